// dressi_rasterize_face_id_noalloc: F::RasterizeFaceId on a fixed,
// library-owned scratch area instead of per-call stream-ordered scratch.
//
// Who needs it: callers that must not allocate device memory during a call
// — a host framework whose caching allocator owns the free memory (a stray
// cudaMallocAsync could fail or fragment its pool), and latency-critical
// render loops where an allocation or release may wait on the device. The
// scratch is a file-scope __device__ array, so it exists on every device
// that loads this library, from module load until process exit.
//
// Set-up: the first call on a device (with that device current) looks the
// array's address up with cudaGetSymbolAddress, which may load the module on
// that device. Make that first call outside any stream capture.
//
// The address is cached per device together with the id of the CUDA context
// it was looked up in. A device reset (cudaDeviceReset) or any other
// destruction and re-creation of the primary context reloads the module and
// can move the array: the next call sees a new context id and looks the
// address up again (that call is then a first call again: keep it outside
// stream capture). Work enqueued before the reset does not survive it.
//
// Calls share the one scratch area per device: two calls that overlap in
// time on the same device (different streams, or host threads without
// ordering between them) race on it.
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <mutex>

#include "../../include/dressi_b200.h"
#include "kernels.h"

namespace dressi {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
unsigned long long g_noalloc_ctx[kMaxDevices] = {};  // context id of the ptr

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Id of the calling thread's current CUDA context (0 if the driver entry
// points are unavailable: the cache then never expires, as before a reset).
unsigned long long current_ctx_id() {
    static CtxGetCurrentFn get_cur = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static bool looked_up = false;
    if (!looked_up) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault,
                                    &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_cur = reinterpret_cast<CtxGetCurrentFn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault,
                                    &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(f);
        looked_up = true;
    }
    if (!get_cur || !get_id) return 0;
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_cur(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Address of this device's scratch, looked up once per device and context.
void* noalloc_scratch(int dev) {
    DRESSI_REQUIRE(dev >= 0 && dev < kMaxDevices,
                   "rasterize_face_id_noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    // cudaSetDevice initialises the device's primary context (or re-creates
    // it after a reset) now, so that its id below is the one the kernels use
    DRESSI_CUDA(cudaSetDevice(dev));
    const unsigned long long ctx = current_ctx_id();
    if (!g_noalloc_ptr[dev] || g_noalloc_ctx[dev] != ctx) {
        void* p = nullptr;
        DRESSI_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_ptr[dev] = p;
        g_noalloc_ctx[dev] = ctx;
    }
    return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace dressi

using namespace dressi;

extern "C" int dressi_rasterize_face_id_noalloc(
        const float* clip, uint32_t n_verts, const float* faces,
        uint32_t n_faces, uint32_t views, uint32_t width, uint32_t height,
        float* out, float* depth_out, uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(clip && out && status && (faces || n_faces == 0),
                       "null pointer");
        DRESSI_REQUIRE(views >= 1 && width >= 1 && height >= 1,
                       "Rasterize: empty screen or no views");
        DRESSI_REQUIRE(width <= 32768 && height <= 32768,
                       "Rasterize: screen larger than 32768");
        DRESSI_REQUIRE(n_faces <= uint32_t(INT_MAX) &&
                               n_verts <= uint32_t(INT_MAX),
                       "Rasterize: face or vertex count above INT_MAX");
        HardDims d;
        d.W = int(width);
        d.H = int(height);
        d.views = int(views);
        d.n_faces = int(n_faces);
        d.n_verts = int(n_verts);
        d.n_comp = 1;
        d.finalize();
        const size_t need = hard_workspace_bytes(d);
        if (need > kNoAllocScratchBytes)
            throw_error(kErrInvalid,
                        "rasterize_face_id_noalloc: needs " +
                                std::to_string(need) +
                                " bytes of scratch, the fixed scratch holds " +
                                std::to_string(kNoAllocScratchBytes) +
                                " (use dressi_rasterize_face_id)",
                        __FILE__, __LINE__);
        int dev = -1;
        DRESSI_CUDA(cudaGetDevice(&dev));
        void* scratch = noalloc_scratch(dev);
        // hard_raster_op zeroes the per-tile counts (the only scratch that
        // must start at zero) on the stream before its first kernel.
        hard_raster_op(d, scratch, clip, nullptr, faces, out, depth_out,
                       status, static_cast<cudaStream_t>(stream));
    });
}
