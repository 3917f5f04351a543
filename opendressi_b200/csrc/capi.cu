// C ABI of libdressi_b200.so (include/dressi_b200.h): argument checking,
// device scratch, plan objects and their CUDA-graph replay.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/dressi_b200.h"
#include "kernels.h"

namespace dressi {

static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }

KernelProfiler*& current_profiler() {
    static thread_local KernelProfiler* p = nullptr;
    return p;
}

void KernelProfiler::begin(const char* name, cudaStream_t s) {
    Rec r{name, nullptr, nullptr};
    DRESSI_CUDA(cudaEventCreate(&r.a));
    DRESSI_CUDA(cudaEventCreate(&r.b));
    DRESSI_CUDA(cudaEventRecord(r.a, s));
    recs.push_back(r);
}

void KernelProfiler::end(cudaStream_t s) {
    if (!recs.empty()) cudaEventRecord(recs.back().b, s);
}

void KernelProfiler::collect(std::vector<const char*>* names,
                             std::vector<double>* ms, std::vector<int>* count) {
    for (auto& r : recs) {
        DRESSI_CUDA(cudaEventSynchronize(r.b));
        float t = 0.f;
        DRESSI_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
        size_t i = 0;
        while (i < names->size() && std::strcmp((*names)[i], r.name) != 0) i++;
        if (i == names->size()) {
            names->push_back(r.name);
            ms->push_back(0.0);
            count->push_back(0);
        }
        (*ms)[i] += t;
        (*count)[i] += 1;
    }
}

KernelProfiler::~KernelProfiler() {
    for (auto& r : recs) {
        if (r.a) cudaEventDestroy(r.a);
        if (r.b) cudaEventDestroy(r.b);
    }
}

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Selects a device for the duration of a call and restores the caller's.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        DRESSI_CUDA(cudaGetDevice(&prev));
        if (prev != dev) DRESSI_CUDA(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0)
            cudaSetDevice(prev);
    }
};

// Stream-ordered scratch for op-level calls.
struct AsyncScratch {
    void* p = nullptr;
    cudaStream_t s;
    AsyncScratch(size_t bytes, cudaStream_t st) : s(st) {
        if (bytes) DRESSI_CUDA(cudaMallocAsync(&p, bytes, s));
    }
    ~AsyncScratch() {
        if (p) cudaFreeAsync(p, s);
    }
};

}  // namespace
}  // namespace dressi

using namespace dressi;

namespace {

// Host-built mesh tables of a silhouette plan's regulariser.
struct RegTables {
    std::vector<float> nbrs, fadj, vf;
    int nbr_deg = 0, vf_deg = 0;
};

void reg_params(SilParams* p, float laplacian, float normal) {
    DRESSI_REQUIRE(std::isfinite(laplacian) && std::isfinite(normal),
                   "silhouette plan: regulariser weights must be finite");
    p->laplacian = laplacian;
    p->normal = normal;
    p->reg = (laplacian != 0.f || normal != 0.f) ? 1 : 0;
}

void reg_tables(const SilParams& p, const float* faces, RegTables* t) {
    if (!p.reg) return;
    sum_all_setup();
    vertex_neighbors_table(faces, p.n_faces, p.n_verts, &t->nbrs,
                           &t->nbr_deg);
    face_neighbors_table(faces, p.n_faces, &t->fadj);
    vertex_faces_table(faces, p.n_faces, p.n_verts, &t->vf, &t->vf_deg);
}

void carve_reg(Arena& a, const SilParams& p, const RegTables& t,
               RegBuffers* r) {
    *r = RegBuffers{};
    if (!p.reg) return;
    const size_t V = size_t(p.n_verts), F = size_t(p.n_faces);
    r->nbrs = a.take<float>(t.nbrs.size());
    r->nbr_deg = t.nbr_deg;
    r->fadj = a.take<float>(t.fadj.size());
    r->vf = a.take<float>(t.vf.size());
    r->vf_deg = t.vf_deg;
    r->term = a.take<float>(F * 3);
    r->glap = a.take<float>(V * 3);
    r->gnrm = a.take<float>(V * 3);
    r->rms = a.take<float>(3);
}

void upload_reg(const RegTables& t, const RegBuffers& r) {
    if (!r.nbrs) return;
    DRESSI_CUDA(cudaMemcpy(r.nbrs, t.nbrs.data(), t.nbrs.size() * 4,
                           cudaMemcpyHostToDevice));
    DRESSI_CUDA(cudaMemcpy(r.fadj, t.fadj.data(), t.fadj.size() * 4,
                           cudaMemcpyHostToDevice));
    DRESSI_CUDA(cudaMemcpy(r.vf, t.vf.data(), t.vf.size() * 4,
                           cudaMemcpyHostToDevice));
}

}  // namespace

struct dressi_plan_s {
    enum Kind { kSil, kFit, kAa, kTex, kPbr } kind = kSil;
    int device = 0;
    void* mem = nullptr;
    size_t mem_bytes = 0;
    struct Slot {
        void* ptr = nullptr;
        size_t bytes = 0;
    } slots[10];
    // silhouette
    SoftDims d;
    SilParams p{};
    SilBuffers b{};
    AaSilBuffers ab{};  // AA plans (ab.sil aliases b)
    // texture plans
    TexParams tp{};
    TexBuffers tb{};
    // PBR plans
    PbrDims pd{};
    PbrBuffers pb{};
    // image fit
    size_t n = 0;
    float lr = 0.f;
    FitBuffers fb{};
    // replay
    cudaStream_t cap_stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaGraphExec_t phase_exec[2] = {nullptr, nullptr};  // exec_phase graphs
    uint32_t kernels_per_iter = 0;
    // silhouette bins live in their own allocation so they can grow
    void* bins_mem = nullptr;
    void* det_mem = nullptr;  // deterministic-mode buffers (b.det_*)
    uint32_t* ovf_host = nullptr;  // pinned: overflow bits of the last
                                   // replayed iteration (written by the graph)

    void alloc_bins() {
        Arena dry;
        carve_soft_bins(dry, d, &b.soft);
        const size_t bytes = dry.used + 256;
        DRESSI_CUDA(cudaMalloc(&bins_mem, bytes));
        Arena a{static_cast<char*>(bins_mem), bytes, 0};
        carve_soft_bins(a, d, &b.soft);
        const size_t vt = size_t(d.views) * d.n_tiles;
        DRESSI_CUDA(cudaMemset(b.soft.bin1.cursor, 0, vt * sizeof(int)));
        DRESSI_CUDA(cudaMemset(b.soft.bin2.cursor, 0, vt * 8 * sizeof(int)));
        DRESSI_CUDA(cudaMemset(b.soft.bin1.spill_n, 0, sizeof(int)));
        DRESSI_CUDA(cudaMemset(b.soft.bin1.parked_n, 0, sizeof(int)));
        DRESSI_CUDA(cudaMemset(b.soft.bin2.spill_n, 0, sizeof(int)));
        DRESSI_CUDA(cudaMemset(b.soft.bin2.open_n, 0, sizeof(int)));
        DRESSI_CUDA(cudaMemset(b.soft.bin2.take, 0, sizeof(int)));
        DRESSI_CUDA(cudaMemset(b.soft.bin2.best, 0xff,
                               size_t(d.views) * d.W * d.H * 8));
    }

    // Reactive growth: a bin set that overflowed in the last replayed
    // iteration (its exact fallback is slow) doubles its capacity, within
    // half of the free device memory; the graph is then re-instantiated.
    void grow_bins_if_needed(cudaStream_t s) {
        if (kind != kSil || !ovf_host) return;
        const uint32_t bits = *reinterpret_cast<volatile uint32_t*>(ovf_host);
        if (!bits) return;
        DRESSI_CUDA(cudaStreamSynchronize(s));
        DRESSI_CUDA(cudaDeviceSynchronize());
        SoftDims nd = d;
        if (bits & 1u) nd.cap1 = std::min(nd.cap1 * 2, 1 << 16);
        if (bits & 2u) nd.cap2 = std::min(nd.cap2 * 2, 1 << 16);
        *ovf_host = 0;
        if (nd.cap1 == d.cap1 && nd.cap2 == d.cap2) return;
        Arena dry;
        SoftBuffers tmp = b.soft;
        carve_soft_bins(dry, nd, &tmp);
        size_t free_b = 0, total_b = 0;
        DRESSI_CUDA(cudaMemGetInfo(&free_b, &total_b));
        if (dry.used > free_b / 2) return;  // keep the (exact) fallback
        if (exec) {
            cudaGraphExecDestroy(exec);
            exec = nullptr;
        }
        for (auto& g : phase_exec) {
            if (g) cudaGraphExecDestroy(g);
            g = nullptr;
        }
        DRESSI_CUDA(cudaFree(bins_mem));
        bins_mem = nullptr;
        d = nd;
        alloc_bins();
    }

    void set_slot(int i, void* ptr, size_t bytes) {
        slots[i].ptr = ptr;
        slots[i].bytes = bytes;
    }

    // the side stream of the regulariser's fork (silhouette plans with a
    // regulariser), created on first use
    StreamFork fork;
    const StreamFork* reg_fork() {
        if (kind != kSil || !p.reg) return nullptr;
        if (!fork.side) {
            DRESSI_CUDA(cudaStreamCreateWithFlags(&fork.side,
                                                  cudaStreamNonBlocking));
            DRESSI_CUDA(cudaEventCreateWithFlags(&fork.begin,
                                                 cudaEventDisableTiming));
            DRESSI_CUDA(cudaEventCreateWithFlags(&fork.end,
                                                 cudaEventDisableTiming));
        }
        return &fork;
    }

    void record_iteration(cudaStream_t s) {
        if (kind == kSil) {
            sil_iteration(d, p, b, s, reg_fork());
            if (ovf_host)
                DRESSI_CUDA(cudaMemcpyAsync(ovf_host, b.soft.status + 1, 4,
                                            cudaMemcpyDeviceToHost, s));
        } else if (kind == kAa) {
            aa_sil_iteration(p, ab, s);
        } else if (kind == kTex) {
            tex_iteration(tp, tb, s);
        } else if (kind == kPbr) {
            pbr_iteration(pd, pb, s);
        } else {
            fit_iteration(n, lr, fb, s);
        }
    }

    void ensure_graph() {
        if (exec) return;
        if (!cap_stream)
            DRESSI_CUDA(cudaStreamCreateWithFlags(&cap_stream,
                                                  cudaStreamNonBlocking));
        cudaGraph_t g = nullptr;
        DRESSI_CUDA(cudaStreamBeginCapture(cap_stream,
                                           cudaStreamCaptureModeThreadLocal));
        try {
            record_iteration(cap_stream);
        } catch (...) {
            cudaStreamEndCapture(cap_stream, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        DRESSI_CUDA(cudaStreamEndCapture(cap_stream, &g));
        size_t n_nodes = 0;
        DRESSI_CUDA(cudaGraphGetNodes(g, nullptr, &n_nodes));
        std::vector<cudaGraphNode_t> nodes(n_nodes);
        DRESSI_CUDA(cudaGraphGetNodes(g, nodes.data(), &n_nodes));
        uint32_t k = 0;
        for (auto nd : nodes) {
            cudaGraphNodeType t;
            DRESSI_CUDA(cudaGraphNodeGetType(nd, &t));
            if (t == cudaGraphNodeTypeKernel) k++;
        }
        kernels_per_iter = k;
        const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        DRESSI_CUDA(e);
    }

    // One phase of a sharded iteration (0: forward/backward into GRAD, 1:
    // the update from GRAD), as exec_phase replays it.
    void record_phase(int phase, cudaStream_t s) {
        if (kind == kTex) {
            if (phase == 0)
                tex_forward_backward(tp, tb, nullptr, s);
            else
                tex_update(tp, tb, s);
        } else if (kind == kPbr) {
            if (phase == 0)
                pbr_forward_backward(pd, pb, s);
            else
                pbr_update(pd, pb, s);
        } else if (kind == kAa) {
            if (phase == 0) {
                aa_sil_forward_backward(p, ab, s);
                sil_grad_reduce(p, b, false, s);
                sil_reg_terms(p, b, s);
            } else {
                sil_update(p, b, s);
            }
        } else if (phase == 0) {
            // the regulariser's terms (pos only) on a parallel branch
            const StreamFork* fk = reg_fork();
            if (fk) {
                DRESSI_CUDA(cudaEventRecord(fk->begin, s));
                DRESSI_CUDA(cudaStreamWaitEvent(fk->side, fk->begin, 0));
                sil_reg_terms(p, b, fk->side);
                DRESSI_CUDA(cudaEventRecord(fk->end, fk->side));
            }
            sil_forward_backward(d, p, b, nullptr, s);
            sil_grad_reduce(p, b, false, s);
            if (fk)
                DRESSI_CUDA(cudaStreamWaitEvent(s, fk->end, 0));
            else
                sil_reg_terms(p, b, s);
            DRESSI_CUDA(cudaMemcpyAsync(ovf_host, b.soft.status + 1, 4,
                                        cudaMemcpyDeviceToHost, s));
        } else {
            sil_update(p, b, s);
        }
    }

    void ensure_phase_graph(int phase) {
        if (phase_exec[phase]) return;
        if (!cap_stream)
            DRESSI_CUDA(cudaStreamCreateWithFlags(&cap_stream,
                                                  cudaStreamNonBlocking));
        cudaGraph_t g = nullptr;
        DRESSI_CUDA(cudaStreamBeginCapture(cap_stream,
                                           cudaStreamCaptureModeThreadLocal));
        try {
            record_phase(phase, cap_stream);
        } catch (...) {
            cudaStreamEndCapture(cap_stream, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        DRESSI_CUDA(cudaStreamEndCapture(cap_stream, &g));
        const cudaError_t e = cudaGraphInstantiate(&phase_exec[phase], g, 0);
        cudaGraphDestroy(g);
        DRESSI_CUDA(e);
    }

    ~dressi_plan_s() {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (exec) cudaGraphExecDestroy(exec);
        for (auto g : phase_exec)
            if (g) cudaGraphExecDestroy(g);
        if (cap_stream) cudaStreamDestroy(cap_stream);
        if (mem) cudaFree(mem);
        if (bins_mem) cudaFree(bins_mem);
        // the render slot is allocated on first use
        if (slots[DRESSI_SLOT_RASTER].ptr) cudaFree(slots[DRESSI_SLOT_RASTER].ptr);
        if (ovf_host) cudaFreeHost(ovf_host);
        if (det_mem) cudaFree(det_mem);
        if (fork.side) cudaStreamDestroy(fork.side);
        if (fork.begin) cudaEventDestroy(fork.begin);
        if (fork.end) cudaEventDestroy(fork.end);
        if (prev >= 0) cudaSetDevice(prev);
    }
};

extern "C" {

int dressi_abi_version(void) { return DRESSI_B200_ABI_VERSION; }

int dressi_last_error(char* buf, size_t len) {
    const std::string& e = g_last_error;
    if (buf && len) {
        const size_t n = std::min(len - 1, e.size());
        std::memcpy(buf, e.data(), n);
        buf[n] = '\0';
    }
    return int(e.size());
}

int dressi_soft_clip(const float* clip, uint32_t n_verts, const float* faces,
                     uint32_t n_faces, uint32_t views, uint32_t width,
                     uint32_t height, float radius_px, float* out,
                     uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(clip && faces && out && status, "null pointer");
        DRESSI_REQUIRE(views >= 1 && width >= 1 && height >= 1,
                       "SoftClip: empty screen or no views");
        DRESSI_REQUIRE(radius_px >= 0.f, "SoftClip: radius_px must be >= 0");
        soft_clip_op(clip, faces, int(views), int(n_verts), int(n_faces),
                     int(width), int(height), radius_px, out, status,
                     as_stream(stream));
    });
}

int dressi_rasterize_soft(const float* soft_clip, uint32_t n_soft,
                          const float* face_id, const float* faces_soft,
                          uint32_t n_faces, const float* hard_clip,
                          uint32_t n_hard, const float* faces_tex,
                          uint32_t views, uint32_t width, uint32_t height,
                          float radius_px, const float* prev_depth,
                          float* out, uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(out && status, "null pointer");
        DRESSI_REQUIRE(n_faces == 0 ||
                               (soft_clip && face_id && faces_soft &&
                                hard_clip && faces_tex),
                       "null pointer");
        DRESSI_REQUIRE(views >= 1 && width >= 1 && height >= 1,
                       "RasterizeSoft: empty screen or no views");
        DRESSI_REQUIRE(width <= 32768 && height <= 32768,
                       "RasterizeSoft: screen larger than 32768");
        DRESSI_REQUIRE(radius_px > 0.f, "RasterizeSoft: radius_px must be > 0");
        DRESSI_REQUIRE(n_soft == 3 * n_faces,
                       "RasterizeSoft: soft vertices must be unwelded "
                       "(3 per face)");
        cudaStream_t s = as_stream(stream);
        SoftDims d;
        d.W = int(width);
        d.H = int(height);
        d.views = int(views);
        d.n_faces = int(n_faces);
        d.n_verts = int(n_hard);
        d.radius = radius_px;
        d.finalize();
        default_caps(&d);
        Arena a;
        SoftBuffers b;
        carve_soft(a, d, &b);
        AsyncScratch scratch(a.used + 256, s);
        a = Arena{static_cast<char*>(scratch.p), a.used + 256, 0};
        carve_soft(a, d, &b);
        init_soft(d, b, s);  // zeroes the counters (and the scratch word)
        b.status = status;   // report into the caller's word
        SoftOpInputs in{soft_clip, face_id, faces_soft, hard_clip, faces_tex,
                        prev_depth, int(n_soft), int(n_hard)};
        soft_raster_op(d, b, in, out, s);
    });
}

int dressi_rasterize_soft_grad(const float* gy, const float* rs,
                               const float* clip, uint32_t n_verts,
                               const float* faces, uint32_t n_faces,
                               uint32_t views, uint32_t width,
                               uint32_t height, float* grad, uint32_t* status,
                               void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(gy && rs && clip && faces && grad && status,
                       "null pointer");
        DRESSI_REQUIRE(views >= 1 && width >= 1 && height >= 1,
                       "RasterizeSoft grad: empty screen or no views");
        dist_grad_op(gy, rs, clip, faces, int(views), int(n_verts),
                     int(n_faces), int(width), int(height), grad, status,
                     as_stream(stream));
    });
}

static int hard_common(const float* clip, uint32_t n_verts, const float* attr,
                       uint32_t n_comp, const float* faces, uint32_t n_faces,
                       uint32_t views, uint32_t width, uint32_t height,
                       float* out, float* depth_out, uint32_t* status,
                       void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(clip && out && status && (faces || n_faces == 0),
                       "null pointer");
        DRESSI_REQUIRE(views >= 1 && width >= 1 && height >= 1,
                       "Rasterize: empty screen or no views");
        DRESSI_REQUIRE(width <= 32768 && height <= 32768,
                       "Rasterize: screen larger than 32768");
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4,
                       "Rasterize: attribute must have 1..4 components");
        DRESSI_REQUIRE(n_faces <= uint32_t(INT_MAX) &&
                               n_verts <= uint32_t(INT_MAX),
                       "Rasterize: face or vertex count above INT_MAX");
        cudaStream_t s = as_stream(stream);
        HardDims d;
        d.W = int(width);
        d.H = int(height);
        d.views = int(views);
        d.n_faces = int(n_faces);
        d.n_verts = int(n_verts);
        d.n_comp = int(n_comp);
        d.finalize();
        AsyncScratch scratch(hard_workspace_bytes(d), s);
        hard_raster_op(d, scratch.p, clip, attr, faces, out, depth_out,
                       status, s);
    });
}

int dressi_rasterize_face_id(const float* clip, uint32_t n_verts,
                             const float* faces, uint32_t n_faces,
                             uint32_t views, uint32_t width, uint32_t height,
                             float* out, float* depth_out, uint32_t* status,
                             void* stream) {
    return hard_common(clip, n_verts, nullptr, 1, faces, n_faces, views,
                       width, height, out, depth_out, status, stream);
}

int dressi_rasterize(const float* clip, uint32_t n_verts, const float* attr,
                     uint32_t n_comp, const float* faces, uint32_t n_faces,
                     uint32_t views, uint32_t width, uint32_t height,
                     float* out, uint32_t* status, void* stream) {
    if (!attr) {
        set_last_error("Rasterize: null attribute");
        return DRESSI_ERR_INVALID;
    }
    return hard_common(clip, n_verts, attr, n_comp, faces, n_faces, views,
                       width, height, out, nullptr, status, stream);
}

static void aa_common_checks(const float* tri, const float* clip,
                             uint32_t n_comp, const float* faces,
                             uint32_t n_faces, uint32_t views, uint32_t width,
                             uint32_t height, uint32_t* status) {
    DRESSI_REQUIRE(tri && clip && status && (faces || n_faces == 0),
                   "null pointer");
    DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4,
                   "AntiAlias: img must have 1..4 components");
    DRESSI_REQUIRE(views >= 1 && width >= 1 && height >= 1,
                   "AntiAlias: empty screen or no views");
    DRESSI_REQUIRE(width <= 32768 && height <= 32768,
                   "AntiAlias: screen larger than 32768");
}

static AaDims aa_dims(uint32_t n_comp, uint32_t n_verts, uint32_t n_faces,
                      uint32_t views, uint32_t width, uint32_t height) {
    AaDims d;
    d.W = int(width);
    d.H = int(height);
    d.views = int(views);
    d.n_faces = int(n_faces);
    d.n_verts = int(n_verts);
    d.n_comp = int(n_comp);
    return d;
}

int dressi_antialias(const float* img, uint32_t n_comp, const float* tri,
                     const float* clip, uint32_t n_verts, const float* faces,
                     uint32_t n_faces, uint32_t views, uint32_t width,
                     uint32_t height, float* out, uint32_t* status,
                     void* stream) {
    return guarded([&] {
        aa_common_checks(tri, clip, n_comp, faces, n_faces, views, width,
                         height, status);
        DRESSI_REQUIRE(img && out, "null pointer");
        cudaStream_t s = as_stream(stream);
        const AaDims d = aa_dims(n_comp, n_verts, n_faces, views, width, height);
        const size_t rec_bytes = size_t(views) * std::max<uint32_t>(n_faces, 1) *
                                 sizeof(AaFace);
        AsyncScratch fr(rec_bytes + sizeof(int) * views, s);
        AaFace* recs = static_cast<AaFace*>(fr.p);
        int* vflags = reinterpret_cast<int*>(static_cast<char*>(fr.p) + rec_bytes);
        aa_face_setup(d, clip, faces, recs, vflags, status, s);
        aa_forward_op(d, recs, vflags, img, tri, out, s);
    });
}

int dressi_antialias_grad(const float* gy, const float* img, uint32_t n_comp,
                          const float* tri, const float* clip,
                          uint32_t n_verts, const float* faces,
                          uint32_t n_faces, const float* vft,
                          uint32_t max_deg, float seed, uint32_t n_samples,
                          uint32_t views, uint32_t width, uint32_t height,
                          float* grad_img, float* grad_clip, uint32_t* status,
                          void* stream) {
    return guarded([&] {
        aa_common_checks(tri, clip, n_comp, faces, n_faces, views, width,
                         height, status);
        DRESSI_REQUIRE(gy, "null pointer");
        DRESSI_REQUIRE(!grad_clip || img, "AntiAlias grad: img is required "
                                          "for the vertex gradient");
        DRESSI_REQUIRE(!grad_clip || n_samples == 0 || (vft && max_deg >= 1),
                       "AntiAlias grad: stochastic samples need the vertex "
                       "-> face table");
        cudaStream_t s = as_stream(stream);
        const AaDims d = aa_dims(n_comp, n_verts, n_faces, views, width, height);
        const size_t rec_bytes = size_t(views) * std::max<uint32_t>(n_faces, 1) *
                                 sizeof(AaFace);
        AsyncScratch fr(rec_bytes + sizeof(int) * views, s);
        AaFace* recs = static_cast<AaFace*>(fr.p);
        int* vflags = reinterpret_cast<int*>(static_cast<char*>(fr.p) + rec_bytes);
        aa_face_setup(d, clip, faces, recs, vflags, status, s);
        if (grad_img) aa_bwd_img_op(d, recs, gy, tri, grad_img, s);
        if (grad_clip)
            aa_bwd_vtx_op(d, recs, gy, img, tri, clip, vft, int(max_deg),
                          seed, int(n_samples), grad_clip, s);
    });
}

// The silhouette plans: RasterizeSoft's own backward (paper = 0) or the
// paper path (paper = 1: peels layers, n_samples FaceFetch edge samples).
static int create_silhouette(const dressi_silhouette_desc* desc, int paper,
                             uint32_t peels, uint32_t n_samples,
                             dressi_plan* out) {
    return guarded([&] {
        DRESSI_REQUIRE(desc && out, "null pointer");
        DRESSI_REQUIRE(desc->struct_size == sizeof(dressi_silhouette_desc),
                       "dressi_silhouette_desc: struct_size mismatch");
        DRESSI_REQUIRE(desc->n_verts > 0 && desc->n_faces > 0 &&
                               desc->n_views > 0 && desc->res > 0,
                       "silhouette plan: empty mesh, views or screen");
        DRESSI_REQUIRE(desc->res <= 32768, "silhouette plan: res > 32768");
        DRESSI_REQUIRE(desc->faces && desc->mvps, "null pointer");
        DRESSI_REQUIRE(desc->radius_px > 0.f && (paper || desc->sigma > 0.f),
                       "silhouette plan: radius_px and sigma must be > 0");
        DRESSI_REQUIRE(!paper || (peels >= 1 && peels <= uint32_t(kPaperMaxPeels)),
                       "paper silhouette plan: peels must be 1..4");
        DRESSI_REQUIRE(n_samples <= 4096, "silhouette plan: n_samples > 4096");
        *out = nullptr;
        DeviceGuard dg(desc->device);
        auto pl = std::make_unique<dressi_plan_s>();
        pl->kind = dressi_plan_s::kSil;
        pl->device = desc->device;
        SoftDims& d = pl->d;
        d.W = d.H = int(desc->res);
        d.views = int(desc->n_views);
        d.n_faces = int(desc->n_faces);
        d.n_verts = int(desc->n_verts);
        d.radius = desc->radius_px;
        d.finalize();
        default_caps(&d);
        SilParams& p = pl->p;
        p.n_verts = int(desc->n_verts);
        p.n_faces = int(desc->n_faces);
        p.views = int(desc->n_views);
        p.res = int(desc->res);
        p.radius = desc->radius_px;
        p.sigma = desc->sigma;
        p.lr = desc->lr;
        p.b1 = desc->beta1;
        p.b2 = desc->beta2;
        p.eps = desc->eps;
        p.k = paper ? 0.f
                    : (2.f / float(desc->res)) * (2.f / float(desc->res)) /
                              desc->sigma;
        p.c = 1.f / float(desc->res * desc->res);
        p.paper = paper;
        p.peels = paper ? int(peels) : 1;
        p.n_samples = int(n_samples);
        p.sigma_scale = 7.f / desc->radius_px;
        reg_params(&p, desc->laplacian, desc->normal);
        RegTables rt;
        reg_tables(p, desc->faces, &rt);
        const int hist = desc->loss_history ? int(desc->loss_history) : 4096;
        const size_t V = desc->n_verts, F = desc->n_faces, NV = desc->n_views;
        const size_t R2 = size_t(desc->res) * desc->res;
        auto carve = [&](Arena& a) {
            SilBuffers& b = pl->b;
            if (paper) {
                b.paper_layers = a.take<float4>(size_t(peels) * NV * R2);
                b.paper_prev = a.take<float>(NV * R2);
                b.paper_gfetch = a.take<float4>(size_t(peels) * 3 * NV * R2);
            }
            b.pos = a.take<float>(V * 3);
            b.adam_m = a.take<float>(V * 3);
            b.adam_v = a.take<float>(V * 3);
            b.scalars = a.take<float>(4);
            b.faces = a.take<float>(F * 3);
            b.mvps = a.take<float>(NV * 16);
            b.targets = a.take<float>(NV * R2);
            b.clip = a.take<float>(NV * V * 4);
            b.gclip = a.take<float>(NV * V * 4);
            b.gpos = a.take<float>(V * 3);
            b.loss_slots = a.take<double>(kLossSlots);
            b.loss_hist = a.take<float>(size_t(hist));
            b.hist_cap = hist;
            b.done = a.take<unsigned>(1);
            carve_soft_main(a, d, &b.soft);
            carve_reg(a, p, rt, &b.reg);
        };
        Arena dry;
        carve(dry);
        pl->mem_bytes = dry.used + 256;
        DRESSI_CUDA(cudaMalloc(&pl->mem, pl->mem_bytes));
        Arena a{static_cast<char*>(pl->mem), pl->mem_bytes, 0};
        carve(a);
        // Everything starts at zero: Adam state, counters, gradients.
        DRESSI_CUDA(cudaMemset(pl->mem, 0, pl->mem_bytes));
        DRESSI_CUDA(cudaMemcpy(pl->b.faces, desc->faces, F * 3 * sizeof(float),
                               cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(pl->b.mvps, desc->mvps, NV * 16 * sizeof(float),
                               cudaMemcpyHostToDevice));
        upload_reg(rt, pl->b.reg);
        pl->alloc_bins();
        DRESSI_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&pl->ovf_host), 4,
                                  cudaHostAllocDefault));
        *pl->ovf_host = 0;
        pl->set_slot(DRESSI_SLOT_PARAM, pl->b.pos, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_M, pl->b.adam_m, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_V, pl->b.adam_v, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_T, pl->b.scalars, 4);
        pl->set_slot(DRESSI_SLOT_TARGET, pl->b.targets, NV * R2 * 4);
        pl->set_slot(DRESSI_SLOT_GRAD, pl->b.gpos, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_LOSS, pl->b.scalars + 3, 4);
        pl->set_slot(DRESSI_SLOT_LOSS_HISTORY, pl->b.loss_hist, size_t(hist) * 4);
        pl->set_slot(DRESSI_SLOT_RASTER, nullptr, NV * R2 * 16);
        pl->set_slot(DRESSI_SLOT_MVP, pl->b.mvps, NV * 16 * 4);
        *out = pl.release();
    });
}

int dressi_silhouette_plan_create(const dressi_silhouette_desc* desc,
                                  dressi_plan* out) {
    return create_silhouette(desc, 0, 1, 0, out);
}

int dressi_paper_silhouette_plan_create(const dressi_silhouette_desc* desc,
                                        uint32_t peels, uint32_t n_samples,
                                        dressi_plan* out) {
    return create_silhouette(desc, 1, peels, n_samples, out);
}

int dressi_aa_silhouette_plan_create(const dressi_aa_silhouette_desc* desc,
                                     dressi_plan* out) {
    return guarded([&] {
        DRESSI_REQUIRE(desc && out, "null pointer");
        DRESSI_REQUIRE(desc->struct_size == sizeof(dressi_aa_silhouette_desc),
                       "dressi_aa_silhouette_desc: struct_size mismatch");
        DRESSI_REQUIRE(desc->n_verts > 0 && desc->n_faces > 0 &&
                               desc->n_views > 0 && desc->res > 0,
                       "AA silhouette plan: empty mesh, views or screen");
        DRESSI_REQUIRE(desc->res <= 32768, "AA silhouette plan: res > 32768");
        DRESSI_REQUIRE(desc->faces && desc->mvps, "null pointer");
        DRESSI_REQUIRE(desc->n_samples <= 4096,
                       "AA silhouette plan: n_samples > 4096");
        *out = nullptr;
        DeviceGuard dg(desc->device);
        auto pl = std::make_unique<dressi_plan_s>();
        pl->kind = dressi_plan_s::kAa;
        pl->device = desc->device;
        SilParams& p = pl->p;
        p.n_verts = int(desc->n_verts);
        p.n_faces = int(desc->n_faces);
        p.views = int(desc->n_views);
        p.res = int(desc->res);
        p.lr = desc->lr;
        p.b1 = desc->beta1;
        p.b2 = desc->beta2;
        p.eps = desc->eps;
        p.c = 1.f / float(desc->res * desc->res);
        p.n_samples = int(desc->n_samples);
        reg_params(&p, desc->laplacian, desc->normal);
        RegTables rt;
        reg_tables(p, desc->faces, &rt);
        const int hist = desc->loss_history ? int(desc->loss_history) : 4096;
        const size_t V = desc->n_verts, F = desc->n_faces, NV = desc->n_views;
        const size_t R2 = size_t(desc->res) * desc->res;
        const size_t ws = aa_sil_workspace_bytes(p);
        auto carve = [&](Arena& a) {
            SilBuffers& b = pl->b;
            b.pos = a.take<float>(V * 3);
            b.adam_m = a.take<float>(V * 3);
            b.adam_v = a.take<float>(V * 3);
            b.scalars = a.take<float>(4);
            b.faces = a.take<float>(F * 3);
            b.mvps = a.take<float>(NV * 16);
            b.targets = a.take<float>(NV * R2);
            b.clip = a.take<float>(NV * V * 4);
            b.gclip = a.take<float>(NV * V * 4);
            b.gpos = a.take<float>(V * 3);
            b.loss_slots = a.take<double>(kLossSlots);
            b.loss_hist = a.take<float>(size_t(hist));
            b.hist_cap = hist;
            b.done = a.take<unsigned>(1);
            AaSilBuffers& ab = pl->ab;
            ab.tri = a.take<float>(NV * R2);
            ab.gy = a.take<float>(NV * R2);
            ab.frs = a.take<AaFace>(NV * F);
            ab.view_flags = a.take<int>(NV);
            ab.status = a.take<uint32_t>(4);
            ab.hard_ws = a.take<char>(ws);
            carve_reg(a, p, rt, &b.reg);
        };
        Arena dry;
        carve(dry);
        pl->mem_bytes = dry.used + 256;
        DRESSI_CUDA(cudaMalloc(&pl->mem, pl->mem_bytes));
        Arena a{static_cast<char*>(pl->mem), pl->mem_bytes, 0};
        carve(a);
        pl->ab.sil = pl->b;
        // Everything starts at zero: Adam state, counters, gradients.
        DRESSI_CUDA(cudaMemset(pl->mem, 0, pl->mem_bytes));
        DRESSI_CUDA(cudaMemcpy(pl->b.faces, desc->faces, F * 3 * sizeof(float),
                               cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(pl->b.mvps, desc->mvps, NV * 16 * sizeof(float),
                               cudaMemcpyHostToDevice));
        upload_reg(rt, pl->b.reg);
        pl->set_slot(DRESSI_SLOT_PARAM, pl->b.pos, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_M, pl->b.adam_m, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_V, pl->b.adam_v, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_T, pl->b.scalars, 4);
        pl->set_slot(DRESSI_SLOT_TARGET, pl->b.targets, NV * R2 * 4);
        pl->set_slot(DRESSI_SLOT_GRAD, pl->b.gpos, V * 3 * 4);
        pl->set_slot(DRESSI_SLOT_LOSS, pl->b.scalars + 3, 4);
        pl->set_slot(DRESSI_SLOT_LOSS_HISTORY, pl->b.loss_hist, size_t(hist) * 4);
        pl->set_slot(DRESSI_SLOT_RASTER, nullptr, NV * R2 * 4);
        pl->set_slot(DRESSI_SLOT_MVP, pl->b.mvps, NV * 16 * 4);
        *out = pl.release();
    });
}

int dressi_rasterize_uvzw(const float* clip_vk, const float* pos_gl,
                          uint32_t n_verts, const float* faces,
                          uint32_t n_faces, uint32_t views, uint32_t width,
                          uint32_t height, float* out, uint32_t* status,
                          void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(clip_vk && pos_gl && out && status &&
                               (faces || n_faces == 0),
                       "null pointer");
        DRESSI_REQUIRE(views >= 1 && width >= 1 && height >= 1,
                       "rasterize: empty screen or no views");
        DRESSI_REQUIRE(width <= 32768 && height <= 32768,
                       "rasterize: screen larger than 32768");
        cudaStream_t s = as_stream(stream);
        HardDims d;
        d.W = int(width);
        d.H = int(height);
        d.views = int(views);
        d.n_faces = int(n_faces);
        d.n_verts = int(n_verts);
        d.n_comp = 4;
        d.uvzw = 1;
        d.finalize();
        AsyncScratch scratch(hard_workspace_bytes(d), s);
        hard_raster_op(d, scratch.p, clip_vk, pos_gl, faces, out, nullptr,
                       status, s);
    });
}

int dressi_interpolate(const float* attr, uint32_t n_comp, uint32_t n_verts,
                       uint32_t attr_views, const float* rast,
                       const float* faces, uint32_t n_faces, uint32_t views,
                       uint32_t width, uint32_t height, float* out,
                       uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(attr && rast && out && status && (faces || n_faces == 0),
                       "null pointer");
        DRESSI_REQUIRE(n_comp >= 1, "interpolate: attr has no components");
        DRESSI_REQUIRE(attr_views == 1 || attr_views == views,
                       "interpolate: attr views must be 1 or the rast views");
        interpolate_op(attr, int(n_comp), int(n_verts), int(attr_views), rast,
                       faces, int(n_faces), int(views), int(width),
                       int(height), out, status, as_stream(stream));
    });
}

int dressi_interpolate_grad(const float* gy, uint32_t n_comp,
                            uint32_t n_verts, uint32_t attr_views,
                            const float* rast, const float* faces,
                            uint32_t n_faces, uint32_t views, uint32_t width,
                            uint32_t height, float* grad_attr,
                            uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(gy && rast && grad_attr && status &&
                               (faces || n_faces == 0),
                       "null pointer");
        DRESSI_REQUIRE(n_comp >= 1, "interpolate grad: no components");
        DRESSI_REQUIRE(attr_views == 1 || attr_views == views,
                       "interpolate grad: attr views must be 1 or the rast "
                       "views");
        interpolate_grad_op(gy, int(n_comp), int(n_verts), int(attr_views),
                            rast, faces, int(n_faces), int(views),
                            int(width), int(height), grad_attr, status,
                            as_stream(stream));
    });
}

int dressi_texture(const float* tex, uint32_t tw, uint32_t th,
                   uint32_t n_comp, const float* uv, uint32_t n_px,
                   uint32_t filter, float* out, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(tex && uv && out, "null pointer");
        DRESSI_REQUIRE(tw >= 1 && th >= 1, "Texture: empty texture");
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4,
                       "Texture: texture must have 1..4 components");
        DRESSI_REQUIRE(filter <= 1, "Texture: filter is 0 (nearest) or 1 "
                                    "(bilinear)");
        texture_sample_op(tex, int(tw), int(th), int(n_comp), int(filter), uv,
                          n_px, out, as_stream(stream));
    });
}

int dressi_texture_grad(const float* gy, uint32_t sw, uint32_t sh,
                        uint32_t n_comp, const float* inv_uv, uint32_t tw,
                        uint32_t th, const float* uv_screen, uint32_t filter,
                        float* grad_tex, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(gy && inv_uv && uv_screen && grad_tex, "null pointer");
        DRESSI_REQUIRE(tw >= 1 && th >= 1 && sw >= 1 && sh >= 1,
                       "Texture grad: empty texture or screen");
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4,
                       "Texture grad: 1..4 components");
        DRESSI_REQUIRE(filter <= 1, "Texture grad: filter is 0 or 1");
        texture_gather_op(gy, int(sw), int(sh), int(n_comp), int(filter),
                          inv_uv, int(tw), int(th), uv_screen, grad_tex,
                          as_stream(stream));
    });
}

namespace {

int copy_table(const std::vector<float>& t, int deg, uint32_t cap, float* out,
               uint32_t* deg_out, const char* what) {
    DRESSI_REQUIRE(uint32_t(deg) <= cap,
                   std::string(what) + ": table height " + std::to_string(deg) +
                           " above cap " + std::to_string(cap));
    std::copy(t.begin(), t.end(), out);
    *deg_out = uint32_t(deg);
    return 0;
}

}  // namespace

int dressi_vertex_faces_tex(const float* faces, uint32_t n_faces,
                            uint32_t n_verts, uint32_t cap, float* out,
                            uint32_t* deg) {
    return guarded([&] {
        DRESSI_REQUIRE(faces && out && deg, "null pointer");
        std::vector<float> t;
        int d = 0;
        vertex_faces_table(faces, int(n_faces), int(n_verts), &t, &d);
        copy_table(t, d, cap, out, deg, "VertexFacesTex");
    });
}

int dressi_vertex_neighbors_tex(const float* faces, uint32_t n_faces,
                                uint32_t n_verts, uint32_t cap, float* out,
                                uint32_t* deg) {
    return guarded([&] {
        DRESSI_REQUIRE(faces && out && deg, "null pointer");
        std::vector<float> t;
        int d = 0;
        vertex_neighbors_table(faces, int(n_faces), int(n_verts), &t, &d);
        copy_table(t, d, cap, out, deg, "VertexNeighborsTex");
    });
}

int dressi_face_neighbors_tex(const float* faces, uint32_t n_faces,
                              float* out) {
    return guarded([&] {
        DRESSI_REQUIRE(faces && out, "null pointer");
        std::vector<float> t;
        face_neighbors_table(faces, int(n_faces), &t);
        std::copy(t.begin(), t.end(), out);
    });
}

int dressi_vertex_neighbor_mean(const float* pos, uint32_t n_verts,
                                const float* nbrs, uint32_t nbr_deg,
                                float* out, uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(pos && nbrs && out, "null pointer");
        vertex_terms_op(pos, int(n_verts), nbrs, int(nbr_deg), false, out,
                        nullptr, nullptr, 0, nullptr, 0, nullptr, status,
                        as_stream(stream));
    });
}

int dressi_normal_consistency_face_term(const float* pos, uint32_t n_verts,
                                        const float* faces, uint32_t n_faces,
                                        const float* face_adj, float* out,
                                        uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(pos && faces && face_adj && out, "null pointer");
        nc_face_term_op(pos, int(n_verts), faces, face_adj, int(n_faces), out,
                        status, as_stream(stream));
    });
}

int dressi_normal_consistency_vertex_grad(const float* term, const float* pos,
                                          uint32_t n_verts, const float* faces,
                                          uint32_t n_faces,
                                          const float* vtx_faces,
                                          uint32_t vf_deg, float* out,
                                          uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(term && pos && faces && vtx_faces && out,
                       "null pointer");
        vertex_terms_op(pos, int(n_verts), nullptr, 0, false, nullptr, term,
                        faces, int(n_faces), vtx_faces, int(vf_deg), out,
                        status, as_stream(stream));
    });
}

int dressi_sum_all(const float* x, uint32_t n_px, uint32_t n_comp, float* out,
                   void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(x && out, "null pointer");
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4, "SumAll: 1..4 components");
        sum_all_setup();
        sum_all_op(x, int(n_px), int(n_comp), out, as_stream(stream));
    });
}

int dressi_regularized_grad(const float* pos, uint32_t n_verts,
                            const float* faces, uint32_t n_faces,
                            const float* nbrs, uint32_t nbr_deg,
                            const float* face_adj, const float* vtx_faces,
                            uint32_t vf_deg, const float* g, float laplacian,
                            float normal, float* out, uint32_t* status,
                            void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(pos && faces && nbrs && face_adj && vtx_faces && g &&
                               out,
                       "null pointer");
        DRESSI_REQUIRE(n_verts > 0, "regularized_grad: no vertices");
        cudaStream_t s = as_stream(stream);
        sum_all_setup();
        const size_t V3 = size_t(n_verts) * 3, F3 = size_t(n_faces) * 3;
        AsyncScratch sc((F3 + 2 * V3 + 3) * sizeof(float), s);
        float* term = static_cast<float*>(sc.p);
        float* glap = term + F3;
        float* gnrm = glap + V3;
        float* rms = gnrm + V3;
        nc_face_term_op(pos, int(n_verts), faces, face_adj, int(n_faces), term,
                        status, s);
        vertex_terms_op(pos, int(n_verts), nbrs, int(nbr_deg), true, glap,
                        term, faces, int(n_faces), vtx_faces, int(vf_deg),
                        gnrm, status, s);
        reg_rms_op(g, glap, gnrm, int(n_verts), rms, s);
        reg_combine_op(g, glap, gnrm, rms, laplacian, normal, int(n_verts),
                       out, s);
    });
}

// ---------------------------------------------------- split-sum IBL ops

namespace {

void ibl_checks(const void* a, const void* b, uint32_t n_comp) {
    DRESSI_REQUIRE(a && b, "null pointer");
    DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4, "IBL op: 1..4 components");
}

}  // namespace

int dressi_equirect_sample(const float* map, uint32_t mw, uint32_t mh,
                           uint32_t n_comp, const float* dir, uint64_t n_px,
                           float* out, void* stream) {
    return guarded([&] {
        ibl_checks(map, dir, n_comp);
        DRESSI_REQUIRE(out, "null pointer");
        DRESSI_REQUIRE(mw >= 1 && mh >= 1, "EquirectSample: empty map");
        equirect_sample_op(map, int(mw), int(mh), int(n_comp), dir,
                           (long long)n_px, out, as_stream(stream));
    });
}

int dressi_equirect_sample_grad(const float* gy, const float* dir,
                                uint64_t n_px, uint32_t mw, uint32_t mh,
                                uint32_t n_comp, float* g_map, void* stream) {
    return guarded([&] {
        ibl_checks(gy, dir, n_comp);
        DRESSI_REQUIRE(g_map, "null pointer");
        DRESSI_REQUIRE(mw >= 1 && mh >= 1, "EquirectSample grad: empty map");
        equirect_sample_bwd_op(gy, dir, (long long)n_px, int(mw), int(mh),
                               int(n_comp), g_map, as_stream(stream));
    });
}

int dressi_irradiance_conv(const float* env, uint32_t sw, uint32_t sh,
                           uint32_t n_comp, uint32_t ow, uint32_t oh,
                           float* out, void* stream) {
    return guarded([&] {
        ibl_checks(env, out, n_comp);
        DRESSI_REQUIRE(sw && sh && ow && oh, "IrradianceConv: empty image");
        cudaStream_t s = as_stream(stream);
        AsyncScratch sc(env_conv_scratch_floats(int(sw), int(sh), int(ow),
                                                int(oh)) * 4, s);
        irradiance_conv_op(env, int(sw), int(sh), int(n_comp), int(ow),
                           int(oh), out, static_cast<float*>(sc.p), s);
    });
}

int dressi_irradiance_conv_grad(const float* gy, uint32_t ow, uint32_t oh,
                                uint32_t n_comp, uint32_t sw, uint32_t sh,
                                float* g_env, void* stream) {
    return guarded([&] {
        ibl_checks(gy, g_env, n_comp);
        DRESSI_REQUIRE(sw && sh && ow && oh, "IrradianceConv grad: empty image");
        cudaStream_t s = as_stream(stream);
        AsyncScratch sc(env_conv_scratch_floats(int(sw), int(sh), int(ow),
                                                int(oh)) * 4, s);
        irradiance_conv_bwd_op(gy, int(ow), int(oh), int(n_comp), int(sw),
                               int(sh), g_env, static_cast<float*>(sc.p), s);
    });
}

int dressi_prefilter_conv(const float* env, uint32_t sw, uint32_t sh,
                          uint32_t n_comp, uint32_t ow, uint32_t oh,
                          float roughness, float* out, void* stream) {
    return guarded([&] {
        ibl_checks(env, out, n_comp);
        DRESSI_REQUIRE(sw && sh && ow && oh, "PrefilterConv: empty image");
        cudaStream_t s = as_stream(stream);
        AsyncScratch sc(env_conv_scratch_floats(int(sw), int(sh), int(ow),
                                                int(oh)) * 4, s);
        prefilter_conv_op(env, int(sw), int(sh), int(n_comp), int(ow),
                          int(oh), roughness, out,
                          static_cast<float*>(sc.p), s);
    });
}

int dressi_prefilter_conv_grad(const float* gy, uint32_t ow, uint32_t oh,
                               uint32_t n_comp, uint32_t sw, uint32_t sh,
                               float roughness, float* g_env, void* stream) {
    return guarded([&] {
        ibl_checks(gy, g_env, n_comp);
        DRESSI_REQUIRE(sw && sh && ow && oh, "PrefilterConv grad: empty image");
        cudaStream_t s = as_stream(stream);
        AsyncScratch sc(env_conv_scratch_floats(int(sw), int(sh), int(ow),
                                                int(oh)) * 4, s);
        prefilter_conv_bwd_op(gy, int(ow), int(oh), int(n_comp), int(sw),
                              int(sh), roughness, g_env,
                              static_cast<float*>(sc.p), s);
    });
}

int dressi_brdf_lut(uint32_t w, uint32_t h, uint32_t n_samples, float* out,
                    void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(out, "null pointer");
        DRESSI_REQUIRE(w && h && n_samples,
                       "BrdfIntegrationLut: empty size or no samples");
        brdf_lut_op(int(w), int(h), int(n_samples), out, as_stream(stream));
    });
}

int dressi_avg_pool2x2(const float* x, uint32_t w, uint32_t h,
                       uint32_t n_comp, float* out, void* stream) {
    return guarded([&] {
        ibl_checks(x, out, n_comp);
        DRESSI_REQUIRE(w >= 2 && h >= 2 && w % 2 == 0 && h % 2 == 0,
                       "AvgPool2x2: even sizes only");
        avg_pool2x2_op(x, int(w), int(h), int(n_comp), out, as_stream(stream));
    });
}

int dressi_avg_pool2x2_grad(const float* gy, uint32_t w, uint32_t h,
                            uint32_t n_comp, float* g_x, void* stream) {
    return guarded([&] {
        ibl_checks(gy, g_x, n_comp);
        DRESSI_REQUIRE(w >= 2 && h >= 2 && w % 2 == 0 && h % 2 == 0,
                       "AvgPool2x2 grad: even sizes only");
        avg_pool2x2_bwd_op(gy, int(w), int(h), int(n_comp), g_x,
                           as_stream(stream));
    });
}

int dressi_screen_coord(uint32_t w, uint32_t h, float* out, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(!(w == 1 && h == 1),
                       "ScreenCoord: size must be non-uniform");
        DRESSI_REQUIRE(out || size_t(w) * h == 0, "null pointer");
        screen_coord_op(int(w), int(h), out, as_stream(stream));
    });
}

int dressi_lookup_faces(const float* attr, uint32_t n_verts, uint32_t n_comp,
                        const float* faces, uint32_t n_faces, uint32_t corner,
                        float* out, uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4, "n_comp must be 1..4");
        DRESSI_REQUIRE(corner < 3, "LookupFaces: corner must be 0, 1 or 2");
        DRESSI_REQUIRE((attr && faces && out) || n_faces == 0,
                       "null pointer");
        lookup_faces_op(attr, int(n_verts), int(n_comp), faces, int(n_faces),
                        int(corner), out, status, as_stream(stream));
    });
}

int dressi_lookup_faces_grad(const float* gy, uint32_t n_comp,
                             const float* faces, uint32_t n_faces,
                             const float* vf, uint32_t n_verts,
                             uint32_t max_deg, uint32_t corner, float* g_attr,
                             uint32_t* status, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4, "n_comp must be 1..4");
        DRESSI_REQUIRE(corner < 3, "LookupFaces: corner must be 0, 1 or 2");
        DRESSI_REQUIRE((gy && faces && vf && g_attr) || n_verts == 0,
                       "null pointer");
        lookup_faces_bwd_op(gy, int(n_comp), faces, int(n_faces), vf,
                            int(n_verts), int(max_deg), int(corner), g_attr,
                            status, as_stream(stream));
    });
}

int dressi_face_fetch(const float* attr, uint32_t n_faces, uint32_t n_comp,
                      const float* idx, uint32_t w, uint32_t h, float* out,
                      void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4, "n_comp must be 1..4");
        DRESSI_REQUIRE((attr || n_faces == 0) && idx && out, "null pointer");
        face_fetch_op(attr, int(n_faces), int(n_comp), idx,
                      (long long)w * h, out, as_stream(stream));
    });
}

int dressi_face_fetch_grad(const float* gy, uint32_t n_comp, const float* idx,
                           uint32_t w, uint32_t h, const float* prj0,
                           const float* prj1, const float* prj2,
                           uint32_t n_faces, float seed, float radius_px,
                           uint32_t n_samples, float* g_attr, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(n_comp >= 1 && n_comp <= 4, "n_comp must be 1..4");
        DRESSI_REQUIRE(radius_px > 0.f || n_samples == 0,
                       "FaceFetch: radius must be positive (or n_samples == 0 "
                       "for the exact backward)");
        DRESSI_REQUIRE((gy && idx && prj0 && prj1 && prj2 && g_attr) ||
                               n_faces == 0,
                       "null pointer");
        face_fetch_bwd_op(gy, int(n_comp), idx, int(w), int(h), prj0, prj1,
                          prj2, int(n_faces), seed, radius_px, int(n_samples),
                          g_attr, as_stream(stream));
    });
}

int dressi_pbr_plan_create(const dressi_pbr_desc* desc, dressi_plan* out) {
    return guarded([&] {
        DRESSI_REQUIRE(desc && out, "null pointer");
        DRESSI_REQUIRE(desc->struct_size == sizeof(dressi_pbr_desc),
                       "dressi_pbr_desc: struct_size mismatch");
        DRESSI_REQUIRE(desc->n_verts > 0 && desc->n_faces > 0 &&
                               desc->n_views > 0 && desc->res > 0,
                       "PBR plan: empty mesh, views or screen");
        DRESSI_REQUIRE(desc->pos && desc->normal && desc->uv && desc->faces &&
                               desc->mvps && desc->frames && desc->light,
                       "null pointer");
        auto pow2 = [](uint32_t x) { return x && !(x & (x - 1)); };
        DRESSI_REQUIRE(desc->tex_size >= 1 && desc->tex_size <= 8192,
                       "PBR plan: tex_size 1..8192");
        DRESSI_REQUIRE(pow2(desc->env_w) && pow2(desc->env_h) &&
                               desc->env_w >= 2 && desc->env_h >= 2,
                       "PBR plan: env sizes must be powers of two");
        DRESSI_REQUIRE(desc->levels >= 2 && desc->levels <= kPbrMaxLevels,
                       "PBR plan: 2..8 prefilter levels");
        DRESSI_REQUIRE(desc->loss_kind == 1 || desc->loss_kind == 2,
                       "PBR plan: loss_kind 1 (L1) or 2 (L2)");
        DRESSI_REQUIRE(desc->lut_size >= 2 && desc->lut_samples >= 1,
                       "PBR plan: lut_size >= 2, lut_samples >= 1");
        DRESSI_REQUIRE(desc->res <= 16384, "PBR plan: res > 16384");
        *out = nullptr;
        DeviceGuard dg(desc->device);
        auto pl = std::make_unique<dressi_plan_s>();
        pl->kind = dressi_plan_s::kPbr;
        pl->device = desc->device;
        PbrDims& d = pl->pd;
        d.views = int(desc->n_views);
        d.res = int(desc->res);
        d.tex = int(desc->tex_size);
        d.ew = int(desc->env_w);
        d.eh = int(desc->env_h);
        d.levels = int(desc->levels);
        d.n_verts = int(desc->n_verts);
        d.n_faces = int(desc->n_faces);
        d.lut_w = d.lut_h = int(desc->lut_size);
        d.lut_samples = int(desc->lut_samples);
        d.loss_kind = int(desc->loss_kind);
        d.inv_n = 1.f / (float(desc->res) * float(desc->res) * 3.f);
        d.lr = desc->lr;
        d.b1 = desc->beta1;
        d.b2 = desc->beta2;
        d.eps = desc->eps;
        // PoolTo (ibl.cpp:14-20): halve until the size fits
        auto pools_to = [&](int mw, int mh) {
            int k = 0, w = d.ew, h = d.eh;
            while (w > mw || h > mh) {
                w /= 2;
                h /= 2;
                k++;
            }
            return k;
        };
        const int ki = pools_to(64, 32), kp = pools_to(128, 64);
        d.n_pool = std::max(ki, kp);
        d.irr_pool = ki - 1;
        d.pref_pool = kp - 1;
        d.irr_sw = d.ew >> ki;
        d.irr_sh = d.eh >> ki;
        d.pref_sw = d.ew >> kp;
        d.pref_sh = d.eh >> kp;
        d.irr_w = 32;
        d.irr_h = 16;
        int off = 0;
        for (int k = 0; k < d.n_pool; k++) {
            d.pool_off[k] = off;
            off += (d.ew >> (k + 1)) * (d.eh >> (k + 1)) * 3;
        }
        d.pool_floats = off;
        // prefilter levels (ibl.cpp:41-60): min(128x64, src), halving
        int lw = std::min(128, d.pref_sw), lh = std::min(64, d.pref_sh);
        int texels = 0;
        d.smem_level0 = d.levels;
        for (int i = 0; i < d.levels; i++) {
            DRESSI_REQUIRE(lw * lh > 1,
                           "PBR plan: a prefilter level would be 1x1");
            d.lw[i] = lw;
            d.lh[i] = lh;
            d.loff[i] = texels;
            texels += lw * lh;
            const float rough = float(i) / float(d.levels - 1);
            d.alpha[i] = prefilter_alpha(rough);
            lw = lw > 1 ? lw / 2 : 1;
            lh = lh > 1 ? lh / 2 : 1;
        }
        d.pref_texels = texels;
        d.loff[d.levels] = texels;
        // the pixel kernel accumulates the irradiance gradient and the
        // prefilter levels from smem_level0 on in shared memory (the levels
        // are at most 128x64, so all of them fit in practice)
        constexpr int kPbrSmemBudget = 200 * 1024;
        d.smem_level0 = 0;
        while (d.smem_level0 < d.levels &&
               size_t(d.irr_w * d.irr_h + texels - d.loff[d.smem_level0]) * 12 >
                       size_t(kPbrSmemBudget))
            d.smem_level0++;
        int dc = 0;
        d.dir_irr_src = dc;
        dc += d.irr_sw * d.irr_sh;
        d.dir_irr_out = dc;
        dc += d.irr_w * d.irr_h;
        d.dir_pref_src = dc;
        dc += d.pref_sw * d.pref_sh;
        for (int i = 0; i < d.levels; i++) {
            d.dir_lvl[i] = dc;
            dc += d.lw[i] * d.lh[i];
        }
        d.dir_count = dc;
        int sms = 0;
        DRESSI_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount,
                                           desc->device));
        d.pixel_ctas = std::max(1, sms) * pbr_pixel_blocks_per_sm(d);
        const int hist = desc->loss_history ? int(desc->loss_history) : 4096;
        const size_t V = desc->n_verts, F = desc->n_faces, NV = desc->n_views;
        const size_t R2 = size_t(desc->res) * desc->res;
        const size_t T2 = size_t(desc->tex_size) * desc->tex_size;
        const size_t E = size_t(desc->env_w) * desc->env_h;
        const size_t NP = T2 * 6 + E * 3;
        auto carve = [&](Arena& a) {
            PbrBuffers& b = pl->pb;
            b.params = a.take<float>(NP);
            b.grad = a.take<float>(NP);
            b.adam_m = a.take<float>(NP);
            b.adam_v = a.take<float>(NP);
            b.scalars = a.take<float>(4);
            b.pools = a.take<float>(std::max(d.pool_floats, 1));
            b.g_pools = a.take<float>(std::max(d.pool_floats, 1));
            b.irr = a.take<float>(size_t(d.irr_w) * d.irr_h * 3);
            b.g_irr = a.take<float>(size_t(d.irr_w) * d.irr_h * 3);
            b.pref = a.take<float>(size_t(texels) * 3);
            b.g_pref = a.take<float>(size_t(texels) * 3);
            b.pref_norm = a.take<float>(size_t(texels));
            b.dirs = a.take<float4>(size_t(dc));
            b.lut = a.take<float>(size_t(d.lut_w) * d.lut_h * 2);
            b.mat4 = a.take<float4>(T2);
            b.metal = a.take<float>(T2);
            b.env4 = a.take<float4>(E);
            b.ibl4 = a.take<float4>(size_t(d.irr_w) * d.irr_h + texels);
            b.gmat4 = a.take<float4>(T2);
            b.gmetal = a.take<float>(T2);
            b.loss_slots = a.take<double>(kLossSlots);
            b.loss_hist = a.take<float>(size_t(hist));
            b.hist_cap = hist;
            b.px = a.take<float>(NV * R2 * 12);
            b.px_side = a.take<float4>(NV * R2);
            b.target = a.take<float>(NV * R2 * 3);
            b.pos = a.take<float>(V * 3);
            b.nrm = a.take<float>(V * 3);
            b.uvh_attr = a.take<float>(V * 4);
            b.faces = a.take<float>(F * 3);
            b.mvps = a.take<float>(NV * 16);
            b.frames = a.take<float>(NV * 12);
            b.light = a.take<float>(6);
            b.status = a.take<uint32_t>(4);
        };
        Arena dry;
        carve(dry);
        pl->mem_bytes = dry.used + 256;
        DRESSI_CUDA(cudaMalloc(&pl->mem, pl->mem_bytes));
        Arena a{static_cast<char*>(pl->mem), pl->mem_bytes, 0};
        carve(a);
        PbrBuffers& b = pl->pb;
        DRESSI_CUDA(cudaMemset(pl->mem, 0, pl->mem_bytes));
        DRESSI_CUDA(cudaMemcpy(b.pos, desc->pos, V * 12, cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(b.nrm, desc->normal, V * 12,
                               cudaMemcpyHostToDevice));
        {
            std::vector<float> uvh(V * 4);
            for (size_t i = 0; i < V; i++) {
                uvh[i * 4 + 0] = desc->uv[i * 2 + 0];
                uvh[i * 4 + 1] = desc->uv[i * 2 + 1];
                uvh[i * 4 + 2] = 1.f;
                uvh[i * 4 + 3] = 0.f;
            }
            DRESSI_CUDA(cudaMemcpy(b.uvh_attr, uvh.data(), V * 16,
                                   cudaMemcpyHostToDevice));
        }
        DRESSI_CUDA(cudaMemcpy(b.faces, desc->faces, F * 12,
                               cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(b.mvps, desc->mvps, NV * 64,
                               cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(b.frames, desc->frames, NV * 48,
                               cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(b.light, desc->light, 24, cudaMemcpyHostToDevice));
        // set-up scratch: clip positions, raster workspace, G-buffer
        HardDims hd;
        hd.W = hd.H = d.res;
        hd.views = d.views;
        hd.n_faces = d.n_faces;
        hd.n_verts = d.n_verts;
        hd.n_comp = 4;
        hd.attr_shared = 1;
        const size_t ws = hard_workspace_bytes(hd);
        Arena st_dry;
        auto carve_setup = [&](Arena& q) {
            b.clip = q.take<float>(NV * V * 4);
            b.hard_ws = q.take<char>(ws);
            b.gbuf_uvh = q.take<float>(NV * R2 * 4);
            b.gbuf_n = q.take<float>(NV * R2 * 3);
            b.gbuf_p = q.take<float>(NV * R2 * 3);
        };
        carve_setup(st_dry);
        void* setup_mem = nullptr;
        DRESSI_CUDA(cudaMalloc(&setup_mem, st_dry.used + 256));
        Arena st{static_cast<char*>(setup_mem), st_dry.used + 256, 0};
        carve_setup(st);
        pbr_static_setup(d, b, nullptr);
        DRESSI_CUDA(cudaDeviceSynchronize());
        cudaFree(setup_mem);
        b.clip = nullptr;
        b.hard_ws = nullptr;
        b.gbuf_uvh = b.gbuf_n = b.gbuf_p = nullptr;
        pl->set_slot(DRESSI_SLOT_PARAM, b.params, NP * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_M, b.adam_m, NP * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_V, b.adam_v, NP * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_T, b.scalars, 4);
        pl->set_slot(DRESSI_SLOT_TARGET, b.target, NV * R2 * 12);
        pl->set_slot(DRESSI_SLOT_GRAD, b.grad, NP * 4);
        pl->set_slot(DRESSI_SLOT_LOSS, b.scalars + 3, 4);
        pl->set_slot(DRESSI_SLOT_LOSS_HISTORY, b.loss_hist, size_t(hist) * 4);
        pl->set_slot(DRESSI_SLOT_RASTER, nullptr, NV * R2 * 12);
        pl->set_slot(DRESSI_SLOT_MVP, b.mvps, NV * 64);
        *out = pl.release();
    });
}

int dressi_texture_plan_create(const dressi_texture_desc* desc,
                               dressi_plan* out) {
    return guarded([&] {
        DRESSI_REQUIRE(desc && out, "null pointer");
        DRESSI_REQUIRE(desc->struct_size == sizeof(dressi_texture_desc),
                       "dressi_texture_desc: struct_size mismatch");
        DRESSI_REQUIRE(desc->n_verts > 0 && desc->n_faces > 0 &&
                               desc->n_views > 0 && desc->res > 0,
                       "texture plan: empty mesh, views or screen");
        DRESSI_REQUIRE(desc->res <= 32768, "texture plan: res > 32768");
        const uint32_t w = desc->tex_size;
        DRESSI_REQUIRE(w >= 1 && (w & (w - 1)) == 0 && w <= 16384,
                       "texture plan: tex_size must be a power of two <= 16384");
        DRESSI_REQUIRE(desc->levels >= 1 && (w >> (desc->levels - 1)) >= 1,
                       "texture plan: more mip levels than the texture has");
        DRESSI_REQUIRE(desc->pos && desc->uv && desc->faces && desc->mvps,
                       "null pointer");
        *out = nullptr;
        DeviceGuard dg(desc->device);
        auto pl = std::make_unique<dressi_plan_s>();
        pl->kind = dressi_plan_s::kTex;
        pl->device = desc->device;
        TexParams& p = pl->tp;
        p.w_tex = int(w);
        p.levels = int(desc->levels);
        p.views = int(desc->n_views);
        p.res = int(desc->res);
        p.n_verts = int(desc->n_verts);
        p.n_faces = int(desc->n_faces);
        p.lr = desc->lr;
        p.b1 = desc->beta1;
        p.b2 = desc->beta2;
        p.eps = desc->eps;
        p.inv_n = 1.f / (float(desc->res) * float(desc->res) * 3.f);
        // the pyramid-gradient scatter: one vector atomic per tap (default:
        // 0.0746 ms per C2 pixel pass on a B200) or the run-merged warp
        // scan with one atomic per run (DRESSI_C2_SCATTER=runs: 0.0772 ms)
        const char* sc = std::getenv("DRESSI_C2_SCATTER");
        p.scatter_runs = (sc && std::strcmp(sc, "runs") == 0) ? 1 : 0;
        const int hist = desc->loss_history ? int(desc->loss_history) : 4096;
        const size_t V = desc->n_verts, F = desc->n_faces, NV = desc->n_views;
        const size_t R2 = size_t(desc->res) * desc->res;
        const size_t T0 = size_t(w) * w * 3;
        const size_t nmip = tex_mip_floats(int(w), p.levels);
        const size_t ws = tex_workspace_bytes(p);
        auto carve = [&](Arena& a) {
            TexBuffers& b = pl->tb;
            b.pyr = a.take<float>(nmip);
            b.gpyr = a.take<float4>(nmip / 3);
            b.grad = a.take<float>(T0);
            b.adam_m = a.take<float>(T0);
            b.adam_v = a.take<float>(T0);
            b.scalars = a.take<float>(4);
            b.clip = a.take<float>(NV * V * 4);
            b.attr = a.take<float>(V * 3);
            b.faces = a.take<float>(F * 3);
            b.gbuf = a.take<float>(NV * R2 * 3);
            b.targets = a.take<float>(NV * R2 * 3);
            b.loss_slots = a.take<double>(kLossSlots);
            b.loss_hist = a.take<float>(size_t(hist));
            b.hist_cap = hist;
            b.status = a.take<uint32_t>(4);
            b.hard_ws = a.take<char>(ws);
        };
        Arena dry;
        carve(dry);
        pl->mem_bytes = dry.used + 256;
        DRESSI_CUDA(cudaMalloc(&pl->mem, pl->mem_bytes));
        Arena a{static_cast<char*>(pl->mem), pl->mem_bytes, 0};
        carve(a);
        DRESSI_CUDA(cudaMemset(pl->mem, 0, pl->mem_bytes));
        // static inputs: faces, the (u, v, 1) attribute, the clip positions
        std::vector<float> attr(V * 3), clip(NV * V * 4);
        for (size_t i = 0; i < V; i++) {
            attr[i * 3 + 0] = desc->uv[i * 2 + 0];
            attr[i * 3 + 1] = desc->uv[i * 2 + 1];
            attr[i * 3 + 2] = 1.f;
        }
        for (size_t v = 0; v < NV; v++) {
            const float* m = desc->mvps + v * 16;
            for (size_t i = 0; i < V; i++) {
                const float4 c = transform_clip(desc->pos[i * 3 + 0],
                                                desc->pos[i * 3 + 1],
                                                desc->pos[i * 3 + 2], m);
                float* o = &clip[(v * V + i) * 4];
                o[0] = c.x;
                o[1] = c.y;
                o[2] = c.z;
                o[3] = c.w;
            }
        }
        DRESSI_CUDA(cudaMemcpy(pl->tb.faces, desc->faces, F * 3 * sizeof(float),
                               cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(pl->tb.attr, attr.data(), V * 3 * sizeof(float),
                               cudaMemcpyHostToDevice));
        DRESSI_CUDA(cudaMemcpy(pl->tb.clip, clip.data(),
                               clip.size() * sizeof(float),
                               cudaMemcpyHostToDevice));
        tex_static_setup(pl->tp, pl->tb, nullptr);
        DRESSI_CUDA(cudaDeviceSynchronize());
        pl->set_slot(DRESSI_SLOT_PARAM, pl->tb.pyr, T0 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_M, pl->tb.adam_m, T0 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_V, pl->tb.adam_v, T0 * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_T, pl->tb.scalars, 4);
        pl->set_slot(DRESSI_SLOT_TARGET, pl->tb.targets, NV * R2 * 3 * 4);
        pl->set_slot(DRESSI_SLOT_GRAD, pl->tb.grad, T0 * 4);
        pl->set_slot(DRESSI_SLOT_LOSS, pl->tb.scalars + 3, 4);
        pl->set_slot(DRESSI_SLOT_LOSS_HISTORY, pl->tb.loss_hist, size_t(hist) * 4);
        pl->set_slot(DRESSI_SLOT_RASTER, nullptr, NV * R2 * 3 * 4);
        pl->set_slot(DRESSI_SLOT_MVP, nullptr, NV * 16 * 4);
        *out = pl.release();
    });
}

int dressi_image_fit_plan_create(uint32_t width, uint32_t height, float lr,
                                 int device, dressi_plan* out) {
    return guarded([&] {
        DRESSI_REQUIRE(out, "null pointer");
        DRESSI_REQUIRE(width > 0 && height > 0, "image fit: empty image");
        *out = nullptr;
        DeviceGuard dg(device);
        auto pl = std::make_unique<dressi_plan_s>();
        pl->kind = dressi_plan_s::kFit;
        pl->device = device;
        pl->n = size_t(width) * height * 4;
        pl->lr = lr;
        const size_t n = pl->n;
        auto carve = [&](Arena& a) {
            FitBuffers& f = pl->fb;
            f.param = a.take<float>(n);
            f.target = a.take<float>(n);
            f.m = a.take<float>(n);
            f.v = a.take<float>(n);
            f.scalars = a.take<float>(4);
            f.loss_acc = a.take<double>(1);
            f.hist_cap = 4096;
            f.loss_hist = a.take<float>(4096);
            f.done = a.take<unsigned>(1);
        };
        Arena dry;
        carve(dry);
        pl->mem_bytes = dry.used + 256;
        DRESSI_CUDA(cudaMalloc(&pl->mem, pl->mem_bytes));
        Arena a{static_cast<char*>(pl->mem), pl->mem_bytes, 0};
        carve(a);
        DRESSI_CUDA(cudaMemset(pl->mem, 0, pl->mem_bytes));
        pl->set_slot(DRESSI_SLOT_PARAM, pl->fb.param, n * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_M, pl->fb.m, n * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_V, pl->fb.v, n * 4);
        pl->set_slot(DRESSI_SLOT_ADAM_T, pl->fb.scalars, 4);
        pl->set_slot(DRESSI_SLOT_TARGET, pl->fb.target, n * 4);
        pl->set_slot(DRESSI_SLOT_LOSS, pl->fb.scalars + 3, 4);
        pl->set_slot(DRESSI_SLOT_LOSS_HISTORY, pl->fb.loss_hist, 4096 * 4);
        *out = pl.release();
    });
}

static dressi_plan_s::Slot& plan_slot(dressi_plan p, int slot) {
    DRESSI_REQUIRE(p, "null plan");
    DRESSI_REQUIRE(slot >= 0 && slot < 10 && p->slots[slot].bytes > 0,
                   "plan has no such slot");
    return p->slots[slot];
}

int dressi_plan_slot_bytes(dressi_plan p, int slot, size_t* bytes) {
    return guarded([&] {
        DRESSI_REQUIRE(bytes, "null pointer");
        *bytes = plan_slot(p, slot).bytes;
    });
}

int dressi_plan_slot_ptr(dressi_plan p, int slot, void** ptr) {
    return guarded([&] {
        DRESSI_REQUIRE(ptr, "null pointer");
        auto& s = plan_slot(p, slot);
        DRESSI_REQUIRE(s.ptr, "slot is not resident (render it first)");
        *ptr = s.ptr;
    });
}

int dressi_plan_upload(dressi_plan p, int slot, const void* src, size_t bytes,
                       int src_is_device, void* stream) {
    return guarded([&] {
        auto& s = plan_slot(p, slot);
        DRESSI_REQUIRE(src, "null pointer");
        DRESSI_REQUIRE(s.ptr, "slot is not uploadable");
        DRESSI_REQUIRE(bytes == s.bytes,
                       "upload size " + std::to_string(bytes) +
                               " != slot size " + std::to_string(s.bytes));
        DeviceGuard dg(p->device);
        DRESSI_CUDA(cudaMemcpyAsync(s.ptr, src, bytes,
                                    src_is_device ? cudaMemcpyDeviceToDevice
                                                  : cudaMemcpyHostToDevice,
                                    as_stream(stream)));
    });
}

int dressi_plan_download(dressi_plan p, int slot, void* dst, size_t bytes,
                         int dst_is_device, void* stream) {
    return guarded([&] {
        auto& s = plan_slot(p, slot);
        DRESSI_REQUIRE(dst, "null pointer");
        DRESSI_REQUIRE(s.ptr, "slot is not resident (render it first)");
        DRESSI_REQUIRE(bytes == s.bytes,
                       "download size " + std::to_string(bytes) +
                               " != slot size " + std::to_string(s.bytes));
        DeviceGuard dg(p->device);
        DRESSI_CUDA(cudaMemcpyAsync(dst, s.ptr, bytes,
                                    dst_is_device ? cudaMemcpyDeviceToDevice
                                                  : cudaMemcpyDeviceToHost,
                                    as_stream(stream)));
    });
}

int dressi_plan_render_targets(dressi_plan p, const float* target_pos_host,
                               void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(p && target_pos_host, "null pointer");
        DRESSI_REQUIRE(p->kind != dressi_plan_s::kFit,
                       "render_targets: not a silhouette or texture plan");
        DeviceGuard dg(p->device);
        cudaStream_t s = as_stream(stream);
        if (p->kind == dressi_plan_s::kPbr) {
            // the ground-truth parameters [albedo | mr | env]
            const size_t n = p->slots[DRESSI_SLOT_PARAM].bytes;
            AsyncScratch gt(n, s);
            DRESSI_CUDA(cudaMemcpyAsync(gt.p, target_pos_host, n,
                                        cudaMemcpyHostToDevice, s));
            pbr_render(p->pd, p->pb, static_cast<const float*>(gt.p),
                       p->pb.target, s);
            DRESSI_CUDA(cudaStreamSynchronize(s));
            return;
        }
        if (p->kind == dressi_plan_s::kTex) {
            const size_t tb = size_t(p->tp.w_tex) * p->tp.w_tex * 3 * sizeof(float);
            AsyncScratch gt(tb, s);
            DRESSI_CUDA(cudaMemcpyAsync(gt.p, target_pos_host, tb,
                                        cudaMemcpyHostToDevice, s));
            tex_render_targets(p->tp, p->tb, static_cast<float*>(gt.p), s);
            DRESSI_CUDA(cudaStreamSynchronize(s));
            return;
        }
        const size_t bytes = size_t(p->p.n_verts) * 3 * sizeof(float);
        AsyncScratch tp(bytes, s);
        DRESSI_CUDA(cudaMemcpyAsync(tp.p, target_pos_host, bytes,
                                    cudaMemcpyHostToDevice, s));
        if (p->kind == dressi_plan_s::kAa)
            aa_render_targets(p->p, p->ab, static_cast<float*>(tp.p), s);
        else
            sil_render_targets(p->d, p->p, p->b, static_cast<float*>(tp.p), s);
        // the host array must stay valid until the copy ran
        DRESSI_CUDA(cudaStreamSynchronize(s));
    });
}

int dressi_plan_exec(dressi_plan p, uint32_t n_iters, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(p, "null plan");
        DeviceGuard dg(p->device);
        p->grow_bins_if_needed(as_stream(stream));
        p->ensure_graph();
        for (uint32_t i = 0; i < n_iters; i++)
            DRESSI_CUDA(cudaGraphLaunch(p->exec, as_stream(stream)));
    });
}

int dressi_plan_exec_phase(dressi_plan p, int phase, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(p, "null plan");
        DRESSI_REQUIRE(p->kind != dressi_plan_s::kFit,
                       "exec_phase: not a silhouette or texture plan");
        DRESSI_REQUIRE(phase == 0 || phase == 1, "exec_phase: phase is 0 or 1");
        DeviceGuard dg(p->device);
        cudaStream_t s = as_stream(stream);
        // each phase is one CUDA-graph replay (captured on first use)
        if (phase == 0 && p->kind == dressi_plan_s::kSil)
            p->grow_bins_if_needed(s);
        p->ensure_phase_graph(phase);
        DRESSI_CUDA(cudaGraphLaunch(p->phase_exec[phase], s));
    });
}

int dressi_plan_set_deterministic(dressi_plan p, int on) {
    return guarded([&] {
        DRESSI_REQUIRE(p, "null plan");
        DRESSI_REQUIRE(p->kind == dressi_plan_s::kSil && !p->p.paper,
                       "set_deterministic: HardSoftRas silhouette plans only");
        DeviceGuard dg(p->device);
        DRESSI_CUDA(cudaDeviceSynchronize());
        if (p->exec) {
            cudaGraphExecDestroy(p->exec);
            p->exec = nullptr;
        }
        for (auto& g : p->phase_exec) {
            if (g) cudaGraphExecDestroy(g);
            g = nullptr;
        }
        SilBuffers& b = p->b;
        if (!on) {
            if (p->det_mem) cudaFree(p->det_mem);
            p->det_mem = nullptr;
            b.det_pix = nullptr;
            b.det_part = nullptr;
            b.det_vf = nullptr;
            b.det_vf_deg = 0;
            b.det_touch = nullptr;
            return;
        }
        if (p->det_mem) return;
        const SilParams& sp = p->p;
        std::vector<float> faces(size_t(sp.n_faces) * 3);
        DRESSI_CUDA(cudaMemcpy(faces.data(), b.faces, faces.size() * 4,
                               cudaMemcpyDeviceToHost));
        std::vector<float> vf;
        int vf_deg = 0;
        vertex_faces_table(faces.data(), sp.n_faces, sp.n_verts, &vf, &vf_deg);
        const size_t px = size_t(sp.views) * sp.res * sp.res;
        auto carve = [&](Arena& a) {
            b.det_pix = a.take<float2>(px);
            b.det_part = a.take<float4>(size_t(sp.views) * sp.n_faces * 3);
            b.det_vf = a.take<float>(vf.size());
            b.det_touch = a.take<uint8_t>(size_t(sp.views) * sp.n_faces);
        };
        Arena dry;
        carve(dry);
        DRESSI_CUDA(cudaMalloc(&p->det_mem, dry.used + 256));
        Arena a{static_cast<char*>(p->det_mem), dry.used + 256, 0};
        carve(a);
        DRESSI_CUDA(cudaMemset(b.det_touch, 0, size_t(sp.views) * sp.n_faces));
        b.det_vf_deg = vf_deg;
        DRESSI_CUDA(cudaMemcpy(const_cast<float*>(b.det_vf), vf.data(),
                               vf.size() * 4, cudaMemcpyHostToDevice));
    });
}

int dressi_plan_record_phase(dressi_plan p, int phase, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(p, "null plan");
        DRESSI_REQUIRE(p->kind != dressi_plan_s::kFit,
                       "record_phase: not a silhouette or texture plan");
        DRESSI_REQUIRE(phase == 0 || phase == 1,
                       "record_phase: phase is 0 or 1");
        DeviceGuard dg(p->device);
        // the phase's kernels go straight onto the stream, so a capture the
        // caller runs on it (with its collective in between) records them
        p->record_phase(phase, as_stream(stream));
    });
}

int dressi_plan_render(dressi_plan p, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(p, "null plan");
        DRESSI_REQUIRE(p->kind != dressi_plan_s::kFit,
                       "render: not a silhouette or texture plan");
        DeviceGuard dg(p->device);
        cudaStream_t s = as_stream(stream);
        auto& slot = p->slots[DRESSI_SLOT_RASTER];
        if (!slot.ptr) DRESSI_CUDA(cudaMalloc(&slot.ptr, slot.bytes));
        if (p->kind == dressi_plan_s::kTex) {
            tex_predict(p->tp, p->tb, static_cast<float*>(slot.ptr), s);
            DRESSI_CUDA(cudaStreamSynchronize(s));
            return;
        }
        if (p->kind == dressi_plan_s::kPbr) {
            pbr_render(p->pd, p->pb, p->pb.params,
                       static_cast<float*>(slot.ptr), s);
            DRESSI_CUDA(cudaStreamSynchronize(s));
            return;
        }
        if (p->kind == dressi_plan_s::kAa) {
            aa_sil_predict(p->p, p->ab, static_cast<float*>(slot.ptr), s);
            DRESSI_CUDA(cudaStreamSynchronize(s));
            return;
        }
        // A forward/backward pass whose side effects are undone: the Adam
        // counter advance is rolled back and the gradient buffers cleared.
        float t_saved = 0.f;
        DRESSI_CUDA(cudaMemcpyAsync(&t_saved, p->b.scalars, 4,
                                    cudaMemcpyDeviceToHost, s));
        DRESSI_CUDA(cudaStreamSynchronize(s));
        sil_forward_backward(p->d, p->p, p->b, static_cast<float*>(slot.ptr),
                             s);
        sil_grad_reduce(p->p, p->b, false, s);
        DRESSI_CUDA(cudaMemcpyAsync(p->b.scalars, &t_saved, 4,
                                    cudaMemcpyHostToDevice, s));
        DRESSI_CUDA(cudaStreamSynchronize(s));
    });
}

int dressi_plan_status(dressi_plan p, uint32_t* word, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(p && word, "null pointer");
        DeviceGuard dg(p->device);
        cudaStream_t s = as_stream(stream);
        *word = 0;
        if (p->kind == dressi_plan_s::kSil) {
            DRESSI_CUDA(cudaMemcpyAsync(word, p->b.soft.status, 4,
                                        cudaMemcpyDeviceToHost, s));
        } else if (p->kind == dressi_plan_s::kAa) {
            DRESSI_CUDA(cudaMemcpyAsync(word, p->ab.status, 4,
                                        cudaMemcpyDeviceToHost, s));
        } else if (p->kind == dressi_plan_s::kTex) {
            DRESSI_CUDA(cudaMemcpyAsync(word, p->tb.status, 4,
                                        cudaMemcpyDeviceToHost, s));
        } else if (p->kind == dressi_plan_s::kPbr) {
            DRESSI_CUDA(cudaMemcpyAsync(word, p->pb.status, 4,
                                        cudaMemcpyDeviceToHost, s));
        }
        DRESSI_CUDA(cudaStreamSynchronize(s));
    });
}

int dressi_plan_launches_per_iter(dressi_plan p, uint32_t* n) {
    return guarded([&] {
        DRESSI_REQUIRE(p && n, "null pointer");
        DeviceGuard dg(p->device);
        p->ensure_graph();
        *n = p->kernels_per_iter;
    });
}

int dressi_plan_profile(dressi_plan p, uint32_t n_iters, void* stream,
                        uint32_t max_kernels, const char** names,
                        float* total_ms, uint32_t* launches,
                        uint32_t* n_kernels) {
    return guarded([&] {
        DRESSI_REQUIRE(p && n_kernels, "null pointer");
        DeviceGuard dg(p->device);
        cudaStream_t s = as_stream(stream);
        KernelProfiler prof;
        current_profiler() = &prof;
        try {
            for (uint32_t i = 0; i < n_iters; i++) p->record_iteration(s);
        } catch (...) {
            current_profiler() = nullptr;
            throw;
        }
        current_profiler() = nullptr;
        std::vector<const char*> nm;
        std::vector<double> ms;
        std::vector<int> cnt;
        prof.collect(&nm, &ms, &cnt);
        *n_kernels = uint32_t(nm.size());
        for (size_t i = 0; i < nm.size() && i < max_kernels; i++) {
            if (names) names[i] = nm[i];  // launch-site string literals
            if (total_ms) total_ms[i] = float(ms[i]);
            if (launches) launches[i] = uint32_t(cnt[i]);
        }
    });
}

int dressi_plan_destroy(dressi_plan p) {
    return guarded([&] { delete p; });
}

}  // extern "C"
