// Attribute interpolation of the dressi.torch-style ops
// (python/dressi/torch/ops.py:169-201 of the reference): per pixel of a
// rasterize output (u, v, z/w, face + 1), the face's three vertex
// attributes (LookupFaces, f_ops.cpp:1568-1619, fetched per pixel by
// FaceFetch, f_ops.cpp:1736-1799) combined as u a0 + v a1 + (1 - u - v) a2,
// and its exact VJP w.r.t. the vertex attributes (FaceFetchBwd's exact scan
// chained with LookupFacesBwd, here a per-pixel scatter).
#include "kernels.h"

namespace dressi {

namespace {

// The face of a rasterize pixel (FaceFetch: int(tid + 0.5) - 1) and its
// vertex ids (LookupFaces: uint32(int64(f + 0.5))); false for background or
// an out-of-range face. Vertex ids out of range set the status bit.
__device__ __forceinline__ bool pixel_face(float tid, const float* faces,
                                           int n_faces, int n_verts,
                                           uint32_t* status, uint32_t vi[3]) {
    const int f = x86_i32(tid + 0.5f) - 1;
    if (f < 0 || f >= n_faces) return false;
    for (int k = 0; k < 3; k++) {
        vi[k] = x86_u32_via_i64(faces[size_t(f) * 3 + k] + 0.5f);
        if (vi[k] >= uint32_t(n_verts)) {
            atomicOr(status, kStatusIndexRange);
            return false;
        }
    }
    return true;
}

__global__ void k_interpolate(const float* attr, int n_comp, int n_verts,
                              int attr_views, const float4* rast,
                              const float* faces, int n_faces, int views,
                              size_t npx_view, float* out, uint32_t* status) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= npx_view * views) return;
    const int v = int(i / npx_view);
    const float4 r = rast[i];
    float* o = out + i * n_comp;
    uint32_t vi[3];
    if (!pixel_face(r.w, faces, n_faces, n_verts, status, vi)) {
        // FaceFetch yields 0 attributes; the combination is then 0
        for (int c = 0; c < n_comp; c++) {
            const float t1 = r.x * 0.f, t2 = r.y * 0.f;
            o[c] = (t1 + t2) + ((1.f - r.x) - r.y) * 0.f;
        }
        return;
    }
    const float* a = attr + size_t(attr_views > 1 ? v : 0) * n_verts * n_comp;
    const float w = (1.f - r.x) - r.y;
    for (int c = 0; c < n_comp; c++) {
        const float t1 = r.x * a[size_t(vi[0]) * n_comp + c];
        const float t2 = r.y * a[size_t(vi[1]) * n_comp + c];
        o[c] = (t1 + t2) + w * a[size_t(vi[2]) * n_comp + c];
    }
}

__global__ void k_interpolate_grad(const float* gy, int n_comp, int n_verts,
                                   int attr_views, const float4* rast,
                                   const float* faces, int n_faces, int views,
                                   size_t npx_view, float* grad,
                                   uint32_t* status) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= npx_view * views) return;
    const int v = int(i / npx_view);
    const float4 r = rast[i];
    uint32_t vi[3];
    if (!pixel_face(r.w, faces, n_faces, n_verts, status, vi)) return;
    float* g = grad + size_t(attr_views > 1 ? v : 0) * n_verts * n_comp;
    const float wgt[3] = {r.x, r.y, (1.f - r.x) - r.y};
    const float* gp = gy + i * n_comp;
    for (int c = 0; c < n_comp; c++) {
        const float gc = gp[c];
        if (gc == 0.f) continue;
        for (int k = 0; k < 3; k++)
            atomicAdd(g + size_t(vi[k]) * n_comp + c, gc * wgt[k]);
    }
}

}  // namespace

void interpolate_op(const float* attr, int n_comp, int n_verts,
                    int attr_views, const float* rast, const float* faces,
                    int n_faces, int views, int W, int H, float* out,
                    uint32_t* status, cudaStream_t s) {
    const size_t npx = size_t(W) * H, n = npx * views;
    if (n == 0) return;
    k_interpolate<<<unsigned((n + 255) / 256), 256, 0, s>>>(
            attr, n_comp, n_verts, attr_views,
            reinterpret_cast<const float4*>(rast), faces, n_faces, views, npx,
            out, status);
    DRESSI_CUDA(cudaGetLastError());
}

void interpolate_grad_op(const float* gy, int n_comp, int n_verts,
                         int attr_views, const float* rast, const float* faces,
                         int n_faces, int views, int W, int H, float* grad,
                         uint32_t* status, cudaStream_t s) {
    const size_t npx = size_t(W) * H, n = npx * views;
    if (n == 0) return;
    k_interpolate_grad<<<unsigned((n + 255) / 256), 256, 0, s>>>(
            gy, n_comp, n_verts, attr_views,
            reinterpret_cast<const float4*>(rast), faces, n_faces, views, npx,
            grad, status);
    DRESSI_CUDA(cudaGetLastError());
}

}  // namespace dressi
