// The paper's HardSoftRas path of the silhouette example as a fused plan
// (examples/silhouette_optimization/run.cpp:229-396), per iteration:
//
//   clip = MVP_v (pos, 1)                                     k_transform
//   K peeled soft layers (dist, face id, hard z, coverage);
//     layer k > 0 drops fragments at or in front of layer k-1's Eq.3
//     shifted depth                                 sweeps + k_paper_prev
//   per pixel: for every layer the face corners fetched (FaceFetch of the
//     LookupFaces clip positions), screen positions, the signed distance to
//     the face's edges, D_k = mask sigmoid(dist 7 / r); Eq.6 union; pred =
//     max(hard, union); loss; the backward to the fetched corners in the
//     reference autodiff's rules              k_paper_pixel (paper_pixel.cu)
//   per (view, layer, face): FaceFetch's backward (hashed edge samples, or
//     the exact bbox scan) and LookupFaces' transpose into g_clip
//                                                       k_paper_fetch_bwd
//   g_pos, regulariser, Adam: the silhouette plan's own kernels.
//
// The raster, the face ids and the sampled pixels are bit-exact with the
// reference (this file keeps the strict flags); the per-pixel chain keeps the
// reference's operation order, so gradients agree within the tolerance of
// its arithmetic and of the order of the gradient sums.
#include "kernels.h"

namespace dressi {

namespace {

__device__ __forceinline__ float step0(float x) { return x < 0.f ? 0.f : 1.f; }
__device__ __forceinline__ float clamp01(float x) {
    return x < 0.f ? 0.f : (1.f < x ? 1.f : x);
}

// Layer k + 1's peeling threshold from layer k: its Eq.3 shifted depth
// rebuilt from the output channels (run.cpp:318-327).
__global__ void k_paper_prev(const float4* layer, long long n, float inv_r,
                             float* prev) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float4 rs = layer[i];
    const float dist = rs.x, cov = rs.w;
    const float ge = step0(dist);
    prev[i] = cov * (ge * (clamp01(rs.z) * 0.5f) +
                     (1.f - ge) * (clamp01(-dist * inv_r) * 0.5f + 0.5f));
}

// FaceFetch's backward for every (view, layer, face), all three corner
// fetches at once (they share the sampling geometry: the face's corners),
// then LookupFaces' transpose: the face's three corner gradients added to
// its vertices' g_clip. The jitter seed is the Adam counter before this
// iteration's step (the example passes its counter leaf).
__global__ void k_paper_fetch_bwd(SilParams p, const float4* layers,
                                  const float4* clip, const float* faces,
                                  const float4* gfetch, const float* scalars,
                                  float* gclip) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y % p.views, k = blockIdx.y / p.views;
    if (f >= p.n_faces) return;
    const long long npx = (long long)p.res * p.res;
    const long long total = npx * p.views;
    const float4* cv = clip + size_t(v) * p.n_verts;
    uint32_t vi[3];
    float s[3][2];
    bool ok = true;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        vi[j] = x86_u32_via_i64(faces[size_t(f) * 3 + j] + 0.5f);
        const float4 c = vi[j] < uint32_t(p.n_verts) ? cv[vi[j]]
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        if (c.w <= 1e-6f) ok = false;
        s[j][0] = (c.x / c.w * 0.5f + 0.5f) * float(p.res);
        s[j][1] = (c.y / c.w * 0.5f + 0.5f) * float(p.res);
    }
    if (!ok) return;
    const float4* lay = layers + size_t(k) * total + size_t(v) * npx;
    const float4* g0 = gfetch + (size_t(k) * 3 + 0) * total + size_t(v) * npx;
    const float4* g1 = gfetch + (size_t(k) * 3 + 1) * total + size_t(v) * npx;
    const float4* g2 = gfetch + (size_t(k) * 3 + 2) * total + size_t(v) * npx;
    float4 acc[3];
#pragma unroll
    for (int j = 0; j < 3; j++) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    auto gather = [&](size_t px) {
        const float4 rs = lay[px];
        if (x86_u32_via_i64((rs.y + 1.f) * rs.w + 0.5f) != uint32_t(f) + 1u)
            return;
        const float4 a = g0[px], b = g1[px], c = g2[px];
        acc[0].x += a.x; acc[0].y += a.y; acc[0].z += a.z; acc[0].w += a.w;
        acc[1].x += b.x; acc[1].y += b.y; acc[1].z += b.z; acc[1].w += b.w;
        acc[2].x += c.x; acc[2].y += c.y; acc[2].z += c.z; acc[2].w += c.w;
    };
    const int W = p.res, H = p.res;
    if (p.n_samples == 0) {
        auto mn = [](float a, float b) { return b < a ? b : a; };
        auto mx = [](float a, float b) { return a < b ? b : a; };
        const int x0 = imax_(x86_i32(floorf(mn(mn(s[0][0], s[1][0]), s[2][0]) - 1.f)), 0);
        const int x1 = imin_(x86_i32(ceilf(mx(mx(s[0][0], s[1][0]), s[2][0]) + 1.f)), W - 1);
        const int y0 = imax_(x86_i32(floorf(mn(mn(s[0][1], s[1][1]), s[2][1]) - 1.f)), 0);
        const int y1 = imin_(x86_i32(ceilf(mx(mx(s[0][1], s[1][1]), s[2][1]) + 1.f)), H - 1);
        for (int iy = y0; iy <= y1; iy++)
            for (int ix = x0; ix <= x1; ix++) gather(size_t(iy) * W + size_t(ix));
    } else {
        const uint32_t seed_u = x86_u32_via_i64((scalars[0] - 1.f) + 0.5f);
        for (int smp = 0; smp < p.n_samples; smp++) {
            const int e = smp % 3;
            const float* a = s[e];
            const float* b = s[(e + 1) % 3];
            const float ex = b[0] - a[0], ey = b[1] - a[1];
            const float len = sqrtf(ex * ex + ey * ey);
            if (len < 1e-6f) continue;
            const float u = hash_to_unit(uint32_t(f), uint32_t(smp), seed_u, 0);
            const float o =
                    (hash_to_unit(uint32_t(f), uint32_t(smp), seed_u, 1) * 2.f - 1.f) *
                    p.radius;
            const int ix = x86_i32(floorf(a[0] + u * ex - o * (ey / len)));
            const int iy = x86_i32(floorf(a[1] + u * ey + o * (ex / len)));
            if (ix < 0 || iy < 0 || ix >= W || iy >= H) continue;
            gather(size_t(iy) * W + size_t(ix));
        }
    }
    float* gv = gclip + size_t(v) * p.n_verts * 4;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        if (vi[j] >= uint32_t(p.n_verts)) continue;
        if (acc[j].x == 0.f && acc[j].y == 0.f && acc[j].w == 0.f) continue;
        float* g = gv + size_t(vi[j]) * 4;
        atomicAdd(g + 0, acc[j].x);
        atomicAdd(g + 1, acc[j].y);
        atomicAdd(g + 2, acc[j].z);
        atomicAdd(g + 3, acc[j].w);
    }
}

void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

}  // namespace

void paper_forward_backward(const SoftDims& d, const SilParams& p,
                            const SilBuffers& b, float* rs_out,
                            cudaStream_t s) {
    sil_transform(p, b, 1, b.soft.rim, d.rim_cells, b.soft.status, s);
    const long long total = (long long)p.res * p.res * p.views;
    const unsigned blocks = unsigned((total + 255) / 256);
    for (int k = 0; k < p.peels; k++) {
        sil_face_setup(d, b, s);
        launch_sweeps(d, b.soft, k > 0 ? b.paper_prev : nullptr,
                      EpiRS{b.paper_layers + size_t(k) * total}, s);
        if (k + 1 < p.peels) {
            k_paper_prev<<<blocks, 256, 0, s>>>(b.paper_layers + size_t(k) * total,
                                                total, 1.f / p.radius,
                                                b.paper_prev);
            check_launch();
        }
    }
    if (rs_out)
        DRESSI_CUDA(cudaMemcpyAsync(rs_out, b.paper_layers, size_t(total) * 16,
                                    cudaMemcpyDeviceToDevice, s));
    {
        ProfScope ps("paper_pixel", s);
        paper_pixel_launch(p, b.paper_layers, b.targets,
                           reinterpret_cast<const float4*>(b.clip), b.faces,
                           b.paper_gfetch, b.loss_slots, blocks, s);
    }
    {
        ProfScope ps("paper_fetch_bwd", s);
        const dim3 g((p.n_faces + 127) / 128, p.views * p.peels);
        k_paper_fetch_bwd<<<g, 128, 0, s>>>(
                p, b.paper_layers, reinterpret_cast<const float4*>(b.clip),
                b.faces, b.paper_gfetch, b.scalars, b.gclip);
    }
    check_launch();
}

}  // namespace dressi
