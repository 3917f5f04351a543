// Soft rasterizer kernels (face setup, binning, sweeps) and the op-level
// launchers for F::SoftClip, F::RasterizeSoft and its dist-channel backward.
// See raster_soft.cuh for the exactness argument.
#include <algorithm>
#include <cstdlib>

#include "kernels.h"

namespace dressi {

// ------------------------------------------------------------- buffers

void default_caps(SoftDims* d) {
    // Sweep-1 bins hold the faces whose hard bbox (+ margin) touches a tile
    // (~4 tiles per face on the configs' meshes); rim bins hold the soft
    // triangles touching an open 8x4 block. Entries past a bin's capacity go
    // to its set's spill list; only a full spill list makes the bin's
    // consumer scan all faces (every path is exact).
    const long long f = d->n_faces, t = std::max(d->n_tiles, 1);
    d->cap1 = int(std::min<long long>(std::max<long long>(256, 8 * ((4 * f + t - 1) / t)),
                                      1 << 16));
    d->cap2 = 1024;
    // Spill lists: room for a few overflowing bins per view.
    const long long sp = std::min<long long>(
            std::max<long long>(1 << 16, 4ll * d->views * t), 1 << 24);
    d->spill1 = d->spill2 = int(sp);
    // Test hooks: DRESSI_B200_BIN_CAP forces a (small) bin capacity so the
    // spill path can be exercised, DRESSI_B200_SPILL_CAP a small spill list
    // so the all-faces fallback can be.
    if (const char* e = std::getenv("DRESSI_B200_BIN_CAP")) {
        const long long c = std::atoll(e);
        if (c > 0) d->cap1 = d->cap2 = int(std::min<long long>(c, 1 << 16));
    }
    if (const char* e = std::getenv("DRESSI_B200_SPILL_CAP")) {
        const long long c = std::atoll(e);
        if (c >= 0) d->spill1 = d->spill2 = int(std::min<long long>(c, 1 << 24));
    }
}

void carve_soft_main(Arena& a, const SoftDims& d, SoftBuffers* b) {
    const size_t vt = size_t(d.views) * d.n_tiles;
    b->recs = a.take<FaceRec>(size_t(d.views) * std::max(d.n_faces, 1));
    b->state = a.take<int2>(size_t(d.views) * d.W * d.H);
    b->active = a.take<uint8_t>(vt * 8);
    b->sat = a.take<int>(size_t(d.views) * (d.tiles_x + 1) * (d.tiles_y + 1));
    b->kept = a.take<int>(size_t(d.views) * std::max(d.n_faces, 1));
    b->kept_n = a.take<int>(size_t(d.views));
    b->rim = a.take<int>(size_t(d.views) * std::max(d.rim_cells, 1));
    b->status = a.take<uint32_t>(4);
}

void carve_soft_bins(Arena& a, const SoftDims& d, SoftBuffers* b) {
    const size_t vt = size_t(d.views) * d.n_tiles;
    const size_t vb = vt * 8;  // 8x4-pixel blocks of the rim phase
    b->bin1.cap = d.cap1;
    b->bin1.cursor = a.take<int>(vt);
    b->bin1.list = a.take<unsigned long long>(vt * d.cap1);
    b->bin1.spill_cap = d.spill1;
    b->bin1.spill_n = a.take<int>(1);
    b->bin1.spill_key = a.take<unsigned long long>(std::max(d.spill1, 1));
    b->bin1.spill_bin = a.take<int>(std::max(d.spill1, 1));
    b->bin1.parked_n = a.take<int>(1);
    b->bin1.parked = a.take<int>(std::max<size_t>(vt, 1));
    b->bin2.cap = d.cap2;
    b->bin2.cursor = a.take<int>(vb);
    b->bin2.list = a.take<int>(vb * d.cap2);
    b->bin2.spill_cap = d.spill2;
    b->bin2.spill_n = a.take<int>(1);
    b->bin2.spill = a.take<int2>(std::max(d.spill2, 1));
    b->bin2.open_n = a.take<int>(1);
    b->bin2.take = a.take<int>(1);
    b->bin2.open = a.take<int>(std::max<size_t>(vb, 1));
    b->bin2.order = a.take<int>(std::max<size_t>(vb, 1));
    b->bin2.seg_block = a.take<int>(std::max<size_t>(kRimSplit * vb, 1));
    b->bin2.seg_index = a.take<int>(std::max<size_t>(kRimSplit * vb, 1));
    b->bin2.split = a.take<int>(std::max<size_t>(vb, 1));
    b->bin2.empty = a.take<int>(std::max<size_t>(vb, 1));
    b->bin2.order_n = a.take<int>(6);
    b->bin2.best = a.take<unsigned long long>(
            std::max<size_t>(size_t(d.views) * d.W * d.H, 1));
}

void carve_soft(Arena& a, const SoftDims& d, SoftBuffers* b) {
    carve_soft_main(a, d, b);
    carve_soft_bins(a, d, b);
}

void init_soft(const SoftDims& d, const SoftBuffers& b, cudaStream_t s) {
    const size_t vt = size_t(d.views) * d.n_tiles;
    DRESSI_CUDA(cudaMemsetAsync(b.bin1.cursor, 0, vt * sizeof(int), s));
    DRESSI_CUDA(cudaMemsetAsync(b.bin2.cursor, 0, vt * 8 * sizeof(int), s));
    DRESSI_CUDA(cudaMemsetAsync(b.bin1.spill_n, 0, sizeof(int), s));
    DRESSI_CUDA(cudaMemsetAsync(b.bin1.parked_n, 0, sizeof(int), s));
    DRESSI_CUDA(cudaMemsetAsync(b.bin2.spill_n, 0, sizeof(int), s));
    DRESSI_CUDA(cudaMemsetAsync(b.bin2.open_n, 0, sizeof(int), s));
    DRESSI_CUDA(cudaMemsetAsync(b.bin2.take, 0, sizeof(int), s));
    DRESSI_CUDA(cudaMemsetAsync(b.bin2.best, 0xff,
                                size_t(d.views) * d.W * d.H * 8, s));
    DRESSI_CUDA(cudaMemsetAsync(b.status, 0, 4 * sizeof(uint32_t), s));
    DRESSI_CUDA(cudaMemsetAsync(b.rim, 0,
                                size_t(d.views) * d.rim_cells * sizeof(int), s));
}

// ---------------------------------------------------------- face setup

// Op-level face setup: explicit soft clip / face ids / faces
// (RasterizeSoftCpu's per-face prologue, cpu_raster.cpp:260-298).
__global__ void k_face_setup_op(SoftDims d, SoftOpInputs in, SoftBuffers b) {
    // the previous rim phase has consumed the rim spill list and work list
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
        *b.bin2.spill_n = 0;
        *b.bin2.open_n = 0;
        *b.bin2.take = 0;
    }
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (f >= d.n_faces) return;
    FaceRec* out = b.recs + size_t(v) * d.n_faces + f;
    const float* sc = in.soft_clip + size_t(v) * in.n_soft * 4;
    const float* fidv = in.face_id + size_t(v) * in.n_soft;
    const float* hc = in.hard_clip + size_t(v) * in.n_hard * 4;
    const float W = float(d.W), H = float(d.H);
    float ss[3][2], sz[3], fid = 0.f;
    bool valid = true;
    for (int k = 0; k < 3; k++) {
        const uint32_t vi = x86_u32_via_i64(in.faces_soft[size_t(f) * 3 + k]);
        if (vi >= uint32_t(in.n_soft)) {
            atomicOr(b.status, kStatusIndexRange);
            valid = false;
            break;
        }
        const float* c = sc + size_t(vi) * 4;
        if (!project_clip(c[0], c[1], c[2], c[3], W, H, &ss[k][0], &ss[k][1],
                          &sz[k])) {
            valid = false;
            break;
        }
        fid = fidv[vi];
    }
    float hs[3][2], hz[3];
    uint32_t hidx[3] = {0, 0, 0};
    if (valid) {
        const uint32_t hf = x86_u32_via_i64(fid + 0.5f);
        if (hf >= uint32_t(d.n_faces)) {
            atomicOr(b.status, kStatusIndexRange);
            valid = false;
        } else {
            for (int k = 0; k < 3; k++) {
                hidx[k] = x86_u32_via_i64(in.faces_tex[size_t(hf) * 3 + k] +
                                          0.5f);
                if (hidx[k] >= uint32_t(in.n_hard)) {
                    atomicOr(b.status, kStatusIndexRange);
                    valid = false;
                    break;
                }
                const float* c = hc + size_t(hidx[k]) * 4;
                if (!project_clip(c[0], c[1], c[2], c[3], W, H, &hs[k][0],
                                  &hs[k][1], &hz[k])) {
                    valid = false;
                    break;
                }
            }
        }
    }
    FaceRec r;
    if (!valid || !build_record(ss, sz, hs, hz, fid, hidx, d.W, d.H, &r)) {
        r.flags = 0;
        *out = r;
        return;
    }
    *out = r;
    bin_sweep1(r, f, d.tiles_x, b.bin1, size_t(v) * d.n_tiles);
    mark_rim_cells(r, b.rim + size_t(v) * d.rim_cells, d.rim_cells_x);
}

static void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

void soft_rim_bins(const SoftDims& d, const SoftBuffers& b, cudaStream_t s) {
    if (d.n_faces == 0) return;
    ProfScope ps("rim_bin", s);
    // per view: which tiles hold open blocks, as a summed-area table
    k_open_sat<<<d.views, 512, 0, s>>>(d.n_tiles, d.tiles_x, d.tiles_y,
                                       b.active, b.sat, b.kept_n);
    check_launch();
    // one thread per face keeps the faces near an open block ...
    const dim3 tg((d.n_faces + 255) / 256, d.views);
    k_rim_filter<<<tg, 256, 0, s>>>(d.n_faces, d.n_tiles, d.tiles_x,
                                    d.tiles_y, b.recs, b.sat, b.kept,
                                    b.kept_n, b.bin2, b.bin1);
    check_launch();
    // ... and one warp per kept face bins it (warps past the count exit)
    const dim3 fg((d.n_faces + 7) / 8, d.views);
    k_rim_bin<<<fg, 256, 0, s>>>(d.n_faces, d.n_tiles, d.tiles_x, b.recs,
                                 b.active, b.kept, b.kept_n, b.bin2);
    check_launch();
}


void soft_raster_op(const SoftDims& d, const SoftBuffers& b,
                    const SoftOpInputs& in, float* out, cudaStream_t s) {
    if (d.n_faces > 0) {
        const dim3 fg((d.n_faces + 127) / 128, d.views);
        ProfScope ps("face_setup_op", s);
        k_face_setup_op<<<fg, 128, 0, s>>>(d, in, b);
        check_launch();
    }
    launch_sweeps(d, b, in.prev_depth, EpiRS{reinterpret_cast<float4*>(out)},
                  s);
}

// ------------------------------------------------- dist-channel backward

// SignedDistGradToTri (cpu_raster.cpp:153-175) + GatherDistGrad's
// screen->clip chain (f_ops.cpp:1335-1349). `c` are the clip vertices.
__device__ __forceinline__ void dist_grad_scatter(
        float px, float py, float g, const float hs[3][2], const float4 c[3],
        const uint32_t idx[3], float W, float H, float* grad /*[V][4]*/) {
    // SignedDistToTri over the hard triangle, then the envelope gradient.
    FaceRec r;
    r.h0x = hs[0][0]; r.h0y = hs[0][1];
    r.h1x = hs[1][0]; r.h1y = hs[1][1];
    r.h2x = hs[2][0]; r.h2y = hs[2][1];
    r.ex0 = hs[1][0] - hs[0][0]; r.ey0 = hs[1][1] - hs[0][1];
    r.ex1 = hs[2][0] - hs[1][0]; r.ey1 = hs[2][1] - hs[1][1];
    r.ex2 = hs[0][0] - hs[2][0]; r.ey2 = hs[0][1] - hs[2][1];
    r.len2_0 = r.ex0 * r.ex0 + r.ey0 * r.ey0;
    r.len2_1 = r.ex1 * r.ex1 + r.ey1 * r.ey1;
    r.len2_2 = r.ex2 * r.ex2 + r.ey2 * r.ey2;
    const TriDist td = signed_dist(px, py, r);
    const float d = fabsf(td.dist);
    if (d < 1e-6f) return;
    const int ia = td.edge, ib = (td.edge + 1) % 3;
    const float qx = hs[ia][0] + td.t * (hs[ib][0] - hs[ia][0]);
    const float qy = hs[ia][1] + td.t * (hs[ib][1] - hs[ia][1]);
    const float sgn = td.dist >= 0.f ? 1.f : -1.f;
    const float nx = (px - qx) / d;
    const float ny = (py - qy) / d;
    float gs[3][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
    gs[ia][0] = -sgn * (1.f - td.t) * nx;
    gs[ia][1] = -sgn * (1.f - td.t) * ny;
    gs[ib][0] = -sgn * td.t * nx;
    gs[ib][1] = -sgn * td.t * ny;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const float gsx = g * gs[k][0];
        const float gsy = g * gs[k][1];
        if (gsx == 0.f && gsy == 0.f) continue;
        float* dst = grad + size_t(idx[k]) * 4;
        atomicAdd(dst + 0, gsx * 0.5f * W / c[k].w);
        atomicAdd(dst + 1, gsy * 0.5f * H / c[k].w);
        atomicAdd(dst + 3, -(gsx * 0.5f * W * c[k].x + gsy * 0.5f * H * c[k].y) /
                                   (c[k].w * c[k].w));
    }
}

__global__ void k_dist_grad(const float* gy, const float4* rs,
                            const float4* clip, const float* faces,
                            int n_verts, int n_faces, int W, int H,
                            float* grad, uint32_t* status) {
    const int v = blockIdx.y;
    const size_t npx = size_t(W) * H;
    for (size_t p = size_t(blockIdx.x) * blockDim.x + threadIdx.x; p < npx;
         p += size_t(gridDim.x) * blockDim.x) {
        const float4 o = rs[v * npx + p];
        if (o.w < 0.5f) continue;
        const float g = gy[v * npx + p];
        if (g == 0.f) continue;
        const uint32_t f = x86_u32_via_i64(o.y + 0.5f);
        if (f >= uint32_t(n_faces)) {
            atomicOr(status, kStatusIndexRange);
            continue;
        }
        uint32_t idx[3];
        float hs[3][2];
        float4 c[3];
        bool valid = true;
        for (int k = 0; k < 3; k++) {
            idx[k] = x86_u32_via_i64(faces[size_t(f) * 3 + k] + 0.5f);
            if (idx[k] >= uint32_t(n_verts)) {
                atomicOr(status, kStatusIndexRange);
                valid = false;
                break;
            }
            c[k] = clip[size_t(v) * n_verts + idx[k]];
            float z;
            if (!project_clip(c[k].x, c[k].y, c[k].z, c[k].w, float(W),
                              float(H), &hs[k][0], &hs[k][1], &z)) {
                valid = false;
                break;
            }
        }
        if (!valid) continue;
        const int y = int(p / W), x = int(p % W);
        dist_grad_scatter(float(x) + 0.5f, float(y) + 0.5f, g, hs, c, idx,
                          float(W), float(H),
                          grad + size_t(v) * n_verts * 4);
    }
}

void dist_grad_op(const float* gy, const float* rs, const float* clip,
                  const float* faces, int views, int n_verts, int n_faces,
                  int W, int H, float* grad, uint32_t* status,
                  cudaStream_t s) {
    const size_t npx = size_t(W) * H;
    const int blocks = int(std::min<size_t>((npx + 255) / 256, 4096));
    k_dist_grad<<<dim3(blocks, views), 256, 0, s>>>(
            gy, reinterpret_cast<const float4*>(rs),
            reinterpret_cast<const float4*>(clip), faces, n_verts, n_faces, W,
            H, grad, status);
    check_launch();
}

// ----------------------------------------------------------- SoftClip op

__global__ void k_soft_clip(const float4* clip, const float* faces, int views,
                            int n_verts, int n_faces, float W, float H,
                            float radius, float4* out, uint32_t* status) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (f >= n_faces) return;
    float4 c[3], o[3];
    for (int k = 0; k < 3; k++) {
        const uint32_t i = x86_u32_via_i64(faces[size_t(f) * 3 + k] + 0.5f);
        if (i >= uint32_t(n_verts)) {
            atomicOr(status, kStatusIndexRange);
            for (int j = 0; j < 3; j++)
                out[(size_t(v) * n_faces + f) * 3 + j] = make_float4(0, 0, 0, 0);
            return;
        }
        c[k] = clip[size_t(v) * n_verts + i];
    }
    soft_clip_face(c, W, H, radius, o);
    for (int k = 0; k < 3; k++) out[(size_t(v) * n_faces + f) * 3 + k] = o[k];
}

void soft_clip_op(const float* clip, const float* faces, int views,
                  int n_verts, int n_faces, int W, int H, float radius,
                  float* out, uint32_t* status, cudaStream_t s) {
    if (n_faces == 0) return;
    k_soft_clip<<<dim3((n_faces + 127) / 128, views), 128, 0, s>>>(
            reinterpret_cast<const float4*>(clip), faces, views, n_verts,
            n_faces, float(W), float(H), radius, reinterpret_cast<float4*>(out),
            status);
    check_launch();
}

}  // namespace dressi
