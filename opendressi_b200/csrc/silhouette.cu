// The fused silhouette iteration (configs C3/C4, HardSoftRas path):
//
//   per view:  clip = MVP_v (pos, 1)                       k_transform
//              soft = SoftClip(clip); face records          k_face_setup_sil
//              RasterizeSoft sweeps 1/2 (exact survivor)    raster_soft.cuh
//              loss image + dL/d dist + GatherDistGrad      k_sweep2_sil
//   all views: g_pos = sum_v MVP_v^T g_clip_v               k_gpos_adam
//              regulariser (laplacian / normal != 0)        regularize.cu
//              in-graph Adam                                k_gpos_adam
//
// It computes what the reference's DressiAD::execStep computes for the
// silhouette graph of examples/silhouette_optimization/run.cpp:228-437 (per
// view: RasterizeSoft of SoftClip(clip), pred = max(hard, soft), loss =
// (target - pred)^2 / R^2, summed over views; the in-graph Adam of
// run.cpp:421-436), with the RasterizeSoft
// output, the loss image and the per-view clip gradients kept on chip
// instead of round-tripping through HBM between passes.
#include <algorithm>

#include "kernels.h"

namespace dressi {

// Per-pixel loss and dL/d dist of the silhouette graph, in the operation
// order of the reference autodiff: pred = max(cov*step(0,d),
// cov*sigmoid(d*|d|*k)), loss = (target - pred)^2 * c. Backward, op by op
// as BuildBackward emits it (src/core/build_backward.cpp:62-149 with the
// rules of src/core/f_ops.cpp): the seed 1 through Mul(., c) gives c; the
// square (Mul(diff, diff)) adds gy*diff twice; Sub gives -g to pred; Max
// passes g to its first operand where hard >= soft (Step(soft, hard)) and
// to the second elsewhere; Sigmoid multiplies by s*(1-s); the product
// d*|d|*k gives g*k*|d| + g*k*d*sign(d) to d (Step has no gradient).
__device__ __forceinline__ float sil_pixel(float dist, float cov, float target,
                                           float k, float c, float* g_dist) {
    const float step = dist < 0.f ? 0.f : 1.f;
    const float hard = cov * step;
    const float a = fabsf(dist);
    const float m1 = dist * a;
    const float m2 = m1 * k;
    const float s = 1.f / (1.f + expf(-m2));
    const float soft = cov * s;
    const float pred = std_max(hard, soft);
    const float diff = target - pred;
    const float lv = diff * diff * c;
    const float g_m4 = 1.f * c;
    const float g_diff = g_m4 * diff + g_m4 * diff;
    const float g_pred = -g_diff;
    const float mask = hard < soft ? 0.f : 1.f;
    const float g_m3 = g_pred * (1.f - mask);
    const float g_sg = g_m3 * cov;
    const float g_m2 = g_sg * (s * (1.f - s));
    const float g_m1 = g_m2 * k;
    const float sgn = float((dist > 0.f) - (dist < 0.f));
    *g_dist = g_m1 * a + (g_m1 * dist) * sgn;
    return lv;
}

// clip[v][u] = MVP_v (pos_u, 1). Block (0,0) also advances the Adam
// counter and the bias corrections of this iteration (the {1,1} part of
// the in-graph Adam: t_new = t + 1, bc = 1 - pow(beta, t_new)).
__global__ void k_transform(const float* pos, const float* mvps, int n_verts,
                            float4* clip, float* scalars, float b1, float b2,
                            int advance, int* rim, int rim_cells,
                            uint32_t* status) {
    const int v = blockIdx.y;
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    if (v == 0 && blockIdx.x == 0 && threadIdx.x == 0) status[1] = 0u;
    if (blockIdx.x == 0) {
        // this iteration's face setup re-marks the rim cells
        for (int i = threadIdx.x; i < rim_cells; i += blockDim.x)
            rim[size_t(v) * rim_cells + i] = 0;
    }
    if (advance && v == 0 && blockIdx.x == 0 && threadIdx.x == 0) {
        const float t_new = scalars[0] + 1.f;
        scalars[0] = t_new;
        scalars[1] = 1.f - powf(b1, t_new);
        scalars[2] = 1.f - powf(b2, t_new);
    }
    __shared__ float m[16];
    if (threadIdx.x < 16) m[threadIdx.x] = mvps[v * 16 + threadIdx.x];
    __syncthreads();
    if (u >= n_verts) return;
    clip[size_t(v) * n_verts + u] =
            transform_clip(pos[u * 3 + 0], pos[u * 3 + 1], pos[u * 3 + 2], m);
}

// Face records of the standard soft geometry (sequential soft faces,
// face_id = f; examples/silhouette_optimization/run.cpp:456-466).
__global__ void k_face_setup_sil(SoftDims d, const float4* clip,
                                 const float* faces, SoftBuffers b) {
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
    const float W = float(d.W), H = float(d.H);
    uint32_t idx[3];
    float4 c[3];
    for (int k = 0; k < 3; k++) {
        idx[k] = x86_u32_via_i64(faces[size_t(f) * 3 + k] + 0.5f);
        if (idx[k] >= uint32_t(d.n_verts)) {
            atomicOr(b.status, kStatusIndexRange);
            out->flags = 0;
            return;
        }
        c[k] = clip[size_t(v) * d.n_verts + idx[k]];
    }
    float4 sc[3];
    soft_clip_face(c, W, H, d.radius, sc);
    float ss[3][2], sz[3], hs[3][2], hz[3];
    bool valid = true;
    for (int k = 0; k < 3 && valid; k++) {
        valid = project_clip(sc[k].x, sc[k].y, sc[k].z, sc[k].w, W, H,
                             &ss[k][0], &ss[k][1], &sz[k]);
    }
    for (int k = 0; k < 3 && valid; k++) {
        valid = project_clip(c[k].x, c[k].y, c[k].z, c[k].w, W, H, &hs[k][0],
                             &hs[k][1], &hz[k]);
    }
    FaceRec r;
    if (!valid || !build_record(ss, sz, hs, hz, float(f), idx, d.W, d.H, &r)) {
        out->flags = 0;
        return;
    }
    *out = r;
    mark_rim_cells(r, b.rim + size_t(v) * d.rim_cells, d.rim_cells_x);
    bin_sweep1(r, f, d.tiles_x, b.bin1, size_t(v) * d.n_tiles);
}

// SignedDistGradToTri (cpu_raster.cpp:153-175) for the survivor's hard
// triangle, then GatherDistGrad's screen->clip chain (f_ops.cpp:1335-1349),
// accumulated straight into the view's clip gradient (its ColSum).
__device__ __forceinline__ void sil_scatter(float px, float py, float g,
                                            const TriDist& td,
                                            const FaceRec& r,
                                            const float4* clip_v, float W,
                                            float H, float* gclip_v) {
    const float d = fabsf(td.dist);
    if (d < 1e-6f) return;
    const float hx[3] = {r.h0x, r.h1x, r.h2x};
    const float hy[3] = {r.h0y, r.h1y, r.h2y};
    const uint32_t idx[3] = {r.i0, r.i1, r.i2};
    const int ia = td.edge, ib = (td.edge + 1) % 3;
    const float qx = hx[ia] + td.t * (hx[ib] - hx[ia]);
    const float qy = hy[ia] + td.t * (hy[ib] - hy[ia]);
    const float sgn = td.dist >= 0.f ? 1.f : -1.f;
    const float nx = (px - qx) / d;
    const float ny = (py - qy) / d;
    const float ga[2] = {-sgn * (1.f - td.t) * nx, -sgn * (1.f - td.t) * ny};
    const float gb[2] = {-sgn * td.t * nx, -sgn * td.t * ny};
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int k = j == 0 ? ia : ib;
        const float* gk = j == 0 ? ga : gb;
        const float gsx = g * gk[0];
        const float gsy = g * gk[1];
        if (gsx == 0.f && gsy == 0.f) continue;
        const float4 c = clip_v[idx[k]];
        float* dst = gclip_v + size_t(idx[k]) * 4;
        atomicAdd(dst + 0, gsx * 0.5f * W / c.w);
        atomicAdd(dst + 1, gsy * 0.5f * H / c.w);
        atomicAdd(dst + 3, -(gsx * 0.5f * W * c.x + gsy * 0.5f * H * c.y) /
                                   (c.w * c.w));
    }
}

// Epilogue of the fused iteration: the loss image (block-summed into the
// loss slots) and, for the rim pixels that carry a gradient, the per-view
// clip gradient. A pixel whose survivor is a hard fragment (dist >= 0) has
// pred = max(1, sigmoid(.)) = 1 exactly and a zero gradient, so its
// distance is never needed.
struct EpiSil {
    const float* targets;   // [views][R][R]
    const float4* clip;     // [views][V]
    float* gclip;           // [views][V][4]
    double* loss_slots;
    float4* rs_out;         // optional RasterizeSoft images
    float k, c;
    int n_verts;
    float2* det_pix;        // deterministic mode: (face, g) per pixel
    uint8_t* det_touch;     // ... and the faces that got a gradient pixel
    __device__ void operator()(const SweepArgs& a, int x, int y, bool in,
                               const Survivor& s) const {
        double lv = 0.0;
        if (in) {
            const size_t pix = size_t(a.v) * a.W * a.H + size_t(y) * a.W + x;
            const float t = targets[pix];
            const float px = float(x) + 0.5f, py = float(y) + 0.5f;
            float g = 0.f;
            if (s.face < 0) {
                lv = sil_pixel(0.f, 0.f, t, k, c, &g);
                if (rs_out) rs_out[pix] = make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
                const FaceRec& r = a.recs[s.face];
                if (s.hard && !rs_out) {
                    const float diff = t - 1.f;
                    lv = diff * diff * c;
                } else {
                    const TriDist td = signed_dist(px, py, r);
                    lv = sil_pixel(td.dist, 1.f, t, k, c, &g);
                    if (rs_out)
                        rs_out[pix] = make_float4(td.dist, r.fid,
                                                  hard_depth(px, py, r), 1.f);
                    if (g != 0.f && !det_pix)
                        sil_scatter(px, py, g, td, r,
                                    clip + size_t(a.v) * n_verts, float(a.W),
                                    float(a.H),
                                    gclip + size_t(a.v) * n_verts * 4);
                }
            }
            if (det_pix) {
                det_pix[pix] = make_float2(
                        __int_as_float(g != 0.f ? s.face : -1), g);
                if (g != 0.f && s.face >= 0)
                    det_touch[size_t(a.v) * a.n_faces + s.face] = 1;
            }
        }
        // warp sum of the loss image (no block barrier: the warps of a
        // tile finish independently)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            lv += __shfl_down_sync(0xffffffffu, lv, o);
        if ((threadIdx.x & 31) == 0) {
            const size_t slot = ((size_t(a.v) * a.n_tiles + blockIdx.x) * 8 +
                                 (threadIdx.x >> 5)) % kLossSlots;
            atomicAdd(&loss_slots[slot], lv);
        }
    }
};

// Small blocks: one thread per vertex and ~10k vertices, so 64 threads put
// a block on every SM.
constexpr int kGposThreads = 64;

// g_pos = sum_v MVP_v^T g_clip_v (TransformToClipVar's backward); zeroes
// g_clip for the next iteration. With `update`, also applies the in-graph
// Adam and (block 0) publishes the loss of this iteration.
__global__ void k_gpos_adam(SilParams p, SilBuffers b, float omb1, float omb2,
                            int do_grad, int update) {
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x == 0 && do_grad) {
        // reduce + clear the loss slots (written by the sweep epilogues);
        // the loads are issued 16 at a time ahead of the dependent adds
        __shared__ double red[kGposThreads];
        double acc = 0.0;
        static_assert(kLossSlots % (kGposThreads * 16) == 0, "slot batches");
        for (int i0 = threadIdx.x; i0 < kLossSlots; i0 += 16 * kGposThreads) {
            double v[16];
#pragma unroll
            for (int k = 0; k < 16; k++) v[k] = b.loss_slots[i0 + k * kGposThreads];
#pragma unroll
            for (int k = 0; k < 16; k++) {
                acc += v[k];
                b.loss_slots[i0 + k * kGposThreads] = 0.0;
            }
        }
        red[threadIdx.x] = acc;
        __syncthreads();
        for (int o = blockDim.x / 2; o > 0; o >>= 1) {
            if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            const float loss = float(red[0]);
            b.scalars[3] = loss;
            const int it = int(b.scalars[0]) - 1;
            if (b.hist_cap > 0 && it >= 0) b.loss_hist[it % b.hist_cap] = loss;
        }
    }
    if (u >= p.n_verts) return;
    float g0, g1, g2;
    if (do_grad) {
        g0 = g1 = g2 = 0.f;
        float4* gc4 = reinterpret_cast<float4*>(b.gclip) + u;
        // all loads first (no store in this loop, so the view loads and the
        // uniform matrix loads pipeline), then the clearing stores
#pragma unroll 8
        for (int v = 0; v < p.views; v++) {
            const float4 gc = __ldcs(gc4 + size_t(v) * p.n_verts);
            const float* m = b.mvps + v * 16;
            g0 += gc.x * m[0] + gc.y * m[1] + gc.z * m[2] + gc.w * m[3];
            g1 += gc.x * m[4] + gc.y * m[5] + gc.z * m[6] + gc.w * m[7];
            g2 += gc.x * m[8] + gc.y * m[9] + gc.z * m[10] + gc.w * m[11];
        }
#pragma unroll 8
        for (int v = 0; v < p.views; v++)
            gc4[size_t(v) * p.n_verts] = make_float4(0.f, 0.f, 0.f, 0.f);
        b.gpos[u * 3 + 0] = g0;
        b.gpos[u * 3 + 1] = g1;
        b.gpos[u * 3 + 2] = g2;
    } else {
        g0 = b.gpos[u * 3 + 0];
        g1 = b.gpos[u * 3 + 1];
        g2 = b.gpos[u * 3 + 2];
    }
    if (!update) return;
    const float bc1 = b.scalars[1], bc2 = b.scalars[2];
    if (p.reg) {
        // g + g_lap * s_lap + g_nrm * s_nrm (run.cpp:419-420), s = rms(g) /
        // rms(term) * weight
        const float sl = b.reg.rms[0] / b.reg.rms[1] * p.laplacian;
        const float sn = b.reg.rms[0] / b.reg.rms[2] * p.normal;
        const float* gl = b.reg.glap + size_t(u) * 3;
        const float* gn = b.reg.gnrm + size_t(u) * 3;
        g0 = (g0 + gl[0] * sl) + gn[0] * sn;
        g1 = (g1 + gl[1] * sl) + gn[1] * sn;
        g2 = (g2 + gl[2] * sl) + gn[2] * sn;
    }
    const float g[3] = {g0, g1, g2};
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const int i = u * 3 + j;
        const float m_new = b.adam_m[i] * p.b1 + g[j] * omb1;
        const float v_new = b.adam_v[i] * p.b2 + g[j] * g[j] * omb2;
        const float step = (m_new / bc1) / (sqrtf(v_new / bc2) + p.eps) * p.lr;
        b.pos[i] = b.pos[i] - step;
        b.adam_m[i] = m_new;
        b.adam_v[i] = v_new;
    }
}

static void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

void sil_transform(const SilParams& p, const SilBuffers& b, int advance,
                   int* rim, int rim_cells, uint32_t* status, cudaStream_t s) {
    ProfScope ps("transform", s);
    const dim3 vg((p.n_verts + 255) / 256, p.views);
    k_transform<<<vg, 256, 0, s>>>(b.pos, b.mvps, p.n_verts,
                                   reinterpret_cast<float4*>(b.clip),
                                   b.scalars, p.b1, p.b2, advance, rim,
                                   rim_cells, status);
    check_launch();
}

void sil_face_setup(const SoftDims& d, const SilBuffers& b, cudaStream_t s) {
    const dim3 fg((d.n_faces + 127) / 128, d.views);
    ProfScope ps("face_setup", s);
    k_face_setup_sil<<<fg, 128, 0, s>>>(
            d, reinterpret_cast<const float4*>(b.clip), b.faces, b.soft);
    check_launch();
}

void sil_forward_backward(const SoftDims& d, const SilParams& p,
                          const SilBuffers& b, float* rs_out,
                          cudaStream_t s) {
    if (p.paper) {
        paper_forward_backward(d, p, b, rs_out, s);
        return;
    }
    sil_transform(p, b, 1, b.soft.rim, d.rim_cells, b.soft.status, s);
    sil_face_setup(d, b, s);
    EpiSil epi{b.targets, reinterpret_cast<const float4*>(b.clip), b.gclip,
               b.loss_slots, reinterpret_cast<float4*>(rs_out), p.k, p.c,
               p.n_verts, b.det_pix, b.det_touch};
    launch_sweeps(d, b.soft, nullptr, epi, s);
    if (b.det_pix) sil_det_gather(d, p, b, s);
}

// Deterministic gradient, part 1: per (view, face), the partials of its
// three corners summed over the pixels whose survivor it is, in row-major
// order over the face's soft bbox (the reference's GatherDistGrad scans a
// face's pixels in the same order); the arithmetic per pixel is
// sil_scatter's.
__global__ void k_det_face(int n_faces, int n_verts, int W, int H,
                           const FaceRec* recs_all, const float2* pix_all,
                           const float4* clip_all, uint8_t* touch_all,
                           float4* part_all) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (f >= n_faces) return;
    const FaceRec& r = recs_all[size_t(v) * n_faces + f];
    float4 acc[3];
#pragma unroll
    for (int k = 0; k < 3; k++) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    // only faces some pixel gave a gradient to have anything to sum
    uint8_t& touched = touch_all[size_t(v) * n_faces + f];
    const bool any = touched != 0;
    if (any) touched = 0;
    if (any && (r.flags & kFaceValid) && r.bx0 <= r.bx1 && r.by0 <= r.by1) {
        const float2* pix = pix_all + size_t(v) * W * H;
        const float4* clip_v = clip_all + size_t(v) * n_verts;
        const float fw = float(W), fh = float(H);
        const float hx[3] = {r.h0x, r.h1x, r.h2x};
        const float hy[3] = {r.h0y, r.h1y, r.h2y};
        const uint32_t idx[3] = {r.i0, r.i1, r.i2};
        for (int y = r.by0; y <= r.by1; y++) {
            for (int x = r.bx0; x <= r.bx1; x++) {
                const float2 e = pix[size_t(y) * W + x];
                if (__float_as_int(e.x) != f) continue;
                const float g = e.y;
                const float px = float(x) + 0.5f, py = float(y) + 0.5f;
                const TriDist td = signed_dist(px, py, r);
                const float d = fabsf(td.dist);
                if (d < 1e-6f) continue;
                const int ia = td.edge, ib = (td.edge + 1) % 3;
                const float qx = hx[ia] + td.t * (hx[ib] - hx[ia]);
                const float qy = hy[ia] + td.t * (hy[ib] - hy[ia]);
                const float sgn = td.dist >= 0.f ? 1.f : -1.f;
                const float nx = (px - qx) / d;
                const float ny = (py - qy) / d;
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int k = j == 0 ? ia : ib;
                    const float wgt = j == 0 ? (1.f - td.t) : td.t;
                    const float gsx = g * (-sgn * wgt * nx);
                    const float gsy = g * (-sgn * wgt * ny);
                    if (gsx == 0.f && gsy == 0.f) continue;
                    const float4 c = clip_v[idx[k]];
                    acc[k].x += gsx * 0.5f * fw / c.w;
                    acc[k].y += gsy * 0.5f * fh / c.w;
                    acc[k].w += -(gsx * 0.5f * fw * c.x +
                                  gsy * 0.5f * fh * c.y) / (c.w * c.w);
                }
            }
        }
    }
    float4* out = part_all + (size_t(v) * n_faces + f) * 3;
#pragma unroll
    for (int k = 0; k < 3; k++) out[k] = acc[k];
}

// Part 2: per (view, vertex), the sum of its incident faces' corner
// partials in the order of the vertex -> face table (the reference's
// ColSum over GatherDistGrad's columns).
__global__ void k_det_vertex(int n_faces, int n_verts, const float* faces,
                             const float* vf, int vf_deg,
                             const float4* part_all, float* gclip_all) {
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (u >= n_verts) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < vf_deg; j++) {
        const float fv = vf[size_t(j) * n_verts + u];
        if (fv < -0.5f) continue;
        const uint32_t f = x86_u32_via_i64(fv + 0.5f);
        if (f >= uint32_t(n_faces)) continue;
        const float4* p = part_all + (size_t(v) * n_faces + f) * 3;
#pragma unroll
        for (int k = 0; k < 3; k++) {
            if (x86_u32_via_i64(faces[size_t(f) * 3 + k] + 0.5f) !=
                uint32_t(u))
                continue;
            acc.x += p[k].x;
            acc.y += p[k].y;
            acc.w += p[k].w;
        }
    }
    float* g = gclip_all + (size_t(v) * n_verts + u) * 4;
    g[0] = acc.x;
    g[1] = acc.y;
    g[2] = 0.f;
    g[3] = acc.w;
}

void sil_det_gather(const SoftDims& d, const SilParams& p, const SilBuffers& b,
                    cudaStream_t s) {
    ProfScope ps("det_gather", s);
    const dim3 fg((p.n_faces + 127) / 128, p.views);
    k_det_face<<<fg, 128, 0, s>>>(p.n_faces, p.n_verts, d.W, d.H, b.soft.recs,
                                  b.det_pix,
                                  reinterpret_cast<const float4*>(b.clip),
                                  b.det_touch, b.det_part);
    check_launch();
    const dim3 vg((p.n_verts + 127) / 128, p.views);
    k_det_vertex<<<vg, 128, 0, s>>>(p.n_faces, p.n_verts, b.faces, b.det_vf,
                                    b.det_vf_deg, b.det_part, b.gclip);
    check_launch();
}

void sil_grad_reduce(const SilParams& p, const SilBuffers& b, bool update,
                     cudaStream_t s) {
    ProfScope ps("gpos_adam", s);
    k_gpos_adam<<<(p.n_verts + kGposThreads - 1) / kGposThreads, kGposThreads,
                  0, s>>>(
            p, b, 1.f - p.b1, 1.f - p.b2, 1, update ? 1 : 0);
    check_launch();
}

void sil_update(const SilParams& p, const SilBuffers& b, cudaStream_t s) {
    sil_reg_scale(p, b, s);
    ProfScope ps("adam", s);
    k_gpos_adam<<<(p.n_verts + kGposThreads - 1) / kGposThreads, kGposThreads,
                  0, s>>>(
            p, b, 1.f - p.b1, 1.f - p.b2, 0, 1);
    check_launch();
}

void sil_iteration(const SoftDims& d, const SilParams& p, const SilBuffers& b,
                   cudaStream_t s, const StreamFork* fork) {
    if (!p.reg) {
        sil_forward_backward(d, p, b, nullptr, s);
        sil_grad_reduce(p, b, true, s);
        return;
    }
    // the regulariser's terms depend on pos only: with a fork they run on
    // the side stream, concurrently with the raster passes
    if (fork) {
        DRESSI_CUDA(cudaEventRecord(fork->begin, s));
        DRESSI_CUDA(cudaStreamWaitEvent(fork->side, fork->begin, 0));
        sil_reg_terms(p, b, fork->side);
        DRESSI_CUDA(cudaEventRecord(fork->end, fork->side));
    }
    sil_forward_backward(d, p, b, nullptr, s);
    // the regulariser needs the whole g before the Adam step
    sil_grad_reduce(p, b, false, s);
    if (fork)
        DRESSI_CUDA(cudaStreamWaitEvent(s, fork->end, 0));
    else
        sil_reg_terms(p, b, s);
    sil_update(p, b, s);
}

}  // namespace dressi
