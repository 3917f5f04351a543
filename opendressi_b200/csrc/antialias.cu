// Screen-space anti-aliasing (Dr.Hair Eq.3-5): F::AntiAlias forward, its
// image transpose and its vertex gradient (exact scan or stochastic edge
// samples), bit-exact with the reference's CPU kernels for the forward and
// image transpose (src/core/f_ops.cpp:2220-2579 over EvalAaPair,
// src/core/cpu_raster.cpp:371-454).
//
// Per pixel s and each of its 8 neighbours n whose triangle ids differ, the
// pair's separating edge is taken from the owner triangle (n's, then s's):
// r = min(|e(s)| / |edge|, 1) blends c(s) toward c(n). The owner triangles'
// screen vertices are computed once per (view, face) by k_aa_face_setup in
// both projections the reference uses (ProjectToScreen's 1/w product for
// the pair test, c/w divisions for the sample placement), so the pair tests
// read 64-byte records instead of re-projecting clip positions.
#include <algorithm>

#include "kernels.h"

namespace dressi {

namespace {

constexpr int kAaQValid = 1;  // all 3 vertices in range and projectable
constexpr int kAaSValid = 2;  // all 3 vertices in range and w > 1e-6
constexpr int kAaViewWild = 1;  // a face of the view has |screen| >= 1e18

__constant__ int kAaOffX[8] = {-1, 0, 1, -1, 1, -1, 0, 1};
__constant__ int kAaOffY[8] = {-1, -1, -1, 0, 0, 1, 1, 1};

struct AaPairD {
    float r;
    uint32_t ia, ib;
    float qax, qay, qbx, qby;
    float es, len;
};

}  // namespace

// Per (view, face): the owner-triangle data of EvalAaPair and the sample
// placement of AntiAliasBwdVtx.
__global__ void k_aa_face_setup(AaDims d, const float4* clip,
                                const float* faces, AaFace* out,
                                int* view_flags, uint32_t* status) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (f >= d.n_faces) return;
    AaFace r;
    float q[6], sc[6];
    uint32_t vi[3];
    int flags = kAaQValid | kAaSValid;
    for (int k = 0; k < 3; k++) {
        vi[k] = x86_u32_via_i64(faces[size_t(f) * 3 + k] + 0.5f);
        if (vi[k] >= uint32_t(d.n_verts)) {
            // EvalAaPair skips the owner; the reference's sampling loop
            // would read out of range (undefined there): reported.
            atomicOr(status, kStatusIndexRange);
            flags = 0;
            q[2 * k] = q[2 * k + 1] = sc[2 * k] = sc[2 * k + 1] = 0.f;
            continue;
        }
        const float4 c = clip[size_t(v) * d.n_verts + vi[k]];
        float z;
        if (!project_clip(c.x, c.y, c.z, c.w, float(d.W), float(d.H),
                          &q[2 * k], &q[2 * k + 1], &z)) {
            flags &= ~kAaQValid;
            q[2 * k] = q[2 * k + 1] = 0.f;
        }
        if (c.w <= 1e-6f) {
            flags &= ~kAaSValid;
            sc[2 * k] = sc[2 * k + 1] = 0.f;
        } else {
            sc[2 * k] = (c.x / c.w * 0.5f + 0.5f) * float(d.W);
            sc[2 * k + 1] = (c.y / c.w * 0.5f + 0.5f) * float(d.H);
        }
    }
    r.qx0 = q[0]; r.qy0 = q[1]; r.qx1 = q[2]; r.qy1 = q[3];
    r.qx2 = q[4]; r.qy2 = q[5];
    r.sx0 = sc[0]; r.sy0 = sc[1]; r.sx1 = sc[2]; r.sy1 = sc[3];
    r.sx2 = sc[4]; r.sy2 = sc[5];
    r.i0 = vi[0]; r.i1 = vi[1]; r.i2 = vi[2];
    r.flags = uint32_t(flags);
    out[size_t(v) * d.n_faces + f] = r;
    // Screen coordinates below 1e18 keep every product of the pair test
    // finite, so r is a number in [0, 1] (see k_aa_forward's shortcut).
    if (flags & kAaQValid) {
        bool tame = true;
        for (int i = 0; i < 6; i++) tame = tame && fabsf(q[i]) < 1e18f;
        if (!tame) atomicOr(&view_flags[v], kAaViewWild);
    }
}

// EvalAaPair over the face records of one view.
__device__ __forceinline__ bool aa_pair(const AaFace* fr, int n_faces,
                                        int its, int itn, float psx,
                                        float psy, float pnx, float pny,
                                        AaPairD* out) {
    if (its == itn) return false;
#pragma unroll
    for (int o = 0; o < 2; o++) {
        const int owner = o == 0 ? itn : its;
        if (owner == 0) continue;
        const uint32_t f = uint32_t(owner) - 1u;
        if (f >= uint32_t(n_faces)) continue;
        const AaFace r = fr[f];
        if (!(r.flags & kAaQValid)) continue;
        const float qx[3] = {r.qx0, r.qx1, r.qx2};
        const float qy[3] = {r.qy0, r.qy1, r.qy2};
        int best_j = -1;
        float best_t = 0.f;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            const int j1 = j == 2 ? 0 : j + 1;
            const float es = (qx[j1] - qx[j]) * (psy - qy[j]) -
                             (qy[j1] - qy[j]) * (psx - qx[j]);
            const float en = (qx[j1] - qx[j]) * (pny - qy[j]) -
                             (qy[j1] - qy[j]) * (pnx - qx[j]);
            if (es * en >= 0.f) continue;
            const float t = es / (es - en);
            if (best_j < 0 || (o == 0 ? t > best_t : t < best_t)) {
                best_t = t;
                best_j = j;
            }
        }
        if (best_j < 0) continue;
        const float ax = best_j == 0 ? qx[0] : best_j == 1 ? qx[1] : qx[2];
        const float ay = best_j == 0 ? qy[0] : best_j == 1 ? qy[1] : qy[2];
        const float bx = best_j == 0 ? qx[1] : best_j == 1 ? qx[2] : qx[0];
        const float by = best_j == 0 ? qy[1] : best_j == 1 ? qy[2] : qy[0];
        const float ex = bx - ax;
        const float ey = by - ay;
        const float len = sqrtf(ex * ex + ey * ey);
        if (len < 1e-6f) continue;
        const float es = ex * (psy - ay) - ey * (psx - ax);
        out->r = std_min(fabsf(es) / len, 1.f);
        out->ia = best_j == 0 ? r.i0 : best_j == 1 ? r.i1 : r.i2;
        out->ib = best_j == 0 ? r.i1 : best_j == 1 ? r.i2 : r.i0;
        out->qax = ax;
        out->qay = ay;
        out->qbx = bx;
        out->qby = by;
        out->es = es;
        out->len = len;
        return true;
    }
    return false;
}

__device__ __forceinline__ int aa_tri_id(float t) { return x86_i32(t + 0.5f); }

// Triangle ids of a 16x16 tile and its 1-pixel halo (INT_MIN outside).
__device__ __forceinline__ void aa_load_ids(const float* tri, int W, int H,
                                            int x0, int y0,
                                            int ids[18][18]) {
    for (int i = threadIdx.x; i < 18 * 18; i += blockDim.x) {
        const int hx = x0 - 1 + i % 18, hy = y0 - 1 + i / 18;
        ids[i / 18][i % 18] = (hx >= 0 && hy >= 0 && hx < W && hy < H)
                                      ? aa_tri_id(tri[size_t(hy) * W + hx])
                                      : INT_MIN;
    }
}

// Forward: out = AntiAlias(img) (f_ops.cpp:2543-2575). Grid (tiles, views).
// The neighbour loops are not unrolled: one copy of the pair test keeps
// the kernels inside the instruction cache.
//
// Shortcut (exact): when c(s) and c(n) have the same bits and are 0 or 1
// in every channel, r * c + (1 - r) * c == c for any r in [0, 1] (for
// c = 1, r + fl(1 - r) rounds to exactly 1), which is what an inactive
// pair adds; such pairs skip the pair test. r is in [0, 1] unless a face
// of the view has wild screen coordinates (view flag), where the shortcut
// is off. On silhouette masks only pixels next to an edge of the mask run
// pair tests.
// r of the pair (s, n), or -1 when the pair is inactive (r itself is >= 0
// or NaN). Out of line: it runs only where the shortcut does not apply, and
// keeps the forward kernel's common path small.
static __device__ __noinline__ float aa_pair_r(const AaFace* fr, int n_faces,
                                               const float* tri_v, int W,
                                               int x, int y, int nx, int ny) {
    AaPairD pr;
    if (!aa_pair(fr, n_faces, aa_tri_id(tri_v[size_t(y) * W + x]),
                 aa_tri_id(tri_v[size_t(ny) * W + nx]), float(x) + 0.5f,
                 float(y) + 0.5f, float(nx) + 0.5f, float(ny) + 0.5f, &pr))
        return -1.f;
    return pr.r;
}

// r of the pair (s, n) from the tile's shared triangle ids.
static __device__ __noinline__ float aa_pair_r_ids(const AaFace* fr,
                                                   int n_faces, int its,
                                                   int itn, int x, int y,
                                                   int nx, int ny) {
    AaPairD pr;
    if (!aa_pair(fr, n_faces, its, itn, float(x) + 0.5f, float(y) + 0.5f,
                 float(nx) + 0.5f, float(ny) + 0.5f, &pr))
        return -1.f;
    return pr.r;
}

// Coverage of a pixel from its triangle id: the mask Rasterize(clip, ones)
// of a covered pixel is (sum_k l_k / w_k) / (sum_k l_k / w_k), which is
// exactly 1 (the two sums are the same products added in the same order)
// whenever that sum is non-zero (it is finite: the raster keeps w > 1e-6),
// and 0 on the background. A zero sum, where the reference's mask is NaN,
// needs an exact cancellation against a rounding-negative barycentric.
__device__ __forceinline__ float aa_mask_of_id(int id) {
    return (id != 0 && id != INT_MIN) ? 1.f : 0.f;
}

// Eight CTAs per SM (32 registers, a few spilled bytes): the kernel is
// latency-bound on its neighbour and face-record loads, so full residency
// beats the unbounded 48 registers (5 CTAs; 1.12 -> 0.87 ms at C4).
// kIdMask (NC == 1): the image is the hard mask of the triangle ids, taken
// from the id tile in shared memory (img unused), so the mask image is
// neither written by the raster nor read here.
template <class Epi, int NC, bool kIdMask = false>
__global__ void __launch_bounds__(256, 8)
        k_aa_forward(AaDims d, const AaFace* frs, const float* img,
                     const float* tri, const int* view_flags, Epi epi) {
    static_assert(!kIdMask || NC == 1, "id masks have one component");
    __shared__ float vals[18][18];  // n_comp == 1: the image tile + halo
    __shared__ int ids_sh[kIdMask ? 18 : 1][kIdMask ? 18 : 1];
    const int v = blockIdx.y;
    const int tiles_x = (d.W + 15) / 16;
    const int x0 = (blockIdx.x % tiles_x) * 16, y0 = (blockIdx.x / tiles_x) * 16;
    const size_t px0 = size_t(v) * d.W * d.H;
    constexpr int nc = NC;
    const float* im = kIdMask ? nullptr : img + px0 * nc;
    if (kIdMask) {
        for (int i = threadIdx.x; i < 18 * 18; i += blockDim.x) {
            const int hx = x0 - 1 + i % 18, hy = y0 - 1 + i / 18;
            const int id = (hx >= 0 && hy >= 0 && hx < d.W && hy < d.H)
                                   ? aa_tri_id(tri[px0 + size_t(hy) * d.W + hx])
                                   : INT_MIN;
            ids_sh[kIdMask ? i / 18 : 0][kIdMask ? i % 18 : 0] = id;
            vals[i / 18][i % 18] = aa_mask_of_id(id);
        }
    } else if (nc == 1) {
        for (int i = threadIdx.x; i < 18 * 18; i += blockDim.x) {
            const int hx = x0 - 1 + i % 18, hy = y0 - 1 + i / 18;
            vals[i / 18][i % 18] = (hx >= 0 && hy >= 0 && hx < d.W && hy < d.H)
                                           ? im[size_t(hy) * d.W + hx]
                                           : 0.f;
        }
    }
    __syncthreads();
    const bool quick = !(view_flags[v] & kAaViewWild);
    const int lx = threadIdx.x & 15, ly = threadIdx.x >> 4;
    const int x = x0 + lx, y = y0 + ly;
    const bool in = x < d.W && y < d.H;
    float dst[4] = {0.f, 0.f, 0.f, 0.f};
    bool flat = false;
    if (in && nc == 1 && quick) {
        // all 8 neighbours (off-screen ones add c too) equal a 0/1 c:
        // c + 8c = 9c is exact and 9c / 9 == c
        const float c0 = vals[ly + 1][lx + 1];
        const uint32_t b0 = __float_as_uint(c0);
        flat = c0 == 0.f || c0 == 1.f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int nx = x + kAaOffX[k], ny = y + kAaOffY[k];
            const bool on = nx >= 0 && ny >= 0 && nx < d.W && ny < d.H;
            flat = flat && (!on || __float_as_uint(vals[ly + 1 + kAaOffY[k]][lx + 1 + kAaOffX[k]]) == b0);
        }
        if (flat) dst[0] = c0;
    }
    if (in && !flat) {
        const AaFace* fr = frs + size_t(v) * d.n_faces;
        float cs[NC];
#pragma unroll
        for (int c = 0; c < nc; c++) {
            cs[c] = nc == 1 ? vals[ly + 1][lx + 1]
                            : im[(size_t(y) * d.W + x) * nc + c];
            dst[c] = cs[c];
        }
#pragma unroll 1
        for (int k = 0; k < 8; k++) {
            const int nx = x + kAaOffX[k], ny = y + kAaOffY[k];
            if (nx < 0 || ny < 0 || nx >= d.W || ny >= d.H) {
#pragma unroll
                for (int c = 0; c < nc; c++) dst[c] += cs[c];
                continue;
            }
            float cn[NC];
#pragma unroll
            for (int c = 0; c < nc; c++)
                cn[c] = nc == 1 ? vals[ly + 1 + kAaOffY[k]][lx + 1 + kAaOffX[k]]
                                : im[(size_t(ny) * d.W + nx) * nc + c];
            if (quick) {
                bool same = true;
#pragma unroll
                for (int c = 0; c < nc; c++)
                    same = same && __float_as_uint(cs[c]) == __float_as_uint(cn[c]) &&
                           (cs[c] == 0.f || cs[c] == 1.f);
                if (same) {
#pragma unroll
                    for (int c = 0; c < nc; c++) dst[c] += cs[c];
                    continue;
                }
            }
            const float r =
                    kIdMask ? aa_pair_r_ids(fr, d.n_faces,
                                            ids_sh[kIdMask ? ly + 1 : 0][kIdMask ? lx + 1 : 0],
                                            ids_sh[kIdMask ? ly + 1 + kAaOffY[k] : 0]
                                                  [kIdMask ? lx + 1 + kAaOffX[k] : 0],
                                            x, y, nx, ny)
                            : aa_pair_r(fr, d.n_faces, tri + px0, d.W, x, y, nx, ny);
            if (r == -1.f) {
#pragma unroll
                for (int c = 0; c < nc; c++) dst[c] += cs[c];
                continue;
            }
#pragma unroll
            for (int c = 0; c < nc; c++) dst[c] += r * cs[c] + (1.f - r) * cn[c];
        }
#pragma unroll
        for (int c = 0; c < nc; c++) dst[c] /= 9.f;
    }
    epi(d, v, x, y, in, dst);  // every thread (epilogues may reduce a warp)
}

// Image transpose (AntiAliasBwdImg, f_ops.cpp:2220-2278).
__global__ void __launch_bounds__(256)
        k_aa_bwd_img(AaDims d, const AaFace* frs, const float* gy,
                     const float* tri, float* out) {
    __shared__ int ids[18][18];
    const int v = blockIdx.y;
    const int tiles_x = (d.W + 15) / 16;
    const int x0 = (blockIdx.x % tiles_x) * 16, y0 = (blockIdx.x / tiles_x) * 16;
    const size_t px0 = size_t(v) * d.W * d.H;
    aa_load_ids(tri + px0, d.W, d.H, x0, y0, ids);
    __syncthreads();
    const int lx = threadIdx.x & 15, ly = threadIdx.x >> 4;
    const int x = x0 + lx, y = y0 + ly;
    if (x >= d.W || y >= d.H) return;
    const AaFace* fr = frs + size_t(v) * d.n_faces;
    const int nc = d.n_comp;
    const float* g = gy + px0 * nc;
    float dst[4] = {0.f, 0.f, 0.f, 0.f};
    float alpha_sum = 0.f;
    const int its = ids[ly + 1][lx + 1];
    const float psx = float(x) + 0.5f, psy = float(y) + 0.5f;
#pragma unroll 1
    for (int k = 0; k < 8; k++) {
        const int nx = x + kAaOffX[k], ny = y + kAaOffY[k];
        if (nx < 0 || ny < 0 || nx >= d.W || ny >= d.H) {
            alpha_sum += 1.f;
            continue;
        }
        const int itn = ids[ly + 1 + kAaOffY[k]][lx + 1 + kAaOffX[k]];
        const float pnx = float(nx) + 0.5f, pny = float(ny) + 0.5f;
        AaPairD pr, pr2;
        alpha_sum += aa_pair(fr, d.n_faces, its, itn, psx, psy, pnx, pny, &pr)
                             ? pr.r
                             : 1.f;
        if (aa_pair(fr, d.n_faces, itn, its, pnx, pny, psx, psy, &pr2)) {
            const float* gn = g + (size_t(ny) * d.W + nx) * nc;
            for (int c = 0; c < nc; c++) dst[c] += (1.f - pr2.r) * gn[c];
        }
    }
    const float* gs = g + (size_t(y) * d.W + x) * nc;
    float* o = out + px0 * nc + (size_t(y) * d.W + x) * nc;
    for (int c = 0; c < nc; c++) {
        dst[c] += gs[c] * (1.f + alpha_sum);
        o[c] = dst[c] / 9.f;
    }
}

// One active pair's vertex gradient (AntiAliasBwdVtx's accumulate,
// f_ops.cpp:2329-2372) added `mult_a` / `mult_b` times to the endpoints.
// (1/9) dot(gy(s), c(s) - c(n)): the pair's weight. Zero -- the pair adds
// nothing -- needs no pair test (the reference returns at this point).
__device__ __forceinline__ float aa_pair_weight(const AaDims& d, int v,
                                                const float* gy,
                                                const float* img, int x, int y,
                                                int nx, int ny) {
    const int nc = d.n_comp;
    const size_t px0 = size_t(v) * d.W * d.H;
    const size_t so = (px0 + size_t(y) * d.W + x) * nc;
    const size_t no = (px0 + size_t(ny) * d.W + nx) * nc;
    float gr = 0.f;
    for (int c = 0; c < nc; c++) gr += gy[so + c] * (img[so + c] - img[no + c]);
    return gr / 9.f;
}

__device__ __forceinline__ void aa_accumulate(const AaDims& d, int v,
                                              float gr, const float4* clip,
                                              int x, int y,
                                              const AaPairD& pr, int mult_a,
                                              int mult_b, float* grad) {
    const float psx = float(x) + 0.5f, psy = float(y) + 0.5f;
    const float sgn = pr.es >= 0.f ? 1.f : -1.f;
    const float inv_l = 1.f / pr.len;
    const float l3 = fabsf(pr.es) * inv_l * inv_l * inv_l;
    const float ex = pr.qbx - pr.qax;
    const float ey = pr.qby - pr.qay;
    const float dq[2][2] = {{sgn * inv_l * (pr.qby - psy) + l3 * ex,
                             sgn * inv_l * (psx - pr.qbx) + l3 * ey},
                            {sgn * inv_l * (psy - pr.qay) - l3 * ex,
                             sgn * inv_l * (pr.qax - psx) - l3 * ey}};
    const uint32_t ids[2] = {pr.ia, pr.ib};
    const int mult[2] = {mult_a, mult_b};
    const float w_scr = float(d.W), h_scr = float(d.H);
#pragma unroll
    for (int e = 0; e < 2; e++) {
        if (mult[e] == 0) continue;
        const float gqx = gr * dq[e][0];
        const float gqy = gr * dq[e][1];
        const float4 c = clip[size_t(v) * d.n_verts + ids[e]];
        const float a0 = gqx * 0.5f * w_scr / c.w;
        const float a1 = gqy * 0.5f * h_scr / c.w;
        const float a3 = -(gqx * 0.5f * w_scr * c.x + gqy * 0.5f * h_scr * c.y) /
                         (c.w * c.w);
        float* gp = grad + (size_t(v) * d.n_verts + ids[e]) * 4;
        for (int m = 0; m < mult[e]; m++) {
            atomicAdd(gp + 0, a0);
            atomicAdd(gp + 1, a1);
            atomicAdd(gp + 3, a3);
        }
    }
}

// Exact vertex gradient (n_samples = 0): every boundary pair of every
// pixel (f_ops.cpp:2373-2396), scattered to both edge endpoints.
template <bool kIdMask = false>
__global__ void __launch_bounds__(256)
        k_aa_bwd_vtx_exact(AaDims d, const AaFace* frs, const float* gy,
                           const float* img, const float* tri,
                           const float4* clip, float* grad) {
    __shared__ int ids[18][18];
    const int v = blockIdx.y;
    const int tiles_x = (d.W + 15) / 16;
    const int x0 = (blockIdx.x % tiles_x) * 16, y0 = (blockIdx.x / tiles_x) * 16;
    aa_load_ids(tri + size_t(v) * d.W * d.H, d.W, d.H, x0, y0, ids);
    __syncthreads();
    const int lx = threadIdx.x & 15, ly = threadIdx.x >> 4;
    const int x = x0 + lx, y = y0 + ly;
    if (x >= d.W || y >= d.H) return;
    const AaFace* fr = frs + size_t(v) * d.n_faces;
    const int its = ids[ly + 1][lx + 1];
    const float psx = float(x) + 0.5f, psy = float(y) + 0.5f;
    #pragma unroll 1
    for (int k = 0; k < 8; k++) {
        const int nx = x + kAaOffX[k], ny = y + kAaOffY[k];
        if (nx < 0 || ny < 0 || nx >= d.W || ny >= d.H) continue;
        const int itn = ids[ly + 1 + kAaOffY[k]][lx + 1 + kAaOffX[k]];
        float gr;
        if (kIdMask) {
            // aa_pair_weight's sum with c = the id mask
            const size_t so = size_t(v) * d.W * d.H + size_t(y) * d.W + x;
            float acc = 0.f;
            acc += gy[so] * (aa_mask_of_id(its) - aa_mask_of_id(itn));
            gr = acc / 9.f;
        } else {
            gr = aa_pair_weight(d, v, gy, img, x, y, nx, ny);
        }
        if (gr == 0.f) continue;
        AaPairD pr;
        if (!aa_pair(fr, d.n_faces, its, itn,
                     psx, psy, float(nx) + 0.5f, float(ny) + 0.5f, &pr) ||
            pr.r >= 1.f)
            continue;
        aa_accumulate(d, v, gr, clip, x, y, pr, 1, 1, grad);
    }
}

// The sample pixel of (face f, sample smp) and the pairs around it
// (f_ops.cpp:2430-2468). `only` >= 0: accumulate to that vertex only
// (multiplicity 1); else to the face's own vertices with their
// multiplicity in the face (the sum over its VertexFacesTex incidences).
// kIdMask: the image is the hard mask of the triangle ids (img unused).
template <bool kIdMask = false>
__device__ __forceinline__ void aa_sample(const AaDims& d, int v,
                                          const AaFace* fr, const AaFace& r,
                                          uint32_t f, uint32_t smp,
                                          uint32_t seed_u, int only,
                                          const float* gy, const float* img,
                                          const float* tri,
                                          const float4* clip, float* grad) {
    const int e = int(smp % 3u);
    const float ax = e == 0 ? r.sx0 : e == 1 ? r.sx1 : r.sx2;
    const float ay = e == 0 ? r.sy0 : e == 1 ? r.sy1 : r.sy2;
    const float bx = e == 0 ? r.sx1 : e == 1 ? r.sx2 : r.sx0;
    const float by = e == 0 ? r.sy1 : e == 1 ? r.sy2 : r.sy0;
    const float ex = bx - ax;
    const float ey = by - ay;
    const float len = sqrtf(ex * ex + ey * ey);
    if (len < 1e-6f) return;
    const float u = hash_to_unit(f, smp, seed_u, 2);
    const float o = (hash_to_unit(f, smp, seed_u, 3) * 2.f - 1.f) * 2.f;
    const int x = x86_i32(floorf(ax + u * ex - o * (ey / len)));
    const int y = x86_i32(floorf(ay + u * ey + o * (ex / len)));
    if (x < 0 || y < 0 || x >= d.W || y >= d.H) return;
    const float* tv = tri + size_t(v) * d.W * d.H;
    const int its = aa_tri_id(tv[size_t(y) * d.W + x]);
    const float psx = float(x) + 0.5f, psy = float(y) + 0.5f;
    #pragma unroll 1
    for (int k = 0; k < 8; k++) {
        const int nx = x + kAaOffX[k], ny = y + kAaOffY[k];
        if (nx < 0 || ny < 0 || nx >= d.W || ny >= d.H) continue;
        int itn = 0;
        float gr;
        if (kIdMask) {
            // aa_pair_weight's sum with c = the id mask
            itn = aa_tri_id(tv[size_t(ny) * d.W + nx]);
            const size_t so = size_t(v) * d.W * d.H + size_t(y) * d.W + x;
            float acc = 0.f;
            acc += gy[so] * (aa_mask_of_id(its) - aa_mask_of_id(itn));
            gr = acc / 9.f;
        } else {
            gr = aa_pair_weight(d, v, gy, img, x, y, nx, ny);
        }
        if (gr == 0.f) continue;
        if (!kIdMask) itn = aa_tri_id(tv[size_t(ny) * d.W + nx]);
        AaPairD pr;
        if (!aa_pair(fr, d.n_faces, its, itn, psx, psy, float(nx) + 0.5f,
                     float(ny) + 0.5f, &pr) ||
            pr.r >= 1.f)
            continue;
        int ma, mb;
        if (only >= 0) {
            ma = pr.ia == uint32_t(only) ? 1 : 0;
            mb = pr.ib == uint32_t(only) ? 1 : 0;
        } else {
            ma = (r.i0 == pr.ia) + (r.i1 == pr.ia) + (r.i2 == pr.ia);
            mb = (r.i0 == pr.ib) + (r.i1 == pr.ib) + (r.i2 == pr.ib);
        }
        if (ma == 0 && mb == 0) continue;
        aa_accumulate(d, v, gr, clip, x, y, pr, ma, mb, grad);
    }
}

// Stochastic vertex gradient exactly as structured by the reference: one
// thread per (vertex, incidence d, sample) of the given VertexFacesTex.
__global__ void k_aa_bwd_vtx_vft(AaDims d, const AaFace* frs, const float* gy,
                                 const float* img, const float* tri,
                                 const float4* clip, const float* vft,
                                 int max_deg, uint32_t seed_u,
                                 const float* seed_dev, int n_samples,
                                 float* grad) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    const long long total = (long long)d.n_verts * max_deg * n_samples;
    if (i >= total) return;
    // seed from device memory (an in-graph {1,1} value) when given
    if (seed_dev) seed_u = x86_u32_via_i64(seed_dev[0] + 0.5f);
    const int smp = int(i % n_samples);
    const long long vd = i / n_samples;
    const int u = int(vd % d.n_verts);
    const int deg = int(vd / d.n_verts);
    const float fv = vft[size_t(deg) * d.n_verts + u];
    if (fv < -0.5f) return;
    const uint32_t f = x86_u32_via_i64(fv + 0.5f);
    if (f >= uint32_t(d.n_faces)) return;
    const AaFace* fr = frs + size_t(v) * d.n_faces;
    const AaFace r = fr[f];
    if (!(r.flags & kAaSValid)) return;
    aa_sample(d, v, fr, r, f, uint32_t(smp), seed_u, u, gy, img, tri, clip,
              grad);
}

// Stochastic vertex gradient, one thread per (face, sample): each sample is
// evaluated once and credited to the face's vertices with their
// multiplicity -- the same sum as the per-incidence form when the adjacency
// is VertexFacesTex of the faces (the plans build it that way).
// Six CTAs per SM (40 registers): 0.58 -> 0.56 ms at C4 against the
// unbounded 59 registers; eight spill and time slower.
template <bool kIdMask = false>
__global__ void __launch_bounds__(256, 6) k_aa_bwd_vtx_faces(AaDims d, const AaFace* frs,
                                   const float* gy, const float* img,
                                   const float* tri, const float4* clip,
                                   const float* t_ptr, float t_add,
                                   int n_samples, float* grad) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const int v = blockIdx.y;
    if (i >= (long long)d.n_faces * n_samples) return;
    const uint32_t f = uint32_t(i / n_samples);
    const uint32_t smp = uint32_t(i % n_samples);
    const AaFace* fr = frs + size_t(v) * d.n_faces;
    const AaFace r = fr[f];
    if (!(r.flags & kAaSValid)) return;
    const uint32_t seed_u = x86_u32_via_i64((t_ptr[0] + t_add) + 0.5f);
    aa_sample<kIdMask>(d, v, fr, r, f, smp, seed_u, -1, gy, img, tri, clip,
                       grad);
}

namespace {

struct EpiAaOut {
    float* out;
    __device__ void operator()(const AaDims& d, int v, int x, int y, bool in,
                               const float* val) const {
        if (!in) return;
        float* o = out + (size_t(v) * d.W * d.H + size_t(y) * d.W + x) * d.n_comp;
        for (int c = 0; c < d.n_comp; c++) o[c] = val[c];
    }
};

void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

dim3 tile_grid(const AaDims& d) {
    return dim3(((d.W + 15) / 16) * ((d.H + 15) / 16), d.views);
}

}  // namespace

void aa_face_setup(const AaDims& d, const float* clip, const float* faces,
                   AaFace* out, int* view_flags, uint32_t* status,
                   cudaStream_t s) {
    ProfScope ps("aa_face_setup", s);
    DRESSI_CUDA(cudaMemsetAsync(view_flags, 0, sizeof(int) * d.views, s));
    if (d.n_faces == 0) return;
    k_aa_face_setup<<<dim3((d.n_faces + 127) / 128, d.views), 128, 0, s>>>(
            d, reinterpret_cast<const float4*>(clip), faces, out, view_flags,
            status);
    check_launch();
}

void aa_forward_op(const AaDims& d, const AaFace* fr, const int* view_flags,
                   const float* img, const float* tri, float* out,
                   cudaStream_t s) {
    ProfScope ps("aa_forward", s);
    const EpiAaOut epi{out};
    switch (d.n_comp) {
    case 1: k_aa_forward<EpiAaOut, 1><<<tile_grid(d), 256, 0, s>>>(d, fr, img, tri, view_flags, epi); break;
    case 2: k_aa_forward<EpiAaOut, 2><<<tile_grid(d), 256, 0, s>>>(d, fr, img, tri, view_flags, epi); break;
    case 3: k_aa_forward<EpiAaOut, 3><<<tile_grid(d), 256, 0, s>>>(d, fr, img, tri, view_flags, epi); break;
    default: k_aa_forward<EpiAaOut, 4><<<tile_grid(d), 256, 0, s>>>(d, fr, img, tri, view_flags, epi); break;
    }
    check_launch();
}

void aa_bwd_img_op(const AaDims& d, const AaFace* fr, const float* gy,
                   const float* tri, float* out, cudaStream_t s) {
    ProfScope ps("aa_bwd_img", s);
    k_aa_bwd_img<<<tile_grid(d), 256, 0, s>>>(d, fr, gy, tri, out);
    check_launch();
}

void aa_bwd_vtx_op(const AaDims& d, const AaFace* fr, const float* gy,
                   const float* img, const float* tri, const float* clip,
                   const float* vft, int max_deg, float seed, int n_samples,
                   float* grad, cudaStream_t s, const float* seed_dev) {
    ProfScope ps("aa_bwd_vtx", s);
    const float4* c4 = reinterpret_cast<const float4*>(clip);
    if (n_samples == 0) {
        k_aa_bwd_vtx_exact<<<tile_grid(d), 256, 0, s>>>(d, fr, gy, img, tri,
                                                        c4, grad);
    } else {
        const long long total = (long long)d.n_verts * max_deg * n_samples;
        if (total == 0) return;
        const uint32_t seed_u = x86_u32_via_i64(seed + 0.5f);
        k_aa_bwd_vtx_vft<<<dim3(unsigned((total + 255) / 256), d.views), 256,
                           0, s>>>(d, fr, gy, img, tri, c4, vft, max_deg,
                                   seed_u, seed_dev, n_samples, grad);
    }
    check_launch();
}

// ------------------------------------------------ AA silhouette (C4)

namespace {

// Per-pixel loss and its gradient w.r.t. the anti-aliased prediction, in
// the reference autodiff's operation order for (t - pred)^2 * c with seed 1
// (as the HardSoftRas iteration): gy = -(c*diff + c*diff). The loss is
// reduced per warp into one of kLossSlots double slots.
struct EpiAaSil {
    const float* targets;
    float* gy;
    double* loss_slots;
    float c;
    __device__ void operator()(const AaDims& d, int v, int x, int y, bool in,
                               const float* val) const {
        float lv = 0.f;
        if (in) {
            const size_t pix = size_t(v) * d.W * d.H + size_t(y) * d.W + x;
            const float diff = targets[pix] - val[0];
            lv = diff * diff * c;
            const float g_m4 = 1.f * c;
            gy[pix] = -(g_m4 * diff + g_m4 * diff);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lv += __shfl_down_sync(0xffffffffu, lv, o);
        if ((threadIdx.x & 31) == 0 && lv != 0.f) {
            const unsigned slot = (unsigned(blockIdx.y) * gridDim.x + blockIdx.x) * 8u +
                                  (threadIdx.x >> 5);
            atomicAdd(&loss_slots[slot % kLossSlots], double(lv));
        }
    }
};

}  // namespace

// Hard mask + triangle ids (one raster sweep), the per-face AA records and
// the anti-aliased image of the plan's current clip positions; epi
// receives the AA value of every pixel.
template <class Epi>
static void aa_sil_render(const SilParams& p, const AaSilBuffers& b,
                          const Epi& epi, cudaStream_t s) {
    HardDims hd;
    hd.W = hd.H = p.res;
    hd.views = p.views;
    hd.n_faces = p.n_faces;
    hd.n_verts = p.n_verts;
    // no attribute: the raster writes the triangle-id image only; the mask
    // Rasterize(clip, ones) is derived from it (aa_mask_of_id)
    hd.attr_ones = 0;
    hard_raster_op(hd, b.hard_ws, b.sil.clip, nullptr, b.sil.faces, b.tri,
                   nullptr, b.status, s, nullptr);
    AaDims d;
    d.W = d.H = p.res;
    d.views = p.views;
    d.n_faces = p.n_faces;
    d.n_verts = p.n_verts;
    d.n_comp = 1;
    aa_face_setup(d, b.sil.clip, b.sil.faces, b.frs, b.view_flags, b.status,
                  s);
    {
        ProfScope ps("aa_forward", s);
        k_aa_forward<Epi, 1, true><<<tile_grid(d), 256, 0, s>>>(
                d, b.frs, nullptr, b.tri, b.view_flags, epi);
    }
    check_launch();
}

size_t aa_sil_workspace_bytes(const SilParams& p) {
    HardDims hd;
    hd.W = hd.H = p.res;
    hd.views = p.views;
    hd.n_faces = p.n_faces;
    hd.n_verts = p.n_verts;
    return hard_workspace_bytes(hd);
}

void aa_sil_forward_backward(const SilParams& p, const AaSilBuffers& b,
                             cudaStream_t s) {
    sil_transform(p, b.sil, 1, nullptr, 0, b.status, s);
    aa_sil_render(p, b, EpiAaSil{b.sil.targets, b.gy, b.sil.loss_slots, p.c},
                  s);
    AaDims d;
    d.W = d.H = p.res;
    d.views = p.views;
    d.n_faces = p.n_faces;
    d.n_verts = p.n_verts;
    d.n_comp = 1;
    const float4* c4 = reinterpret_cast<const float4*>(b.sil.clip);
    ProfScope ps("aa_bwd_vtx", s);
    if (p.n_samples == 0) {
        k_aa_bwd_vtx_exact<true><<<tile_grid(d), 256, 0, s>>>(
                d, b.frs, b.gy, nullptr, b.tri, c4, b.sil.gclip);
    } else {
        // the sampling seed is the Adam counter before this iteration's
        // update: scalars[0] - 1 once the transform has advanced it (exact
        // for counters below 2^24)
        const long long n = (long long)p.n_faces * p.n_samples;
        k_aa_bwd_vtx_faces<true><<<dim3(unsigned((n + 255) / 256), p.views),
                                   256, 0, s>>>(d, b.frs, b.gy, nullptr, b.tri, c4,
                                     b.sil.scalars, -1.f, p.n_samples,
                                     b.sil.gclip);
    }
    check_launch();
}

void aa_sil_iteration(const SilParams& p, const AaSilBuffers& b,
                      cudaStream_t s) {
    aa_sil_forward_backward(p, b, s);
    if (!p.reg) {
        sil_grad_reduce(p, b.sil, true, s);
        return;
    }
    sil_grad_reduce(p, b.sil, false, s);
    sil_reg_terms(p, b.sil, s);
    sil_update(p, b.sil, s);
}

void aa_sil_predict(const SilParams& p, const AaSilBuffers& b, float* out,
                    cudaStream_t s) {
    sil_transform(p, b.sil, 0, nullptr, 0, b.status, s);
    aa_sil_render(p, b, EpiAaOut{out}, s);
}

void aa_render_targets(const SilParams& p, const AaSilBuffers& b,
                       const float* target_pos, cudaStream_t s) {
    // target clip positions go through the plan's clip buffer (overwritten
    // by every iteration's transform)
    sil_transform_plain(p, b.sil, target_pos, s);
    aa_sil_render(p, b, EpiAaOut{b.sil.targets}, s);
}

}  // namespace dressi
