// Texturing.
//
// Op level (drop-ins for the reference's ops): F::TextureBilinear's
// forward (BilerpClamp, src/core/ibl_math.h:91-115) and its backward
// GatherByInverseUVBilinear (src/core/f_ops.cpp:2650-2732), bit-exact with
// the reference's CPU kernels; F::Texture's nearest sampling and its
// GatherByInverseUV, restated from the reference's GLSL and sampler
// (src/codegen/glsl_codegen.cpp:658-709, src/vk/executor.cpp:193-202).
//
// Config C2 (no reference implementation of mips; defined from first
// principles, the definition is spelled out beside
// dressi_texture_plan_create in the public header): a box-filtered mip
// pyramid of the
// optimised texture, per-pixel trilinear sampling at a lod taken from the
// G-buffer's uv differences, the loss of the reference's texture graph
// (examples/texture_optimization/run.cpp:115-126: per view
// Mean((target - mask * sample)^2)), the exact transpose of the sampling
// scattered into the pyramid's gradient, folded down to level 0, and Adam.
#include <algorithm>

#include "kernels.h"

namespace dressi {

namespace {

__device__ __forceinline__ int iclamp(int x, int lo, int hi) {
    return x < lo ? lo : (x > hi ? hi : x);
}

// BilerpClamp (ibl_math.h:91-115): 4-tap, clamp-to-edge.
template <int N>
__device__ __forceinline__ void bilerp_clamp(const float* data, int w, int h,
                                             float u, float v, float* out) {
    const float sx = u * float(w) - 0.5f;
    const float sy = v * float(h) - 0.5f;
    const int ix = x86_i32(floorf(sx));
    const int iy = x86_i32(floorf(sy));
    const float fx = sx - float(ix);
    const float fy = sy - float(iy);
#pragma unroll
    for (int c = 0; c < N; c++) out[c] = 0.f;
#pragma unroll
    for (int dy = 0; dy <= 1; dy++) {
#pragma unroll
        for (int dx = 0; dx <= 1; dx++) {
            const int x = iclamp(ix + dx, 0, w - 1);
            const int y = iclamp(iy + dy, 0, h - 1);
            const float wgt = (dx == 0 ? 1.f - fx : fx) * (dy == 0 ? 1.f - fy : fy);
            const float* p = data + (size_t(y) * w + size_t(x)) * N;
#pragma unroll
            for (int c = 0; c < N; c++) out[c] += wgt * p[c];
        }
    }
}

template <int N>
__global__ void k_tex_sample(const float* tex, int tw, int th, int filter,
                             const float* uv, size_t npx, float* out) {
    const size_t p = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p >= npx) return;
    const float u = uv[p * 2], v = uv[p * 2 + 1];
    float* o = out + p * N;
    if (filter == 1) {
        bilerp_clamp<N>(tex, tw, th, u, v, o);
        return;
    }
    const int x = iclamp(x86_i32(floorf(u * float(tw))), 0, tw - 1);
    const int y = iclamp(x86_i32(floorf(v * float(th))), 0, th - 1);
    const float* q = tex + (size_t(y) * tw + x) * N;
#pragma unroll
    for (int c = 0; c < N; c++) o[c] = q[c];
}

// Anchor of texel (tx, ty) in the inverse-UV table (its entry, else the
// first valid one of the 9x9 neighbourhood in row order).
__device__ __forceinline__ bool inv_uv_anchor(const float4* iv_t, int tw,
                                              int th, int tx, int ty,
                                              float4* out) {
    float4 iv = iv_t[size_t(ty) * tw + tx];
    for (int ny = -4; ny <= 4 && iv.z < 0.5f; ny++) {
        for (int nx = -4; nx <= 4; nx++) {
            const int px = tx + nx, py = ty + ny;
            if (px < 0 || py < 0 || px >= tw || py >= th) continue;
            iv = iv_t[size_t(py) * tw + px];
            if (iv.z > 0.5f) break;
        }
    }
    *out = iv;
    return iv.z > 0.5f;
}

template <int N>
__global__ void k_tex_gather(const float* gy, int sw, int sh, int filter,
                             const float4* inv_uv, int tw, int th,
                             const float2* uv_screen, float* out) {
    const int tx = blockIdx.x * blockDim.x + threadIdx.x;
    const int ty = blockIdx.y;
    if (tx >= tw) return;
    float o[N];
#pragma unroll
    for (int c = 0; c < N; c++) o[c] = 0.f;
    float4 iv;
    if (inv_uv_anchor(inv_uv, tw, th, tx, ty, &iv)) {
        const int scx = x86_i32(iv.x), scy = x86_i32(iv.y);
        bool found = false;
        for (int dy = -3; dy <= 3 && !found; dy++) {
            for (int dx = -3; dx <= 3; dx++) {
                const int spx = scx + dx, spy = scy + dy;
                if (spx < 0 || spy < 0 || spx >= sw || spy >= sh) continue;
                const float2 suv = uv_screen[size_t(spy) * sw + spx];
                const float* g = gy + (size_t(spy) * sw + spx) * N;
                if (filter == 1) {
                    const float stx = suv.x * float(tw) - 0.5f;
                    const float sty = suv.y * float(th) - 0.5f;
                    const float w = std_max(0.f, 1.f - fabsf(stx - float(tx))) *
                                    std_max(0.f, 1.f - fabsf(sty - float(ty)));
                    if (w > 0.f) {
#pragma unroll
                        for (int c = 0; c < N; c++) o[c] += g[c] * w;
                    }
                } else {
                    const int stx = x86_i32(suv.x * float(tw));
                    const int sty = x86_i32(suv.y * float(th));
                    if (stx == tx && sty == ty) {
#pragma unroll
                        for (int c = 0; c < N; c++) o[c] = g[c];
                        found = true;
                        break;
                    }
                }
            }
        }
    }
    float* dst = out + (size_t(ty) * tw + tx) * N;
#pragma unroll
    for (int c = 0; c < N; c++) dst[c] = o[c];
}

void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

}  // namespace

void texture_sample_op(const float* tex, int tw, int th, int n, int filter,
                       const float* uv, size_t npx, float* out,
                       cudaStream_t s) {
    if (npx == 0) return;
    const unsigned blocks = unsigned((npx + 255) / 256);
    switch (n) {
    case 1: k_tex_sample<1><<<blocks, 256, 0, s>>>(tex, tw, th, filter, uv, npx, out); break;
    case 2: k_tex_sample<2><<<blocks, 256, 0, s>>>(tex, tw, th, filter, uv, npx, out); break;
    case 3: k_tex_sample<3><<<blocks, 256, 0, s>>>(tex, tw, th, filter, uv, npx, out); break;
    default: k_tex_sample<4><<<blocks, 256, 0, s>>>(tex, tw, th, filter, uv, npx, out); break;
    }
    check_launch();
}

void texture_gather_op(const float* gy, int sw, int sh, int n, int filter,
                       const float* inv_uv, int tw, int th,
                       const float* uv_screen, float* out, cudaStream_t s) {
    const dim3 grid((tw + 127) / 128, th);
    const float4* iv = reinterpret_cast<const float4*>(inv_uv);
    const float2* us = reinterpret_cast<const float2*>(uv_screen);
    switch (n) {
    case 1: k_tex_gather<1><<<grid, 128, 0, s>>>(gy, sw, sh, filter, iv, tw, th, us, out); break;
    case 2: k_tex_gather<2><<<grid, 128, 0, s>>>(gy, sw, sh, filter, iv, tw, th, us, out); break;
    case 3: k_tex_gather<3><<<grid, 128, 0, s>>>(gy, sw, sh, filter, iv, tw, th, us, out); break;
    default: k_tex_gather<4><<<grid, 128, 0, s>>>(gy, sw, sh, filter, iv, tw, th, us, out); break;
    }
    check_launch();
}

// ------------------------------------------------------------------ C2

size_t tex_mip_floats(int w, int levels) {
    size_t n = 0;
    for (int l = 0; l < levels; l++) n += size_t(w >> l) * size_t(w >> l) * 3;
    return n;
}

namespace {

__host__ __device__ __forceinline__ size_t mip_off(int w, int level) {
    size_t off = 0;
    for (int l = 0; l < level; l++) off += size_t(w >> l) * size_t(w >> l) * 3;
    return off;
}

// Level l+1 from level l (2x2 box, row-major order); zeroes the matching
// gradient entries for this iteration.
__global__ void k_mip_level(float* pyr, float4* gpyr, int w, int level) {
    const int s = w >> level, t = s >> 1;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(t) * t * 3) return;
    const int c = int(i % 3), px = int(i / 3);
    const int x = px % t, y = px / t;
    const float* src = pyr + mip_off(w, level);
    const float a = src[(size_t(2 * y) * s + 2 * x) * 3 + c];
    const float b = src[(size_t(2 * y) * s + 2 * x + 1) * 3 + c];
    const float cc = src[(size_t(2 * y + 1) * s + 2 * x) * 3 + c];
    const float d = src[(size_t(2 * y + 1) * s + 2 * x + 1) * 3 + c];
    const size_t o = mip_off(w, level + 1) + i;
    pyr[o] = 0.25f * (((a + b) + cc) + d);
    if (gpyr && c == 0) gpyr[o / 3] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// Levels 1..nlev (nlev <= 5) of one 32x32 level-0 tile per block, the
// intermediate levels kept in shared memory; every value is k_mip_level's
// 0.25 (((a + b) + c) + d) of the same four inputs.
constexpr int kMipTile = 32;
__global__ void __launch_bounds__(256)
        k_mip_tiles(float* pyr, float4* gpyr, int w, int nlev) {
    __shared__ float buf[2][(kMipTile / 2) * (kMipTile / 2) * 3];
    const int tiles = w / kMipTile;
    const int tx = blockIdx.x % tiles, ty = blockIdx.x / tiles;
    for (int k = 1; k <= nlev; k++) {
        const int n = kMipTile >> k;          // this level's tile side
        const int sl = w >> k;                // this level's image side
        float* dst = buf[k & 1];
        const float* src = buf[(k - 1) & 1];
        const int ps = 2 * n;                 // the source tile side
        const size_t off = mip_off(w, k);
        float* out = pyr + off;
        const float* lvl0 = pyr;
        for (int i = threadIdx.x; i < n * n * 3; i += blockDim.x) {
            const int c = i % 3, q = i / 3, x = q % n, y = q / n;
            float a, b, cc, d;
            if (k == 1) {
                const size_t r0 = size_t(ty * kMipTile + 2 * y) * w +
                                  tx * kMipTile + 2 * x;
                a = lvl0[r0 * 3 + c];
                b = lvl0[(r0 + 1) * 3 + c];
                cc = lvl0[(r0 + w) * 3 + c];
                d = lvl0[(r0 + w + 1) * 3 + c];
            } else {
                const int r0 = (2 * y) * ps + 2 * x;
                a = src[r0 * 3 + c];
                b = src[(r0 + 1) * 3 + c];
                cc = src[(r0 + ps) * 3 + c];
                d = src[(r0 + ps + 1) * 3 + c];
            }
            const float v = 0.25f * (((a + b) + cc) + d);
            dst[i] = v;
            const size_t texel = size_t(ty * n + y) * sl + tx * n + x;
            out[texel * 3 + c] = v;
            if (gpyr && c == 0)
                gpyr[off / 3 + texel] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
    }
}

// Levels from + 1 .. levels - 1 by one block (level `from` at most 64x64),
// level by level; the block's barrier orders its own global writes.
__global__ void __launch_bounds__(1024)
        k_mip_top(float* pyr, float4* gpyr, int w, int from, int levels) {
    for (int l = from; l + 1 < levels; l++) {
        const int sp = w >> l, t = sp >> 1;
        const float* src = pyr + mip_off(w, l);
        const size_t o0 = mip_off(w, l + 1);
        for (int i = threadIdx.x; i < t * t * 3; i += blockDim.x) {
            const int c = i % 3, q = i / 3, x = q % t, y = q / t;
            const float a = src[(size_t(2 * y) * sp + 2 * x) * 3 + c];
            const float b = src[(size_t(2 * y) * sp + 2 * x + 1) * 3 + c];
            const float cc = src[(size_t(2 * y + 1) * sp + 2 * x) * 3 + c];
            const float d = src[(size_t(2 * y + 1) * sp + 2 * x + 1) * 3 + c];
            pyr[o0 + i] = 0.25f * (((a + b) + cc) + d);
            if (gpyr && c == 0)
                gpyr[(o0 + i) / 3] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
    }
}

// lod from the level-0 footprint rho: e + (m - 1) for rho = m * 2^e,
// m in [1, 2) (piecewise-linear log2, exact in float), clamped.
__device__ __forceinline__ float lod_of(float rho, int levels) {
    if (!(rho > 1.f)) return 0.f;
    int e;
    const float m2 = frexpf(rho, &e);
    const float lod = float(e - 1) + (m2 * 2.f - 1.f);
    const float top = float(levels - 1);
    return lod < top ? lod : top;
}

__device__ __forceinline__ float pixel_rho(const float* gb, int W, int H,
                                           int x, int y, float w_tex) {
    float du[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    const float* c = gb + (size_t(y) * W + x) * 3;
#pragma unroll
    for (int axis = 0; axis < 2; axis++) {
        const int ax = axis == 0 ? 1 : 0, ay = axis == 0 ? 0 : 1;
        const int x1 = x + ax, y1 = y + ay, x0 = x - ax, y0 = y - ay;
        if (x1 < W && y1 < H && gb[(size_t(y1) * W + x1) * 3 + 2] > 0.5f) {
            const float* q = gb + (size_t(y1) * W + x1) * 3;
            du[axis][0] = q[0] - c[0];
            du[axis][1] = q[1] - c[1];
        } else if (x0 >= 0 && y0 >= 0 && gb[(size_t(y0) * W + x0) * 3 + 2] > 0.5f) {
            const float* q = gb + (size_t(y0) * W + x0) * 3;
            du[axis][0] = c[0] - q[0];
            du[axis][1] = c[1] - q[1];
        }
    }
    const float ax_ = du[0][0] * w_tex, ay_ = du[0][1] * w_tex;
    const float bx_ = du[1][0] * w_tex, by_ = du[1][1] * w_tex;
    const float rx = sqrtf(ax_ * ax_ + ay_ * ay_);
    const float ry = sqrtf(bx_ * bx_ + by_ * by_);
    return std_max(rx, ry);
}

// Per view pixel: lod, trilinear sample of the pyramid. train: the loss of
// the pixel (warp-summed into loss_slots) and the exact transpose of its
// sampling scattered into gpyr; out (nullable) gets mask * sample.
// Eight CTAs per SM (32 registers instead of 40): 0.121 -> 0.120 ms per
// C2 iteration.
//
// Scatter of the transpose (kRuns): each lane's bilinear tap quad of a level
// is one (four texels, four weights) set. With kRuns = false every tap is a
// float4 vector atomic (red.v4.f32); with kRuns = true the lanes of a warp
// whose quads name the same four texels (neighbouring pixels of a row in a
// magnified region) are first summed by a segmented warp scan and one lane
// per run issues the atomics (warp-aggregated accumulation).
template <bool kRuns>
__global__ void __launch_bounds__(256, kRuns ? 4 : 8)
        k_c2_pixel(TexParams p, const float* pyr, const float* gbuf,
                   const float* targets, float4* gpyr, double* loss_slots,
                   float* out, int train) {
    // the quads of the (up to) two levels this lane scatters into
    int qkey[2][4] = {{-1, -1, -1, -1}, {-1, -1, -1, -1}};
    float qw[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    float gq[3] = {0.f, 0.f, 0.f};
    const int v = blockIdx.y;
    const int tiles_x = (p.res + 15) / 16;
    const int x = (blockIdx.x % tiles_x) * 16 + (threadIdx.x & 15);
    const int y = (blockIdx.x / tiles_x) * 16 + (threadIdx.x >> 4);
    const bool in = x < p.res && y < p.res;
    const float* gb = gbuf + size_t(v) * p.res * p.res * 3;
    float lv = 0.f;
    if (in) {
        const size_t pix = size_t(y) * p.res + x;
        const float u = gb[pix * 3], vv = gb[pix * 3 + 1], mask = gb[pix * 3 + 2];
        const float lod = mask > 0.5f
                                  ? lod_of(pixel_rho(gb, p.res, p.res, x, y,
                                                     float(p.w_tex)),
                                           p.levels)
                                  : 0.f;
        const int l0 = x86_i32(floorf(lod));
        const float f = lod - float(l0);
        const int s0 = p.w_tex >> l0;
        float smp[3], s1[3];
        bilerp_clamp<3>(pyr + mip_off(p.w_tex, l0), s0, s0, u, vv, smp);
        const bool two = f > 0.f && l0 + 1 < p.levels;
        if (two) {
            bilerp_clamp<3>(pyr + mip_off(p.w_tex, l0 + 1), s0 >> 1, s0 >> 1,
                            u, vv, s1);
#pragma unroll
            for (int c = 0; c < 3; c++) smp[c] = smp[c] * (1.f - f) + s1[c] * f;
        }
        const size_t o = (size_t(v) * p.res * p.res + pix) * 3;
        if (!train) {
#pragma unroll
            for (int c = 0; c < 3; c++) out[o + c] = mask * smp[c];
        } else {
            float g[3];
#pragma unroll
            for (int c = 0; c < 3; c++) {
                const float pred = mask * smp[c];
                if (out) out[o + c] = pred;
                const float diff = targets[o + c] - pred;
                lv += diff * diff * p.inv_n;
                const float g_m = 1.f * p.inv_n;
                g[c] = -(g_m * diff + g_m * diff) * mask;
            }
            if (g[0] != 0.f || g[1] != 0.f || g[2] != 0.f) {
                for (int lvl = 0; lvl < 1 + (two ? 1 : 0); lvl++) {
                    const int level = l0 + lvl;
                    const float lw = two ? (lvl == 0 ? 1.f - f : f) : 1.f;
                    const int s = p.w_tex >> level;
                    const float sx = u * float(s) - 0.5f;
                    const float sy = vv * float(s) - 0.5f;
                    const int ix = x86_i32(floorf(sx));
                    const int iy = x86_i32(floorf(sy));
                    const float fx = sx - float(ix);
                    const float fy = sy - float(iy);
                    const size_t lbase = mip_off(p.w_tex, level) / 3;
                    float4* gl = gpyr + lbase;
#pragma unroll
                    for (int dy = 0; dy <= 1; dy++)
#pragma unroll
                        for (int dx = 0; dx <= 1; dx++) {
                            const int tx = iclamp(ix + dx, 0, s - 1);
                            const int ty = iclamp(iy + dy, 0, s - 1);
                            const float wt = (dx == 0 ? 1.f - fx : fx) *
                                             (dy == 0 ? 1.f - fy : fy);
                            if (kRuns) {
                                qkey[lvl][dy * 2 + dx] =
                                        int(lbase + size_t(ty) * s + tx);
                                qw[lvl][dy * 2 + dx] = lw * wt;
                            } else {
                                // one vector atomic per tap (rgb + unused)
                                atomicAdd(gl + size_t(ty) * s + tx,
                                          make_float4(g[0] * lw * wt,
                                                      g[1] * lw * wt,
                                                      g[2] * lw * wt, 0.f));
                            }
                        }
                }
                if (kRuns) {
#pragma unroll
                    for (int c = 0; c < 3; c++) gq[c] = g[c];
                }
            }
        }
    }
    if (kRuns && train) {
        // every lane of the warp takes part (lanes without taps carry key
        // -1 and form runs of their own)
#pragma unroll
        for (int lvl = 0; lvl < 2; lvl++) {
            const bool on = qkey[lvl][0] >= 0;
            if (!__any_sync(0xffffffffu, on)) continue;
            const int lane = threadIdx.x & 31;
            bool head = lane == 0;
#pragma unroll
            for (int k = 0; k < 4; k++)
                head |= __shfl_up_sync(0xffffffffu, qkey[lvl][k], 1) !=
                        qkey[lvl][k];
            const unsigned heads = __ballot_sync(0xffffffffu, head);
            const int start = 31 - __clz(heads & (0xffffffffu >> (31 - lane)));
            const unsigned longest = __reduce_max_sync(
                    0xffffffffu, unsigned(lane - start + 1));
            const int steps = longest <= 1u ? 0 : 32 - __clz(longest - 1u);
            float val[12];
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int c = 0; c < 3; c++)
                    val[k * 3 + c] = on ? gq[c] * qw[lvl][k] : 0.f;
            for (int st = 0; st < steps; st++) {
                const int off = 1 << st;
                const bool take = lane - off >= start;
#pragma unroll
                for (int q = 0; q < 12; q++) {
                    const float o = __shfl_up_sync(0xffffffffu, val[q], off);
                    if (take) val[q] += o;
                }
            }
            const bool tail = lane == 31 || ((heads >> (lane + 1)) & 1u);
            if (on && tail) {
#pragma unroll
                for (int k = 0; k < 4; k++)
                    atomicAdd(gpyr + qkey[lvl][k],
                              make_float4(val[k * 3], val[k * 3 + 1],
                                          val[k * 3 + 2], 0.f));
            }
        }
    }
    if (train) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lv += __shfl_down_sync(0xffffffffu, lv, o);
        if ((threadIdx.x & 31) == 0 && lv != 0.f) {
            const unsigned slot = (unsigned(blockIdx.y) * gridDim.x + blockIdx.x) * 8u +
                                  (threadIdx.x >> 5);
            atomicAdd(&loss_slots[slot % kLossSlots], double(lv));
        }
    }
}

__device__ __forceinline__ float comp3(const float4& q, int c) {
    return c == 0 ? q.x : (c == 1 ? q.y : q.z);
}

// Folds the pyramid gradient down to level 0 (the transpose of the box
// mips: each level adds 0.25 of its parent, from the top level down, which
// per level-0 texel and channel is the chain acc_l = g_l + 0.25 acc_{l+1})
// into grad; zeroes level 0 of gpyr. One thread per level-0 texel. Block 0
// also publishes the iteration's loss and advances the Adam counter.
__global__ void k_mip_fold(TexParams p, float4* gpyr, float* grad,
                           float* scalars, double* loss_slots,
                           float* loss_hist, int hist_cap) {
    if (blockIdx.x == 0) {
        __shared__ double red[256];
        double acc = 0.0;
        for (int i = threadIdx.x; i < kLossSlots; i += blockDim.x) {
            acc += loss_slots[i];
            loss_slots[i] = 0.0;
        }
        red[threadIdx.x] = acc;
        __syncthreads();
        for (int o = blockDim.x / 2; o > 0; o >>= 1) {
            if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            const float t_new = scalars[0] + 1.f;
            scalars[0] = t_new;
            scalars[1] = 1.f - powf(p.b1, t_new);
            scalars[2] = 1.f - powf(p.b2, t_new);
            const float loss = float(red[0]);
            scalars[3] = loss;
            const int it = int(t_new) - 1;
            if (hist_cap > 0) loss_hist[it % hist_cap] = loss;
        }
    }
    const size_t n0 = size_t(p.w_tex) * p.w_tex;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n0) return;
    const int x = int(i % p.w_tex), y = int(i / p.w_tex);
    const float4 q0 = gpyr[i];
    float g0[3] = {q0.x, q0.y, q0.z};
    if (p.levels > 1) {
        const int top = p.levels - 1;
        // texel offsets of the levels walked down from the top
        size_t off = mip_off(p.w_tex, top) / 3;
        const int st = p.w_tex >> top;
        const float4 qt = gpyr[off + size_t(y >> top) * st + (x >> top)];
        float acc[3] = {qt.x, qt.y, qt.z};
        for (int l = top - 1; l >= 1; l--) {
            const int sl = p.w_tex >> l;
            off -= size_t(sl) * size_t(sl);
            const float4 q = gpyr[off + size_t(y >> l) * sl + (x >> l)];
#pragma unroll
            for (int c = 0; c < 3; c++) acc[c] = comp3(q, c) + 0.25f * acc[c];
        }
#pragma unroll
        for (int c = 0; c < 3; c++) g0[c] = g0[c] + 0.25f * acc[c];
    }
#pragma unroll
    for (int c = 0; c < 3; c++) grad[i * 3 + c] = g0[c];
    gpyr[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

__global__ void k_tex_adam(TexParams p, float* param, const float* grad,
                           float* m, float* v, const float* scalars,
                           float omb1, float omb2) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(p.w_tex) * p.w_tex * 3) return;
    const float bc1 = scalars[1], bc2 = scalars[2];
    const float g = grad[i];
    const float m_new = m[i] * p.b1 + g * omb1;
    const float v_new = v[i] * p.b2 + g * g * omb2;
    const float step = (m_new / bc1) / (sqrtf(v_new / bc2) + p.eps) * p.lr;
    param[i] = param[i] - step;
    m[i] = m_new;
    v[i] = v_new;
}

void mip_build(const TexParams& p, float* pyr, float4* gpyr, cudaStream_t s) {
    ProfScope ps("mip_build", s);
    const int w = p.w_tex;
    int l = 0;
    if (p.levels > 1 && w % kMipTile == 0) {
        // levels 1..5 tile by tile
        const int nlev = std::min(5, p.levels - 1);
        const int tiles = w / kMipTile;
        k_mip_tiles<<<unsigned(tiles * tiles), 256, 0, s>>>(pyr, gpyr, w, nlev);
        l = nlev;
    }
    if (l + 1 < p.levels && (w >> l) <= 64) {
        // the small top levels in one block
        k_mip_top<<<1, 1024, 0, s>>>(pyr, gpyr, w, l, p.levels);
    } else {
        for (; l + 1 < p.levels; l++) {
            const int t = (w >> l) >> 1;
            const size_t n = size_t(t) * t * 3;
            k_mip_level<<<unsigned((n + 255) / 256), 256, 0, s>>>(pyr, gpyr,
                                                                  w, l);
        }
    }
    check_launch();
}

void gbuffer(const TexParams& p, const TexBuffers& b, cudaStream_t s) {
    HardDims hd;
    hd.W = hd.H = p.res;
    hd.views = p.views;
    hd.n_faces = p.n_faces;
    hd.n_verts = p.n_verts;
    hd.n_comp = 3;
    hd.attr_shared = 1;
    hard_raster_op(hd, b.hard_ws, b.clip, b.attr, b.faces, b.gbuf, nullptr,
                   b.status, s);
}

dim3 pixel_grid(const TexParams& p) {
    const int t = (p.res + 15) / 16;
    return dim3(t * t, p.views);
}

}  // namespace

size_t tex_workspace_bytes(const TexParams& p) {
    HardDims hd;
    hd.W = hd.H = p.res;
    hd.views = p.views;
    hd.n_faces = p.n_faces;
    hd.n_verts = p.n_verts;
    hd.n_comp = 3;
    return hard_workspace_bytes(hd);
}

void tex_static_setup(const TexParams& p, const TexBuffers& b,
                      cudaStream_t s) {
    gbuffer(p, b, s);
}

void tex_forward_backward(const TexParams& p, const TexBuffers& b,
                          float* pred_out, cudaStream_t s) {
    mip_build(p, b.pyr, b.gpyr, s);
    {
        ProfScope ps("c2_pixel", s);
        if (p.scatter_runs)
            k_c2_pixel<true><<<pixel_grid(p), 256, 0, s>>>(
                    p, b.pyr, b.gbuf, b.targets, b.gpyr, b.loss_slots,
                    pred_out, 1);
        else
            k_c2_pixel<false><<<pixel_grid(p), 256, 0, s>>>(
                    p, b.pyr, b.gbuf, b.targets, b.gpyr, b.loss_slots,
                    pred_out, 1);
    }
    check_launch();
    {
        ProfScope ps("mip_fold", s);
        const size_t n0 = size_t(p.w_tex) * p.w_tex;
        k_mip_fold<<<unsigned((n0 + 255) / 256), 256, 0, s>>>(
                p, b.gpyr, b.grad, b.scalars, b.loss_slots, b.loss_hist,
                b.hist_cap);
    }
    check_launch();
}

void tex_update(const TexParams& p, const TexBuffers& b, cudaStream_t s) {
    ProfScope ps("tex_adam", s);
    const size_t n0 = size_t(p.w_tex) * p.w_tex * 3;
    k_tex_adam<<<unsigned((n0 + 255) / 256), 256, 0, s>>>(
            p, b.pyr, b.grad, b.adam_m, b.adam_v, b.scalars, 1.f - p.b1,
            1.f - p.b2);
    check_launch();
}

void tex_iteration(const TexParams& p, const TexBuffers& b, cudaStream_t s) {
    tex_forward_backward(p, b, nullptr, s);
    tex_update(p, b, s);
}

void tex_predict(const TexParams& p, const TexBuffers& b, float* out,
                 cudaStream_t s) {
    mip_build(p, b.pyr, nullptr, s);
    k_c2_pixel<false><<<pixel_grid(p), 256, 0, s>>>(
            p, b.pyr, b.gbuf, nullptr, nullptr, nullptr, out, 0);
    check_launch();
}

void tex_render_targets(const TexParams& p, const TexBuffers& b,
                        const float* gt_tex, cudaStream_t s) {
    const size_t nmip = tex_mip_floats(p.w_tex, p.levels);
    void* tmp = nullptr;
    DRESSI_CUDA(cudaMallocAsync(&tmp, nmip * sizeof(float), s));
    float* gt_pyr = static_cast<float*>(tmp);
    DRESSI_CUDA(cudaMemcpyAsync(gt_pyr, gt_tex,
                                size_t(p.w_tex) * p.w_tex * 3 * sizeof(float),
                                cudaMemcpyDeviceToDevice, s));
    mip_build(p, gt_pyr, nullptr, s);
    k_c2_pixel<false><<<pixel_grid(p), 256, 0, s>>>(
            p, gt_pyr, b.gbuf, nullptr, nullptr, nullptr, b.targets, 0);
    check_launch();
    DRESSI_CUDA(cudaFreeAsync(tmp, s));
}

}  // namespace dressi
