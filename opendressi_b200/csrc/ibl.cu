// Split-sum IBL ops (config C5) of the reference's f_ops.cpp:2785-3415 and
// ibl_math.h, op level:
//
//   EquirectSample / its map transpose     k_equirect_sample / _bwd
//   IrradianceConv / transpose              k_irradiance_conv / _bwd
//   PrefilterConvNorm / PrefilterConv / T   k_prefilter_norm / _conv / _bwd
//   BrdfIntegrationLut                      k_brdf_lut
//   AvgPool2x2 / transpose                  k_avg_pool2x2 / _bwd
//
// Every expression keeps the reference's operation order. The
// transcendentals (sinf, cosf, atan2f, acosf, powf) are CUDA's, which agree
// with the host libm to a few ulps, as the reference's own GLSL twins do
// (ibl_math.h:6-9): these ops match the reference within the float
// tolerance, except AvgPool2x2, which is bit-exact. The convolutions are
// dense out x src sums (FP32-ALU-bound): one block per output (or source)
// texel reduces over the other side with the directions precomputed.
#include <algorithm>

#include "kernels.h"

namespace dressi {

namespace {

constexpr float kPiF = 3.14159265358979323846f;
constexpr float kTwoPiF = 6.28318530717958647692f;
constexpr float kInvPiF = 0.31830988618379067154f;
constexpr float kInvTwoPiF = 0.15915494309189533577f;

__device__ __forceinline__ float dot3(const float* a, const float* b) {
    return a[0] * b[0] + a[1] * b[1] + a[2] * b[2];
}

// EquirectUvFromDir (ibl_math.h:39-44)
__device__ __forceinline__ void equirect_uv(const float d[3], float* u,
                                            float* v) {
    *u = atan2f(d[2], d[0]) * kInvTwoPiF + 0.5f;
    const float y = d[1] < -1.f ? -1.f : (1.f < d[1] ? 1.f : d[1]);
    *v = acosf(y) * kInvPiF;
}

// DirFromEquirectUv (ibl_math.h:47-52)
__device__ __forceinline__ void equirect_dir(float u, float v, float d[3]) {
    const float phi = (u - 0.5f) * kTwoPiF;
    const float theta = v * kPiF;
    const float st = sinf(theta);
    d[0] = st * cosf(phi);
    d[1] = cosf(theta);
    d[2] = st * sinf(phi);
}

// The 4 taps of BilerpWrap (ibl_math.h:56-86): u wraps, v clamps; (dy, dx)
// order.
__device__ __forceinline__ void wrap_taps(int w, int h, float u, float v,
                                          int idx[4], float wt[4]) {
    const float sx = u * float(w) - 0.5f;
    const float sy = v * float(h) - 0.5f;
    const int ix = x86_i32(floorf(sx));
    const int iy = x86_i32(floorf(sy));
    const float fx = sx - float(ix);
    const float fy = sy - float(iy);
#pragma unroll
    for (int dy = 0; dy <= 1; dy++)
#pragma unroll
        for (int dx = 0; dx <= 1; dx++) {
            int x = ix + dx;
            if (x < 0) x += w;
            if (x >= w) x -= w;
            int y = iy + dy;
            y = y < 0 ? 0 : (y > h - 1 ? h - 1 : y);
            const int k = dy * 2 + dx;
            idx[k] = y * w + x;
            wt[k] = (dx == 0 ? 1.f - fx : fx) * (dy == 0 ? 1.f - fy : fy);
        }
}

// Unit direction of a dir pixel; false for |d| < 1e-8 (background).
__device__ __forceinline__ bool unit_dir(const float* p, float d[3]) {
    d[0] = p[0];
    d[1] = p[1];
    d[2] = p[2];
    const float len = sqrtf(dot3(d, d));
    if (len < 1e-8f) return false;
    d[0] = d[0] / len;
    d[1] = d[1] / len;
    d[2] = d[2] / len;
    return true;
}

// GgxConvWeight (ibl_math.h:160-168)
__device__ __forceinline__ float ggx_conv_weight(float c, float alpha) {
    if (c <= 0.f) return 0.f;
    const float ch2 = (1.f + c) * 0.5f;
    const float a2 = alpha * alpha;
    const float d = ch2 * (a2 - 1.f) + 1.f;
    return a2 / (kPiF * d * d) * c;
}

template <int NC>
__global__ void k_equirect_sample(const float* map, int mw, int mh,
                                  const float* dir, long long n_px,
                                  float* out) {
    const long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (p >= n_px) return;
    float o[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) o[c] = 0.f;
    float d[3];
    if (unit_dir(dir + p * 3, d)) {
        float u, v;
        equirect_uv(d, &u, &v);
        int idx[4];
        float wt[4];
        wrap_taps(mw, mh, u, v, idx, wt);
#pragma unroll
        for (int k = 0; k < 4; k++)
#pragma unroll
            for (int c = 0; c < NC; c++)
                o[c] += wt[k] * map[size_t(idx[k]) * NC + c];
    }
#pragma unroll
    for (int c = 0; c < NC; c++) out[p * NC + c] = o[c];
}

// The map transpose: each pixel scatters gy * weight into its 4 taps
// (float atomics; the reference sums the same terms per texel in pixel
// order, so the two agree within float rounding).
template <int NC>
__global__ void k_equirect_sample_bwd(const float* gy, const float* dir,
                                      long long n_px, int mw, int mh,
                                      float* g_map) {
    const long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (p >= n_px) return;
    float d[3];
    if (!unit_dir(dir + p * 3, d)) return;
    float u, v;
    equirect_uv(d, &u, &v);
    int idx[4];
    float wt[4];
    wrap_taps(mw, mh, u, v, idx, wt);
#pragma unroll
    for (int k = 0; k < 4; k++)
#pragma unroll
        for (int c = 0; c < NC; c++)
            atomicAdd(&g_map[size_t(idx[k]) * NC + c], gy[p * NC + c] * wt[k]);
}

// Direction and sin(theta) of every texel of a w x h equirect map.
__global__ void k_texel_dirs(int w, int h, float4* out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= w * h) return;
    const int x = i % w, y = i / w;
    const float v = (float(y) + 0.5f) / float(h);
    float d[3];
    equirect_dir((float(x) + 0.5f) / float(w), v, d);
    out[i] = make_float4(d[0], d[1], d[2], sinf(v * kPiF));
}

constexpr int kConvThreads = 256;

// Block-wide sum of NC floats per thread (result in thread 0's v).
template <int NC>
__device__ __forceinline__ void block_sum(float v[NC], float (*red)[NC]) {
#pragma unroll
    for (int c = 0; c < NC; c++) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            v[c] += __shfl_down_sync(0xffffffffu, v[c], o);
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0)
#pragma unroll
        for (int c = 0; c < NC; c++) red[w][c] = v[c];
    __syncthreads();
    if (w == 0) {
#pragma unroll
        for (int c = 0; c < NC; c++) {
            v[c] = lane < int(blockDim.x >> 5) ? red[lane][c] : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                v[c] += __shfl_down_sync(0xffffffffu, v[c], o);
        }
    }
}

// Irradiance / prefilter convolution forward: one block per output texel
// (dirs_out[blockIdx.x]), threads strided over the sources. kind 0:
// max(N.d, 0) sin * scale; kind 1: GgxConvWeight(R.d, alpha) sin / W(t).
template <int NC, int kKind>
__global__ void __launch_bounds__(kConvThreads)
k_env_conv(const float* env, const float4* src_dirs, int n_src,
           const float4* out_dirs, float scale_or_alpha, const float* norm,
           float* out) {
    __shared__ float red[kConvThreads / 32][NC];
    const int t = blockIdx.x;
    const float4 r4 = out_dirs[t];
    const float r[3] = {r4.x, r4.y, r4.z};
    float acc[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) acc[c] = 0.f;
    for (int s = threadIdx.x; s < n_src; s += blockDim.x) {
        const float4 d4 = src_dirs[s];
        const float d[3] = {d4.x, d4.y, d4.z};
        float w;
        if (kKind == 0) {
            const float nd = dot3(r, d);
            w = (nd < 0.f ? 0.f : nd) * d4.w;
        } else {
            w = ggx_conv_weight(dot3(r, d), scale_or_alpha) * d4.w;
        }
#pragma unroll
        for (int c = 0; c < NC; c++) acc[c] += env[size_t(s) * NC + c] * w;
    }
    block_sum<NC>(acc, red);
    if (threadIdx.x == 0) {
        if (kKind == 0) {
#pragma unroll
            for (int c = 0; c < NC; c++) out[size_t(t) * NC + c] = acc[c] * scale_or_alpha;
        } else {
            const float wn = fmaxf(norm[t], 1e-12f);
#pragma unroll
            for (int c = 0; c < NC; c++) out[size_t(t) * NC + c] = acc[c] / wn;
        }
    }
}

// The transposes: one block per source texel, threads strided over the
// output texels.
template <int NC, int kKind>
__global__ void __launch_bounds__(kConvThreads)
k_env_conv_bwd(const float* gy, const float4* out_dirs, int n_out,
               const float4* src_dirs, float scale_or_alpha,
               const float* norm, float* g_env, int acc) {
    __shared__ float red[kConvThreads / 32][NC];
    const int s = blockIdx.x;
    const float4 d4 = src_dirs[s];
    const float d[3] = {d4.x, d4.y, d4.z};
    float sum[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) sum[c] = 0.f;
    for (int t = threadIdx.x; t < n_out; t += blockDim.x) {
        const float4 r4 = out_dirs[t];
        const float r[3] = {r4.x, r4.y, r4.z};
        float w;
        if (kKind == 0) {
            const float nd = dot3(r, d);
            w = (nd < 0.f ? 0.f : nd) * d4.w;
        } else {
            const float g = ggx_conv_weight(dot3(r, d), scale_or_alpha);
            if (g <= 0.f) continue;
            w = g / fmaxf(norm[t], 1e-12f);
        }
#pragma unroll
        for (int c = 0; c < NC; c++) sum[c] += gy[size_t(t) * NC + c] * w;
    }
    block_sum<NC>(sum, red);
    if (threadIdx.x == 0) {
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const float v = kKind == 0 ? sum[c] * scale_or_alpha
                                       : sum[c] * d4.w;
            g_env[size_t(s) * NC + c] = acc ? g_env[size_t(s) * NC + c] + v : v;
        }
    }
}

// PrefilterConvNorm: W(t) = sum_s GgxConvWeight(R_t . d_s) sin(theta_s).
__global__ void __launch_bounds__(kConvThreads)
k_prefilter_norm(const float4* src_dirs, int n_src, const float4* out_dirs,
                 float alpha, float* norm) {
    __shared__ float red[kConvThreads / 32][1];
    const float4 r4 = out_dirs[blockIdx.x];
    const float r[3] = {r4.x, r4.y, r4.z};
    float acc[1] = {0.f};
    for (int s = threadIdx.x; s < n_src; s += blockDim.x) {
        const float4 d4 = src_dirs[s];
        const float d[3] = {d4.x, d4.y, d4.z};
        acc[0] += ggx_conv_weight(dot3(r, d), alpha) * d4.w;
    }
    block_sum<1>(acc, red);
    if (threadIdx.x == 0) norm[blockIdx.x] = acc[0];
}

// RadicalInverse (ibl_math.h:119-126)
__device__ __forceinline__ float radical_inverse(uint32_t b) {
    b = (b << 16u) | (b >> 16u);
    b = ((b & 0x55555555u) << 1u) | ((b & 0xAAAAAAAAu) >> 1u);
    b = ((b & 0x33333333u) << 2u) | ((b & 0xCCCCCCCCu) >> 2u);
    b = ((b & 0x0F0F0F0Fu) << 4u) | ((b & 0xF0F0F0F0u) >> 4u);
    b = ((b & 0x00FF00FFu) << 8u) | ((b & 0xFF00FF00u) >> 8u);
    return float(b) * 2.3283064365386963e-10f;
}

__device__ __forceinline__ void normalize3(float v[3]) {
    const float len = sqrtf(dot3(v, v));
    v[0] = v[0] / len;
    v[1] = v[1] / len;
    v[2] = v[2] / len;
}

// BrdfIntegrationLut (f_ops.cpp:3350-3408): one thread per texel, the
// samples in order (ImportanceSampleGGX about +Z, ibl_math.h:135-150).
__global__ void k_brdf_lut(int w, int h, int n_samples, float2* out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= w * h) return;
    const int ox = i % w, oy = i / w;
    const float rough = (float(oy) + 0.5f) / float(h);
    const float k = rough * rough / 2.f;
    const float ndv = (float(ox) + 0.5f) / float(w);
    const float s2 = 1.f - ndv * ndv;
    const float V[3] = {sqrtf(s2 < 0.f ? 0.f : s2), 0.f, ndv};
    // tangent frame of N = +Z (up = +X): tx = normalize(up x N), ty = N x tx
    float tx[3] = {0.f * 1.f - 0.f * 0.f, 0.f * 0.f - 1.f * 1.f,
                   1.f * 0.f - 0.f * 0.f};
    normalize3(tx);
    const float ty[3] = {0.f * tx[2] - 1.f * tx[1], 1.f * tx[0] - 0.f * tx[2],
                         0.f * tx[1] - 0.f * tx[0]};
    const float a = rough * rough;
    float sa = 0.f, sb = 0.f;
    for (int s = 0; s < n_samples; s++) {
        const float xi0 = float(s) / float(n_samples);
        const float xi1 = radical_inverse(uint32_t(s));
        const float phi = kTwoPiF * xi0;
        const float ct = sqrtf((1.f - xi1) / (1.f + (a * a - 1.f) * xi1));
        const float st2 = 1.f - ct * ct;
        const float st = sqrtf(st2 < 0.f ? 0.f : st2);
        const float ht[3] = {cosf(phi) * st, sinf(phi) * st, ct};
        float hv[3] = {tx[0] * ht[0] + ty[0] * ht[1] + 0.f * ht[2],
                       tx[1] * ht[0] + ty[1] * ht[1] + 0.f * ht[2],
                       tx[2] * ht[0] + ty[2] * ht[1] + 1.f * ht[2]};
        normalize3(hv);
        const float vdh2 = 2.f * dot3(V, hv);
        float l[3] = {vdh2 * hv[0] - V[0], vdh2 * hv[1] - V[1],
                      vdh2 * hv[2] - V[2]};
        normalize3(l);
        const float nol = l[2] < 0.f ? 0.f : l[2];
        const float noh = hv[2] < 0.f ? 0.f : hv[2];
        const float vh = dot3(V, hv);
        const float voh = vh < 0.f ? 0.f : vh;
        if (nol > 0.f) {
            const float g = (ndv / (ndv * (1.f - k) + k)) *
                            (nol / (nol * (1.f - k) + k));
            const float den = noh * ndv;
            const float gv = g * voh / (den < 1e-8f ? 1e-8f : den);
            const float fc = powf(1.f - voh, 5.f);
            sa += (1.f - fc) * gv;
            sb += fc * gv;
        }
    }
    out[i] = make_float2(sa / float(n_samples), sb / float(n_samples));
}

// AvgPool2x2: ((a + b) + c + d) * 0.25 in the reference's order (bit-exact)
__global__ void k_avg_pool2x2(const float* x, int w, int h, int n,
                              float* out) {
    const int ow = w / 2, oh = h / 2;
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)ow * oh * n) return;
    const int c = int(i % n);
    const long long p = i / n;
    const int ox = int(p % ow), oy = int(p / ow);
    const float* r0 = x + (size_t(2 * oy) * w + 2 * ox) * n + c;
    const float* r1 = r0 + size_t(w) * n;
    out[i] = (((r0[0] + r0[n]) + r1[0]) + r1[n]) * 0.25f;
}

// Its transpose: every source texel receives 0.25 * its output's gradient.
__global__ void k_avg_pool2x2_bwd(const float* gy, int w, int h, int n,
                                  float* g) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)w * h * n) return;
    const int c = int(i % n);
    const long long p = i / n;
    const int x = int(p % w), y = int(p / w);
    g[i] = gy[(size_t(y / 2) * (w / 2) + x / 2) * n + c] * 0.25f;
}

inline unsigned grid_for(long long n, int threads) {
    return unsigned((n + threads - 1) / threads);
}

void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

}  // namespace

// ------------------------------------------------------------ op entries

void equirect_sample_op(const float* map, int mw, int mh, int n,
                        const float* dir, long long n_px, float* out,
                        cudaStream_t s) {
    if (n_px <= 0) return;
    ProfScope ps("equirect_sample", s);
    const unsigned g = grid_for(n_px, 256);
    switch (n) {
        case 1: k_equirect_sample<1><<<g, 256, 0, s>>>(map, mw, mh, dir, n_px, out); break;
        case 2: k_equirect_sample<2><<<g, 256, 0, s>>>(map, mw, mh, dir, n_px, out); break;
        case 3: k_equirect_sample<3><<<g, 256, 0, s>>>(map, mw, mh, dir, n_px, out); break;
        default: k_equirect_sample<4><<<g, 256, 0, s>>>(map, mw, mh, dir, n_px, out); break;
    }
    check_launch();
}

void equirect_sample_bwd_op(const float* gy, const float* dir, long long n_px,
                            int mw, int mh, int n, float* g_map,
                            cudaStream_t s) {
    DRESSI_CUDA(cudaMemsetAsync(g_map, 0, size_t(mw) * mh * n * 4, s));
    if (n_px <= 0) return;
    ProfScope ps("equirect_sample_bwd", s);
    const unsigned g = grid_for(n_px, 256);
    switch (n) {
        case 1: k_equirect_sample_bwd<1><<<g, 256, 0, s>>>(gy, dir, n_px, mw, mh, g_map); break;
        case 2: k_equirect_sample_bwd<2><<<g, 256, 0, s>>>(gy, dir, n_px, mw, mh, g_map); break;
        case 3: k_equirect_sample_bwd<3><<<g, 256, 0, s>>>(gy, dir, n_px, mw, mh, g_map); break;
        default: k_equirect_sample_bwd<4><<<g, 256, 0, s>>>(gy, dir, n_px, mw, mh, g_map); break;
    }
    check_launch();
}

void texel_dirs_op(int w, int h, float4* out, cudaStream_t s) {
    k_texel_dirs<<<grid_for((long long)w * h, 256), 256, 0, s>>>(w, h, out);
    check_launch();
}

size_t env_conv_scratch_floats(int sw, int sh, int ow, int oh) {
    // 256-byte aligned float4 tables of both sides plus the norm
    auto al = [](size_t f) { return (f + 63) / 64 * 64; };
    return al(size_t(sw) * sh * 4) + al(size_t(ow) * oh * 4) +
           al(size_t(ow) * oh);
}

namespace {

struct ConvTables {
    float4* src;
    float4* out;
    float* norm;
};

ConvTables carve_conv(float* scratch, int sw, int sh, int ow, int oh) {
    auto al = [](size_t f) { return (f + 63) / 64 * 64; };
    ConvTables t;
    t.src = reinterpret_cast<float4*>(scratch);
    t.out = reinterpret_cast<float4*>(scratch + al(size_t(sw) * sh * 4));
    t.norm = scratch + al(size_t(sw) * sh * 4) + al(size_t(ow) * oh * 4);
    return t;
}

template <int kKind>
void env_conv_launch(const float* env, int n, const ConvTables& t, int n_src,
                     int n_out, float scale_or_alpha, float* out,
                     cudaStream_t s) {
    switch (n) {
        case 1: k_env_conv<1, kKind><<<n_out, kConvThreads, 0, s>>>(env, t.src, n_src, t.out, scale_or_alpha, t.norm, out); break;
        case 2: k_env_conv<2, kKind><<<n_out, kConvThreads, 0, s>>>(env, t.src, n_src, t.out, scale_or_alpha, t.norm, out); break;
        case 3: k_env_conv<3, kKind><<<n_out, kConvThreads, 0, s>>>(env, t.src, n_src, t.out, scale_or_alpha, t.norm, out); break;
        default: k_env_conv<4, kKind><<<n_out, kConvThreads, 0, s>>>(env, t.src, n_src, t.out, scale_or_alpha, t.norm, out); break;
    }
    check_launch();
}

template <int kKind>
void env_conv_bwd_launch(const float* gy, int n, const ConvTables& t,
                         int n_src, int n_out, float scale_or_alpha,
                         float* g_env, cudaStream_t s) {
    switch (n) {
        case 1: k_env_conv_bwd<1, kKind><<<n_src, kConvThreads, 0, s>>>(gy, t.out, n_out, t.src, scale_or_alpha, t.norm, g_env, 0); break;
        case 2: k_env_conv_bwd<2, kKind><<<n_src, kConvThreads, 0, s>>>(gy, t.out, n_out, t.src, scale_or_alpha, t.norm, g_env, 0); break;
        case 3: k_env_conv_bwd<3, kKind><<<n_src, kConvThreads, 0, s>>>(gy, t.out, n_out, t.src, scale_or_alpha, t.norm, g_env, 0); break;
        default: k_env_conv_bwd<4, kKind><<<n_src, kConvThreads, 0, s>>>(gy, t.out, n_out, t.src, scale_or_alpha, t.norm, g_env, 0); break;
    }
    check_launch();
}

}  // namespace

void env_conv_run(int kind, const float* env, int n, const float4* src_dirs,
                  int n_src, const float4* out_dirs, int n_out,
                  float scale_or_alpha, const float* norm, float* out,
                  cudaStream_t s) {
    const ConvTables t{const_cast<float4*>(src_dirs),
                       const_cast<float4*>(out_dirs),
                       const_cast<float*>(norm)};
    if (kind == 0)
        env_conv_launch<0>(env, n, t, n_src, n_out, scale_or_alpha, out, s);
    else
        env_conv_launch<1>(env, n, t, n_src, n_out, scale_or_alpha, out, s);
}

void env_conv_bwd_run(int kind, const float* gy, int n,
                      const float4* src_dirs, int n_src,
                      const float4* out_dirs, int n_out, float scale_or_alpha,
                      const float* norm, float* g_env, bool accumulate,
                      cudaStream_t s) {
    const int acc = accumulate ? 1 : 0;
#define DRESSI_BWD(NC, K)                                                    \
    k_env_conv_bwd<NC, K><<<n_src, kConvThreads, 0, s>>>(                    \
            gy, out_dirs, n_out, src_dirs, scale_or_alpha, norm, g_env, acc)
    if (kind == 0) {
        if (n == 3) DRESSI_BWD(3, 0); else if (n == 1) DRESSI_BWD(1, 0);
        else if (n == 2) DRESSI_BWD(2, 0); else DRESSI_BWD(4, 0);
    } else {
        if (n == 3) DRESSI_BWD(3, 1); else if (n == 1) DRESSI_BWD(1, 1);
        else if (n == 2) DRESSI_BWD(2, 1); else DRESSI_BWD(4, 1);
    }
#undef DRESSI_BWD
    check_launch();
}

void prefilter_norm_op(const float4* src_dirs, int n_src,
                       const float4* out_dirs, int n_out, float alpha,
                       float* norm, cudaStream_t s) {
    k_prefilter_norm<<<n_out, kConvThreads, 0, s>>>(src_dirs, n_src, out_dirs,
                                                    alpha, norm);
    check_launch();
}

void irradiance_conv_op(const float* env, int sw, int sh, int n, int ow,
                        int oh, float* out, float* scratch, cudaStream_t s) {
    ProfScope ps("irradiance_conv", s);
    const ConvTables t = carve_conv(scratch, sw, sh, ow, oh);
    texel_dirs_op(sw, sh, t.src, s);
    texel_dirs_op(ow, oh, t.out, s);
    env_conv_launch<0>(env, n, t, sw * sh, ow * oh,
                       kTwoPiF / (float(sw) * float(sh)), out, s);
}

void irradiance_conv_bwd_op(const float* gy, int ow, int oh, int n, int sw,
                            int sh, float* g_env, float* scratch,
                            cudaStream_t s) {
    ProfScope ps("irradiance_conv_bwd", s);
    const ConvTables t = carve_conv(scratch, sw, sh, ow, oh);
    texel_dirs_op(sw, sh, t.src, s);
    texel_dirs_op(ow, oh, t.out, s);
    env_conv_bwd_launch<0>(gy, n, t, sw * sh, ow * oh,
                           kTwoPiF / (float(sw) * float(sh)), g_env, s);
}

float prefilter_alpha(float roughness) {
    const float r = std::max(roughness, 0.045f);
    return r * r;
}

void prefilter_conv_op(const float* env, int sw, int sh, int n, int ow,
                       int oh, float roughness, float* out, float* scratch,
                       cudaStream_t s) {
    ProfScope ps("prefilter_conv", s);
    const ConvTables t = carve_conv(scratch, sw, sh, ow, oh);
    const float alpha = prefilter_alpha(roughness);
    texel_dirs_op(sw, sh, t.src, s);
    texel_dirs_op(ow, oh, t.out, s);
    prefilter_norm_op(t.src, sw * sh, t.out, ow * oh, alpha, t.norm, s);
    env_conv_launch<1>(env, n, t, sw * sh, ow * oh, alpha, out, s);
}

void prefilter_conv_bwd_op(const float* gy, int ow, int oh, int n, int sw,
                           int sh, float roughness, float* g_env,
                           float* scratch, cudaStream_t s) {
    ProfScope ps("prefilter_conv_bwd", s);
    const ConvTables t = carve_conv(scratch, sw, sh, ow, oh);
    const float alpha = prefilter_alpha(roughness);
    texel_dirs_op(sw, sh, t.src, s);
    texel_dirs_op(ow, oh, t.out, s);
    prefilter_norm_op(t.src, sw * sh, t.out, ow * oh, alpha, t.norm, s);
    env_conv_bwd_launch<1>(gy, n, t, sw * sh, ow * oh, alpha, g_env, s);
}

void brdf_lut_op(int w, int h, int n_samples, float* out, cudaStream_t s) {
    ProfScope ps("brdf_lut", s);
    k_brdf_lut<<<grid_for((long long)w * h, 128), 128, 0, s>>>(
            w, h, n_samples, reinterpret_cast<float2*>(out));
    check_launch();
}

void avg_pool2x2_op(const float* x, int w, int h, int n, float* out,
                    cudaStream_t s) {
    const long long total = (long long)(w / 2) * (h / 2) * n;
    if (total <= 0) return;
    ProfScope ps("avg_pool2x2", s);
    k_avg_pool2x2<<<grid_for(total, 256), 256, 0, s>>>(x, w, h, n, out);
    check_launch();
}

void avg_pool2x2_bwd_op(const float* gy, int w, int h, int n, float* g,
                        cudaStream_t s) {
    const long long total = (long long)w * h * n;
    if (total <= 0) return;
    ProfScope ps("avg_pool2x2_bwd", s);
    k_avg_pool2x2_bwd<<<grid_for(total, 256), 256, 0, s>>>(gy, w, h, n, g);
    check_launch();
}

}  // namespace dressi
