// Exact-arithmetic building blocks shared by the rasterizer kernels.
//
// The triangle-ID / coverage / distance outputs must be bit-identical to the
// reference CPU rasterizer (src/core/cpu_raster.cpp). That holds when every
// float expression here keeps the reference's operation order with IEEE
// rounding and no contraction: the library is compiled with -fmad=false
// (and the default -prec-div / -prec-sqrt / -ftz=false), so `a * b + c` is a
// rounded multiply followed by a rounded add, exactly as on x86-64 SSE.
//
// Two C++ library behaviours of the reference are restated explicitly:
//  * std::min(a, b) == (b < a) ? b : a and std::max(a, b) == (a < b) ? b : a
//    (these differ from fminf/fmaxf for NaN and for signed zeros);
//  * int(float) / int64_t(float) on x86-64 (cvttss2si) yield INT_MIN /
//    INT64_MIN for NaN or out-of-range inputs, whereas a CUDA conversion
//    saturates. The reference's bbox loops and index reads depend on it.
#pragma once

#include <climits>
#include <cstdint>

namespace dressi {

__host__ __device__ __forceinline__ float std_min(float a, float b) {
    return (b < a) ? b : a;
}
__host__ __device__ __forceinline__ float std_max(float a, float b) {
    return (a < b) ? b : a;
}

// int(x) as compiled for x86-64.
__host__ __device__ __forceinline__ int x86_i32(float x) {
    return (x >= -2147483648.0f && x < 2147483648.0f) ? int(x) : INT_MIN;
}

// uint32_t(int64_t(x)) as compiled for x86-64 (INT64_MIN has zero low bits).
__host__ __device__ __forceinline__ uint32_t x86_u32_via_i64(float x) {
    return (x >= -9223372036854775808.0f && x < 9223372036854775808.0f)
                   ? uint32_t(uint64_t(int64_t(x)))
                   : 0u;
}

// Wang's integer hash and its [0,1) mapping (f_ops.cpp:1473-1487).
__host__ __device__ __forceinline__ uint32_t wang_hash(uint32_t x) {
    x = (x ^ 61u) ^ (x >> 16);
    x *= 9u;
    x ^= x >> 4;
    x *= 0x27d4eb2du;
    x ^= x >> 15;
    return x;
}
__host__ __device__ __forceinline__ float hash_to_unit(uint32_t f, uint32_t s,
                                                       uint32_t seed,
                                                       uint32_t salt) {
    const uint32_t h = wang_hash(f * 9781u ^ s * 6151u ^ seed * 26699u ^
                                 salt * 42589u);
    return float(h & 0xFFFFFFu) / 16777216.f;
}

__host__ __device__ __forceinline__ int imin_(int a, int b) {
    return a < b ? a : b;
}
__host__ __device__ __forceinline__ int imax_(int a, int b) {
    return a > b ? a : b;
}

// ProjectClipToScreen (cpu_raster.cpp:227-239, via ProjectToScreen 19-27):
// false when |w| <= 1e-6 or w < 0.
__host__ __device__ __forceinline__ bool project_clip(float cx, float cy,
                                                      float cz, float cw,
                                                      float sw, float sh,
                                                      float* x, float* y,
                                                      float* z) {
    if (fabsf(cw) <= 1e-6f || cw < 0.f) return false;
    const float inv_w = 1.f / cw;
    *x = (cx * inv_w * 0.5f + 0.5f) * sw;
    *y = (cy * inv_w * 0.5f + 0.5f) * sh;
    *z = cz * inv_w;
    return true;
}

// Inclusive pixel range of a bbox, RasterizeCore's
// floor(min - 0.5) .. ceil(max - 0.5) clamped to the screen
// (cpu_raster.cpp:73-78).
__host__ __device__ __forceinline__ void bbox_range(float mn, float mx,
                                                    int size, int* lo,
                                                    int* hi) {
    *lo = imax_(0, x86_i32(floorf(mn - 0.5f)));
    *hi = imin_(size - 1, x86_i32(ceilf(mx - 0.5f)));
}

// Clip transform of one vertex: row r = x*m[r] + y*m[4+r] + z*m[8+r] +
// m[12+r] (examples/common/geometry_utils.cpp:391-402; column-major m).
__host__ __device__ __forceinline__ float4 transform_clip(float x, float y,
                                                          float z,
                                                          const float* m) {
    float4 c;
    c.x = x * m[0] + y * m[4] + z * m[8] + m[12];
    c.y = x * m[1] + y * m[5] + z * m[9] + m[13];
    c.z = x * m[2] + y * m[6] + z * m[10] + m[14];
    c.w = x * m[3] + y * m[7] + z * m[11] + m[15];
    return c;
}

}  // namespace dressi
