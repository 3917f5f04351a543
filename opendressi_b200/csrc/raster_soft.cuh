// HardSoftRas soft rasterizer for sm_100a: tile-binned, order-independent,
// bit-exact with the reference's sequential RasterizeSoftCpu
// (src/core/cpu_raster.cpp:241-355).
//
// Why order-independent is exact: the reference walks faces in order and
// keeps a fragment when `depth <= zbuf`, so the survivor of a pixel is the
// fragment with the smallest (depth, -face) key -- the latest face wins ties.
// Each thread here owns one pixel and folds fragments into that key in any
// order, which gives the same survivor (for finite depths).
//
// Work split (per view, 16x16-pixel tiles, one CTA per tile):
//  sweep 1: every fragment inside a face's *sweep-1 region* -- the hard
//           triangle's bbox grown by kHardMargin pixels (or the whole soft
//           bbox for faces flagged unsafe) -- is evaluated in full.
//  sweep 2: only tiles that still hold a pixel whose best depth is > 0.5
//           (not covered by a hard fragment) see the remaining soft-rim
//           fragments of safe faces (soft bbox minus sweep-1 region).
// A fragment outside the hard bbox + margin of a *safe* face is provably a
// rim fragment with dist <= -kHardMargin, hence depth > 0.5, so it can never
// beat a hard fragment: skipping it for tiles whose pixels all have
// depth <= 0.5 cannot change any output. "Safe" bounds the sign-test
// rounding error: every angle of the hard triangle must satisfy
// sin(theta/2) > kSafeSlope * L, L the largest pixel distance the face's
// soft bbox reaches from a hard vertex (the rounding error of the edge
// function is <= ~5u*|e|*L, its exact value outside the margin is
// >= 2*sin(theta/2)*|e| * kHardMargin/2); faces failing it, or with huge
// coordinates, are evaluated exhaustively in sweep 1.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "exact.cuh"

namespace dressi {

constexpr int kTile = 16;                // tile edge in pixels
constexpr int kTileThreads = kTile * kTile;
constexpr int kHardMargin = 2;           // sweep-1 bbox growth (pixels)
constexpr float kSafeSlope = 1.5e-6f;    // see header comment
constexpr float kCoordLimit = 1048576.f; // |screen coord| bound for "safe"

// Device status word bits (mirrored in include/dressi_b200.h).
constexpr uint32_t kStatusIndexRange = 0x1u;
constexpr uint32_t kStatusBinOverflow = 0x2u;
constexpr uint32_t kStatusNonFinite = 0x4u;

enum FaceFlags : uint32_t {
    kFaceValid = 1u,     // produces fragments
    kFaceHardBary = 2u,  // hard ScreenBarycentric succeeds
    kFaceSafe = 4u,      // sweep-2 skipping is exact for this face
};

// Per-(view, face) constants hoisted out of the per-pixel loop. Every value
// is computed with the reference's own expression, so hoisting is exact.
struct __align__(16) FaceRec {
    float s0x, s0y, s1x, s1y;  // soft triangle, screen px
    float s2x, s2y, s_inv_area, fid;
    float sz0, sz1, sz2, pad0;  // soft vertex NDC depth
    float h0x, h0y, h1x, h1y;   // hard triangle, screen px
    float h2x, h2y, h_inv_area, hz0;
    float hz1, hz2, ex0, ey0;   // hard edges e_k = h[k+1] - h[k]
    float ex1, ey1, ex2, ey2;
    float len2_0, len2_1, len2_2, pad1;
    int bx0, bx1, by0, by1;  // soft bbox pixel range (inclusive)
    int rx0, rx1, ry0, ry1;  // sweep-1 region pixel range (inclusive)
    uint32_t flags, i0, i1, i2;  // flags + hard vertex indices
};
static_assert(sizeof(FaceRec) == 176, "FaceRec layout");
constexpr int kRecVec4 = sizeof(FaceRec) / 16;

// Per-pixel survivor carried from sweep 1 to sweep 2.
struct __align__(16) PixState {
    float depth;  // Eq.3 shifted depth of the survivor (1 = clear)
    int face;     // soft face index of the survivor (-1 = none)
    float dist;   // signed distance to its hard triangle
    float hard_z; // unclamped hard depth
};

struct TriDist {
    float dist;
    int edge;
    float t;
};

// SignedDistToTri (cpu_raster.cpp:114-151) with the per-edge constants
// (e, |e|^2) read from the record.
__device__ __forceinline__ TriDist signed_dist(float px, float py,
                                               const FaceRec& r) {
    const float ax[3] = {r.h0x, r.h1x, r.h2x};
    const float ay[3] = {r.h0y, r.h1y, r.h2y};
    const float exs[3] = {r.ex0, r.ex1, r.ex2};
    const float eys[3] = {r.ey0, r.ey1, r.ey2};
    const float l2s[3] = {r.len2_0, r.len2_1, r.len2_2};
    TriDist best{0.f, 0, 0.f};
    float best_d2 = -1.f;
    int n_pos = 0, n_neg = 0;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const float ex = exs[k], ey = eys[k], len2 = l2s[k];
        float t = 0.f;
        if (len2 > 1e-6f * 1e-6f) {
            t = ((px - ax[k]) * ex + (py - ay[k]) * ey) / len2;
            t = std_min(std_max(t, 0.f), 1.f);
        }
        const float qx = ax[k] + t * ex;
        const float qy = ay[k] + t * ey;
        const float dx = px - qx;
        const float dy = py - qy;
        const float d2 = dx * dx + dy * dy;
        if (best_d2 < 0.f || d2 < best_d2) {
            best_d2 = d2;
            best.edge = k;
            best.t = t;
        }
        const float cr = ex * (py - ay[k]) - ey * (px - ax[k]);
        n_pos += (cr >= 0.f);
        n_neg += (cr <= 0.f);
    }
    const float sgn = (n_pos == 3 || n_neg == 3) ? 1.f : -1.f;
    best.dist = sgn * sqrtf(std_max(best_d2, 0.f));
    return best;
}

// Unclamped hard depth: ScreenBarycentric on the hard triangle, 0.5 when it
// is degenerate (cpu_raster.cpp:323-328).
__device__ __forceinline__ float hard_depth(float px, float py,
                                            const FaceRec& r) {
    if (!(r.flags & kFaceHardBary)) return 0.5f;
    const float l0 = ((r.h1x - px) * (r.h2y - py) - (r.h1y - py) * (r.h2x - px)) *
                     r.h_inv_area;
    const float l1 = ((r.h2x - px) * (r.h0y - py) - (r.h2y - py) * (r.h0x - px)) *
                     r.h_inv_area;
    const float l2 = 1.f - l0 - l1;
    return l0 * r.hz0 + l1 * r.hz1 + l2 * r.hz2;
}

// Soft coverage test (ScreenBarycentric of the soft triangle, all lambdas
// >= 0) and the soft depth range test (cpu_raster.cpp:310-321).
__device__ __forceinline__ bool soft_covers(float px, float py,
                                            const FaceRec& r) {
    const float l0 = ((r.s1x - px) * (r.s2y - py) - (r.s1y - py) * (r.s2x - px)) *
                     r.s_inv_area;
    const float l1 = ((r.s2x - px) * (r.s0y - py) - (r.s2y - py) * (r.s0x - px)) *
                     r.s_inv_area;
    const float l2 = 1.f - l0 - l1;
    if (l0 < 0.f || l1 < 0.f || l2 < 0.f) return false;
    const float z = l0 * r.sz0 + l1 * r.sz1 + l2 * r.sz2;
    return !(z < 0.f || z > 1.f);
}

// Eq.3 depth shift (cpu_raster.cpp:329-334).
__device__ __forceinline__ float shifted_depth(float dist, float hard_z,
                                               float radius) {
    return dist >= 0.f ? 0.5f * std_min(std_max(hard_z, 0.f), 1.f)
                       : 0.5f + 0.5f * std_min(-dist / radius, 1.f);
}

// Fold a fragment into the survivor key (smaller depth, later face on ties).
__device__ __forceinline__ bool beats(float depth, int face, float best_depth,
                                      int best_face) {
    return depth < best_depth || (depth == best_depth && face > best_face);
}

// ----------------------------------------------------------- record setup

// Fills the record of a soft face from its projected soft and hard
// triangles. Returns false when the face yields no fragment.
__device__ __forceinline__ bool build_record(
        const float ss[3][2], const float sz[3], const float hs[3][2],
        const float hz[3], float fid, const uint32_t hidx[3], int W, int H,
        FaceRec* out) {
    FaceRec r;
    // Soft barycentric denominator (ScreenBarycentric, cpu_raster.cpp:177-193)
    const float s_area = (ss[1][0] - ss[0][0]) * (ss[2][1] - ss[0][1]) -
                         (ss[1][1] - ss[0][1]) * (ss[2][0] - ss[0][0]);
    // Soft bbox (cpu_raster.cpp:299-307)
    const float mnx = std_min(std_min(ss[0][0], ss[1][0]), ss[2][0]);
    const float mxx = std_max(std_max(ss[0][0], ss[1][0]), ss[2][0]);
    const float mny = std_min(std_min(ss[0][1], ss[1][1]), ss[2][1]);
    const float mxy = std_max(std_max(ss[0][1], ss[1][1]), ss[2][1]);
    bbox_range(mnx, mxx, W, &r.bx0, &r.bx1);
    bbox_range(mny, mxy, H, &r.by0, &r.by1);
    uint32_t flags = 0;
    // A degenerate soft triangle makes ScreenBarycentric fail for every
    // pixel: no fragments.
    if (!(fabsf(s_area) < 1e-6f) && r.bx0 <= r.bx1 && r.by0 <= r.by1) {
        flags |= kFaceValid;
    }
    r.s0x = ss[0][0]; r.s0y = ss[0][1];
    r.s1x = ss[1][0]; r.s1y = ss[1][1];
    r.s2x = ss[2][0]; r.s2y = ss[2][1];
    r.s_inv_area = 1.f / s_area;
    r.fid = fid;
    r.sz0 = sz[0]; r.sz1 = sz[1]; r.sz2 = sz[2];
    r.pad0 = 0.f;
    r.h0x = hs[0][0]; r.h0y = hs[0][1];
    r.h1x = hs[1][0]; r.h1y = hs[1][1];
    r.h2x = hs[2][0]; r.h2y = hs[2][1];
    const float h_area = (hs[1][0] - hs[0][0]) * (hs[2][1] - hs[0][1]) -
                         (hs[1][1] - hs[0][1]) * (hs[2][0] - hs[0][0]);
    if (!(fabsf(h_area) < 1e-6f)) flags |= kFaceHardBary;
    r.h_inv_area = 1.f / h_area;
    r.hz0 = hz[0]; r.hz1 = hz[1]; r.hz2 = hz[2];
    float exs[3], eys[3], l2s[3];
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const int k2 = (k + 1) % 3;
        exs[k] = hs[k2][0] - hs[k][0];
        eys[k] = hs[k2][1] - hs[k][1];
        l2s[k] = exs[k] * exs[k] + eys[k] * eys[k];
    }
    r.ex0 = exs[0]; r.ey0 = eys[0]; r.ex1 = exs[1]; r.ey1 = eys[1];
    r.ex2 = exs[2]; r.ey2 = eys[2];
    r.len2_0 = l2s[0]; r.len2_1 = l2s[1]; r.len2_2 = l2s[2];
    r.pad1 = 0.f;
    r.i0 = hidx[0]; r.i1 = hidx[1]; r.i2 = hidx[2];

    // Safety classification (all in double; only decides how much work is
    // done, never a result).
    bool safe = true;
    double hmnx = 1e300, hmxx = -1e300, hmny = 1e300, hmxy = -1e300;
    for (int k = 0; k < 3; k++) {
        const double x = hs[k][0], y = hs[k][1];
        if (!(fabs(x) < kCoordLimit && fabs(y) < kCoordLimit)) safe = false;
        hmnx = fmin(hmnx, x); hmxx = fmax(hmxx, x);
        hmny = fmin(hmny, y); hmxy = fmax(hmxy, y);
    }
    if (safe) {
        double L = 0.0;
        const double cx[2] = {double(r.bx0) - 1.0, double(r.bx1) + 2.0};
        const double cy[2] = {double(r.by0) - 1.0, double(r.by1) + 2.0};
        for (int k = 0; k < 3; k++)
            for (int a = 0; a < 2; a++)
                for (int b = 0; b < 2; b++) {
                    const double dx = cx[a] - hs[k][0], dy = cy[b] - hs[k][1];
                    L = fmax(L, sqrt(dx * dx + dy * dy));
                }
        for (int k = 0; k < 3 && safe; k++) {
            const int k1 = (k + 1) % 3, k2 = (k + 2) % 3;
            const double ux = hs[k1][0] - hs[k][0], uy = hs[k1][1] - hs[k][1];
            const double vx = hs[k2][0] - hs[k][0], vy = hs[k2][1] - hs[k][1];
            const double nu = sqrt(ux * ux + uy * uy), nv = sqrt(vx * vx + vy * vy);
            if (!(nu > 1e-3 && nv > 1e-3)) { safe = false; break; }
            const double cs = (ux * vx + uy * vy) / (nu * nv);
            // sin(theta/2) = sqrt((1 - cos theta) / 2)
            const double sh = sqrt(fmax(0.0, (1.0 - cs) * 0.5));
            if (!(sh > double(kSafeSlope) * L)) safe = false;
        }
    }
    if (safe) {
        flags |= kFaceSafe;
        int hx0, hx1, hy0, hy1;
        hx0 = int(floor(hmnx - 0.5)) - kHardMargin;
        hx1 = int(ceil(hmxx - 0.5)) + kHardMargin;
        hy0 = int(floor(hmny - 0.5)) - kHardMargin;
        hy1 = int(ceil(hmxy - 0.5)) + kHardMargin;
        r.rx0 = imax_(r.bx0, hx0);
        r.rx1 = imin_(r.bx1, hx1);
        r.ry0 = imax_(r.by0, hy0);
        r.ry1 = imin_(r.by1, hy1);
    } else {
        r.rx0 = r.bx0; r.rx1 = r.bx1; r.ry0 = r.by0; r.ry1 = r.by1;
    }
    r.flags = flags;
    *out = r;
    return (flags & kFaceValid) != 0;
}

// SoftClip of one face (f_ops.cpp:1917-1978) from its three hard clip
// vertices; writes the three soft clip vertices.
__device__ __forceinline__ void soft_clip_face(const float4 c[3], float W,
                                               float H, float radius,
                                               float4 out[3]) {
    float s[3][2];
    bool valid = true;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        float z;
        if (c[k].w <= 1e-6f ||
            !project_clip(c[k].x, c[k].y, c[k].z, c[k].w, W, H, &s[k][0],
                          &s[k][1], &z)) {
            valid = false;
        }
    }
    float scale = 1.f, cx = 0.f, cy = 0.f;
    if (valid) {
        cx = (s[0][0] + s[1][0] + s[2][0]) / 3.f;
        cy = (s[0][1] + s[1][1] + s[2][1]) / 3.f;
        float d_min = 1e30f;
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const int k2 = (k + 1) % 3;
            const float ex = s[k2][0] - s[k][0];
            const float ey = s[k2][1] - s[k][1];
            const float len = sqrtf(ex * ex + ey * ey);
            if (len < 1e-6f) continue;
            d_min = std_min(d_min,
                            fabsf(ex * (cy - s[k][1]) - ey * (cx - s[k][0])) /
                                    len);
        }
        scale = d_min < 1e29f
                        ? std_min(1.f + radius / std_max(d_min, 1e-3f), 8.f)
                        : 1.f;
    }
#pragma unroll
    for (int k = 0; k < 3; k++) {
        out[k] = c[k];
        if (valid) {
            const float sx = cx + (s[k][0] - cx) * scale;
            const float sy = cy + (s[k][1] - cy) * scale;
            out[k].x = (sx / W * 2.f - 1.f) * c[k].w;
            out[k].y = (sy / H * 2.f - 1.f) * c[k].w;
        }
    }
}

// ---------------------------------------------------------------- binning

struct BinSet {
    int* count;     // [views * tiles]   zeroed by the scan after use
    int* offset;    // [views * tiles]   exclusive scan of count
    int* cursor;    // [views * tiles]   offset + entries written so far
    int* list;      // [views * cap]
    int* overflow;  // [views]           1 -> sweep falls back to all faces
    int cap;        // list entries per view
};

__device__ __forceinline__ void tile_range(int x0, int x1, int y0, int y1,
                                           int* tx0, int* tx1, int* ty0,
                                           int* ty1) {
    *tx0 = x0 / kTile;
    *tx1 = x1 / kTile;
    *ty0 = y0 / kTile;
    *ty1 = y1 / kTile;
}

// Exclusive scan of one view's tile counts (grid = views, block = 1024).
// Zeroes the counts for the next use and flags views whose lists exceed the
// capacity.
static __global__ void k_bin_scan(BinSet b, int n_tiles, uint32_t* status) {
    const int v = blockIdx.x;
    int* cnt = b.count + size_t(v) * n_tiles;
    int* off = b.offset + size_t(v) * n_tiles;
    int* cur = b.cursor + size_t(v) * n_tiles;
    const int per = (n_tiles + blockDim.x - 1) / blockDim.x;
    const int beg = threadIdx.x * per;
    const int end = imin_(beg + per, n_tiles);
    int local = 0;
    for (int i = beg; i < end; i++) local += cnt[i];
    // block exclusive scan of `local`
    __shared__ int warp_sums[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const int nw = blockDim.x >> 5;
        int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += n;
        }
        if (lane < nw) warp_sums[lane] = s;
    }
    __syncthreads();
    int run = incl - local + (wid > 0 ? warp_sums[wid - 1] : 0);
    for (int i = beg; i < end; i++) {
        const int c = cnt[i];
        off[i] = run;
        cur[i] = run;
        cnt[i] = 0;
        run += c;
    }
    if (threadIdx.x == blockDim.x - 1) {
        const int total = warp_sums[(blockDim.x >> 5) - 1];
        const int of = total > b.cap ? 1 : 0;
        b.overflow[v] = of;
        if (of) atomicOr(status, kStatusBinOverflow);
    }
}

// ------------------------------------------------------------ tile sweeps

// Cooperative load of `n` records into shared memory.
__device__ __forceinline__ void load_recs(FaceRec* sh, const FaceRec* recs,
                                          const int* list, int base, int n,
                                          bool identity) {
    const float4* src = reinterpret_cast<const float4*>(recs);
    float4* dst = reinterpret_cast<float4*>(sh);
    for (int i = threadIdx.x; i < n * kRecVec4; i += blockDim.x) {
        const int j = i / kRecVec4, w = i % kRecVec4;
        const int f = identity ? base + j : list[base + j];
        dst[i] = src[size_t(f) * kRecVec4 + w];
    }
}

constexpr int kRecChunk = 64;

struct SweepView {
    const FaceRec* recs;  // this view's records [n_faces]
    int n_faces;
    int W, H, tiles_x, n_tiles;
    float radius;
};

// Sweep 1: full evaluation inside each face's sweep-1 region.
// State out: PixState per pixel, active flag per tile.
static __device__ void sweep1_tile(const SweepView& sv, const BinSet& b, int v,
                            int tile, const float* prev_depth,
                            PixState* state, int* active) {
    __shared__ FaceRec sh[kRecChunk];
    const int tx = tile % sv.tiles_x, ty = tile / sv.tiles_x;
    const int x = tx * kTile + (threadIdx.x % kTile);
    const int y = ty * kTile + (threadIdx.x / kTile);
    const bool in = x < sv.W && y < sv.H;
    const float px = float(x) + 0.5f, py = float(y) + 0.5f;
    const size_t pix = size_t(y) * sv.W + x;
    const float prev = (in && prev_depth) ? prev_depth[pix] : 0.f;

    float best_depth = 1.f, best_dist = 0.f, best_hz = 0.f;
    int best_face = -1;

    const bool identity = b.overflow[v] != 0;
    const int tl = v * sv.n_tiles + tile;
    const int beg = identity ? 0 : b.offset[tl];
    const int end = identity ? sv.n_faces : b.cursor[tl];
    const int* list = b.list + size_t(v) * b.cap;
    for (int base = beg; base < end; base += kRecChunk) {
        const int n = imin_(kRecChunk, end - base);
        __syncthreads();
        load_recs(sh, sv.recs, list, base, n, identity);
        __syncthreads();
        if (!in) continue;
        for (int i = 0; i < n; i++) {
            const FaceRec& r = sh[i];
            if (!(r.flags & kFaceValid)) continue;
            if (x < r.rx0 || x > r.rx1 || y < r.ry0 || y > r.ry1) continue;
            if (!soft_covers(px, py, r)) continue;
            const TriDist td = signed_dist(px, py, r);
            const float hz = hard_depth(px, py, r);
            const float depth = shifted_depth(td.dist, hz, sv.radius);
            if (prev_depth && depth <= prev + 1e-4f) continue;
            const int f = identity ? base + i : list[base + i];
            if (beats(depth, f, best_depth, best_face)) {
                best_depth = depth;
                best_face = f;
                best_dist = td.dist;
                best_hz = hz;
            }
        }
    }
    if (in) {
        state[size_t(v) * sv.W * sv.H + pix] =
                PixState{best_depth, best_face, best_dist, best_hz};
    }
    const int act = __syncthreads_or(in && best_depth > 0.5f);
    if (threadIdx.x == 0) active[tl] = act;
}

// Sweep 2: soft-rim fragments of safe faces outside their sweep-1 region,
// for pixels still uncovered by a hard fragment. Returns the survivor.
static __device__ PixState sweep2_tile(const SweepView& sv, const BinSet& b, int v,
                                int tile, const float* prev_depth,
                                const PixState* state, const int* active,
                                int* out_x, int* out_y, bool* out_in) {
    __shared__ FaceRec sh[kRecChunk];
    const int tx = tile % sv.tiles_x, ty = tile / sv.tiles_x;
    const int x = tx * kTile + (threadIdx.x % kTile);
    const int y = ty * kTile + (threadIdx.x / kTile);
    const bool in = x < sv.W && y < sv.H;
    const float px = float(x) + 0.5f, py = float(y) + 0.5f;
    const size_t pix = size_t(y) * sv.W + x;
    *out_x = x;
    *out_y = y;
    *out_in = in;
    PixState s{1.f, -1, 0.f, 0.f};
    if (in) s = state[size_t(v) * sv.W * sv.H + pix];
    const int tl = v * sv.n_tiles + tile;
    if (!active[tl]) return s;
    const float prev = (in && prev_depth) ? prev_depth[pix] : 0.f;
    const bool identity = b.overflow[v] != 0;
    const int beg = identity ? 0 : b.offset[tl];
    const int end = identity ? sv.n_faces : b.cursor[tl];
    const int* list = b.list + size_t(v) * b.cap;
    const bool open = in && s.depth > 0.5f;
    for (int base = beg; base < end; base += kRecChunk) {
        const int n = imin_(kRecChunk, end - base);
        __syncthreads();
        load_recs(sh, sv.recs, list, base, n, identity);
        __syncthreads();
        if (!open) continue;
        for (int i = 0; i < n; i++) {
            const FaceRec& r = sh[i];
            const uint32_t need = kFaceValid | kFaceSafe;
            if ((r.flags & need) != need) continue;
            if (x < r.bx0 || x > r.bx1 || y < r.by0 || y > r.by1) continue;
            if (x >= r.rx0 && x <= r.rx1 && y >= r.ry0 && y <= r.ry1) continue;
            if (!soft_covers(px, py, r)) continue;
            const TriDist td = signed_dist(px, py, r);
            // dist < 0 here for safe faces; the hard-type branch is kept so
            // the expression is the reference's in every case.
            const float hz = td.dist >= 0.f ? hard_depth(px, py, r) : 0.f;
            const float depth = shifted_depth(td.dist, hz, sv.radius);
            if (prev_depth && depth <= prev + 1e-4f) continue;
            const int f = identity ? base + i : list[base + i];
            if (beats(depth, f, s.depth, s.face)) {
                s.depth = depth;
                s.face = f;
                s.dist = td.dist;
                s.hard_z = td.dist >= 0.f ? hz : hard_depth(px, py, r);
            }
        }
    }
    return s;
}

}  // namespace dressi
