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
// Work split per view:
//  sweep 1 (16x16-pixel tiles, one CTA each): the faces whose *sweep-1
//           region* -- the hard triangle's bbox grown by kHardMargin pixels,
//           or the whole soft bbox for faces flagged unsafe -- touches the
//           tile. Inside (hard) and boundary fragments are folded; fragments
//           provably more than 0.008 px outside (see classify) are rim
//           fragments with depth > 0.5 and are deferred.
//  rim phase (8x4-pixel blocks, one warp each): only blocks that still hold
//           a pixel whose best depth is > 0.5 (no hard fragment) see the
//           rim fragments of safe faces: the deferred ones and those outside
//           the sweep-1 region.
// A fragment outside the hard bbox + margin of a *safe* face is provably a
// rim fragment with dist <= -(kHardMargin + 1) (the region's integer bounds
// floor(min - 0.5) - margin .. ceil(max - 0.5) + margin leave every pixel
// centre outside it at least margin + 1 px from the bbox), hence depth >
// 0.5, so it can never beat a hard fragment: leaving it out for pixels whose
// depth is <= 0.5 cannot change any output. "Safe" bounds the sign-test
// rounding error: every angle of the hard triangle must satisfy
// sin(theta/2) > kSafeSlope * L, L the largest pixel distance the face's
// soft bbox reaches from a hard vertex (the rounding error of the edge
// function is <= ~5u*|e|*L, its exact value outside the margin is >=
// 2*sin(theta/2)*|e| * (kHardMargin + 1)/2 >= 2*sin(theta/2)*|e|);
// faces failing it, or with huge coordinates, are evaluated exhaustively in
// sweep 1.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "exact.cuh"

namespace dressi {

constexpr int kTile = 16;                // tile edge in pixels
constexpr int kTileThreads = kTile * kTile;
#ifndef DRESSI_HARD_MARGIN
#define DRESSI_HARD_MARGIN 1
#endif
constexpr int kHardMargin = DRESSI_HARD_MARGIN;  // sweep-1 bbox growth (px)
static_assert(kHardMargin >= 1, "the safety bound needs centres >= 2 px out");
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
    kFaceFast = 8u,      // the "far" classification is exact for this face
    kFaceSoftInside = 16u,  // an inside fragment is always soft-covered
};

constexpr float kMaxFastRadius = 1e3f;  // rim depth stays > 0.5 below it

// Per-(view, face) constants hoisted out of the per-pixel loop. Every value
// is computed with the reference's own expression, so hoisting is exact.
struct __align__(16) FaceRec {
    float s0x, s0y, s1x, s1y;  // soft triangle, screen px
    float s2x, s2y, s_inv_area, fid;
    float sz0, sz1, sz2, orient;  // soft vertex NDC depth; sign of hard area
    float h0x, h0y, h1x, h1y;     // hard triangle, screen px
    float h2x, h2y, h_inv_area, hz0;
    float hz1, hz2, ex0, ey0;     // hard edges e_k = h[k+1] - h[k]
    float ex1, ey1, ex2, ey2;
    float len2_0, len2_1, len2_2, near2;  // near2: tau^2 of classify()
    float lbx0, lbx1, lby0, lby1;  // hard bbox grown by rounding slack
    int bx0, bx1, by0, by1;  // soft bbox pixel range (inclusive)
    int rx0, rx1, ry0, ry1;  // sweep-1 region pixel range (inclusive)
    uint32_t flags, i0, i1, i2;  // flags + hard vertex indices
};
static_assert(sizeof(FaceRec) == 192, "FaceRec layout");
constexpr int kRecVec4 = sizeof(FaceRec) / 16;
// the 16-byte word holding (lbx0, lbx1, lby0, lby1)
constexpr int kRecLbVec4 = 8;
static_assert(offsetof(FaceRec, lbx0) == kRecLbVec4 * 16 &&
                      offsetof(FaceRec, lby1) == kRecLbVec4 * 16 + 12,
              "FaceRec bbox word");

// Survivor of a pixel: Eq.3 depth, soft face index (-1 = none) and whether
// its signed distance is >= 0 (a "hard" fragment). The distance and hard
// depth themselves are recomputed once, for the survivor only, from its
// record -- the same expressions, hence the same values.
struct Survivor {
    float depth;
    int face;
    bool hard;
};
// Packed form kept in HBM between the sweeps (8 B / pixel).
__device__ __forceinline__ int2 pack(const Survivor& s) {
    return make_int2(__float_as_int(s.depth),
                     s.face < 0 ? -1 : (s.face | (s.hard ? int(0x80000000u) : 0)));
}
__device__ __forceinline__ Survivor unpack(int2 p) {
    Survivor s;
    s.depth = __int_as_float(p.x);
    s.face = p.y == -1 ? -1 : (p.y & 0x7fffffff);
    s.hard = p.y != -1 && (p.y & int(0x80000000u)) != 0;
    return s;
}

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

// Fragment classes of the two-pass sweep.
enum FragClass : int {
    kInside = 0,    // SignedDistToTri's sign test says inside: dist >= 0
    kFar = 1,       // provably dist < 0 with depth > 0.5: a rim fragment
    kBoundary = 2,  // anything else: evaluate in full
};

// The inside test is SignedDistToTri's own sign test (same expressions).
// Otherwise the reference's distance is -sqrt(best_d2), which is -0 -- a
// hard-type fragment -- only when some closest point q_k = a_k + t e_k
// rounds exactly onto the pixel centre. That puts the centre within
// |q rounding| + |cr rounding| / |e_k| of edge k's line, a bound tau the
// record stores as near2 = tau^2 (kFaceFast faces only, see build_record).
// A centre farther than tau from all three lines therefore has d2 > 0 and
// |dist| > 1.2e-4 px, so with radius < kMaxFastRadius its Eq.3 depth
// 0.5 + 0.5 |dist| / radius rounds strictly above 0.5.
__device__ __forceinline__ int classify(float px, float py, const FaceRec& r) {
    const float cr0 = r.ex0 * (py - r.h0y) - r.ey0 * (px - r.h0x);
    const float cr1 = r.ex1 * (py - r.h1y) - r.ey1 * (px - r.h1x);
    const float cr2 = r.ex2 * (py - r.h2y) - r.ey2 * (px - r.h2x);
    const int n_pos = (cr0 >= 0.f) + (cr1 >= 0.f) + (cr2 >= 0.f);
    const int n_neg = (cr0 <= 0.f) + (cr1 <= 0.f) + (cr2 <= 0.f);
    if (n_pos == 3 || n_neg == 3) return kInside;
    if (!(r.flags & 8u /* kFaceFast */)) return kBoundary;
    const bool near = cr0 * cr0 <= r.near2 * r.len2_0 ||
                      cr1 * cr1 <= r.near2 * r.len2_1 ||
                      cr2 * cr2 <= r.near2 * r.len2_2;
    return near ? kBoundary : kFar;
}

// Lower bound of a rim fragment's depth from the distance to the face's
// (slack-grown) hard bbox; never above the reference's depth (monotone).
__device__ __forceinline__ float rim_depth_lb(float px, float py,
                                              const FaceRec& r, float radius) {
    const float dx = fmaxf(fmaxf(r.lbx0 - px, px - r.lbx1), 0.f);
    const float dy = fmaxf(fmaxf(r.lby0 - py, py - r.lby1), 0.f);
    const float d = sqrtf(dx * dx + dy * dy) * 0.999f;
    return 0.5f + 0.5f * std_min(d / radius, 1.f);
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
    r.orient = 0.f;
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
    r.near2 = 0.f;
    r.i0 = hidx[0]; r.i1 = hidx[1]; r.i2 = hidx[2];
    {
        // bbox of the segments a_k + t e_k the distance is measured to,
        // grown by their rounding slack
        float mnx = hs[0][0], mxx = hs[0][0], mny = hs[0][1], mxy = hs[0][1];
        float amax = 0.f;
        for (int k = 0; k < 3; k++) {
            const float ax = hs[k][0], ay = hs[k][1];
            const float bx = ax + exs[k], by = ay + eys[k];
            mnx = fminf(mnx, fminf(ax, bx)); mxx = fmaxf(mxx, fmaxf(ax, bx));
            mny = fminf(mny, fminf(ay, by)); mxy = fmaxf(mxy, fmaxf(ay, by));
            amax = fmaxf(amax, fmaxf(fabsf(ax), fabsf(ay)));
        }
        const float slack = 1e-3f + 4e-7f * amax;
        r.lbx0 = mnx - slack; r.lbx1 = mxx + slack;
        r.lby0 = mny - slack; r.lby1 = mxy + slack;
    }

    // Safety classification. Float arithmetic with explicit rounding
    // allowances (u = 2^-24); it only decides how much work is done, the
    // results never depend on it beyond the guarantees stated per flag.
    constexpr float kU = 5.9604645e-8f;
    bool safe = true;
    float hmnx = hs[0][0], hmxx = hs[0][0], hmny = hs[0][1], hmxy = hs[0][1];
    float cmax = 0.f, emax = 0.f;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const float x = hs[k][0], y = hs[k][1];
        if (!(fabsf(x) < kCoordLimit && fabsf(y) < kCoordLimit)) safe = false;
        hmnx = fminf(hmnx, x); hmxx = fmaxf(hmxx, x);
        hmny = fminf(hmny, y); hmxy = fmaxf(hmxy, y);
        cmax = fmaxf(cmax, fmaxf(fabsf(x), fabsf(y)));
        emax = fmaxf(emax, sqrtf(l2s[k]));
    }
    // L: largest distance from a hard vertex to a (grown) soft-bbox corner,
    // rounded up
    float L = 0.f;
    if (safe) {
        const float cx[2] = {float(r.bx0) - 1.f, float(r.bx1) + 2.f};
        const float cy[2] = {float(r.by0) - 1.f, float(r.by1) + 2.f};
#pragma unroll
        for (int k = 0; k < 3; k++)
#pragma unroll
            for (int a = 0; a < 2; a++)
#pragma unroll
                for (int b = 0; b < 2; b++) {
                    const float dx = cx[a] - hs[k][0], dy = cy[b] - hs[k][1];
                    L = fmaxf(L, sqrtf(dx * dx + dy * dy));
                }
        L *= 1.001f;
        // every angle: sin(theta/2) >= sin(theta)/2 = |u x v| / (2|u||v|),
        // with the cross product's rounding subtracted
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const int k1 = (k + 1) % 3, k2 = (k + 2) % 3;
            const float ux = hs[k1][0] - hs[k][0], uy = hs[k1][1] - hs[k][1];
            const float vx = hs[k2][0] - hs[k][0], vy = hs[k2][1] - hs[k][1];
            const float nu = sqrtf(ux * ux + uy * uy), nv = sqrtf(vx * vx + vy * vy);
            const float p1 = ux * vy, p2 = uy * vx;
            const float cross = fabsf(p1 - p2) - 8.f * kU * (fabsf(p1) + fabsf(p2));
            const float sh = cross / (2.f * nu * nv * 1.001f);
            if (!(nu > 1e-3f && nv > 1e-3f && sh > kSafeSlope * L)) safe = false;
        }
    }
    if (safe && (flags & kFaceHardBary)) {
        // "far" classification (classify()): coordinates < 4096 keep the
        // edge endpoints within 2.5e-4 px of the next vertex; the reach L
        // of the soft bbox bounds the edge-function rounding error by
        // 4u|e|L < 0.001|e|; the area keeps the three edge functions from
        // all taking the outside sign.
        if (cmax < 4096.f && L < 4000.f &&
            fabsf(h_area) >= fmaxf(1.f, 1e-4f * emax * L * 1.001f)) {
            flags |= kFaceFast;
            r.orient = h_area > 0.f ? 1.f : -1.f;
            // tau (classify): rounding of q = a + t e (<= 4u|coords|) plus
            // that of the edge function over the reach L (4u L), doubled,
            // plus 2.5e-4 px, which keeps |dist| >= 2^-23 * kMaxFastRadius
            // so the Eq.3 depth of a deferred fragment rounds above 0.5
            const float tau = 2.f * (4.f * kU * L + 4.f * kU * cmax) + 2.5e-4f;
            r.near2 = tau * tau;
            // Soft coverage of inside fragments: if every hard vertex has
            // soft barycentrics >= 0.01 (convexity extends that to the whole
            // hard triangle, and an inside-classified pixel is within 1e-3
            // px of it) and the vertex depths stay 1e-5 inside [0, 1], the
            // reference's soft test passes for every inside fragment. The
            // barycentrics here carry a rounding allowance of 1e-5 times
            // the magnitude of their terms.
            bool si = !(fabsf(s_area) < 1e-6f);
            const float ia = fabsf(1.f / s_area);
#pragma unroll
            for (int k = 0; k < 3; k++) {
                const float px = hs[k][0], py = hs[k][1];
                const float a0 = (ss[1][0] - px) * (ss[2][1] - py),
                            b0 = (ss[1][1] - py) * (ss[2][0] - px);
                const float a1 = (ss[2][0] - px) * (ss[0][1] - py),
                            b1 = (ss[2][1] - py) * (ss[0][0] - px);
                const float l0 = (a0 - b0) / s_area, l1 = (a1 - b1) / s_area;
                const float tol = 0.01f + 1e-5f * (1.f + (fabsf(a0) + fabsf(b0) +
                                                          fabsf(a1) + fabsf(b1)) * ia);
                si = si && l0 >= tol && l1 >= tol && 1.f - l0 - l1 >= tol;
                si = si && sz[k] > 1e-5f && sz[k] < 1.f - 1e-5f;
            }
            if (si) flags |= kFaceSoftInside;
        }
    }
    if (safe) {
        flags |= kFaceSafe;
        // |coords| < 2^20: floorf/ceilf of x - 0.5 are exact
        const int hx0 = int(floorf(hmnx - 0.5f)) - kHardMargin;
        const int hx1 = int(ceilf(hmxx - 0.5f)) + kHardMargin;
        const int hy0 = int(floorf(hmny - 0.5f)) - kHardMargin;
        const int hy1 = int(ceilf(hmxy - 0.5f)) + kHardMargin;
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

constexpr int kRecChunk = 64;
constexpr int kRimCell = 32;     // pixels per side of a rim-flag cell
constexpr int kRimChunk = 8;     // records per rim staging buffer (2/warp)


// Fixed-capacity bins filled in one pass: entry i of bin k lives at
// list[k * cap + i]; the bin's cursor counts every append. Appends past the
// capacity go to one shared spill list, tagged with their bin; the consumer
// of an overflowed bin reads its own entries and then scans the spill list
// for its tag. Only when the spill list itself overflows does the consumer
// fall back to scanning all faces (still exact). The consumer resets the
// cursor; the spill counter is reset by the kernel after the consumer.
struct FixedBins {
    int* cursor;  // [views * bins]
    int* list;    // [views * bins * cap]
    int cap;
    int* spill_n;     // [1] appends past the capacity (all bins)
    int2* spill;      // [spill_cap] (global bin, face)
    int spill_cap;
    // work list of the rim phase: the open 8x4 blocks (global tile * 8 +
    // block), appended by sweep 1, taken by the rim warps through `take`
    int* open_n;      // [1]
    int* open;        // [views * tiles * 8]
    int* take;        // [1]
    // the work list reordered by k_rim_order, whole blocks with the long
    // lists at the front and the others from the back, so the rim warps
    // take the long lists first and no long block starts last
    int* order;       // [views * tiles * 8]
    // split blocks: their segments (block, segment) for k_rim_seg and the
    // blocks themselves for k_rim_split_epi
    int* seg_block;   // [kRimSplit * views * tiles * 8]
    int* seg_index;   // [kRimSplit * views * tiles * 8]
    int* split;       // [views * tiles * 8]
    // open blocks whose bins stayed empty: no fragment left to fold, only
    // the epilogue of their sweep-1 survivors (k_rim_empty)
    int* empty;       // [views * tiles * 8]
    // [0] front and [1] back whole blocks placed, [2] segments, [3] split
    // blocks, [4] k_rim_seg's work cursor, [5] empty blocks (all reset by
    // k_rim_filter)
    int* order_n;
    // per pixel, the best fragment the segments of a heavy block found
    // (rim_key_of; ~0 = none), consumed and reset by rim_split_finish
    unsigned long long* best;  // [views * H * W]
};

// Sweep-1 bins: 64-bit entries, high word = a lower bound of the depth of
// every fragment of the face (float bits, >= 0), low word = face << 8 |
// 8-bit block mask. Sorting them front to back lets a pixel stop at the
// first face whose bound exceeds its survivor's depth.
struct FixedBins1 {
    int* cursor;                 // [views * tiles]
    unsigned long long* list;    // [views * tiles * cap]
    int cap;
    int* spill_n;                     // [1]
    unsigned long long* spill_key;    // [spill_cap]
    int* spill_bin;                   // [spill_cap] global bin of each key
    int spill_cap;
    int* parked_n;                    // [1] overflowed tiles left to finish
    int* parked;                      // [views * tiles] their global bins
};
constexpr int kSortMax = 256;    // keys gathered per round by k_sweep1_spill
#ifndef DRESSI_WARP_SORT
#define DRESSI_WARP_SORT 128
#endif
constexpr int kWarpSort = DRESSI_WARP_SORT;  // longest per-warp list sorted
#ifndef DRESSI_RIM_SORT
#define DRESSI_RIM_SORT 256
#endif
constexpr int kRimSort = DRESSI_RIM_SORT;  // longest rim-block list ordered
constexpr int kRimBuckets = 65;  // rim depth-bound buckets (rim_bucket_order)
// Bucket of a rim block bound lbb in [0.5, 1]: (lbb - 0.5) * 128 is exact
// (lbb - 0.5 by Sterbenz, the product a power of two), so its floor puts lbb
// at or above the bucket's edge 0.5 + b/128; lbb == 1 alone takes 64.
// (Clamped so that a NaN bound, which converts to 0, or any other stray
// value stays inside the count array.)
__device__ __forceinline__ int rim_bucket_of(float lbb) {
    return lbb >= 1.f ? 64 : imin_(imax_(int((lbb - 0.5f) * 128.f), 0), 63);
}
#ifndef DRESSI_WARP_RECS
#define DRESSI_WARP_RECS 16
#endif
constexpr int kWarpRecs = DRESSI_WARP_RECS;  // records staged per warp and round
// warp_sort_smem pads a list to a power of two of at least 64 keys inside
// the buffer these size
static_assert(kWarpSort >= 64 && (kWarpSort & (kWarpSort - 1)) == 0,
              "DRESSI_WARP_SORT must be a power of two >= 64");
static_assert(kRimSort >= 64 && (kRimSort & (kRimSort - 1)) == 0,
              "DRESSI_RIM_SORT must be a power of two >= 64");
static_assert(2 * kRimChunk * sizeof(FaceRec) >=
                      kRimSort * sizeof(unsigned long long),
              "rim_bucket_order's scratch is a warp's record buffer");
static_assert(kWarpRecs >= 1 && kWarpRecs <= 32,
              "DRESSI_WARP_RECS must lie in [1, 32]");
constexpr int kSpillBlocks = 296;  // grid of k_sweep1_spill (2 per SM)
static_assert(kSortMax >= kTileThreads, "spill gathers need blockDim keys");

// Thread -> pixel of a 16x16 tile: 8 warps of 8x4 pixels (2-D warp
// footprints keep more lanes inside a small triangle's bbox).
__device__ __forceinline__ void tile_xy(int tile, int tiles_x, int* x,
                                        int* y) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    *x = (tile % tiles_x) * kTile + (w & 1) * 8 + (l & 7);
    *y = (tile / tiles_x) * kTile + (w >> 1) * 4 + (l >> 3);
}

// 8-bit mask of the 8x4 blocks of tile (tx, ty) that a pixel rectangle
// touches (bit w = warp w of tile_xy).
__device__ __forceinline__ int block_mask(int tx, int ty, int x0, int x1,
                                          int y0, int y1) {
    int m = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const int bx0 = tx * kTile + (w & 1) * 8, by0 = ty * kTile + (w >> 1) * 4;
        if (x0 <= bx0 + 7 && x1 >= bx0 && y0 <= by0 + 3 && y1 >= by0) m |= 1 << w;
    }
    return m;
}

struct SweepArgs {
    const FaceRec* recs;  // this view's records [n_faces]
    int n_faces, W, H, tiles_x, n_tiles, v;
    float radius;
    const float* prev;    // this view's peeling depth [H][W] or null
    int rim_cells_x;
    const int* rim;       // this view's rim-possible flags per cell
    uint32_t* status;     // [0] sticky status word, [1] per-iteration
                          // overflow bits (1: sweep-1 bins, 2: rim bins)
};

__device__ __forceinline__ void fold(Survivor& s, float depth, int f,
                                     bool hard) {
    if (beats(depth, f, s.depth, s.face)) {
        s.depth = depth;
        s.face = f;
        s.hard = hard;
    }
}

// Full evaluation of a fragment the way RasterizeSoftCpu does it (the
// caller has checked soft coverage).
__device__ __forceinline__ void eval_full(Survivor& s, float px, float py,
                                          const FaceRec& r, int f,
                                          float radius, bool peel,
                                          float prev) {
    const TriDist td = signed_dist(px, py, r);
    const float hz = td.dist >= 0.f ? hard_depth(px, py, r) : 0.f;
    const float depth = shifted_depth(td.dist, hz, radius);
    if (peel && depth <= prev + 1e-4f) return;
    fold(s, depth, f, td.dist >= 0.f);
}

// Lower bound of the Eq.3 depth of every fragment of a face: inside (and
// distance-zero) fragments of a kFaceFast face lie within 1.2e-3 of the
// triangle in barycentric units (the area criterion of build_record), so
// their hard depth is >= zmin - 3.6e-3 (zmax - zmin) less rounding; rim
// fragments are >= 0.5. Faces without the guarantees get 0.
__device__ __forceinline__ float face_depth_lb(const FaceRec& r) {
    if (!(r.flags & kFaceFast)) return 0.f;
    const float zmin = fminf(fminf(r.hz0, r.hz1), r.hz2);
    const float zmax = fmaxf(fmaxf(r.hz0, r.hz1), r.hz2);
    const float zlb = zmin - 0.1f * (zmax - zmin) - 1e-6f;
    return 0.5f * fminf(fmaxf(zlb, 0.f), 1.f) * 0.99999f;
}

// Appends face f to the sweep-1 bins of the tiles its region touches; the
// entry carries the face's depth bound and the 8-bit block mask.
__device__ __forceinline__ void bin_sweep1(const FaceRec& r, int f,
                                           int tiles_x, FixedBins1 b1,
                                           size_t view_bin0) {
    if (r.rx0 > r.rx1 || r.ry0 > r.ry1) return;
    const unsigned long long hi =
            (unsigned long long)__float_as_uint(face_depth_lb(r)) << 32;
    for (int ty = r.ry0 / kTile; ty <= r.ry1 / kTile; ty++)
        for (int tx = r.rx0 / kTile; tx <= r.rx1 / kTile; tx++) {
            const size_t bin = view_bin0 + size_t(ty) * tiles_x + tx;
            const unsigned long long key =
                    hi | uint32_t((f << 8) |
                                  block_mask(tx, ty, r.rx0, r.rx1, r.ry0, r.ry1));
            const int slot = atomicAdd(&b1.cursor[bin], 1);
            if (slot < b1.cap) {
                b1.list[bin * b1.cap + slot] = key;
            } else {
                const int sp = atomicAdd(b1.spill_n, 1);
                if (sp < b1.spill_cap) {
                    b1.spill_key[sp] = key;
                    b1.spill_bin[sp] = int(bin);
                }
            }
        }
}

// Ascending bitonic sort of one key per lane across a full warp.
__device__ __forceinline__ unsigned long long warp_sort_asc(
        unsigned long long k) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, j);
            const bool up = (lane & size) == 0;
            const bool lower = (lane & j) == 0;
            const unsigned long long lo = k < o ? k : o;
            const unsigned long long hi = k < o ? o : k;
            k = (lower == up) ? lo : hi;
        }
    }
    return k;
}

// Ascending bitonic sort of one 32-bit key per lane across a full warp.
__device__ __forceinline__ uint32_t warp_sort_asc32(uint32_t k) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xffffffffu, k, j);
            const bool up = (lane & size) == 0;
            const bool lower = (lane & j) == 0;
            const uint32_t lo = k < o ? k : o;
            const uint32_t hi = k < o ? o : k;
            k = (lower == up) ? lo : hi;
        }
    }
    return k;
}

// Folds the spilled entries of an overflowed sweep-1 bin (gathered from the
// spill list blockDim at a time) into the pixel's survivor -- or, when the
// spill list itself overflowed (all_faces), every face. Faces already folded
// by sweep 1 fold again to the same survivor. Called by every thread of the
// block (it has barriers); used only by k_sweep1_spill.
__device__ __forceinline__ void sweep1_spilled(
        const SweepArgs& a, const FixedBins1& b1, int bin, int ns,
        bool all_faces, int x, int y, bool in, bool peel, float prev,
        bool fast_ok, FaceRec* sh, unsigned long long* keys, int* n_match,
        Survivor& s) {
    const int w = threadIdx.x >> 5;
    const float px = float(x) + 0.5f, py = float(y) + 0.5f;
    const int total = all_faces ? a.n_faces : ns;
    for (int sb = 0; sb < total; sb += blockDim.x) {
        __syncthreads();
        if (threadIdx.x == 0) *n_match = 0;
        __syncthreads();
        const int i = sb + threadIdx.x;
        if (all_faces) {
            if (i < total) keys[threadIdx.x] = (unsigned long long)((i << 8) | 0xff);
            if (threadIdx.x == 0) *n_match = imin_(int(blockDim.x), total - sb);
        } else if (i < ns && b1.spill_bin[i] == bin) {
            keys[atomicAdd(n_match, 1)] = b1.spill_key[i];
        }
        __syncthreads();
        const int m = *n_match;
        for (int c = 0; c < m; c += kRecChunk) {
            const int n = imin_(kRecChunk, m - c);
            __syncthreads();
            const float4* src = reinterpret_cast<const float4*>(a.recs);
            float4* dst = reinterpret_cast<float4*>(sh);
            for (int t = threadIdx.x; t < n * kRecVec4; t += blockDim.x) {
                const int j = t / kRecVec4, q = t % kRecVec4;
                const int f = int(uint32_t(keys[c + j])) >> 8;
                dst[t] = src[size_t(f) * kRecVec4 + q];
            }
            __syncthreads();
            if (!in) continue;
            for (int j = 0; j < n; j++) {
                const int ent = int(uint32_t(keys[c + j]));
                if (!((ent >> w) & 1)) continue;
                const FaceRec& r = sh[j];
                if (x < r.rx0 || x > r.rx1 || y < r.ry0 || y > r.ry1) continue;
                if (!(r.flags & kFaceValid)) continue;
                const int f = ent >> 8;
                int cl = classify(px, py, r);
                if (cl == kFar && !fast_ok) cl = kBoundary;
                if (cl == kInside) {
                    if (!(r.flags & kFaceSoftInside) && !soft_covers(px, py, r))
                        continue;
                    const float depth =
                            0.5f * std_min(std_max(hard_depth(px, py, r), 0.f), 1.f);
                    if (peel && depth <= prev + 1e-4f) continue;
                    fold(s, depth, f, true);
                } else if (cl == kBoundary) {
                    if (!soft_covers(px, py, r)) continue;
                    eval_full(s, px, py, r, f, a.radius, peel, prev);
                }
            }
        }
    }
}

// End of a sweep-1 tile: each warp (an 8x4-pixel block) reports whether it
// still holds an open pixel (depth > 0.5) inside some face's soft reach.
// Tiles without such blocks finish through the epilogue; the others store
// their survivors and the open-block mask for the rim phase.
template <class Epi>
__device__ __forceinline__ void sweep1_finish(const SweepArgs& a, size_t bin,
                                              int x, int y, bool in,
                                              const Survivor& s, int2* state,
                                              uint8_t* active,
                                              const FixedBins& b2, Epi& epi) {
    const int w = threadIdx.x >> 5;
    const int cell = (y / kRimCell) * a.rim_cells_x + (x / kRimCell);
    const bool open = __ballot_sync(0xffffffffu, in && s.depth > 0.5f &&
                                                         a.rim[cell] != 0) != 0u;
    if ((threadIdx.x & 31) == 0) active[bin * 8 + w] = open ? 1 : 0;
    if (open) {
        // open block: survivors stored, the block queued for the rim phase
        if (in) state[size_t(a.v) * a.W * a.H + size_t(y) * a.W + x] = pack(s);
        if ((threadIdx.x & 31) == 0)
            b2.open[atomicAdd(b2.open_n, 1)] = int(bin) * 8 + w;
    } else {
        epi(a, x, y, in, s);
    }
}

// Ascending bitonic sort of n <= kWarpSort keys in a warp's shared buffer
// (padded with ~0 to a power of two), by the warp alone.
__device__ __forceinline__ void warp_sort_smem(unsigned long long* k, int n) {
    const int lane = threadIdx.x & 31;
    int p = 64;
    while (p < n) p <<= 1;
    for (int i = n + lane; i < p; i += 32) k[i] = ~0ull;
    __syncwarp();
    for (int size = 2; size <= p; size <<= 1) {
        for (int j = size >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < p; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = k[i], b = k[ixj];
                    const bool up = (i & size) == 0;
                    if (up ? a > b : a < b) {
                        k[i] = b;
                        k[ixj] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// Stages the records of keys[0, n) (n <= kWarpRecs) into the warp's shared
// slots: lane l copies 16-byte word l % 12 of record l / 12, ... .
__device__ __forceinline__ void stage_records(const FaceRec* recs,
                                              const unsigned long long* keys,
                                              int n, FaceRec* dst_recs) {
    const int lane = threadIdx.x & 31;
    const float4* src = reinterpret_cast<const float4*>(recs);
    float4* dst = reinterpret_cast<float4*>(dst_recs);
    for (int i = lane; i < n * kRecVec4; i += 32) {
        const int j = i / kRecVec4, q = i - j * kRecVec4;
        const int f = int(uint32_t(keys[j])) >> 8;
        dst[i] = src[size_t(f) * kRecVec4 + q];
    }
    __syncwarp();
}

// Sweep 1 runs kSweepWarps warps per 16x16 tile, each over kSweepPx of the
// tile's 8x4 blocks, one pixel of each per lane, so the warp's list
// filtering, sorting and record staging serve 32 kSweepPx pixels.
#ifndef DRESSI_SWEEP_WARPS
#define DRESSI_SWEEP_WARPS 4
#endif
constexpr int kSweepWarps = DRESSI_SWEEP_WARPS;
constexpr int kSweepPx = 8 / kSweepWarps;
constexpr int kSweep1Threads = 32 * kSweepWarps;

// Pixel j of this lane in sweep-1 warp W: block w = kSweepPx W + j of the
// tile, numbered as tile_xy's warps (w & 1: x half, w >> 1: row of blocks).
__device__ __forceinline__ void sweep1_xy(int tile, int tiles_x, int wb,
                                          int lane, int* x, int* y) {
    *x = (tile % tiles_x) * kTile + (wb & 1) * 8 + (lane & 7);
    *y = (tile / tiles_x) * kTile + (wb >> 1) * 4 + (lane >> 3);
}

// Sweep 1 over the tile's bin, every warp on its own (no block barrier):
// the warp keeps the list entries whose block mask meets its four blocks,
// sorts them front to back (up to kWarpSort) and folds inside and boundary
// fragments into each lane's four survivors; far (rim) fragments are left
// to the rim phase. A block still holding an open pixel (depth > 0.5)
// inside some face's soft reach stores its survivors and is queued for the
// rim phase; the others finish here through the epilogue. A tile whose bin
// overflowed folds the entries it holds, stores its survivors and is parked
// for k_sweep1_spill (this kernel keeps no spill code: compiled in, it
// slowed the common path). The bin's cursor is reset by k_rim_bin.
template <class Epi>
static __device__ void sweep1_tile(const SweepArgs& a, FixedBins1 b1,
                                   const FixedBins& b2, int tile, int2* state,
                                   uint8_t* active, Epi& epi) {
    __shared__ FaceRec sh_all[kSweepWarps][kWarpRecs];
    __shared__ unsigned long long keys_all[kSweepWarps][kWarpSort];
    const int wq = threadIdx.x >> 5, lane = threadIdx.x & 31;
    FaceRec* sh = sh_all[wq];
    unsigned long long* keys = keys_all[wq];
    const bool peel = a.prev != nullptr;
    const bool fast_ok = a.radius < kMaxFastRadius;
    int xs[kSweepPx], ys[kSweepPx];
    bool ins[kSweepPx];
    float prevs[kSweepPx];
#pragma unroll
    for (int j = 0; j < kSweepPx; j++) {
        sweep1_xy(tile, a.tiles_x, kSweepPx * wq + j, lane, &xs[j], &ys[j]);
        ins[j] = xs[j] < a.W && ys[j] < a.H;
        prevs[j] = (ins[j] && peel) ? a.prev[size_t(ys[j]) * a.W + xs[j]] : 0.f;
    }
    const size_t bin = size_t(a.v) * a.n_tiles + tile;
    const unsigned long long* list = b1.list + bin * b1.cap;
    // the list's first 32 slots are read together with its count (slots
    // past the count hold stale entries and are masked below), so the two
    // loads overlap instead of the list waiting on the count
    const unsigned long long first = lane < b1.cap ? list[lane] : 0ull;
    const int nent = b1.cursor[bin];
    // overflow: the own list's entries are folded here, the tile is then
    // parked for k_sweep1_spill (spilled entries, or all faces)
    const bool over = nent > b1.cap;
    if (over && threadIdx.x == 0) {
        atomicOr(&a.status[0], kStatusBinOverflow);  // sticky report
        atomicOr(&a.status[1], 1u);  // this iteration: grow the sweep-1 bins
        b1.parked[atomicAdd(b1.parked_n, 1)] = int(bin);
    }
    const int end = over ? b1.cap : nent;
    const unsigned lt = (1u << lane) - 1u;
    const uint32_t wmask = ((1u << kSweepPx) - 1u) << (kSweepPx * wq);

    // this warp's entries, in list order (first kWarpSort of them)
    int cnt = 0;
    for (int base = 0; base < end; base += 32) {
        const unsigned long long k =
                base + lane < end ? (base == 0 ? first : list[base + lane])
                                  : 0ull;
        const bool mine = (uint32_t(k) & wmask) != 0u;
        const unsigned bal = __ballot_sync(0xffffffffu, mine);
        const int slot = cnt + __popc(bal & lt);
        if (mine && slot < kWarpSort) keys[slot] = k;
        cnt += __popc(bal);
    }
    __syncwarp();
    // front-to-back order when the warp's list fits the sort buffer
    const bool sorted = !over && cnt <= kWarpSort;
    if (sorted && cnt <= 32) {
        // sorted as 32-bit keys: the bound's bits with the low five cleared
        // (non-negative floats order as their bits, and the truncated value
        // is still a lower bound) over the entry's slot; the entries are
        // then rewritten in that order with the truncated bound
        const uint32_t k = warp_sort_asc32(
                lane < cnt ? ((uint32_t(keys[lane] >> 32) & ~31u) | uint32_t(lane))
                           : 0xffffffffu);
        const unsigned long long src = keys[k & 31u];  // lanes >= cnt: unused
        __syncwarp();
        if (lane < cnt) keys[lane] = (uint64_t(k & ~31u) << 32) | uint32_t(src);
        __syncwarp();
    } else if (sorted) {
        warp_sort_smem(keys, cnt);
    }

    Survivor s[kSweepPx];
    bool done[kSweepPx];
    auto all_done = [&]() {
        bool d = true;
#pragma unroll
        for (int j = 0; j < kSweepPx; j++) d = d && done[j];
        return d;
    };
#pragma unroll
    for (int j = 0; j < kSweepPx; j++) {
        s[j] = Survivor{1.f, -1, false};
        done[j] = !ins[j];  // sorted lists: every later face is behind
    }
    // unsorted lists (over kWarpSort entries, or an overflowed tile) are
    // walked in list order, re-gathered kWarpRecs at a time
    int lpos = 0;
    for (int base = 0; base < cnt; base += kWarpRecs) {
        if (__all_sync(0xffffffffu, all_done())) break;
        int n;
        const unsigned long long* kb;
        if (sorted) {
            n = imin_(kWarpRecs, cnt - base);
            kb = keys + base;
        } else {
            // next kWarpRecs of this warp's entries from the list
            n = 0;
            while (n < kWarpRecs && lpos < end) {
                const int i = lpos + lane;
                const unsigned long long k = i < end ? list[i] : 0ull;
                const bool mine = (uint32_t(k) & wmask) != 0u;
                const unsigned bal = __ballot_sync(0xffffffffu, mine);
                const int slot = n + __popc(bal & lt);
                const int take = imin_(__popc(bal), kWarpRecs - n);
                // entries past the room are revisited from their position
                if (mine && slot < kWarpRecs) keys[slot] = k;
                if (take < __popc(bal)) {
                    // lane of the first entry left over
                    unsigned rest = bal;
                    for (int t = 0; t < take; t++) rest &= rest - 1u;
                    lpos += __ffs(rest) - 1;
                } else {
                    lpos += 32;
                }
                n += take;
            }
            __syncwarp();
            kb = keys;
        }
        stage_records(a.recs, kb, n, sh);
        for (int i = 0; i < n; i++) {
            if (all_done()) continue;
            const unsigned long long key = kb[i];
            const int ent = int(uint32_t(key));
            const float bound = __uint_as_float(uint32_t(key >> 32));
            const FaceRec& r = sh[i];
            const int f = ent >> 8;
#pragma unroll
            for (int j = 0; j < kSweepPx; j++) {
                if (done[j]) continue;
                if (sorted && s[j].depth < bound) {
                    done[j] = true;  // this face and all later ones lose
                    continue;
                }
                if (!((ent >> (kSweepPx * wq + j)) & 1)) continue;
                const int x = xs[j], y = ys[j];
                if (x < r.rx0 || x > r.rx1 || y < r.ry0 || y > r.ry1) continue;
                if (!(r.flags & kFaceValid)) continue;
                const float px = float(x) + 0.5f, py = float(y) + 0.5f;
                int c = classify(px, py, r);
                if (c == kFar && !fast_ok) c = kBoundary;
                if (c == kInside) {
                    if (!(r.flags & kFaceSoftInside) && !soft_covers(px, py, r))
                        continue;
                    const float depth = 0.5f * std_min(
                            std_max(hard_depth(px, py, r), 0.f), 1.f);
                    if (peel && depth <= prevs[j] + 1e-4f) continue;
                    fold(s[j], depth, f, true);
                } else if (c == kBoundary) {
                    if (!soft_covers(px, py, r)) continue;
                    eval_full(s[j], px, py, r, f, a.radius, peel, prevs[j]);
                }
            }
        }
        __syncwarp();  // sh / keys reuse by the next round
        if (!sorted && lpos >= end) break;
    }
#pragma unroll
    for (int j = 0; j < kSweepPx; j++) {
        const int wb = kSweepPx * wq + j;
        const int x = xs[j], y = ys[j];
        const int cell = (y / kRimCell) * a.rim_cells_x + (x / kRimCell);
        // a parked tile reports every block open, so its survivors are stored
        const bool open =
                __ballot_sync(0xffffffffu, (ins[j] && s[j].depth > 0.5f &&
                                            a.rim[cell] != 0) ||
                                                   over) != 0u;
        if (lane == 0) active[bin * 8 + wb] = open ? 1 : 0;
        if (open) {
            // open block (or a parked tile): survivors stored; an open block
            // of an unparked tile is queued for the rim phase
            if (ins[j])
                state[size_t(a.v) * a.W * a.H + size_t(y) * a.W + x] = pack(s[j]);
            if (!over && lane == 0)
                b2.open[atomicAdd(b2.open_n, 1)] = int(bin) * 8 + wb;
        } else {
            epi(a, x, y, ins[j], s[j]);
        }
    }
}

// Conservative test whether the soft triangle can cover a pixel centre of
// 8x4 block (bx, by): false only if, for one barycentric coordinate, its
// maximum over the rectangle of the block's pixel centres is below
// -margin. The coordinates are affine in the pixel centre, so that maximum
// is the value at the rectangle's centre plus |gradient| times the half
// extents (3.5, 1.5); the margin (~80 float ulps of the largest magnitude
// the products reach over the block) bounds the rounding of this float
// evaluation and of soft_covers' own. TriBlockTest holds the per-face
// constants (the soft vertices, the gradients' half-extent terms), computed
// once per face by tri_block_test_of with the same expressions.
struct TriBlockTest {
    float s0x, s0y, s1x, s1y, s2x, s2y, inv, ia, e0, e1, e2;
};
__device__ __forceinline__ TriBlockTest tri_block_test_of(const FaceRec& r) {
    TriBlockTest t;
    t.s0x = r.s0x; t.s0y = r.s0y; t.s1x = r.s1x; t.s1y = r.s1y;
    t.s2x = r.s2x; t.s2y = r.s2y;
    t.inv = r.s_inv_area;
    t.ia = fabsf(r.s_inv_area);
    const float g0x = (r.s1y - r.s2y) * r.s_inv_area;
    const float g0y = (r.s2x - r.s1x) * r.s_inv_area;
    const float g1x = (r.s2y - r.s0y) * r.s_inv_area;
    const float g1y = (r.s0x - r.s2x) * r.s_inv_area;
    t.e0 = fabsf(g0x) * 3.5f + fabsf(g0y) * 1.5f;
    t.e1 = fabsf(g1x) * 3.5f + fabsf(g1y) * 1.5f;
    t.e2 = fabsf(g0x + g1x) * 3.5f + fabsf(g0y + g1y) * 1.5f;
    return t;
}
__device__ __forceinline__ bool tri_touches_block(const TriBlockTest& t,
                                                  int bx, int by) {
    const float cx = float(bx * 8) + 4.f, cy = float(by * 4) + 2.f;
    const float a0 = (t.s1x - cx) * (t.s2y - cy), b0 = (t.s1y - cy) * (t.s2x - cx);
    const float a1 = (t.s2x - cx) * (t.s0y - cy), b1 = (t.s2y - cy) * (t.s0x - cx);
    const float l0 = (a0 - b0) * t.inv;
    const float l1 = (a1 - b1) * t.inv;
    // an upper bound of the products' magnitudes at every pixel centre of
    // the block (each factor widened by the half extent)
    const float u0x = fabsf(t.s0x - cx) + 3.5f, u0y = fabsf(t.s0y - cy) + 1.5f;
    const float u1x = fabsf(t.s1x - cx) + 3.5f, u1y = fabsf(t.s1y - cy) + 1.5f;
    const float u2x = fabsf(t.s2x - cx) + 3.5f, u2y = fabsf(t.s2y - cy) + 1.5f;
    const float mag = (u1x * u2y + u1y * u2x + u2x * u0y + u2y * u0x) * t.ia;
    const float margin = 1e-5f * (1.f + mag);
    return !(l0 + t.e0 < -margin || l1 + t.e1 < -margin ||
             (1.f - l0 - l1) + t.e2 < -margin);
}

// Summed-area table of the open blocks per 16x16 tile of one view (block
// = view): sat[(ty + 1) (tiles_x + 1) + tx + 1] = the open blocks of the
// tiles (0..tx, 0..ty); row 0 and column 0 are zero. Rows are prefix-summed
// by one warp each (warp scans over 32 tiles at a time), then columns.
// Also zeroes the view's count of faces kept for the rim binning.
static __global__ void k_open_sat(int n_tiles, int tiles_x, int tiles_y,
                                  const uint8_t* active, int* sat_all,
                                  int* kept_n) {
    const int v = blockIdx.x;
    if (threadIdx.x == 0) kept_n[v] = 0;
    const int w1 = tiles_x + 1;
    int* sat = sat_all + size_t(v) * w1 * (tiles_y + 1);
    const uint8_t* act = active + size_t(v) * n_tiles * 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_warps = blockDim.x >> 5;
    for (int x = threadIdx.x; x < w1; x += blockDim.x) sat[x] = 0;
    // rows: one warp per row, 32 tiles per step, a warp scan per step
    for (int ty = warp; ty < tiles_y; ty += n_warps) {
        int* row = sat + size_t(ty + 1) * w1;
        const uint2* a = reinterpret_cast<const uint2*>(act) +
                         size_t(ty) * tiles_x;
        if (lane == 0) row[0] = 0;
        int carry = 0;
        for (int t0 = 0; t0 < tiles_x; t0 += 32) {
            const int tx = t0 + lane;
            int c = 0;
            if (tx < tiles_x) {
                const uint2 b = a[tx];  // the tile's 8 block flags (0 / 1)
                c = __popc(b.x) + __popc(b.y);
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, c, o);
                if (lane >= o) c += n;
            }
            if (tx < tiles_x) row[tx + 1] = carry + c;
            carry += __shfl_sync(0xffffffffu, c, 31);
        }
    }
    __syncthreads();
    // columns: one warp per column, 32 rows per step
    for (int x = warp; x < w1; x += n_warps) {
        int carry = 0;
        for (int r0 = 1; r0 <= tiles_y; r0 += 32) {
            const int ty = r0 + lane;
            int c = ty <= tiles_y ? sat[size_t(ty) * w1 + x] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, c, o);
                if (lane >= o) c += n;
            }
            if (ty <= tiles_y) sat[size_t(ty) * w1 + x] = carry + c;
            carry += __shfl_sync(0xffffffffu, c, 31);
        }
    }
}

// Rim-phase face filter: one thread per face asks the view's summed-area
// table whether any tile under the face's soft bbox holds an open block
// (most faces lie away from every open block); the kept faces of a view are
// appended to its list. Also resets what sweep 1 consumed (the sweep-1
// bins, the spill list and the parked tiles) and the rim order counters.
static __global__ void k_rim_filter(int n_faces, int n_tiles, int tiles_x,
                                    int tiles_y, const FaceRec* recs_all,
                                    const int* sat_all, int* kept_all,
                                    int* kept_n, FixedBins b2,
                                    FixedBins1 b1) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
        *b1.spill_n = 0;
        *b1.parked_n = 0;
        for (int i = 0; i < 6; i++) b2.order_n[i] = 0;
    }
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n_tiles;
         t += gridDim.x * blockDim.x)
        b1.cursor[size_t(blockIdx.y) * n_tiles + t] = 0;
    const int v = blockIdx.y;
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t need = kFaceValid | kFaceSafe;
    bool keep = false;
    if (f < n_faces) {
        const FaceRec& r = recs_all[size_t(v) * n_faces + f];
        if ((r.flags & need) == need && r.bx0 <= r.bx1 && r.by0 <= r.by1) {
            const int w1 = tiles_x + 1;
            const int* sat = sat_all + size_t(v) * w1 * (tiles_y + 1);
            const int tx0 = r.bx0 >> 4, tx1 = (r.bx1 >> 4) + 1;
            const int ty0 = r.by0 >> 4, ty1 = (r.by1 >> 4) + 1;
            const int open = sat[ty1 * w1 + tx1] - sat[ty0 * w1 + tx1] -
                             sat[ty1 * w1 + tx0] + sat[ty0 * w1 + tx0];
            keep = open > 0;
        }
    }
    // warp-aggregated append
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    const int lane = threadIdx.x & 31;
    int base = 0;
    if (lane == 0 && m) base = atomicAdd(&kept_n[v], __popc(m));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (keep)
        kept_all[size_t(v) * n_faces + base +
                 __popc(m & ((1u << lane) - 1u))] = f;
}

// Rim-phase binning: a kept face enters the bin of every open 8x4 block its
// soft triangle may touch. One warp per kept face, lanes striding over the
// blocks of its soft bbox (the face's test constants in registers).
static __global__ void k_rim_bin(int n_faces, int n_tiles, int tiles_x,
                                 const FaceRec* recs_all,
                                 const uint8_t* active, const int* kept_all,
                                 const int* kept_n, FixedBins b2) {
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int v = blockIdx.y;
    if (i >= kept_n[v]) return;
    const int f = kept_all[size_t(v) * n_faces + i];
    const FaceRec& r = recs_all[size_t(v) * n_faces + f];
    const TriBlockTest tb = tri_block_test_of(r);
    const int bx0 = r.bx0 >> 3, bx1 = r.bx1 >> 3;
    const int by0 = r.by0 >> 2, by1 = r.by1 >> 2;
    const int blocks_x = tiles_x * 2;
    const uint8_t* act = active + size_t(v) * n_tiles * 8;
    const size_t bin0 = size_t(v) * n_tiles * 8;
    // lanes tile the block range 8 wide x 4 tall (no integer division)
    const int lx = lane & 7, ly = lane >> 3;
    for (int by = by0 + ly; by <= by1; by += 4) {
        for (int bx = bx0 + lx; bx <= bx1; bx += 8) {
            if (!act[((by >> 2) * tiles_x + (bx >> 1)) * 8 + (by & 3) * 2 +
                     (bx & 1)])
                continue;
            if (!tri_touches_block(tb, bx, by)) continue;
            const size_t bin = bin0 + size_t(by) * blocks_x + bx;
            const int slot = atomicAdd(&b2.cursor[bin], 1);
            if (slot < b2.cap) {
                b2.list[bin * b2.cap + slot] = f;
            } else {
                const int sp = atomicAdd(b2.spill_n, 1);
                if (sp < b2.spill_cap) b2.spill[sp] = make_int2(int(bin), f);
            }
        }
    }
}

// The rim work list with the longest lists first: blocks whose bins hold
// more than kRimSplitMin entries as kRimSplit segments when the open blocks
// are few, then those above kRimHeavy whole, then the others; within each
// class the order is arbitrary. Open blocks whose bins stayed empty go to
// the epilogue-only list.
constexpr int kRimHeavy = 96;
// lists longer than this are split into segments when the open blocks are
// few (below kRimSort, which bounds the ordered lists, so that at few views
// the long lists run on several warps)
constexpr int kRimSplitMin = 128;
constexpr int kRimSplit = 4;  // segments of a heavy block (strided entries)
// Splitting costs work (each segment prunes against its own survivor only)
// and pays only when the open blocks are too few to fill the machine and
// the longest list sets the phase's time (few views per GPU).
#ifndef DRESSI_RIM_SPLIT_MAX_OPEN
#define DRESSI_RIM_SPLIT_MAX_OPEN 16384
#endif
constexpr int kRimSplitMaxOpen = DRESSI_RIM_SPLIT_MAX_OPEN;
static __global__ void k_rim_order(FixedBins b2, int n_tiles, int tiles_x) {
    const int n = *b2.open_n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += gridDim.x * blockDim.x) {
        const int e = b2.open[i];
        const int tbin = e >> 3, w = e & 7;
        const int v = tbin / n_tiles, tile = tbin - v * n_tiles;
        // the block's rim bin, indexed as in rim_block
        const int bx = (tile % tiles_x) * 2 + (w & 1);
        const int by = (tile / tiles_x) * 4 + (w >> 1);
        const size_t bin = size_t(v) * n_tiles * 8 + size_t(by) * (tiles_x * 2) + bx;
        const int cnt = b2.cursor[bin];
        if (cnt == 0) {
            // nothing to fold (an empty bin spilled nothing either)
            b2.empty[atomicAdd(&b2.order_n[5], 1)] = e;
        } else if (n < kRimSplitMaxOpen && cnt > kRimSplitMin &&
                   cnt <= b2.cap) {
            // a list too long to sort (and not spilled): kRimSplit warps
            // fold a strided share each, k_rim_split_epi finishes the block
            const int slot = atomicAdd(&b2.order_n[2], kRimSplit);
            for (int sg = 0; sg < kRimSplit; sg++) {
                b2.seg_block[slot + sg] = e;
                b2.seg_index[slot + sg] = sg;
            }
            b2.split[atomicAdd(&b2.order_n[3], 1)] = e;
        } else if (cnt > kRimHeavy) {
            // long but sorted: one warp, early in the list
            b2.order[atomicAdd(&b2.order_n[0], 1)] = e;
        } else {
            b2.order[n - 1 - atomicAdd(&b2.order_n[1], 1)] = e;
        }
    }
}

// The 64-bit key of a survivor: ascending keys order as `beats` does
// (lower depth first; at equal depth the later face; no face last), with
// the hard bit alongside.
__device__ __forceinline__ unsigned long long rim_key_of(const Survivor& s) {
    const uint32_t lo = s.face < 0 ? 0xffffffffu
                                   : ((uint32_t(0x7fffffff - s.face) << 1) |
                                      (s.hard ? 1u : 0u));
    return (uint64_t(__float_as_uint(s.depth)) << 32) | lo;
}
__device__ __forceinline__ Survivor rim_survivor_of(unsigned long long k) {
    Survivor s;
    s.depth = __uint_as_float(uint32_t(k >> 32));
    const uint32_t lo = uint32_t(k);
    s.face = lo == 0xffffffffu ? -1 : 0x7fffffff - int(lo >> 1);
    s.hard = lo != 0xffffffffu && (lo & 1u);
    return s;
}

// Asynchronous 16-byte global -> shared copies (cp.async), committed and
// waited for per thread in groups.
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src) {
    const unsigned d =
            static_cast<unsigned>(__cvta_generic_to_shared(dst_smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(d),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kPending) : "memory");
}

// Starts the copy of the records ids[0, cn) into a warp's buffer (one
// commit group per lane).
__device__ __forceinline__ void rim_issue(const FaceRec* recs, const int* ids,
                                          int cn, FaceRec* buf) {
    const int lane = threadIdx.x & 31;
    const float4* src = reinterpret_cast<const float4*>(recs);
    float4* dst = reinterpret_cast<float4*>(buf);
    for (int i = lane; i < cn * kRecVec4; i += 32) {
        const int j = i / kRecVec4, q = i - j * kRecVec4;
        cp_async16(dst + i, src + size_t(ids[j]) * kRecVec4 + q);
    }
    cp_async_commit();
}

// Folds the staged records buf[0, cn) of faces ids[0, cn) into the pixel's
// survivor (kb: their sort keys, or null). The bounds are explained at
// rim_block.
__device__ __forceinline__ void rim_fold_chunk(
        const SweepArgs& a, int x, int y, float px, float py, bool peel,
        float prev, int cn, const FaceRec* buf, const int* ids,
        const unsigned long long* kb, Survivor& s, bool& done) {
    const float r2 = a.radius * a.radius;
    for (int j = 0; j < cn; j++) {
        if (done) break;
        if (kb && s.depth < __uint_as_float(uint32_t(kb[j] >> 32))) {
            done = true;  // this entry and all later ones lose
            break;
        }
        const int f = ids[j];
        const FaceRec& r = buf[j];
        const uint32_t need = kFaceValid | kFaceSafe;
        if ((r.flags & need) != need) continue;
        if (x < r.bx0 || x > r.bx1 || y < r.by0 || y > r.by1) continue;
        const float dx = fmaxf(fmaxf(r.lbx0 - px, px - r.lbx1), 0.f);
        const float dy = fmaxf(fmaxf(r.lby0 - py, py - r.lby1), 0.f);
        const float d2 = (dx * dx + dy * dy) * 0.998f;
        if (s.depth < 1.f) {
            const float t = 2.f * s.depth - 1.f + 2.3841858e-7f;
            if (d2 > t * t * r2) continue;  // bound above the survivor
        }
        const bool far = d2 >= r2;  // depth exactly 1
        if (far && f < s.face) continue;  // 1.0 tie, older face
        if (!soft_covers(px, py, r)) continue;
        if (far) {
            if (peel && 1.f <= prev + 1e-4f) continue;
            fold(s, 1.f, f, false);
        } else {
            eval_full(s, px, py, r, f, a.radius, peel, prev);
        }
    }
}

// Face ids of the list entries [base, base + cn) of a rim block into ids
// (lane < cn): from the sorted keys, the bin's list, or (identity) all
// faces from the last.
__device__ __forceinline__ void rim_load_ids(const SweepArgs& a,
                                             const unsigned long long* keys,
                                             const int* lst, bool sorted,
                                             bool identity, int base, int cn,
                                             int* ids) {
    const int lane = threadIdx.x & 31;
    if (lane < cn) {
        if (sorted) {
            const unsigned long long k = keys[base + lane];
            const uint32_t lo = uint32_t(k);
            ids[lane] = int(uint32_t(k >> 32) == __float_as_uint(1.f)
                                    ? 0xffffffffu - lo
                                    : lo);
        } else {
            ids[lane] = identity ? a.n_faces - 1 - (base + lane)
                                 : lst[base + lane];
        }
    }
    __syncwarp();
}

// Front-to-back order of a rim block's list without a comparison sort: the
// keys (block depth bound lbb | face word) are counted into kRimBuckets
// buckets of lbb -- 0.5 + b/128 <= lbb < 0.5 + (b+1)/128 for b < 64, and
// lbb == 1 in the last -- and scattered in bucket order through the scratch
// `tmp` (n <= kRimSort keys). Each key's high word becomes its bucket's
// lower edge, which is exact (a multiple of 2^-7 plus 0.5) and <= the
// key's own bound, so the edges are ascending along the list and a pixel
// whose survivor lies below an edge is done with every later entry, as
// with sorted bounds. The face words are kept (the last bucket's stay
// inverted). Order within a bucket is arbitrary: the fold is
// order-independent.
static __device__ __noinline__ void rim_bucket_order(unsigned long long* keys,
                                                 int n,
                                                 unsigned long long* tmp,
                                                 int* cnt) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < kRimBuckets; i += 32) cnt[i] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
        const unsigned long long k = keys[i];
        tmp[i] = k;
        const float lbb = __uint_as_float(uint32_t(k >> 32));
        atomicAdd(&cnt[rim_bucket_of(lbb)], 1);
    }
    __syncwarp();
    // exclusive scan of the counts (kRimBuckets = 65: lanes hold 0..31,
    // 32..63, and lane 0 the last)
    const int c0 = cnt[lane], c1 = cnt[lane + 32];
    int s0 = c0, s1 = c1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u0 = __shfl_up_sync(0xffffffffu, s0, o);
        const int u1 = __shfl_up_sync(0xffffffffu, s1, o);
        if (lane >= o) {
            s0 += u0;
            s1 += u1;
        }
    }
    const int t0 = __shfl_sync(0xffffffffu, s0, 31);
    const int t1 = __shfl_sync(0xffffffffu, s1, 31);
    __syncwarp();
    cnt[lane] = s0 - c0;
    cnt[lane + 32] = t0 + s1 - c1;
    if (lane == 0) cnt[64] = t0 + t1;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
        const unsigned long long k = tmp[i];
        const float lbb = __uint_as_float(uint32_t(k >> 32));
        const int b = rim_bucket_of(lbb);
        const float edge = b == 64 ? 1.f : 0.5f + float(b) * 0.0078125f;
        keys[atomicAdd(&cnt[b], 1)] =
                (uint64_t(__float_as_uint(edge)) << 32) | uint32_t(k);
    }
    __syncwarp();
}

// Rim phase for the open pixels of an open 8x4 block: folds every fragment
// of the faces in the block's bin (records staged per warp in shared
// memory, the next chunk's copy in flight while one is folded), pruned by
// the bbox depth bound. Fragments at |dist| >= radius all have depth
// exactly 1, where the latest covering face wins: once a pixel holds such
// a survivor, older faces at depth 1 are skipped without a coverage test.
//
// The per-fragment bound is rim_depth_lb's, tested on squared distances:
// with q = 0.999 d / R, lb = 0.5 + 0.5 min(q, 1) > depth  <=>  q > t =
// 2 depth - 1 (t < 1), i.e. d^2 0.999^2 > t^2 R^2, and lb = 1 <=> d^2
// 0.999^2 >= R^2. Using 0.998 < 0.999^2 keeps both bounds below the true
// depth with the same ~1e-3 slack against rounding (~1e-7). A skipped
// fragment must also round to a depth strictly above the survivor's (an
// equal depth is a tie that the later face wins): t is raised by 2^-22,
// two units in the last place of depths in [0.5, 1), so the skip holds
// for survivors at any distance, not only where the relative slack
// exceeds an ulp.
template <class Epi>
static __device__ __forceinline__ void rim_block(const SweepArgs& a, FixedBins b2, int tile,
                                 int w, const int2* state, FaceRec* recs_w,
                                 int* ids_w, unsigned long long* keys_w,
                                 int* cnt_w, Epi& epi) {
    const int lane = threadIdx.x & 31;
    const int x = (tile % a.tiles_x) * kTile + (w & 1) * 8 + (lane & 7);
    const int y = (tile / a.tiles_x) * kTile + (w >> 1) * 4 + (lane >> 3);
    const bool in = x < a.W && y < a.H;
    const float px = float(x) + 0.5f, py = float(y) + 0.5f;
    const size_t pix = size_t(y) * a.W + x;
    const bool peel = a.prev != nullptr;
    const float prev = (in && peel) ? a.prev[pix] : 0.f;
    Survivor s{1.f, -1, false};
    if (in) s = unpack(state[size_t(a.v) * a.W * a.H + pix]);
    const bool open = in && s.depth > 0.5f;
    const int bx = (tile % a.tiles_x) * 2 + (w & 1);
    const int by = (tile / a.tiles_x) * 4 + (w >> 1);
    const size_t bin = size_t(a.v) * a.n_tiles * 8 +
                       size_t(by) * (a.tiles_x * 2) + bx;
    // the list's first 32 slots are read together with its count (slots
    // past the count are never used)
    const int* lst = b2.list + bin * b2.cap;
    const int first = lane < b2.cap ? lst[lane] : 0;
    int n = 0, ns = 0;
    if (lane == 0) {
        n = b2.cursor[bin];
        b2.cursor[bin] = 0;  // ready for the next use
        if (n > b2.cap) ns = *b2.spill_n;
    }
    n = __shfl_sync(0xffffffffu, n, 0);
    ns = __shfl_sync(0xffffffffu, ns, 0);
    const bool over = n > b2.cap;  // the rest of the list is spilled
    const bool identity = over && ns > b2.spill_cap;  // spill lost
    if (over && lane == 0) {
        atomicOr(&a.status[0], kStatusBinOverflow);  // sticky report
        atomicOr(&a.status[1], 2u);  // this iteration: grow the rim bins
    }
    const int end = identity ? a.n_faces : (over ? b2.cap : n);
    const float4* src = reinterpret_cast<const float4*>(a.recs);
    // Front-to-back order when the list fits the key buffer: per entry the
    // depth bound of the whole block (rim_depth_lb at the distance from the
    // block's pixel-centre rectangle to the face's bbox; rounding is
    // monotonic, so it is <= every pixel's own bound), ascending; entries
    // whose bound is 1 (|dist| >= radius: depth exactly 1, latest face
    // wins) by descending face. A pixel is done at the first entry whose
    // bound is above its survivor's depth.
    const bool sorted = !over && end > 0 && end <= kRimSort;
    if (sorted) {
        const float xlo = float(bx * 8) + 0.5f, xhi = float(bx * 8) + 7.5f;
        const float ylo = float(by * 4) + 0.5f, yhi = float(by * 4) + 3.5f;
        for (int i = lane; i < end; i += 32) {
            const int f = i < 32 ? first : lst[i];
            const float4 lbq = src[size_t(f) * kRecVec4 + kRecLbVec4];
            const float dx = fmaxf(fmaxf(lbq.x - xhi, xlo - lbq.y), 0.f);
            const float dy = fmaxf(fmaxf(lbq.z - yhi, ylo - lbq.w), 0.f);
            const float d = sqrtf(dx * dx + dy * dy) * 0.999f;
            const float lbb = 0.5f + 0.5f * std_min(d / a.radius, 1.f);
            const uint32_t lo = lbb == 1.f ? 0xffffffffu - uint32_t(f)
                                           : uint32_t(f);
            keys_w[i] = (uint64_t(__float_as_uint(lbb)) << 32) | lo;
        }
        __syncwarp();
        if (end <= 32) {
            unsigned long long k = lane < end ? keys_w[lane] : ~0ull;
            k = warp_sort_asc(k);
            __syncwarp();
            keys_w[lane] = k;
            __syncwarp();
        } else {
            rim_bucket_order(keys_w, end, reinterpret_cast<unsigned long long*>(recs_w),
                             cnt_w);
        }
    }
    bool done = !open;
    // double-buffered pass over the list: chunk c folds from buffer c & 1
    // while chunk c + 1 is copied into the other
    if (end > 0 && !__all_sync(0xffffffffu, done)) {
        int cn = imin_(kRimChunk, end);
        rim_load_ids(a, keys_w, lst, sorted, identity, 0, cn, ids_w);
        rim_issue(a.recs, ids_w, cn, recs_w);
        for (int base = 0, c = 0; base < end; base += kRimChunk, c ^= 1) {
            const int nbase = base + kRimChunk;
            const bool more = nbase < end && !__all_sync(0xffffffffu, done);
            const int ncn = more ? imin_(kRimChunk, end - nbase) : 0;
            if (more) {
                int* nids = ids_w + (c ^ 1) * kRimChunk;
                rim_load_ids(a, keys_w, lst, sorted, identity, nbase, ncn,
                             nids);
                rim_issue(a.recs, nids, ncn, recs_w + (c ^ 1) * kRimChunk);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncwarp();
            if (open)
                rim_fold_chunk(a, x, y, px, py, peel, prev, cn,
                               recs_w + c * kRimChunk, ids_w + c * kRimChunk,
                               sorted ? keys_w + base : nullptr, s, done);
            __syncwarp();  // buffer c is refilled two chunks on
            if (!more) break;
            cn = ncn;
        }
    }
    if (over && !identity) {
        // this block's spilled entries, kRimChunk scanned per step
        for (int sb = 0; sb < ns; sb += kRimChunk) {
            const int i = sb + lane;
            int2 e = make_int2(-1, 0);
            if (lane < kRimChunk && i < ns) e = b2.spill[i];
            const bool match = e.x == int(bin);
            const unsigned mm = __ballot_sync(0xffffffffu, match);
            if (mm == 0u) continue;
            __syncwarp();
            if (match) ids_w[__popc(mm & ((1u << lane) - 1u))] = e.y;
            __syncwarp();
            rim_issue(a.recs, ids_w, __popc(mm), recs_w);
            cp_async_wait<0>();
            __syncwarp();
            if (open)
                rim_fold_chunk(a, x, y, px, py, peel, prev, __popc(mm),
                               recs_w, ids_w, nullptr, s, done);
            __syncwarp();
        }
    }
    epi(a, x, y, in, s);
    __syncwarp();  // buffers reused by the warp's next block
}

// One segment of a heavy rim block: the list entries seg, seg + kRimSplit,
// ... folded into the sweep-1 survivors of the block's open pixels and
// merged into b2.best (atomic minimum of rim_key_of). The argmin is
// order-free, so the segments' merge equals one warp's whole pass.
static __device__ __forceinline__ void rim_segment(const SweepArgs& a,
                                                   FixedBins b2, int tile,
                                                   int w, int seg,
                                                   const int2* state,
                                                   FaceRec* recs_w,
                                                   int* ids_w) {
    const int lane = threadIdx.x & 31;
    const int x = (tile % a.tiles_x) * kTile + (w & 1) * 8 + (lane & 7);
    const int y = (tile / a.tiles_x) * kTile + (w >> 1) * 4 + (lane >> 3);
    const bool in = x < a.W && y < a.H;
    const float px = float(x) + 0.5f, py = float(y) + 0.5f;
    const size_t pix = size_t(y) * a.W + x;
    const bool peel = a.prev != nullptr;
    const float prev = (in && peel) ? a.prev[pix] : 0.f;
    Survivor s{1.f, -1, false};
    if (in) s = unpack(state[size_t(a.v) * a.W * a.H + pix]);
    const bool open = in && s.depth > 0.5f;
    const int bx = (tile % a.tiles_x) * 2 + (w & 1);
    const int by = (tile / a.tiles_x) * 4 + (w >> 1);
    const size_t bin = size_t(a.v) * a.n_tiles * 8 +
                       size_t(by) * (a.tiles_x * 2) + bx;
    const int n = b2.cursor[bin];  // <= cap (heavy blocks are not spilled)
    const int* lst = b2.list + bin * b2.cap;
    const int ns = n > seg ? (n - seg + kRimSplit - 1) / kRimSplit : 0;
    bool done = !open;
    for (int base = 0; base < ns; base += kRimChunk) {
        if (__all_sync(0xffffffffu, done)) break;
        const int cn = imin_(kRimChunk, ns - base);
        if (lane < cn) ids_w[lane] = lst[seg + (base + lane) * kRimSplit];
        __syncwarp();
        rim_issue(a.recs, ids_w, cn, recs_w);
        cp_async_wait<0>();
        __syncwarp();
        if (open)
            rim_fold_chunk(a, x, y, px, py, peel, prev, cn, recs_w, ids_w,
                           nullptr, s, done);
        __syncwarp();
    }
    if (open) atomicMin(&b2.best[size_t(a.v) * a.W * a.H + pix], rim_key_of(s));
}

// Finishes a split rim block (its segments ran in k_rim_seg): per pixel the
// best of the sweep-1 survivor and the segments' fragments, then the
// epilogue; resets b2.best and the block's bin cursor for the next use.
template <class Epi>
__device__ __forceinline__ void rim_split_finish(const SweepArgs& a, FixedBins b2,
                                                 int tile, int w,
                                                 const int2* state,
                                                 const Epi& epi) {
    const int lane = threadIdx.x & 31;
    const int x = (tile % a.tiles_x) * kTile + (w & 1) * 8 + (lane & 7);
    const int y = (tile / a.tiles_x) * kTile + (w >> 1) * 4 + (lane >> 3);
    const bool in = x < a.W && y < a.H;
    Survivor s{1.f, -1, false};
    if (in) {
        const size_t pi = size_t(a.v) * a.W * a.H + size_t(y) * a.W + x;
        s = unpack(state[pi]);
        const unsigned long long k = b2.best[pi];
        if (k != ~0ull) {
            if (k < rim_key_of(s)) s = rim_survivor_of(k);
            b2.best[pi] = ~0ull;
        }
    }
    if (lane == 0) {
        const int bx = (tile % a.tiles_x) * 2 + (w & 1);
        const int by = (tile / a.tiles_x) * 4 + (w >> 1);
        b2.cursor[size_t(a.v) * a.n_tiles * 8 + size_t(by) * (a.tiles_x * 2) +
                  bx] = 0;
    }
    epi(a, x, y, in, s);
}

// Epilogue of the op-level RasterizeSoft: the reference's output channels
// (dist, face_id, hard_z, coverage) recomputed for the survivor.
struct EpiRS {
    float4* out;  // [views][H][W]
    __device__ void operator()(const SweepArgs& a, int x, int y, bool in,
                               const Survivor& s) const {
        if (!in) return;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s.face >= 0) {
            const FaceRec& r = a.recs[s.face];
            const float px = float(x) + 0.5f, py = float(y) + 0.5f;
            o.x = signed_dist(px, py, r).dist;
            o.y = r.fid;
            o.z = hard_depth(px, py, r);
            o.w = 1.f;
        }
        out[size_t(a.v) * a.W * a.H + size_t(y) * a.W + x] = o;
    }
};

// Nine CTAs per SM (56 registers): issue-bound, so residency pays over the
// few spilled bytes (7 CTAs at the unbounded 72 registers; 8, 10 and 12 per
// SM timed slower).
template <class Epi>
#ifndef DRESSI_SWEEP1_CTAS
#define DRESSI_SWEEP1_CTAS 9
#endif
__global__ void __launch_bounds__(kSweep1Threads, DRESSI_SWEEP1_CTAS)
        k_sweep1(SweepArgs a0, FixedBins1 b1, FixedBins b2, int2* state,
                 uint8_t* active, size_t view_stride_recs,
                 size_t view_stride_px, size_t view_stride_rim, Epi epi) {
    SweepArgs a = a0;
    a.v = blockIdx.y;
    a.recs = a0.recs + a.v * view_stride_recs;
    a.rim = a0.rim + a.v * view_stride_rim;
    if (a0.prev) a.prev = a0.prev + a.v * view_stride_px;
    sweep1_tile(a, b1, b2, blockIdx.x, state, active, epi);
}

// Finishes the sweep-1 tiles whose bins overflowed into the spill list:
// their survivors over the own-list entries were stored by sweep 1; the
// spilled entries are folded here, then the tile ends as in sweep 1. A grid
// of any size strides over the parked tiles (none: every block exits).
template <class Epi>
__global__ void __launch_bounds__(kTileThreads)
        k_sweep1_spill(SweepArgs a0, FixedBins1 b1, FixedBins b2, int2* state,
                       uint8_t* active, size_t view_stride_recs,
                       size_t view_stride_px, size_t view_stride_rim,
                       Epi epi) {
    __shared__ FaceRec sh[kRecChunk];
    __shared__ unsigned long long keys[kSortMax];
    __shared__ int n_match;
    const int n_parked = *b1.parked_n;
    const int ns_all = *b1.spill_n;
    const bool all_faces = ns_all > b1.spill_cap;  // spill entries were lost
    const int ns = imin_(ns_all, b1.spill_cap);
    for (int k = blockIdx.x; k < n_parked; k += gridDim.x) {
        const int bin = b1.parked[k];
        SweepArgs a = a0;
        a.v = bin / a0.n_tiles;
        const int tile = bin - a.v * a0.n_tiles;
        a.recs = a0.recs + a.v * view_stride_recs;
        a.rim = a0.rim + a.v * view_stride_rim;
        if (a0.prev) a.prev = a0.prev + a.v * view_stride_px;
        int x, y;
        tile_xy(tile, a.tiles_x, &x, &y);
        const bool in = x < a.W && y < a.H;
        const size_t pix = size_t(y) * a.W + x;
        const bool peel = a.prev != nullptr;
        const float prev = (in && peel) ? a.prev[pix] : 0.f;
        Survivor s{1.f, -1, false};
        if (in) s = unpack(state[size_t(a.v) * a.W * a.H + pix]);
        sweep1_spilled(a, b1, bin, ns, all_faces, x, y, in, peel, prev,
                       a.radius < kMaxFastRadius, sh, keys, &n_match, s);
        sweep1_finish(a, size_t(bin), x, y, in, s, state, active, b2, epi);
        __syncthreads();  // sh reuse by the next parked tile
    }
}

// The segments of the split rim blocks (few open blocks, lists too long to
// sort), by persistent warps; k_rim_split_epi finishes those blocks.
static __global__ void __launch_bounds__(kTileThreads)
        k_rim_seg(SweepArgs a0, FixedBins b2, const int2* state,
                  size_t view_stride_recs, size_t view_stride_px,
                  size_t view_stride_rim) {
    __shared__ FaceRec recs_sh[8][kRimChunk];
    __shared__ int ids_sh[8][kRimChunk];
    const int wc = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_seg = b2.order_n[2];
    for (;;) {
        int item = 0;
        if (lane == 0) item = atomicAdd(&b2.order_n[4], 1);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item >= n_seg) break;
        const int e = b2.seg_block[item];
        const int tbin = e >> 3, w = e & 7;
        SweepArgs a = a0;
        a.v = tbin / a0.n_tiles;
        const int tile = tbin - a.v * a0.n_tiles;
        a.recs = a0.recs + a.v * view_stride_recs;
        a.rim = a0.rim + a.v * view_stride_rim;
        if (a0.prev) a.prev = a0.prev + a.v * view_stride_px;
        rim_segment(a, b2, tile, w, b2.seg_index[item], state, recs_sh[wc],
                    ids_sh[wc]);
    }
}

// The rim phase: persistent warps take the open 8x4 blocks queued by sweep
// 1 from the work list (an atomic cursor balances blocks of very different
// cost), so every resident warp has work.
template <class Epi>
__global__ void __launch_bounds__(kTileThreads)
        k_rim(SweepArgs a0, FixedBins b2, const int2* state,
              size_t view_stride_recs, size_t view_stride_px,
              size_t view_stride_rim, Epi epi) {
    __shared__ FaceRec recs_sh[8][2 * kRimChunk];
    __shared__ int ids_sh[8][2 * kRimChunk];
    __shared__ unsigned long long keys_sh[8][kRimSort];
    __shared__ int cnt_sh[8][kRimBuckets];
    const int wc = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_open = *b2.open_n;
    const int n_front = b2.order_n[0], n_back = b2.order_n[1];
    for (;;) {
        int item = 0;
        if (lane == 0) item = atomicAdd(b2.take, 1);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item >= n_front + n_back) break;
        // the long lists first (the split blocks are not in this list)
        const int e = b2.order[item < n_front ? item
                                              : n_open - 1 - (item - n_front)];
        const int tbin = e >> 3, w = e & 7;
        SweepArgs a = a0;
        a.v = tbin / a0.n_tiles;
        const int tile = tbin - a.v * a0.n_tiles;
        a.recs = a0.recs + a.v * view_stride_recs;
        a.rim = a0.rim + a.v * view_stride_rim;
        if (a0.prev) a.prev = a0.prev + a.v * view_stride_px;
        rim_block(a, b2, tile, w, state, recs_sh[wc], ids_sh[wc], keys_sh[wc],
                  cnt_sh[wc], epi);
    }
}

// The split blocks' epilogues (rim_split_finish), one warp per block, after
// k_rim_seg.
template <class Epi>
__global__ void __launch_bounds__(256)
        k_rim_split_epi(SweepArgs a0, FixedBins b2, const int2* state,
                        size_t view_stride_recs, size_t view_stride_px,
                        size_t view_stride_rim, Epi epi) {
    const int n_split = b2.order_n[3];
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < n_split;
         t += (gridDim.x * blockDim.x) >> 5) {
        const int e = b2.split[t];
        const int tbin = e >> 3, w = e & 7;
        SweepArgs a = a0;
        a.v = tbin / a0.n_tiles;
        const int tile = tbin - a.v * a0.n_tiles;
        a.recs = a0.recs + a.v * view_stride_recs;
        a.rim = a0.rim + a.v * view_stride_rim;
        if (a0.prev) a.prev = a0.prev + a.v * view_stride_px;
        rim_split_finish(a, b2, tile, w, state, epi);
    }
}
// The open blocks whose rim bins stayed empty (most of them: the rim-flag
// cells are coarse): the rim phase would fold nothing into their sweep-1
// survivors, so one warp per block only runs the epilogue, as rim_block
// does for an empty list.
template <class Epi>
__global__ void __launch_bounds__(256)
        k_rim_empty(SweepArgs a0, FixedBins b2, const int2* state,
                    size_t view_stride_recs, size_t view_stride_px,
                    size_t view_stride_rim, Epi epi) {
    const int n_empty = b2.order_n[5];
    const int lane = threadIdx.x & 31;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < n_empty;
         t += (gridDim.x * blockDim.x) >> 5) {
        const int e = b2.empty[t];
        const int tbin = e >> 3, w = e & 7;
        SweepArgs a = a0;
        a.v = tbin / a0.n_tiles;
        const int tile = tbin - a.v * a0.n_tiles;
        a.recs = a0.recs + a.v * view_stride_recs;
        a.rim = a0.rim + a.v * view_stride_rim;
        if (a0.prev) a.prev = a0.prev + a.v * view_stride_px;
        const int x = (tile % a.tiles_x) * kTile + (w & 1) * 8 + (lane & 7);
        const int y = (tile / a.tiles_x) * kTile + (w >> 1) * 4 + (lane >> 3);
        const bool in = x < a.W && y < a.H;
        Survivor s{1.f, -1, false};
        if (in)
            s = unpack(state[size_t(a.v) * a.W * a.H + size_t(y) * a.W + x]);
        epi(a, x, y, in, s);
    }
}
constexpr int kRimCtas = 148 * 4;  // persistent grid of k_rim

// Marks the rim-flag cells a safe face's soft bbox reaches: a superset of
// where the rim phase can find fragments (those outside the sweep-1 region
// and the deferred far ones inside it).
__device__ __forceinline__ void mark_rim_cells(const FaceRec& r, int* rim,
                                               int cells_x) {
    const uint32_t need = kFaceValid | kFaceSafe;
    if ((r.flags & need) != need) return;
    for (int cy = r.by0 / kRimCell; cy <= r.by1 / kRimCell; cy++)
        for (int cx = r.bx0 / kRimCell; cx <= r.bx1 / kRimCell; cx++)
            rim[cy * cells_x + cx] = 1;
}

}  // namespace dressi
