/*
 * TEST INFRASTRUCTURE ONLY -- see oracle.h. A plain-C restatement of the
 * reference CPU algorithms; every float expression keeps the reference's
 * operation order (no FMA: built with -ffp-contract=off) so raster outputs
 * are bit-identical to the reference's CpuEvaluator.
 *
 * std::min / std::max are restated as the comparisons libstdc++ uses
 * ((b < a) ? b : a and (a < b) ? b : a), and float->int conversions as the
 * x86-64 cvttss2si result (INT_MIN / INT64_MIN for NaN or out-of-range), so
 * NaN and overflow behave as in the compiled reference.
 */
#define _POSIX_C_SOURCE 200809L
#include "oracle.h"

#include <limits.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[256];

static int fail(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return 1;
}

const char* orc_last_error(void) { return g_err; }

/* ---------------------------------------------------------------- helpers */

static inline float smin(float a, float b) { return (b < a) ? b : a; }
static inline float smax(float a, float b) { return (a < b) ? b : a; }

/* int(x) as x86-64 cvttss2si: truncation, INT_MIN when not representable */
static inline int to_i32(float x) {
    if (!(x >= -2147483648.0f && x < 2147483648.0f)) return INT_MIN;
    return (int)x;
}
/* uint32_t(int64_t(x)): 64-bit truncation (INT64_MIN when unrepresentable),
 * then the low 32 bits */
static inline uint32_t to_u32_via_i64(float x) {
    int64_t v;
    if (!(x >= -9223372036854775808.0f && x < 9223372036854775808.0f))
        v = INT64_MIN;
    else
        v = (int64_t)x;
    return (uint32_t)(uint64_t)v;
}
static inline int imax(int a, int b) { return a > b ? a : b; }
static inline int imin(int a, int b) { return a < b ? a : b; }

typedef struct {
    float x, y, z, inv_w;
} sv_t;

/* ProjectToScreen (cpu_raster.cpp:19-27) */
static inline sv_t project(const float* c, uint32_t w, uint32_t h) {
    sv_t v;
    const float inv_w = 1.f / c[3];
    v.x = (c[0] * inv_w * 0.5f + 0.5f) * (float)w;
    v.y = (c[1] * inv_w * 0.5f + 0.5f) * (float)h;
    v.z = c[2] * inv_w;
    v.inv_w = inv_w;
    return v;
}

/* ProjectClipToScreen (cpu_raster.cpp:227-239) */
static inline int project_ok(const float* c, uint32_t w, uint32_t h,
                             float s[2], float* z) {
    if (fabsf(c[3]) <= 1e-6f || c[3] < 0.f) return 0;
    sv_t v = project(c, w, h);
    s[0] = v.x;
    s[1] = v.y;
    if (z) *z = v.z;
    return 1;
}

typedef struct {
    float dist;
    int edge;
    float t;
} tridist_t;

/* SignedDistToTri (cpu_raster.cpp:114-151) */
static tridist_t signed_dist(const float p[2], const float s[3][2]) {
    tridist_t best = {0.f, 0, 0.f};
    float best_d2 = -1.f;
    int n_pos = 0, n_neg = 0;
    for (int k = 0; k < 3; k++) {
        const float* a = s[k];
        const float* b = s[(k + 1) % 3];
        const float ex = b[0] - a[0];
        const float ey = b[1] - a[1];
        const float len2 = ex * ex + ey * ey;
        float t = 0.f;
        if (len2 > 1e-6f * 1e-6f) {
            t = ((p[0] - a[0]) * ex + (p[1] - a[1]) * ey) / len2;
            t = smin(smax(t, 0.f), 1.f);
        }
        const float qx = a[0] + t * ex;
        const float qy = a[1] + t * ey;
        const float dx = p[0] - qx;
        const float dy = p[1] - qy;
        const float d2 = dx * dx + dy * dy;
        if (best_d2 < 0.f || d2 < best_d2) {
            best_d2 = d2;
            best.edge = k;
            best.t = t;
        }
        const float cr = ex * (p[1] - a[1]) - ey * (p[0] - a[0]);
        n_pos += (cr >= 0.f);
        n_neg += (cr <= 0.f);
    }
    const float sgn = (n_pos == 3 || n_neg == 3) ? 1.f : -1.f;
    best.dist = sgn * sqrtf(smax(best_d2, 0.f));
    return best;
}

/* SignedDistGradToTri (cpu_raster.cpp:153-175) */
static void signed_dist_grad(const float p[2], const float s[3][2],
                             tridist_t td, float g[3][2]) {
    memset(g, 0, sizeof(float) * 6);
    const float d = fabsf(td.dist);
    if (d < 1e-6f) return;
    const int ia = td.edge, ib = (td.edge + 1) % 3;
    const float qx = s[ia][0] + td.t * (s[ib][0] - s[ia][0]);
    const float qy = s[ia][1] + td.t * (s[ib][1] - s[ia][1]);
    const float sgn = td.dist >= 0.f ? 1.f : -1.f;
    const float nx = (p[0] - qx) / d;
    const float ny = (p[1] - qy) / d;
    g[ia][0] = -sgn * (1.f - td.t) * nx;
    g[ia][1] = -sgn * (1.f - td.t) * ny;
    g[ib][0] = -sgn * td.t * nx;
    g[ib][1] = -sgn * td.t * ny;
}

/* ScreenBarycentric (cpu_raster.cpp:177-193) */
static int screen_bary(const float p[2], const float s[3][2], float l[3]) {
    const float area = (s[1][0] - s[0][0]) * (s[2][1] - s[0][1]) -
                       (s[1][1] - s[0][1]) * (s[2][0] - s[0][0]);
    if (fabsf(area) < 1e-6f) return 0;
    const float inv_area = 1.f / area;
    l[0] = ((s[1][0] - p[0]) * (s[2][1] - p[1]) -
            (s[1][1] - p[1]) * (s[2][0] - p[0])) *
           inv_area;
    l[1] = ((s[2][0] - p[0]) * (s[0][1] - p[1]) -
            (s[2][1] - p[1]) * (s[0][0] - p[0])) *
           inv_area;
    l[2] = 1.f - l[0] - l[1];
    return 1;
}

/* ------------------------------------------------------------ rasterizers */

typedef void (*shade_fn)(void* ctx, int x, int y, uint32_t f,
                         const uint32_t idx[3], const sv_t sv[3],
                         const float l[3]);

/* RasterizeCore (cpu_raster.cpp:31-110): sequential faces, LessOrEqual depth
 * test against a clear of 1 (later face wins ties). */
static int raster_core(const float* clip, uint32_t n_verts,
                       const float* faces, uint32_t n_faces, uint32_t w,
                       uint32_t h, shade_fn shade, void* ctx) {
    float* zbuf = (float*)malloc(sizeof(float) * (size_t)w * h);
    if (!zbuf) return fail("oom");
    for (size_t i = 0; i < (size_t)w * h; i++) zbuf[i] = 1.f;
    for (uint32_t f = 0; f < n_faces; f++) {
        uint32_t idx[3];
        sv_t sv[3];
        int skip = 0;
        for (int k = 0; k < 3; k++) {
            idx[k] = to_u32_via_i64(faces[(size_t)f * 3 + k]);
            if (idx[k] >= n_verts) {
                free(zbuf);
                return fail("CPU raster: face index range");
            }
            const float* c = &clip[(size_t)idx[k] * 4];
            if (fabsf(c[3]) <= 1e-6f || c[3] < 0.f) {
                skip = 1;
                break;
            }
            sv[k] = project(c, w, h);
        }
        if (skip) continue;
        const float area = (sv[1].x - sv[0].x) * (sv[2].y - sv[0].y) -
                           (sv[1].y - sv[0].y) * (sv[2].x - sv[0].x);
        if (fabsf(area) < 1e-6f) continue;
        const float inv_area = 1.f / area;
        const float min_xf = smin(smin(sv[0].x, sv[1].x), sv[2].x);
        const float max_xf = smax(smax(sv[0].x, sv[1].x), sv[2].x);
        const float min_yf = smin(smin(sv[0].y, sv[1].y), sv[2].y);
        const float max_yf = smax(smax(sv[0].y, sv[1].y), sv[2].y);
        const int x0 = imax(0, to_i32(floorf(min_xf - 0.5f)));
        const int x1 = imin((int)w - 1, to_i32(ceilf(max_xf - 0.5f)));
        const int y0 = imax(0, to_i32(floorf(min_yf - 0.5f)));
        const int y1 = imin((int)h - 1, to_i32(ceilf(max_yf - 0.5f)));
        for (int y = y0; y <= y1; y++) {
            for (int x = x0; x <= x1; x++) {
                const float px = (float)x + 0.5f;
                const float py = (float)y + 0.5f;
                const float l0 = ((sv[1].x - px) * (sv[2].y - py) -
                                  (sv[1].y - py) * (sv[2].x - px)) *
                                 inv_area;
                const float l1 = ((sv[2].x - px) * (sv[0].y - py) -
                                  (sv[2].y - py) * (sv[0].x - px)) *
                                 inv_area;
                const float l2 = 1.f - l0 - l1;
                if (l0 < 0.f || l1 < 0.f || l2 < 0.f) continue;
                const float z = l0 * sv[0].z + l1 * sv[1].z + l2 * sv[2].z;
                if (z < 0.f || z > 1.f) continue;
                float* zb = &zbuf[(size_t)y * w + x];
                if (z > *zb) continue;
                *zb = z;
                const float l[3] = {l0, l1, l2};
                shade(ctx, x, y, f, idx, sv, l);
            }
        }
    }
    free(zbuf);
    return 0;
}

typedef struct {
    float* out;
    uint32_t w;
} fid_ctx;

static void shade_face_id(void* vc, int x, int y, uint32_t f,
                          const uint32_t idx[3], const sv_t sv[3],
                          const float l[3]) {
    (void)idx;
    (void)sv;
    (void)l;
    fid_ctx* c = (fid_ctx*)vc;
    c->out[(size_t)y * c->w + x] = (float)f + 1.f;
}

int orc_rasterize_face_id(const float* clip, uint32_t n_verts,
                          const float* faces, uint32_t n_faces, uint32_t w,
                          uint32_t h, float* out) {
    memset(out, 0, sizeof(float) * (size_t)w * h);
    fid_ctx c = {out, w};
    return raster_core(clip, n_verts, faces, n_faces, w, h, shade_face_id,
                       &c);
}

typedef struct {
    float* out;
    const float* attr;
    uint32_t w, nc;
} hard_ctx;

/* RasterizeHardCpu's shade lambda (cpu_raster.cpp:205-223) */
static void shade_hard(void* vc, int x, int y, uint32_t f,
                       const uint32_t idx[3], const sv_t sv[3],
                       const float l[3]) {
    (void)f;
    hard_ctx* c = (hard_ctx*)vc;
    const float denom =
            l[0] * sv[0].inv_w + l[1] * sv[1].inv_w + l[2] * sv[2].inv_w;
    float* dst = &c->out[((size_t)y * c->w + x) * c->nc];
    for (uint32_t ch = 0; ch < c->nc; ch++) {
        float num = 0.f;
        for (int k = 0; k < 3; k++) {
            num += l[k] * sv[k].inv_w * c->attr[(size_t)idx[k] * c->nc + ch];
        }
        dst[ch] = num / denom;
    }
}

int orc_rasterize_hard(const float* clip, uint32_t n_verts, const float* attr,
                       uint32_t n_comp, const float* faces, uint32_t n_faces,
                       uint32_t w, uint32_t h, float* out) {
    memset(out, 0, sizeof(float) * (size_t)w * h * n_comp);
    hard_ctx c = {out, attr, w, n_comp};
    return raster_core(clip, n_verts, faces, n_faces, w, h, shade_hard, &c);
}

/* F::SoftClip's CPU kernel (f_ops.cpp:1917-1978) */
int orc_soft_clip(const float* clip, uint32_t n_verts, const float* faces,
                  uint32_t n_faces, uint32_t w, uint32_t h, float radius,
                  float* out) {
    memset(out, 0, sizeof(float) * (size_t)n_faces * 12);
    for (uint32_t f = 0; f < n_faces; f++) {
        uint32_t idx[3];
        float s[3][2];
        const float* c[3];
        int valid = 1;
        for (int k = 0; k < 3; k++) {
            idx[k] = to_u32_via_i64(faces[(size_t)f * 3 + k] + 0.5f);
            if (idx[k] >= n_verts) return fail("SoftClip: vertex index range");
            c[k] = &clip[(size_t)idx[k] * 4];
            if (c[k][3] <= 1e-6f || !project_ok(c[k], w, h, s[k], NULL))
                valid = 0;
        }
        float scale = 1.f, cx = 0.f, cy = 0.f;
        if (valid) {
            cx = (s[0][0] + s[1][0] + s[2][0]) / 3.f;
            cy = (s[0][1] + s[1][1] + s[2][1]) / 3.f;
            float d_min = 1e30f;
            for (int k = 0; k < 3; k++) {
                const int k2 = (k + 1) % 3;
                const float ex = s[k2][0] - s[k][0];
                const float ey = s[k2][1] - s[k][1];
                const float len = sqrtf(ex * ex + ey * ey);
                if (len < 1e-6f) continue;
                d_min = smin(d_min, fabsf(ex * (cy - s[k][1]) -
                                          ey * (cx - s[k][0])) /
                                            len);
            }
            scale = d_min < 1e29f
                            ? smin(1.f + radius / smax(d_min, 1e-3f), 8.f)
                            : 1.f;
        }
        for (int k = 0; k < 3; k++) {
            float* dst = &out[((size_t)f * 3 + (size_t)k) * 4];
            for (int j = 0; j < 4; j++) dst[j] = c[k][j];
            if (valid) {
                const float sx = cx + (s[k][0] - cx) * scale;
                const float sy = cy + (s[k][1] - cy) * scale;
                dst[0] = (sx / (float)w * 2.f - 1.f) * c[k][3];
                dst[1] = (sy / (float)h * 2.f - 1.f) * c[k][3];
            }
        }
    }
    return 0;
}

/* RasterizeSoftCpu (cpu_raster.cpp:241-355) */
int orc_rasterize_soft(const float* soft_clip, uint32_t n_soft,
                       const float* face_id, const float* faces_soft,
                       uint32_t n_faces, const float* hard_clip,
                       uint32_t n_hard, const float* faces_tex, uint32_t w,
                       uint32_t h, float radius, const float* prev_depth,
                       float* out) {
    const size_t npx = (size_t)w * h;
    memset(out, 0, sizeof(float) * npx * 4);
    float* zbuf = (float*)malloc(sizeof(float) * npx);
    if (!zbuf) return fail("oom");
    for (size_t i = 0; i < npx; i++) zbuf[i] = 1.f;
    for (uint32_t f = 0; f < n_faces; f++) {
        float ss[3][2], sz[3], fid = 0.f;
        int valid = 1;
        for (int k = 0; k < 3; k++) {
            const uint32_t vi = to_u32_via_i64(faces_soft[(size_t)f * 3 + k]);
            if (vi >= n_soft) {
                free(zbuf);
                return fail("RasterizeSoftCpu: soft index range");
            }
            if (!project_ok(&soft_clip[(size_t)vi * 4], w, h, ss[k], &sz[k])) {
                valid = 0;
                break;
            }
            fid = face_id[vi];
        }
        if (!valid) continue;
        const uint32_t hf = to_u32_via_i64(fid + 0.5f);
        if (hf >= n_faces) {
            free(zbuf);
            return fail("RasterizeSoftCpu: face id range");
        }
        float hs[3][2], hz[3];
        for (int k = 0; k < 3; k++) {
            const uint32_t vi =
                    to_u32_via_i64(faces_tex[(size_t)hf * 3 + k] + 0.5f);
            if (vi >= n_hard) {
                free(zbuf);
                return fail("RasterizeSoftCpu: hard index range");
            }
            if (!project_ok(&hard_clip[(size_t)vi * 4], w, h, hs[k], &hz[k])) {
                valid = 0;
                break;
            }
        }
        if (!valid) continue;
        const float min_x = smin(smin(ss[0][0], ss[1][0]), ss[2][0]);
        const float max_x = smax(smax(ss[0][0], ss[1][0]), ss[2][0]);
        const float min_y = smin(smin(ss[0][1], ss[1][1]), ss[2][1]);
        const float max_y = smax(smax(ss[0][1], ss[1][1]), ss[2][1]);
        const int x0 = imax(0, to_i32(floorf(min_x - 0.5f)));
        const int x1 = imin((int)w - 1, to_i32(ceilf(max_x - 0.5f)));
        const int y0 = imax(0, to_i32(floorf(min_y - 0.5f)));
        const int y1 = imin((int)h - 1, to_i32(ceilf(max_y - 0.5f)));
        for (int y = y0; y <= y1; y++) {
            for (int x = x0; x <= x1; x++) {
                const float p[2] = {(float)x + 0.5f, (float)y + 0.5f};
                float sl[3];
                if (!screen_bary(p, ss, sl) || sl[0] < 0.f || sl[1] < 0.f ||
                    sl[2] < 0.f)
                    continue;
                const float soft_z = sl[0] * sz[0] + sl[1] * sz[1] +
                                     sl[2] * sz[2];
                if (soft_z < 0.f || soft_z > 1.f) continue;
                const tridist_t td = signed_dist(p, hs);
                float hl[3];
                float hard_z = 0.5f;
                if (screen_bary(p, hs, hl))
                    hard_z = hl[0] * hz[0] + hl[1] * hz[1] + hl[2] * hz[2];
                const float depth =
                        td.dist >= 0.f
                                ? 0.5f * smin(smax(hard_z, 0.f), 1.f)
                                : 0.5f + 0.5f * smin(-td.dist / radius, 1.f);
                if (prev_depth &&
                    depth <= prev_depth[(size_t)y * w + x] + 1e-4f)
                    continue;
                float* zb = &zbuf[(size_t)y * w + x];
                if (depth > *zb) continue;
                *zb = depth;
                float* dst = &out[((size_t)y * w + x) * 4];
                dst[0] = td.dist;
                dst[1] = fid;
                dst[2] = hard_z;
                dst[3] = 1.f;
            }
        }
    }
    free(zbuf);
    return 0;
}

/* GatherDistGrad's CPU kernel (f_ops.cpp:1289-1352) summed straight into
 * {V} (the ColSum of the wide partials, f_ops.cpp:1218-1246) */
int orc_dist_grad(const float* gy, const float* rs, const float* clip,
                  uint32_t n_verts, const float* faces, uint32_t n_faces,
                  uint32_t w, uint32_t h, float* grad) {
    memset(grad, 0, sizeof(float) * (size_t)n_verts * 4);
    const float w_scr = (float)w, h_scr = (float)h;
    for (uint32_t y = 0; y < h; y++) {
        for (uint32_t x = 0; x < w; x++) {
            const size_t o = ((size_t)y * w + x) * 4;
            if (rs[o + 3] < 0.5f) continue;
            const float g = gy[(size_t)y * w + x];
            if (g == 0.f) continue;
            const uint32_t f = to_u32_via_i64(rs[o + 1] + 0.5f);
            if (f >= n_faces) return fail("dist grad: face id range");
            uint32_t idx[3];
            float s[3][2];
            int valid = 1;
            for (int k = 0; k < 3; k++) {
                idx[k] = to_u32_via_i64(faces[(size_t)f * 3 + k] + 0.5f);
                if (idx[k] >= n_verts)
                    return fail("dist grad: vertex index range");
                if (!project_ok(&clip[(size_t)idx[k] * 4], w, h, s[k], NULL)) {
                    valid = 0;
                    break;
                }
            }
            if (!valid) continue;
            const float p[2] = {(float)x + 0.5f, (float)y + 0.5f};
            const tridist_t td = signed_dist(p, s);
            float gs[3][2];
            signed_dist_grad(p, s, td, gs);
            for (int k = 0; k < 3; k++) {
                const float gsx = g * gs[k][0];
                const float gsy = g * gs[k][1];
                if (gsx == 0.f && gsy == 0.f) continue;
                const float* c = &clip[(size_t)idx[k] * 4];
                float* dst = &grad[(size_t)idx[k] * 4];
                dst[0] += gsx * 0.5f * w_scr / c[3];
                dst[1] += gsy * 0.5f * h_scr / c[3];
                dst[3] += -(gsx * 0.5f * w_scr * c[0] +
                            gsy * 0.5f * h_scr * c[1]) /
                          (c[3] * c[3]);
            }
        }
    }
    return 0;
}

void orc_transform_clip(const float* pos, uint32_t n_verts, const float* m,
                        float* clip) {
    for (uint32_t i = 0; i < n_verts; i++) {
        const float x = pos[i * 3 + 0], y = pos[i * 3 + 1],
                    z = pos[i * 3 + 2];
        for (int r = 0; r < 4; r++) {
            clip[i * 4 + r] =
                    x * m[0 * 4 + r] + y * m[1 * 4 + r] + z * m[2 * 4 + r] +
                    m[3 * 4 + r];
        }
    }
}

/* ------------------------------------------------- silhouette iteration */

/* Per-pixel loss and dist-channel gradient of the silhouette graph
 * (ref_driver.cpp SilViewLoss), in the operation order the reference
 * autodiff produces (build_backward.cpp:62-149 over the f_ops.cpp
 * backward generators): see the derivation in the repository's design
 * notes. Returns the pixel's loss; *g_dist = dL/d dist. */
static inline float sil_pixel(const float* rs4, float target, float k,
                              float c, float* g_dist) {
    const float dist = rs4[0], cov = rs4[3];
    const float step = dist < 0.f ? 0.f : 1.f;            /* Step(0, dist) */
    const float hard = cov * step;
    const float a = fabsf(dist);                          /* Abs */
    const float m1 = dist * a;                            /* dist*|dist| */
    const float m2 = m1 * k;
    const float s = 1.f / (1.f + expf(-m2));              /* Sigmoid */
    const float soft = cov * s;
    const float pred = smax(hard, soft);                  /* Max */
    const float diff = target - pred;
    const float lv = diff * diff * c;
    /* backward (seed 1 per pixel) */
    const float g_m4 = 1.f * c;
    const float g_diff = g_m4 * diff + g_m4 * diff;
    const float g_pred = -g_diff;
    const float mask = hard < soft ? 0.f : 1.f;           /* Step(soft,hard)*/
    const float g_m3 = g_pred * (1.f - mask);
    const float g_sg = g_m3 * cov;
    const float g_m2 = g_sg * (s * (1.f - s));
    const float g_m1 = g_m2 * k;
    const float sgn = (float)((dist > 0.f) - (dist < 0.f));
    *g_dist = g_m1 * a + (g_m1 * dist) * sgn;
    return lv;
}

static int sil_view(const float* pos, uint32_t n_verts, const float* faces,
                    uint32_t n_faces, uint32_t res, float radius, float sigma,
                    const float* mvp, const float* target, double* loss,
                    float* gpos, float* rs_out) {
    const size_t npx = (size_t)res * res;
    int rc = 1;
    float* clip = (float*)malloc(sizeof(float) * n_verts * 4);
    float* soft = (float*)malloc(sizeof(float) * n_faces * 12);
    float* fid = (float*)malloc(sizeof(float) * n_faces * 3);
    float* fs = (float*)malloc(sizeof(float) * n_faces * 3);
    float* rs = rs_out ? rs_out : (float*)malloc(sizeof(float) * npx * 4);
    float* gd = (float*)malloc(sizeof(float) * npx);
    float* gc = (float*)malloc(sizeof(float) * n_verts * 4);
    if (!clip || !soft || !fid || !fs || !rs || !gd || !gc) {
        fail("oom");
        goto done;
    }
    for (uint32_t f = 0; f < n_faces; f++)
        for (uint32_t k = 0; k < 3; k++) {
            fid[f * 3 + k] = (float)f;
            fs[f * 3 + k] = (float)(f * 3 + k);
        }
    orc_transform_clip(pos, n_verts, mvp, clip);
    if (orc_soft_clip(clip, n_verts, faces, n_faces, res, res, radius, soft))
        goto done;
    if (orc_rasterize_soft(soft, n_faces * 3, fid, fs, n_faces, clip, n_verts,
                           faces, res, res, radius, NULL, rs))
        goto done;
    const float k = (2.f / (float)res) * (2.f / (float)res) / sigma;
    const float c = 1.f / (float)(res * res);
    double l = 0.0;
    for (size_t i = 0; i < npx; i++) l += sil_pixel(&rs[i * 4], target[i], k, c, &gd[i]);
    *loss = l;
    if (orc_dist_grad(gd, rs, clip, n_verts, faces, n_faces, res, res, gc))
        goto done;
    /* clip -> pos (TransformToClipVar's backward) */
    for (uint32_t i = 0; i < n_verts; i++) {
        const float* g = &gc[i * 4];
        for (int j = 0; j < 3; j++) {
            gpos[i * 3 + j] = g[0] * mvp[j * 4 + 0] + g[1] * mvp[j * 4 + 1] +
                              g[2] * mvp[j * 4 + 2] + g[3] * mvp[j * 4 + 3];
        }
    }
    rc = 0;
done:
    free(clip);
    free(soft);
    free(fid);
    free(fs);
    if (!rs_out) free(rs);
    free(gd);
    free(gc);
    return rc;
}

typedef struct {
    const float* pos;
    uint32_t n_verts, n_faces, n_views, res;
    const float* faces;
    float radius, sigma;
    const float* mvps;
    const float* targets;
    double* vloss;
    float* vgrad; /* n_views * V*3 */
    float* rs_out;
    int next, err;
    pthread_mutex_t mu;
} sil_job;

static void* sil_worker(void* arg) {
    sil_job* j = (sil_job*)arg;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        const int v = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (v >= (int)j->n_views) break;
        const size_t npx = (size_t)j->res * j->res;
        if (sil_view(j->pos, j->n_verts, j->faces, j->n_faces, j->res,
                     j->radius, j->sigma, j->mvps + (size_t)v * 16,
                     j->targets + (size_t)v * npx, &j->vloss[v],
                     j->vgrad + (size_t)v * j->n_verts * 3,
                     j->rs_out ? j->rs_out + (size_t)v * npx * 4 : NULL)) {
            j->err = 1;
        }
    }
    return NULL;
}

static int sil_loss_grad_mt(const float* pos, uint32_t n_verts,
                            const float* faces, uint32_t n_faces,
                            uint32_t n_views, uint32_t res, float radius,
                            float sigma, const float* mvps,
                            const float* targets, double* loss, float* grad,
                            float* rs_out, uint32_t threads) {
    sil_job j;
    memset(&j, 0, sizeof(j));
    j.pos = pos;
    j.n_verts = n_verts;
    j.n_faces = n_faces;
    j.n_views = n_views;
    j.res = res;
    j.faces = faces;
    j.radius = radius;
    j.sigma = sigma;
    j.mvps = mvps;
    j.targets = targets;
    j.rs_out = rs_out;
    j.vloss = (double*)calloc(n_views, sizeof(double));
    j.vgrad = (float*)calloc((size_t)n_views * n_verts * 3, sizeof(float));
    if (!j.vloss || !j.vgrad) {
        free(j.vloss);
        free(j.vgrad);
        return fail("oom");
    }
    pthread_mutex_init(&j.mu, NULL);
    if (threads < 1) threads = 1;
    if (threads > n_views) threads = n_views;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * threads);
    for (uint32_t i = 1; i < threads; i++)
        pthread_create(&th[i], NULL, sil_worker, &j);
    sil_worker(&j);
    for (uint32_t i = 1; i < threads; i++) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&j.mu);
    int rc = j.err;
    if (!rc) {
        double l = 0.0;
        memset(grad, 0, sizeof(float) * n_verts * 3);
        for (uint32_t v = 0; v < n_views; v++) {
            l += j.vloss[v];
            const float* g = j.vgrad + (size_t)v * n_verts * 3;
            for (size_t i = 0; i < (size_t)n_verts * 3; i++) grad[i] += g[i];
        }
        *loss = l;
    }
    free(j.vloss);
    free(j.vgrad);
    return rc;
}

int orc_silhouette_loss_grad(const float* pos, uint32_t n_verts,
                             const float* faces, uint32_t n_faces,
                             uint32_t n_views, uint32_t res, float radius,
                             float sigma, const float* mvps,
                             const float* targets, double* loss, float* grad,
                             float* rs_out) {
    return sil_loss_grad_mt(pos, n_verts, faces, n_faces, n_views, res,
                            radius, sigma, mvps, targets, loss, grad, rs_out,
                            1);
}

/* In-graph Adam (examples/silhouette_optimization/run.cpp:421-436) */
void orc_adam(float* p, float* m, float* v, float* t, const float* g,
              uint32_t n, float lr, float b1, float b2, float eps) {
    const float t_new = *t + 1.f;
    const float bc1 = 1.f - powf(b1, t_new);
    const float bc2 = 1.f - powf(b2, t_new);
    for (uint32_t i = 0; i < n; i++) {
        const float m_new = m[i] * b1 + g[i] * (1.f - b1);
        const float v_new = v[i] * b2 + g[i] * g[i] * (1.f - b2);
        const float step = (m_new / bc1) / (sqrtf(v_new / bc2) + eps) * lr;
        p[i] = p[i] - step;
        m[i] = m_new;
        v[i] = v_new;
    }
    *t = t_new;
}

int orc_silhouette_run(float* pos, uint32_t n_verts, const float* faces,
                       uint32_t n_faces, uint32_t n_views, uint32_t res,
                       float radius, float sigma, float lr, const float* mvps,
                       const float* targets, uint32_t n_iters,
                       uint32_t threads, float* loss_trace) {
    const size_t n = (size_t)n_verts * 3;
    float* m = (float*)calloc(n, sizeof(float));
    float* v = (float*)calloc(n, sizeof(float));
    float* g = (float*)calloc(n, sizeof(float));
    float t = 0.f;
    int rc = 0;
    if (!m || !v || !g) rc = fail("oom");
    for (uint32_t it = 0; it < n_iters && !rc; it++) {
        double l = 0.0;
        rc = sil_loss_grad_mt(pos, n_verts, faces, n_faces, n_views, res,
                              radius, sigma, mvps, targets, &l, g, NULL,
                              threads);
        if (rc) break;
        loss_trace[it] = (float)l;
        orc_adam(pos, m, v, &t, g, (uint32_t)n, lr, 0.9f, 0.999f, 1e-8f);
    }
    free(m);
    free(v);
    free(g);
    return rc;
}

/* ------------------------------------------------------ screen-space AA */

typedef struct {
    float r;
    uint32_t ia, ib;     /* vertex ids of the chosen edge */
    float qa[2], qb[2];  /* its screen endpoints */
    float es, len;       /* edge function at s's centre, edge length */
} aa_pair_t;

static const int kAaOffs[8][2] = {{-1, -1}, {0, -1}, {1, -1}, {-1, 0},
                                  {1, 0},   {-1, 1}, {0, 1},  {1, 1}};

/* EvalAaPair (cpu_raster.cpp:371-454): the silhouette edge crossed between
 * pixel s and its neighbour n, taken from the owner triangle (n's first,
 * then s's), with r = min(|e(s)| / |edge|, 1). */
static int aa_pair(const float* tri, const float* clip, uint32_t n_verts,
                   const float* faces, uint32_t n_faces, uint32_t w,
                   uint32_t h, int sx, int sy, int nx, int ny,
                   aa_pair_t* out) {
    const int its = to_i32(tri[(size_t)sy * w + sx] + 0.5f);
    const int itn = to_i32(tri[(size_t)ny * w + nx] + 0.5f);
    if (its == itn) return 0;
    const float ps[2] = {(float)sx + 0.5f, (float)sy + 0.5f};
    const float pn[2] = {(float)nx + 0.5f, (float)ny + 0.5f};
    for (int o = 0; o < 2; o++) {
        const int owner = o == 0 ? itn : its;
        if (owner == 0) continue;
        const uint32_t f = (uint32_t)owner - 1u;
        if (f >= n_faces) continue;
        uint32_t vi[3];
        float q[3][2];
        int ok = 1;
        for (int k = 0; k < 3; k++) {
            vi[k] = to_u32_via_i64(faces[(size_t)f * 3 + k] + 0.5f);
            if (vi[k] >= n_verts ||
                !project_ok(&clip[(size_t)vi[k] * 4], w, h, q[k], NULL)) {
                ok = 0;
                break;
            }
        }
        if (!ok) continue;
        int best_j = -1;
        float best_t = 0.f;
        for (int j = 0; j < 3; j++) {
            const float* a = q[j];
            const float* b = q[(j + 1) % 3];
            const float es = (b[0] - a[0]) * (ps[1] - a[1]) -
                             (b[1] - a[1]) * (ps[0] - a[0]);
            const float en = (b[0] - a[0]) * (pn[1] - a[1]) -
                             (b[1] - a[1]) * (pn[0] - a[0]);
            if (es * en >= 0.f) continue;
            const float t = es / (es - en);
            if (best_j < 0 || (o == 0 ? t > best_t : t < best_t)) {
                best_t = t;
                best_j = j;
            }
        }
        if (best_j < 0) continue;
        const float* a = q[best_j];
        const float* b = q[(best_j + 1) % 3];
        const float ex = b[0] - a[0];
        const float ey = b[1] - a[1];
        const float len = sqrtf(ex * ex + ey * ey);
        if (len < 1e-6f) continue;
        const float es = ex * (ps[1] - a[1]) - ey * (ps[0] - a[0]);
        out->r = smin(fabsf(es) / len, 1.f);
        out->ia = vi[best_j];
        out->ib = vi[(best_j + 1) % 3];
        out->qa[0] = a[0];
        out->qa[1] = a[1];
        out->qb[0] = b[0];
        out->qb[1] = b[1];
        out->es = es;
        out->len = len;
        return 1;
    }
    return 0;
}

static inline int aa_inside(int x, int y, uint32_t w, uint32_t h) {
    return x >= 0 && y >= 0 && x < (int)w && y < (int)h;
}

int orc_antialias(const float* img, uint32_t n_comp, const float* tri,
                  const float* clip, uint32_t n_verts, const float* faces,
                  uint32_t n_faces, uint32_t w, uint32_t h, float* out) {
    if (n_comp < 1 || n_comp > 4) return fail("antialias: n_comp 1..4");
    for (int y = 0; y < (int)h; y++) {
        for (int x = 0; x < (int)w; x++) {
            const size_t so = ((size_t)y * w + x) * n_comp;
            const float* cs = &img[so];
            float* dst = &out[so];
            for (uint32_t c = 0; c < n_comp; c++) dst[c] = cs[c];
            for (int k = 0; k < 8; k++) {
                const int nx = x + kAaOffs[k][0], ny = y + kAaOffs[k][1];
                aa_pair_t pr;
                if (!aa_inside(nx, ny, w, h) ||
                    !aa_pair(tri, clip, n_verts, faces, n_faces, w, h, x, y,
                             nx, ny, &pr)) {
                    for (uint32_t c = 0; c < n_comp; c++) dst[c] += cs[c];
                    continue;
                }
                const float* cn = &img[((size_t)ny * w + nx) * n_comp];
                for (uint32_t c = 0; c < n_comp; c++)
                    dst[c] += pr.r * cs[c] + (1.f - pr.r) * cn[c];
            }
            for (uint32_t c = 0; c < n_comp; c++) dst[c] /= 9.f;
        }
    }
    return 0;
}

int orc_antialias_bwd_img(const float* gy, uint32_t n_comp, const float* tri,
                          const float* clip, uint32_t n_verts,
                          const float* faces, uint32_t n_faces, uint32_t w,
                          uint32_t h, float* out) {
    if (n_comp < 1 || n_comp > 4) return fail("antialias: n_comp 1..4");
    for (int y = 0; y < (int)h; y++) {
        for (int x = 0; x < (int)w; x++) {
            const size_t so = ((size_t)y * w + x) * n_comp;
            float alpha_sum = 0.f;
            float* dst = &out[so];
            for (uint32_t c = 0; c < n_comp; c++) dst[c] = 0.f;
            for (int k = 0; k < 8; k++) {
                const int nx = x + kAaOffs[k][0], ny = y + kAaOffs[k][1];
                if (!aa_inside(nx, ny, w, h)) {
                    alpha_sum += 1.f;
                    continue;
                }
                aa_pair_t pr, pr2;
                alpha_sum += aa_pair(tri, clip, n_verts, faces, n_faces, w, h,
                                     x, y, nx, ny, &pr)
                                     ? pr.r
                                     : 1.f;
                if (aa_pair(tri, clip, n_verts, faces, n_faces, w, h, nx, ny,
                            x, y, &pr2)) {
                    const size_t no = ((size_t)ny * w + nx) * n_comp;
                    for (uint32_t c = 0; c < n_comp; c++)
                        dst[c] += (1.f - pr2.r) * gy[no + c];
                }
            }
            for (uint32_t c = 0; c < n_comp; c++) {
                dst[c] += gy[so + c] * (1.f + alpha_sum);
                dst[c] /= 9.f;
            }
        }
    }
    return 0;
}

/* Wang's integer hash and its [0,1) mapping (f_ops.cpp:1473-1487) */
static inline uint32_t wang_hash(uint32_t x) {
    x = (x ^ 61u) ^ (x >> 16);
    x *= 9u;
    x ^= x >> 4;
    x *= 0x27d4eb2du;
    x ^= x >> 15;
    return x;
}

static inline float hash_to_unit(uint32_t f, uint32_t s, uint32_t seed,
                                 uint32_t salt) {
    const uint32_t hsh = wang_hash(f * 9781u ^ s * 6151u ^ seed * 26699u ^
                                   salt * 42589u);
    return (float)(hsh & 0xFFFFFFu) / 16777216.f;
}

float orc_hash_to_unit(uint32_t f, uint32_t s, uint32_t seed, uint32_t salt) {
    return hash_to_unit(f, s, seed, salt);
}

/* One active pair's vertex gradient (AntiAliasBwdVtx's accumulate lambda,
 * f_ops.cpp:2329-2372): into dst_v for vertex v only (only_v), else into
 * both endpoint rows of out. */
static void aa_accumulate(const float* gy, const float* img, uint32_t n_comp,
                          const float* clip, uint32_t w, uint32_t h,
                          uint32_t v, int x, int y, int nx, int ny,
                          const aa_pair_t* pr, int only_v, float* dst_v,
                          float* out) {
    const size_t so = ((size_t)y * w + x) * n_comp;
    const size_t no = ((size_t)ny * w + nx) * n_comp;
    const float w_scr = (float)w, h_scr = (float)h;
    float gr = 0.f;
    for (uint32_t c = 0; c < n_comp; c++)
        gr += gy[so + c] * (img[so + c] - img[no + c]);
    gr /= 9.f;
    if (gr == 0.f) return;
    const float ps[2] = {(float)x + 0.5f, (float)y + 0.5f};
    const float sgn = pr->es >= 0.f ? 1.f : -1.f;
    const float inv_l = 1.f / pr->len;
    const float l3 = fabsf(pr->es) * inv_l * inv_l * inv_l;
    const float ex = pr->qb[0] - pr->qa[0];
    const float ey = pr->qb[1] - pr->qa[1];
    const float dqa[2] = {sgn * inv_l * (pr->qb[1] - ps[1]) + l3 * ex,
                          sgn * inv_l * (ps[0] - pr->qb[0]) + l3 * ey};
    const float dqb[2] = {sgn * inv_l * (ps[1] - pr->qa[1]) - l3 * ex,
                          sgn * inv_l * (pr->qa[0] - ps[0]) - l3 * ey};
    const uint32_t ids[2] = {pr->ia, pr->ib};
    const float* dqs[2] = {dqa, dqb};
    for (int e = 0; e < 2; e++) {
        if (only_v && ids[e] != v) continue;
        const float gqx = gr * dqs[e][0];
        const float gqy = gr * dqs[e][1];
        const float* c = &clip[(size_t)ids[e] * 4];
        float* dst = only_v ? dst_v : &out[(size_t)ids[e] * 4];
        dst[0] += gqx * 0.5f * w_scr / c[3];
        dst[1] += gqy * 0.5f * h_scr / c[3];
        dst[3] += -(gqx * 0.5f * w_scr * c[0] + gqy * 0.5f * h_scr * c[1]) /
                  (c[3] * c[3]);
    }
}

int orc_antialias_bwd_vtx(const float* gy, const float* img, uint32_t n_comp,
                          const float* tri, const float* clip,
                          uint32_t n_verts, const float* faces,
                          uint32_t n_faces, const float* vft,
                          uint32_t max_deg, float seed, uint32_t n_samples,
                          uint32_t w, uint32_t h, float* grad) {
    if (n_comp < 1 || n_comp > 4) return fail("antialias: n_comp 1..4");
    memset(grad, 0, sizeof(float) * (size_t)n_verts * 4);
    if (n_samples == 0) {
        /* exact: every boundary pixel pair (f_ops.cpp:2373-2396) */
        for (int y = 0; y < (int)h; y++)
            for (int x = 0; x < (int)w; x++)
                for (int k = 0; k < 8; k++) {
                    const int nx = x + kAaOffs[k][0], ny = y + kAaOffs[k][1];
                    if (!aa_inside(nx, ny, w, h)) continue;
                    aa_pair_t pr;
                    if (!aa_pair(tri, clip, n_verts, faces, n_faces, w, h, x,
                                 y, nx, ny, &pr) ||
                        pr.r >= 1.f)
                        continue;
                    aa_accumulate(gy, img, n_comp, clip, w, h, 0, x, y, nx,
                                  ny, &pr, 0, NULL, grad);
                }
        return 0;
    }
    /* stochastic, wide layout {V, max_deg} + ColSum (f_ops.cpp:2397-2470,
     * 2567-2572; ColSum 1218-1246: rows summed in order) */
    float* part = (float*)calloc((size_t)n_verts * max_deg * 4, sizeof(float));
    if (!part) return fail("oom");
    const uint32_t seed_u = to_u32_via_i64(seed + 0.5f);
    const float w_scr = (float)w, h_scr = (float)h;
    for (uint32_t v = 0; v < n_verts; v++) {
        for (uint32_t d = 0; d < max_deg; d++) {
            float* dst_v = &part[((size_t)d * n_verts + v) * 4];
            const float fv = vft[(size_t)d * n_verts + v];
            if (fv < -0.5f) continue;
            const uint32_t f = to_u32_via_i64(fv + 0.5f);
            if (f >= n_faces) continue; /* the reference reads out of range */
            float s3[3][2];
            int ok = 1;
            for (int k = 0; k < 3; k++) {
                const uint32_t vi = to_u32_via_i64(faces[(size_t)f * 3 + k] + 0.5f);
                if (vi >= n_verts) { ok = 0; break; }
                const float* c = &clip[(size_t)vi * 4];
                if (c[3] <= 1e-6f) { ok = 0; break; }
                s3[k][0] = (c[0] / c[3] * 0.5f + 0.5f) * w_scr;
                s3[k][1] = (c[1] / c[3] * 0.5f + 0.5f) * h_scr;
            }
            if (!ok) continue;
            for (uint32_t smp = 0; smp < n_samples; smp++) {
                const int e = (int)(smp % 3);
                const float* a = s3[e];
                const float* b = s3[(e + 1) % 3];
                const float ex = b[0] - a[0];
                const float ey = b[1] - a[1];
                const float len = sqrtf(ex * ex + ey * ey);
                if (len < 1e-6f) continue;
                const float u = hash_to_unit(f, smp, seed_u, 2);
                const float o = (hash_to_unit(f, smp, seed_u, 3) * 2.f - 1.f) * 2.f;
                const int x = to_i32(floorf(a[0] + u * ex - o * (ey / len)));
                const int y = to_i32(floorf(a[1] + u * ey + o * (ex / len)));
                if (!aa_inside(x, y, w, h)) continue;
                for (int k = 0; k < 8; k++) {
                    const int nx = x + kAaOffs[k][0], ny = y + kAaOffs[k][1];
                    if (!aa_inside(nx, ny, w, h)) continue;
                    aa_pair_t pr;
                    if (!aa_pair(tri, clip, n_verts, faces, n_faces, w, h, x,
                                 y, nx, ny, &pr) ||
                        pr.r >= 1.f)
                        continue;
                    if (pr.ia != v && pr.ib != v) continue;
                    aa_accumulate(gy, img, n_comp, clip, w, h, v, x, y, nx,
                                  ny, &pr, 1, dst_v, NULL);
                }
            }
        }
    }
    for (uint32_t d = 0; d < max_deg; d++)
        for (size_t i = 0; i < (size_t)n_verts * 4; i++)
            grad[i] += part[(size_t)d * n_verts * 4 + i];
    free(part);
    return 0;
}

/* ------------------------------------------- AA silhouette iteration (C4) */

/* Hard mask, triangle ids and their anti-aliased image of one view
 * (examples/silhouette_optimization/run.cpp:230-238): mask =
 * Rasterize(clip, ones), tri = RasterizeFaceId(clip), aa = AntiAlias(mask,
 * tri, clip). Buffers are W*W. */
static int aa_view_fwd(const float* clip, uint32_t n_verts, const float* faces,
                       uint32_t n_faces, uint32_t res, float* mask,
                       float* tri, float* aa) {
    float* ones = (float*)malloc(sizeof(float) * n_verts);
    if (!ones) return fail("oom");
    for (uint32_t i = 0; i < n_verts; i++) ones[i] = 1.f;
    int rc = orc_rasterize_hard(clip, n_verts, ones, 1, faces, n_faces, res,
                                res, mask);
    free(ones);
    if (rc) return rc;
    rc = orc_rasterize_face_id(clip, n_verts, faces, n_faces, res, res, tri);
    if (rc) return rc;
    return orc_antialias(mask, 1, tri, clip, n_verts, faces, n_faces, res,
                         res, aa);
}

int orc_aa_targets(const float* target_pos, uint32_t n_verts,
                   const float* faces, uint32_t n_faces, uint32_t n_views,
                   uint32_t res, const float* mvps, float* out) {
    const size_t npx = (size_t)res * res;
    float* clip = (float*)malloc(sizeof(float) * n_verts * 4);
    float* mask = (float*)malloc(sizeof(float) * npx);
    float* tri = (float*)malloc(sizeof(float) * npx);
    int rc = (!clip || !mask || !tri) ? fail("oom") : 0;
    for (uint32_t v = 0; v < n_views && !rc; v++) {
        orc_transform_clip(target_pos, n_verts, mvps + (size_t)v * 16, clip);
        rc = aa_view_fwd(clip, n_verts, faces, n_faces, res, mask, tri,
                         out + (size_t)v * npx);
    }
    free(clip);
    free(mask);
    free(tri);
    return rc;
}

/* One view of the C4 graph: loss = sum_px (t - aa)^2 / R^2, the backward
 * of (t - pred)^2 * c in the reference AD's operation order (as sil_pixel),
 * the AntiAlias vertex backward (n_samples, seed) and the clip transform's
 * backward. */
static int aa_view(const float* pos, uint32_t n_verts, const float* faces,
                   uint32_t n_faces, const float* vft, uint32_t max_deg,
                   uint32_t res, uint32_t n_samples, float seed,
                   const float* mvp, const float* target, double* loss,
                   float* gpos, float* pred_out) {
    const size_t npx = (size_t)res * res;
    int rc = 1;
    float* clip = (float*)malloc(sizeof(float) * n_verts * 4);
    float* mask = (float*)malloc(sizeof(float) * npx);
    float* tri = (float*)malloc(sizeof(float) * npx);
    float* pred = pred_out ? pred_out : (float*)malloc(sizeof(float) * npx);
    float* gy = (float*)malloc(sizeof(float) * npx);
    float* gc = (float*)malloc(sizeof(float) * n_verts * 4);
    if (!clip || !mask || !tri || !pred || !gy || !gc) {
        fail("oom");
        goto done;
    }
    orc_transform_clip(pos, n_verts, mvp, clip);
    if (aa_view_fwd(clip, n_verts, faces, n_faces, res, mask, tri, pred))
        goto done;
    const float c = 1.f / (float)(res * res);
    double l = 0.0;
    for (size_t i = 0; i < npx; i++) {
        const float diff = target[i] - pred[i];
        l += diff * diff * c;
        const float g_m4 = 1.f * c;
        gy[i] = -(g_m4 * diff + g_m4 * diff);
    }
    *loss = l;
    if (orc_antialias_bwd_vtx(gy, mask, 1, tri, clip, n_verts, faces, n_faces,
                              vft, max_deg, seed, n_samples, res, res, gc))
        goto done;
    for (uint32_t i = 0; i < n_verts; i++) {
        const float* g = &gc[i * 4];
        for (int j = 0; j < 3; j++) {
            gpos[i * 3 + j] = g[0] * mvp[j * 4 + 0] + g[1] * mvp[j * 4 + 1] +
                              g[2] * mvp[j * 4 + 2] + g[3] * mvp[j * 4 + 3];
        }
    }
    rc = 0;
done:
    free(clip);
    free(mask);
    free(tri);
    if (!pred_out) free(pred);
    free(gy);
    free(gc);
    return rc;
}

typedef struct {
    const float* pos;
    uint32_t n_verts, n_faces, n_views, res, max_deg, n_samples;
    const float* faces;
    const float* vft;
    float seed;
    const float* mvps;
    const float* targets;
    double* vloss;
    float* vgrad;
    float* pred_out;
    int next, err;
    pthread_mutex_t mu;
} aa_job;

static void* aa_worker(void* arg) {
    aa_job* j = (aa_job*)arg;
    for (;;) {
        pthread_mutex_lock(&j->mu);
        const int v = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (v >= (int)j->n_views) break;
        const size_t npx = (size_t)j->res * j->res;
        if (aa_view(j->pos, j->n_verts, j->faces, j->n_faces, j->vft,
                    j->max_deg, j->res, j->n_samples, j->seed,
                    j->mvps + (size_t)v * 16, j->targets + (size_t)v * npx,
                    &j->vloss[v], j->vgrad + (size_t)v * j->n_verts * 3,
                    j->pred_out ? j->pred_out + (size_t)v * npx : NULL))
            j->err = 1;
    }
    return NULL;
}

int orc_aa_silhouette_loss_grad(const float* pos, uint32_t n_verts,
                                const float* faces, uint32_t n_faces,
                                const float* vft, uint32_t max_deg,
                                uint32_t n_views, uint32_t res,
                                uint32_t n_samples, float seed,
                                const float* mvps, const float* targets,
                                uint32_t threads, double* loss, float* grad,
                                float* pred_out) {
    aa_job j;
    memset(&j, 0, sizeof(j));
    j.pos = pos;
    j.n_verts = n_verts;
    j.n_faces = n_faces;
    j.n_views = n_views;
    j.res = res;
    j.max_deg = max_deg;
    j.n_samples = n_samples;
    j.faces = faces;
    j.vft = vft;
    j.seed = seed;
    j.mvps = mvps;
    j.targets = targets;
    j.pred_out = pred_out;
    j.vloss = (double*)calloc(n_views, sizeof(double));
    j.vgrad = (float*)calloc((size_t)n_views * n_verts * 3, sizeof(float));
    if (!j.vloss || !j.vgrad) {
        free(j.vloss);
        free(j.vgrad);
        return fail("oom");
    }
    pthread_mutex_init(&j.mu, NULL);
    if (threads < 1) threads = 1;
    if (threads > n_views) threads = n_views;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * threads);
    for (uint32_t i = 1; i < threads; i++)
        pthread_create(&th[i], NULL, aa_worker, &j);
    aa_worker(&j);
    for (uint32_t i = 1; i < threads; i++) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&j.mu);
    int rc = j.err;
    if (!rc) {
        double l = 0.0;
        memset(grad, 0, sizeof(float) * n_verts * 3);
        for (uint32_t v = 0; v < n_views; v++) {
            l += j.vloss[v];
            const float* g = j.vgrad + (size_t)v * n_verts * 3;
            for (size_t i = 0; i < (size_t)n_verts * 3; i++) grad[i] += g[i];
        }
        *loss = l;
    }
    free(j.vloss);
    free(j.vgrad);
    return rc;
}

int orc_aa_silhouette_run(float* pos, uint32_t n_verts, const float* faces,
                          uint32_t n_faces, const float* vft,
                          uint32_t max_deg, uint32_t n_views, uint32_t res,
                          uint32_t n_samples, float lr, const float* mvps,
                          const float* targets, uint32_t n_iters,
                          uint32_t threads, float* loss_trace) {
    const size_t n = (size_t)n_verts * 3;
    float* m = (float*)calloc(n, sizeof(float));
    float* v = (float*)calloc(n, sizeof(float));
    float* g = (float*)calloc(n, sizeof(float));
    float t = 0.f;
    int rc = 0;
    if (!m || !v || !g) rc = fail("oom");
    for (uint32_t it = 0; it < n_iters && !rc; it++) {
        double l = 0.0;
        /* the in-graph counter (before its update) seeds the sampling */
        rc = orc_aa_silhouette_loss_grad(pos, n_verts, faces, n_faces, vft,
                                         max_deg, n_views, res, n_samples, t,
                                         mvps, targets, threads, &l, g, NULL);
        if (rc) break;
        loss_trace[it] = (float)l;
        orc_adam(pos, m, v, &t, g, (uint32_t)n, lr, 0.9f, 0.999f, 1e-8f);
    }
    free(m);
    free(v);
    free(g);
    return rc;
}

/* --------------------------------------------------------- image fitting */

/* Sum (f_ops.cpp:1037-1043, the Reduce2x2Sum chain 998-1033) followed by
 * CompSum and the Mean scale (1045-1050) */
static float mean_2x2(const float* x, uint32_t w, uint32_t h, uint32_t nc) {
    float* cur = (float*)malloc(sizeof(float) * (size_t)w * h * nc);
    memcpy(cur, x, sizeof(float) * (size_t)w * h * nc);
    uint32_t cw = w, ch = h;
    while (!(cw == 1 && ch == 1)) {
        const uint32_t nw = (cw + 1) / 2, nh = (ch + 1) / 2;
        float* nx = (float*)calloc((size_t)nw * nh * nc, sizeof(float));
        for (uint32_t py = 0; py < ch; py++)
            for (uint32_t px = 0; px < cw; px++)
                for (uint32_t c = 0; c < nc; c++)
                    nx[((size_t)(py / 2) * nw + px / 2) * nc + c] +=
                            cur[((size_t)py * cw + px) * nc + c];
        free(cur);
        cur = nx;
        cw = nw;
        ch = nh;
    }
    float acc = 0.f;
    for (uint32_t c = 0; c < nc; c++) acc += cur[c];
    free(cur);
    const float inv_n = 1.f / ((float)w * (float)h * (float)nc);
    return acc * inv_n;
}

int orc_image_fit_run(float* param, const float* target, uint32_t w,
                      uint32_t h, float lr, uint32_t n_iters,
                      float* loss_trace) {
    const size_t n = (size_t)w * h * 4;
    float* m = (float*)calloc(n, sizeof(float));
    float* v = (float*)calloc(n, sizeof(float));
    float* g = (float*)calloc(n, sizeof(float));
    float* sq = (float*)calloc(n, sizeof(float));
    if (!m || !v || !g || !sq) return fail("oom");
    const float inv_n = 1.f / ((float)w * (float)h * 4.f);
    float t = 0.f;
    for (uint32_t it = 0; it < n_iters; it++) {
        for (size_t i = 0; i < n; i++) {
            const float diff = param[i] - target[i];
            sq[i] = diff * diff;
            const float g_sq = 1.f * inv_n;
            g[i] = g_sq * diff + g_sq * diff;
        }
        loss_trace[it] = mean_2x2(sq, w, h, 4);
        orc_adam(param, m, v, &t, g, (uint32_t)n, lr, 0.9f, 0.999f, 1e-8f);
    }
    free(m);
    free(v);
    free(g);
    free(sq);
    return 0;
}

/* ---------------------------------------------------------- adjacency */

int orc_vertex_faces_tex(const float* faces, uint32_t n_faces,
                         uint32_t n_verts, uint32_t cap, float* out,
                         uint32_t* max_deg) {
    uint32_t* deg = (uint32_t*)calloc(n_verts, sizeof(uint32_t));
    if (!deg) return fail("oom");
    uint32_t md = 1;
    for (uint32_t f = 0; f < n_faces; f++)
        for (int k = 0; k < 3; k++) {
            const uint32_t v = (uint32_t)faces[(size_t)f * 3 + k];
            if (v >= n_verts) {
                free(deg);
                return fail("vertex_faces_tex: vertex index range");
            }
            deg[v]++;
            if (deg[v] > md) md = deg[v];
        }
    if (md > cap) {
        free(deg);
        return fail("vertex_faces_tex: capacity %u < max degree %u", cap, md);
    }
    for (size_t i = 0; i < (size_t)n_verts * md; i++) out[i] = -1.f;
    memset(deg, 0, sizeof(uint32_t) * n_verts);
    for (uint32_t f = 0; f < n_faces; f++)
        for (int k = 0; k < 3; k++) {
            const uint32_t v = (uint32_t)faces[(size_t)f * 3 + k];
            out[(size_t)deg[v]++ * n_verts + v] = (float)f;
        }
    *max_deg = md;
    free(deg);
    return 0;
}
