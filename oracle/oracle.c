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

/* orc_silhouette_loss_grad with the views spread over `threads` host
 * threads (the per-view results are summed in view order, as above). */
int orc_silhouette_loss_grad_mt(const float* pos, uint32_t n_verts,
                                const float* faces, uint32_t n_faces,
                                uint32_t n_views, uint32_t res, float radius,
                                float sigma, const float* mvps,
                                const float* targets, double* loss,
                                float* grad, float* rs_out,
                                uint32_t threads) {
    return sil_loss_grad_mt(pos, n_verts, faces, n_faces, n_views, res,
                            radius, sigma, mvps, targets, loss, grad, rs_out,
                            threads);
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

/* Mesh tables + scratch of the optimizer-side regulariser of the silhouette
 * runs (laplacian = normal = 0: none, the gradient passes unchanged). */
typedef struct {
    float *vn, *fa, *vf, *g2;
    uint32_t vn_deg, vf_deg;
} reg_state_t;

static void reg_free(reg_state_t* r) {
    free(r->vn);
    free(r->fa);
    free(r->vf);
    free(r->g2);
    memset(r, 0, sizeof(*r));
}

static int reg_init(reg_state_t* r, const float* faces, uint32_t n_faces,
                    uint32_t n_verts, float laplacian, float normal) {
    memset(r, 0, sizeof(*r));
    if (laplacian == 0.f && normal == 0.f) return 0;
    r->vn = (float*)malloc(sizeof(float) * (size_t)n_verts * 64);
    r->vf = (float*)malloc(sizeof(float) * (size_t)n_verts * 64);
    r->fa = (float*)malloc(sizeof(float) * (size_t)n_faces * 3);
    r->g2 = (float*)malloc(sizeof(float) * (size_t)n_verts * 3);
    if (!r->vn || !r->vf || !r->fa || !r->g2) {
        reg_free(r);
        return fail("oom");
    }
    int rc = orc_vertex_neighbors_tex(faces, n_faces, n_verts, 64, r->vn,
                                      &r->vn_deg);
    if (!rc) rc = orc_face_neighbors_tex(faces, n_faces, r->fa);
    if (!rc)
        rc = orc_vertex_faces_tex(faces, n_faces, n_verts, 64, r->vf,
                                  &r->vf_deg);
    if (rc) reg_free(r);
    return rc;
}

/* g <- the regularised gradient (run.cpp:407-420), when enabled. */
static int reg_apply(reg_state_t* r, const float* pos, uint32_t n_verts,
                     const float* faces, uint32_t n_faces, float laplacian,
                     float normal, float* g) {
    if (!r->vn) return 0;
    const int rc = orc_regularized_grad(pos, n_verts, faces, n_faces, r->vn,
                                        r->vn_deg, r->fa, r->vf, r->vf_deg, g,
                                        laplacian, normal, r->g2);
    if (!rc) memcpy(g, r->g2, sizeof(float) * (size_t)n_verts * 3);
    return rc;
}

int orc_silhouette_run(float* pos, uint32_t n_verts, const float* faces,
                       uint32_t n_faces, uint32_t n_views, uint32_t res,
                       float radius, float sigma, float lr, const float* mvps,
                       const float* targets, uint32_t n_iters,
                       uint32_t threads, float laplacian, float normal,
                       float* loss_trace) {
    const size_t n = (size_t)n_verts * 3;
    float* m = (float*)calloc(n, sizeof(float));
    float* v = (float*)calloc(n, sizeof(float));
    float* g = (float*)calloc(n, sizeof(float));
    float t = 0.f;
    reg_state_t reg;
    int rc = reg_init(&reg, faces, n_faces, n_verts, laplacian, normal);
    if (!rc && (!m || !v || !g)) rc = fail("oom");
    for (uint32_t it = 0; it < n_iters && !rc; it++) {
        double l = 0.0;
        rc = sil_loss_grad_mt(pos, n_verts, faces, n_faces, n_views, res,
                              radius, sigma, mvps, targets, &l, g, NULL,
                              threads);
        if (!rc)
            rc = reg_apply(&reg, pos, n_verts, faces, n_faces, laplacian,
                           normal, g);
        if (rc) break;
        loss_trace[it] = (float)l;
        orc_adam(pos, m, v, &t, g, (uint32_t)n, lr, 0.9f, 0.999f, 1e-8f);
    }
    reg_free(&reg);
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
                          uint32_t threads, float laplacian, float normal,
                          float* loss_trace) {
    const size_t n = (size_t)n_verts * 3;
    float* m = (float*)calloc(n, sizeof(float));
    float* v = (float*)calloc(n, sizeof(float));
    float* g = (float*)calloc(n, sizeof(float));
    float t = 0.f;
    reg_state_t reg;
    int rc = reg_init(&reg, faces, n_faces, n_verts, laplacian, normal);
    if (!rc && (!m || !v || !g)) rc = fail("oom");
    for (uint32_t it = 0; it < n_iters && !rc; it++) {
        double l = 0.0;
        /* the in-graph counter (before its update) seeds the sampling */
        rc = orc_aa_silhouette_loss_grad(pos, n_verts, faces, n_faces, vft,
                                         max_deg, n_views, res, n_samples, t,
                                         mvps, targets, threads, &l, g, NULL);
        if (!rc)
            rc = reg_apply(&reg, pos, n_verts, faces, n_faces, laplacian,
                           normal, g);
        if (rc) break;
        loss_trace[it] = (float)l;
        orc_adam(pos, m, v, &t, g, (uint32_t)n, lr, 0.9f, 0.999f, 1e-8f);
    }
    reg_free(&reg);
    free(m);
    free(v);
    free(g);
    return rc;
}

/* ---------------------------------------------------------- texturing */

static inline int iclamp(int x, int lo, int hi) {
    return x < lo ? lo : (x > hi ? hi : x);
}

/* BilerpClamp (ibl_math.h:91-115): 4-tap, clamp-to-edge */
static void bilerp_clamp(const float* data, uint32_t w, uint32_t h,
                         uint32_t n, float u, float v, float* out) {
    const float sx = u * (float)w - 0.5f;
    const float sy = v * (float)h - 0.5f;
    const int ix = to_i32(floorf(sx));
    const int iy = to_i32(floorf(sy));
    const float fx = sx - (float)ix;
    const float fy = sy - (float)iy;
    for (uint32_t c = 0; c < n; c++) out[c] = 0.f;
    for (int dy = 0; dy <= 1; dy++) {
        for (int dx = 0; dx <= 1; dx++) {
            const int x = iclamp(ix + dx, 0, (int)w - 1);
            const int y = iclamp(iy + dy, 0, (int)h - 1);
            const float wgt = (dx == 0 ? 1.f - fx : fx) * (dy == 0 ? 1.f - fy : fy);
            const float* p = data + ((size_t)y * w + (size_t)x) * n;
            for (uint32_t c = 0; c < n; c++) out[c] += wgt * p[c];
        }
    }
}

int orc_texture_bilinear(const float* tex, uint32_t tw, uint32_t th,
                         uint32_t n, const float* uv, uint32_t npx,
                         float* out) {
    if (n < 1 || n > 4) return fail("texture: n_comp 1..4");
    for (uint32_t p = 0; p < npx; p++)
        bilerp_clamp(tex, tw, th, n, uv[(size_t)p * 2], uv[(size_t)p * 2 + 1],
                     out + (size_t)p * n);
    return 0;
}

/* The inverse-UV anchor of texel (tx, ty): its table entry, else the first
 * valid entry of the 9x9 neighbourhood in row order (f_ops.cpp:2681-2702;
 * glsl_codegen.cpp:674-690). Returns 0 when none is valid. */
static int inv_uv_anchor(const float* iv_t, int tw, int th, int tx, int ty,
                         float iv[4]) {
    const float* iv0 = &iv_t[((size_t)ty * tw + tx) * 4];
    for (int k = 0; k < 4; k++) iv[k] = iv0[k];
    for (int ny = -4; ny <= 4 && iv[2] < 0.5f; ny++) {
        for (int nx = -4; nx <= 4; nx++) {
            const int px = tx + nx, py = ty + ny;
            if (px < 0 || py < 0 || px >= tw || py >= th) continue;
            const float* q = &iv_t[((size_t)py * tw + px) * 4];
            for (int k = 0; k < 4; k++) iv[k] = q[k];
            if (iv[2] > 0.5f) break;
        }
    }
    return iv[2] > 0.5f;
}

/* GatherByInverseUVBilinear (f_ops.cpp:2650-2732) */
int orc_gather_inv_uv_bilinear(const float* gy, uint32_t sw, uint32_t sh,
                               uint32_t n, const float* inv_uv, uint32_t tw,
                               uint32_t th, const float* uv_screen,
                               float* out) {
    if (n < 1 || n > 4) return fail("gather: n_comp 1..4");
    memset(out, 0, sizeof(float) * (size_t)tw * th * n);
    for (int ty = 0; ty < (int)th; ty++) {
        for (int tx = 0; tx < (int)tw; tx++) {
            float iv[4];
            if (!inv_uv_anchor(inv_uv, (int)tw, (int)th, tx, ty, iv)) continue;
            const int scx = to_i32(iv[0]), scy = to_i32(iv[1]);
            float* o = &out[((size_t)ty * tw + tx) * n];
            for (int dy = -3; dy <= 3; dy++) {
                for (int dx = -3; dx <= 3; dx++) {
                    const int spx = scx + dx, spy = scy + dy;
                    if (spx < 0 || spy < 0 || spx >= (int)sw || spy >= (int)sh)
                        continue;
                    const float* suv = &uv_screen[((size_t)spy * sw + spx) * 2];
                    const float stx = suv[0] * (float)tw - 0.5f;
                    const float sty = suv[1] * (float)th - 0.5f;
                    const float w = smax(0.f, 1.f - fabsf(stx - (float)tx)) *
                                    smax(0.f, 1.f - fabsf(sty - (float)ty));
                    if (w > 0.f) {
                        const float* g = &gy[((size_t)spy * sw + spx) * n];
                        for (uint32_t c = 0; c < n; c++) o[c] += g[c] * w;
                    }
                }
            }
        }
    }
    return 0;
}

/* Nearest texture() of a clamp-to-edge nearest sampler (the reference's
 * Texture on its Vulkan path, f_ops.cpp:2605-2639, executor.cpp:193-202):
 * texel (clamp(floor(u*W)), clamp(floor(v*H))). Restated from the GLSL /
 * Vulkan sampling rules; the reference has no CPU kernel for it. */
int orc_texture_nearest(const float* tex, uint32_t tw, uint32_t th,
                        uint32_t n, const float* uv, uint32_t npx,
                        float* out) {
    if (n < 1 || n > 4) return fail("texture: n_comp 1..4");
    for (uint32_t p = 0; p < npx; p++) {
        const int x = iclamp(to_i32(floorf(uv[(size_t)p * 2] * (float)tw)), 0,
                             (int)tw - 1);
        const int y = iclamp(to_i32(floorf(uv[(size_t)p * 2 + 1] * (float)th)),
                             0, (int)th - 1);
        const float* q = tex + ((size_t)y * tw + x) * n;
        for (uint32_t c = 0; c < n; c++) out[(size_t)p * n + c] = q[c];
    }
    return 0;
}

/* GatherByInverseUV, restated from its GLSL (glsl_codegen.cpp:658-709):
 * the gradient of the first screen pixel of the anchor's 7x7 window (row
 * order) whose uv truncates to this texel. */
int orc_gather_inv_uv(const float* gy, uint32_t sw, uint32_t sh, uint32_t n,
                      const float* inv_uv, uint32_t tw, uint32_t th,
                      const float* uv_screen, float* out) {
    if (n < 1 || n > 4) return fail("gather: n_comp 1..4");
    memset(out, 0, sizeof(float) * (size_t)tw * th * n);
    for (int ty = 0; ty < (int)th; ty++) {
        for (int tx = 0; tx < (int)tw; tx++) {
            float iv[4];
            if (!inv_uv_anchor(inv_uv, (int)tw, (int)th, tx, ty, iv)) continue;
            const int scx = to_i32(iv[0]), scy = to_i32(iv[1]);
            float* o = &out[((size_t)ty * tw + tx) * n];
            int found = 0;
            for (int dy = -3; dy <= 3 && !found; dy++) {
                for (int dx = -3; dx <= 3; dx++) {
                    const int spx = scx + dx, spy = scy + dy;
                    if (spx < 0 || spy < 0 || spx >= (int)sw || spy >= (int)sh)
                        continue;
                    const float* suv = &uv_screen[((size_t)spy * sw + spx) * 2];
                    const int stx = to_i32(suv[0] * (float)tw);
                    const int sty = to_i32(suv[1] * (float)th);
                    if (stx == tx && sty == ty) {
                        const float* g = &gy[((size_t)spy * sw + spx) * n];
                        for (uint32_t c = 0; c < n; c++) o[c] = g[c];
                        found = 1;
                        break;
                    }
                }
            }
        }
    }
    return 0;
}

/* UvAsClip / ScreenAttr (mesh_utils.cpp:180-203): the inverse-UV table is
 * Rasterize(UvAsClip(uv), ScreenAttr(clip), faces, tex_size). */
void orc_uv_as_clip(const float* uv, uint32_t n_verts, float* out) {
    for (uint32_t i = 0; i < n_verts; i++) {
        out[i * 4 + 0] = uv[i * 2 + 0] * 2.f - 1.f;
        out[i * 4 + 1] = uv[i * 2 + 1] * 2.f - 1.f;
        out[i * 4 + 2] = 0.5f;
        out[i * 4 + 3] = 1.f;
    }
}

void orc_screen_attr(const float* clip, uint32_t n_verts, uint32_t sw,
                     uint32_t sh, float* out) {
    for (uint32_t i = 0; i < n_verts; i++) {
        const float w = clip[i * 4 + 3];
        const float ndc_x = clip[i * 4 + 0] / w;
        const float ndc_y = clip[i * 4 + 1] / w;
        out[i * 4 + 0] = (ndc_x * 0.5f + 0.5f) * (float)sw;
        out[i * 4 + 1] = (ndc_y * 0.5f + 0.5f) * (float)sh;
        out[i * 4 + 2] = 1.f;
        out[i * 4 + 3] = 0.f;
    }
}

/* ---- C2: mip pyramid, trilinear sampling, exact transpose -------------
 * No reference implementation (the reference samples one level); defined
 * here from first principles and documented as such:
 *  - level l+1 texel = 0.25 * (((a + b) + c) + d) of its 2x2 children
 *    (row-major order), square power-of-two textures;
 *  - per pixel, rho = max(|d uv/dx|, |d uv/dy|) in level-0 texels from the
 *    G-buffer's forward differences (backward at the right / bottom edge or
 *    next to background; 0 when neither neighbour is covered);
 *  - lod = e + (m - 1) for rho = m * 2^e, m in [1, 2) (piecewise-linear
 *    log2, exact in float), clamped to [0, levels - 1];
 *  - trilinear = (1 - f) * bilerp(level l) + f * bilerp(level l + 1). */

static inline size_t mip_offset(uint32_t w, uint32_t level, uint32_t n) {
    size_t off = 0;
    for (uint32_t l = 0; l < level; l++) {
        const size_t s = w >> l;
        off += s * s * n;
    }
    return off;
}

int orc_mip_build(const float* tex0, uint32_t w, uint32_t n, uint32_t levels,
                  float* pyr) {
    if ((w & (w - 1)) || (w >> (levels - 1)) < 1) return fail("mip: size");
    memcpy(pyr, tex0, sizeof(float) * (size_t)w * w * n);
    for (uint32_t l = 0; l + 1 < levels; l++) {
        const uint32_t s = w >> l, t = s >> 1;
        const float* src = pyr + mip_offset(w, l, n);
        float* dst = pyr + mip_offset(w, l + 1, n);
        for (uint32_t y = 0; y < t; y++)
            for (uint32_t x = 0; x < t; x++)
                for (uint32_t c = 0; c < n; c++) {
                    const float a = src[((size_t)(2 * y) * s + 2 * x) * n + c];
                    const float b = src[((size_t)(2 * y) * s + 2 * x + 1) * n + c];
                    const float cc = src[((size_t)(2 * y + 1) * s + 2 * x) * n + c];
                    const float d = src[((size_t)(2 * y + 1) * s + 2 * x + 1) * n + c];
                    dst[((size_t)y * t + x) * n + c] = 0.25f * (((a + b) + cc) + d);
                }
    }
    return 0;
}

/* lod of a pixel from its level-0 footprint rho (texels per pixel) */
static inline float lod_of(float rho, uint32_t levels) {
    if (!(rho > 1.f)) return 0.f;
    int e;
    const float m2 = frexpf(rho, &e);      /* rho = m2 * 2^e, m2 in [0.5,1) */
    const float lod = (float)(e - 1) + (m2 * 2.f - 1.f);
    const float top = (float)(levels - 1);
    return lod < top ? lod : top;
}

/* rho of pixel (x, y): uv [H][W][2], mask [H][W] (>0.5 covered), w_tex =
 * level-0 size */
static float pixel_rho(const float* uv, const float* mask, int W, int H,
                       int x, int y, float w_tex) {
    float du[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int axis = 0; axis < 2; axis++) {
        const int ax = axis == 0 ? 1 : 0, ay = axis == 0 ? 0 : 1;
        const int x1 = x + ax, y1 = y + ay, x0 = x - ax, y0 = y - ay;
        const float* c = &uv[((size_t)y * W + x) * 2];
        if (x1 < W && y1 < H && mask[(size_t)y1 * W + x1] > 0.5f) {
            const float* q = &uv[((size_t)y1 * W + x1) * 2];
            du[axis][0] = q[0] - c[0];
            du[axis][1] = q[1] - c[1];
        } else if (x0 >= 0 && y0 >= 0 && mask[(size_t)y0 * W + x0] > 0.5f) {
            const float* q = &uv[((size_t)y0 * W + x0) * 2];
            du[axis][0] = c[0] - q[0];
            du[axis][1] = c[1] - q[1];
        }
    }
    const float ax_ = du[0][0] * w_tex, ay_ = du[0][1] * w_tex;
    const float bx_ = du[1][0] * w_tex, by_ = du[1][1] * w_tex;
    const float rx = sqrtf(ax_ * ax_ + ay_ * ay_);
    const float ry = sqrtf(bx_ * bx_ + by_ * by_);
    return smax(rx, ry);
}

int orc_texture_lod(const float* uv, const float* mask, uint32_t W,
                    uint32_t H, uint32_t w_tex, uint32_t levels, float* lod) {
    for (int y = 0; y < (int)H; y++)
        for (int x = 0; x < (int)W; x++)
            lod[(size_t)y * W + x] =
                    mask[(size_t)y * W + x] > 0.5f
                            ? lod_of(pixel_rho(uv, mask, (int)W, (int)H, x, y,
                                               (float)w_tex), levels)
                            : 0.f;
    return 0;
}

int orc_texture_trilinear(const float* pyr, uint32_t w, uint32_t n,
                          uint32_t levels, const float* uv, const float* lod,
                          uint32_t npx, float* out) {
    float s0[4], s1[4];
    for (uint32_t p = 0; p < npx; p++) {
        const float l = lod[p];
        const int l0 = to_i32(floorf(l));
        const float f = l - (float)l0;
        const float u = uv[(size_t)p * 2], v = uv[(size_t)p * 2 + 1];
        const uint32_t s = w >> l0;
        bilerp_clamp(pyr + mip_offset(w, (uint32_t)l0, n), s, s, n, u, v, s0);
        float* o = out + (size_t)p * n;
        if (f > 0.f && (uint32_t)l0 + 1 < levels) {
            bilerp_clamp(pyr + mip_offset(w, (uint32_t)l0 + 1, n), s >> 1,
                         s >> 1, n, u, v, s1);
            for (uint32_t c = 0; c < n; c++) o[c] = s0[c] * (1.f - f) + s1[c] * f;
        } else {
            for (uint32_t c = 0; c < n; c++) o[c] = s0[c];
        }
    }
    return 0;
}

/* The bilinear taps of (u, v) on an s x s level: texel indices + weights */
static void bilerp_taps(uint32_t s, float u, float v, int tx[4], int ty[4],
                        float tw_[4]) {
    const float sx = u * (float)s - 0.5f;
    const float sy = v * (float)s - 0.5f;
    const int ix = to_i32(floorf(sx));
    const int iy = to_i32(floorf(sy));
    const float fx = sx - (float)ix;
    const float fy = sy - (float)iy;
    int k = 0;
    for (int dy = 0; dy <= 1; dy++)
        for (int dx = 0; dx <= 1; dx++, k++) {
            tx[k] = iclamp(ix + dx, 0, (int)s - 1);
            ty[k] = iclamp(iy + dy, 0, (int)s - 1);
            tw_[k] = (dx == 0 ? 1.f - fx : fx) * (dy == 0 ? 1.f - fy : fy);
        }
}

/* Exact transpose of orc_texture_trilinear: adds g [npx][n] into the
 * pyramid gradient gpyr. */
int orc_texture_trilinear_grad(const float* g, uint32_t w, uint32_t n,
                               uint32_t levels, const float* uv,
                               const float* lod, uint32_t npx, float* gpyr) {
    for (uint32_t p = 0; p < npx; p++) {
        const float l = lod[p];
        const int l0 = to_i32(floorf(l));
        const float f = l - (float)l0;
        const float u = uv[(size_t)p * 2], v = uv[(size_t)p * 2 + 1];
        const int two = f > 0.f && (uint32_t)l0 + 1 < levels;
        for (int lv = 0; lv < 1 + two; lv++) {
            const uint32_t level = (uint32_t)l0 + (uint32_t)lv;
            const float lw = two ? (lv == 0 ? 1.f - f : f) : 1.f;
            const uint32_t s = w >> level;
            int tx[4], ty[4];
            float wt[4];
            bilerp_taps(s, u, v, tx, ty, wt);
            float* gl = gpyr + mip_offset(w, level, n);
            for (int k = 0; k < 4; k++)
                for (uint32_t c = 0; c < n; c++)
                    gl[((size_t)ty[k] * s + tx[k]) * n + c] +=
                            g[(size_t)p * n + c] * lw * wt[k];
        }
    }
    return 0;
}

/* Transpose of orc_mip_build: level l texel += 0.25 * its parent's
 * gradient, from the top level down; gpyr level 0 then holds d/d tex0. */
void orc_mip_fold(float* gpyr, uint32_t w, uint32_t n, uint32_t levels) {
    for (int l = (int)levels - 2; l >= 0; l--) {
        const uint32_t s = w >> l, t = s >> 1;
        float* dst = gpyr + mip_offset(w, (uint32_t)l, n);
        const float* src = gpyr + mip_offset(w, (uint32_t)l + 1, n);
        for (uint32_t y = 0; y < s; y++)
            for (uint32_t x = 0; x < s; x++)
                for (uint32_t c = 0; c < n; c++)
                    dst[((size_t)y * s + x) * n + c] +=
                            0.25f * src[((size_t)(y / 2) * t + x / 2) * n + c];
    }
}

size_t orc_mip_floats(uint32_t w, uint32_t n, uint32_t levels) {
    return mip_offset(w, levels, n);
}

/* One C2 iteration (first principles on the reference's graph shape,
 * examples/texture_optimization/run.cpp:115-126 with trilinear sampling):
 * per view, G-buffer (uv, mask) = Rasterize(clip, (u, v, 1)); pred = mask *
 * trilinear(mips(tex), uv); loss_v = Mean((target - pred)^2) over W*H*3;
 * loss = sum_v loss_v; grad = d loss / d tex (level 0). gbuf (nullable)
 * [views][R][R][3] receives the G-buffers, pred_out (nullable) the
 * predictions. */
int orc_c2_loss_grad(const float* tex, uint32_t w_tex, uint32_t levels,
                     const float* pos, const float* uv_v, uint32_t n_verts,
                     const float* faces, uint32_t n_faces, const float* mvps,
                     uint32_t n_views, uint32_t res, const float* targets,
                     double* loss, float* grad, float* pred_out) {
    const uint32_t n = 3;
    const size_t npx = (size_t)res * res;
    const size_t nmip = orc_mip_floats(w_tex, n, levels);
    float* pyr = (float*)malloc(sizeof(float) * nmip);
    float* gpyr = (float*)calloc(nmip, sizeof(float));
    float* clip = (float*)malloc(sizeof(float) * n_verts * 4);
    float* attr = (float*)malloc(sizeof(float) * n_verts * 3);
    float* gb = (float*)malloc(sizeof(float) * npx * 3);
    float* uv = (float*)malloc(sizeof(float) * npx * 2);
    float* mask = (float*)malloc(sizeof(float) * npx);
    float* lod = (float*)malloc(sizeof(float) * npx);
    float* smp = (float*)malloc(sizeof(float) * npx * n);
    float* g = (float*)malloc(sizeof(float) * npx * n);
    int rc = 1;
    if (!pyr || !gpyr || !clip || !attr || !gb || !uv || !mask || !lod ||
        !smp || !g) {
        fail("oom");
        goto done;
    }
    orc_mip_build(tex, w_tex, n, levels, pyr);
    for (uint32_t i = 0; i < n_verts; i++) {
        attr[i * 3 + 0] = uv_v[i * 2 + 0];
        attr[i * 3 + 1] = uv_v[i * 2 + 1];
        attr[i * 3 + 2] = 1.f;
    }
    const float inv_n = 1.f / ((float)res * (float)res * (float)n);
    double l = 0.0;
    for (uint32_t v = 0; v < n_views; v++) {
        orc_transform_clip(pos, n_verts, mvps + (size_t)v * 16, clip);
        if (orc_rasterize_hard(clip, n_verts, attr, 3, faces, n_faces, res, res,
                               gb))
            goto done;
        for (size_t i = 0; i < npx; i++) {
            uv[i * 2] = gb[i * 3];
            uv[i * 2 + 1] = gb[i * 3 + 1];
            mask[i] = gb[i * 3 + 2];
        }
        orc_texture_lod(uv, mask, res, res, w_tex, levels, lod);
        orc_texture_trilinear(pyr, w_tex, n, levels, uv, lod, (uint32_t)npx, smp);
        const float* t = targets + (size_t)v * npx * n;
        for (size_t i = 0; i < npx; i++) {
            for (uint32_t c = 0; c < n; c++) {
                const float pred = mask[i] * smp[i * n + c];
                if (pred_out) pred_out[((size_t)v * npx + i) * n + c] = pred;
                const float diff = t[i * n + c] - pred;
                l += (double)(diff * diff * inv_n);
                const float g_m = 1.f * inv_n;
                const float g_pred = -(g_m * diff + g_m * diff);
                g[i * n + c] = g_pred * mask[i];
            }
        }
        orc_texture_trilinear_grad(g, w_tex, n, levels, uv, lod, (uint32_t)npx,
                                   gpyr);
    }
    orc_mip_fold(gpyr, w_tex, n, levels);
    memcpy(grad, gpyr, sizeof(float) * (size_t)w_tex * w_tex * n);
    *loss = l;
    rc = 0;
done:
    free(pyr);
    free(gpyr);
    free(clip);
    free(attr);
    free(gb);
    free(uv);
    free(mask);
    free(lod);
    free(smp);
    free(g);
    return rc;
}

int orc_c2_run(float* tex, uint32_t w_tex, uint32_t levels, const float* pos,
               const float* uv_v, uint32_t n_verts, const float* faces,
               uint32_t n_faces, const float* mvps, uint32_t n_views,
               uint32_t res, const float* targets, float lr, uint32_t n_iters,
               float* loss_trace) {
    const size_t nt = (size_t)w_tex * w_tex * 3;
    float* m = (float*)calloc(nt, sizeof(float));
    float* v = (float*)calloc(nt, sizeof(float));
    float* g = (float*)calloc(nt, sizeof(float));
    float t = 0.f;
    int rc = (!m || !v || !g) ? fail("oom") : 0;
    for (uint32_t it = 0; it < n_iters && !rc; it++) {
        double l = 0.0;
        rc = orc_c2_loss_grad(tex, w_tex, levels, pos, uv_v, n_verts, faces,
                              n_faces, mvps, n_views, res, targets, &l, g,
                              NULL);
        if (rc) break;
        loss_trace[it] = (float)l;
        orc_adam(tex, m, v, &t, g, (uint32_t)nt, lr, 0.9f, 0.999f, 1e-8f);
    }
    free(m);
    free(v);
    free(g);
    return rc;
}

/* ------------------------------------------------------- regularisers */

static int cmp_u32(const void* a, const void* b) {
    const uint32_t x = *(const uint32_t*)a, y = *(const uint32_t*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/* VertexNeighborsTex (mesh_utils.cpp:10-28, 73-86): sorted neighbour sets,
 * {V, max_deg} row d at out[d*V], -1 padding. */
int orc_vertex_neighbors_tex(const float* faces, uint32_t n_faces,
                             uint32_t n_verts, uint32_t cap, float* out,
                             uint32_t* max_deg) {
    uint32_t* lst = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)n_verts * 64);
    uint32_t* cnt = (uint32_t*)calloc(n_verts, sizeof(uint32_t));
    if (!lst || !cnt) {
        free(lst);
        free(cnt);
        return fail("oom");
    }
    int rc = 0;
    for (uint32_t f = 0; f < n_faces && !rc; f++) {
        uint32_t idx[3];
        for (int k = 0; k < 3; k++) idx[k] = (uint32_t)faces[(size_t)f * 3 + k];
        for (int k = 0; k < 3 && !rc; k++) {
            const uint32_t v = idx[k];
            if (v >= n_verts) { rc = fail("neighbors: vertex index"); break; }
            const uint32_t nb[2] = {idx[(k + 1) % 3], idx[(k + 2) % 3]};
            for (int j = 0; j < 2; j++) {
                int seen = 0;
                for (uint32_t i = 0; i < cnt[v]; i++)
                    if (lst[(size_t)v * 64 + i] == nb[j]) seen = 1;
                if (!seen) {
                    if (cnt[v] >= 64) { rc = fail("neighbors: degree > 64"); break; }
                    lst[(size_t)v * 64 + cnt[v]++] = nb[j];
                }
            }
        }
    }
    uint32_t md = 1;
    for (uint32_t v = 0; v < n_verts && !rc; v++) {
        qsort(&lst[(size_t)v * 64], cnt[v], sizeof(uint32_t), cmp_u32);
        if (cnt[v] > md) md = cnt[v];
    }
    if (!rc && md > cap) rc = fail("neighbors: capacity %u < %u", cap, md);
    if (!rc) {
        for (size_t i = 0; i < (size_t)n_verts * md; i++) out[i] = -1.f;
        for (uint32_t v = 0; v < n_verts; v++)
            for (uint32_t d = 0; d < cnt[v]; d++)
                out[(size_t)d * n_verts + v] = (float)lst[(size_t)v * 64 + d];
        *max_deg = md;
    }
    free(lst);
    free(cnt);
    return rc;
}

typedef struct {
    uint32_t a, b, f;
} edge_face_t;

static int cmp_edge_face(const void* x, const void* y) {
    const edge_face_t* p = (const edge_face_t*)x;
    const edge_face_t* q = (const edge_face_t*)y;
    if (p->a != q->a) return p->a < q->a ? -1 : 1;
    if (p->b != q->b) return p->b < q->b ? -1 : 1;
    return p->f < q->f ? -1 : (p->f > q->f ? 1 : 0);  /* insertion order */
}

/* FaceNeighborsTex (mesh_utils.cpp:30-52, 88-101): for each edge (ordered
 * by (min, max) vertex) every pair of its faces, in face order; each face
 * keeps its first 3 neighbours. out [F][3], -1 padding. */
int orc_face_neighbors_tex(const float* faces, uint32_t n_faces, float* out) {
    edge_face_t* e = (edge_face_t*)malloc(sizeof(edge_face_t) * (size_t)n_faces * 3);
    uint32_t* n_adj = (uint32_t*)calloc(n_faces, sizeof(uint32_t));
    if (!e || !n_adj) {
        free(e);
        free(n_adj);
        return fail("oom");
    }
    for (uint32_t f = 0; f < n_faces; f++)
        for (int k = 0; k < 3; k++) {
            const uint32_t a = (uint32_t)faces[(size_t)f * 3 + k];
            const uint32_t b = (uint32_t)faces[(size_t)f * 3 + (k + 1) % 3];
            edge_face_t* t = &e[(size_t)f * 3 + k];
            t->a = a < b ? a : b;
            t->b = a < b ? b : a;
            t->f = f;
        }
    qsort(e, (size_t)n_faces * 3, sizeof(edge_face_t), cmp_edge_face);
    for (size_t i = 0; i < (size_t)n_faces * 3; i++) out[i] = -1.f;
    size_t i = 0;
    while (i < (size_t)n_faces * 3) {
        size_t j = i;
        while (j < (size_t)n_faces * 3 && e[j].a == e[i].a && e[j].b == e[i].b) j++;
        for (size_t x = i; x < j; x++)
            for (size_t y = x + 1; y < j; y++) {
                const uint32_t pr[2] = {e[x].f, e[y].f};
                for (int s = 0; s < 2; s++) {
                    const uint32_t f = pr[s], g = pr[1 - s];
                    if (n_adj[f] < 3) out[(size_t)f * 3 + n_adj[f]++] = (float)g;
                }
            }
        i = j;
    }
    free(e);
    free(n_adj);
    return 0;
}

static void cross_of_face(const float* pos, const float* faces, uint32_t f,
                          uint32_t idx[3], float c[3]) {
    for (int k = 0; k < 3; k++)
        idx[k] = to_u32_via_i64(faces[(size_t)f * 3 + k] + 0.5f);
    const float* p0 = &pos[(size_t)idx[0] * 3];
    const float* p1 = &pos[(size_t)idx[1] * 3];
    const float* p2 = &pos[(size_t)idx[2] * 3];
    const float e1[3] = {p1[0] - p0[0], p1[1] - p0[1], p1[2] - p0[2]};
    const float e2[3] = {p2[0] - p0[0], p2[1] - p0[1], p2[2] - p0[2]};
    c[0] = e1[1] * e2[2] - e1[2] * e2[1];
    c[1] = e1[2] * e2[0] - e1[0] * e2[2];
    c[2] = e1[0] * e2[1] - e1[1] * e2[0];
}

/* SumAll over n floats (f_ops.cpp:1119-1149 with SumPartial 1087-1115):
 * above 256 elements, 64 strided partial sums in double (each rounded to
 * float), then their double sum rounded to float. `elems` is the pixel
 * count, `n` the components per pixel. */
static float sum_all(const float* x, size_t elems, uint32_t n) {
    if (elems <= 256) {
        double s = 0.0;
        for (size_t i = 0; i < elems * n; i++) s += x[i];
        return (float)s;
    }
    double s = 0.0;
    for (uint32_t p = 0; p < 64; p++) {
        double q = 0.0;
        for (size_t i = p; i < elems; i += 64)
            for (uint32_t c = 0; c < n; c++) q += x[i * n + c];
        s += (double)(float)q;
    }
    return (float)s;
}

/* rms(x) = sqrt(SumAll(x * x) * inv_cnt + 1e-24) (run.cpp:410-413) */
static float reg_rms(const float* x, uint32_t n_verts, float* tmp) {
    const float inv_cnt = 1.f / (float)(n_verts * 3);
    for (size_t i = 0; i < (size_t)n_verts * 3; i++) tmp[i] = x[i] * x[i];
    return sqrtf(sum_all(tmp, n_verts, 3) * inv_cnt + 1e-24f);
}

/* VertexNeighborMean (f_ops.cpp:1983-2029): the mean of the listed
 * neighbours in table order; pos itself without neighbours. */
void orc_vertex_neighbor_mean(const float* pos, uint32_t n_verts,
                              const float* vnbrs, uint32_t nbr_deg,
                              float* out) {
    for (uint32_t v = 0; v < n_verts; v++) {
        float mean[3] = {0.f, 0.f, 0.f};
        uint32_t count = 0;
        for (uint32_t d = 0; d < nbr_deg; d++) {
            const float nv = vnbrs[(size_t)d * n_verts + v];
            if (nv < -0.5f) continue;
            const size_t nb = (size_t)to_u32_via_i64(nv + 0.5f);
            for (int c = 0; c < 3; c++) mean[c] += pos[nb * 3 + c];
            count++;
        }
        for (int c = 0; c < 3; c++)
            out[(size_t)v * 3 + c] =
                    count > 0 ? mean[c] / (float)count : pos[(size_t)v * 3 + c];
    }
}

/* NormalConsistencyFaceTerm (f_ops.cpp:2031-2098): per face a (skipped
 * when |c_a| < 1e-12), the sum over its edge neighbours b (|c_b| >= 1e-12)
 * of -(n_b - (n_a . n_b) n_a) / |c_a|. */
void orc_nc_face_term(const float* pos, const float* faces, uint32_t n_faces,
                      const float* fadj, float* term) {
    for (uint32_t f = 0; f < n_faces; f++) {
        uint32_t ia[3];
        float ca[3];
        float gg[3] = {0.f, 0.f, 0.f};
        cross_of_face(pos, faces, f, ia, ca);
        const float la = sqrtf(ca[0] * ca[0] + ca[1] * ca[1] + ca[2] * ca[2]);
        if (la >= 1e-12f) {
            const float na[3] = {ca[0] / la, ca[1] / la, ca[2] / la};
            for (int j = 0; j < 3; j++) {
                const float gv = fadj[(size_t)f * 3 + j];
                if (gv < -0.5f) continue;
                uint32_t ib[3];
                float cb[3];
                cross_of_face(pos, faces, to_u32_via_i64(gv + 0.5f), ib, cb);
                const float lb =
                        sqrtf(cb[0] * cb[0] + cb[1] * cb[1] + cb[2] * cb[2]);
                if (lb < 1e-12f) continue;
                const float nb[3] = {cb[0] / lb, cb[1] / lb, cb[2] / lb};
                const float d = na[0] * nb[0] + na[1] * nb[1] + na[2] * nb[2];
                for (int c = 0; c < 3; c++) gg[c] += -(nb[c] - d * na[c]) / la;
            }
        }
        for (int c = 0; c < 3; c++) term[(size_t)f * 3 + c] = gg[c];
    }
}

/* NormalConsistencyVertexGrad (f_ops.cpp:2100-2181): per vertex over its
 * incident faces in table order, the transpose of the cross product
 * c = e1 x e2 applied to the face term. */
void orc_nc_vertex_grad(const float* term, const float* pos, uint32_t n_verts,
                        const float* faces, const float* vft,
                        uint32_t vft_deg, float* out) {
    for (uint32_t v = 0; v < n_verts; v++) {
        float acc[3] = {0.f, 0.f, 0.f};
        for (uint32_t d = 0; d < vft_deg; d++) {
            const float fv = vft[(size_t)d * n_verts + v];
            if (fv < -0.5f) continue;
            const uint32_t f = to_u32_via_i64(fv + 0.5f);
            uint32_t idx[3];
            for (int k = 0; k < 3; k++)
                idx[k] = to_u32_via_i64(faces[(size_t)f * 3 + k] + 0.5f);
            const float* p0 = &pos[(size_t)idx[0] * 3];
            const float* p1 = &pos[(size_t)idx[1] * 3];
            const float* p2 = &pos[(size_t)idx[2] * 3];
            const float e1[3] = {p1[0] - p0[0], p1[1] - p0[1], p1[2] - p0[2]};
            const float e2[3] = {p2[0] - p0[0], p2[1] - p0[1], p2[2] - p0[2]};
            const float* t = &term[(size_t)f * 3];
            const float g1[3] = {e2[1] * t[2] - e2[2] * t[1],
                                 e2[2] * t[0] - e2[0] * t[2],
                                 e2[0] * t[1] - e2[1] * t[0]};
            const float g2[3] = {t[1] * e1[2] - t[2] * e1[1],
                                 t[2] * e1[0] - t[0] * e1[2],
                                 t[0] * e1[1] - t[1] * e1[0]};
            for (int c = 0; c < 3; c++) {
                if (idx[1] == v) acc[c] += g1[c];
                if (idx[2] == v) acc[c] += g2[c];
                if (idx[0] == v) acc[c] -= g1[c] + g2[c];
            }
        }
        for (int c = 0; c < 3; c++) out[(size_t)v * 3 + c] = acc[c];
    }
}

float orc_sum_all(const float* x, size_t n_px, uint32_t n_comp) {
    return sum_all(x, n_px, n_comp);
}

/* The regularised gradient of the reference's silhouette optimizer
 * (examples/silhouette_optimization/run.cpp:407-420): g + g_lap *
 * (rms(g) / rms(g_lap) * laplacian) + g_nrm * (rms(g) / rms(g_nrm) *
 * normal), g_lap = pos - VertexNeighborMean(pos), g_nrm =
 * NormalConsistencyVertexGrad(NormalConsistencyFaceTerm(pos)).
 * vnbrs {V,nbr_deg}, fadj [F][3], vft {V,vft_deg}. */
int orc_regularized_grad(const float* pos, uint32_t n_verts, const float* faces,
                         uint32_t n_faces, const float* vnbrs, uint32_t nbr_deg,
                         const float* fadj, const float* vft, uint32_t vft_deg,
                         const float* g, float laplacian, float normal,
                         float* out) {
    const size_t n3 = (size_t)n_verts * 3;
    float* glap = (float*)malloc(sizeof(float) * n3);
    float* gnrm = (float*)malloc(sizeof(float) * n3);
    float* term = (float*)malloc(sizeof(float) * (size_t)n_faces * 3);
    float* tmp = (float*)malloc(sizeof(float) * n3);
    if (!glap || !gnrm || !term || !tmp) {
        free(glap); free(gnrm); free(term); free(tmp);
        return fail("oom");
    }
    orc_vertex_neighbor_mean(pos, n_verts, vnbrs, nbr_deg, glap);
    for (size_t i = 0; i < n3; i++) glap[i] = pos[i] - glap[i];
    orc_nc_face_term(pos, faces, n_faces, fadj, term);
    orc_nc_vertex_grad(term, pos, n_verts, faces, vft, vft_deg, gnrm);
    const float data_rms = reg_rms(g, n_verts, tmp);
    const float s_lap = data_rms / reg_rms(glap, n_verts, tmp) * laplacian;
    const float s_nrm = data_rms / reg_rms(gnrm, n_verts, tmp) * normal;
    for (size_t i = 0; i < n3; i++)
        out[i] = (g[i] + glap[i] * s_lap) + gnrm[i] * s_nrm;
    free(glap);
    free(gnrm);
    free(term);
    free(tmp);
    return 0;
}

/* ------------------------------------------------ split-sum IBL (C5) */

/* Constants of src/core/ibl_math.h:16-19 (float literals). */
#define IBL_PI 3.14159265358979323846f
#define IBL_TWO_PI 6.28318530717958647692f
#define IBL_INV_PI 0.31830988618379067154f
#define IBL_INV_TWO_PI 0.15915494309189533577f

static inline float dot3(const float a[3], const float b[3]) {
    return a[0] * b[0] + a[1] * b[1] + a[2] * b[2];
}

/* EquirectUvFromDir (ibl_math.h:39-44): u wraps at the atan2 seam, v = 0
 * at +Y. */
static void equirect_uv(const float d[3], float* u, float* v) {
    *u = atan2f(d[2], d[0]) * IBL_INV_TWO_PI + 0.5f;
    const float y = d[1] < -1.f ? -1.f : (d[1] > 1.f ? 1.f : d[1]);
    *v = acosf(y) * IBL_INV_PI;
}

/* DirFromEquirectUv (ibl_math.h:47-52) */
static void equirect_dir(float u, float v, float d[3]) {
    const float phi = (u - 0.5f) * IBL_TWO_PI;
    const float theta = v * IBL_PI;
    const float st = sinf(theta);
    d[0] = st * cosf(phi);
    d[1] = cosf(theta);
    d[2] = st * sinf(phi);
}

/* BilerpWrap (ibl_math.h:56-86): 4 taps, u wraps, v clamps; taps in (dy,
 * dx) order. Calls tap(x, y, weight) through the caller's loop instead of
 * summing when out is NULL (used by the transposes). */
static void bilerp_wrap_taps(uint32_t w, uint32_t h, float u, float v,
                             int tx[4], int ty[4], float tw[4]) {
    const float sx = u * (float)w - 0.5f;
    const float sy = v * (float)h - 0.5f;
    const int ix = to_i32(floorf(sx));
    const int iy = to_i32(floorf(sy));
    const float fx = sx - (float)ix;
    const float fy = sy - (float)iy;
    int k = 0;
    for (int dy = 0; dy <= 1; dy++)
        for (int dx = 0; dx <= 1; dx++, k++) {
            int x = ix + dx;
            if (x < 0) x += (int)w;
            if (x >= (int)w) x -= (int)w;
            int y = iy + dy;
            y = y < 0 ? 0 : (y > (int)h - 1 ? (int)h - 1 : y);
            tx[k] = x;
            ty[k] = y;
            tw[k] = (dx == 0 ? 1.f - fx : fx) * (dy == 0 ? 1.f - fy : fy);
        }
}

/* The direction of a dir-image pixel, normalised; 0 for |d| < 1e-8 (the
 * rasterizer's background; f_ops.cpp:2944-2950). */
static int unit_dir(const float* p, float d[3]) {
    d[0] = p[0];
    d[1] = p[1];
    d[2] = p[2];
    const float len = sqrtf(dot3(d, d));
    if (len < 1e-8f) return 0;
    d[0] = d[0] / len;
    d[1] = d[1] / len;
    d[2] = d[2] / len;
    return 1;
}

/* EquirectSample (f_ops.cpp:2913-2964): map [mh][mw][n] sampled along dir
 * [n_px][3] -> out [n_px][n]. */
void orc_equirect_sample(const float* map, uint32_t mw, uint32_t mh,
                         uint32_t n, const float* dir, size_t n_px,
                         float* out) {
    for (size_t p = 0; p < n_px; p++) {
        float* o = &out[p * n];
        for (uint32_t c = 0; c < n; c++) o[c] = 0.f;
        float d[3], u, v;
        if (!unit_dir(&dir[p * 3], d)) continue;
        equirect_uv(d, &u, &v);
        int tx[4], ty[4];
        float tw[4];
        bilerp_wrap_taps(mw, mh, u, v, tx, ty, tw);
        for (int k = 0; k < 4; k++) {
            const float* e = &map[((size_t)ty[k] * mw + tx[k]) * n];
            for (uint32_t c = 0; c < n; c++) o[c] += tw[k] * e[c];
        }
    }
}

/* EquirectSampleBwd + TileSum (f_ops.cpp:2831-2909, 2785-2821): the exact
 * transpose w.r.t. the map, accumulated in k band partials of the dir
 * image (k = the smallest power of two with map texels * k >= 65536, at
 * most the dir height), each summed in pixel order, then added in band
 * order. gy [dh][dw][n], dir [dh][dw][3] -> g_map [mh][mw][n]. */
int orc_equirect_sample_bwd(const float* gy, const float* dir, uint32_t dw,
                            uint32_t dh, uint32_t mw, uint32_t mh, uint32_t n,
                            float* g_map) {
    uint32_t k = 1;
    while ((size_t)mw * mh * k < 65536 && k < dh) k *= 2;
    const uint32_t rows_per = (dh + k - 1) / k;
    const size_t plane = (size_t)mw * mh * n;
    float* part = (float*)calloc(plane * k, sizeof(float));
    if (!part) return fail("oom");
    for (uint32_t py = 0; py < dh; py++) {
        float* dst = part + plane * (py / rows_per);
        for (uint32_t px = 0; px < dw; px++) {
            const size_t p = (size_t)py * dw + px;
            float d[3], u, v;
            if (!unit_dir(&dir[p * 3], d)) continue;
            equirect_uv(d, &u, &v);
            int tx[4], ty[4];
            float tw[4];
            bilerp_wrap_taps(mw, mh, u, v, tx, ty, tw);
            for (int q = 0; q < 4; q++) {
                float* o = &dst[((size_t)ty[q] * mw + tx[q]) * n];
                for (uint32_t c = 0; c < n; c++) o[c] += gy[p * n + c] * tw[q];
            }
        }
    }
    for (size_t i = 0; i < plane; i++) g_map[i] = 0.f;
    for (uint32_t b = 0; b < k; b++)
        for (size_t i = 0; i < plane; i++) g_map[i] += part[plane * b + i];
    free(part);
    return 0;
}

/* IrradianceConv (f_ops.cpp:3023-3105): out(N) = 2 pi / (sw sh) * sum_s
 * max(N . d_s, 0) sin(theta_s) env(s), summed in source row-major order
 * per output texel. env [sh][sw][n] -> out [oh][ow][n]. */
void orc_irradiance_conv(const float* env, uint32_t sw, uint32_t sh,
                         uint32_t n, uint32_t ow, uint32_t oh, float* out) {
    const float scale = IBL_TWO_PI / ((float)sw * (float)sh);
    for (uint32_t oy = 0; oy < oh; oy++)
        for (uint32_t ox = 0; ox < ow; ox++) {
            float N[3];
            equirect_dir(((float)ox + 0.5f) / (float)ow,
                         ((float)oy + 0.5f) / (float)oh, N);
            float* o = &out[((size_t)oy * ow + ox) * n];
            for (uint32_t c = 0; c < n; c++) o[c] = 0.f;
            for (uint32_t sy = 0; sy < sh; sy++) {
                const float sv = ((float)sy + 0.5f) / (float)sh;
                const float sin_th = sinf(sv * IBL_PI);
                for (uint32_t sx = 0; sx < sw; sx++) {
                    float d[3];
                    equirect_dir(((float)sx + 0.5f) / (float)sw, sv, d);
                    const float nd = dot3(N, d);
                    const float w = (nd < 0.f ? 0.f : nd) * sin_th;
                    const float* e = &env[((size_t)sy * sw + sx) * n];
                    for (uint32_t c = 0; c < n; c++) o[c] += e[c] * w;
                }
            }
            for (uint32_t c = 0; c < n; c++) o[c] *= scale;
        }
}

/* IrradianceConvBwd (f_ops.cpp:2970-3019): the exact transpose, per source
 * texel the sum over output texels in row-major order, times sin and the
 * scale. gy [oh][ow][n] -> g_env [sh][sw][n]. */
void orc_irradiance_conv_bwd(const float* gy, uint32_t ow, uint32_t oh,
                             uint32_t n, uint32_t sw, uint32_t sh,
                             float* g_env) {
    const float scale = IBL_TWO_PI / ((float)sw * (float)sh);
    for (uint32_t sy = 0; sy < sh; sy++) {
        const float sv = ((float)sy + 0.5f) / (float)sh;
        const float sin_th = sinf(sv * IBL_PI);
        for (uint32_t sx = 0; sx < sw; sx++) {
            float d[3];
            equirect_dir(((float)sx + 0.5f) / (float)sw, sv, d);
            float* o = &g_env[((size_t)sy * sw + sx) * n];
            for (uint32_t c = 0; c < n; c++) o[c] = 0.f;
            for (uint32_t ty = 0; ty < oh; ty++)
                for (uint32_t tx = 0; tx < ow; tx++) {
                    float N[3];
                    equirect_dir(((float)tx + 0.5f) / (float)ow,
                                 ((float)ty + 0.5f) / (float)oh, N);
                    const float nd = dot3(N, d);
                    const float w = (nd < 0.f ? 0.f : nd) * sin_th;
                    const float* g = &gy[((size_t)ty * ow + tx) * n];
                    for (uint32_t c = 0; c < n; c++) o[c] += g[c] * w;
                }
            for (uint32_t c = 0; c < n; c++) o[c] *= scale;
        }
    }
}

/* GgxConvWeight (ibl_math.h:160-168) */
static inline float ggx_conv_weight(float c, float alpha) {
    if (c <= 0.f) return 0.f;
    const float ch2 = (1.f + c) * 0.5f;
    const float a2 = alpha * alpha;
    const float d = ch2 * (a2 - 1.f) + 1.f;
    return a2 / (IBL_PI * d * d) * c;
}

/* alpha of PrefilterConv (f_ops.cpp:3280-3283): max(r, 0.045)^2 */
float orc_prefilter_alpha(float roughness) {
    const float r = roughness < 0.045f ? 0.045f : roughness;
    return r * r;
}

/* PrefilterConvNorm (f_ops.cpp:3166-3205): W(t) = sum_s w(R_t . d_s)
 * sin(theta_s), a float sum in source row-major order. */
void orc_prefilter_conv_norm(uint32_t ow, uint32_t oh, uint32_t sw,
                             uint32_t sh, float alpha, float* out) {
    for (uint32_t oy = 0; oy < oh; oy++)
        for (uint32_t ox = 0; ox < ow; ox++) {
            float r[3];
            equirect_dir(((float)ox + 0.5f) / (float)ow,
                         ((float)oy + 0.5f) / (float)oh, r);
            float acc = 0.f;
            for (uint32_t sy = 0; sy < sh; sy++) {
                const float sv = ((float)sy + 0.5f) / (float)sh;
                const float sin_th = sinf(sv * IBL_PI);
                for (uint32_t sx = 0; sx < sw; sx++) {
                    float d[3];
                    equirect_dir(((float)sx + 0.5f) / (float)sw, sv, d);
                    acc += ggx_conv_weight(dot3(r, d), alpha) * sin_th;
                }
            }
            out[(size_t)oy * ow + ox] = acc;
        }
}

/* PrefilterConv (f_ops.cpp:3272-3345): pref(t) = sum_s w sin env(s) /
 * max(W(t), 1e-12). */
void orc_prefilter_conv(const float* env, uint32_t sw, uint32_t sh,
                        uint32_t n, const float* norm, uint32_t ow,
                        uint32_t oh, float alpha, float* out) {
    for (uint32_t oy = 0; oy < oh; oy++)
        for (uint32_t ox = 0; ox < ow; ox++) {
            float r[3];
            equirect_dir(((float)ox + 0.5f) / (float)ow,
                         ((float)oy + 0.5f) / (float)oh, r);
            float* o = &out[((size_t)oy * ow + ox) * n];
            for (uint32_t c = 0; c < n; c++) o[c] = 0.f;
            for (uint32_t sy = 0; sy < sh; sy++) {
                const float sv = ((float)sy + 0.5f) / (float)sh;
                const float sin_th = sinf(sv * IBL_PI);
                for (uint32_t sx = 0; sx < sw; sx++) {
                    float d[3];
                    equirect_dir(((float)sx + 0.5f) / (float)sw, sv, d);
                    const float w = ggx_conv_weight(dot3(r, d), alpha) * sin_th;
                    const float* e = &env[((size_t)sy * sw + sx) * n];
                    for (uint32_t c = 0; c < n; c++) o[c] += e[c] * w;
                }
            }
            const float nv = norm[(size_t)oy * ow + ox];
            const float wn = nv < 1e-12f ? 1e-12f : nv;
            for (uint32_t c = 0; c < n; c++) o[c] /= wn;
        }
}

/* PrefilterConvBwd (f_ops.cpp:3210-3268): g_env(s) = sin(theta_s) sum_t
 * gy(t) w(t, s) / max(W(t), 1e-12), skipping w <= 0. */
void orc_prefilter_conv_bwd(const float* gy, const float* norm, uint32_t ow,
                            uint32_t oh, uint32_t n, uint32_t sw, uint32_t sh,
                            float alpha, float* g_env) {
    for (uint32_t sy = 0; sy < sh; sy++) {
        const float sv = ((float)sy + 0.5f) / (float)sh;
        const float sin_th = sinf(sv * IBL_PI);
        for (uint32_t sx = 0; sx < sw; sx++) {
            float d[3];
            equirect_dir(((float)sx + 0.5f) / (float)sw, sv, d);
            float* o = &g_env[((size_t)sy * sw + sx) * n];
            for (uint32_t c = 0; c < n; c++) o[c] = 0.f;
            for (uint32_t ty = 0; ty < oh; ty++)
                for (uint32_t tx = 0; tx < ow; tx++) {
                    float r[3];
                    equirect_dir(((float)tx + 0.5f) / (float)ow,
                                 ((float)ty + 0.5f) / (float)oh, r);
                    const float w = ggx_conv_weight(dot3(r, d), alpha);
                    if (w <= 0.f) continue;
                    const float nv = norm[(size_t)ty * ow + tx];
                    const float wn = w / (nv < 1e-12f ? 1e-12f : nv);
                    const float* g = &gy[((size_t)ty * ow + tx) * n];
                    for (uint32_t c = 0; c < n; c++) o[c] += g[c] * wn;
                }
            for (uint32_t c = 0; c < n; c++) o[c] *= sin_th;
        }
    }
}

/* RadicalInverse / Hammersley (ibl_math.h:119-131) */
static float radical_inverse(uint32_t b) {
    b = (b << 16u) | (b >> 16u);
    b = ((b & 0x55555555u) << 1u) | ((b & 0xAAAAAAAAu) >> 1u);
    b = ((b & 0x33333333u) << 2u) | ((b & 0xCCCCCCCCu) >> 2u);
    b = ((b & 0x0F0F0F0Fu) << 4u) | ((b & 0xF0F0F0F0u) >> 4u);
    b = ((b & 0x00FF00FFu) << 8u) | ((b & 0xFF00FF00u) >> 8u);
    return (float)b * 2.3283064365386963e-10f;
}

static void normalize3(float v[3]) {
    const float len = sqrtf(dot3(v, v));
    v[0] = v[0] / len;
    v[1] = v[1] / len;
    v[2] = v[2] / len;
}

/* ImportanceSampleGGX about N = +Z (ibl_math.h:135-150; the tangent frame
 * of +Z is built from up = (1, 0, 0)). */
static void ggx_sample_z(float xi0, float xi1, float rough, float h[3]) {
    const float a = rough * rough;
    const float phi = IBL_TWO_PI * xi0;
    const float ct = sqrtf((1.f - xi1) / (1.f + (a * a - 1.f) * xi1));
    const float st2 = 1.f - ct * ct;
    const float st = sqrtf(st2 < 0.f ? 0.f : st2);
    const float ht[3] = {cosf(phi) * st, sinf(phi) * st, ct};
    /* up = (1,0,0) since |n.z| = 1 >= 0.999; tx = normalize(up x n),
     * ty = n x tx with n = (0,0,1) */
    float tx[3] = {0.f * 1.f - 0.f * 0.f, 0.f * 0.f - 1.f * 1.f,
                   1.f * 0.f - 0.f * 0.f};
    normalize3(tx);
    const float ty[3] = {0.f * tx[2] - 1.f * tx[1], 1.f * tx[0] - 0.f * tx[2],
                         0.f * tx[1] - 0.f * tx[0]};
    h[0] = tx[0] * ht[0] + ty[0] * ht[1] + 0.f * ht[2];
    h[1] = tx[1] * ht[0] + ty[1] * ht[1] + 0.f * ht[2];
    h[2] = tx[2] * ht[0] + ty[2] * ht[1] + 1.f * ht[2];
    normalize3(h);
}

/* BrdfIntegrationLut (f_ops.cpp:3350-3408): (A, B) over (NdotV, rough)
 * texel centres, n_samples Hammersley GGX samples, Smith G with k =
 * rough^2 / 2. out [h][w][2]. */
void orc_brdf_lut(uint32_t w, uint32_t h, uint32_t n_samples, float* out) {
    for (uint32_t oy = 0; oy < h; oy++) {
        const float rough = ((float)oy + 0.5f) / (float)h;
        const float k = rough * rough / 2.f;
        for (uint32_t ox = 0; ox < w; ox++) {
            const float ndv = ((float)ox + 0.5f) / (float)w;
            const float s2 = 1.f - ndv * ndv;
            const float V[3] = {sqrtf(s2 < 0.f ? 0.f : s2), 0.f, ndv};
            float a = 0.f, b = 0.f;
            for (uint32_t i = 0; i < n_samples; i++) {
                const float xi0 = (float)i / (float)n_samples;
                const float xi1 = radical_inverse(i);
                float hv[3];
                ggx_sample_z(xi0, xi1, rough, hv);
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
                    a += (1.f - fc) * gv;
                    b += fc * gv;
                }
            }
            out[((size_t)oy * w + ox) * 2 + 0] = a / (float)n_samples;
            out[((size_t)oy * w + ox) * 2 + 1] = b / (float)n_samples;
        }
    }
}

/* AvgPool2x2 = Reduce2x2Sum * 0.25 (f_ops.cpp:3411-3415, 995-1033): each
 * output sums its 2x2 sources in row-major order. w, h even. */
void orc_avg_pool2x2(const float* x, uint32_t w, uint32_t h, uint32_t n,
                     float* out) {
    const uint32_t ow = w / 2, oh = h / 2;
    for (uint32_t oy = 0; oy < oh; oy++)
        for (uint32_t ox = 0; ox < ow; ox++)
            for (uint32_t c = 0; c < n; c++) {
                const float a = x[((size_t)(2 * oy) * w + 2 * ox) * n + c];
                const float b = x[((size_t)(2 * oy) * w + 2 * ox + 1) * n + c];
                const float cc = x[((size_t)(2 * oy + 1) * w + 2 * ox) * n + c];
                const float d = x[((size_t)(2 * oy + 1) * w + 2 * ox + 1) * n + c];
                out[((size_t)oy * ow + ox) * n + c] = (((a + b) + cc) + d) * 0.25f;
            }
}

/* ---------------------------------------------- PBR shading graph (C5) */

/* BilerpClamp of a [h][w][n] image at (u, v) (ibl_math.h:91-115); the taps
 * and weights, (dy, dx) order, both axes clamped. */
static void clamp_taps(uint32_t w, uint32_t h, float u, float v, int idx[4],
                       float wt[4]) {
    const float sx = u * (float)w - 0.5f;
    const float sy = v * (float)h - 0.5f;
    const int ix = to_i32(floorf(sx));
    const int iy = to_i32(floorf(sy));
    const float fx = sx - (float)ix;
    const float fy = sy - (float)iy;
    int k = 0;
    for (int dy = 0; dy <= 1; dy++)
        for (int dx = 0; dx <= 1; dx++, k++) {
            int x = ix + dx, y = iy + dy;
            x = x < 0 ? 0 : (x > (int)w - 1 ? (int)w - 1 : x);
            y = y < 0 ? 0 : (y > (int)h - 1 ? (int)h - 1 : y);
            idx[k] = y * (int)w + x;
            wt[k] = (dx == 0 ? 1.f - fx : fx) * (dy == 0 ? 1.f - fy : fy);
        }
}

static void sample_clamp(const float* img, uint32_t w, uint32_t h, uint32_t n,
                         float u, float v, float* out) {
    int idx[4];
    float wt[4];
    clamp_taps(w, h, u, v, idx, wt);
    for (uint32_t c = 0; c < n; c++) out[c] = 0.f;
    for (int k = 0; k < 4; k++)
        for (uint32_t c = 0; c < n; c++) out[c] += wt[k] * img[(size_t)idx[k] * n + c];
}

static void scatter_clamp(float* g, uint32_t w, uint32_t h, uint32_t n,
                          float u, float v, const float* gy) {
    int idx[4];
    float wt[4];
    clamp_taps(w, h, u, v, idx, wt);
    for (int k = 0; k < 4; k++)
        for (uint32_t c = 0; c < n; c++) g[(size_t)idx[k] * n + c] += gy[c] * wt[k];
}

/* EquirectSample of a VEC3 map along d (0 for |d| < 1e-8) and its
 * transpose (scatter, any order). */
static void sample_equirect3(const float* map, uint32_t w, uint32_t h,
                             const float dir[3], float out[3]) {
    orc_equirect_sample(map, w, h, 3, dir, 1, out);
}

static void scatter_equirect3(float* g, uint32_t w, uint32_t h,
                              const float dir[3], const float gy[3]) {
    float d[3], u, v;
    if (!unit_dir(dir, d)) return;
    equirect_uv(d, &u, &v);
    int tx[4], ty[4];
    float tw[4];
    bilerp_wrap_taps(w, h, u, v, tx, ty, tw);
    for (int q = 0; q < 4; q++)
        for (int c = 0; c < 3; c++)
            g[((size_t)ty[q] * w + tx[q]) * 3 + c] += gy[c] * tw[q];
}

/* SafeNormalize (pbr_graph.cpp:17-19): v * InverseSqrt(dot(v, v) + 1e-12),
 * InverseSqrt = 1 / sqrt. */
static void safe_normalize(const float v[3], float out[3]) {
    const float is = 1.f / sqrtf(dot3(v, v) + 1e-12f);
    out[0] = v[0] * is;
    out[1] = v[1] * is;
    out[2] = v[2] * is;
}

static inline float fmax_ref(float a, float b) { return (a < b) ? b : a; }

/* The pixel-static terms of BuildPbrShade (pbr_graph.cpp:47-138) without
 * normal mapping: everything that depends on the G-buffer and the frame
 * only. */
void orc_pbr_static(const float g_n[3], const float g_p[3],
                    const float cam_pos[3], const float light_pos[3],
                    const float light_col[3], float out[ORC_PBR_STATIC]) {
    float n[3], v[3], l[3], h[3], vl[3], cp[3], tl[3];
    safe_normalize(g_n, n);
    for (int c = 0; c < 3; c++) cp[c] = cam_pos[c] - g_p[c];
    safe_normalize(cp, v);
    const float ndv = fmax_ref(dot3(n, v), 1e-4f);
    for (int c = 0; c < 3; c++) tl[c] = light_pos[c] - g_p[c];
    const float dist2 = fmax_ref(dot3(tl, tl), 1e-4f);
    safe_normalize(tl, l);
    for (int c = 0; c < 3; c++) vl[c] = v[c] + l[c];
    safe_normalize(vl, h);
    const float ndl = fmax_ref(dot3(n, l), 0.f);
    const float ndh = fmax_ref(dot3(n, h), 0.f);
    const float vdh = fmax_ref(dot3(v, h), 0.f);
    /* Reflect(-v, n) = I - (2 dot(n, I)) n (f_ops.cpp:737-741) */
    const float I[3] = {-v[0], -v[1], -v[2]};
    const float k2 = 2.f * dot3(n, I);
    out[0] = ndv;
    out[1] = ndl;
    out[2] = ndh;
    out[3] = vdh;
    out[4] = powf(1.f - ndv, 5.f);
    out[5] = powf(1.f - vdh, 5.f);
    for (int c = 0; c < 3; c++) out[6 + c] = light_col[c] / dist2;
    for (int c = 0; c < 3; c++) out[9 + c] = n[c];
    for (int c = 0; c < 3; c++) out[12 + c] = I[c] - k2 * n[c];
}

/* One pixel of BuildPbrShade (no normal mapping) and the gradient of its
 * loss term, in the reference autodiff's rules (f_ops.cpp: Max/Min give a
 * tie to the first operand, Clamp passes inside [lo, hi] inclusive, Abs ->
 * Sign, Pow -> p x^(p-1); broadcast FLOAT operands receive the component
 * sum). st: orc_pbr_static; A, mr, E: the material samples, ao the ao
 * sample; irr, P[L], bg: the environment samples; ab the LUT sample.
 * Writes hdr / mapped and the gradients of loss = wgt * |T - mapped| summed
 * (loss_kind 1) or wgt * (T - mapped)^2 (loss_kind 2). */
typedef struct {
    float gA[3], g_rough, g_metal, g_irr[3], g_bg[3];
    float g_P[ORC_PBR_MAX_LEVELS][3];
    float mapped[3];
    double loss;
} pbr_px_out_t;

static void pbr_pixel(const float* st, float mask, const float A[3],
                      float rough_raw, float metal, float ao, const float E[3],
                      const float irr[3], const float (*P)[3], int L,
                      const float ab[2], const float bg[3], const float T[3],
                      int loss_kind, float wgt, pbr_px_out_t* o) {
    const float ndv = st[0], ndl = st[1], ndh = st[2];
    const float p5v = st[4], p5h = st[5];
    const float* rad = &st[6];
    const float pi = IBL_PI;
    /* ---- forward */
    const float rough = rough_raw < 0.045f ? 0.045f
                        : (1.f < rough_raw ? 1.f : rough_raw);
    float f0[3], fres[3], kdd[3], fibl[3], kdi[3], mx[3];
    for (int c = 0; c < 3; c++) f0[c] = 0.04f + (A[c] - 0.04f) * metal;
    const float alpha = rough * rough;
    const float alpha2 = alpha * alpha;
    const float dd = ndh * ndh * (alpha2 - 1.f) + 1.f;
    const float D = pi * dd * dd;
    const float dist_d = alpha2 / D;
    const float r1a = rough + 1.f, r1b = rough + 1.f;
    const float k = r1a * r1b / 8.f;
    const float omk = 1.f - k;
    const float den_v = ndv * omk + k;
    const float gv = ndv / den_v;
    const float ndlc = fmax_ref(ndl, 1e-4f);
    const float den_l = ndlc * omk + k;
    const float gl = ndlc / den_l;
    for (int c = 0; c < 3; c++) fres[c] = f0[c] + (1.f - f0[c]) * p5h;
    const float num = dist_d * gv * gl;
    const float den_s = 4.f * ndv * ndl + 1e-4f;
    const float sd = num / den_s;
    const float om_metal = 1.f - metal;
    for (int c = 0; c < 3; c++) kdd[c] = (1.f - fres[c]) * om_metal;
    float lo[3], w1[3];
    for (int c = 0; c < 3; c++) {
        w1[c] = kdd[c] * A[c] / pi + fres[c] * sd;
        lo[c] = w1[c] * rad[c] * ndl;
    }
    const float omr = 1.f - rough;
    for (int c = 0; c < 3; c++) {
        mx[c] = fmax_ref(omr, f0[c]);
        fibl[c] = f0[c] + (mx[c] - f0[c]) * p5v;
        kdi[c] = (1.f - fibl[c]) * om_metal;
    }
    const float lod = rough * (float)(L - 1);
    float wl[ORC_PBR_MAX_LEVELS], xl[ORC_PBR_MAX_LEVELS];
    float pref[3] = {0.f, 0.f, 0.f};
    for (int i = 0; i < L; i++) {
        xl[i] = 1.f - fabsf(lod - (float)i);
        wl[i] = xl[i] < 0.f ? 0.f : (1.f < xl[i] ? 1.f : xl[i]);
    }
    /* at most two non-zero terms: their sum does not depend on the order */
    for (int i = 0; i < L; i++)
        for (int c = 0; c < 3; c++)
            if (wl[i] != 0.f) pref[c] += P[i][c] * wl[i];
    float q[3], spec_ibl[3], amb[3], shaded[3], hdr[3];
    for (int c = 0; c < 3; c++) {
        q[c] = f0[c] * ab[0] + ab[1];
        spec_ibl[c] = pref[c] * q[c];
        amb[c] = (kdi[c] * irr[c] * A[c] + spec_ibl[c]) * ao;
        shaded[c] = lo[c] + amb[c] + E[c];
        hdr[c] = mask * shaded[c] + (1.f - mask) * bg[c];
        o->mapped[c] = hdr[c] / (hdr[c] + 1.f);
    }
    /* ---- loss and backward */
    float g_hdr[3];
    o->loss = 0.0;
    for (int c = 0; c < 3; c++) {
        const float diff = T[c] - o->mapped[c];
        float g_diff;
        if (loss_kind == 1) {
            o->loss += (double)(fabsf(diff) * wgt);
            g_diff = wgt * (float)((diff > 0.f) - (diff < 0.f));
        } else {
            o->loss += (double)(diff * diff * wgt);
            g_diff = wgt * diff + wgt * diff;
        }
        const float g_m = -g_diff;
        const float h1 = hdr[c] + 1.f;
        g_hdr[c] = g_m / h1 + -(g_m * hdr[c] / (h1 * h1));
    }
    float g_sh[3], g_A[3] = {0.f, 0.f, 0.f}, g_f0[3] = {0.f, 0.f, 0.f};
    float g_rough = 0.f, g_metal = 0.f;
    for (int c = 0; c < 3; c++) {
        g_sh[c] = g_hdr[c] * mask;
        o->g_bg[c] = g_hdr[c] * (1.f - mask);
    }
    /* ambient = ((kdi * irr) * A + spec_ibl) * ao */
    float g_kdi[3], g_q[3], g_pref[3];
    for (int c = 0; c < 3; c++) {
        const float g_t1 = g_sh[c] * ao;
        const float g_ki = g_t1 * A[c];
        g_A[c] += g_t1 * (kdi[c] * irr[c]);
        g_kdi[c] = g_ki * irr[c];
        o->g_irr[c] = g_ki * kdi[c];
        g_pref[c] = g_t1 * q[c];
        g_q[c] = g_t1 * pref[c];
        g_f0[c] += g_q[c] * ab[0];
    }
    /* pref = sum_i P_i w_i, w_i = Clamp(1 - |lod - i|, 0, 1) */
    float g_lod = 0.f;
    for (int i = 0; i < L; i++) {
        float gw = 0.f;
        for (int c = 0; c < 3; c++) {
            o->g_P[i][c] = g_pref[c] * wl[i];
            gw += g_pref[c] * P[i][c];
        }
        const float inside = (xl[i] >= 0.f && 1.f >= xl[i]) ? 1.f : 0.f;
        const float g_x = gw * inside;
        const float dl = lod - (float)i;
        const float sgn = (float)((dl > 0.f) - (dl < 0.f));
        g_lod += -g_x * sgn;
    }
    g_rough += g_lod * (float)(L - 1);
    /* kdi = (1 - fibl) * (1 - metal) */
    float g_fibl[3], g_omm = 0.f;
    for (int c = 0; c < 3; c++) {
        g_fibl[c] = -(g_kdi[c] * om_metal);
        g_omm += g_kdi[c] * (1.f - fibl[c]);
    }
    /* fibl = f0 + (Max(1 - rough, f0) - f0) * p5v */
    float g_omr = 0.f;
    for (int c = 0; c < 3; c++) {
        g_f0[c] += g_fibl[c];
        const float g_mx = g_fibl[c] * p5v;
        g_f0[c] += -g_mx;
        const float m = (omr >= f0[c]) ? 1.f : 0.f;
        g_omr += g_mx * m;
        g_f0[c] += g_mx * (1.f - m);
    }
    g_rough += -g_omr;
    /* lo = ((kdd * A / pi + fres * sd) * rad) * ndl */
    float g_kdd[3], g_fres[3] = {0.f, 0.f, 0.f}, g_sd = 0.f;
    for (int c = 0; c < 3; c++) {
        const float g_w1 = g_sh[c] * ndl * rad[c];
        const float g_kA = g_w1 / pi;
        g_kdd[c] = g_kA * A[c];
        g_A[c] += g_kA * kdd[c];
        g_fres[c] += g_w1 * sd;
        g_sd += g_w1 * fres[c];
    }
    /* kdd = (1 - fres) * (1 - metal) */
    for (int c = 0; c < 3; c++) {
        g_fres[c] += -(g_kdd[c] * om_metal);
        g_omm += g_kdd[c] * (1.f - fres[c]);
    }
    g_metal += -g_omm;
    /* fres = f0 + (1 - f0) * p5h */
    for (int c = 0; c < 3; c++) {
        g_f0[c] += g_fres[c];
        g_f0[c] += -(g_fres[c] * p5h);
    }
    /* sd = ((dist_d * gv) * gl) / den_s */
    const float g_num = g_sd / den_s;
    const float g_dg = g_num * gl;
    const float g_gl = g_num * (dist_d * gv);
    const float g_dist = g_dg * gv;
    const float g_gv = g_dg * dist_d;
    /* gv = ndv / (ndv * (1 - k) + k), gl likewise */
    float g_k = 0.f;
    {
        const float g_den = -(g_gv * ndv / (den_v * den_v));
        g_k += g_den;
        g_k += -(g_den * ndv);
        const float g_den2 = -(g_gl * ndlc / (den_l * den_l));
        g_k += g_den2;
        g_k += -(g_den2 * ndlc);
    }
    /* k = ((rough + 1) * (rough + 1)) / 8 */
    const float g_sq = g_k / 8.f;
    g_rough += g_sq * r1b + g_sq * r1a;
    /* dist_d = alpha2 / ((pi * dd) * dd), dd = (ndh ndh)(alpha2 - 1) + 1 */
    float g_a2 = g_dist / D;
    const float g_D = -(g_dist * alpha2 / (D * D));
    const float g_pdd = g_D * dd;
    const float g_dd = g_D * (pi * dd) + g_pdd * pi;
    g_a2 += g_dd * (ndh * ndh);
    const float g_alpha = g_a2 * alpha + g_a2 * alpha;
    g_rough += g_alpha * rough + g_alpha * rough;
    /* f0 = 0.04 + (A - 0.04) * metal */
    for (int c = 0; c < 3; c++) {
        g_A[c] += g_f0[c] * metal;
        g_metal += g_f0[c] * (A[c] - 0.04f);
    }
    for (int c = 0; c < 3; c++) o->gA[c] = g_A[c];
    /* rough = Clamp(mr.y, 0.045, 1) */
    const int rin = rough_raw >= 0.045f && 1.f >= rough_raw;
    o->g_rough = rin ? g_rough : 0.f;
    o->g_metal = g_metal;
}

/* PoolTo (ibl.cpp:14-20) by halving until it fits; returns the level. */
static float* pool_to(const float* env, uint32_t w, uint32_t h, uint32_t mw,
                      uint32_t mh, uint32_t* ow, uint32_t* oh) {
    float* cur = (float*)malloc(sizeof(float) * (size_t)w * h * 3);
    memcpy(cur, env, sizeof(float) * (size_t)w * h * 3);
    while (w > mw || h > mh) {
        float* nx = (float*)malloc(sizeof(float) * (size_t)(w / 2) * (h / 2) * 3);
        orc_avg_pool2x2(cur, w, h, 3, nx);
        free(cur);
        cur = nx;
        w /= 2;
        h /= 2;
    }
    *ow = w;
    *oh = h;
    return cur;
}

/* g of the level at (w, h) -> g of the source env, through the pooling
 * chain's transposes (each 2x2 source texel receives 0.25 g). */
static void unpool_add(const float* g, uint32_t w, uint32_t h, uint32_t ew,
                       uint32_t eh, float* g_env) {
    float* cur = (float*)malloc(sizeof(float) * (size_t)w * h * 3);
    memcpy(cur, g, sizeof(float) * (size_t)w * h * 3);
    while (w < ew) {
        float* nx = (float*)malloc(sizeof(float) * (size_t)w * h * 12);
        for (uint32_t y = 0; y < 2 * h; y++)
            for (uint32_t x = 0; x < 2 * w; x++)
                for (int c = 0; c < 3; c++)
                    nx[((size_t)y * 2 * w + x) * 3 + c] =
                            cur[((size_t)(y / 2) * w + x / 2) * 3 + c] * 0.25f;
        free(cur);
        cur = nx;
        w *= 2;
        h *= 2;
    }
    for (size_t i = 0; i < (size_t)ew * eh * 3; i++) g_env[i] += cur[i];
    free(cur);
}

/* The split-sum IBL maps of an env (pbr_graph.cpp:23-34 with the
 * differentiable prefilter; ibl.cpp:22-60): irradiance 32x16 of the env
 * pooled to <= 64x32, L PrefilterConv levels from the env pooled to <=
 * 128x64 (level i at roughness i / (L-1), sizes halving from min(128x64,
 * src)). */
typedef struct {
    uint32_t ew, eh, iw, ih, irr_sw, irr_sh, pw, ph, L;
    float* irr_src;
    float* irr;
    float* pref_src;
    float* pref[ORC_PBR_MAX_LEVELS];
    uint32_t lw[ORC_PBR_MAX_LEVELS], lh[ORC_PBR_MAX_LEVELS];
    float* norm[ORC_PBR_MAX_LEVELS];
} ibl_maps_t;

static void ibl_free(ibl_maps_t* m) {
    free(m->irr_src);
    free(m->irr);
    free(m->pref_src);
    for (uint32_t i = 0; i < m->L; i++) {
        free(m->pref[i]);
        free(m->norm[i]);
    }
}

static void ibl_build(const float* env, uint32_t ew, uint32_t eh, uint32_t L,
                      ibl_maps_t* m) {
    memset(m, 0, sizeof(*m));
    m->ew = ew;
    m->eh = eh;
    m->L = L;
    m->iw = 32;
    m->ih = 16;
    m->irr_src = pool_to(env, ew, eh, 64, 32, &m->irr_sw, &m->irr_sh);
    m->irr = (float*)malloc(sizeof(float) * 32 * 16 * 3);
    orc_irradiance_conv(m->irr_src, m->irr_sw, m->irr_sh, 3, 32, 16, m->irr);
    m->pref_src = pool_to(env, ew, eh, 128, 64, &m->pw, &m->ph);
    uint32_t w = m->pw < 128 ? m->pw : 128, h = m->ph < 64 ? m->ph : 64;
    for (uint32_t i = 0; i < L; i++) {
        const float rough = (float)i / (float)(L - 1);
        const float alpha = orc_prefilter_alpha(rough);
        m->lw[i] = w;
        m->lh[i] = h;
        m->norm[i] = (float*)malloc(sizeof(float) * w * h);
        orc_prefilter_conv_norm(w, h, m->pw, m->ph, alpha, m->norm[i]);
        m->pref[i] = (float*)malloc(sizeof(float) * w * h * 3);
        orc_prefilter_conv(m->pref_src, m->pw, m->ph, 3, m->norm[i], w, h,
                           alpha, m->pref[i]);
        w = w > 1 ? w / 2 : 1;
        h = h > 1 ? h / 2 : 1;
    }
}

/* BuildPbrShade with per-pixel G-buffer and material images sampled at
 * pixel centres (identity uv: the w x h material "textures" are the
 * per-pixel values), the L1 / L2 loss against T (Mean per image), and its
 * gradients w.r.t. albedo, mr and the env through the whole IBL chain
 * (EquirectSample / IrradianceConv / PrefilterConv / pooling transposes).
 * Images [h][w][c]; env [eh][ew][3]; frame: cam_pos, cam_fwd, cam_right,
 * cam_up, light_pos, light_col (3 each); lut [lh][lw][2]. */
int orc_pbr_shade_grad(uint32_t w, uint32_t h, const float* g_n,
                       const float* g_p, const float* mask,
                       const float* albedo, const float* mr, const float* ao,
                       const float* emissive, const float* frame,
                       const float* env, uint32_t ew, uint32_t eh, uint32_t L,
                       const float* lut, uint32_t lw, uint32_t lh,
                       const float* target, int loss_kind, float* mapped,
                       double* loss, float* g_albedo, float* g_mr,
                       float* g_env) {
    memset(g_albedo, 0, sizeof(float) * (size_t)w * h * 3);
    memset(g_mr, 0, sizeof(float) * (size_t)w * h * 3);
    memset(g_env, 0, sizeof(float) * (size_t)ew * eh * 3);
    return orc_pbr_shade_grad_uv(w, h, g_n, g_p, mask, NULL, w, h, albedo,
                                 mr, ao, emissive, frame, env, ew, eh, L, lut,
                                 lw, lh, target, loss_kind, mapped, loss,
                                 g_albedo, g_mr, g_env);
}

/* The same with material textures of tw x th sampled at the G-buffer's uv
 * [h][w][2] (NULL: pixel centres with tw x th = w x h). With a uv image ao
 * and emissive are constant 1 x 1 textures (ao = 1 and emissive = 0 in
 * the C5 plan), otherwise [th][tw][3] images. The material gradients are
 * the exact transpose of the bilinear samples (scatter); every gradient is
 * accumulated (+=), so views sum by repeated calls. */
int orc_pbr_shade_grad_uv(uint32_t w, uint32_t h, const float* g_n,
                          const float* g_p, const float* mask,
                          const float* uv_img, uint32_t tw, uint32_t th,
                          const float* albedo, const float* mr,
                          const float* ao, const float* emissive,
                          const float* frame, const float* env, uint32_t ew,
                          uint32_t eh, uint32_t L, const float* lut,
                          uint32_t lw, uint32_t lh, const float* target,
                          int loss_kind, float* mapped, double* loss,
                          float* g_albedo, float* g_mr, float* g_env) {
    if (L < 2 || L > ORC_PBR_MAX_LEVELS) return fail("pbr: levels 2..%d", ORC_PBR_MAX_LEVELS);
    {
        /* the reference's prefilter levels must stay non-uniform (> 1x1) */
        uint32_t w0 = ew, h0 = eh;
        while (w0 > 128 || h0 > 64) {
            w0 /= 2;
            h0 /= 2;
        }
        for (uint32_t i = 1; i < L; i++) {
            w0 = w0 > 1 ? w0 / 2 : 1;
            h0 = h0 > 1 ? h0 / 2 : 1;
        }
        if (w0 * h0 <= 1) return fail("pbr: prefilter level %u would be 1x1", L - 1);
    }
    ibl_maps_t m;
    ibl_build(env, ew, eh, L, &m);
    const float wgt = 1.f / ((float)w * (float)h * 3.f);
    float* g_irr = (float*)calloc(32 * 16 * 3, sizeof(float));
    float* g_pref[ORC_PBR_MAX_LEVELS];
    for (uint32_t i = 0; i < L; i++)
        g_pref[i] = (float*)calloc((size_t)m.lw[i] * m.lh[i] * 3, sizeof(float));
    double tot = 0.0;
    const int const_ao = tw != w || th != h || uv_img != NULL;
    const float* cam_pos = frame;
    const float* fwd = frame + 3;
    const float* right = frame + 6;
    const float* up = frame + 9;
    const float* light_pos = frame + 12;
    const float* light_col = frame + 15;
    for (uint32_t py = 0; py < h; py++)
        for (uint32_t px = 0; px < w; px++) {
            const size_t p = (size_t)py * w + px;
            float st[ORC_PBR_STATIC];
            orc_pbr_static(&g_n[p * 3], &g_p[p * 3], cam_pos, light_pos,
                           light_col, st);
            const float u = uv_img ? uv_img[p * 2 + 0]
                                   : ((float)px + 0.5f) / (float)w;
            const float v = uv_img ? uv_img[p * 2 + 1]
                                   : ((float)py + 0.5f) / (float)h;
            float A[3], MR[3], AO[3], E[3], irr[3], bg[3], ab[2];
            float P[ORC_PBR_MAX_LEVELS][3];
            sample_clamp(albedo, tw, th, 3, u, v, A);
            sample_clamp(mr, tw, th, 3, u, v, MR);
            if (const_ao) {
                /* 1x1 textures: every tap reads the one texel */
                sample_clamp(ao, 1, 1, 3, u, v, AO);
                sample_clamp(emissive, 1, 1, 3, u, v, E);
            } else {
                sample_clamp(ao, tw, th, 3, u, v, AO);
                sample_clamp(emissive, tw, th, 3, u, v, E);
            }
            sample_equirect3(m.irr, 32, 16, &st[9], irr);
            for (uint32_t i = 0; i < L; i++)
                sample_equirect3(m.pref[i], m.lw[i], m.lh[i], &st[12], P[i]);
            const float rough = MR[1] < 0.045f ? 0.045f
                                : (1.f < MR[1] ? 1.f : MR[1]);
            sample_clamp(lut, lw, lh, 2, st[0], rough, ab);
            /* background ray (pbr_graph.cpp:115-121) */
            const float ndc_x = ((float)px + 0.5f) * (2.f / (float)w) - 1.f;
            const float ndc_y = ((float)py + 0.5f) * (2.f / (float)h) - 1.f;
            float ray[3];
            for (int c = 0; c < 3; c++)
                ray[c] = fwd[c] + right[c] * ndc_x - up[c] * ndc_y;
            sample_equirect3(env, ew, eh, ray, bg);
            pbr_px_out_t o;
            pbr_pixel(st, mask[p], A, MR[1], MR[2], AO[0], E, irr,
                      (const float(*)[3])P, (int)L, ab, bg, &target[p * 3],
                      loss_kind, wgt, &o);
            tot += o.loss;
            for (int c = 0; c < 3; c++) mapped[p * 3 + c] = o.mapped[c];
            scatter_clamp(g_albedo, tw, th, 3, u, v, o.gA);
            const float gmr[3] = {0.f, o.g_rough, o.g_metal};
            scatter_clamp(g_mr, tw, th, 3, u, v, gmr);
            scatter_equirect3(g_irr, 32, 16, &st[9], o.g_irr);
            for (uint32_t i = 0; i < L; i++)
                scatter_equirect3(g_pref[i], m.lw[i], m.lh[i], &st[12], o.g_P[i]);
            scatter_equirect3(g_env, ew, eh, ray, o.g_bg);
        }
    *loss = tot;
    /* the IBL chain's transposes */
    float* g_isrc = (float*)malloc(sizeof(float) * (size_t)m.irr_sw * m.irr_sh * 3);
    orc_irradiance_conv_bwd(g_irr, 32, 16, 3, m.irr_sw, m.irr_sh, g_isrc);
    unpool_add(g_isrc, m.irr_sw, m.irr_sh, ew, eh, g_env);
    float* g_psrc = (float*)calloc((size_t)m.pw * m.ph * 3, sizeof(float));
    float* tmp = (float*)malloc(sizeof(float) * (size_t)m.pw * m.ph * 3);
    for (uint32_t i = 0; i < L; i++) {
        orc_prefilter_conv_bwd(g_pref[i], m.norm[i], m.lw[i], m.lh[i], 3,
                               m.pw, m.ph,
                               orc_prefilter_alpha((float)i / (float)(L - 1)),
                               tmp);
        for (size_t j = 0; j < (size_t)m.pw * m.ph * 3; j++) g_psrc[j] += tmp[j];
    }
    unpool_add(g_psrc, m.pw, m.ph, ew, eh, g_env);
    free(tmp);
    free(g_psrc);
    free(g_isrc);
    free(g_irr);
    for (uint32_t i = 0; i < L; i++) free(g_pref[i]);
    ibl_free(&m);
    return 0;
}

/* ---------------------------------------------- indexed access (HSR) */

/* ScreenCoord (f_ops.cpp:1490-1513): out [h][w][2] = (x + 0.5, y + 0.5). */
void orc_screen_coord(uint32_t w, uint32_t h, float* out) {
    for (uint32_t py = 0; py < h; py++)
        for (uint32_t px = 0; px < w; px++) {
            const size_t o = ((size_t)py * w + px) * 2;
            out[o + 0] = (float)px + 0.5f;
            out[o + 1] = (float)py + 0.5f;
        }
}

/* LookupFaces (f_ops.cpp:1568-1619): out[f] = attr[faces[f][corner]]
 * (n components). A vertex id out of range is an error here (the reference
 * reads out of bounds). */
int orc_lookup_faces(const float* attr, uint32_t n_verts, uint32_t n,
                     const float* faces, uint32_t n_faces, uint32_t corner,
                     float* out) {
    if (corner > 2) return fail("lookup_faces: corner must be 0..2");
    for (uint32_t f = 0; f < n_faces; f++) {
        const uint32_t vi = to_u32_via_i64(faces[(size_t)f * 3 + corner] + 0.5f);
        if (vi >= n_verts) return fail("lookup_faces: vertex index range");
        for (uint32_t c = 0; c < n; c++)
            out[(size_t)f * n + c] = attr[(size_t)vi * n + c];
    }
    return 0;
}

/* LookupFacesBwd (f_ops.cpp:1521-1564): out[v] = sum, in the order of the
 * vertex's incident-face list vf {V, max_deg} (-1 padding), of gy[f] over
 * the faces whose corner `corner` is v. */
int orc_lookup_faces_bwd(const float* gy, uint32_t n, const float* faces,
                         uint32_t n_faces, const float* vf, uint32_t n_verts,
                         uint32_t max_deg, uint32_t corner, float* out) {
    if (corner > 2) return fail("lookup_faces_bwd: corner must be 0..2");
    for (size_t i = 0; i < (size_t)n_verts * n; i++) out[i] = 0.f;
    for (uint32_t v = 0; v < n_verts; v++)
        for (uint32_t d = 0; d < max_deg; d++) {
            const float fv = vf[(size_t)d * n_verts + v];
            if (fv < -0.5f) continue;
            const uint32_t f = to_u32_via_i64(fv + 0.5f);
            if (f >= n_faces) return fail("lookup_faces_bwd: face index range");
            const uint32_t vi =
                    to_u32_via_i64(faces[(size_t)f * 3 + corner] + 0.5f);
            if (vi != v) continue;
            for (uint32_t c = 0; c < n; c++)
                out[(size_t)v * n + c] += gy[(size_t)f * n + c];
        }
    return 0;
}

/* FaceFetch (f_ops.cpp:1736-1799): out(p) = attr[idx(p) - 1], 0 for the
 * background and for ids past the attribute table. */
void orc_face_fetch(const float* attr, uint32_t n_faces, uint32_t n,
                    const float* idx, size_t n_px, float* out) {
    for (size_t p = 0; p < n_px; p++) {
        /* int(x) - 1 wraps INT_MIN to INT_MAX on x86: skipped either way */
        const int64_t f = (int64_t)to_i32(idx[p] + 0.5f) - 1;
        for (uint32_t c = 0; c < n; c++)
            out[p * n + c] = (f < 0 || f >= (int64_t)n_faces)
                                     ? 0.f
                                     : attr[(size_t)f * n + c];
    }
}

/* FaceFetchBwd (f_ops.cpp:1631-1732). n_samples == 0: the exact VJP, the
 * face's screen bbox (+-1 px) scanned row by row, summing gy where the id
 * image names the face. n_samples > 0: the paper's edge samples -- sample
 * s on edge s % 3 at HashToUnit(f, s, seed, 0) along it and an offset of
 * (2 HashToUnit(f, s, seed, 1) - 1) radius_px across it, gathered where the
 * id image confirms the face. prj[k] [F][4]: corner k's clip position. */
void orc_face_fetch_bwd(const float* gy, uint32_t n, const float* idx,
                        uint32_t w, uint32_t h, const float* prj0,
                        const float* prj1, const float* prj2,
                        uint32_t n_faces, float seed, float radius_px,
                        uint32_t n_samples, float* out) {
    const float* prj[3] = {prj0, prj1, prj2};
    const uint32_t seed_u = to_u32_via_i64(seed + 0.5f);
    for (size_t i = 0; i < (size_t)n_faces * n; i++) out[i] = 0.f;
    for (uint32_t f = 0; f < n_faces; f++) {
        float s[3][2];
        int ok = 1;
        for (int k = 0; k < 3; k++) {
            const float* c = &prj[k][(size_t)f * 4];
            if (c[3] <= 1e-6f) {
                ok = 0;
                break;
            }
            s[k][0] = (c[0] / c[3] * 0.5f + 0.5f) * (float)w;
            s[k][1] = (c[1] / c[3] * 0.5f + 0.5f) * (float)h;
        }
        if (!ok) continue;
        float* dst = &out[(size_t)f * n];
        if (n_samples == 0) {
            const float lo_x = smin(smin(s[0][0], s[1][0]), s[2][0]);
            const float hi_x = smax(smax(s[0][0], s[1][0]), s[2][0]);
            const float lo_y = smin(smin(s[0][1], s[1][1]), s[2][1]);
            const float hi_y = smax(smax(s[0][1], s[1][1]), s[2][1]);
            const int x0 = imax(to_i32(floorf(lo_x - 1.f)), 0);
            const int x1 = imin(to_i32(ceilf(hi_x + 1.f)), (int)w - 1);
            const int y0 = imax(to_i32(floorf(lo_y - 1.f)), 0);
            const int y1 = imin(to_i32(ceilf(hi_y + 1.f)), (int)h - 1);
            for (int iy = y0; iy <= y1; iy++)
                for (int ix = x0; ix <= x1; ix++) {
                    const size_t p = (size_t)iy * w + (size_t)ix;
                    if (to_u32_via_i64(idx[p] + 0.5f) != f + 1) continue;
                    for (uint32_t c = 0; c < n; c++) dst[c] += gy[p * n + c];
                }
            continue;
        }
        for (uint32_t smp = 0; smp < n_samples; smp++) {
            const int e = (int)(smp % 3);
            const float* a = s[e];
            const float* b = s[(e + 1) % 3];
            const float ex = b[0] - a[0];
            const float ey = b[1] - a[1];
            const float len = sqrtf(ex * ex + ey * ey);
            if (len < 1e-6f) continue;
            const float u = hash_to_unit(f, smp, seed_u, 0);
            const float o = (hash_to_unit(f, smp, seed_u, 1) * 2.f - 1.f) *
                            radius_px;
            const float px = a[0] + u * ex - o * (ey / len);
            const float py = a[1] + u * ey + o * (ex / len);
            const int ix = to_i32(floorf(px));
            const int iy = to_i32(floorf(py));
            if (ix < 0 || iy < 0 || ix >= (int)w || iy >= (int)h) continue;
            const size_t p = (size_t)iy * w + (size_t)ix;
            if (to_u32_via_i64(idx[p] + 0.5f) != f + 1) continue;
            for (uint32_t c = 0; c < n; c++) dst[c] += gy[p * n + c];
        }
    }
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
