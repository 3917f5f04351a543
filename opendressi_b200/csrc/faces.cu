// Indexed access of the paper's HardSoftRas path (f_ops.cpp:1490-1799):
// ScreenCoord, LookupFaces and its exact transpose, FaceFetch and its
// backward (the exact bbox scan, or the hashed edge samples of the paper's
// Alg. 1). Every output keeps the reference's summation order (one thread
// per output element, its terms in the reference's loop order), so all of
// them are bit-exact with the reference's CPU kernels.
#include "kernels.h"

namespace dressi {

namespace {

constexpr int kThreads = 256;

__global__ void k_screen_coord(int w, int h, float2* out) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)w * h) return;
    const int px = int(i % w), py = int(i / w);
    out[i] = make_float2(float(px) + 0.5f, float(py) + 0.5f);
}

// out[f][c] = attr[faces[f][corner]][c]
__global__ void k_lookup_faces(const float* attr, int n_verts, int n,
                               const float* faces, int n_faces, int corner,
                               float* out, uint32_t* status) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)n_faces * n) return;
    const long long f = i / n;
    const int c = int(i % n);
    const uint32_t vi = x86_u32_via_i64(faces[f * 3 + corner] + 0.5f);
    if (vi >= uint32_t(n_verts)) {
        if (status) atomicOr(status, kStatusIndexRange);
        out[i] = 0.f;
        return;
    }
    out[i] = attr[size_t(vi) * n + c];
}

// out[v] = sum over v's incident faces (table order) whose corner `corner`
// is v of gy[f] (LookupFacesBwd, f_ops.cpp:1521-1564).
__global__ void k_lookup_faces_bwd(const float* gy, int n, const float* faces,
                                   int n_faces, const float* vf, int n_verts,
                                   int max_deg, int corner, float* out,
                                   uint32_t* status) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n_verts) return;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < max_deg; d++) {
        const float fv = vf[size_t(d) * n_verts + v];
        if (fv < -0.5f) continue;
        const uint32_t f = x86_u32_via_i64(fv + 0.5f);
        if (f >= uint32_t(n_faces)) {
            if (status) atomicOr(status, kStatusIndexRange);
            continue;
        }
        const uint32_t vi = x86_u32_via_i64(faces[size_t(f) * 3 + corner] + 0.5f);
        if (vi != uint32_t(v)) continue;
        for (int c = 0; c < n; c++) acc[c] += gy[size_t(f) * n + c];
    }
    for (int c = 0; c < n; c++) out[size_t(v) * n + c] = acc[c];
}

// out(p) = attr[idx(p) - 1]; 0 for the background and ids past the table
__global__ void k_face_fetch(const float* attr, int n_faces, int n,
                             const float* idx, long long n_px, float* out) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= n_px * n) return;
    const long long p = i / n;
    const int c = int(i % n);
    // int(x) - 1 as on x86 (INT_MIN wraps to INT_MAX): skipped either way
    const long long f = (long long)x86_i32(idx[p] + 0.5f) - 1;
    out[i] = (f < 0 || f >= n_faces) ? 0.f : attr[size_t(f) * n + c];
}

// FaceFetchBwd (f_ops.cpp:1631-1732), one thread per face.
__global__ void k_face_fetch_bwd(const float* gy, int n, const float* idx,
                                 int w, int h, const float4* prj0,
                                 const float4* prj1, const float4* prj2,
                                 int n_faces, uint32_t seed_u,
                                 const float* seed_dev, float radius_px,
                                 int n_samples, float* out) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= n_faces) return;
    // seed from device memory (an in-graph {1,1} value) when given
    if (seed_dev) seed_u = x86_u32_via_i64(seed_dev[0] + 0.5f);
    const float4 c4[3] = {prj0[f], prj1[f], prj2[f]};
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float s[3][2];
    bool ok = true;
    for (int k = 0; k < 3; k++) {
        if (c4[k].w <= 1e-6f) {
            ok = false;
            break;
        }
        s[k][0] = (c4[k].x / c4[k].w * 0.5f + 0.5f) * float(w);
        s[k][1] = (c4[k].y / c4[k].w * 0.5f + 0.5f) * float(h);
    }
    if (ok && n_samples == 0) {
        // exact: the screen bbox (+-1 px), rows then columns
        auto mn = [](float a, float b) { return b < a ? b : a; };
        auto mx = [](float a, float b) { return a < b ? b : a; };
        const float lo_x = mn(mn(s[0][0], s[1][0]), s[2][0]);
        const float hi_x = mx(mx(s[0][0], s[1][0]), s[2][0]);
        const float lo_y = mn(mn(s[0][1], s[1][1]), s[2][1]);
        const float hi_y = mx(mx(s[0][1], s[1][1]), s[2][1]);
        const int x0 = imax_(x86_i32(floorf(lo_x - 1.f)), 0);
        const int x1 = imin_(x86_i32(ceilf(hi_x + 1.f)), w - 1);
        const int y0 = imax_(x86_i32(floorf(lo_y - 1.f)), 0);
        const int y1 = imin_(x86_i32(ceilf(hi_y + 1.f)), h - 1);
        for (int iy = y0; iy <= y1; iy++)
            for (int ix = x0; ix <= x1; ix++) {
                const size_t p = size_t(iy) * w + size_t(ix);
                if (x86_u32_via_i64(idx[p] + 0.5f) != uint32_t(f) + 1u) continue;
                for (int c = 0; c < n; c++) acc[c] += gy[p * n + c];
            }
    } else if (ok) {
        for (int smp = 0; smp < n_samples; smp++) {
            const int e = smp % 3;
            const float* a = s[e];
            const float* b = s[(e + 1) % 3];
            const float ex = b[0] - a[0];
            const float ey = b[1] - a[1];
            const float len = sqrtf(ex * ex + ey * ey);
            if (len < 1e-6f) continue;
            const float u = hash_to_unit(uint32_t(f), uint32_t(smp), seed_u, 0);
            const float o =
                    (hash_to_unit(uint32_t(f), uint32_t(smp), seed_u, 1) * 2.f - 1.f) *
                    radius_px;
            const float px = a[0] + u * ex - o * (ey / len);
            const float py = a[1] + u * ey + o * (ex / len);
            const int ix = x86_i32(floorf(px));
            const int iy = x86_i32(floorf(py));
            if (ix < 0 || iy < 0 || ix >= w || iy >= h) continue;
            const size_t p = size_t(iy) * w + size_t(ix);
            if (x86_u32_via_i64(idx[p] + 0.5f) != uint32_t(f) + 1u) continue;
            for (int c = 0; c < n; c++) acc[c] += gy[p * n + c];
        }
    }
    for (int c = 0; c < n; c++) out[size_t(f) * n + c] = acc[c];
}

unsigned blocks_for(long long n) { return unsigned((n + kThreads - 1) / kThreads); }

void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

}  // namespace

void screen_coord_op(int w, int h, float* out, cudaStream_t s) {
    ProfScope ps("screen_coord", s);
    const long long n = (long long)w * h;
    if (n == 0) return;
    k_screen_coord<<<blocks_for(n), kThreads, 0, s>>>(
            w, h, reinterpret_cast<float2*>(out));
    check_launch();
}

void lookup_faces_op(const float* attr, int n_verts, int n, const float* faces,
                     int n_faces, int corner, float* out, uint32_t* status,
                     cudaStream_t s) {
    ProfScope ps("lookup_faces", s);
    const long long total = (long long)n_faces * n;
    if (total == 0) return;
    k_lookup_faces<<<blocks_for(total), kThreads, 0, s>>>(
            attr, n_verts, n, faces, n_faces, corner, out, status);
    check_launch();
}

void lookup_faces_bwd_op(const float* gy, int n, const float* faces,
                         int n_faces, const float* vf, int n_verts,
                         int max_deg, int corner, float* out,
                         uint32_t* status, cudaStream_t s) {
    ProfScope ps("lookup_faces_bwd", s);
    if (n_verts == 0) return;
    k_lookup_faces_bwd<<<blocks_for(n_verts), kThreads, 0, s>>>(
            gy, n, faces, n_faces, vf, n_verts, max_deg, corner, out, status);
    check_launch();
}

void face_fetch_op(const float* attr, int n_faces, int n, const float* idx,
                   long long n_px, float* out, cudaStream_t s) {
    ProfScope ps("face_fetch", s);
    if (n_px * n == 0) return;
    k_face_fetch<<<blocks_for(n_px * n), kThreads, 0, s>>>(attr, n_faces, n,
                                                          idx, n_px, out);
    check_launch();
}

void face_fetch_bwd_op(const float* gy, int n, const float* idx, int w, int h,
                       const float* prj0, const float* prj1, const float* prj2,
                       int n_faces, float seed, float radius_px,
                       int n_samples, float* out, cudaStream_t s,
                       const float* seed_dev) {
    ProfScope ps("face_fetch_bwd", s);
    if (n_faces == 0) return;
    k_face_fetch_bwd<<<blocks_for(n_faces), kThreads, 0, s>>>(
            gy, n, idx, w, h, reinterpret_cast<const float4*>(prj0),
            reinterpret_cast<const float4*>(prj1),
            reinterpret_cast<const float4*>(prj2), n_faces,
            x86_u32_via_i64(seed + 0.5f), seed_dev, radius_px, n_samples,
            out);
    check_launch();
}

}  // namespace dressi
