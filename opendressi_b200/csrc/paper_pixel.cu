// The per-pixel part of the paper path (the plan in paper.cu): for every
// layer the face corners fetched (FaceFetch of the LookupFaces clip
// positions), their screen positions, the signed distance to the face's
// edges, D_k = mask * sigmoid(dist * 7 / r); the Eq.6 union; pred =
// max(hard, union); the loss; and the backward to the fetched corners in
// the reference autodiff's rules (Min ties to the first operand, Clamp's
// inclusive interior, a broadcast FLOAT receives the component sum).
//
// This file is compiled with FMA contraction and the fast (<= 2 ulp)
// division: its outputs (the loss and the per-pixel gradients) have a
// tolerance contract with the reference. The raster, the face ids and the
// sampled pixels, which must be exact, are computed elsewhere.
#include "kernels.h"

namespace dressi {

namespace {

__device__ __forceinline__ float step0(float x) { return x < 0.f ? 0.f : 1.f; }
__device__ __forceinline__ float clamp01(float x) {
    return x < 0.f ? 0.f : (1.f < x ? 1.f : x);
}

// One edge of the signed-distance term: |pc - (a + clamp(t) e)| with its
// intermediate values (for the backward).
struct EdgeFwd {
    float ex, ey, num, den, ratio, t, ddx, ddy, ed;
};

__device__ __forceinline__ EdgeFwd edge_fwd(float ax, float ay, float bx,
                                            float by, float pcx, float pcy) {
    EdgeFwd e;
    e.ex = bx - ax;
    e.ey = by - ay;
    e.num = (pcx - ax) * e.ex + (pcy - ay) * e.ey;
    e.den = (e.ex * e.ex + e.ey * e.ey) + 1e-12f;
    e.ratio = e.num / e.den;
    e.t = clamp01(e.ratio);
    e.ddx = pcx - (ax + e.t * e.ex);
    e.ddy = pcy - (ay + e.t * e.ey);
    e.ed = sqrtf((e.ddx * e.ddx + e.ddy * e.ddy) + 1e-12f);
    return e;
}

// d ed / d (a, b) times g (accumulated).
__device__ __forceinline__ void edge_bwd(const EdgeFwd& e, float g, float ax,
                                         float ay, float pcx, float pcy,
                                         float* gax, float* gay, float* gbx,
                                         float* gby) {
    const float g_dd2 = g * 0.5f / e.ed;
    const float g_ddx = g_dd2 * e.ddx + g_dd2 * e.ddx;
    const float g_ddy = g_dd2 * e.ddy + g_dd2 * e.ddy;
    // dd = pc - (a + t e)
    const float g_qx = -g_ddx, g_qy = -g_ddy;
    float g_ax = g_qx, g_ay = g_qy;
    const float g_t = g_qx * e.ex + g_qy * e.ey;  // a broadcast FLOAT
    float g_ex = g_qx * e.t, g_ey = g_qy * e.t;
    // t = clamp(ratio, 0, 1), inclusive interior
    const float g_ratio = (e.ratio >= 0.f && e.ratio <= 1.f) ? g_t : 0.f;
    const float g_num = g_ratio / e.den;
    const float g_den = -(g_ratio * e.num / (e.den * e.den));
    g_ex += g_den * e.ex + g_den * e.ex;
    g_ey += g_den * e.ey + g_den * e.ey;
    g_ax += -(g_num * e.ex);
    g_ay += -(g_num * e.ey);
    g_ex += g_num * (pcx - ax);
    g_ey += g_num * (pcy - ay);
    // e = b - a
    *gbx += g_ex;
    *gby += g_ey;
    *gax += g_ax - g_ex;
    *gay += g_ay - g_ey;
}

// One layer's D = mask * sigmoid(signed edge distance * scale) from the
// fetched corner clip positions c[3]; with want_grad the gradient of g_D * D
// w.r.t. c (x, y, 0, w) into gc.
__device__ __forceinline__ float paper_layer(const float4 c[3], float mask,
                                             float pcx, float pcy, float R,
                                             float scale, bool want_grad,
                                             float g_D, float4 gc[3]) {
    float w[3], sx[3], sy[3];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        w[j] = c[j].w + (1.f - mask);
        sx[j] = (c[j].x / w[j] * 0.5f + 0.5f) * R;
        sy[j] = (c[j].y / w[j] * 0.5f + 0.5f) * R;
    }
    const EdgeFwd e01 = edge_fwd(sx[0], sy[0], sx[1], sy[1], pcx, pcy);
    const EdgeFwd e12 = edge_fwd(sx[1], sy[1], sx[2], sy[2], pcx, pcy);
    const EdgeFwd e20 = edge_fwd(sx[2], sy[2], sx[0], sy[0], pcx, pcy);
    // Min: the minimum; ties go to the first operand
    const float m = e12.ed < e01.ed ? e12.ed : e01.ed;
    const float dmin = e20.ed < m ? e20.ed : m;
    float cr[3];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const int j2 = (j + 1) % 3;
        const float ex = sx[j2] - sx[j], ey = sy[j2] - sy[j];
        cr[j] = ex * (pcy - sy[j]) - ey * (pcx - sx[j]);
    }
    const float in_sum = step0(cr[0]) * step0(cr[1]) * step0(cr[2]) +
                         step0(-cr[0]) * step0(-cr[1]) * step0(-cr[2]);
    const float inside = in_sum < 1.f ? in_sum : 1.f;
    const float sgn = inside * 2.f - 1.f;
    const float dist = sgn * dmin;
    const float sg = 1.f / (1.f + expf(-(dist * scale)));
    const float D = mask * sg;
    if (!want_grad) return D;
    const float g_sg = g_D * mask;
    const float g_z = g_sg * (sg * (1.f - sg));
    const float g_dist = g_z * scale;
    const float g_dmin = g_dist * sgn;
    const float g_m = e20.ed < m ? 0.f : g_dmin;
    const float g_e20 = e20.ed < m ? g_dmin : 0.f;
    const float g_e01 = e12.ed < e01.ed ? 0.f : g_m;
    const float g_e12 = e12.ed < e01.ed ? g_m : 0.f;
    float gsx[3] = {0.f, 0.f, 0.f}, gsy[3] = {0.f, 0.f, 0.f};
    edge_bwd(e01, g_e01, sx[0], sy[0], pcx, pcy, &gsx[0], &gsy[0], &gsx[1],
             &gsy[1]);
    edge_bwd(e12, g_e12, sx[1], sy[1], pcx, pcy, &gsx[1], &gsy[1], &gsx[2],
             &gsy[2]);
    edge_bwd(e20, g_e20, sx[2], sy[2], pcx, pcy, &gsx[2], &gsy[2], &gsx[0],
             &gsy[0]);
#pragma unroll
    for (int j = 0; j < 3; j++) {
        // s = (c / w * 0.5 + 0.5) * R
        const float grx = gsx[j] * R * 0.5f, gry = gsy[j] * R * 0.5f;
        const float ww = w[j] * w[j];
        gc[j] = make_float4(grx / w[j], gry / w[j], 0.f,
                            -(grx * c[j].x / ww) + -(gry * c[j].y / ww));
    }
    return D;
}

// The face of a layer's id (FaceFetch: int(idx + 0.5) - 1) and its corner
// clip positions (LookupFaces); false for the background or ids past the
// tables.
__device__ __forceinline__ bool fetch_corners(float idx, const float* faces,
                                              int n_faces, const float4* clip,
                                              int n_verts, float4 c[3]) {
    const long long f = (long long)x86_i32(idx + 0.5f) - 1;
    if (f < 0 || f >= n_faces) {
        c[0] = c[1] = c[2] = make_float4(0.f, 0.f, 0.f, 0.f);
        return false;
    }
#pragma unroll
    for (int j = 0; j < 3; j++) {
        const uint32_t vi = x86_u32_via_i64(faces[size_t(f) * 3 + j] + 0.5f);
        c[j] = vi < uint32_t(n_verts) ? clip[vi] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return true;
}

// Per pixel of every view: the loss and the gradient w.r.t. each layer's
// three fetched corners (gfetch[k][j], written where the layer has a face).
__global__ void __launch_bounds__(256)
        k_paper_pixel(SilParams p, const float4* layers, const float* targets,
                      const float4* clip, const float* faces, float4* gfetch,
                      double* loss_slots) {
    const long long npx = (long long)p.res * p.res;
    const long long total = npx * p.views;
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    float lv = 0.f;
    if (i < total) {
        const int v = int(i / npx);
        const long long pix = i - v * npx;
        const float pcx = float(pix % p.res) + 0.5f;
        const float pcy = float(pix / p.res) + 0.5f;
        const float R = float(p.res);
        const float4* cv = clip + size_t(v) * p.n_verts;
        float D[kPaperMaxPeels], q[kPaperMaxPeels], P[kPaperMaxPeels];
        float4 rsk[kPaperMaxPeels];
        float hard = 0.f, om = 1.f;
        for (int k = 0; k < p.peels; k++) {
            const float4 rs = layers[size_t(k) * total + i];
            rsk[k] = rs;
            if (k == 0) hard = rs.w * step0(rs.x);
            const float idx = (rs.y + 1.f) * rs.w;
            const float mask = idx > 0.5f ? 1.f : 0.f;
            float4 c[3], gdummy[3];
            // no face: FaceFetch gives zeros and D = 0 * sigmoid(.) = 0
            D[k] = 0.f;
            if (mask != 0.f) {
                fetch_corners(idx, faces, p.n_faces, cv, p.n_verts, c);
                D[k] = paper_layer(c, mask, pcx, pcy, R, p.sigma_scale, false,
                                   0.f, gdummy);
            }
            q[k] = 1.f - D[k];
            om = om * q[k];
            P[k] = om;
        }
        const float soft = 1.f - om;
        const float pred = hard < soft ? soft : hard;
        const float diff = targets[i] - pred;
        lv = diff * diff * p.c;
        const float g_diff = p.c * diff + p.c * diff;
        const float g_pred = -g_diff;
        const float g_soft = hard < soft ? g_pred : 0.f;
        float g_P = -g_soft;
        for (int k = p.peels - 1; k >= 0; k--) {
            const float prevP = k > 0 ? P[k - 1] : 1.f;
            const float g_q = g_P * prevP;
            g_P = g_P * q[k];
            const float4 rs = rsk[k];
            const float idx = (rs.y + 1.f) * rs.w;
            const float mask = idx > 0.5f ? 1.f : 0.f;
            if (mask == 0.f) continue;  // FaceFetch's backward never reads it
            float4 c[3], gc[3];
            fetch_corners(idx, faces, p.n_faces, cv, p.n_verts, c);
            paper_layer(c, mask, pcx, pcy, R, p.sigma_scale, true, -g_q, gc);
#pragma unroll
            for (int j = 0; j < 3; j++)
                gfetch[(size_t(k) * 3 + j) * total + i] = gc[j];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lv += __shfl_down_sync(0xffffffffu, lv, o);
    if ((threadIdx.x & 31) == 0 && lv != 0.f)
        atomicAdd(&loss_slots[(blockIdx.x * 8u + (threadIdx.x >> 5)) % kLossSlots],
                  double(lv));
}

}  // namespace

void paper_pixel_launch(const SilParams& p, const float4* layers,
                        const float* targets, const float4* clip,
                        const float* faces, float4* gfetch,
                        double* loss_slots, unsigned blocks, cudaStream_t s) {
    k_paper_pixel<<<blocks, 256, 0, s>>>(p, layers, targets, clip, faces,
                                         gfetch, loss_slots);
    DRESSI_CUDA(cudaGetLastError());
}

}  // namespace dressi
