// Optimizer-side regulariser of the silhouette optimisation
// (examples/silhouette_optimization/run.cpp:407-420), applied to the
// all-reduced vertex gradient g before Adam:
//
//   g_lap = pos - VertexNeighborMean(pos, nbrs)        k_vertex_terms
//   term  = NormalConsistencyFaceTerm(pos, faces, adj)  k_nc_face_term
//   g_nrm = NormalConsistencyVertexGrad(term, ...)      k_vertex_terms
//   s_lap = rms(g) / rms(g_lap) * laplacian             k_reg_scale
//   s_nrm = rms(g) / rms(g_nrm) * normal                k_reg_scale
//   g'    = (g + g_lap * s_lap) + g_nrm * s_nrm         k_gpos_adam
//
// rms(x) = sqrt(SumAll(x * x) * (1 / 3V) + 1e-24). SumAll is restated
// with the reference's own summation order (f_ops.cpp:1087-1149: above 256
// elements, 64 strided partial sums in double, each rounded to float, then
// their double sum), so with -fmad=false and IEEE division / square root
// every value here is bit-identical to the reference's CPU evaluator for
// the same g. The mesh tables keep the reference's layout (mesh_utils.cpp:
// 53-101): ids stored as float, -1 padding, {V, max_deg} tables row-major
// with row d at [d * V].
#include <algorithm>
#include <map>
#include <utility>
#include <vector>

#include "kernels.h"

namespace dressi {

namespace {

__device__ __forceinline__ int tab_id(float x) { return int(x + 0.5f); }

// A table id in [0, n): true; otherwise the status word's index bit is set
// (status nullable) and the entry is skipped.
__device__ __forceinline__ bool id_ok(float x, int n, uint32_t* status) {
    if (x > -0.5f && x < float(n) - 0.5f) return true;
    if (status) atomicOr(status, kStatusIndexRange);
    return false;
}

// The vertex ids of face f, all checked against n_verts.
__device__ __forceinline__ bool face_ids(const float* faces, int f,
                                         int n_verts, uint32_t* status,
                                         int idx[3]) {
    bool ok = true;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const float x = faces[size_t(f) * 3 + k];
        ok = ok && id_ok(x, n_verts, status);
        idx[k] = ok ? tab_id(x) : 0;
    }
    return ok;
}

// CrossOfFace (f_ops.cpp:1872-1885): (p1 - p0) x (p2 - p0); a face with an
// id out of range is zero (skipped like a degenerate one).
__device__ __forceinline__ void face_cross(const float* pos,
                                           const float* faces, int f,
                                           int n_verts, uint32_t* status,
                                           int idx[3], float c[3]) {
    if (!face_ids(faces, f, n_verts, status, idx)) {
        c[0] = c[1] = c[2] = 0.f;
        return;
    }
    const float* p0 = pos + size_t(idx[0]) * 3;
    const float* p1 = pos + size_t(idx[1]) * 3;
    const float* p2 = pos + size_t(idx[2]) * 3;
    const float e1[3] = {p1[0] - p0[0], p1[1] - p0[1], p1[2] - p0[2]};
    const float e2[3] = {p2[0] - p0[0], p2[1] - p0[1], p2[2] - p0[2]};
    c[0] = e1[1] * e2[2] - e1[2] * e2[1];
    c[1] = e1[2] * e2[0] - e1[0] * e2[2];
    c[2] = e1[0] * e2[1] - e1[1] * e2[0];
}

}  // namespace

// NormalConsistencyFaceTerm (f_ops.cpp:2031-2098): per face a, with
// n = c / |c| and faces closer to degenerate than |c| < 1e-12 skipped,
// term_a = sum over edge neighbours b of -(n_b - (n_a . n_b) n_a) / |c_a|.
__global__ void k_nc_face_term(const float* pos, int n_verts,
                               const float* faces, const float* fadj,
                               int n_faces, float* term, uint32_t* status) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= n_faces) return;
    int ia[3];
    float ca[3];
    face_cross(pos, faces, f, n_verts, status, ia, ca);
    const float la = sqrtf(ca[0] * ca[0] + ca[1] * ca[1] + ca[2] * ca[2]);
    float gg[3] = {0.f, 0.f, 0.f};
    if (la >= 1e-12f) {
        const float na[3] = {ca[0] / la, ca[1] / la, ca[2] / la};
#pragma unroll 1
        for (int j = 0; j < 3; j++) {
            const float gv = fadj[size_t(f) * 3 + j];
            if (gv < -0.5f || !id_ok(gv, n_faces, status)) continue;
            int ib[3];
            float cb[3];
            face_cross(pos, faces, tab_id(gv), n_verts, status, ib, cb);
            const float lb =
                    sqrtf(cb[0] * cb[0] + cb[1] * cb[1] + cb[2] * cb[2]);
            if (lb < 1e-12f) continue;
            const float nb[3] = {cb[0] / lb, cb[1] / lb, cb[2] / lb};
            const float d = na[0] * nb[0] + na[1] * nb[1] + na[2] * nb[2];
#pragma unroll
            for (int c = 0; c < 3; c++) gg[c] += -(nb[c] - d * na[c]) / la;
        }
    }
#pragma unroll
    for (int c = 0; c < 3; c++) term[size_t(f) * 3 + c] = gg[c];
}

// Per vertex: VertexNeighborMean (f_ops.cpp:1983-2029; the mean of the
// listed neighbours in table order, pos itself without neighbours) as
// `mean` or, with `lap_diff`, pos - mean; and NormalConsistencyVertexGrad
// (f_ops.cpp:2100-2181) over the vertex's incident faces in table order.
// Either output may be null.
__global__ void k_vertex_terms(const float* pos, int n_verts,
                               const float* nbrs, int nbr_deg, int lap_diff,
                               float* lap_out, const float* term,
                               const float* faces, int n_faces,
                               const float* vf, int vf_deg, float* nrm_out,
                               uint32_t* status) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n_verts) return;
    const float* pv = pos + size_t(v) * 3;
    if (lap_out) {
        float mean[3] = {0.f, 0.f, 0.f};
        int count = 0;
#pragma unroll 1
        for (int d = 0; d < nbr_deg; d++) {
            const float nv = nbrs[size_t(d) * n_verts + v];
            if (nv < -0.5f || !id_ok(nv, n_verts, status)) continue;
            const float* pn = pos + size_t(tab_id(nv)) * 3;
            mean[0] += pn[0];
            mean[1] += pn[1];
            mean[2] += pn[2];
            count++;
        }
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const float m = count > 0 ? mean[c] / float(count) : pv[c];
            lap_out[size_t(v) * 3 + c] = lap_diff ? pv[c] - m : m;
        }
    }
    if (nrm_out) {
        float acc[3] = {0.f, 0.f, 0.f};
#pragma unroll 1
        for (int d = 0; d < vf_deg; d++) {
            const float fv = vf[size_t(d) * n_verts + v];
            if (fv < -0.5f || !id_ok(fv, n_faces, status)) continue;
            const int f = tab_id(fv);
            int idx[3];
            if (!face_ids(faces, f, n_verts, status, idx)) continue;
            const float* p0 = pos + size_t(idx[0]) * 3;
            const float* p1 = pos + size_t(idx[1]) * 3;
            const float* p2 = pos + size_t(idx[2]) * 3;
            const float e1[3] = {p1[0] - p0[0], p1[1] - p0[1], p1[2] - p0[2]};
            const float e2[3] = {p2[0] - p0[0], p2[1] - p0[1], p2[2] - p0[2]};
            const float* t = term + size_t(f) * 3;
            const float g1[3] = {e2[1] * t[2] - e2[2] * t[1],
                                 e2[2] * t[0] - e2[0] * t[2],
                                 e2[0] * t[1] - e2[1] * t[0]};
            const float g2[3] = {t[1] * e1[2] - t[2] * e1[1],
                                 t[2] * e1[0] - t[0] * e1[2],
                                 t[0] * e1[1] - t[1] * e1[0]};
#pragma unroll
            for (int c = 0; c < 3; c++) {
                if (idx[1] == v) acc[c] += g1[c];
                if (idx[2] == v) acc[c] += g2[c];
                if (idx[0] == v) acc[c] -= g1[c] + g2[c];
            }
        }
#pragma unroll
        for (int c = 0; c < 3; c++) nrm_out[size_t(v) * 3 + c] = acc[c];
    }
}

namespace {

constexpr int kSumParts = 64;  // SumPartial's part count (f_ops.cpp:1127)

// Element value fed to SumAll: x, or x * x rounded to float (the
// reference squares in its own float node before summing).
template <bool kSq>
__device__ __forceinline__ double sum_elem(float x) {
    return kSq ? double(x * x) : double(x);
}

// SumPartial's part p (f_ops.cpp:1087-1115): the elements of pixels p,
// p + 64, ... in pixel-then-component order, summed in double and rounded
// to float. Pixel loads are issued eight at a time so the dependent double
// additions wait on one load latency per batch.
template <bool kSq>
__device__ float sum_partial(const float* x, int n_px, int nc, int p) {
    double s = 0.0;
    int i = p;
    for (; i + 7 * kSumParts < n_px; i += 8 * kSumParts) {
        float v[8][4];
#pragma unroll
        for (int k = 0; k < 8; k++)
#pragma unroll
            for (int c = 0; c < 4; c++)
                if (c < nc) v[k][c] = x[size_t(i + k * kSumParts) * nc + c];
#pragma unroll
        for (int k = 0; k < 8; k++)
#pragma unroll
            for (int c = 0; c < 4; c++)
                if (c < nc) s += sum_elem<kSq>(v[k][c]);
    }
    for (; i < n_px; i += kSumParts)
        for (int c = 0; c < nc; c++) s += sum_elem<kSq>(x[size_t(i) * nc + c]);
    return float(s);
}

// SumAll (f_ops.cpp:1119-1149) by a group of `kSumParts` threads (lane =
// index in the group); the result is valid in lane 0. `parts` is the
// group's shared scratch. Every thread of the block calls it with the same
// n_px (it holds a block barrier).
template <bool kSq>
__device__ float sum_all_block(const float* x, int n_px, int nc, int lane,
                               float* parts) {
    if (n_px <= 256) {
        // one serial pass over every element
        if (lane != 0) return 0.f;
        double s = 0.0;
        for (size_t i = 0; i < size_t(n_px) * nc; i++)
            s += sum_elem<kSq>(x[i]);
        return float(s);
    }
    parts[lane] = sum_partial<kSq>(x, n_px, nc, lane);
    __syncthreads();
    if (lane != 0) return 0.f;
    double s = 0.0;
    for (int q = 0; q < kSumParts; q++) s += double(parts[q]);
    return float(s);
}

}  // namespace

// out[0] = SumAll(x) for x [n_px][nc] (op level).
__global__ void k_sum_all(const float* x, int n_px, int nc, float* out) {
    __shared__ float parts[kSumParts];
    const float s = sum_all_block<false>(x, n_px, nc, threadIdx.x, parts);
    if (threadIdx.x == 0) out[0] = s;
}

// The three RMS values of the regulariser, one group of 64 threads each
// (g, g_lap, g_nrm), then scale = {s_lap, s_nrm}.
__global__ void k_reg_scale(const float* g, const float* glap,
                            const float* gnrm, int n_verts, float inv_cnt,
                            float laplacian, float normal, float* scale) {
    __shared__ float parts[3][kSumParts];
    __shared__ float rms[3];
    const int grp = threadIdx.x / kSumParts, lane = threadIdx.x % kSumParts;
    const float* x = grp == 0 ? g : (grp == 1 ? glap : gnrm);
    const float s = sum_all_block<true>(x, n_verts, 3, lane, parts[grp]);
    if (lane == 0) rms[grp] = sqrtf(s * inv_cnt + 1e-24f);
    __syncthreads();
    if (threadIdx.x == 0) {
        scale[0] = rms[0] / rms[1] * laplacian;
        scale[1] = rms[0] / rms[2] * normal;
    }
}

static void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

void nc_face_term_op(const float* pos, int n_verts, const float* faces,
                     const float* fadj, int n_faces, float* term,
                     uint32_t* status, cudaStream_t s) {
    if (n_faces <= 0) return;
    ProfScope ps("nc_face_term", s);
    k_nc_face_term<<<(n_faces + 127) / 128, 128, 0, s>>>(
            pos, n_verts, faces, fadj, n_faces, term, status);
    check_launch();
}

void vertex_terms_op(const float* pos, int n_verts, const float* nbrs,
                     int nbr_deg, bool lap_diff, float* lap_out,
                     const float* term, const float* faces, int n_faces,
                     const float* vf, int vf_deg, float* nrm_out,
                     uint32_t* status, cudaStream_t s) {
    if (n_verts <= 0) return;
    ProfScope ps("vertex_terms", s);
    k_vertex_terms<<<(n_verts + 127) / 128, 128, 0, s>>>(
            pos, n_verts, nbrs, nbr_deg, lap_diff ? 1 : 0, lap_out, term,
            faces, n_faces, vf, vf_deg, nrm_out, status);
    check_launch();
}

void reg_scale_op(const float* g, const float* glap, const float* gnrm,
                  int n_verts, float laplacian, float normal, float* scale,
                  cudaStream_t s) {
    ProfScope ps("reg_scale", s);
    k_reg_scale<<<1, 3 * kSumParts, 0, s>>>(g, glap, gnrm, n_verts,
                                            1.f / float(n_verts * 3),
                                            laplacian, normal, scale);
    check_launch();
}

// out = (g + glap * scale[0]) + gnrm * scale[1] (op level; out may alias g)
__global__ void k_reg_combine(const float* g, const float* glap,
                              const float* gnrm, const float* scale, int n,
                              float* out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = (g[i] + glap[i] * scale[0]) + gnrm[i] * scale[1];
}

void reg_combine_op(const float* g, const float* glap, const float* gnrm,
                    const float* scale, int n, float* out, cudaStream_t s) {
    if (n <= 0) return;
    ProfScope ps("reg_combine", s);
    k_reg_combine<<<(n + 255) / 256, 256, 0, s>>>(g, glap, gnrm, scale, n,
                                                  out);
    check_launch();
}

void sum_all_op(const float* x, int n_px, int nc, float* out,
                cudaStream_t s) {
    ProfScope ps("sum_all", s);
    k_sum_all<<<1, kSumParts, 0, s>>>(x, n_px, nc, out);
    check_launch();
}

// The plan's tables are built on the host from faces already checked at
// plan creation, so the plan passes no status word.
void sil_reg_terms(const SilParams& p, const SilBuffers& b, cudaStream_t s) {
    if (!p.reg) return;
    const RegBuffers& r = b.reg;
    nc_face_term_op(b.pos, p.n_verts, b.faces, r.fadj, p.n_faces, r.term,
                    nullptr, s);
    vertex_terms_op(b.pos, p.n_verts, r.nbrs, r.nbr_deg, true, r.glap,
                    r.term, b.faces, p.n_faces, r.vf, r.vf_deg, r.gnrm,
                    nullptr, s);
}

void sil_reg_scale(const SilParams& p, const SilBuffers& b, cudaStream_t s) {
    if (!p.reg) return;
    const RegBuffers& r = b.reg;
    reg_scale_op(b.gpos, r.glap, r.gnrm, p.n_verts, p.laplacian, p.normal,
                 r.scale, s);
}

// ---- host: the reference's mesh tables (mesh_utils.cpp:53-101) ----

void vertex_faces_table(const float* faces, int n_faces, int n_verts,
                        std::vector<float>* out, int* max_deg) {
    std::vector<std::vector<int>> lst(static_cast<size_t>(n_verts));
    for (int f = 0; f < n_faces; f++)
        for (int k = 0; k < 3; k++) {
            const float x = faces[size_t(f) * 3 + k];
            DRESSI_REQUIRE(x >= 0.f && x < float(n_verts),
                           "mesh tables: vertex index out of range");
            lst[size_t(x)].push_back(f);
        }
    int md = 1;
    for (const auto& l : lst) md = std::max(md, int(l.size()));
    out->assign(size_t(md) * n_verts, -1.f);
    for (int v = 0; v < n_verts; v++)
        for (size_t d = 0; d < lst[v].size(); d++)
            (*out)[d * n_verts + v] = float(lst[v][d]);
    *max_deg = md;
}

void vertex_neighbors_table(const float* faces, int n_faces, int n_verts,
                            std::vector<float>* out, int* max_deg) {
    std::vector<std::vector<int>> lst(static_cast<size_t>(n_verts));
    for (int f = 0; f < n_faces; f++) {
        int idx[3];
        for (int k = 0; k < 3; k++) {
            const float x = faces[size_t(f) * 3 + k];
            DRESSI_REQUIRE(x >= 0.f && x < float(n_verts),
                           "mesh tables: vertex index out of range");
            idx[k] = int(x);
        }
        for (int k = 0; k < 3; k++) {
            lst[idx[k]].push_back(idx[(k + 1) % 3]);
            lst[idx[k]].push_back(idx[(k + 2) % 3]);
        }
    }
    int md = 1;
    for (auto& l : lst) {
        std::sort(l.begin(), l.end());
        l.erase(std::unique(l.begin(), l.end()), l.end());
        md = std::max(md, int(l.size()));
    }
    out->assign(size_t(md) * n_verts, -1.f);
    for (int v = 0; v < n_verts; v++)
        for (size_t d = 0; d < lst[v].size(); d++)
            (*out)[d * n_verts + v] = float(lst[v][d]);
    *max_deg = md;
}

void face_neighbors_table(const float* faces, int n_faces,
                          std::vector<float>* out) {
    // faces of each undirected edge, keyed by (min, max) vertex, in face
    // order; every pair of an edge's faces links both ways; a face keeps
    // its first three links
    std::map<std::pair<int, int>, std::vector<int>> edges;
    for (int f = 0; f < n_faces; f++)
        for (int k = 0; k < 3; k++) {
            const int a = int(faces[size_t(f) * 3 + k]);
            const int b = int(faces[size_t(f) * 3 + (k + 1) % 3]);
            edges[{std::min(a, b), std::max(a, b)}].push_back(f);
        }
    out->assign(size_t(n_faces) * 3, -1.f);
    std::vector<int> n_adj(size_t(n_faces), 0);
    auto link = [&](int f, int g) {
        if (n_adj[f] < 3) (*out)[size_t(f) * 3 + n_adj[f]++] = float(g);
    };
    for (const auto& e : edges) {
        const auto& fs = e.second;
        for (size_t i = 0; i < fs.size(); i++)
            for (size_t j = i + 1; j < fs.size(); j++) {
                link(fs[i], fs[j]);
                link(fs[j], fs[i]);
            }
    }
}

}  // namespace dressi
