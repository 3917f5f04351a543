// Optimizer-side regulariser of the silhouette optimisation
// (examples/silhouette_optimization/run.cpp:407-420), applied to the
// all-reduced vertex gradient g before Adam:
//
//   g_lap = pos - VertexNeighborMean(pos, nbrs)        k_vertex_terms
//   term  = NormalConsistencyFaceTerm(pos, faces, adj)  k_nc_face_term
//   g_nrm = NormalConsistencyVertexGrad(term, ...)      k_vertex_terms
//   rms(g), rms(g_lap), rms(g_nrm)                     k_reg_rms
//   s_lap = rms(g) / rms(g_lap) * laplacian             k_gpos_adam
//   s_nrm = rms(g) / rms(g_nrm) * normal                k_gpos_adam
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
// The three neighbours' crosses are loaded up front (independent loads);
// the sum keeps the table order.
__global__ void __launch_bounds__(128)
k_nc_face_term(const float* pos, int n_verts, const float* faces,
               const float* fadj, int n_faces, float* term,
               uint32_t* status) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= n_faces) return;
    float gv[3];
#pragma unroll
    for (int j = 0; j < 3; j++) gv[j] = fadj[size_t(f) * 3 + j];
    int ia[3];
    float ca[3];
    face_cross(pos, faces, f, n_verts, status, ia, ca);
    bool okb[3];
    float cb[3][3];
#pragma unroll
    for (int j = 0; j < 3; j++) {
        int ib[3];
        okb[j] = !(gv[j] < -0.5f) && id_ok(gv[j], n_faces, status);
        if (okb[j]) {
            face_cross(pos, faces, tab_id(gv[j]), n_verts, status, ib, cb[j]);
        } else {
            cb[j][0] = cb[j][1] = cb[j][2] = 0.f;
        }
    }
    const float la = sqrtf(ca[0] * ca[0] + ca[1] * ca[1] + ca[2] * ca[2]);
    float gg[3] = {0.f, 0.f, 0.f};
    if (la >= 1e-12f) {
        const float na[3] = {ca[0] / la, ca[1] / la, ca[2] / la};
#pragma unroll
        for (int j = 0; j < 3; j++) {
            if (!okb[j]) continue;
            const float* c = cb[j];
            const float lb = sqrtf(c[0] * c[0] + c[1] * c[1] + c[2] * c[2]);
            if (lb < 1e-12f) continue;
            const float nb[3] = {c[0] / lb, c[1] / lb, c[2] / lb};
            const float d = na[0] * nb[0] + na[1] * nb[1] + na[2] * nb[2];
#pragma unroll
            for (int k = 0; k < 3; k++) gg[k] += -(nb[k] - d * na[k]) / la;
        }
    }
#pragma unroll
    for (int k = 0; k < 3; k++) term[size_t(f) * 3 + k] = gg[k];
}

namespace {

constexpr int kVtxThreads = 64;  // ~10k vertices: a block on every SM
constexpr int kNbrBatch = 8;     // neighbour slots loaded per round
constexpr int kFaceBatch = 4;    // incident faces loaded per round

// VertexNeighborMean of vertex v (f_ops.cpp:1983-2029): the mean of the
// listed neighbours in table order, pos itself without neighbours.
__device__ __forceinline__ void neighbor_mean(const float* pos, int n_verts,
                                              const float* nbrs, int nbr_deg,
                                              int v, uint32_t* status,
                                              float m[3]) {
    float mean[3] = {0.f, 0.f, 0.f};
    int count = 0;
    for (int d0 = 0; d0 < nbr_deg; d0 += kNbrBatch) {
        float nv[kNbrBatch];
#pragma unroll
        for (int k = 0; k < kNbrBatch; k++)
            nv[k] = d0 + k < nbr_deg ? nbrs[size_t(d0 + k) * n_verts + v]
                                     : -1.f;
        bool ok[kNbrBatch];
        float pn[kNbrBatch][3];
#pragma unroll
        for (int k = 0; k < kNbrBatch; k++) {
            ok[k] = !(nv[k] < -0.5f) && id_ok(nv[k], n_verts, status);
            const float* q = pos + size_t(ok[k] ? tab_id(nv[k]) : v) * 3;
            pn[k][0] = q[0];
            pn[k][1] = q[1];
            pn[k][2] = q[2];
        }
#pragma unroll
        for (int k = 0; k < kNbrBatch; k++) {
            if (!ok[k]) continue;
            mean[0] += pn[k][0];
            mean[1] += pn[k][1];
            mean[2] += pn[k][2];
            count++;
        }
    }
    const float* pv = pos + size_t(v) * 3;
#pragma unroll
    for (int c = 0; c < 3; c++)
        m[c] = count > 0 ? mean[c] / float(count) : pv[c];
}

// NormalConsistencyVertexGrad of vertex v (f_ops.cpp:2100-2181): over its
// incident faces in table order, the transpose of c = e1 x e2 applied to
// the face term.
__device__ __forceinline__ void nc_vertex_grad(const float* term,
                                               const float* pos, int n_verts,
                                               const float* faces, int n_faces,
                                               const float* vf, int vf_deg,
                                               int v, uint32_t* status,
                                               float acc[3]) {
    acc[0] = acc[1] = acc[2] = 0.f;
    for (int d0 = 0; d0 < vf_deg; d0 += kFaceBatch) {
        float fv[kFaceBatch];
#pragma unroll
        for (int k = 0; k < kFaceBatch; k++)
            fv[k] = d0 + k < vf_deg ? vf[size_t(d0 + k) * n_verts + v] : -1.f;
        bool ok[kFaceBatch];
        int idx[kFaceBatch][3];
#pragma unroll
        for (int k = 0; k < kFaceBatch; k++) {
            ok[k] = !(fv[k] < -0.5f) && id_ok(fv[k], n_faces, status);
            ok[k] = ok[k] &&
                    face_ids(faces, tab_id(fv[k]), n_verts, status, idx[k]);
        }
        float e1[kFaceBatch][3], e2[kFaceBatch][3], t[kFaceBatch][3];
#pragma unroll
        for (int k = 0; k < kFaceBatch; k++) {
            const int f = ok[k] ? tab_id(fv[k]) : 0;
            const int i0 = ok[k] ? idx[k][0] : 0;
            const int i1 = ok[k] ? idx[k][1] : 0;
            const int i2 = ok[k] ? idx[k][2] : 0;
            const float* p0 = pos + size_t(i0) * 3;
            const float* p1 = pos + size_t(i1) * 3;
            const float* p2 = pos + size_t(i2) * 3;
#pragma unroll
            for (int c = 0; c < 3; c++) {
                e1[k][c] = p1[c] - p0[c];
                e2[k][c] = p2[c] - p0[c];
                t[k][c] = term[size_t(f) * 3 + c];
            }
        }
#pragma unroll
        for (int k = 0; k < kFaceBatch; k++) {
            if (!ok[k]) continue;
            const float* a = e1[k];
            const float* b = e2[k];
            const float* tt = t[k];
            const float g1[3] = {b[1] * tt[2] - b[2] * tt[1],
                                 b[2] * tt[0] - b[0] * tt[2],
                                 b[0] * tt[1] - b[1] * tt[0]};
            const float g2[3] = {tt[1] * a[2] - tt[2] * a[1],
                                 tt[2] * a[0] - tt[0] * a[2],
                                 tt[0] * a[1] - tt[1] * a[0]};
#pragma unroll
            for (int c = 0; c < 3; c++) {
                if (idx[k][1] == v) acc[c] += g1[c];
                if (idx[k][2] == v) acc[c] += g2[c];
                if (idx[k][0] == v) acc[c] -= g1[c] + g2[c];
            }
        }
    }
}

}  // namespace

// Per vertex, part 0: VertexNeighborMean as `mean` or, with lap_diff, pos -
// mean; part 1: NormalConsistencyVertexGrad. part = part0 + blockIdx.y, so
// both parts of a vertex run in separate threads.
__global__ void __launch_bounds__(kVtxThreads)
k_vertex_terms(const float* pos, int n_verts, const float* nbrs, int nbr_deg,
               int lap_diff, float* lap_out, const float* term,
               const float* faces, int n_faces, const float* vf, int vf_deg,
               float* nrm_out, uint32_t* status, int part0) {
    const int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n_verts) return;
    float r[3];
    if (part0 + int(blockIdx.y) == 0) {
        neighbor_mean(pos, n_verts, nbrs, nbr_deg, v, status, r);
        const float* pv = pos + size_t(v) * 3;
#pragma unroll
        for (int c = 0; c < 3; c++)
            lap_out[size_t(v) * 3 + c] = lap_diff ? pv[c] - r[c] : r[c];
    } else {
        nc_vertex_grad(term, pos, n_verts, faces, n_faces, vf, vf_deg, v,
                       status, r);
#pragma unroll
        for (int c = 0; c < 3; c++) nrm_out[size_t(v) * 3 + c] = r[c];
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

constexpr int kRmsThreads = 1024;
// dynamic shared staging buffer of the SumAll kernels (floats): 19200
// pixels x 3 components per round, within the 227 KB a block may opt into
constexpr int kStageFloats = kSumParts * 900;
constexpr int kStageBytes = kStageFloats * 4 + kSumParts * 4;
static_assert(kStageBytes <= 227 * 1024, "SumAll staging above 227 KB");
constexpr int kLoadBatch = 8;  // global loads in flight per thread

// SumAll (f_ops.cpp:1119-1149, SumPartial 1087-1115) of x [n_px][kNc] by
// one block of kRmsThreads threads; the result is valid in thread 0.
// Above 256 pixels, part p (thread p < 64) sums the elements of pixels p,
// p + 64, ... in pixel-then-component order in double, rounded to float;
// the 64 parts are summed in double. The pixels are staged in shared
// memory by the whole block (all of a batch's loads issued before its
// stores), so each part's serial chain reads shared memory only.
template <bool kSq, int kNc>
__device__ float sum_all_block(const float* x, int n_px, float* stage,
                               float* parts) {
    constexpr int nc = kNc;
    constexpr int round_px = kStageFloats / nc / kSumParts * kSumParts;
    const int tid = threadIdx.x;
    if (n_px <= 256) {
        // one serial pass over every element
        double s = 0.0;
        if (tid == 0)
            for (size_t i = 0; i < size_t(n_px) * nc; i++)
                s += sum_elem<kSq>(x[i]);
        return float(s);
    }
    double s = 0.0;
    for (int base = 0; base < n_px; base += round_px) {
        const int np = min(round_px, n_px - base);
        const float* src = x + size_t(base) * nc;
        const int total = np * nc;
        for (int i0 = tid; i0 < total; i0 += kLoadBatch * kRmsThreads) {
            float v[kLoadBatch];
#pragma unroll
            for (int k = 0; k < kLoadBatch; k++) {
                const int i = i0 + k * kRmsThreads;
                v[k] = i < total ? src[i] : 0.f;
            }
#pragma unroll
            for (int k = 0; k < kLoadBatch; k++) {
                const int i = i0 + k * kRmsThreads;
                if (i < total) stage[i] = v[k];
            }
        }
        __syncthreads();
        if (tid < kSumParts) {
            // shared loads four pixels ahead of the dependent double adds
            int j = tid;
            for (; j + 3 * kSumParts < np; j += 4 * kSumParts) {
                float v[4][nc];
#pragma unroll
                for (int k = 0; k < 4; k++)
#pragma unroll
                    for (int c = 0; c < nc; c++)
                        v[k][c] = stage[(j + k * kSumParts) * nc + c];
#pragma unroll
                for (int k = 0; k < 4; k++)
#pragma unroll
                    for (int c = 0; c < nc; c++) s += sum_elem<kSq>(v[k][c]);
            }
            for (; j < np; j += kSumParts)
#pragma unroll
                for (int c = 0; c < nc; c++)
                    s += sum_elem<kSq>(stage[j * nc + c]);
        }
        __syncthreads();
    }
    if (tid < kSumParts) parts[tid] = float(s);
    __syncthreads();
    double t = 0.0;
    if (tid == 0)
        for (int q = 0; q < kSumParts; q++) t += double(parts[q]);
    return float(t);
}

}  // namespace

// out[0] = SumAll(x) for x [n_px][nc] (op level).
__global__ void __launch_bounds__(kRmsThreads)
k_sum_all(const float* x, int n_px, int nc, float* out) {
    extern __shared__ float dyn[];
    float* stage = dyn;
    float* parts = dyn + kStageFloats;
    float s = 0.f;
    switch (nc) {
        case 1: s = sum_all_block<false, 1>(x, n_px, stage, parts); break;
        case 2: s = sum_all_block<false, 2>(x, n_px, stage, parts); break;
        case 3: s = sum_all_block<false, 3>(x, n_px, stage, parts); break;
        default: s = sum_all_block<false, 4>(x, n_px, stage, parts); break;
    }
    if (threadIdx.x == 0) out[0] = s;
}

// rms[b] = sqrt(SumAll(x_b * x_b) * inv_cnt + 1e-24) for x = (g, g_lap,
// g_nrm), one block each.
__global__ void __launch_bounds__(kRmsThreads)
k_reg_rms(const float* g, const float* glap, const float* gnrm, int n_verts,
          float inv_cnt, float* rms) {
    extern __shared__ float dyn[];
    float* stage = dyn;
    float* parts = dyn + kStageFloats;
    const float* x = blockIdx.x == 0 ? g : (blockIdx.x == 1 ? glap : gnrm);
    const float s = sum_all_block<true, 3>(x, n_verts, stage, parts);
    if (threadIdx.x == 0) rms[blockIdx.x] = sqrtf(s * inv_cnt + 1e-24f);
}

// Opts the SumAll kernels into kStageBytes of dynamic shared memory on the
// current device (host side, outside any stream capture).
void sum_all_setup() {
    DRESSI_CUDA(cudaFuncSetAttribute(
            k_sum_all, cudaFuncAttributeMaxDynamicSharedMemorySize,
            kStageBytes));
    DRESSI_CUDA(cudaFuncSetAttribute(
            k_reg_rms, cudaFuncAttributeMaxDynamicSharedMemorySize,
            kStageBytes));
}

// out = (g + glap * s_lap) + gnrm * s_nrm with s = rms(g) / rms(term) *
// weight (op level; out may alias g).
__global__ void k_reg_combine(const float* g, const float* glap,
                              const float* gnrm, const float* rms,
                              float laplacian, float normal, int n,
                              float* out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float sl = rms[0] / rms[1] * laplacian;
    const float sn = rms[0] / rms[2] * normal;
    out[i] = (g[i] + glap[i] * sl) + gnrm[i] * sn;
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
    if (n_verts <= 0 || (!lap_out && !nrm_out)) return;
    ProfScope ps("vertex_terms", s);
    const int part0 = lap_out ? 0 : 1;
    const int parts = (lap_out && nrm_out) ? 2 : 1;
    const dim3 grid((n_verts + kVtxThreads - 1) / kVtxThreads, parts);
    k_vertex_terms<<<grid, kVtxThreads, 0, s>>>(
            pos, n_verts, nbrs, nbr_deg, lap_diff ? 1 : 0, lap_out, term,
            faces, n_faces, vf, vf_deg, nrm_out, status, part0);
    check_launch();
}

void sum_all_op(const float* x, int n_px, int nc, float* out,
                cudaStream_t s) {
    ProfScope ps("sum_all", s);
    k_sum_all<<<1, kRmsThreads, kStageBytes, s>>>(x, n_px, nc, out);
    check_launch();
}

void reg_rms_op(const float* g, const float* glap, const float* gnrm,
                int n_verts, float* rms, cudaStream_t s) {
    ProfScope ps("reg_rms", s);
    k_reg_rms<<<3, kRmsThreads, kStageBytes, s>>>(
            g, glap, gnrm, n_verts, 1.f / float(n_verts * 3), rms);
    check_launch();
}

void reg_combine_op(const float* g, const float* glap, const float* gnrm,
                    const float* rms, float laplacian, float normal,
                    int n_verts, float* out, cudaStream_t s) {
    const int n = n_verts * 3;
    if (n <= 0) return;
    ProfScope ps("reg_combine", s);
    k_reg_combine<<<(n + 255) / 256, 256, 0, s>>>(g, glap, gnrm, rms,
                                                  laplacian, normal, n, out);
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
    reg_rms_op(b.gpos, r.glap, r.gnrm, p.n_verts, r.rms, s);
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
