// Internal host-side interface between the C ABI (capi.cu) and the kernel
// translation units. Not installed; the public surface is
// include/dressi_b200.h.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <vector>

#include "common.h"
#include "raster_soft.cuh"

namespace dressi {

// Shape of one soft-raster launch (all views share W, H and the face count).
struct SoftDims {
    int W = 0, H = 0, views = 1, n_faces = 0, n_verts = 0;
    float radius = 1.f;
    int tiles_x = 0, tiles_y = 0, n_tiles = 0;
    int rim_cells_x = 0, rim_cells = 0;
    int cap1 = 0, cap2 = 0;  // entries per sweep-1 tile / rim block bin
    int spill1 = 0, spill2 = 0;  // spill-list entries (all bins of a set)

    void finalize() {
        tiles_x = (W + kTile - 1) / kTile;
        tiles_y = (H + kTile - 1) / kTile;
        n_tiles = tiles_x * tiles_y;
        rim_cells_x = (W + kRimCell - 1) / kRimCell;
        rim_cells = rim_cells_x * ((H + kRimCell - 1) / kRimCell);
    }

    // Sweep arguments of view 0 (the kernels offset them per view).
    SweepArgs args(const FaceRec* recs, const int* rim, const float* prev,
                   uint32_t* status) const {
        SweepArgs a;
        a.recs = recs;
        a.n_faces = n_faces;
        a.W = W;
        a.H = H;
        a.tiles_x = tiles_x;
        a.n_tiles = n_tiles;
        a.v = 0;
        a.radius = radius;
        a.prev = prev;
        a.rim_cells_x = rim_cells_x;
        a.rim = rim;
        a.status = status;
        return a;
    }
};

// Device scratch of the soft rasterizer, carved from one allocation.
struct SoftBuffers {
    FaceRec* recs = nullptr;   // [views * n_faces]
    FixedBins1 bin1{};         // sweep-1 bins per 16x16 tile
    FixedBins bin2{};          // rim-phase bins per 8x4 block
    int2* state = nullptr;     // packed survivors [views * W * H]
    uint8_t* active = nullptr; // open flag per 8x4 block [views*n_tiles*8]
    // summed-area table of the open blocks per 16x16 tile, with a zero
    // first row and column: [views][(tiles_y + 1) * (tiles_x + 1)]
    int* sat = nullptr;
    int* kept = nullptr;    // faces near an open block [views][n_faces]
    int* kept_n = nullptr;  // their count per view [views]
    int* rim = nullptr;        // rim-possible flags [views * rim_cells]
    uint32_t* status = nullptr;
};

// Carves SoftBuffers out of `a` (a dry run with a.base == nullptr measures
// the size). The count arrays must be zero before the first use; the scan
// re-zeroes them after every use.
void carve_soft(Arena& a, const SoftDims& d, SoftBuffers* b);
// The same split in two: everything but the bins / the two bin sets (so a
// plan can grow its bins alone).
void carve_soft_main(Arena& a, const SoftDims& d, SoftBuffers* b);
void carve_soft_bins(Arena& a, const SoftDims& d, SoftBuffers* b);
// Zeroes the persistent counters of freshly carved buffers.
void init_soft(const SoftDims& d, const SoftBuffers& b, cudaStream_t s);

// Default tile-list capacities for a scene (entries per view).
void default_caps(SoftDims* d);

// The face-setup kernels fill the sweep-1 bins; after sweep 1 the rim
// binning fills the per-block bins of the open blocks.
void soft_rim_bins(const SoftDims& d, const SoftBuffers& b, cudaStream_t s);

// Launches sweep 1, the rim binning and the rim phase with an epilogue.
template <class Epi>
void launch_sweeps(const SoftDims& d, const SoftBuffers& b,
                   const float* prev_depth, const Epi& epi, cudaStream_t s) {
    const SweepArgs a = d.args(b.recs, b.rim, prev_depth, b.status);
    const dim3 grid(d.n_tiles, d.views);
    const size_t sr = size_t(d.n_faces), sp = size_t(d.W) * d.H,
                 sm = size_t(d.rim_cells);
    {
        ProfScope ps("sweep1", s);
        k_sweep1<Epi><<<grid, kSweep1Threads, 0, s>>>(a, b.bin1, b.bin2, b.state,
                                                    b.active, sr, sp, sm, epi);
    }
    DRESSI_CUDA(cudaGetLastError());
    {
        // tiles whose bins overflowed into the spill list (usually none)
        ProfScope ps("sweep1_spill", s);
        k_sweep1_spill<Epi><<<kSpillBlocks, kTileThreads, 0, s>>>(
                a, b.bin1, b.bin2, b.state, b.active, sr, sp, sm, epi);
    }
    DRESSI_CUDA(cudaGetLastError());
    soft_rim_bins(d, b, s);
    {
        ProfScope ps("rim_order", s);
        k_rim_order<<<148 * 2, 256, 0, s>>>(b.bin2, d.n_tiles, d.tiles_x);
    }
    DRESSI_CUDA(cudaGetLastError());
    {
        // split long lists (only when the open blocks are few)
        ProfScope ps("rim_seg", s);
        k_rim_seg<<<kRimCtas, kTileThreads, 0, s>>>(a, b.bin2, b.state, sr, sp,
                                                    sm);
    }
    DRESSI_CUDA(cudaGetLastError());
    {
        ProfScope ps("rim", s);
        k_rim<Epi><<<kRimCtas, kTileThreads, 0, s>>>(a, b.bin2, b.state, sr,
                                                     sp, sm, epi);
    }
    DRESSI_CUDA(cudaGetLastError());
    {
        ProfScope ps("rim_split_epi", s);
        k_rim_split_epi<Epi><<<148 * 2, 256, 0, s>>>(a, b.bin2, b.state, sr,
                                                     sp, sm, epi);
    }
    DRESSI_CUDA(cudaGetLastError());
    {
        ProfScope ps("rim_empty", s);
        k_rim_empty<Epi><<<148 * 4, 256, 0, s>>>(a, b.bin2, b.state, sr, sp,
                                                 sm, epi);
    }
    DRESSI_CUDA(cudaGetLastError());
}

// --- op-level soft raster (explicit soft geometry, one or more views) ---
struct SoftOpInputs {
    const float* soft_clip;   // [views][n_soft][4]
    const float* face_id;     // [views][n_soft]
    const float* faces_soft;  // [n_faces][3]  (shared by all views)
    const float* hard_clip;   // [views][n_hard][4]
    const float* faces_tex;   // [n_faces][3]  (shared)
    const float* prev_depth;  // [views][H][W] or null
    int n_soft, n_hard;
};
// Enqueues face setup, binning and both sweeps; writes out[views][H][W][4].
void soft_raster_op(const SoftDims& d, const SoftBuffers& b,
                    const SoftOpInputs& in, float* out, cudaStream_t s);

// --- exact GatherDistGrad + ColSum (op level) ---
// grad[views][n_verts][4] += d/d clip of sum_px gy * dist.
void dist_grad_op(const float* gy, const float* rs, const float* clip,
                  const float* faces, int views, int n_verts, int n_faces,
                  int W, int H, float* grad, uint32_t* status,
                  cudaStream_t s);

// --- SoftClip (op level) ---
void soft_clip_op(const float* clip, const float* faces, int views,
                  int n_verts, int n_faces, int W, int H, float radius,
                  float* out, uint32_t* status, cudaStream_t s);

// --- silhouette iteration (plan level) ---
struct SilParams {
    int n_verts, n_faces, views, res;
    float radius, sigma, lr, b1, b2, eps;
    float k;  // (2/R)^2 / sigma
    float c;  // 1 / R^2
    int n_samples;  // AA plans: stochastic edge samples (0: exact)
    // optimizer-side regulariser weights (run.cpp:407-420); reg = either
    // weight non-zero
    float laplacian, normal;
    int reg;
    // the paper's HardSoftRas path (paper.cu): peels layers, D = mask *
    // sigmoid(dist * sigma_scale) with sigma_scale = 7 / radius; n_samples
    // edge samples per face in FaceFetch's backward (0: exact)
    int paper, peels;
    float sigma_scale;
};
constexpr int kPaperMaxPeels = 4;
// Mesh tables and scratch of the regulariser (ids as float, -1 padding).
struct RegBuffers {
    float* nbrs;     // [nbr_deg][V] VertexNeighborsTex
    int nbr_deg;
    float* fadj;     // [F][3] FaceNeighborsTex
    float* vf;       // [vf_deg][V] VertexFacesTex
    int vf_deg;
    float* term;     // [F][3] NormalConsistencyFaceTerm
    float* glap;     // [V][3] pos - VertexNeighborMean
    float* gnrm;     // [V][3] NormalConsistencyVertexGrad
    float* rms;      // [3] rms(g), rms(g_lap), rms(g_nrm)
};
struct SilBuffers {
    float* pos;       // [V*3]
    float* adam_m;    // [V*3]
    float* adam_v;    // [V*3]
    float* scalars;   // [0]=t  [1]=bc1 [2]=bc2 [3]=last loss
    float* faces;     // [F*3]
    float* mvps;      // [views*16]
    float* targets;   // [views*R*R]
    float* clip;      // [views*V*4]
    float* gclip;     // [views*V*4]  zeroed by the Adam step
    float* gpos;      // [V*3]        last gradient (for inspection)
    double* loss_slots;  // [kLossSlots] zeroed by the Adam step
    float* loss_hist;    // [hist_cap]
    int hist_cap;
    unsigned* done;      // block-completion counter of the Adam step
    SoftBuffers soft;
    RegBuffers reg;      // p.reg only
    // p.paper only: the soft layers [peels][views*R*R], the peeling
    // threshold [views*R*R], the per-pixel gradients of the fetched corners
    // [peels][3][views*R*R]
    float4* paper_layers;
    float* paper_prev;
    float4* paper_gfetch;
    // Deterministic gradient mode (null = off): the epilogue writes each
    // pixel's (survivor face, dL/d dist) instead of scattering with float
    // atomics; det_face_op then gathers per face in pixel order and per
    // vertex in vertex -> face table order (the reference's GatherDistGrad
    // + ColSum order).
    float2* det_pix;   // [views*R*R] (face as int bits or -1, g)
    float4* det_part;  // [views*F*3] per-face corner partials (x, y, -, w)
    const float* det_vf;  // VertexFacesTex [vf_deg][V] (ids as float)
    int det_vf_deg;
    // faces that received a gradient pixel this iteration [views*F]: set by
    // the epilogue, read and cleared by the per-face gather
    uint8_t* det_touch;
};
constexpr int kLossSlots = 4096;
// Deterministic mode: partials per face, then g_clip per vertex.
void sil_det_gather(const SoftDims& d, const SilParams& p, const SilBuffers& b,
                    cudaStream_t s);
// Transform, raster, loss and per-view clip gradients (advances the Adam
// counter). rs_out (nullable) receives the RasterizeSoft images.
void sil_forward_backward(const SoftDims& d, const SilParams& p,
                          const SilBuffers& b, float* rs_out, cudaStream_t s);
// The soft-raster face records and bins of this iteration's clip positions.
void sil_face_setup(const SoftDims& d, const SilBuffers& b, cudaStream_t s);
// The paper path's per-pixel loss and fetched-corner gradients
// (paper_pixel.cu): one thread per pixel of every view.
void paper_pixel_launch(const SilParams& p, const float4* layers,
                        const float* targets, const float4* clip,
                        const float* faces, float4* gfetch,
                        double* loss_slots, unsigned blocks, cudaStream_t s);
// The paper path's forward/backward into g_clip (p.paper; called by
// sil_forward_backward). rs_out (nullable) receives layer 0.
void paper_forward_backward(const SoftDims& d, const SilParams& p,
                            const SilBuffers& b, float* rs_out,
                            cudaStream_t s);
// g_pos = sum_v MVP_v^T g_clip_v, the loss of the iteration, and (update)
// the Adam step.
void sil_grad_reduce(const SilParams& p, const SilBuffers& b, bool update,
                     cudaStream_t s);
// Adam step from an externally reduced g_pos (multi-GPU: after the
// all-reduce).
void sil_update(const SilParams& p, const SilBuffers& b, cudaStream_t s);
// clip = MVP (pos, 1) for every view; with `advance` also the Adam
// counter / bias corrections of the iteration. rim (nullable) rim flags to
// clear; status[1] is reset.
void sil_transform(const SilParams& p, const SilBuffers& b, int advance,
                   int* rim, int rim_cells, uint32_t* status, cudaStream_t s);
// clip = MVP (target_pos, 1) into b.clip (target rendering).
void sil_transform_plain(const SilParams& p, const SilBuffers& b,
                         const float* target_pos, cudaStream_t s);
// Regulariser terms of the current pos (g_lap, NC face term, g_nrm);
// depend on pos only, so they run before the gradient all-reduce.
void sil_reg_terms(const SilParams& p, const SilBuffers& b, cudaStream_t s);
// The regulariser's scales from the reduced g_pos (before the Adam step).
void sil_reg_scale(const SilParams& p, const SilBuffers& b, cudaStream_t s);
// The reference's mesh tables (mesh_utils.cpp:53-101), host side.
void vertex_faces_table(const float* faces, int n_faces, int n_verts,
                        std::vector<float>* out, int* max_deg);
void vertex_neighbors_table(const float* faces, int n_faces, int n_verts,
                            std::vector<float>* out, int* max_deg);
void face_neighbors_table(const float* faces, int n_faces,
                          std::vector<float>* out);
// Op level: NormalConsistencyFaceTerm, VertexNeighborMean (lap_diff: pos -
// mean) + NormalConsistencyVertexGrad (either output nullable), SumAll.
// Table ids out of range set kStatusIndexRange in status (nullable)
// and are skipped.
void nc_face_term_op(const float* pos, int n_verts, const float* faces,
                     const float* fadj, int n_faces, float* term,
                     uint32_t* status, cudaStream_t s);
void vertex_terms_op(const float* pos, int n_verts, const float* nbrs,
                     int nbr_deg, bool lap_diff, float* lap_out,
                     const float* term, const float* faces, int n_faces,
                     const float* vf, int vf_deg, float* nrm_out,
                     uint32_t* status, cudaStream_t s);
void sum_all_op(const float* x, int n_px, int nc, float* out, cudaStream_t s);
// Dynamic shared memory opt-in of the SumAll kernels on the current device;
// call before launching them (and before any stream capture).
void sum_all_setup();
// rms = {rms(g), rms(glap), rms(gnrm)} over [n_verts][3] each; out =
// (g + glap s_lap) + gnrm s_nrm, s = rms[0] / rms[1 | 2] * weight.
void reg_rms_op(const float* g, const float* glap, const float* gnrm,
                int n_verts, float* rms, cudaStream_t s);
void reg_combine_op(const float* g, const float* glap, const float* gnrm,
                    const float* rms, float laplacian, float normal,
                    int n_verts, float* out, cudaStream_t s);
// --- split-sum IBL ops (ibl.cu) ---
void equirect_sample_op(const float* map, int mw, int mh, int n,
                        const float* dir, long long n_px, float* out,
                        cudaStream_t s);
// g_map [mh][mw][n] is overwritten (zeroed, then scattered into).
void equirect_sample_bwd_op(const float* gy, const float* dir, long long n_px,
                            int mw, int mh, int n, float* g_map,
                            cudaStream_t s);
// Scratch floats of the convolutions: direction tables of both sides and
// the prefilter normaliser.
size_t env_conv_scratch_floats(int sw, int sh, int ow, int oh);
void irradiance_conv_op(const float* env, int sw, int sh, int n, int ow,
                        int oh, float* out, float* scratch, cudaStream_t s);
void irradiance_conv_bwd_op(const float* gy, int ow, int oh, int n, int sw,
                            int sh, float* g_env, float* scratch,
                            cudaStream_t s);
float prefilter_alpha(float roughness);
void prefilter_conv_op(const float* env, int sw, int sh, int n, int ow,
                       int oh, float roughness, float* out, float* scratch,
                       cudaStream_t s);
void prefilter_conv_bwd_op(const float* gy, int ow, int oh, int n, int sw,
                           int sh, float roughness, float* g_env,
                           float* scratch, cudaStream_t s);
void brdf_lut_op(int w, int h, int n_samples, float* out, cudaStream_t s);
void avg_pool2x2_op(const float* x, int w, int h, int n, float* out,
                    cudaStream_t s);
void avg_pool2x2_bwd_op(const float* gy, int w, int h, int n, float* g,
                        cudaStream_t s);
// Direction + sin(theta) table of a w x h equirect map.
void texel_dirs_op(int w, int h, float4* out, cudaStream_t s);
void prefilter_norm_op(const float4* src_dirs, int n_src,
                       const float4* out_dirs, int n_out, float alpha,
                       float* norm, cudaStream_t s);
// The convolutions over precomputed direction tables (kind 0 irradiance
// with scale 2 pi / n_src, kind 1 prefilter with alpha and norm);
// the transpose optionally accumulates into g_env.
void env_conv_run(int kind, const float* env, int n, const float4* src_dirs,
                  int n_src, const float4* out_dirs, int n_out,
                  float scale_or_alpha, const float* norm, float* out,
                  cudaStream_t s);
void env_conv_bwd_run(int kind, const float* gy, int n,
                      const float4* src_dirs, int n_src,
                      const float4* out_dirs, int n_out, float scale_or_alpha,
                      const float* norm, float* g_env, bool accumulate,
                      cudaStream_t s);

// A side stream and the two events of a fork / join, so that independent
// work of an iteration runs concurrently (a fork inside a stream capture
// becomes parallel branches of the graph).
struct StreamFork {
    cudaStream_t side = nullptr;
    cudaEvent_t begin = nullptr, end = nullptr;
};
// One full single-device iteration (fork: the regulariser's terms on the
// side stream; null: all on s).
void sil_iteration(const SoftDims& d, const SilParams& p,
                   const SilBuffers& b, cudaStream_t s,
                   const StreamFork* fork = nullptr);
// Renders hard silhouettes (face id > 0) of pos into targets (setup only).
void sil_render_targets(const SoftDims& d, const SilParams& p,
                        const SilBuffers& b, const float* target_pos,
                        cudaStream_t s);

// --- hard rasterizer (face id / attribute interpolation) ---
struct HardDims {
    int W = 0, H = 0, views = 1, n_faces = 0, n_verts = 0, n_comp = 1;
    int attr_ones = 0;  // the attribute is 1 at every vertex (a mask)
    int attr_shared = 0;  // one attribute array [V][n_comp] for all views
    // nvdiffrast-style output (dressi.torch rasterize): out [views][H][W][4]
    // = (u, v, z/w, face + 1) from the corner attributes (1,0,z,w), (0,1,
    // z,w), (0,0,z,w) with z, w = attr[views][V][4] (the GL clip position)
    int uvzw = 0;
    int tiles_x = 0, tiles_y = 0, n_tiles = 0, cap = 0;
    void finalize() {
        tiles_x = (W + kTile - 1) / kTile;
        tiles_y = (H + kTile - 1) / kTile;
        n_tiles = tiles_x * tiles_y;
    }
};
size_t hard_workspace_bytes(const HardDims& d);
// clip [views][V][4]; attr [views][V][n_comp] (null for face id, or with
// d.attr_ones for a constant 1); faces [F][3] shared. out: face id image
// [views][H][W] (no attribute) or the interpolated attribute
// [views][H][W][n_comp]. depth_out / id_out (nullable) also get the
// survivor's depth / the face-id image.
void hard_raster_op(const HardDims& d, void* workspace, const float* clip,
                    const float* attr, const float* faces, float* out,
                    float* depth_out, uint32_t* status, cudaStream_t s,
                    float* id_out = nullptr);

// --- screen-space AA (F::AntiAlias and its backward) ---
// Per (view, face): screen vertices in both projections the reference uses
// and the vertex ids (64 B).
struct __align__(16) AaFace {
    float qx0, qy0, qx1, qy1;  // ProjectToScreen (1/w product): pair tests
    float qx2, qy2;
    uint32_t i0, i1;
    float sx0, sy0, sx1, sy1;  // (c / w * 0.5 + 0.5) * size: sample placement
    float sx2, sy2;
    uint32_t i2, flags;        // 1: pair data valid, 2: sample data valid
};
static_assert(sizeof(AaFace) == 64, "AaFace layout");
struct AaDims {
    int W = 0, H = 0, views = 1, n_faces = 0, n_verts = 0, n_comp = 1;
};
// clip [views][V][4], faces [F][3] -> out [views][F]; view_flags
// [views] (zeroed here) marks views with wild screen coordinates.
void aa_face_setup(const AaDims& d, const float* clip, const float* faces,
                   AaFace* out, int* view_flags, uint32_t* status,
                   cudaStream_t s);
// img / out [views][H][W][n_comp], tri [views][H][W] (face id + 1).
void aa_forward_op(const AaDims& d, const AaFace* fr, const int* view_flags,
                   const float* img, const float* tri, float* out,
                   cudaStream_t s);
void aa_bwd_img_op(const AaDims& d, const AaFace* fr, const float* gy,
                   const float* tri, float* out, cudaStream_t s);
// grad [views][V][4] += d(sum gy * aa)/d clip; n_samples 0 = exact scan,
// else stochastic over vft [max_deg][V] seeded by `seed`.
// seed_dev (nullable): read the seed from device memory instead of `seed`.
void aa_bwd_vtx_op(const AaDims& d, const AaFace* fr, const float* gy,
                   const float* img, const float* tri, const float* clip,
                   const float* vft, int max_deg, float seed, int n_samples,
                   float* grad, cudaStream_t s,
                   const float* seed_dev = nullptr);

// --- AA silhouette (C4): hard raster + AntiAlias + stochastic vertex
// gradient, sharing the HardSoftRas plan's transform, gradient reduction
// and Adam.
struct AaSilBuffers {
    SilBuffers sil;     // pos / Adam / targets / clip / gclip / loss ...
    float* tri;         // [views][R][R] face id + 1 (the mask Rasterize(
                        // clip, ones) is 1 exactly where it is non-zero)
    float* gy;          // [views][R][R] dL / d pred
    AaFace* frs;        // [views][F]
    int* view_flags;    // [views]
    void* hard_ws;      // hard raster workspace (aa_sil_workspace_bytes)
    uint32_t* status;   // [4]
};
size_t aa_sil_workspace_bytes(const SilParams& p);
void aa_sil_forward_backward(const SilParams& p, const AaSilBuffers& b,
                             cudaStream_t s);
void aa_sil_iteration(const SilParams& p, const AaSilBuffers& b,
                      cudaStream_t s);
// The anti-aliased predictions of the current positions into out
// [views][R][R] (no gradient, counter unchanged).
void aa_sil_predict(const SilParams& p, const AaSilBuffers& b, float* out,
                    cudaStream_t s);
// targets = AntiAlias of the target mesh's mask (seed 0, forward only).
void aa_render_targets(const SilParams& p, const AaSilBuffers& b,
                       const float* target_pos, cudaStream_t s);

// --- texturing: op-level sampling and inverse-UV gathers ---
// filter: 0 nearest (GLSL texture() of a clamp-to-edge nearest sampler),
// 1 bilinear (BilerpClamp). tex [th][tw][n]; uv / out per pixel.
void texture_sample_op(const float* tex, int tw, int th, int n, int filter,
                       const float* uv, size_t npx, float* out,
                       cudaStream_t s);
// GatherByInverseUV (filter 0) / GatherByInverseUVBilinear (1): gy
// [sh][sw][n], inv_uv [th][tw][4], uv_screen [sh][sw][2] -> out [th][tw][n].
void texture_gather_op(const float* gy, int sw, int sh, int n, int filter,
                       const float* inv_uv, int tw, int th,
                       const float* uv_screen, float* out, cudaStream_t s);

// --- C2 texture optimisation (first principles: box mips, trilinear
// sampling, exact scatter transpose, Adam on level 0) ---
struct TexParams {
    int w_tex, levels, views, res, n_verts, n_faces;
    float lr, b1, b2, eps;
    float inv_n;  // 1 / (R * R * 3): the per-view Mean
    int scatter_runs;  // 1: run-merged warp scatter, 0: one atomic per tap
};
struct TexBuffers {
    float* pyr;       // mip pyramid, level 0 = the optimised texture
    float4* gpyr;     // its gradient, one (r, g, b, unused) per texel
                      // (levels > 0 zeroed by the mip build)
    float* grad;      // d loss / d level 0 [w][w][3]
    float* adam_m;    // [w][w][3]
    float* adam_v;
    float* scalars;   // [0]=t [1]=bc1 [2]=bc2 [3]=last loss
    float* clip;      // [views][V][4] (static)
    float* attr;      // [V][3] = (u, v, 1)
    float* faces;     // [F][3]
    float* gbuf;      // [views][R][R][3] = (u, v, mask)
    float* targets;   // [views][R][R][3]
    double* loss_slots;
    float* loss_hist;
    int hist_cap;
    void* hard_ws;
    uint32_t* status;
};
size_t tex_mip_floats(int w, int levels);
size_t tex_workspace_bytes(const TexParams& p);
// Forward + loss + d loss / d level 0 into grad (advances the Adam counter).
// The G-buffer (uv, mask) of every view: the geometry and cameras are fixed,
// so it is rasterised once at plan creation.
void tex_static_setup(const TexParams& p, const TexBuffers& b,
                      cudaStream_t s);
void tex_forward_backward(const TexParams& p, const TexBuffers& b,
                          float* pred_out, cudaStream_t s);
// Adam on level 0 from grad (and the loss of the iteration).
void tex_update(const TexParams& p, const TexBuffers& b, cudaStream_t s);
void tex_iteration(const TexParams& p, const TexBuffers& b, cudaStream_t s);
// out [views][R][R][3] = mask * trilinear(mips(texture)) of the current
// texture (no gradient, counter unchanged).
void tex_predict(const TexParams& p, const TexBuffers& b, float* out,
                 cudaStream_t s);
// targets = mask * trilinear(mips(gt_tex)) per view (gt_tex on the device).
void tex_render_targets(const TexParams& p, const TexBuffers& b,
                        const float* gt_tex, cudaStream_t s);

// --- indexed access of the paper's HardSoftRas (faces.cu) ---
void screen_coord_op(int w, int h, float* out, cudaStream_t s);
void lookup_faces_op(const float* attr, int n_verts, int n, const float* faces,
                     int n_faces, int corner, float* out, uint32_t* status,
                     cudaStream_t s);
void lookup_faces_bwd_op(const float* gy, int n, const float* faces,
                         int n_faces, const float* vf, int n_verts,
                         int max_deg, int corner, float* out,
                         uint32_t* status, cudaStream_t s);
void face_fetch_op(const float* attr, int n_faces, int n, const float* idx,
                   long long n_px, float* out, cudaStream_t s);
void face_fetch_bwd_op(const float* gy, int n, const float* idx, int w, int h,
                       const float* prj0, const float* prj1, const float* prj2,
                       int n_faces, float seed, float radius_px,
                       int n_samples, float* out, cudaStream_t s,
                       const float* seed_dev = nullptr);

// --- C5 PBR material + environment optimisation (pbr.cu) ---
constexpr int kPbrThreads = 512;
constexpr int kPbrMaxLevels = 8;
struct PbrDims {
    int views, res, tex, ew, eh, levels, n_verts, n_faces;
    int lut_w, lut_h, lut_samples, loss_kind;
    float inv_n;  // 1 / (R * R * 3): the per-view Mean
    float lr, b1, b2, eps;
    // IBL: irradiance out 32x16 from the env pooled to <= 64x32; the
    // prefilter levels from the env pooled to <= 128x64
    int irr_w, irr_h, irr_sw, irr_sh, pref_sw, pref_sh;
    int n_pool, pool_floats, pool_off[8];  // pooled levels ew/2, ew/4, ...
    int irr_pool, pref_pool;               // their source level (-1: env)
    int lw[kPbrMaxLevels], lh[kPbrMaxLevels];
    int loff[kPbrMaxLevels + 1];  // texel offsets; loff[levels] = the total
    int pref_texels;
    float alpha[kPbrMaxLevels];
    int dir_irr_src, dir_irr_out, dir_pref_src, dir_lvl[kPbrMaxLevels];
    int dir_count;
    int smem_level0;  // first prefilter level accumulated in shared memory
    int pixel_ctas;
};
struct PbrBuffers {
    float* px;        // [views][R*R][3 float4] pixel-static records
    float4* px_side;  // [views][R*R] (mask, background u, v, 0)
    float* target;    // [views][R*R][3] tone-mapped targets
    float* params;    // albedo [T*T*3] | mr [T*T*3] | env [eh*ew*3]
    float* grad;      // same layout
    float* adam_m;
    float* adam_v;
    float* scalars;   // t, bc1, bc2, loss
    float* pools;     // pooled env levels
    float* g_pools;
    float* irr;       // [16][32][3]
    float* g_irr;
    float* pref;      // levels concatenated [texels][3]
    float* g_pref;
    float* pref_norm; // [texels]
    float4* dirs;     // direction tables
    float* lut;       // [lut_h][lut_w][2]
    // per-iteration float4 copies gathered by the pixel kernel
    float4* mat4;     // [T*T] (albedo rgb, roughness)
    float* metal;     // [T*T]
    float4* env4;     // [eh*ew] (rgb, 0)
    float4* ibl4;     // irradiance texels, then the prefilter texels
    // material gradient accumulators (folded into grad, then cleared)
    float4* gmat4;    // [T*T] (d albedo rgb, d roughness)
    float* gmetal;    // [T*T]
    double* loss_slots;
    float* loss_hist;
    int hist_cap;
    // set-up only
    float* pos;       // [V][3] (also the world-position attribute)
    float* nrm;       // [V][3]
    float* uvh_attr;  // [V][4] = (u, v, 1, 0)
    float* faces;     // [F][3]
    float* mvps;      // [views][16]
    float* frames;    // [views][12]
    float* light;     // [6]
    float* clip;      // [views][V][4]
    void* hard_ws;
    float* gbuf_uvh;  // [views][R*R][4]
    float* gbuf_n;    // [views][R*R][3]
    float* gbuf_p;    // [views][R*R][3]
    uint32_t* status;
};
__global__ void k_pbr_static(PbrDims d, const float* uvh, const float* nrm,
                             const float* wpos, const float* frames,
                             const float* light, float4* rec,
                             float4* side);
size_t pbr_smem_bytes(const PbrDims& d);
// Sets the pixel kernel's shared-memory limit; its resident CTAs per SM.
int pbr_pixel_blocks_per_sm(const PbrDims& d);
// Direction tables, normalisers, the LUT, the G-buffer and the
// pixel-static records (plan creation).
void pbr_static_setup(const PbrDims& d, const PbrBuffers& b, cudaStream_t s);
// Forward + loss + gradient of [albedo | mr | env] into grad (advances the
// Adam counter; publishes the loss).
void pbr_forward_backward(const PbrDims& d, const PbrBuffers& b,
                          cudaStream_t s);
void pbr_update(const PbrDims& d, const PbrBuffers& b, cudaStream_t s);
void pbr_iteration(const PbrDims& d, const PbrBuffers& b, cudaStream_t s);
// out [views][R][R][3] = the tone-mapped render of params.
void pbr_render(const PbrDims& d, const PbrBuffers& b, const float* params,
                float* out, cudaStream_t s);

// --- dressi.torch-style interpolation (interp.cu) ---// --- dressi.torch-style interpolation (interp.cu) ---
// attr [attr_views][V][n_comp] (attr_views 1: shared), rast
// [views][H][W][4] -> out [views][H][W][n_comp]; the grad ADDS into
// grad [attr_views][V][n_comp].
void interpolate_op(const float* attr, int n_comp, int n_verts,
                    int attr_views, const float* rast, const float* faces,
                    int n_faces, int views, int W, int H, float* out,
                    uint32_t* status, cudaStream_t s);
void interpolate_grad_op(const float* gy, int n_comp, int n_verts,
                         int attr_views, const float* rast, const float* faces,
                         int n_faces, int views, int W, int H, float* grad,
                         uint32_t* status, cudaStream_t s);

// --- image fitting (C1) ---
struct FitBuffers {
    float* param;   // [n]
    float* target;  // [n]
    float* m;       // [n]
    float* v;       // [n]
    float* scalars; // [0]=t [3]=last loss
    double* loss_acc;  // [1]
    float* loss_hist;
    int hist_cap;
    unsigned* done;
};
void fit_iteration(size_t n, float lr, const FitBuffers& b, cudaStream_t s);

}  // namespace dressi
