/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for opendressi_b200.
 *
 * A plain-C restatement of the reference (unclearness/opendressi) CPU
 * algorithms on the Dressi-AD silhouette hot path. Each function cites the
 * reference file:line it follows. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference arm may load liboracle.so; the product
 * path never calls it.
 *
 * Pinned against: (1) the reference's own known-answer tests, re-expressed
 * in tests/test_oracle.py (tests/test_softras.cpp:92-137,
 * tests/test_cpu_eval.cpp:310-474 of the reference), and (2) the compiled
 * reference itself (oracle/_ref, ref_driver.cpp) on seeded random scenes,
 * bit-exact for raster outputs; see tests/golden/make_golden.py.
 *
 * Conventions (reference src/core/cpu_raster.h:8-13): screen =
 * (clip.xy / clip.w * 0.5 + 0.5) * (W, H), row 0 on top, pixel centres at
 * +0.5, depth = clip.z / clip.w in [0, 1]. Images are row-major with
 * interleaved components. Index arrays ("faces") are float-valued, as in
 * the reference's image leaves.
 */
#ifndef DRESSI_ORACLE_H
#define DRESSI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error text of the last failing call on this thread. */
const char* orc_last_error(void);

/* F::SoftClip -> out[3F*4] (f_ops.cpp:1890-1981). */
int orc_soft_clip(const float* clip, uint32_t n_verts, const float* faces,
                  uint32_t n_faces, uint32_t w, uint32_t h, float radius,
                  float* out);

/* RasterizeSoftCpu -> out[W*H*4] = (dist_px, face_id, hard_z, coverage)
 * (cpu_raster.cpp:241-355). prev_depth (nullable) = depth-peeling input. */
int orc_rasterize_soft(const float* soft_clip, uint32_t n_soft,
                       const float* face_id, const float* faces_soft,
                       uint32_t n_faces, const float* hard_clip,
                       uint32_t n_hard, const float* faces_tex, uint32_t w,
                       uint32_t h, float radius, const float* prev_depth,
                       float* out);

/* RasterizeFaceIdCpu -> out[W*H] (cpu_raster.cpp:357-369). */
int orc_rasterize_face_id(const float* clip, uint32_t n_verts,
                          const float* faces, uint32_t n_faces, uint32_t w,
                          uint32_t h, float* out);

/* RasterizeHardCpu -> out[W*H*n_comp] (cpu_raster.cpp:195-225). */
int orc_rasterize_hard(const float* clip, uint32_t n_verts, const float* attr,
                       uint32_t n_comp, const float* faces, uint32_t n_faces,
                       uint32_t w, uint32_t h, float* out);

/* ColSum(GatherDistGrad(gy, rs, clip, faces, vft)) -> grad[V*4]: the
 * gradient of sum_px gy(px)*dist(px) w.r.t. the hard clip positions
 * (f_ops.cpp:1248-1358 with ColSum 1218-1246). gy is W*H (the dist
 * channel's incoming gradient), rs the RasterizeSoft output. */
int orc_dist_grad(const float* gy, const float* rs, const float* clip,
                  uint32_t n_verts, const float* faces, uint32_t n_faces,
                  uint32_t w, uint32_t h, float* grad);

/* Clip transform (examples/common/geometry_utils.cpp:391-402):
 * clip[V*4] = rows x*m[r] + y*m[4+r] + z*m[8+r] + m[12+r]. */
void orc_transform_clip(const float* pos, uint32_t n_verts, const float* mvp,
                        float* clip);

/* One silhouette iteration's loss and position gradient (no update): the
 * graph of ref_driver.cpp's SilViewLoss summed over views. Returns the loss
 * (sum over pixels and views) in *loss; grad[V*3]. rs_out (nullable) gets
 * n_views*W*W*4 raster outputs. */
int orc_silhouette_loss_grad(const float* pos, uint32_t n_verts,
                             const float* faces, uint32_t n_faces,
                             uint32_t n_views, uint32_t res, float radius,
                             float sigma, const float* mvps,
                             const float* targets, double* loss, float* grad,
                             float* rs_out);
int orc_silhouette_loss_grad_mt(const float* pos, uint32_t n_verts,
                                const float* faces, uint32_t n_faces,
                                uint32_t n_views, uint32_t res, float radius,
                                float sigma, const float* mvps,
                                const float* targets, double* loss,
                                float* grad, float* rs_out,
                                uint32_t threads);

/* In-graph Adam of examples/silhouette_optimization/run.cpp:421-436, one
 * step over n params; t is the counter BEFORE the step (updated in place). */
void orc_adam(float* param, float* m, float* v, float* t, const float* grad,
              uint32_t n, float lr, float b1, float b2, float eps);

/* Full silhouette run: n_iters of loss/grad + Adam (lr, 0.9, 0.999, 1e-8).
 * loss_trace[n_iters]; pos updated in place. threads > 1 evaluates views
 * on that many threads (gradients summed in view order). */
int orc_silhouette_run(float* pos, uint32_t n_verts, const float* faces,
                       uint32_t n_faces, uint32_t n_views, uint32_t res,
                       float radius, float sigma, float lr, const float* mvps,
                       const float* targets, uint32_t n_iters,
                       uint32_t threads, float laplacian, float normal,
                       float* loss_trace);

/* F::AntiAlias forward (f_ops.cpp:2543-2575 over EvalAaPair,
 * cpu_raster.cpp:371-454): img/out W*H*n_comp, tri W*H (face id + 1). */
int orc_antialias(const float* img, uint32_t n_comp, const float* tri,
                  const float* clip, uint32_t n_verts, const float* faces,
                  uint32_t n_faces, uint32_t w, uint32_t h, float* out);

/* AntiAliasBwdImg (f_ops.cpp:2220-2278): out = d(sum gy*aa)/d img. */
int orc_antialias_bwd_img(const float* gy, uint32_t n_comp, const float* tri,
                          const float* clip, uint32_t n_verts,
                          const float* faces, uint32_t n_faces, uint32_t w,
                          uint32_t h, float* out);

/* AntiAliasBwdVtx (f_ops.cpp:2284-2476): grad[V*4] = d(sum gy*aa)/d clip.
 * n_samples == 0: the exact scan; > 0: the stochastic edge samples seeded
 * by `seed` (the {V,max_deg} partials summed in row order, as ColSum).
 * vft = VertexFacesTex {V,max_deg} (row d at vft[d*V]). */
int orc_antialias_bwd_vtx(const float* gy, const float* img, uint32_t n_comp,
                          const float* tri, const float* clip,
                          uint32_t n_verts, const float* faces,
                          uint32_t n_faces, const float* vft,
                          uint32_t max_deg, float seed, uint32_t n_samples,
                          uint32_t w, uint32_t h, float* grad);

/* HashToUnit (f_ops.cpp:1481-1486) over Wang's integer hash. */
float orc_hash_to_unit(uint32_t f, uint32_t s, uint32_t seed, uint32_t salt);

/* Anti-aliased target masks of a mesh (run.cpp:352-362 with seed 0 and the
 * exact backward): out[n_views*W*W]. */
int orc_aa_targets(const float* target_pos, uint32_t n_verts,
                   const float* faces, uint32_t n_faces, uint32_t n_views,
                   uint32_t res, const float* mvps, float* out);

/* One AA-silhouette iteration (C4; run.cpp:230-238 + 386-396): loss and
 * position gradient, views on `threads` threads. pred_out (nullable) gets
 * the n_views*W*W anti-aliased predictions. */
int orc_aa_silhouette_loss_grad(const float* pos, uint32_t n_verts,
                                const float* faces, uint32_t n_faces,
                                const float* vft, uint32_t max_deg,
                                uint32_t n_views, uint32_t res,
                                uint32_t n_samples, float seed,
                                const float* mvps, const float* targets,
                                uint32_t threads, double* loss, float* grad,
                                float* pred_out);

/* Full AA-silhouette run: n_iters of loss/grad (sampling seeded by the
 * in-graph Adam counter) + Adam (lr, 0.9, 0.999, 1e-8). */
int orc_aa_silhouette_run(float* pos, uint32_t n_verts, const float* faces,
                          uint32_t n_faces, const float* vft,
                          uint32_t max_deg, uint32_t n_views, uint32_t res,
                          uint32_t n_samples, float lr, const float* mvps,
                          const float* targets, uint32_t n_iters,
                          uint32_t threads, float laplacian, float normal,
                          float* loss_trace);

/* F::TextureBilinear forward (f_ops.cpp:2767-2778 over BilerpClamp,
 * ibl_math.h:91-115): tex [th][tw][n], uv [npx][2] -> out [npx][n]. */
int orc_texture_bilinear(const float* tex, uint32_t tw, uint32_t th,
                         uint32_t n, const float* uv, uint32_t npx,
                         float* out);
/* GatherByInverseUVBilinear (f_ops.cpp:2650-2732): gy [sh][sw][n], inv_uv
 * [th][tw][4], uv_screen [sh][sw][2] -> out [th][tw][n]. */
int orc_gather_inv_uv_bilinear(const float* gy, uint32_t sw, uint32_t sh,
                               uint32_t n, const float* inv_uv, uint32_t tw,
                               uint32_t th, const float* uv_screen,
                               float* out);
/* Nearest Texture / GatherByInverseUV: restated from the reference's GLSL
 * and sampler (no CPU kernel there; unpinned by reference outputs). */
int orc_texture_nearest(const float* tex, uint32_t tw, uint32_t th,
                        uint32_t n, const float* uv, uint32_t npx,
                        float* out);
int orc_gather_inv_uv(const float* gy, uint32_t sw, uint32_t sh, uint32_t n,
                      const float* inv_uv, uint32_t tw, uint32_t th,
                      const float* uv_screen, float* out);
/* UvAsClip / ScreenAttr (mesh_utils.cpp:180-203). */
void orc_uv_as_clip(const float* uv, uint32_t n_verts, float* out);
void orc_screen_attr(const float* clip, uint32_t n_verts, uint32_t sw,
                     uint32_t sh, float* out);

/* C2 texture path, first principles (no reference implementation): box
 * mip pyramid of a square power-of-two texture (levels concatenated,
 * orc_mip_floats floats), per-pixel lod from the G-buffer, trilinear
 * sampling and its exact transpose, and the mip-chain fold. */
size_t orc_mip_floats(uint32_t w, uint32_t n, uint32_t levels);
int orc_mip_build(const float* tex0, uint32_t w, uint32_t n, uint32_t levels,
                  float* pyr);
int orc_texture_lod(const float* uv, const float* mask, uint32_t W,
                    uint32_t H, uint32_t w_tex, uint32_t levels, float* lod);
int orc_texture_trilinear(const float* pyr, uint32_t w, uint32_t n,
                          uint32_t levels, const float* uv, const float* lod,
                          uint32_t npx, float* out);
int orc_texture_trilinear_grad(const float* g, uint32_t w, uint32_t n,
                               uint32_t levels, const float* uv,
                               const float* lod, uint32_t npx, float* gpyr);
void orc_mip_fold(float* gpyr, uint32_t w, uint32_t n, uint32_t levels);
/* One C2 iteration (loss, d loss / d tex) and a full Adam run. */
int orc_c2_loss_grad(const float* tex, uint32_t w_tex, uint32_t levels,
                     const float* pos, const float* uv_v, uint32_t n_verts,
                     const float* faces, uint32_t n_faces, const float* mvps,
                     uint32_t n_views, uint32_t res, const float* targets,
                     double* loss, float* grad, float* pred_out);
int orc_c2_run(float* tex, uint32_t w_tex, uint32_t levels, const float* pos,
               const float* uv_v, uint32_t n_verts, const float* faces,
               uint32_t n_faces, const float* mvps, uint32_t n_views,
               uint32_t res, const float* targets, float lr, uint32_t n_iters,
               float* loss_trace);

/* Mesh tables of the regularisers: VertexNeighborsTex (mesh_utils.cpp:
 * 73-86; {V,max_deg} row d at out[d*V]) and FaceNeighborsTex (88-101;
 * [F][3]); -1 padding. */
int orc_vertex_neighbors_tex(const float* faces, uint32_t n_faces,
                             uint32_t n_verts, uint32_t cap, float* out,
                             uint32_t* max_deg);
int orc_face_neighbors_tex(const float* faces, uint32_t n_faces, float* out);
/* The regulariser's ops: VertexNeighborMean (f_ops.cpp:1983-2029),
 * NormalConsistencyFaceTerm (2031-2098), NormalConsistencyVertexGrad
 * (2100-2181), SumAll (1119-1149, with SumPartial 1087-1115). */
void orc_vertex_neighbor_mean(const float* pos, uint32_t n_verts,
                              const float* vnbrs, uint32_t nbr_deg,
                              float* out);
void orc_nc_face_term(const float* pos, const float* faces, uint32_t n_faces,
                      const float* fadj, float* term);
void orc_nc_vertex_grad(const float* term, const float* pos, uint32_t n_verts,
                        const float* faces, const float* vft,
                        uint32_t vft_deg, float* out);
float orc_sum_all(const float* x, size_t n_px, uint32_t n_comp);
/* The silhouette optimizer's regularised gradient (run.cpp:407-420):
 * out = g + g_lap (rms(g)/rms(g_lap) laplacian) + g_nrm (rms(g)/rms(g_nrm)
 * normal); pos, g, out [V][3]. */
int orc_regularized_grad(const float* pos, uint32_t n_verts, const float* faces,
                         uint32_t n_faces, const float* vnbrs, uint32_t nbr_deg,
                         const float* fadj, const float* vft, uint32_t vft_deg,
                         const float* g, float laplacian, float normal,
                         float* out);

/* Split-sum IBL ops (C5; f_ops.cpp:2785-3415, ibl_math.h). Images are
 * [h][w][n] row-major, directions [n_px][3]. */
void orc_equirect_sample(const float* map, uint32_t mw, uint32_t mh,
                         uint32_t n, const float* dir, size_t n_px,
                         float* out);
int orc_equirect_sample_bwd(const float* gy, const float* dir, uint32_t dw,
                            uint32_t dh, uint32_t mw, uint32_t mh, uint32_t n,
                            float* g_map);
void orc_irradiance_conv(const float* env, uint32_t sw, uint32_t sh,
                         uint32_t n, uint32_t ow, uint32_t oh, float* out);
void orc_irradiance_conv_bwd(const float* gy, uint32_t ow, uint32_t oh,
                             uint32_t n, uint32_t sw, uint32_t sh,
                             float* g_env);
float orc_prefilter_alpha(float roughness);
void orc_prefilter_conv_norm(uint32_t ow, uint32_t oh, uint32_t sw,
                             uint32_t sh, float alpha, float* out);
void orc_prefilter_conv(const float* env, uint32_t sw, uint32_t sh,
                        uint32_t n, const float* norm, uint32_t ow,
                        uint32_t oh, float alpha, float* out);
void orc_prefilter_conv_bwd(const float* gy, const float* norm, uint32_t ow,
                            uint32_t oh, uint32_t n, uint32_t sw, uint32_t sh,
                            float alpha, float* g_env);
void orc_brdf_lut(uint32_t w, uint32_t h, uint32_t n_samples, float* out);
void orc_avg_pool2x2(const float* x, uint32_t w, uint32_t h, uint32_t n,
                     float* out);

/* PBR shading graph (C5; examples/common/pbr_graph.cpp:47-138, no normal
 * mapping). orc_pbr_static: the pixel-static terms (ndv, ndl, ndh, vdh,
 * (1-ndv)^5, (1-vdh)^5, radiance[3], n[3], refl[3]). orc_pbr_shade_grad:
 * per-pixel G-buffer and material images (identity uv), L1 (loss_kind 1)
 * or L2 (2) Mean loss against target, gradients w.r.t. albedo, mr and the
 * env through the IBL chain. frame = cam_pos, cam_fwd, cam_right, cam_up,
 * light_pos, light_col. */
#define ORC_PBR_STATIC 15
#define ORC_PBR_MAX_LEVELS 8
void orc_pbr_static(const float g_n[3], const float g_p[3],
                    const float cam_pos[3], const float light_pos[3],
                    const float light_col[3], float out[ORC_PBR_STATIC]);
int orc_pbr_shade_grad(uint32_t w, uint32_t h, const float* g_n,
                       const float* g_p, const float* mask,
                       const float* albedo, const float* mr, const float* ao,
                       const float* emissive, const float* frame,
                       const float* env, uint32_t ew, uint32_t eh, uint32_t L,
                       const float* lut, uint32_t lw, uint32_t lh,
                       const float* target, int loss_kind, float* mapped,
                       double* loss, float* g_albedo, float* g_mr,
                       float* g_env);
/* uv_img [h][w][2] (NULL: pixel centres); textures [th][tw][3]; with a uv
 * image ao / emissive are 1x1; gradients accumulate (+=). */
int orc_pbr_shade_grad_uv(uint32_t w, uint32_t h, const float* g_n,
                          const float* g_p, const float* mask,
                          const float* uv_img, uint32_t tw, uint32_t th,
                          const float* albedo, const float* mr,
                          const float* ao, const float* emissive,
                          const float* frame, const float* env, uint32_t ew,
                          uint32_t eh, uint32_t L, const float* lut,
                          uint32_t lw, uint32_t lh, const float* target,
                          int loss_kind, float* mapped, double* loss,
                          float* g_albedo, float* g_mr, float* g_env);

/* Indexed access of the paper's HardSoftRas (f_ops.cpp:1490-1799):
 * ScreenCoord; LookupFaces and its exact transpose over the vertex-face
 * table vf {V, max_deg} (row-major [max_deg][V], -1 padding); FaceFetch
 * and its backward (n_samples == 0: exact bbox scan; > 0: the hashed edge
 * samples). Gradients are written (not accumulated). */
void orc_screen_coord(uint32_t w, uint32_t h, float* out);
int orc_lookup_faces(const float* attr, uint32_t n_verts, uint32_t n,
                     const float* faces, uint32_t n_faces, uint32_t corner,
                     float* out);
int orc_lookup_faces_bwd(const float* gy, uint32_t n, const float* faces,
                         uint32_t n_faces, const float* vf, uint32_t n_verts,
                         uint32_t max_deg, uint32_t corner, float* out);
void orc_face_fetch(const float* attr, uint32_t n_faces, uint32_t n,
                    const float* idx, size_t n_px, float* out);
void orc_face_fetch_bwd(const float* gy, uint32_t n, const float* idx,
                        uint32_t w, uint32_t h, const float* prj0,
                        const float* prj1, const float* prj2,
                        uint32_t n_faces, float seed, float radius_px,
                        uint32_t n_samples, float* out);

/* 2-D image fitting (C1): loss = Mean((p - t)^2) over W*H*4, Adam on p.
 * loss_trace[n_iters] = loss at the start of each iteration. */
int orc_image_fit_run(float* param, const float* target, uint32_t w,
                      uint32_t h, float lr, uint32_t n_iters,
                      float* loss_trace);

/* VertexFacesTex (mesh_utils.cpp:53-69): out[V*cap] row-major {V,max_deg},
 * -1 padding; *max_deg set. Nonzero if cap is too small. */
int orc_vertex_faces_tex(const float* faces, uint32_t n_faces,
                         uint32_t n_verts, uint32_t cap, float* out,
                         uint32_t* max_deg);

#ifdef __cplusplus
}
#endif

#endif /* DRESSI_ORACLE_H */
