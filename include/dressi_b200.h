/*
 * dressi_b200.h -- C ABI of libdressi_b200.so, the B200 (sm_100a) device
 * layer of the Dressi-AD per-iteration hot path.
 *
 * Conventions
 *  - Plain C: pointers, sizes and an int status. 0 = success; on failure
 *    dressi_last_error() returns the message (thread-local), mirroring the
 *    reference's DressiError text (include/dressi/types.h:110-123).
 *  - Images are row-major with interleaved components and no VEC3 padding
 *    (the reference's CpuImage layout, include/dressi/types.h:72-88).
 *    Index images ("faces") are float-valued as in the reference's leaves.
 *  - Op-level entry points take DEVICE pointers and enqueue on `stream`
 *    (a cudaStream_t passed as void*; NULL = legacy default stream). Their
 *    scratch memory is allocated stream-ordered (cudaMallocAsync) and freed
 *    on the same stream.
 *  - Kernels never trap. A condition the reference reports by throwing
 *    (index out of range) sets a bit in a device status word instead; read it
 *    with dressi_plan_status() or the `status` argument of op-level calls
 *    (a device uint32_t the caller zeroes).
 *
 * Reference interfaces replaced (paths inside unclearness/opendressi):
 *  - DressiAD::execStep / sendImg / recvImg    include/dressi/dressi_ad.h:95-131
 *  - BuildGpuPlan / ExecuteGpuPlan             src/vk/executor.h:43-66
 *  - F::SoftClip                               include/dressi/f.h:236-242
 *  - F::RasterizeSoft (+ peel variant)         include/dressi/f.h:131-160
 *  - F::RasterizeFaceId / F::Rasterize         include/dressi/f.h:162-169, 116-118
 *  - RasterizeSoft backward (ColSum(GatherDistGrad))
 *                                              src/core/f_ops.cpp:1218-1358
 *  - dressi.torch.rasterize_soft / rasterize   python/dressi/torch/ops.py:682, 118
 *  - F::EquirectSample / IrradianceConv / PrefilterConv /
 *    BrdfIntegrationLut / AvgPool2x2      include/dressi/f.h (IBL ops)
 *  - F::VertexNeighborMean / NormalConsistency* / SumAll and the mesh
 *    tables of the silhouette optimizer         include/dressi/f.h:97, 240-255;
 *                                              include/dressi/mesh_utils.h:26-34
 */
#ifndef DRESSI_B200_H
#define DRESSI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DRESSI_B200_ABI_VERSION 1

/* status codes */
#define DRESSI_OK 0
#define DRESSI_ERR_INVALID 1  /* bad argument / shape (DressiError)        */
#define DRESSI_ERR_CUDA 2     /* CUDA runtime error                         */
#define DRESSI_ERR_OOM 3      /* device allocation failed                   */
#define DRESSI_ERR_DEVICE 4   /* device status word reported an error       */

/* device status word bits */
#define DRESSI_STATUS_INDEX_RANGE 0x1u  /* face/vertex index out of range   */
#define DRESSI_STATUS_BIN_OVERFLOW 0x2u /* tile list capacity exceeded; the */
                                        /* excess went to the spill lists   */
                                        /* (results stay exact)             */

/* ABI version of the loaded library (DRESSI_B200_ABI_VERSION). */
int dressi_abi_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to len). Returns its full length. */
int dressi_last_error(char* buf, size_t len);

/* ------------------------------------------------------------------------
 * Op-level entry points (device pointers)
 * --------------------------------------------------------------------- */

/* F::SoftClip (reference src/core/f_ops.cpp:1890-1981) for `views` stacked
 * clip images: clip [views][n_verts][4], faces [n_faces][3] (shared),
 * out [views][3*n_faces][4]. */
int dressi_soft_clip(const float* clip, uint32_t n_verts, const float* faces,
                     uint32_t n_faces, uint32_t views, uint32_t width,
                     uint32_t height, float radius_px, float* out,
                     uint32_t* status, void* stream);

/* F::RasterizeSoft (reference src/core/cpu_raster.cpp:241-355), bit-exact.
 *   soft_clip  [views][n_soft][4]   face_id [views][n_soft]
 *   faces_soft [n_faces][3]         hard_clip [views][n_hard][4]
 *   faces_tex  [n_faces][3]         prev_depth [views][H][W] or NULL
 *   out        [views][H][W][4] = (signed_dist_px, face_id, hard_z, coverage)
 * prev_depth != NULL selects the depth-peeling variant (f.h:149-160). */
int dressi_rasterize_soft(const float* soft_clip, uint32_t n_soft,
                          const float* face_id, const float* faces_soft,
                          uint32_t n_faces, const float* hard_clip,
                          uint32_t n_hard, const float* faces_tex,
                          uint32_t views, uint32_t width, uint32_t height,
                          float radius_px, const float* prev_depth,
                          float* out, uint32_t* status, void* stream);

/* RasterizeSoft's dist-channel backward, ColSum(GatherDistGrad(...))
 * (reference src/core/f_ops.cpp:1248-1358): ADDS to grad [views][n_verts][4]
 * the gradient of sum_px gy(px) * dist(px) w.r.t. the hard clip positions.
 * gy [views][H][W] (the dist channel's incoming gradient), rs the forward
 * output [views][H][W][4], clip [views][n_verts][4], faces [n_faces][3]. */
int dressi_rasterize_soft_grad(const float* gy, const float* rs,
                               const float* clip, uint32_t n_verts,
                               const float* faces, uint32_t n_faces,
                               uint32_t views, uint32_t width,
                               uint32_t height, float* grad, uint32_t* status,
                               void* stream);

/* F::RasterizeFaceId (cpu_raster.cpp:357-369), bit-exact: out [views][H][W]
 * = float(face)+1, 0 = background. depth_out (nullable) [views][H][W] gets
 * the survivor's NDC depth (1 = background). */
int dressi_rasterize_face_id(const float* clip, uint32_t n_verts,
                             const float* faces, uint32_t n_faces,
                             uint32_t views, uint32_t width, uint32_t height,
                             float* out, float* depth_out, uint32_t* status,
                             void* stream);

/* dressi_rasterize_face_id on a fixed scratch area; no counterpart in the
 * reference. Same arguments and output as dressi_rasterize_face_id, but it
 * allocates no device memory: its scratch is a 16 MiB file-scope device
 * array that every device loading the library holds until process exit.
 * For callers that cannot allocate during a call (a host framework's
 * allocator owns the free memory; latency-critical loops). A call whose
 * scratch need exceeds 16 MiB fails with DRESSI_ERR_INVALID; the need is
 * about views * (96 F + 12 T + 4 max(16 F, 4 T) + 16 K) bytes for F faces
 * and T 16x16-pixel tiles (one 1024x1024 view of 20480 faces: 3.4 MB).
 * The first call on a device looks up the scratch address (and may load the
 * module): make it outside any stream capture. A device reset
 * (cudaDeviceReset, or the primary context destroyed and re-created) can
 * move the array; the next call notices the new context and looks the
 * address up again, so it counts as a first call too. Calls that overlap in
 * time on one device share the scratch and race. */
int dressi_rasterize_face_id_noalloc(const float* clip, uint32_t n_verts,
                                     const float* faces, uint32_t n_faces,
                                     uint32_t views, uint32_t width,
                                     uint32_t height, float* out,
                                     float* depth_out, uint32_t* status,
                                     void* stream);

/* F::Rasterize (cpu_raster.cpp:195-225), bit-exact: perspective-correct
 * interpolation of attr [views][n_verts][n_comp] (n_comp 1..4);
 * out [views][H][W][n_comp]; background 0. */
int dressi_rasterize(const float* clip, uint32_t n_verts, const float* attr,
                     uint32_t n_comp, const float* faces, uint32_t n_faces,
                     uint32_t views, uint32_t width, uint32_t height,
                     float* out, uint32_t* status, void* stream);

/* F::AntiAlias (f_ops.cpp:2480-2579 over EvalAaPair, cpu_raster.cpp:
 * 371-454), bit-exact: Dr.Hair screen-space anti-aliasing of img
 * [views][H][W][n_comp] (n_comp 1..4) given the triangle-id image tri
 * [views][H][W] (float(face)+1, 0 = background), clip [views][n_verts][4]
 * and faces [n_faces][3]; out like img. */
int dressi_antialias(const float* img, uint32_t n_comp, const float* tri,
                     const float* clip, uint32_t n_verts, const float* faces,
                     uint32_t n_faces, uint32_t views, uint32_t width,
                     uint32_t height, float* out, uint32_t* status,
                     void* stream);

/* AntiAlias backward for an incoming gradient gy (like img):
 * grad_img (nullable, like img) = AntiAliasBwdImg (f_ops.cpp:2220-2278),
 * bit-exact; grad_clip (nullable) [views][n_verts][4] += AntiAliasBwdVtx
 * (f_ops.cpp:2284-2476): n_samples == 0 the exact scan of every boundary
 * pair, else n_samples stochastic edge samples per incident face, seeded
 * by `seed` (the graph's seed value) over the vertex -> face table vft
 * [max_deg][n_verts] (VertexFacesTex, mesh_utils.cpp:53-69; -1 padding). */
int dressi_antialias_grad(const float* gy, const float* img, uint32_t n_comp,
                          const float* tri, const float* clip,
                          uint32_t n_verts, const float* faces,
                          uint32_t n_faces, const float* vft,
                          uint32_t max_deg, float seed, uint32_t n_samples,
                          uint32_t views, uint32_t width, uint32_t height,
                          float* grad_img, float* grad_clip, uint32_t* status,
                          void* stream);

/* dressi.torch rasterize (python/dressi/torch/ops.py:96-163): out
 * [views][H][W][4] = (u, v, z/w, face + 1), 0 = background, computed as
 * the reference does it -- Rasterize of the unwelded corner attributes
 * (1,0,z,w), (0,1,z,w), (0,0,z,w) with clip_vk, RasterizeFaceId, and
 * z/w = g.z / (g.w + (1 - mask)) -- bit-exact. clip_vk [views][V][4] is the
 * Vulkan-depth clip position (z_vk = 0.5 (z_gl + w)), pos_gl [views][V][4]
 * the GL one whose z, w are interpolated. */
int dressi_rasterize_uvzw(const float* clip_vk, const float* pos_gl,
                          uint32_t n_verts, const float* faces,
                          uint32_t n_faces, uint32_t views, uint32_t width,
                          uint32_t height, float* out, uint32_t* status,
                          void* stream);

/* dressi.torch interpolate (ops.py:169-298): per pixel of a rasterize
 * output, u a0 + v a1 + (1 - u - v) a2 of the face's vertex attributes
 * (LookupFaces + FaceFetch, f_ops.cpp:1568-1799), bit-exact. attr
 * [attr_views][n_verts][n_comp] (attr_views 1: shared by the views). */
int dressi_interpolate(const float* attr, uint32_t n_comp, uint32_t n_verts,
                       uint32_t attr_views, const float* rast,
                       const float* faces, uint32_t n_faces, uint32_t views,
                       uint32_t width, uint32_t height, float* out,
                       uint32_t* status, void* stream);

/* Its exact VJP w.r.t. attr (FaceFetchBwd n=0 + LookupFacesBwd):
 * grad_attr [attr_views][n_verts][n_comp] += ..., gy like out. */
int dressi_interpolate_grad(const float* gy, uint32_t n_comp,
                            uint32_t n_verts, uint32_t attr_views,
                            const float* rast, const float* faces,
                            uint32_t n_faces, uint32_t views, uint32_t width,
                            uint32_t height, float* grad_attr,
                            uint32_t* status, void* stream);

/* F::Texture (filter 0: nearest, the reference's clamp-to-edge nearest
 * sampler, f_ops.cpp:2605-2639) / F::TextureBilinear (filter 1: BilerpClamp,
 * f_ops.cpp:2736-2780, bit-exact): tex [th][tw][n_comp] (n_comp 1..4)
 * sampled at uv [n_px][2] -> out [n_px][n_comp]. */
int dressi_texture(const float* tex, uint32_t tw, uint32_t th,
                   uint32_t n_comp, const float* uv, uint32_t n_px,
                   uint32_t filter, float* out, void* stream);

/* The texture gradient of dressi_texture through the inverse-UV table:
 * filter 0 GatherByInverseUV (restated from glsl_codegen.cpp:658-709),
 * filter 1 GatherByInverseUVBilinear (f_ops.cpp:2650-2732, bit-exact).
 * gy [sh][sw][n_comp], inv_uv [th][tw][4] (Rasterize(UvAsClip(uv),
 * ScreenAttr(clip)), mesh_utils.cpp:180-203), uv_screen [sh][sw][2] ->
 * grad_tex [th][tw][n_comp] (written). */
int dressi_texture_grad(const float* gy, uint32_t sw, uint32_t sh,
                        uint32_t n_comp, const float* inv_uv, uint32_t tw,
                        uint32_t th, const float* uv_screen, uint32_t filter,
                        float* grad_tex, void* stream);

/* Optimizer-side regulariser ops of the silhouette example
 * (examples/silhouette_optimization/run.cpp:407-420). Tables keep the
 * reference's layout: ids as float, -1 padding, {V, deg} tables row-major
 * with row d at [d * n_verts].
 *
 * VertexFacesTex / VertexNeighborsTex / FaceNeighborsTex (mesh_utils.cpp:
 * 53-101; HOST pointers, no device work): out holds cap * n_verts floats
 * ({V, deg} tables; *deg receives the table height, an error when above
 * cap) or 3 * n_faces floats (face neighbours). */
int dressi_vertex_faces_tex(const float* faces, uint32_t n_faces,
                            uint32_t n_verts, uint32_t cap, float* out,
                            uint32_t* deg);
int dressi_vertex_neighbors_tex(const float* faces, uint32_t n_faces,
                                uint32_t n_verts, uint32_t cap, float* out,
                                uint32_t* deg);
int dressi_face_neighbors_tex(const float* faces, uint32_t n_faces,
                              float* out);

/* F::VertexNeighborMean (f_ops.cpp:1983-2029): out [V][3] = mean of the
 * listed neighbours of each vertex (pos itself when it has none). In these
 * ops a table id out of range sets DRESSI_STATUS_INDEX_RANGE in `status`
 * (a device word, nullable) and is skipped. */
int dressi_vertex_neighbor_mean(const float* pos, uint32_t n_verts,
                                const float* nbrs, uint32_t nbr_deg,
                                float* out, uint32_t* status, void* stream);

/* F::NormalConsistencyFaceTerm (f_ops.cpp:2031-2098): out [F][3] from pos
 * [V][3], faces [F][3] and face_adj [F][3]. */
int dressi_normal_consistency_face_term(const float* pos, uint32_t n_verts,
                                        const float* faces, uint32_t n_faces,
                                        const float* face_adj, float* out,
                                        uint32_t* status, void* stream);

/* F::NormalConsistencyVertexGrad (f_ops.cpp:2100-2181): out [V][3] from
 * the face term [F][3], pos, faces and vtx_faces {V, vf_deg}. */
int dressi_normal_consistency_vertex_grad(const float* term, const float* pos,
                                          uint32_t n_verts, const float* faces,
                                          uint32_t n_faces,
                                          const float* vtx_faces,
                                          uint32_t vf_deg, float* out,
                                          uint32_t* status, void* stream);

/* F::SumAll (f_ops.cpp:1119-1149, with SumPartial's 64 strided double
 * partials above 256 pixels): out (1 device float) = the sum of x
 * [n_px][n_comp], bit-identical to the reference's CPU evaluator. */
int dressi_sum_all(const float* x, uint32_t n_px, uint32_t n_comp, float* out,
                   void* stream);

/* The whole regulariser: out [V][3] = g + g_lap (rms(g) / rms(g_lap)
 * laplacian) + g_nrm (rms(g) / rms(g_nrm) normal), g_lap = pos -
 * VertexNeighborMean(pos), g_nrm = NormalConsistencyVertexGrad(
 * NormalConsistencyFaceTerm(pos)), rms(x) = sqrt(SumAll(x*x) / (3V) +
 * 1e-24); out may alias g. */
int dressi_regularized_grad(const float* pos, uint32_t n_verts,
                            const float* faces, uint32_t n_faces,
                            const float* nbrs, uint32_t nbr_deg,
                            const float* face_adj, const float* vtx_faces,
                            uint32_t vf_deg, const float* g, float laplacian,
                            float normal, float* out, uint32_t* status,
                            void* stream);

/* Split-sum IBL ops (config C5; f_ops.cpp:2785-3415, ibl_math.h). Maps
 * are equirect images [h][w][n_comp] (n_comp 1..4), directions [n_px][3].
 * Within float tolerance of the reference (its transcendentals are the
 * host libm's, here CUDA's); AvgPool2x2 bit-exact.
 *
 * F::EquirectSample: 4-tap bilinear (u wraps, v clamps) along the
 * normalised direction, 0 for |dir| < 1e-8; its map transpose (g_map
 * written). */
int dressi_equirect_sample(const float* map, uint32_t mw, uint32_t mh,
                           uint32_t n_comp, const float* dir, uint64_t n_px,
                           float* out, void* stream);
int dressi_equirect_sample_grad(const float* gy, const float* dir,
                                uint64_t n_px, uint32_t mw, uint32_t mh,
                                uint32_t n_comp, float* g_map, void* stream);
/* F::IrradianceConv (E(N)/pi of env [sh][sw] into [oh][ow]) and its exact
 * transpose (g_env written). */
int dressi_irradiance_conv(const float* env, uint32_t sw, uint32_t sh,
                           uint32_t n_comp, uint32_t ow, uint32_t oh,
                           float* out, void* stream);
int dressi_irradiance_conv_grad(const float* gy, uint32_t ow, uint32_t oh,
                                uint32_t n_comp, uint32_t sw, uint32_t sh,
                                float* g_env, void* stream);
/* F::PrefilterConv (GGX-NDF-weighted, normalised by PrefilterConvNorm,
 * alpha = max(roughness, 0.045)^2) and its exact transpose. */
int dressi_prefilter_conv(const float* env, uint32_t sw, uint32_t sh,
                          uint32_t n_comp, uint32_t ow, uint32_t oh,
                          float roughness, float* out, void* stream);
int dressi_prefilter_conv_grad(const float* gy, uint32_t ow, uint32_t oh,
                               uint32_t n_comp, uint32_t sw, uint32_t sh,
                               float roughness, float* g_env, void* stream);
/* F::BrdfIntegrationLut: out [h][w][2] = (A, B) over (NdotV, roughness). */
int dressi_brdf_lut(uint32_t w, uint32_t h, uint32_t n_samples, float* out,
                    void* stream);
/* F::AvgPool2x2 (even sizes; out [h/2][w/2][n]) and its transpose (g_x
 * [h][w][n] written). */
int dressi_avg_pool2x2(const float* x, uint32_t w, uint32_t h,
                       uint32_t n_comp, float* out, void* stream);
int dressi_avg_pool2x2_grad(const float* gy, uint32_t w, uint32_t h,
                            uint32_t n_comp, float* g_x, void* stream);

/* ------------------------------------------------------------------------
 * Indexed access of the paper's HardSoftRas (f_ops.cpp:1490-1799). Device
 * pointers, float ids (the reference's leaves), n_comp 1..4; each output is
 * written. A table id out of range sets DRESSI_STATUS_INDEX_RANGE in
 * `status` (nullable) and reads nothing.
 * ---------------------------------------------------------------------- */

/* F::ScreenCoord({w, h}): out [h][w][2] = (x + 0.5, y + 0.5); a uniform
 * size ({1, 1}) is rejected, as by the reference. */
int dressi_screen_coord(uint32_t w, uint32_t h, float* out, void* stream);

/* F::LookupFaces(vtx_attr, faces, vtx_faces, corner): out [F][n] =
 * attr[faces[f][corner]]. */
int dressi_lookup_faces(const float* attr, uint32_t n_verts, uint32_t n_comp,
                        const float* faces, uint32_t n_faces, uint32_t corner,
                        float* out, uint32_t* status, void* stream);
/* Its exact transpose (LookupFacesBwd): g_attr [V][n] = sum of gy[f] over
 * the faces of v's VertexFacesTex list (vf {V, max_deg}: [max_deg][V], -1
 * padding) whose corner `corner` is v, in list order. */
int dressi_lookup_faces_grad(const float* gy, uint32_t n_comp,
                             const float* faces, uint32_t n_faces,
                             const float* vf, uint32_t n_verts,
                             uint32_t max_deg, uint32_t corner, float* g_attr,
                             uint32_t* status, void* stream);

/* F::FaceFetch forward: out [h][w][n] = attr[idx(p) - 1] (0 where idx is
 * 0 or past the table). */
int dressi_face_fetch(const float* attr, uint32_t n_faces, uint32_t n_comp,
                      const float* idx, uint32_t w, uint32_t h, float* out,
                      void* stream);
/* FaceFetchBwd: g_attr [F][n]. n_samples == 0: the exact VJP (each face's
 * screen bbox +-1 px scanned); > 0: the paper's hashed edge samples
 * (band +-radius_px, jitter `seed`). prj0..2 [F][4]: the corners' clip
 * positions (LookupFaces of the clip positions). */
int dressi_face_fetch_grad(const float* gy, uint32_t n_comp, const float* idx,
                           uint32_t w, uint32_t h, const float* prj0,
                           const float* prj1, const float* prj2,
                           uint32_t n_faces, float seed, float radius_px,
                           uint32_t n_samples, float* g_attr, void* stream);

/* ------------------------------------------------------------------------
 * Plans: one fused fwd + bwd + Adam iteration, resident on one device,
 * replayed as a CUDA graph with no per-iteration host traffic
 * (the reference's one pre-recorded command buffer per execStep,
 * src/vk/executor.cpp:42-907, :1020-1026).
 * --------------------------------------------------------------------- */

typedef struct dressi_plan_s* dressi_plan;

/* Buffer slots of a plan (upload / download / buffer address). */
enum {
    DRESSI_SLOT_PARAM = 0,   /* optimised parameter (pos [V][3] / image)   */
    DRESSI_SLOT_ADAM_M = 1,  /* Adam first moment (same shape)             */
    DRESSI_SLOT_ADAM_V = 2,  /* Adam second moment                         */
    DRESSI_SLOT_ADAM_T = 3,  /* Adam counter t (1 float)                   */
    DRESSI_SLOT_TARGET = 4,  /* target images                              */
    DRESSI_SLOT_GRAD = 5,    /* last gradient of the parameter             */
    DRESSI_SLOT_LOSS = 6,    /* loss of the last iteration (1 float)       */
    DRESSI_SLOT_LOSS_HISTORY = 7, /* ring of per-iteration losses          */
    DRESSI_SLOT_RASTER = 8,  /* silhouette: images of the last             */
                             /* dressi_plan_render(): RasterizeSoft        */
                             /* [views][R][R][4], AA predictions [views][R][R] */
    DRESSI_SLOT_MVP = 9      /* silhouette: view matrices [views][16]      */
};

/* Silhouette optimisation (configs C3/C4): HardSoftRas with RasterizeSoft's
 * exact dist-channel backward. Per view v: clip = MVP_v (pos, 1);
 * rs = RasterizeSoft(SoftClip(clip)); pred = max(cov*step(0,d),
 * cov*sigmoid(d*|d|*k)), k = (2/R)^2/sigma; loss = sum (target - pred)^2/R^2;
 * Adam on pos. faces/mvps are host arrays copied at creation. */
typedef struct {
    uint32_t struct_size;  /* sizeof(dressi_silhouette_desc) */
    uint32_t n_verts, n_faces, n_views, res;
    float radius_px, sigma, lr, beta1, beta2, eps;
    const float* faces;    /* host [n_faces][3] */
    const float* mvps;     /* host [n_views][16], column-major */
    uint32_t loss_history; /* ring capacity (0 -> 4096) */
    int device;            /* CUDA device ordinal */
    /* optimizer-side regulariser weights relative to the data-gradient RMS
     * (run.cpp:407-420; the example's defaults are 0.15 / 0.4); 0 / 0 =
     * none */
    float laplacian, normal;
} dressi_silhouette_desc;

int dressi_silhouette_plan_create(const dressi_silhouette_desc* desc,
                                  dressi_plan* out);

/* The silhouette example's own HardSoftRas technique, the paper path
 * (examples/silhouette_optimization/run.cpp:229-396): `peels` (1..4) soft
 * layers, each pixel's D_k = mask * sigmoid(signed distance to its face's
 * edges * 7 / radius_px) from the corners fetched with FaceFetch of
 * LookupFaces, pred = max(hard, 1 - prod_k (1 - D_k)); FaceFetch's backward
 * takes n_samples hashed edge samples per face (0: the exact bbox scan),
 * jittered by the Adam counter. Same descriptor as above (sigma unused),
 * same slots, targets, regulariser and phases. */
int dressi_paper_silhouette_plan_create(const dressi_silhouette_desc* desc,
                                        uint32_t peels, uint32_t n_samples,
                                        dressi_plan* out);

/* AA silhouette optimisation (config C4; examples/silhouette_optimization/
 * run.cpp:230-238): per view v, clip = MVP_v (pos, 1); mask =
 * Rasterize(clip, ones); tri = RasterizeFaceId(clip); pred =
 * AntiAlias(mask, tri, clip) with the vertex gradient from n_samples
 * stochastic edge samples per face seeded by the Adam counter (0: the
 * exact scan); loss = sum (target - pred)^2 / R^2; Adam on pos. Targets
 * (dressi_plan_render_targets) are the anti-aliased target masks. */
typedef struct {
    uint32_t struct_size;  /* sizeof(dressi_aa_silhouette_desc) */
    uint32_t n_verts, n_faces, n_views, res;
    uint32_t n_samples;    /* 8 in the reference example; 0 = exact */
    float lr, beta1, beta2, eps;
    const float* faces;    /* host [n_faces][3] */
    const float* mvps;     /* host [n_views][16], column-major */
    uint32_t loss_history; /* ring capacity (0 -> 4096) */
    int device;            /* CUDA device ordinal */
    /* regulariser weights as in dressi_silhouette_desc (the example's
     * defaults for this technique are 0.5 / 0.5); 0 / 0 = none */
    float laplacian, normal;
} dressi_aa_silhouette_desc;

int dressi_aa_silhouette_plan_create(const dressi_aa_silhouette_desc* desc,
                                     dressi_plan* out);

/* Texture optimisation (config C2): a fixed UV-mapped mesh seen from
 * n_views cameras; per view the G-buffer (uv, mask) = Rasterize(clip,
 * (u, v, 1)), pred = mask * trilinear(mips(tex), uv) with `levels` box-
 * filtered mip levels and a per-pixel lod from the uv differences, loss =
 * sum_v Mean((target - pred)^2); Adam on the [tex_size][tex_size][3]
 * texture (PARAM slot). Targets: dressi_plan_render_targets with the
 * target TEXTURE (host [tex_size][tex_size][3]).
 * The mip path has no counterpart in the reference (which samples one
 * level); it is defined here:
 *  - level l + 1 texel (x, y) = 0.25 * (((a + b) + c) + d) of the level-l
 *    texels a = (2x, 2y), b = (2x+1, 2y), c = (2x, 2y+1), d = (2x+1, 2y+1);
 *  - per covered pixel, du_x = uv(x+1, y) - uv(x, y) if the right
 *    neighbour is covered and inside the screen, else uv(x, y) - uv(x-1, y)
 *    if the left one is, else 0 (du_y likewise with the rows);
 *    rho = max(|du_x|, |du_y|) * tex_size (Euclidean lengths);
 *  - lod = 0 for rho <= 1, else e + (m - 1) with rho = m 2^e, m in [1, 2)
 *    (a piecewise-linear log2, exact in float), clamped to levels - 1;
 *  - sample = (1 - f) B(l0) + f B(l0 + 1), l0 = floor(lod), f = lod - l0,
 *    B(l) the clamp-to-edge bilinear tap set of level l at uv (the
 *    reference's BilerpClamp); f = 0 or l0 = levels - 1 uses B(l0) alone;
 *  - the backward is the exact transpose: every tap weight times the
 *    pixel's gradient added to the level's texel, then the chain
 *    acc_l = g_l + 0.25 acc_(l+1) folded down to level 0. */
typedef struct {
    uint32_t struct_size;  /* sizeof(dressi_texture_desc) */
    uint32_t n_verts, n_faces, n_views, res;
    uint32_t tex_size;     /* square, power of two */
    uint32_t levels;       /* mip levels (1 = level 0 only) */
    float lr, beta1, beta2, eps;
    const float* pos;      /* host [n_verts][3] */
    const float* uv;       /* host [n_verts][2] */
    const float* faces;    /* host [n_faces][3] */
    const float* mvps;     /* host [n_views][16], column-major */
    uint32_t loss_history; /* ring capacity (0 -> 4096) */
    int device;
} dressi_texture_desc;

int dressi_texture_plan_create(const dressi_texture_desc* desc,
                               dressi_plan* out);

/* 2-D image fitting (config C1): loss = Mean((param - target)^2) over a
 * [h][w][4] image, Adam(lr, 0.9, 0.999, 1e-8) on param. */
/* PBR material + environment optimisation (config C5): a fixed UV mesh
 * seen from n_views cameras, GGX Cook-Torrance with split-sum IBL
 * (examples/common/pbr_graph.cpp:47-138, no normal mapping, ao = 1,
 * emissive = 0; irradiance 32x16 from the env pooled to <= 64x32,
 * `levels` PrefilterConv levels from the env pooled to <= 128x64, a
 * lut_size^2 BRDF LUT), a per-view Mean L1 (loss_kind 1) or L2 (2) of the
 * Reinhard-mapped render against the targets, Adam on the PARAM slot
 * [albedo tex^2 x 3 | metallic-roughness tex^2 x 3 (G = roughness, B =
 * metallic) | env env_h x env_w x 3] with the maps clamped to [0, 1] and
 * the env to >= 0. Targets: dressi_plan_render_targets with the
 * ground-truth parameters in that layout (host). */
typedef struct {
    uint32_t struct_size;  /* sizeof(dressi_pbr_desc) */
    uint32_t n_verts, n_faces, n_views, res;
    uint32_t tex_size;     /* square material maps */
    uint32_t env_w, env_h; /* powers of two */
    uint32_t levels;       /* prefilter levels, 2..8 */
    uint32_t lut_size, lut_samples;  /* 256, 512 in the reference */
    uint32_t loss_kind;    /* 1 = L1, 2 = L2 */
    float lr, beta1, beta2, eps;
    const float* pos;      /* host [n_verts][3] world positions */
    const float* normal;   /* host [n_verts][3] */
    const float* uv;       /* host [n_verts][2] */
    const float* faces;    /* host [n_faces][3] */
    const float* mvps;     /* host [n_views][16], column-major */
    const float* frames;   /* host [n_views][12]: cam_pos, cam_fwd,
                              cam_right * tan(fov/2) * aspect,
                              cam_up * tan(fov/2) */
    const float* light;    /* host [6]: light position, light colour */
    uint32_t loss_history; /* ring capacity (0 -> 4096) */
    int device;
} dressi_pbr_desc;

int dressi_pbr_plan_create(const dressi_pbr_desc* desc, dressi_plan* out);

int dressi_image_fit_plan_create(uint32_t width, uint32_t height, float lr,
                                 int device, dressi_plan* out);

/* Host (or device, if src_is_device) -> slot copy on `stream`; `bytes` must
 * equal the slot size (sizes in dressi_plan_slot_bytes). */
int dressi_plan_upload(dressi_plan p, int slot, const void* src, size_t bytes,
                       int src_is_device, void* stream);
int dressi_plan_download(dressi_plan p, int slot, void* dst, size_t bytes,
                         int dst_is_device, void* stream);
int dressi_plan_slot_bytes(dressi_plan p, int slot, size_t* bytes);
/* Device address of a slot (for zero-copy wrapping by bindings). */
int dressi_plan_slot_ptr(dressi_plan p, int slot, void** ptr);

/* Silhouette plans: renders the targets of target_pos (host [n_verts][3])
 * into the TARGET slot -- hard silhouettes (HardSoftRas plans) or
 * anti-aliased masks (AA plans); setup, not part of the iteration. */
int dressi_plan_render_targets(dressi_plan p, const float* target_pos_host,
                               void* stream);

/* Runs n_iters full iterations on `stream` (CUDA-graph replays; the graph
 * is instantiated on first use). */
int dressi_plan_exec(dressi_plan p, uint32_t n_iters, void* stream);

/* Multi-device split of one iteration (view-sharded data parallelism):
 *  phase 0: forward + backward, leaves the local gradient in the GRAD slot;
 *  phase 1: Adam from the GRAD slot (after the caller all-reduced it). */
int dressi_plan_exec_phase(dressi_plan p, int phase, void* stream);

/* The same phase with its kernels launched directly on `stream` instead of
 * as the plan's own CUDA graph, so that a stream capture the caller runs
 * records them: phase 0, the caller's collective on the GRAD slot and phase
 * 1 then replay as ONE graph (no host round trip per iteration). Make the
 * first call outside capture. Within the caller's graph the bins do not
 * grow after an overflow; the overflow path stays exact. */
int dressi_plan_record_phase(dressi_plan p, int phase, void* stream);

/* Deterministic gradient mode of a HardSoftRas silhouette plan (on = 1):
 * instead of float atomics per pixel, the iteration stores each pixel's
 * (survivor face, dL/d dist), sums each face's corner partials over its
 * pixels in row-major order and each vertex's over its incident faces in
 * the order of the vertex -> face table -- the order of the reference's
 * GatherDistGrad + ColSum -- so that repeated runs give bit-identical
 * gradients and positions. Costs extra passes (one thread per face scans
 * its soft bbox) and [views][R][R] float2 + [views][F][3] float4 of device
 * memory. Re-captures the plan's graphs. */
int dressi_plan_set_deterministic(dressi_plan p, int on);

/* Silhouette plans: forward pass writing the RASTER slot (no update). */
int dressi_plan_render(dressi_plan p, void* stream);

/* Synchronises `stream`, returns the plan's device status word. */
int dressi_plan_status(dressi_plan p, uint32_t* word, void* stream);

/* Kernel launches one dressi_plan_exec iteration enqueues. */
int dressi_plan_launches_per_iter(dressi_plan p, uint32_t* n);

/* Debug timing outside the CUDA graph: runs n_iters iterations launching
 * every kernel directly, each bracketed by a pair of CUDA events on
 * `stream`. Fills up to max_kernels entries (one per distinct kernel, in
 * launch order): names[i] (static strings owned by the library),
 * total_ms[i] summed over its launches, launches[i]; *n_kernels = number of
 * distinct kernels. Any output array may be NULL. */
int dressi_plan_profile(dressi_plan p, uint32_t n_iters, void* stream,
                        uint32_t max_kernels, const char** names,
                        float* total_ms, uint32_t* launches,
                        uint32_t* n_kernels);

int dressi_plan_destroy(dressi_plan p);

/* ------------------------------------------------------------------------
 * Graph path: Variables, F:: ops, BuildBackward and DressiAD
 *
 * Replaces (unclearness/opendressi):
 *  - Variable handles, VType, ImgSize     include/dressi/variable.h:18-49,
 *                                         include/dressi/types.h:12-33
 *  - the F:: op library                    include/dressi/f.h:12-317
 *  - DressiAD (setLossVar, setOptimizer, addUpdate, markOutput,
 *    setGradOutputsEnabled, inputGrads, setRebuildCounts, execStep,
 *    sendImg, recvImg)                     include/dressi/dressi_ad.h:44-131
 *  - BuildBackward, the packer and the Vulkan executor behind execStep
 *                                         src/core/build_backward.cpp:62-149,
 *                                         src/pack/greedy_packer.cpp:388-586,
 *                                         src/vk/executor.h:43-66
 * A graph is built on the host from Variable handles; execStep lowers it
 * (reverse graph, optimizer graph, fusion of the pixel-wise ops into pixel
 * programs, reductions and rendering kernels) into one CUDA graph on the
 * DressiAD's device and replays it. Values are float images [h][w][ncomp]
 * (integer VTypes hold their values as floats, as the reference's CPU
 * tensors do). Host-only calls (graph building) need no GPU.
 * --------------------------------------------------------------------- */

/* VType values: the reference's enumeration order. */
#define DRESSI_VT_FLOAT 0
#define DRESSI_VT_VEC2 1
#define DRESSI_VT_VEC3 2
#define DRESSI_VT_VEC4 3
#define DRESSI_VT_MAT2 4
#define DRESSI_VT_MAT3 5
#define DRESSI_VT_MAT4 6
#define DRESSI_VT_INT 7
#define DRESSI_VT_IVEC2 8
#define DRESSI_VT_IVEC3 9
#define DRESSI_VT_IVEC4 10
#define DRESSI_VT_UINT 11

/* A reference to a graph Variable. Every handle returned by the library is
 * owned by the caller and released with dressi_var_release; the Variable
 * lives while a handle, a graph node consuming it or a DressiAD holds it. */
typedef struct dressi_var_s* dressi_var;
typedef struct dressi_ad_s* dressi_ad;

/* Variable(VType, ImgSize) (variable.h:20): a leaf image of w x h. */
int dressi_var_create(int vtype, uint32_t w, uint32_t h, dressi_var* out);
/* A second handle to the same Variable. */
int dressi_var_clone(dressi_var v, dressi_var* out);
int dressi_var_release(dressi_var v);
/* Type, size, creation id, and whether an op computes it (1) or it is a
 * leaf (0); any output pointer may be NULL. */
int dressi_var_info(dressi_var v, int* vtype, uint32_t* w, uint32_t* h,
                    uint64_t* id, int* computed);
/* setRequiresGrad / setRequiresGradRecursively (recursive = 1: the
 * Variable and everything computed from it so far). */
int dressi_var_set_requires_grad(dressi_var v, int req, int recursive);
int dressi_var_requires_grad(dressi_var v, int* req);
/* setDirty / setDirtyRecursively (the reactive cache's change marks). */
int dressi_var_set_dirty(dressi_var v, int dirty, int recursive);

/* Any F:: op by its reference name ("Add", "Sigmoid", "RasterizeSoft",
 * "Mean", "Vec3", "GetX", ...) over inputs xs, with its float parameters
 * (constants, radius_px, roughness) and integer parameters (image sizes as
 * (w, h), n_samples, corner, offsets). Argument errors (types, sizes,
 * counts) are DRESSI_ERR_INVALID with the reference's message. */
int dressi_op(const char* name, const dressi_var* xs, uint32_t n_xs,
              const float* fparams, uint32_t n_f, const int64_t* iparams,
              uint32_t n_i, dressi_var* out);

/* DressiAD::Optimizer: given the requires-grad leaves xs and their
 * gradients gxs (handles borrowed for the call), write one new handle per
 * input into out (the library takes them over); return 0 on success. The
 * callback may call dressi_ad_add_update for optimizer state. */
typedef int (*dressi_optimizer_fn)(void* user, const dressi_var* xs,
                                   const dressi_var* gxs, uint32_t n,
                                   dressi_var* out);

int dressi_ad_create(int device, dressi_ad* out);
int dressi_ad_destroy(dressi_ad ad);
int dressi_ad_set_loss(dressi_ad ad, dressi_var loss);
int dressi_ad_set_optimizer(dressi_ad ad, dressi_optimizer_fn fn, void* user);
int dressi_ad_add_update(dressi_ad ad, dressi_var input_leaf,
                         dressi_var updated);
int dressi_ad_mark_output(dressi_ad ad, dressi_var v);
int dressi_ad_set_grad_outputs(dressi_ad ad, int enable);
/* setRebuildCounts: stable iterations before the reactive re-plan that
 * prunes cached static branches (0 disables that trigger). */
int dressi_ad_set_rebuild_counts(dressi_ad ad, uint32_t fast, uint32_t full);
/* Upper bound on the ops fused into one pixel program (default 512; 1 =
 * one kernel per op, the reference's Naive packing mode). */
int dressi_ad_set_max_fusion(dressi_ad ad, uint32_t max_ops);
/* inputGrads(): up to cap (leaf, gradient) pairs as new handles; *n gets
 * the total. Valid after the first exec_step. */
int dressi_ad_input_grads(dressi_ad ad, dressi_var* xs, dressi_var* gxs,
                          uint32_t cap, uint32_t* n);
/* execStep(): (re)builds when needed, then replays the iteration's CUDA
 * graph on `stream` (asynchronous). */
int dressi_ad_exec_step(dressi_ad ad, void* stream);
/* sendImg / recvImg: n_floats = w * h * ncomp; host (on_device = 0,
 * synchronous) or device pointers (asynchronous on `stream`). A send marks
 * the Variable dirty. recv needs a Variable with a device image: a root
 * (loss, optimizer outputs, markOutput, gradients when enabled) or an
 * input of any step. */
int dressi_ad_send(dressi_ad ad, dressi_var v, const float* data,
                   size_t n_floats, int on_device, void* stream);
int dressi_ad_recv(dressi_ad ad, dressi_var v, float* data, size_t n_floats,
                   int on_device, void* stream);

typedef struct {
    uint32_t n_funcs;          /* ops of the full graph (getFuncCount) */
    uint32_t n_exec_funcs;     /* ops executed per iteration after pruning */
    uint32_t n_steps;          /* lowered steps (programs + kernels) */
    uint32_t n_programs;       /* fused pixel programs */
    uint32_t n_fused_ops;      /* ops inside the programs */
    uint32_t n_program_instructions;
    uint32_t max_program_regs;
    uint32_t n_materialized;   /* values with a device image */
    uint32_t kernels_per_iter; /* kernel nodes of the CUDA graph */
    uint32_t rebuilds;
    uint32_t pruning_active;
} dressi_ad_stats_t;

int dressi_ad_stats(dressi_ad ad, dressi_ad_stats_t* out);
/* Device status word (DRESSI_STATUS_* bits) accumulated by the graph's
 * kernels; synchronises the device; clear = 1 resets it. */
int dressi_ad_status(dressi_ad ad, uint32_t* word, int clear);

#ifdef __cplusplus
}
#endif

#endif /* DRESSI_B200_H */
