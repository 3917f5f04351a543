// Test infrastructure only: a C entry-point shim over the UNMODIFIED
// reference implementation (unclearness/opendressi), compiled in place from
// the reference checkout by oracle/Makefile into oracle/_ref/. Nothing in the
// product links this file; tests/ and bench.py's reference arm load it via
// ctypes as the checker / CPU baseline.
//
// Every graph here is built with the reference's public graph API
// (include/dressi/f.h) and evaluated by its CPU interpreter
// (src/core/cpu_eval.cpp:25-63) after its autodiff
// (src/core/build_backward.cpp:62-149) -- i.e. exactly what the reference's
// Vulkan executor computes per execStep (src/dressi_ad.cpp:280-530), minus
// the graphics API.

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <cctype>
#include <cstdlib>
#include <string>
#include <thread>
#include <vector>

#include "core/build_backward.h"
#include "core/cpu_eval.h"
#include "core/cpu_raster.h"
#include "dressi/dressi.h"
#include "dressi/ibl.h"
#include "dressi/mesh_utils.h"
#include "pbr_graph.h"

using namespace dressi;

namespace {

thread_local std::string g_err;

CpuTensor Tensor(VType vt, ImgSize sz, const float* data) {
    CpuTensor t;
    t.vtype = vt;
    t.size = sz;
    t.data.assign(data, data + size_t(sz.w) * sz.h * NumComponents(vt));
    return t;
}

void CopyOut(const CpuTensor& t, float* out) {
    std::memcpy(out, t.data.data(), t.data.size() * sizeof(float));
}

template <typename Fn>
int Guard(Fn&& fn) {
    try {
        fn();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 1;
    }
}

// Clip transform of examples/common/geometry_utils.cpp:391-402 rebuilt with
// the public ops: row r = x*m[r] + y*m[4+r] + z*m[8+r] + m[12+r].
Variable ClipOf(const Variable& pos, const float* m) {
    Variable x = F::GetX(pos), y = F::GetY(pos), z = F::GetZ(pos);
    auto row = [&](int r) {
        return x * m[0 * 4 + r] + y * m[1 * 4 + r] + z * m[2 * 4 + r] +
               m[3 * 4 + r];
    };
    return F::Vec4(row(0), row(1), row(2), row(3));
}

// The optimizer-side regulariser of examples/silhouette_optimization/
// run.cpp:407-420 on graph leaves, with its mesh tables built by the
// reference's own helpers (mesh_utils.cpp:53-101):
//   out = g + g_lap * (rms(g) / rms(g_lap) * laplacian)
//           + g_nrm * (rms(g) / rms(g_nrm) * normal)
struct RegGraph {
    uint32_t n_verts = 0;
    float laplacian = 0.f, normal = 0.f;
    Variable faces, vnb, vfa, vvf;
    CpuTensor t_faces, t_vnb, t_vfa, t_vvf;

    RegGraph(const float* faces_f, uint32_t n_faces, uint32_t nv, float lap,
             float nrm)
        : n_verts(nv), laplacian(lap), normal(nrm) {
        CpuImage fimg(n_faces, 1, 3);
        std::copy(faces_f, faces_f + size_t(n_faces) * 3, fimg.data.begin());
        const CpuImage vn = VertexNeighborsTex(fimg, nv);
        const CpuImage fa = FaceNeighborsTex(fimg);
        const CpuImage vf = VertexFacesTex(fimg, nv);
        faces = Variable(VEC3, {n_faces, 1});
        vnb = Variable(FLOAT, {nv, vn.height});
        vfa = Variable(VEC3, {n_faces, 1});
        vvf = Variable(FLOAT, {nv, vf.height});
        t_faces = Tensor(VEC3, {n_faces, 1}, faces_f);
        t_vnb = Tensor(FLOAT, {nv, vn.height}, vn.data.data());
        t_vfa = Tensor(VEC3, {n_faces, 1}, fa.data.data());
        t_vvf = Tensor(FLOAT, {nv, vf.height}, vf.data.data());
    }
    Variable Apply(const Variable& pos, const Variable& g) const {
        const float inv_cnt = 1.f / float(n_verts * 3);
        const auto rms = [&](const Variable& x) {
            return F::Sqrt(F::SumAll(x * x) * inv_cnt + 1e-24f);
        };
        Variable data_rms = rms(g);
        Variable g_lap = pos - F::VertexNeighborMean(pos, vnb);
        Variable g_nrm = F::NormalConsistencyVertexGrad(
                F::NormalConsistencyFaceTerm(pos, faces, vfa), pos, faces,
                vvf);
        return g + g_lap * (data_rms / rms(g_lap) * laplacian) +
               g_nrm * (data_rms / rms(g_nrm) * normal);
    }
    void Bind(CpuEvaluator& ev) const {
        ev.bind(faces, t_faces);
        ev.bind(vnb, t_vnb);
        ev.bind(vfa, t_vfa);
        ev.bind(vvf, t_vvf);
    }
};

// Host-side form for the view-parallel drivers: g <- Apply(pos, g).
struct RegStep {
    RegGraph rg;
    Variable pos, g, out;
    RegStep(const float* faces_f, uint32_t n_faces, uint32_t nv, float lap,
            float nrm)
        : rg(faces_f, n_faces, nv, lap, nrm),
          pos(VEC3, {nv, 1}),
          g(VEC3, {nv, 1}) {
        out = rg.Apply(pos, g);
    }
    void Run(const std::vector<float>& p, std::vector<float>& grad) const {
        CpuEvaluator ev;
        rg.Bind(ev);
        ev.bind(pos, Tensor(VEC3, {rg.n_verts, 1}, p.data()));
        ev.bind(g, Tensor(VEC3, {rg.n_verts, 1}, grad.data()));
        grad = ev.eval(out).data;
    }
};

struct SilInputs {
    uint32_t n_verts, n_faces, res, max_deg;
    float radius_px, sigma;
};

// The silhouette prediction of one view (HardSoftRas, RasterizeSoft's own
// exact dist-channel backward):
//   rs    = RasterizeSoft(SoftClip(clip), ..., clip, ...)
//   hard  = cov * step(0, dist)
//   soft  = cov * sigmoid(dist * |dist| * k),  k = (2/R)^2 / sigma
//   pred  = max(hard, soft)                    (examples/silhouette_
//                                               optimization/run.cpp:339-342)
//   loss  = (target - pred)^2 / R^2
struct SilGraph {
    Variable faces_f, vft, face_id, faces_soft;
    std::vector<Variable> targets;
    Variables view_losses;
};

Variable SilViewLoss(const Variable& clip, const SilGraph& g,
                     const Variable& target, const SilInputs& in) {
    const ImgSize screen = {in.res, in.res};
    Variable soft_clip = F::SoftClip(clip, g.faces_f, screen, in.radius_px);
    Variable rs = F::RasterizeSoft(soft_clip, g.face_id, g.faces_soft, clip,
                                   g.faces_f, g.vft, screen, in.radius_px);
    Variable dist = F::GetX(rs);
    Variable cov = F::GetW(rs);
    Variable zero = F::Float(0.f);
    const float k = (2.f / float(in.res)) * (2.f / float(in.res)) / in.sigma;
    Variable hard = cov * F::Step(zero, dist);
    Variable soft = cov * F::Sigmoid(dist * F::Abs(dist) * k);
    Variable pred = F::Max(hard, soft);
    Variable diff = F::StopGradient(target) - pred;
    return diff * diff * (1.f / float(in.res * in.res));
}

// The paper's HardSoftRas prediction of one view, composed as the
// silhouette example composes it (examples/silhouette_optimization/
// run.cpp:229-345): K soft layers (stop-gradient; layer k > 0 discards
// fragments at or in front of layer k-1's Eq.3 shifted depth), per layer
// D_k = mask * sigmoid(dist * 7 / r) with the pixel's signed distance to
// its face's edges, the corners fetched per pixel (FaceFetch of the
// LookupFaces corner positions; backward: the face's edge samples, jitter
// `seed`); Eq.6 I_s = 1 - prod_k (1 - D_k); pred = max(hard, I_s).
Variable PaperViewPred(const Variable& clip, const SilGraph& g,
                       const SilInputs& in, uint32_t peels, uint32_t samples,
                       const Variable& seed) {
    const ImgSize screen = {in.res, in.res};
    const float sigma_scale = 7.f / in.radius_px;
    Variable soft_clip = F::SoftClip(clip, g.faces_f, screen, in.radius_px);
    Variable tri0 = F::LookupFaces(clip, g.faces_f, g.vft, 0);
    Variable tri1 = F::LookupFaces(clip, g.faces_f, g.vft, 1);
    Variable tri2 = F::LookupFaces(clip, g.faces_f, g.vft, 2);
    Variable pc = F::ScreenCoord(screen);
    Variable zero = F::Float(0.f);
    Variable one = F::Float(1.f);
    const auto soft_prob = [&](const Variable& idx) {
        Variable mask = F::Greater(idx, F::Float(0.5f));
        const auto fetch = [&](const Variable& tri) {
            return F::FaceFetch(tri, idx, tri0, tri1, tri2, seed,
                                in.radius_px, samples);
        };
        const auto screen_of = [&](const Variable& c) {
            Variable w = F::GetW(c) + (1.f - mask);
            Variable sx = (F::GetX(c) / w * 0.5f + 0.5f) * float(screen.w);
            Variable sy = (F::GetY(c) / w * 0.5f + 0.5f) * float(screen.h);
            return F::Vec2(sx, sy);
        };
        Variable s0 = screen_of(fetch(tri0));
        Variable s1 = screen_of(fetch(tri1));
        Variable s2 = screen_of(fetch(tri2));
        const auto edge_dist = [&](const Variable& a, const Variable& b) {
            Variable e = b - a;
            Variable t = F::Clamp(F::Dot(pc - a, e) / (F::Dot(e, e) + 1e-12f),
                                  zero, one);
            Variable dd = pc - (a + t * e);
            return F::Sqrt(F::Dot(dd, dd) + 1e-12f);
        };
        const auto edge_cross = [&](const Variable& a, const Variable& b) {
            Variable e = b - a;
            return F::GetX(e) * (F::GetY(pc) - F::GetY(a)) -
                   F::GetY(e) * (F::GetX(pc) - F::GetX(a));
        };
        Variable dmin = F::Min(F::Min(edge_dist(s0, s1), edge_dist(s1, s2)),
                               edge_dist(s2, s0));
        Variable cr0 = edge_cross(s0, s1);
        Variable cr1 = edge_cross(s1, s2);
        Variable cr2 = edge_cross(s2, s0);
        Variable inside = F::Min(
                F::Step(zero, cr0) * F::Step(zero, cr1) * F::Step(zero, cr2) +
                        F::Step(zero, -cr0) * F::Step(zero, -cr1) *
                                F::Step(zero, -cr2),
                one);
        Variable dist = (inside * 2.f - 1.f) * dmin;
        return mask * F::Sigmoid(dist * sigma_scale);
    };
    Variable one_minus = one;
    Variable prev_shift(nullptr);
    Variable hard(nullptr);
    for (uint32_t peel = 0; peel < peels; peel++) {
        Variable rs = F::StopGradient(
                peel == 0 ? F::RasterizeSoft(soft_clip, g.face_id,
                                             g.faces_soft, clip, g.faces_f,
                                             g.vft, screen, in.radius_px)
                          : F::RasterizeSoft(soft_clip, g.face_id,
                                             g.faces_soft, clip, g.faces_f,
                                             g.vft, prev_shift, screen,
                                             in.radius_px));
        Variable dist_c = F::GetX(rs);
        Variable cov = F::GetW(rs);
        Variable ge = F::Step(zero, dist_c);
        prev_shift = cov * (ge * (F::Clamp(F::GetZ(rs), zero, one) * 0.5f) +
                            (1.f - ge) *
                                    (F::Clamp(-dist_c * (1.f / in.radius_px),
                                              zero, one) *
                                             0.5f +
                                     0.5f));
        Variable idx = (F::GetY(rs) + 1.f) * cov;
        one_minus = one_minus * (1.f - soft_prob(idx));
        if (peel == 0) hard = cov * ge;
    }
    Variable soft_sil = 1.f - one_minus;
    return F::Max(hard, soft_sil);
}

double SumAll(const CpuTensor& t) {
    double s = 0.0;
    for (float v : t.data) s += v;
    return s;
}

VType CompType(uint32_t n) {
    DRESSI_CHECK(n >= 1 && n <= 4, "n_comp 1..4");
    return n == 1 ? FLOAT : n == 2 ? VEC2 : n == 3 ? VEC3 : VEC4;
}

// y = op(x) for one image leaf x {xw, xh, n}; out receives y, and with gy
// (y's shape) g_x receives d(sum gy * y)/dx from BuildBackward.
template <typename Op>
void RunLeafOp(const float* x, uint32_t xw, uint32_t xh, uint32_t n, Op op,
               const float* gy, float* out, float* g_x) {
    const VType vt = CompType(n);
    Variable vx(vt, {xw, xh});
    Variable y = op(vx);
    CpuEvaluator ev;
    ev.bind(vx, Tensor(vt, {xw, xh}, x));
    CpuTensor ty = ev.eval(y);
    CopyOut(ty, out);
    if (!gy || !g_x) return;
    Variable vgy(y.getVType(), y.getImgSize());
    ev.bind(vgy, Tensor(y.getVType(), y.getImgSize(), gy));
    Variable loss = F::StopGradient(vgy) * y;
    Variable vx_mut = vx;
    vx_mut.setRequiresGradRecursively();
    auto [xs, gxs] = BuildBackward(loss);
    for (size_t i = 0; i < xs.size(); i++)
        if (xs[i] == vx) CopyOut(ev.eval(gxs[i]), g_x);
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// F::RasterizeSoft forward (src/core/f_ops.cpp:1362-1420 ->
// src/core/cpu_raster.cpp:241-355); out = W*H*4.
int ref_rasterize_soft(const float* soft_clip, const float* face_id,
                       const float* faces_soft, uint32_t n_faces,
                       const float* hard_clip, uint32_t n_hard,
                       const float* faces_tex, const float* vft,
                       uint32_t max_deg, uint32_t w, uint32_t h,
                       float radius, const float* prev_depth, float* out) {
    return Guard([&] {
        Variable sc(VEC4, {n_faces * 3, 1}), fid(FLOAT, {n_faces * 3, 1}),
                fs(IVEC3, {n_faces, 1}), hc(VEC4, {n_hard, 1}),
                ft(VEC3, {n_faces, 1}), vf(FLOAT, {n_hard, max_deg}),
                pd(FLOAT, {w, h});
        Variable rs = prev_depth
                              ? F::RasterizeSoft(sc, fid, fs, hc, ft, vf, pd,
                                                 {w, h}, radius)
                              : F::RasterizeSoft(sc, fid, fs, hc, ft, vf,
                                                 {w, h}, radius);
        CpuEvaluator ev;
        ev.bind(sc, Tensor(VEC4, {n_faces * 3, 1}, soft_clip));
        ev.bind(fid, Tensor(FLOAT, {n_faces * 3, 1}, face_id));
        ev.bind(fs, Tensor(IVEC3, {n_faces, 1}, faces_soft));
        ev.bind(hc, Tensor(VEC4, {n_hard, 1}, hard_clip));
        ev.bind(ft, Tensor(VEC3, {n_faces, 1}, faces_tex));
        ev.bind(vf, Tensor(FLOAT, {n_hard, max_deg}, vft));
        if (prev_depth) ev.bind(pd, Tensor(FLOAT, {w, h}, prev_depth));
        CopyOut(ev.eval(rs), out);
    });
}

// F::SoftClip (src/core/f_ops.cpp:1890-1981); out = 3F*4.
int ref_soft_clip(const float* clip, uint32_t n_verts, const float* faces,
                  uint32_t n_faces, uint32_t w, uint32_t h, float radius,
                  float* out) {
    return Guard([&] {
        Variable c(VEC4, {n_verts, 1}), f(VEC3, {n_faces, 1});
        Variable y = F::SoftClip(c, f, {w, h}, radius);
        CpuEvaluator ev;
        ev.bind(c, Tensor(VEC4, {n_verts, 1}, clip));
        ev.bind(f, Tensor(VEC3, {n_faces, 1}, faces));
        CopyOut(ev.eval(y), out);
    });
}

// F::RasterizeFaceId (src/core/f_ops.cpp:2183-2209); out = W*H.
int ref_rasterize_face_id(const float* clip, uint32_t n_verts,
                          const float* faces, uint32_t n_faces, uint32_t w,
                          uint32_t h, float* out) {
    return Guard([&] {
        Variable c(VEC4, {n_verts, 1}), a(FLOAT, {n_verts, 1}),
                f(IVEC3, {n_faces, 1});
        Variable y = F::RasterizeFaceId(c, a, f, {w, h});
        CpuEvaluator ev;
        std::vector<float> ones(n_verts, 1.f);
        ev.bind(c, Tensor(VEC4, {n_verts, 1}, clip));
        ev.bind(a, Tensor(FLOAT, {n_verts, 1}, ones.data()));
        ev.bind(f, Tensor(IVEC3, {n_faces, 1}, faces));
        CopyOut(ev.eval(y), out);
    });
}

// F::Rasterize (src/core/f_ops.cpp:1182-1207); attr has n_comp (1..4)
// components; out = W*H*n_comp.
int ref_rasterize_hard(const float* clip, uint32_t n_verts, const float* attr,
                       uint32_t n_comp, const float* faces, uint32_t n_faces,
                       uint32_t w, uint32_t h, float* out) {
    return Guard([&] {
        const VType at = VecVTypeOf(n_comp);
        Variable c(VEC4, {n_verts, 1}), a(at, {n_verts, 1}),
                f(IVEC3, {n_faces, 1});
        Variable y = F::Rasterize(c, a, f, {w, h});
        CpuEvaluator ev;
        ev.bind(c, Tensor(VEC4, {n_verts, 1}, clip));
        ev.bind(a, Tensor(at, {n_verts, 1}, attr));
        ev.bind(f, Tensor(IVEC3, {n_faces, 1}, faces));
        CopyOut(ev.eval(y), out);
    });
}

// Gradient of sum_px gy(px) * dist(px) w.r.t. the hard clip positions via
// the reference autodiff: RasterizeSoft's backward is
// ColSum(GatherDistGrad(...)) (src/core/f_ops.cpp:1407-1416, 1248-1358).
// out_grad = n_hard*4; out_rs (optional) = W*H*4.
int ref_dist_grad(const float* soft_clip, const float* face_id,
                  const float* faces_soft, uint32_t n_faces,
                  const float* hard_clip, uint32_t n_hard,
                  const float* faces_tex, const float* vft, uint32_t max_deg,
                  uint32_t w, uint32_t h, float radius, const float* gy,
                  float* out_grad, float* out_rs) {
    return Guard([&] {
        Variable sc(VEC4, {n_faces * 3, 1}), fid(FLOAT, {n_faces * 3, 1}),
                fs(IVEC3, {n_faces, 1}), hc(VEC4, {n_hard, 1}),
                ft(VEC3, {n_faces, 1}), vf(FLOAT, {n_hard, max_deg}),
                g(FLOAT, {w, h});
        Variable rs =
                F::RasterizeSoft(sc, fid, fs, hc, ft, vf, {w, h}, radius);
        Variable loss = F::GetX(rs) * F::StopGradient(g);
        Variable hc_mut = hc;
        hc_mut.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        Variable grad(nullptr);
        for (size_t i = 0; i < xs.size(); i++) {
            if (xs[i] == hc) grad = gxs[i];
        }
        DRESSI_CHECK(grad, "no gradient reached the hard clip leaf");
        CpuEvaluator ev;
        ev.bind(sc, Tensor(VEC4, {n_faces * 3, 1}, soft_clip));
        ev.bind(fid, Tensor(FLOAT, {n_faces * 3, 1}, face_id));
        ev.bind(fs, Tensor(IVEC3, {n_faces, 1}, faces_soft));
        ev.bind(hc, Tensor(VEC4, {n_hard, 1}, hard_clip));
        ev.bind(ft, Tensor(VEC3, {n_faces, 1}, faces_tex));
        ev.bind(vf, Tensor(FLOAT, {n_hard, max_deg}, vft));
        ev.bind(g, Tensor(FLOAT, {w, h}, gy));
        CopyOut(ev.eval(grad), out_grad);
        if (out_rs) CopyOut(ev.eval(rs), out_rs);
    });
}

// Full silhouette optimisation (fwd + bwd + in-graph Adam) exactly as the
// reference's DressiAD runs it: one graph over all views whose per-view loss
// images are summed with SumPixelWise (examples/silhouette_optimization/
// run.cpp:386-396), BuildBackward on the image loss (per-pixel seed 1), and
// the in-graph Adam of run.cpp:421-436 (no regularisers). Each iteration
// evaluates the updated leaves on one evaluator and re-binds them
// (the copy-backs of src/vk/executor.cpp:883-898).
//
// loss_trace[i] = sum over pixels of the loss image at the START of
// iteration i. grad0 (optional, V*3) = the position gradient of iteration 0.
// threads > 1 evaluates views on separate threads (one graph per view,
// gradients summed in view order, then the same Adam arithmetic).
int ref_silhouette_run(uint32_t n_verts, uint32_t n_faces, uint32_t n_views,
                       uint32_t res, float radius_px, float sigma, float lr,
                       const float* pos0, const float* faces,
                       const float* vft, uint32_t max_deg,
                       const float* mvps, const float* targets,
                       uint32_t n_iters, uint32_t threads, float laplacian,
                       float normal, float* loss_trace, float* pos_out,
                       float* grad0, double* seconds) {
    return Guard([&] {
        SilInputs in{n_verts, n_faces, res, max_deg, radius_px, sigma};
        const bool reg = laplacian != 0.f || normal != 0.f;
        const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
        std::vector<float> face_id(size_t(n_faces) * 3),
                faces_soft(size_t(n_faces) * 3);
        for (uint32_t f = 0; f < n_faces; f++) {
            for (uint32_t k = 0; k < 3; k++) {
                face_id[f * 3 + k] = float(f);
                faces_soft[f * 3 + k] = float(f * 3 + k);
            }
        }
        const size_t px = size_t(res) * res;
        CpuTensor t_faces = Tensor(VEC3, {n_faces, 1}, faces);
        CpuTensor t_vft = Tensor(FLOAT, {n_verts, max_deg}, vft);
        CpuTensor t_fid = Tensor(FLOAT, {n_faces * 3, 1}, face_id.data());
        CpuTensor t_fs = Tensor(IVEC3, {n_faces, 1}, faces_soft.data());

        auto make_graph = [&](SilGraph& g) {
            g.faces_f = Variable(VEC3, {n_faces, 1});
            g.vft = Variable(FLOAT, {n_verts, max_deg});
            g.face_id = Variable(FLOAT, {n_faces * 3, 1});
            g.faces_soft = Variable(IVEC3, {n_faces, 1});
        };
        auto bind_static = [&](CpuEvaluator& ev, const SilGraph& g) {
            ev.bind(g.faces_f, t_faces);
            ev.bind(g.vft, t_vft);
            ev.bind(g.face_id, t_fid);
            ev.bind(g.faces_soft, t_fs);
        };

        std::vector<float> pos(pos0, pos0 + size_t(n_verts) * 3);
        const auto t0 = std::chrono::steady_clock::now();

        if (threads <= 1) {
            SilGraph g;
            make_graph(g);
            Variable vpos(VEC3, {n_verts, 1}), am(VEC3, {n_verts, 1}),
                    av(VEC3, {n_verts, 1}), at(FLOAT, {1, 1});
            Variables losses;
            for (uint32_t v = 0; v < n_views; v++) {
                g.targets.emplace_back(FLOAT, ImgSize{res, res});
                losses.push_back(SilViewLoss(ClipOf(vpos, mvps + v * 16), g,
                                             g.targets.back(), in));
            }
            Variable loss = F::SumPixelWise(losses);
            vpos.setRequiresGradRecursively();
            auto [xs, gxs] = BuildBackward(loss);
            DRESSI_CHECK(xs.size() == 1 && xs[0] == vpos,
                         "expected pos as the only gradient leaf");
            Variable gdata = gxs[0];
            std::unique_ptr<RegGraph> rg;
            if (reg)
                rg = std::make_unique<RegGraph>(faces, n_faces, n_verts,
                                                laplacian, normal);
            Variable gp = rg ? rg->Apply(vpos, gdata) : gdata;
            Variable t_new = at + 1.f;
            Variable m_new = am * b1 + gp * (1.f - b1);
            Variable v_new = av * b2 + gp * gp * (1.f - b2);
            Variable bc1 = 1.f - F::Pow(F::Float(b1), t_new);
            Variable bc2 = 1.f - F::Pow(F::Float(b2), t_new);
            Variable step = (m_new / bc1) / (F::Sqrt(v_new / bc2) + eps) * lr;
            Variable pos_new = vpos - step;
            CpuTensor tm = Tensor(VEC3, {n_verts, 1},
                                  std::vector<float>(n_verts * 3, 0.f).data());
            CpuTensor tv = tm;
            float tt = 0.f;
            for (uint32_t it = 0; it < n_iters; it++) {
                CpuEvaluator ev;
                bind_static(ev, g);
                if (rg) rg->Bind(ev);
                for (uint32_t v = 0; v < n_views; v++) {
                    ev.bind(g.targets[v],
                            Tensor(FLOAT, {res, res}, targets + v * px));
                }
                ev.bind(vpos, Tensor(VEC3, {n_verts, 1}, pos.data()));
                ev.bind(am, tm);
                ev.bind(av, tv);
                ev.bind(at, Tensor(FLOAT, {1, 1}, &tt));
                loss_trace[it] = float(SumAll(ev.eval(loss)));
                if (it == 0 && grad0) CopyOut(ev.eval(gdata), grad0);
                CpuTensor np = ev.eval(pos_new);
                tm = ev.eval(m_new);
                tv = ev.eval(v_new);
                tt = ev.eval(t_new).data[0];
                pos = np.data;
            }
        } else {
            // View-parallel: one graph per view, evaluated concurrently
            struct ViewG {
                SilGraph g;
                Variable vpos, target, loss, grad;
            };
            std::vector<ViewG> vg(n_views);
            for (uint32_t v = 0; v < n_views; v++) {
                make_graph(vg[v].g);
                vg[v].vpos = Variable(VEC3, {n_verts, 1});
                vg[v].target = Variable(FLOAT, {res, res});
                vg[v].loss = SilViewLoss(ClipOf(vg[v].vpos, mvps + v * 16),
                                         vg[v].g, vg[v].target, in);
                vg[v].vpos.setRequiresGradRecursively();
                auto [xs, gxs] = BuildBackward(vg[v].loss);
                DRESSI_CHECK(xs.size() == 1, "expected one gradient leaf");
                vg[v].grad = gxs[0];
            }
            std::vector<float> m(size_t(n_verts) * 3, 0.f), vv = m;
            float t = 0.f;
            std::vector<std::vector<float>> grads(n_views);
            std::vector<double> vloss(n_views);
            std::unique_ptr<RegStep> rstep;
            if (reg)
                rstep = std::make_unique<RegStep>(faces, n_faces, n_verts,
                                                  laplacian, normal);
            for (uint32_t it = 0; it < n_iters; it++) {
                std::atomic<uint32_t> next{0};
                std::vector<std::string> errs(threads);
                auto work = [&](uint32_t tid) {
                    try {
                        for (uint32_t v; (v = next++) < n_views;) {
                            CpuEvaluator ev;
                            bind_static(ev, vg[v].g);
                            ev.bind(vg[v].target,
                                    Tensor(FLOAT, {res, res},
                                           targets + v * px));
                            ev.bind(vg[v].vpos,
                                    Tensor(VEC3, {n_verts, 1}, pos.data()));
                            vloss[v] = SumAll(ev.eval(vg[v].loss));
                            grads[v] = ev.eval(vg[v].grad).data;
                        }
                    } catch (const std::exception& e) {
                        errs[tid] = e.what();
                    }
                };
                std::vector<std::thread> pool;
                for (uint32_t i = 0; i < threads; i++) pool.emplace_back(work, i);
                for (auto& th : pool) th.join();
                for (auto& e : errs) DRESSI_CHECK(e.empty(), e);
                double ls = 0.0;
                for (double l : vloss) ls += l;
                loss_trace[it] = float(ls);
                std::vector<float> g(size_t(n_verts) * 3, 0.f);
                for (uint32_t v = 0; v < n_views; v++) {
                    for (size_t i = 0; i < g.size(); i++) g[i] += grads[v][i];
                }
                if (it == 0 && grad0) std::copy(g.begin(), g.end(), grad0);
                if (rstep) rstep->Run(pos, g);
                t = t + 1.f;
                const float bc1 = 1.f - std::pow(b1, t);
                const float bc2 = 1.f - std::pow(b2, t);
                for (size_t i = 0; i < g.size(); i++) {
                    m[i] = m[i] * b1 + g[i] * (1.f - b1);
                    vv[i] = vv[i] * b2 + g[i] * g[i] * (1.f - b2);
                    pos[i] = pos[i] - (m[i] / bc1) /
                                              (std::sqrt(vv[i] / bc2) + eps) *
                                              lr;
                }
            }
        }
        const auto t1 = std::chrono::steady_clock::now();
        if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
        std::copy(pos.begin(), pos.end(), pos_out);
    });
}

// F::AntiAlias on fixed leaves (img/tri/clip/faces/vertex-faces/seed), its
// image gradient and clip gradient for an incoming gradient gy: both from
// BuildBackward on sum(StopGradient(gy) * AntiAlias(...)). out_img_grad /
// out_clip_grad are nullable.
int ref_antialias(const float* img, uint32_t n_comp, const float* tri,
                  const float* clip, uint32_t n_verts, const float* faces,
                  uint32_t n_faces, const float* vft, uint32_t max_deg,
                  float seed, uint32_t n_samples, uint32_t w, uint32_t h,
                  const float* gy, float* out, float* out_img_grad,
                  float* out_clip_grad) {
    return Guard([&] {
        DRESSI_CHECK(n_comp >= 1 && n_comp <= 4, "n_comp 1..4");
        const VType it = n_comp == 1 ? FLOAT : n_comp == 2 ? VEC2
                                         : n_comp == 3   ? VEC3
                                                         : VEC4;
        Variable vimg(it, {w, h}), vtri(FLOAT, {w, h}), vclip(VEC4, {n_verts, 1}),
                vfaces(VEC3, {n_faces, 1}), vvf(FLOAT, {n_verts, max_deg}),
                vseed(FLOAT, {1, 1}), vgy(it, {w, h});
        Variable aa = F::AntiAlias(vimg, vtri, vclip, vfaces, vvf, vseed,
                                   n_samples);
        CpuEvaluator ev;
        ev.bind(vimg, Tensor(it, {w, h}, img));
        ev.bind(vtri, Tensor(FLOAT, {w, h}, tri));
        ev.bind(vclip, Tensor(VEC4, {n_verts, 1}, clip));
        ev.bind(vfaces, Tensor(VEC3, {n_faces, 1}, faces));
        ev.bind(vvf, Tensor(FLOAT, {n_verts, max_deg}, vft));
        ev.bind(vseed, Tensor(FLOAT, {1, 1}, &seed));
        CopyOut(ev.eval(aa), out);
        if (!out_img_grad && !out_clip_grad) return;
        ev.bind(vgy, Tensor(it, {w, h}, gy));
        Variable loss = F::StopGradient(vgy) * aa;
        Variable vimg_mut = vimg, vclip_mut = vclip;
        vimg_mut.setRequiresGradRecursively();
        vclip_mut.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        for (size_t i = 0; i < xs.size(); i++) {
            if (xs[i] == vimg && out_img_grad) CopyOut(ev.eval(gxs[i]), out_img_grad);
            if (xs[i] == vclip && out_clip_grad) CopyOut(ev.eval(gxs[i]), out_clip_grad);
        }
    });
}

// The AA silhouette prediction of one view (C4; examples/silhouette_
// optimization/run.cpp:230-238): mask = Rasterize(clip, ones), tri =
// RasterizeFaceId(clip), pred = AntiAlias(mask, tri, clip, faces,
// vertex-faces, seed, n_samples); loss = (target - pred)^2 / R^2.
struct AaGraph {
    Variable ones, faces_i, faces_f, vft, seed;
};

Variable AaViewLoss(const Variable& clip, const AaGraph& g,
                    const Variable& target, uint32_t res, uint32_t n_samples) {
    const ImgSize screen = {res, res};
    Variable mask = F::Rasterize(clip, g.ones, g.faces_i, screen);
    Variable tri = F::RasterizeFaceId(clip, g.ones, g.faces_i, screen);
    Variable pred = F::AntiAlias(mask, tri, clip, g.faces_f, g.vft, g.seed,
                                 n_samples);
    Variable diff = F::StopGradient(target) - pred;
    return diff * diff * (1.f / float(res * res));
}

// Full AA-silhouette optimisation: the graph of AaViewLoss over all views
// (SumPixelWise), BuildBackward, and the in-graph Adam whose counter is also
// the sampling seed (run.cpp:238, 421-436). threads > 1: one graph per view
// on separate threads, gradients summed in view order, then the same Adam
// arithmetic (as ref_silhouette_run).
int ref_aa_silhouette_run(uint32_t n_verts, uint32_t n_faces, uint32_t n_views,
                          uint32_t res, uint32_t n_samples, float lr,
                          const float* pos0, const float* faces,
                          const float* vft, uint32_t max_deg,
                          const float* mvps, const float* targets,
                          uint32_t n_iters, uint32_t threads,
                          float laplacian, float normal, float* loss_trace,
                          float* pos_out, float* grad0, double* seconds) {
    return Guard([&] {
        const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
        std::unique_ptr<RegStep> rstep;
        if (laplacian != 0.f || normal != 0.f)
            rstep = std::make_unique<RegStep>(faces, n_faces, n_verts,
                                              laplacian, normal);
        const size_t px = size_t(res) * res;
        CpuTensor t_faces = Tensor(VEC3, {n_faces, 1}, faces);
        CpuTensor t_faces_i = t_faces;
        t_faces_i.vtype = IVEC3;
        CpuTensor t_vft = Tensor(FLOAT, {n_verts, max_deg}, vft);
        std::vector<float> ones(n_verts, 1.f);
        CpuTensor t_ones = Tensor(FLOAT, {n_verts, 1}, ones.data());
        auto make_graph = [&](AaGraph& g) {
            g.ones = Variable(FLOAT, {n_verts, 1});
            g.faces_i = Variable(IVEC3, {n_faces, 1});
            g.faces_f = Variable(VEC3, {n_faces, 1});
            g.vft = Variable(FLOAT, {n_verts, max_deg});
            g.seed = Variable(FLOAT, {1, 1});
        };
        auto bind_static = [&](CpuEvaluator& ev, const AaGraph& g) {
            ev.bind(g.ones, t_ones);
            ev.bind(g.faces_i, t_faces_i);
            ev.bind(g.faces_f, t_faces);
            ev.bind(g.vft, t_vft);
        };
        std::vector<float> pos(pos0, pos0 + size_t(n_verts) * 3);
        const auto t0 = std::chrono::steady_clock::now();
        struct ViewG {
            AaGraph g;
            Variable vpos, target, loss, grad;
        };
        const uint32_t n_graphs = threads <= 1 ? 1 : n_views;
        std::vector<ViewG> vg(n_graphs);
        Variables all_losses;
        std::vector<Variable> all_targets;
        if (threads <= 1) {
            // one graph over every view: SumPixelWise of the view losses
            make_graph(vg[0].g);
            vg[0].vpos = Variable(VEC3, {n_verts, 1});
            for (uint32_t v = 0; v < n_views; v++) {
                all_targets.emplace_back(FLOAT, ImgSize{res, res});
                all_losses.push_back(AaViewLoss(ClipOf(vg[0].vpos, mvps + v * 16),
                                                vg[0].g, all_targets.back(),
                                                res, n_samples));
            }
            vg[0].loss = F::SumPixelWise(all_losses);
            vg[0].vpos.setRequiresGradRecursively();
            auto [xs, gxs] = BuildBackward(vg[0].loss);
            DRESSI_CHECK(xs.size() == 1, "expected one gradient leaf");
            vg[0].grad = gxs[0];
        } else {
            for (uint32_t v = 0; v < n_views; v++) {
                make_graph(vg[v].g);
                vg[v].vpos = Variable(VEC3, {n_verts, 1});
                vg[v].target = Variable(FLOAT, {res, res});
                vg[v].loss = AaViewLoss(ClipOf(vg[v].vpos, mvps + v * 16),
                                        vg[v].g, vg[v].target, res, n_samples);
                vg[v].vpos.setRequiresGradRecursively();
                auto [xs, gxs] = BuildBackward(vg[v].loss);
                DRESSI_CHECK(xs.size() == 1, "expected one gradient leaf");
                vg[v].grad = gxs[0];
            }
        }
        std::vector<float> m(size_t(n_verts) * 3, 0.f), vv = m;
        float t = 0.f;
        std::vector<std::vector<float>> grads(n_graphs);
        std::vector<double> vloss(n_graphs);
        for (uint32_t it = 0; it < n_iters; it++) {
            std::atomic<uint32_t> next{0};
            const uint32_t nt = std::max(1u, std::min(threads, n_graphs));
            std::vector<std::string> errs(nt);
            auto work = [&](uint32_t tid) {
                try {
                    for (uint32_t v; (v = next++) < n_graphs;) {
                        CpuEvaluator ev;
                        bind_static(ev, vg[v].g);
                        ev.bind(vg[v].g.seed, Tensor(FLOAT, {1, 1}, &t));
                        if (n_graphs == 1) {
                            for (uint32_t k = 0; k < n_views; k++)
                                ev.bind(all_targets[k],
                                        Tensor(FLOAT, {res, res}, targets + k * px));
                        } else {
                            ev.bind(vg[v].target,
                                    Tensor(FLOAT, {res, res}, targets + v * px));
                        }
                        ev.bind(vg[v].vpos, Tensor(VEC3, {n_verts, 1}, pos.data()));
                        vloss[v] = SumAll(ev.eval(vg[v].loss));
                        grads[v] = ev.eval(vg[v].grad).data;
                    }
                } catch (const std::exception& e) {
                    errs[tid] = e.what();
                }
            };
            std::vector<std::thread> pool;
            for (uint32_t i = 1; i < nt; i++) pool.emplace_back(work, i);
            work(0);
            for (auto& th : pool) th.join();
            for (auto& e : errs) DRESSI_CHECK(e.empty(), e);
            double ls = 0.0;
            for (double l : vloss) ls += l;
            loss_trace[it] = float(ls);
            std::vector<float> g(size_t(n_verts) * 3, 0.f);
            for (uint32_t v = 0; v < n_graphs; v++)
                for (size_t i = 0; i < g.size(); i++) g[i] += grads[v][i];
            if (it == 0 && grad0) std::copy(g.begin(), g.end(), grad0);
            if (rstep) rstep->Run(pos, g);
            t = t + 1.f;
            const float bc1 = 1.f - std::pow(b1, t);
            const float bc2 = 1.f - std::pow(b2, t);
            for (size_t i = 0; i < g.size(); i++) {
                m[i] = m[i] * b1 + g[i] * (1.f - b1);
                vv[i] = vv[i] * b2 + g[i] * g[i] * (1.f - b2);
                pos[i] = pos[i] - (m[i] / bc1) / (std::sqrt(vv[i] / bc2) + eps) * lr;
            }
        }
        const auto t1 = std::chrono::steady_clock::now();
        if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
        std::copy(pos.begin(), pos.end(), pos_out);
    });
}

// F::TextureBilinear on fixed leaves: out = TextureBilinear(tex, uv, inv_uv)
// [sh][sw][n]; out_grad (nullable) = d(sum gy * out)/d tex through
// BuildBackward (GatherByInverseUVBilinear).
int ref_texture_bilinear(const float* tex, uint32_t tw, uint32_t th,
                         uint32_t n, const float* uv, uint32_t sw, uint32_t sh,
                         const float* inv_uv, const float* gy, float* out,
                         float* out_grad) {
    return Guard([&] {
        DRESSI_CHECK(n >= 1 && n <= 4, "n_comp 1..4");
        const VType vt = n == 1 ? FLOAT : n == 2 ? VEC2 : n == 3 ? VEC3 : VEC4;
        Variable vtex(vt, {tw, th}), vuv(VEC2, {sw, sh}),
                viv(VEC4, {tw, th}), vgy(vt, {sw, sh});
        Variable y = F::TextureBilinear(vtex, vuv, viv);
        CpuEvaluator ev;
        ev.bind(vtex, Tensor(vt, {tw, th}, tex));
        ev.bind(vuv, Tensor(VEC2, {sw, sh}, uv));
        ev.bind(viv, Tensor(VEC4, {tw, th}, inv_uv));
        CopyOut(ev.eval(y), out);
        if (!out_grad) return;
        ev.bind(vgy, Tensor(vt, {sw, sh}, gy));
        Variable loss = F::StopGradient(vgy) * y;
        Variable vtex_mut = vtex;
        vtex_mut.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        for (size_t i = 0; i < xs.size(); i++) {
            if (xs[i] == vtex) CopyOut(ev.eval(gxs[i]), out_grad);
        }
    });
}

// Mesh tables of the regularisers built by the reference's own helpers
// (mesh_utils.cpp:73-101): vnbrs {V,max_deg} (row-major, -1 padding; cap
// floats per row limit) and fadj [F][3].
int ref_mesh_tables(const float* faces, uint32_t n_faces, uint32_t n_verts,
                    uint32_t cap, float* vnbrs, uint32_t* nbr_deg,
                    float* fadj) {
    return Guard([&] {
        CpuImage fimg(n_faces, 1, 3);
        std::copy(faces, faces + size_t(n_faces) * 3, fimg.data.begin());
        const CpuImage vn = VertexNeighborsTex(fimg, n_verts);
        DRESSI_CHECK(vn.height <= cap, "capacity too small");
        *nbr_deg = vn.height;
        std::copy(vn.data.begin(), vn.data.end(), vnbrs);
        const CpuImage fa = FaceNeighborsTex(fimg);
        std::copy(fa.data.begin(), fa.data.end(), fadj);
    });
}

// The regularised gradient of examples/silhouette_optimization/
// run.cpp:407-420 built with the reference's ops and evaluated by its CPU
// evaluator: out = g + g_lap * (rms(g) / rms(g_lap) * laplacian) + g_nrm *
// (rms(g) / rms(g_nrm) * normal).
int ref_regularized_grad(const float* pos, uint32_t n_verts, const float* faces,
                         uint32_t n_faces, const float* g, float laplacian,
                         float normal, float* out) {
    return Guard([&] {
        RegStep rs(faces, n_faces, n_verts, laplacian, normal);
        std::vector<float> p(pos, pos + size_t(n_verts) * 3);
        std::vector<float> gr(g, g + size_t(n_verts) * 3);
        rs.Run(p, gr);
        std::copy(gr.begin(), gr.end(), out);
    });
}

// F::SumAll of x {n_px, 1} with n_comp components (f_ops.cpp:1119-1149).
int ref_sum_all(const float* x, uint32_t n_px, uint32_t n_comp, float* out) {
    return Guard([&] {
        const VType vt = n_comp == 1   ? FLOAT
                         : n_comp == 2 ? VEC2
                         : n_comp == 3 ? VEC3
                                       : VEC4;
        Variable vx(vt, {n_px, 1});
        CpuEvaluator ev;
        ev.bind(vx, Tensor(vt, {n_px, 1}, x));
        *out = ev.eval(F::SumAll(vx)).data[0];
    });
}

// ---------------------------------------------------------------- IBL (C5)

// F::EquirectSample(map, dir) (f_ops.cpp:2913-2964) and its map gradient.
int ref_equirect_sample(const float* map, uint32_t mw, uint32_t mh,
                                   uint32_t n, const float* dir, uint32_t dw,
                                   uint32_t dh, const float* gy, float* out,
                                   float* g_map) {
    return Guard([&] {
        Variable vdir(VEC3, {dw, dh});
        CpuTensor tdir = Tensor(VEC3, {dw, dh}, dir);
        const VType vt = CompType(n);
        Variable vmap(vt, {mw, mh});
        Variable y = F::EquirectSample(vmap, vdir);
        CpuEvaluator ev;
        ev.bind(vmap, Tensor(vt, {mw, mh}, map));
        ev.bind(vdir, tdir);
        CopyOut(ev.eval(y), out);
        if (!gy || !g_map) return;
        Variable vgy(vt, {dw, dh});
        ev.bind(vgy, Tensor(vt, {dw, dh}, gy));
        Variable loss = F::StopGradient(vgy) * y;
        Variable vm = vmap;
        vm.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        for (size_t i = 0; i < xs.size(); i++)
            if (xs[i] == vmap) CopyOut(ev.eval(gxs[i]), g_map);
    });
}

// F::IrradianceConv(env, {ow, oh}) (f_ops.cpp:3023-3105) and its env
// gradient.
int ref_irradiance_conv(const float* env, uint32_t sw, uint32_t sh,
                                   uint32_t n, uint32_t ow, uint32_t oh,
                                   const float* gy, float* out, float* g_env) {
    return Guard([&] {
        RunLeafOp(env, sw, sh, n,
                  [&](const Variable& x) {
                      return F::IrradianceConv(x, ImgSize{ow, oh});
                  },
                  gy, out, g_env);
    });
}

// F::PrefilterConv(env, {ow, oh}, roughness) (f_ops.cpp:3272-3345) and its
// env gradient.
int ref_prefilter_conv(const float* env, uint32_t sw, uint32_t sh,
                                  uint32_t n, uint32_t ow, uint32_t oh,
                                  float roughness, const float* gy,
                                  float* out, float* g_env) {
    return Guard([&] {
        RunLeafOp(env, sw, sh, n,
                  [&](const Variable& x) {
                      return F::PrefilterConv(x, ImgSize{ow, oh}, roughness);
                  },
                  gy, out, g_env);
    });
}

// F::AvgPool2x2(x) (f_ops.cpp:3411-3415) and its gradient.
int ref_avg_pool2x2(const float* x, uint32_t w, uint32_t h,
                               uint32_t n, const float* gy, float* out,
                               float* g_x) {
    return Guard([&] {
        RunLeafOp(x, w, h, n, [](const Variable& v) { return F::AvgPool2x2(v); },
                  gy, out, g_x);
    });
}

// F::BrdfIntegrationLut({w, h}, n_samples) (f_ops.cpp:3350-3408).
int ref_brdf_lut(uint32_t w, uint32_t h, uint32_t n_samples,
                            float* out) {
    return Guard([&] {
        Variable y = F::BrdfIntegrationLut(ImgSize{w, h}, n_samples);
        CpuEvaluator ev;
        CopyOut(ev.eval(y), out);
    });
}

// BuildPbrShade (examples/common/pbr_graph.cpp:47-138, no normal mapping)
// over per-pixel G-buffer leaves and w x h material textures sampled at the
// pixel centres (identity uv and inverse-uv table), with the IBL maps of
// the env built as the envmap example does (differentiable prefilter; L
// levels), the Mean L1 (loss_kind 1) or L2 (2) loss against target, and
// the gradients w.r.t. the albedo and mr textures and the env from
// BuildBackward. frame = cam_pos, cam_fwd, cam_right, cam_up, light_pos,
// light_col.
int ref_pbr_shade_grad(uint32_t w, uint32_t h, const float* g_n,
                       const float* g_p, const float* mask,
                       const float* albedo, const float* mr, const float* ao,
                       const float* emissive, const float* frame,
                       const float* env, uint32_t ew, uint32_t eh, uint32_t L,
                       uint32_t lut_w, uint32_t lut_h, uint32_t lut_samples,
                       const float* target, int loss_kind, float* mapped,
                       float* loss, float* g_albedo, float* g_mr,
                       float* g_env) {
    return Guard([&] {
        using namespace dressi_examples;
        const ImgSize scr{w, h};
        std::vector<float> uvi(size_t(w) * h * 2), inv(size_t(w) * h * 4);
        for (uint32_t y = 0; y < h; y++)
            for (uint32_t x = 0; x < w; x++) {
                const size_t p = size_t(y) * w + x;
                uvi[p * 2 + 0] = (float(x) + 0.5f) / float(w);
                uvi[p * 2 + 1] = (float(y) + 0.5f) / float(h);
                inv[p * 4 + 0] = float(x) + 0.5f;
                inv[p * 4 + 1] = float(y) + 0.5f;
                inv[p * 4 + 2] = 1.f;
                inv[p * 4 + 3] = 1.f;
            }
        Variable venv(VEC3, {ew, eh});
        PbrIblMaps ibl;
        ibl.env = venv;
        ibl.irr = BuildIrradianceSample(venv);
        ibl.pref = BuildPrefEnvironmentSampleConv(venv, L);
        ibl.lut = BuildBrdfIntegrationMap({lut_w, lut_h}, lut_samples);
        PbrGBuffer gb;
        gb.uv = Variable(VEC2, scr);
        gb.mask = Variable(FLOAT, scr);
        gb.handed = Variable(FLOAT, scr);
        gb.g_n = Variable(VEC3, scr);
        gb.g_t = Variable(VEC3, scr);
        gb.g_p = Variable(VEC3, scr);
        PbrMaterialLeaves mat;
        mat.albedo = Variable(VEC3, scr);
        mat.mr = Variable(VEC3, scr);
        mat.normal_map = Variable(VEC3, scr);
        mat.ao = Variable(VEC3, scr);
        mat.emissive = Variable(VEC3, scr);
        PbrFrameLeaves fr;
        fr.cam_pos = Variable(VEC3, {1, 1});
        fr.cam_fwd = Variable(VEC3, {1, 1});
        fr.cam_right = Variable(VEC3, {1, 1});
        fr.cam_up = Variable(VEC3, {1, 1});
        fr.light_pos = Variable(VEC3, {1, 1});
        fr.light_col = Variable(VEC3, {1, 1});
        Variable vinv(VEC4, scr), vtgt(VEC3, scr);
        const PbrOutputs out = BuildPbrShade(gb, mat, fr, ibl, vinv, scr,
                                             false);
        Variable diff = F::StopGradient(vtgt) - out.mapped;
        Variable vloss = loss_kind == 1 ? F::Mean(F::Abs(diff))
                                        : F::Mean(diff * diff);
        CpuEvaluator ev;
        const size_t np = size_t(w) * h;
        std::vector<float> zeros(np * 3, 0.f), ones(np, 1.f);
        ev.bind(gb.uv, Tensor(VEC2, scr, uvi.data()));
        ev.bind(gb.mask, Tensor(FLOAT, scr, mask));
        ev.bind(gb.handed, Tensor(FLOAT, scr, ones.data()));
        ev.bind(gb.g_n, Tensor(VEC3, scr, g_n));
        ev.bind(gb.g_t, Tensor(VEC3, scr, zeros.data()));
        ev.bind(gb.g_p, Tensor(VEC3, scr, g_p));
        ev.bind(mat.albedo, Tensor(VEC3, scr, albedo));
        ev.bind(mat.mr, Tensor(VEC3, scr, mr));
        ev.bind(mat.normal_map, Tensor(VEC3, scr, zeros.data()));
        ev.bind(mat.ao, Tensor(VEC3, scr, ao));
        ev.bind(mat.emissive, Tensor(VEC3, scr, emissive));
        const Variable* fv[6] = {&fr.cam_pos, &fr.cam_fwd, &fr.cam_right,
                                 &fr.cam_up, &fr.light_pos, &fr.light_col};
        for (int i = 0; i < 6; i++)
            ev.bind(*fv[i], Tensor(VEC3, {1, 1}, frame + 3 * i));
        ev.bind(venv, Tensor(VEC3, {ew, eh}, env));
        ev.bind(vinv, Tensor(VEC4, scr, inv.data()));
        ev.bind(vtgt, Tensor(VEC3, scr, target));
        CopyOut(ev.eval(out.mapped), mapped);
        *loss = ev.eval(vloss).data[0];
        Variable a_mut = mat.albedo, m_mut = mat.mr, e_mut = venv;
        a_mut.setRequiresGradRecursively();
        m_mut.setRequiresGradRecursively();
        e_mut.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(vloss);
        for (size_t i = 0; i < xs.size(); i++) {
            if (xs[i] == mat.albedo) CopyOut(ev.eval(gxs[i]), g_albedo);
            if (xs[i] == mat.mr) CopyOut(ev.eval(gxs[i]), g_mr);
            if (xs[i] == venv) CopyOut(ev.eval(gxs[i]), g_env);
        }
    });
}

// 2-D image fitting (examples/image_fitting/run.cpp:40-63 with the in-graph
// Adam of the silhouette example): loss = Mean((param - target)^2) over a
// VEC4 image; Adam lr on param. loss_trace[i] is the Mean loss at the start
// of iteration i.
int ref_image_fit_run(uint32_t w, uint32_t h, const float* param0,
                      const float* target, float lr, uint32_t n_iters,
                      float* loss_trace, float* param_out, double* seconds) {
    return Guard([&] {
        const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
        Variable p(VEC4, {w, h}), tg(VEC4, {w, h}), am(VEC4, {w, h}),
                av(VEC4, {w, h}), at(FLOAT, {1, 1});
        Variable diff = p - F::StopGradient(tg);
        Variable loss = F::Mean(diff * diff);
        p.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        DRESSI_CHECK(xs.size() == 1 && xs[0] == p, "expected param leaf");
        Variable g = gxs[0];
        Variable t_new = at + 1.f;
        Variable m_new = am * b1 + g * (1.f - b1);
        Variable v_new = av * b2 + g * g * (1.f - b2);
        Variable bc1 = 1.f - F::Pow(F::Float(b1), t_new);
        Variable bc2 = 1.f - F::Pow(F::Float(b2), t_new);
        Variable step = (m_new / bc1) / (F::Sqrt(v_new / bc2) + eps) * lr;
        Variable p_new = p - step;
        const size_t n = size_t(w) * h * 4;
        CpuTensor tp = Tensor(VEC4, {w, h}, param0);
        CpuTensor tt = Tensor(VEC4, {w, h}, target);
        std::vector<float> zeros(n, 0.f);
        CpuTensor tm = Tensor(VEC4, {w, h}, zeros.data()), tv = tm;
        float t = 0.f;
        const auto t0 = std::chrono::steady_clock::now();
        for (uint32_t it = 0; it < n_iters; it++) {
            CpuEvaluator ev;
            ev.bind(p, tp);
            ev.bind(tg, tt);
            ev.bind(am, tm);
            ev.bind(av, tv);
            ev.bind(at, Tensor(FLOAT, {1, 1}, &t));
            loss_trace[it] = ev.eval(loss).data[0];
            CpuTensor np = ev.eval(p_new);
            tm = ev.eval(m_new);
            tv = ev.eval(v_new);
            t = ev.eval(t_new).data[0];
            tp = np;
        }
        const auto t1 = std::chrono::steady_clock::now();
        if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
        CopyOut(tp, param_out);
    });
}

// One evaluation of the paper-path silhouette loss over all views
// (SumPixelWise of (target - pred)^2 / R^2, BuildBackward): loss_out = the
// summed loss image, grad_out [V][3] = d loss / d pos, pred_out (nullable)
// [views][R][R]. `seed` is FaceFetch's jitter (the example passes its Adam
// counter).
int ref_paper_sil_grad(uint32_t n_verts, uint32_t n_faces, uint32_t n_views,
                       uint32_t res, float radius_px, uint32_t samples,
                       uint32_t peels, const float* pos, const float* faces,
                       const float* vft, uint32_t max_deg, const float* mvps,
                       const float* targets, float seed, float* loss_out,
                       float* grad_out, float* pred_out) {
    return Guard([&] {
        SilInputs in{n_verts, n_faces, res, max_deg, radius_px, 0.f};
        std::vector<float> face_id(size_t(n_faces) * 3),
                faces_soft(size_t(n_faces) * 3);
        for (uint32_t f = 0; f < n_faces; f++)
            for (uint32_t k = 0; k < 3; k++) {
                face_id[f * 3 + k] = float(f);
                faces_soft[f * 3 + k] = float(f * 3 + k);
            }
        SilGraph g;
        g.faces_f = Variable(VEC3, {n_faces, 1});
        g.vft = Variable(FLOAT, {n_verts, max_deg});
        g.face_id = Variable(FLOAT, {n_faces * 3, 1});
        g.faces_soft = Variable(IVEC3, {n_faces, 1});
        Variable vpos(VEC3, {n_verts, 1});
        Variable vseed(FLOAT, {1, 1});
        Variables losses, preds;
        for (uint32_t v = 0; v < n_views; v++) {
            g.targets.emplace_back(FLOAT, ImgSize{res, res});
            preds.push_back(PaperViewPred(ClipOf(vpos, mvps + v * 16), g, in,
                                          peels, samples, vseed));
            Variable diff = g.targets.back() - preds.back();
            losses.push_back(diff * diff * (1.f / float(res * res)));
        }
        Variable loss = F::SumPixelWise(losses);
        vpos.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        DRESSI_CHECK(xs.size() == 1 && xs[0] == vpos,
                     "expected pos as the only gradient leaf");
        CpuEvaluator ev;
        ev.bind(g.faces_f, Tensor(VEC3, {n_faces, 1}, faces));
        ev.bind(g.vft, Tensor(FLOAT, {n_verts, max_deg}, vft));
        ev.bind(g.face_id, Tensor(FLOAT, {n_faces * 3, 1}, face_id.data()));
        ev.bind(g.faces_soft, Tensor(IVEC3, {n_faces, 1}, faces_soft.data()));
        const size_t px = size_t(res) * res;
        for (uint32_t v = 0; v < n_views; v++)
            ev.bind(g.targets[v], Tensor(FLOAT, {res, res}, targets + v * px));
        ev.bind(vpos, Tensor(VEC3, {n_verts, 1}, pos));
        ev.bind(vseed, Tensor(FLOAT, {1, 1}, &seed));
        *loss_out = float(SumAll(ev.eval(loss)));
        CopyOut(ev.eval(gxs[0]), grad_out);
        if (pred_out)
            for (uint32_t v = 0; v < n_views; v++)
                CopyOut(ev.eval(preds[v]), pred_out + v * px);
    });
}

// ------------------------------------------------ indexed access (HSR)

// F::ScreenCoord({w, h}) (f_ops.cpp:1490-1513).
int ref_screen_coord(uint32_t w, uint32_t h, float* out) {
    return Guard([&] {
        CpuEvaluator ev;
        CopyOut(ev.eval(F::ScreenCoord({w, h})), out);
    });
}

// F::LookupFaces(attr, faces, vf, corner) (f_ops.cpp:1568-1619) and, with
// gy [F][n], the attribute gradient BuildBackward gives (LookupFacesBwd).
// vf: {V, max_deg} row-major [max_deg][V].
int ref_lookup_faces(const float* attr, uint32_t n_verts, uint32_t n,
                     const float* faces, uint32_t n_faces, const float* vf,
                     uint32_t max_deg, uint32_t corner, const float* gy,
                     float* out, float* g_attr) {
    return Guard([&] {
        const VType vt = CompType(n);
        Variable va(vt, {n_verts, 1});
        Variable vfaces(VEC3, {n_faces, 1});
        Variable vvf(FLOAT, {n_verts, max_deg});
        Variable y = F::LookupFaces(va, vfaces, vvf, corner);
        CpuEvaluator ev;
        ev.bind(va, Tensor(vt, {n_verts, 1}, attr));
        ev.bind(vfaces, Tensor(VEC3, {n_faces, 1}, faces));
        ev.bind(vvf, Tensor(FLOAT, {n_verts, max_deg}, vf));
        CopyOut(ev.eval(y), out);
        if (!gy || !g_attr) return;
        Variable vgy(vt, {n_faces, 1});
        ev.bind(vgy, Tensor(vt, {n_faces, 1}, gy));
        Variable loss = F::StopGradient(vgy) * y;
        Variable vm = va;
        vm.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        for (size_t i = 0; i < xs.size(); i++)
            if (xs[i] == va) CopyOut(ev.eval(gxs[i]), g_attr);
    });
}

// F::FaceFetch(attr, idx, prj0, prj1, prj2, seed, radius_px, n_samples)
// (f_ops.cpp:1736-1799) and, with gy [h][w][n], the attribute gradient of
// BuildBackward (FaceFetchBwd, f_ops.cpp:1631-1732). prj*: [F][4].
int ref_face_fetch(const float* attr, uint32_t n_faces, uint32_t n,
                   const float* idx, uint32_t w, uint32_t h,
                   const float* prj0, const float* prj1, const float* prj2,
                   float seed, float radius_px, uint32_t n_samples,
                   const float* gy, float* out, float* g_attr) {
    return Guard([&] {
        const VType vt = CompType(n);
        Variable va(vt, {n_faces, 1});
        Variable vidx(FLOAT, {w, h});
        Variable vp[3] = {Variable(VEC4, {n_faces, 1}),
                          Variable(VEC4, {n_faces, 1}),
                          Variable(VEC4, {n_faces, 1})};
        Variable vseed(FLOAT, {1, 1});
        Variable y = F::FaceFetch(va, vidx, vp[0], vp[1], vp[2], vseed,
                                  radius_px, n_samples);
        CpuEvaluator ev;
        ev.bind(va, Tensor(vt, {n_faces, 1}, attr));
        ev.bind(vidx, Tensor(FLOAT, {w, h}, idx));
        const float* prj[3] = {prj0, prj1, prj2};
        for (int k = 0; k < 3; k++)
            ev.bind(vp[k], Tensor(VEC4, {n_faces, 1}, prj[k]));
        ev.bind(vseed, Tensor(FLOAT, {1, 1}, &seed));
        CopyOut(ev.eval(y), out);
        if (!gy || !g_attr) return;
        Variable vgy(vt, {w, h});
        ev.bind(vgy, Tensor(vt, {w, h}, gy));
        Variable loss = F::StopGradient(vgy) * y;
        Variable vm = va;
        vm.setRequiresGradRecursively();
        auto [xs, gxs] = BuildBackward(loss);
        for (size_t i = 0; i < xs.size(); i++)
            if (xs[i] == va) CopyOut(ev.eval(gxs[i]), g_attr);
    });
}

// Vertex -> incident-face adjacency (src/core/mesh_utils.cpp:53-69).
// Returns max_deg via *max_deg; out must hold n_verts*cap floats and is
// written row-major {V, max_deg} (-1 padding). Returns nonzero if cap is
// too small.
int ref_vertex_faces_tex(const float* faces, uint32_t n_faces,
                         uint32_t n_verts, uint32_t cap, float* out,
                         uint32_t* max_deg) {
    return Guard([&] {
        CpuImage fi(n_faces, 1, 3);
        std::copy(faces, faces + size_t(n_faces) * 3, fi.data.begin());
        CpuImage t = VertexFacesTex(fi, n_verts);
        DRESSI_CHECK(t.height <= cap, "vertex_faces_tex: capacity");
        *max_deg = t.height;
        std::copy(t.data.begin(), t.data.end(), out);
    });
}

}  // extern "C"

// ------------------------------------------------------------------------
// Generic graph programs: the same op list the library's graph path builds
// (tests/graph_programs.py writes it), built here with the reference's own
// F:: API, differentiated by its BuildBackward and evaluated by its
// CpuEvaluator. One item per line:
//   leaf <id> <vtype> <w> <h> <requires_grad 0|1>
//   op <id> <Name> <n_in> <in ids> <n_f> <floats> <n_i> <ints>
//   loss <id>                 the Variable BuildBackward differentiates
//   grad <id> <leaf id>       that leaf's gradient Variable (after `loss`)
//   eval <id>                 a value to return, in order
// leaf_data: the leaves' images concatenated in declaration order; out:
// the evaluated images concatenated in `eval` order.
namespace {

Variable RefNamedOp(const std::string& name, const Variables& xs,
                    const std::vector<float>& fp,
                    const std::vector<long long>& ip) {
    auto S = [&](size_t i) {
        return ImgSize{uint32_t(ip.at(i)), uint32_t(ip.at(i + 1))};
    };
    if (name == "Float") return F::Float(fp.at(0));
    if (name == "Vec2")
        return xs.empty() ? F::Vec2(fp.at(0), fp.at(1))
                          : F::Vec2(xs.at(0), xs.at(1));
    if (name == "Vec3") {
        if (xs.empty()) return F::Vec3(fp.at(0), fp.at(1), fp.at(2));
        if (xs.size() == 2) return F::Vec3(xs[0], xs[1]);
        return F::Vec3(xs.at(0), xs.at(1), xs.at(2));
    }
    if (name == "Vec4") {
        if (xs.empty()) return F::Vec4(fp.at(0), fp.at(1), fp.at(2), fp.at(3));
        if (xs.size() == 2) return F::Vec4(xs[0], xs[1]);
        return F::Vec4(xs.at(0), xs.at(1), xs.at(2), xs.at(3));
    }
    if (name == "Add") return F::Add(xs.at(0), xs.at(1));
    if (name == "Sub") return F::Sub(xs.at(0), xs.at(1));
    if (name == "Mul") return F::Mul(xs.at(0), xs.at(1));
    if (name == "Div") return F::Div(xs.at(0), xs.at(1));
    if (name == "Neg") return F::Neg(xs.at(0));
    if (name == "Sin") return F::Sin(xs.at(0));
    if (name == "Cos") return F::Cos(xs.at(0));
    if (name == "Tan") return F::Tan(xs.at(0));
    if (name == "Asin") return F::Asin(xs.at(0));
    if (name == "Acos") return F::Acos(xs.at(0));
    if (name == "Atan") return F::Atan(xs.at(0));
    if (name == "Atan2") return F::Atan2(xs.at(0), xs.at(1));
    if (name == "Exp") return F::Exp(xs.at(0));
    if (name == "Exp2") return F::Exp2(xs.at(0));
    if (name == "Log") return F::Log(xs.at(0));
    if (name == "Log2") return F::Log2(xs.at(0));
    if (name == "Sqrt") return F::Sqrt(xs.at(0));
    if (name == "InverseSqrt") return F::InverseSqrt(xs.at(0));
    if (name == "Abs") return F::Abs(xs.at(0));
    if (name == "Sign") return F::Sign(xs.at(0));
    if (name == "Floor") return F::Floor(xs.at(0));
    if (name == "Fract") return F::Fract(xs.at(0));
    if (name == "Mod") return F::Mod(xs.at(0), xs.at(1));
    if (name == "Pow") return F::Pow(xs.at(0), xs.at(1));
    if (name == "Max") return F::Max(xs.at(0), xs.at(1));
    if (name == "Min") return F::Min(xs.at(0), xs.at(1));
    if (name == "Clamp") return F::Clamp(xs.at(0), xs.at(1), xs.at(2));
    if (name == "Mix") return F::Mix(xs.at(0), xs.at(1), xs.at(2));
    if (name == "Step") return F::Step(xs.at(0), xs.at(1));
    if (name == "SmoothStep")
        return F::SmoothStep(xs.at(0), xs.at(1), xs.at(2));
    if (name == "Sigmoid") return F::Sigmoid(xs.at(0));
    if (name == "Less") return F::Less(xs.at(0), xs.at(1));
    if (name == "LessEqual") return F::LessEqual(xs.at(0), xs.at(1));
    if (name == "Greater") return F::Greater(xs.at(0), xs.at(1));
    if (name == "GreaterEqual") return F::GreaterEqual(xs.at(0), xs.at(1));
    if (name == "GetX") return F::GetX(xs.at(0));
    if (name == "GetY") return F::GetY(xs.at(0));
    if (name == "GetZ") return F::GetZ(xs.at(0));
    if (name == "GetW") return F::GetW(xs.at(0));
    if (name == "Dot") return F::Dot(xs.at(0), xs.at(1));
    if (name == "Cross") return F::Cross(xs.at(0), xs.at(1));
    if (name == "Length") return F::Length(xs.at(0));
    if (name == "Distance") return F::Distance(xs.at(0), xs.at(1));
    if (name == "Normalize") return F::Normalize(xs.at(0));
    if (name == "Reflect") return F::Reflect(xs.at(0), xs.at(1));
    if (name == "CompSum") return F::CompSum(xs.at(0));
    if (name == "MatMul") return F::MatMul(xs.at(0), xs.at(1));
    if (name == "Transpose") return F::Transpose(xs.at(0));
    if (name == "OuterProduct") return F::OuterProduct(xs.at(0), xs.at(1));
    if (name == "SumPixelWise") return F::SumPixelWise(xs);
    if (name == "Sum") return F::Sum(xs.at(0));
    if (name == "Mean") return F::Mean(xs.at(0));
    if (name == "SumAll") return F::SumAll(xs.at(0));
    if (name == "Broadcast") return F::Broadcast(xs.at(0), S(0));
    if (name == "StopGradient") return F::StopGradient(xs.at(0));
    if (name == "SetFragDepth") return F::SetFragDepth(xs.at(0));
    if (name == "ScreenCoord") return F::ScreenCoord(S(0));
    if (name == "Rasterize")
        return F::Rasterize(xs.at(0), xs.at(1), xs.at(2), S(0));
    if (name == "RasterizeFaceId")
        return F::RasterizeFaceId(xs.at(0), xs.at(1), xs.at(2), S(0));
    if (name == "RasterizeSoft") {
        if (xs.size() == 7)
            return F::RasterizeSoft(xs[0], xs[1], xs[2], xs[3], xs[4], xs[5],
                                    xs[6], S(0), fp.at(0));
        return F::RasterizeSoft(xs.at(0), xs.at(1), xs.at(2), xs.at(3),
                                xs.at(4), xs.at(5), S(0), fp.at(0));
    }
    if (name == "SoftClip")
        return F::SoftClip(xs.at(0), xs.at(1), S(0), fp.at(0));
    if (name == "AntiAlias")
        return F::AntiAlias(xs.at(0), xs.at(1), xs.at(2), xs.at(3), xs.at(4),
                            xs.at(5), ip.empty() ? 8u : uint32_t(ip[0]));
    if (name == "VertexNeighborMean")
        return F::VertexNeighborMean(xs.at(0), xs.at(1));
    if (name == "NormalConsistencyFaceTerm")
        return F::NormalConsistencyFaceTerm(xs.at(0), xs.at(1), xs.at(2));
    if (name == "NormalConsistencyVertexGrad")
        return F::NormalConsistencyVertexGrad(xs.at(0), xs.at(1), xs.at(2),
                                              xs.at(3));
    if (name == "LookupFaces")
        return F::LookupFaces(xs.at(0), xs.at(1), xs.at(2),
                              uint32_t(ip.at(0)));
    if (name == "FaceFetch")
        return F::FaceFetch(xs.at(0), xs.at(1), xs.at(2), xs.at(3), xs.at(4),
                            xs.at(5), fp.at(0),
                            ip.empty() ? 4u : uint32_t(ip[0]));
    if (name == "Texture") return F::Texture(xs.at(0), xs.at(1), xs.at(2));
    if (name == "TextureBilinear")
        return F::TextureBilinear(xs.at(0), xs.at(1), xs.at(2));
    if (name == "EquirectSample") return F::EquirectSample(xs.at(0), xs.at(1));
    if (name == "IrradianceConv") return F::IrradianceConv(xs.at(0), S(0));
    if (name == "PrefilterConv")
        return F::PrefilterConv(xs.at(0), S(0), fp.at(0));
    if (name == "BrdfIntegrationLut")
        return F::BrdfIntegrationLut(S(0),
                                     ip.size() > 2 ? uint32_t(ip[2]) : 512u);
    if (name == "AvgPool2x2") return F::AvgPool2x2(xs.at(0));
    if (name == "PixelFetch")
        return F::PixelFetch(xs.at(0), uint32_t(ip.at(0)), xs.at(1));
    if (name == "TileFetch")
        return F::TileFetch(xs.at(0), xs.at(1), uint32_t(ip.at(0)));
    DRESSI_CHECK(false, "ref_graph_eval: unknown op " + name);
    return nullptr;
}

}  // namespace

// Whitespace tokenizer of the program text (no iostreams: their locale
// facets are not safe to use from every host process that loads this
// library).
struct Tokens {
    const char* p;
    bool next(std::string* out) {
        while (*p && std::isspace(static_cast<unsigned char>(*p))) p++;
        if (!*p) return false;
        const char* b = p;
        while (*p && !std::isspace(static_cast<unsigned char>(*p))) p++;
        out->assign(b, p);
        return true;
    }
    std::string str() {
        std::string t;
        DRESSI_CHECK(next(&t), "ref_graph_eval: truncated program");
        return t;
    }
    long long i64() { return std::strtoll(str().c_str(), nullptr, 10); }
    float f32() { return std::strtof(str().c_str(), nullptr); }
};

extern "C" int ref_graph_eval(const char* program, const float* leaf_data,
                              float* out) {
    return Guard([&] {
        std::map<long long, Variable> vars;
        std::vector<Variable> leaves, evals;
        Variable loss(nullptr);
        std::map<Variable, Variable> grads;
        bool have_grads = false;
        Tokens in{program};
        std::string kind;
        while (in.next(&kind)) {
            if (kind == "leaf") {
                const long long id = in.i64();
                const int vt = int(in.i64());
                const uint32_t w = uint32_t(in.i64());
                const uint32_t h = uint32_t(in.i64());
                const int rg = int(in.i64());
                Variable v(VType(vt), {w, h});
                if (rg) v.setRequiresGrad(true);
                vars[id] = v;
                leaves.push_back(v);
            } else if (kind == "op") {
                const long long id = in.i64();
                const std::string name = in.str();
                size_t n = size_t(in.i64());
                Variables xs(n);
                for (auto& x : xs) x = vars.at(in.i64());
                std::vector<float> fp(size_t(in.i64()));
                for (auto& f : fp) f = in.f32();
                std::vector<long long> ip(size_t(in.i64()));
                for (auto& i : ip) i = in.i64();
                vars[id] = RefNamedOp(name, xs, fp, ip);
            } else if (kind == "loss") {
                loss = vars.at(in.i64());
            } else if (kind == "grad") {
                const long long id = in.i64();
                const long long leaf = in.i64();
                DRESSI_CHECK(loss, "ref_graph_eval: grad before loss");
                if (!have_grads) {
                    // requires-grad marks reach everything computed so far
                    for (auto& l : leaves)
                        if (l.getRequiresGrad())
                            l.setRequiresGradRecursively(true);
                    auto [xs, gxs] = BuildBackward(loss);
                    for (size_t i = 0; i < xs.size(); i++)
                        grads[xs[i]] = gxs[i];
                    have_grads = true;
                }
                auto it = grads.find(vars.at(leaf));
                DRESSI_CHECK(it != grads.end(),
                             "ref_graph_eval: leaf without gradient");
                vars[id] = it->second;
            } else if (kind == "eval") {
                evals.push_back(vars.at(in.i64()));
            } else {
                DRESSI_CHECK(false, "ref_graph_eval: bad line " + kind);
            }
        }
        CpuEvaluator ev;
        size_t off = 0;
        for (auto& l : leaves) {
            const size_t n = size_t(l.getImgSize().w) * l.getImgSize().h *
                             NumComponents(l.getVType());
            ev.bind(l, Tensor(l.getVType(), l.getImgSize(), leaf_data + off));
            off += n;
        }
        size_t o = 0;
        for (auto& e : evals) {
            CpuTensor t = ev.eval(e);
            CopyOut(t, out + o);
            o += t.data.size();
        }
    });
}
