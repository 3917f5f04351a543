// Graph nodes, the F:: op constructors (output type / size inference and
// argument checks) and each op's backward rule.
//
// The rules follow the reference op by op (src/core/f_ops.cpp, cited per
// group below): a rule builds its gradient from F:: ops, so BuildBackward
// yields a graph of the same elementwise expressions the reference
// evaluates, and the planner fuses those like the forward ops.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <functional>
#include <unordered_set>

#include "graph.h"

namespace dressi {
namespace graph {

// ------------------------------------------------------------------ types

uint32_t ncomp(VType t) {
    switch (t) {
    case FLOAT: case INT: case UINT: return 1;
    case VEC2: case IVEC2: return 2;
    case VEC3: case IVEC3: return 3;
    case VEC4: case IVEC4: case MAT2: return 4;
    case MAT3: return 9;
    case MAT4: return 16;
    }
    return 1;
}
bool is_int(VType t) {
    return t == INT || t == IVEC2 || t == IVEC3 || t == IVEC4 || t == UINT;
}
bool is_mat(VType t) { return t == MAT2 || t == MAT3 || t == MAT4; }
bool is_vec(VType t) {
    return t == VEC2 || t == VEC3 || t == VEC4 || t == IVEC2 || t == IVEC3 ||
           t == IVEC4;
}
VType vec_of(uint32_t n, bool integer) {
    DRESSI_REQUIRE(n >= 1 && n <= 4, "vector width must be 1..4");
    static const VType f[] = {FLOAT, VEC2, VEC3, VEC4};
    static const VType i[] = {INT, IVEC2, IVEC3, IVEC4};
    return integer ? i[n - 1] : f[n - 1];
}
uint32_t mat_dim(VType t) { return t == MAT2 ? 2 : t == MAT3 ? 3 : 4; }

const char* op_name(Op op) {
    static const char* names[] = {
        "Const", "Add", "Sub", "Mul", "Div", "Neg", "Sin", "Cos", "Tan",
        "Asin", "Acos", "Atan", "Atan2", "Exp", "Exp2", "Log", "Log2", "Sqrt",
        "InverseSqrt", "Abs", "Sign", "Floor", "Fract", "Mod", "Pow", "Max",
        "Min", "Clamp", "Mix", "Step", "SmoothStep", "Sigmoid", "Less",
        "LessEqual", "Greater", "GreaterEqual", "Compose", "ExtractComps",
        "Dot", "Cross", "Length", "Normalize", "CompSum", "MatMul",
        "Transpose", "OuterProduct", "SumPixelWise", "StopGradient",
        "SetFragDepth", "Broadcast", "ScreenCoord", "Sum", "SumPartial",
        "SumAll", "Rasterize", "RasterizeFaceId", "RasterizeSoft",
        "RasterizeSoftGrad", "SoftClip", "AntiAlias", "AntiAliasBwdImg",
        "AntiAliasBwdVtx", "VertexNeighborMean", "NormalConsistencyFaceTerm",
        "NormalConsistencyVertexGrad", "LookupFaces", "LookupFacesBwd",
        "FaceFetch", "FaceFetchBwd", "Texture", "TextureBilinear",
        "GatherByInverseUV", "GatherByInverseUVBilinear", "EquirectSample",
        "EquirectSampleBwd", "IrradianceConv", "IrradianceConvBwd",
        "PrefilterConv", "PrefilterConvBwd", "BrdfIntegrationLut",
        "AvgPool2x2", "AvgPool2x2Bwd", "PixelFetch", "TileFetch"};
    static_assert(sizeof(names) / sizeof(names[0]) == size_t(Op::kCount),
                  "op names");
    return names[int(op)];
}

bool is_pixelwise(Op op) { return int(op) <= int(Op::ScreenCoord); }

// ------------------------------------------------------------------ nodes

uint64_t next_node_id() {
    static std::atomic<uint64_t> next{1};
    return next.fetch_add(1);
}

Var make_op(Op op, const Vars& xs, VType vt, ImgSize size,
            std::vector<float> fp, std::vector<int64_t> ip) {
    auto f = std::make_shared<FuncNode>();
    f->id = next_node_id();
    f->op = op;
    f->fp = std::move(fp);
    f->ip = std::move(ip);
    for (const auto& x : xs) {
        DRESSI_REQUIRE(x, std::string(op_name(op)) + ": null input");
        f->xs.push_back(x);
        x->users.push_back(f);
    }
    auto y = std::make_shared<VarNode>();
    y->id = next_node_id();
    y->vtype = vt;
    y->size = size;
    y->creator = f;
    f->y = y;
    return y;
}

Var make_leaf(VType vt, ImgSize size) {
    DRESSI_REQUIRE(size.w >= 1 && size.h >= 1, "Variable: empty image size");
    auto y = std::make_shared<VarNode>();
    y->id = next_node_id();
    y->vtype = vt;
    y->size = size;
    return y;
}

namespace {

// `set` on v and on every variable computed downstream of it (the
// reference's ForEachDownstream, src/core/node.cpp:152-177).
void for_each_downstream(const Var& start,
                         const std::function<void(VarNode&)>& set) {
    std::vector<Var> stack{start};
    std::unordered_set<uint64_t> seen;
    while (!stack.empty()) {
        Var v = stack.back();
        stack.pop_back();
        if (!seen.insert(v->id).second) continue;
        set(*v);
        for (auto& wu : v->users) {
            if (auto u = wu.lock())
                if (auto y = u->y.lock()) stack.push_back(y);
        }
    }
}

// ------------------------------------------------------------ inference

ImgSize common_size(const Vars& xs) {
    ImgSize c;
    for (const auto& x : xs) {
        if (x->size.uniform()) continue;
        if (c.uniform())
            c = x->size;
        else
            DRESSI_REQUIRE(c == x->size,
                           "Image size mismatch: non-uniform inputs must "
                           "have the same size");
    }
    return c;
}

// InferElementwise (src/core/infer.cpp:26-49): scalars broadcast, vector
// and matrix types must agree, ints and floats do not mix.
VType elementwise_type(const Vars& xs) {
    bool any_int = false, any_float = false;
    VType widest = FLOAT;
    uint32_t widest_n = 0;
    for (const auto& x : xs) {
        const VType t = x->vtype;
        (is_int(t) ? any_int : any_float) = true;
        const uint32_t n = ncomp(t);
        if (n > 1)
            DRESSI_REQUIRE(widest_n <= 1 || t == widest,
                           "Vector/matrix type mismatch between inputs");
        if (n > widest_n) {
            widest_n = n;
            widest = t;
        }
    }
    DRESSI_REQUIRE(!(any_int && any_float),
                   "Int and float inputs cannot mix implicitly; use a cast");
    return widest;
}

Var ew(Op op, const Vars& xs) {
    return make_op(op, xs, elementwise_type(xs), common_size(xs));
}

Var fixed(Op op, const Vars& xs, VType vt) {
    return make_op(op, xs, vt, common_size(xs));
}

bool is_const_val(const Var& v, float val) {
    return v->is_const && v->cval.size() == 1 && v->cval[0] == val;
}

}  // namespace

void set_requires_grad_recursively(const Var& v, bool req) {
    for_each_downstream(v, [req](VarNode& n) { n.req_grad = req; });
}

void set_dirty_recursively(const Var& v, bool dirty) {
    for_each_downstream(v, [dirty](VarNode& n) { n.dirty = dirty; });
}

// ------------------------------------------------------------------- F::

namespace F {

Var Float(float v) {
    Var y = make_op(Op::Const, {}, FLOAT, {1, 1});
    y->is_const = true;
    y->cval = {v};
    return y;
}

Var Vec(const std::vector<float>& vals) {
    DRESSI_REQUIRE(vals.size() >= 2 && vals.size() <= 4,
                   "Vec: 2..4 components");
    Var y = make_op(Op::Const, {}, vec_of(uint32_t(vals.size())), {1, 1});
    y->is_const = true;
    y->cval = vals;
    return y;
}

Var Add(const Var& a, const Var& b) { return ew(Op::Add, {a, b}); }
Var Sub(const Var& a, const Var& b) { return ew(Op::Sub, {a, b}); }
Var Mul(const Var& a, const Var& b) {
    DRESSI_REQUIRE(!is_mat(a->vtype) || b->vtype == FLOAT,
                   "Use F::MatMul for matrix products");
    DRESSI_REQUIRE(!is_mat(b->vtype) || a->vtype == FLOAT,
                   "Use F::MatMul for matrix products");
    return ew(Op::Mul, {a, b});
}
Var Div(const Var& a, const Var& b) {
    DRESSI_REQUIRE(!is_mat(b->vtype), "Division by a matrix is not supported");
    return ew(Op::Div, {a, b});
}
Var Neg(const Var& x) { return ew(Op::Neg, {x}); }

Var Unary(Op op, const Var& x) { return ew(op, {x}); }

Var Binary(Op op, const Var& a, const Var& b) {
    if (op == Op::Less || op == Op::LessEqual || op == Op::Greater ||
        op == Op::GreaterEqual) {
        DRESSI_REQUIRE(a->vtype == FLOAT && b->vtype == FLOAT,
                       "Comparison ops require scalar FLOAT inputs");
        return fixed(op, {a, b}, FLOAT);
    }
    return ew(op, {a, b});
}

Var Ternary(Op op, const Var& a, const Var& b, const Var& c) {
    return ew(op, {a, b, c});
}

// Compose / ExtractComps (f_ops.cpp:35-124)
Var Compose(const Vars& parts) {
    uint32_t total = 0;
    for (const auto& p : parts) {
        DRESSI_REQUIRE(p && !is_int(p->vtype) && !is_mat(p->vtype),
                       "Compose expects float scalar/vector parts");
        total += ncomp(p->vtype);
    }
    DRESSI_REQUIRE(total >= 2 && total <= 4,
                   "Compose: invalid component count");
    return fixed(Op::Compose, parts, vec_of(total));
}

Var Extract(const Var& v, uint32_t ofs, uint32_t n) {
    const uint32_t src_n = ncomp(v->vtype);
    DRESSI_REQUIRE(ofs + n <= src_n && n >= 1, "ExtractComps out of range");
    if (n == src_n) return v;
    return make_op(Op::Extract, {v}, vec_of(n), v->size, {},
                   {int64_t(ofs), int64_t(n)});
}

Var Dot(const Var& a, const Var& b) {
    DRESSI_REQUIRE(is_vec(a->vtype) && a->vtype == b->vtype,
                   "Dot requires two equal vector types");
    return fixed(Op::Dot, {a, b}, FLOAT);
}

Var Cross(const Var& a, const Var& b) {
    DRESSI_REQUIRE(a->vtype == VEC3 && b->vtype == VEC3,
                   "Cross requires VEC3 inputs");
    return fixed(Op::Cross, {a, b}, VEC3);
}

Var Length(const Var& v) {
    DRESSI_REQUIRE(is_vec(v->vtype) || v->vtype == FLOAT,
                   "Length requires a float vector");
    return fixed(Op::Length, {v}, FLOAT);
}

Var Normalize(const Var& v) { return ew(Op::Normalize, {v}); }

Var CompSum(const Var& v) {
    if (v->vtype == FLOAT) return v;
    DRESSI_REQUIRE(is_vec(v->vtype) && !is_int(v->vtype),
                   "CompSum requires a float vector");
    return fixed(Op::CompSum, {v}, FLOAT);
}

Var MatMul(const Var& a, const Var& b) {
    DRESSI_REQUIRE(is_mat(a->vtype), "MatMul: lhs must be a matrix");
    const uint32_t dim = mat_dim(a->vtype);
    const bool vec_rhs = is_vec(b->vtype);
    if (vec_rhs)
        DRESSI_REQUIRE(ncomp(b->vtype) == dim, "MatMul: dimension mismatch");
    else
        DRESSI_REQUIRE(b->vtype == a->vtype,
                       "MatMul: rhs must match lhs matrix type");
    return fixed(Op::MatMul, {a, b}, vec_rhs ? b->vtype : a->vtype);
}

Var Transpose(const Var& m) {
    DRESSI_REQUIRE(is_mat(m->vtype), "Transpose requires a matrix");
    return fixed(Op::Transpose, {m}, m->vtype);
}

Var OuterProduct(const Var& c, const Var& r) {
    DRESSI_REQUIRE(is_vec(c->vtype) && r->vtype == c->vtype,
                   "OuterProduct requires two equal float vectors");
    const uint32_t d = ncomp(c->vtype);
    return fixed(Op::OuterProduct, {c, r},
                 d == 2 ? MAT2 : d == 3 ? MAT3 : MAT4);
}

// SumPixelWise (f_ops.cpp:893-948): a tree of flat nodes of arity <= 4.
Var SumPixelWise(const Vars& xs) {
    DRESSI_REQUIRE(!xs.empty(), "SumPixelWise requires inputs");
    if (xs.size() == 1) return xs[0];
    Vars level = xs;
    while (level.size() > 1) {
        Vars next;
        for (size_t i = 0; i < level.size(); i += 4) {
            const size_t n = std::min<size_t>(4, level.size() - i);
            if (n == 1)
                next.push_back(level[i]);
            else
                next.push_back(ew(Op::SumPixelWise,
                                  Vars(level.begin() + i,
                                       level.begin() + i + n)));
        }
        level = std::move(next);
    }
    return level[0];
}

// Sum: the whole-image reduction to {1,1}. The reference chains
// Reduce2x2Sum nodes (f_ops.cpp:1034-1040); here it is one node whose
// kernel walks the same quad tree (so the float sums are identical) and
// whose backward broadcasts (the transpose of the chain).
Var Sum(const Var& x) {
    if (x->size.uniform()) return x;
    return make_op(Op::Sum, {x}, x->vtype, {1, 1});
}

// Mean (f_ops.cpp:1042-1048)
Var Mean(const Var& x) {
    const uint32_t n = ncomp(x->vtype);
    const float inv_n =
            1.f / (float(x->size.w) * float(x->size.h) * float(n));
    return Mul(CompSum(Sum(x)), Float(inv_n));
}

// SumAll = SumPartial(64) + a serial double sum for inputs above 256
// pixels (f_ops.cpp:1087-1149).
Var SumAll(const Var& x) {
    DRESSI_REQUIRE(!is_int(x->vtype) && !is_mat(x->vtype),
                   "SumAll: input must be a float image");
    Var src = x;
    if (x->size.pixels() > 256)
        src = make_op(Op::SumPartial, {x}, FLOAT, {64, 1}, {}, {64});
    return make_op(Op::SumAll, {src}, FLOAT, {1, 1});
}

Var Broadcast(const Var& x, ImgSize size) {
    DRESSI_REQUIRE(x->size.uniform(),
                   "Broadcast: input must be a uniform {1,1} Variable");
    if (size.uniform()) return x;
    return make_op(Op::Broadcast, {x}, x->vtype, size);
}

Var StopGradient(const Var& x) { return ew(Op::StopGradient, {x}); }
Var SetFragDepth(const Var& x) { return ew(Op::SetFragDepth, {x}); }

Var ScreenCoord(ImgSize size) {
    return make_op(Op::ScreenCoord, {}, VEC2, size);
}

// ----------------------------------------------------- rasterization

Var Rasterize(const Var& clip, const Var& attr, const Var& faces,
              ImgSize screen) {
    DRESSI_REQUIRE(clip->vtype == VEC4 && clip->size.h == 1,
                   "Rasterize: vtx_clip_pos must be VEC4 {V,1}");
    DRESSI_REQUIRE(!is_int(attr->vtype) && !is_mat(attr->vtype),
                   "Rasterize: attribute must be a float scalar/vector");
    DRESSI_REQUIRE(attr->size == clip->size,
                   "Rasterize: attribute count must match vertex count");
    DRESSI_REQUIRE(faces->vtype == IVEC3 && faces->size.h == 1,
                   "Rasterize: faces must be IVEC3 {F,1}");
    return make_op(Op::Rasterize, {clip, attr, faces}, attr->vtype, screen);
}

Var RasterizeFaceId(const Var& clip, const Var& dummy, const Var& faces,
                    ImgSize screen) {
    DRESSI_REQUIRE(clip->vtype == VEC4 && clip->size.h == 1,
                   "RasterizeFaceId: vtx_clip_pos must be VEC4 {V,1}");
    DRESSI_REQUIRE(faces->vtype == IVEC3 && faces->size.h == 1,
                   "RasterizeFaceId: faces must be IVEC3 {F,1}");
    return make_op(Op::RasterizeFaceId, {clip, dummy, faces}, FLOAT, screen);
}

// RasterizeSoft (+ peel) (f_ops.cpp:1362-1465)
Var RasterizeSoft(const Var& soft_clip, const Var& face_id,
                  const Var& faces_soft, const Var& clip_hard,
                  const Var& faces_tex, const Var& vft,
                  const Var& prev_depth, ImgSize screen, float radius_px) {
    DRESSI_REQUIRE(soft_clip->vtype == VEC4 && soft_clip->size.h == 1,
                   "RasterizeSoft: vtx_clip_soft must be VEC4 {3F,1}");
    DRESSI_REQUIRE(face_id->vtype == FLOAT && face_id->size == soft_clip->size,
                   "RasterizeSoft: face_id must be FLOAT {3F,1}");
    DRESSI_REQUIRE(faces_soft->vtype == IVEC3 && faces_soft->size.h == 1,
                   "RasterizeSoft: faces_soft must be IVEC3 {F,1}");
    DRESSI_REQUIRE(soft_clip->size.w == faces_soft->size.w * 3,
                   "RasterizeSoft: soft vertices must be unwelded "
                   "(3 per face)");
    DRESSI_REQUIRE(clip_hard->vtype == VEC4 && clip_hard->size.h == 1,
                   "RasterizeSoft: vtx_clip_hard_tex must be VEC4 {V,1}");
    DRESSI_REQUIRE(faces_tex->vtype == VEC3 &&
                           faces_tex->size == faces_soft->size,
                   "RasterizeSoft: faces_tex must be VEC3 {F,1}");
    DRESSI_REQUIRE(vft->vtype == FLOAT && vft->size.w == clip_hard->size.w,
                   "RasterizeSoft: vtx_faces_tex must be FLOAT {V,max_deg}");
    DRESSI_REQUIRE(radius_px > 0.f, "RasterizeSoft: radius_px must be > 0");
    Vars xs{soft_clip, face_id, faces_soft, clip_hard, faces_tex, vft};
    if (prev_depth) {
        DRESSI_REQUIRE(prev_depth->vtype == FLOAT && prev_depth->size == screen,
                       "RasterizeSoft: prev_shifted_depth must be FLOAT {S,S}");
        xs.push_back(prev_depth);
    }
    return make_op(Op::RasterizeSoft, xs, VEC4, screen, {radius_px});
}

Var SoftClip(const Var& clip_hard, const Var& faces_tex, ImgSize screen,
             float radius_px) {
    DRESSI_REQUIRE(clip_hard->vtype == VEC4 && clip_hard->size.h == 1,
                   "SoftClip: vtx_clip_hard_tex must be VEC4 {V,1}");
    DRESSI_REQUIRE(faces_tex->vtype == VEC3 && faces_tex->size.h == 1,
                   "SoftClip: faces_tex must be VEC3 {F,1}");
    DRESSI_REQUIRE(radius_px >= 0.f, "SoftClip: radius_px must be >= 0");
    return make_op(Op::SoftClip, {clip_hard, faces_tex}, VEC4,
                   {faces_tex->size.w * 3, 1},
                   {radius_px, float(screen.w), float(screen.h)});
}

// AntiAlias (f_ops.cpp:2480-2579)
Var AntiAlias(const Var& img, const Var& tri_id, const Var& clip,
              const Var& faces, const Var& vft, const Var& seed,
              uint32_t n_samples) {
    DRESSI_REQUIRE(!is_int(img->vtype) && !is_mat(img->vtype) &&
                           ncomp(img->vtype) <= 4,
                   "AntiAlias: img must be a float image of 1..4 components");
    DRESSI_REQUIRE(tri_id->vtype == FLOAT && tri_id->size == img->size,
                   "AntiAlias: tri_id must be FLOAT of img's size");
    DRESSI_REQUIRE(clip->vtype == VEC4 && clip->size.h == 1,
                   "AntiAlias: vtx_clip must be VEC4 {V,1}");
    DRESSI_REQUIRE(faces->vtype == VEC3 && faces->size.h == 1,
                   "AntiAlias: faces must be VEC3 {F,1}");
    DRESSI_REQUIRE(vft->vtype == FLOAT && vft->size.w == clip->size.w,
                   "AntiAlias: vtx_faces_tex must be FLOAT {V,max_deg}");
    DRESSI_REQUIRE(seed->vtype == FLOAT && seed->size.uniform(),
                   "AntiAlias: seed must be FLOAT {1,1}");
    return make_op(Op::AntiAlias, {img, tri_id, clip, faces, vft, seed},
                   img->vtype, img->size, {}, {int64_t(n_samples)});
}

Var VertexNeighborMean(const Var& pos, const Var& nbrs) {
    DRESSI_REQUIRE(pos->vtype == VEC3 && pos->size.h == 1,
                   "VertexNeighborMean: pos_tex must be VEC3 {V,1}");
    DRESSI_REQUIRE(nbrs->vtype == FLOAT && nbrs->size.w == pos->size.w,
                   "VertexNeighborMean: vtx_neighbors_tex must be FLOAT "
                   "{V,max_deg}");
    return make_op(Op::VertexNeighborMean, {pos, nbrs}, VEC3, pos->size);
}

Var NormalConsistencyFaceTerm(const Var& pos, const Var& faces,
                              const Var& fadj) {
    DRESSI_REQUIRE(pos->vtype == VEC3 && pos->size.h == 1,
                   "NormalConsistencyFaceTerm: pos_tex must be VEC3 {V,1}");
    DRESSI_REQUIRE(faces->vtype == VEC3 && faces->size.h == 1 &&
                           fadj->vtype == VEC3 && fadj->size == faces->size,
                   "NormalConsistencyFaceTerm: faces_tex / face_adj_tex "
                   "must be VEC3 {F,1}");
    return make_op(Op::NormalConsistencyFaceTerm, {pos, faces, fadj}, VEC3,
                   faces->size);
}

Var NormalConsistencyVertexGrad(const Var& term, const Var& pos,
                                const Var& faces, const Var& vft) {
    DRESSI_REQUIRE(term->vtype == VEC3 && term->size == faces->size,
                   "NormalConsistencyVertexGrad: face_term must be VEC3 "
                   "{F,1}");
    DRESSI_REQUIRE(vft->vtype == FLOAT && vft->size.w == pos->size.w,
                   "NormalConsistencyVertexGrad: vtx_faces_tex must be "
                   "FLOAT {V,max_deg}");
    return make_op(Op::NormalConsistencyVertexGrad, {term, pos, faces, vft},
                   VEC3, pos->size);
}

// LookupFaces (f_ops.cpp:1568-1619)
Var LookupFaces(const Var& attr, const Var& faces_tex, const Var& vft,
                uint32_t corner) {
    DRESSI_REQUIRE(!is_int(attr->vtype) && !is_mat(attr->vtype) &&
                           attr->size.h == 1,
                   "LookupFaces: vtx_attr must be a float {V,1} Variable");
    DRESSI_REQUIRE(faces_tex->vtype == VEC3 && faces_tex->size.h == 1,
                   "LookupFaces: faces_tex must be VEC3 {F,1}");
    DRESSI_REQUIRE(vft->vtype == FLOAT && vft->size.w == attr->size.w,
                   "LookupFaces: vtx_faces_tex must be FLOAT {V,max_deg}");
    DRESSI_REQUIRE(corner < 3, "LookupFaces: corner must be 0, 1 or 2");
    return make_op(Op::LookupFaces, {attr, faces_tex, vft}, attr->vtype,
                   {faces_tex->size.w, 1}, {}, {int64_t(corner)});
}

// FaceFetch (f_ops.cpp:1736-1799)
Var FaceFetch(const Var& tri_attr, const Var& idx, const Var& prj0,
              const Var& prj1, const Var& prj2, const Var& seed,
              float radius_px, uint32_t n_samples) {
    DRESSI_REQUIRE(!is_int(tri_attr->vtype) && !is_mat(tri_attr->vtype) &&
                           tri_attr->size.h == 1,
                   "FaceFetch: tri_attr must be a float {F,1} Variable");
    DRESSI_REQUIRE(idx->vtype == FLOAT, "FaceFetch: idx_img must be FLOAT");
    for (const Var& p : {prj0, prj1, prj2})
        DRESSI_REQUIRE(p->vtype == VEC4 && p->size == tri_attr->size,
                       "FaceFetch: tri_prj_k must be VEC4 {F,1}");
    DRESSI_REQUIRE(seed->vtype == FLOAT && seed->size.uniform(),
                   "FaceFetch: seed must be FLOAT {1,1}");
    return make_op(Op::FaceFetch, {tri_attr, idx, prj0, prj1, prj2, seed},
                   tri_attr->vtype, idx->size, {radius_px},
                   {int64_t(n_samples)});
}

// Texture / TextureBilinear (f_ops.cpp:2605-2780). The inverse-UV table
// is a third input here (the reference captures it in the backward).
Var Texture(const Var& tex, const Var& uv, const Var& inv_uv) {
    DRESSI_REQUIRE(!is_int(tex->vtype) && !is_mat(tex->vtype),
                   "Texture: tex must be a float image");
    DRESSI_REQUIRE(uv->vtype == VEC2, "Texture: uv must be VEC2");
    DRESSI_REQUIRE(inv_uv->vtype == VEC4 && inv_uv->size == tex->size,
                   "Texture: inv_uv must be VEC4 of the texture's size");
    return make_op(Op::Texture, {tex, uv, inv_uv}, tex->vtype, uv->size);
}

Var TextureBilinear(const Var& tex, const Var& uv, const Var& inv_uv) {
    DRESSI_REQUIRE(!is_int(tex->vtype) && !is_mat(tex->vtype),
                   "TextureBilinear: tex must be a float image");
    DRESSI_REQUIRE(uv->vtype == VEC2, "TextureBilinear: uv must be VEC2");
    DRESSI_REQUIRE(inv_uv->vtype == VEC4 && inv_uv->size == tex->size,
                   "TextureBilinear: inv_uv must be VEC4 of the texture's "
                   "size");
    return make_op(Op::TextureBilinear, {tex, uv, inv_uv}, tex->vtype,
                   uv->size);
}

// IBL (f_ops.cpp:2785-3419)
Var EquirectSample(const Var& map, const Var& dir) {
    DRESSI_REQUIRE(!is_int(map->vtype) && !is_mat(map->vtype),
                   "EquirectSample: map must be a float image");
    DRESSI_REQUIRE(dir->vtype == VEC3, "EquirectSample: dir must be VEC3");
    return make_op(Op::EquirectSample, {map, dir}, map->vtype, dir->size);
}

Var IrradianceConv(const Var& env, ImgSize out) {
    DRESSI_REQUIRE(!is_int(env->vtype) && !is_mat(env->vtype),
                   "IrradianceConv: env must be a float image");
    return make_op(Op::IrradianceConv, {env}, env->vtype, out);
}

Var PrefilterConv(const Var& env, ImgSize out, float roughness) {
    DRESSI_REQUIRE(!is_int(env->vtype) && !is_mat(env->vtype),
                   "PrefilterConv: env must be a float image");
    DRESSI_REQUIRE(!out.uniform(), "PrefilterConv: 1x1 output level");
    return make_op(Op::PrefilterConv, {env}, env->vtype, out, {roughness});
}

Var BrdfIntegrationLut(ImgSize size, uint32_t n_samples) {
    return make_op(Op::BrdfLut, {}, VEC2, size, {}, {int64_t(n_samples)});
}

Var AvgPool2x2(const Var& x) {
    DRESSI_REQUIRE(!x->size.uniform(), "AvgPool2x2 on {1,1} input");
    return make_op(Op::AvgPool2x2, {x}, x->vtype,
                   {(x->size.w + 1) / 2, (x->size.h + 1) / 2});
}

// PixelFetch / TileFetch (f_ops.cpp:1803-1866)
Var PixelFetch(const Var& tex, uint32_t x_index, const Var& row_idx) {
    DRESSI_REQUIRE(!is_int(tex->vtype) && !is_mat(tex->vtype),
                   "PixelFetch: tex must be a float image");
    DRESSI_REQUIRE(x_index < tex->size.w, "PixelFetch: x out of range");
    DRESSI_REQUIRE(row_idx->vtype == FLOAT && row_idx->size.uniform(),
                   "PixelFetch: row_idx must be FLOAT {1,1}");
    return make_op(Op::PixelFetch, {tex, row_idx}, tex->vtype, {1, 1}, {},
                   {int64_t(x_index)});
}

Var TileFetch(const Var& atlas, const Var& tile_idx, uint32_t tile_h) {
    DRESSI_REQUIRE(tile_h >= 1 && !is_int(atlas->vtype) &&
                           !is_mat(atlas->vtype) &&
                           atlas->size.h % tile_h == 0,
                   "TileFetch: atlas height must be a multiple of tile_h");
    DRESSI_REQUIRE(tile_idx->vtype == FLOAT && tile_idx->size.uniform(),
                   "TileFetch: tile_idx must be FLOAT {1,1}");
    return make_op(Op::TileFetch, {atlas, tile_idx}, atlas->vtype,
                   {atlas->size.w, tile_h}, {}, {int64_t(tile_h)});
}

}  // namespace F

// ------------------------------------------------------------ by name

namespace {

const std::map<std::string, Op>& unary_ops() {
    static const std::map<std::string, Op> m = {
        {"Sin", Op::Sin}, {"Cos", Op::Cos}, {"Tan", Op::Tan},
        {"Asin", Op::Asin}, {"Acos", Op::Acos}, {"Atan", Op::Atan},
        {"Exp", Op::Exp}, {"Exp2", Op::Exp2}, {"Log", Op::Log},
        {"Log2", Op::Log2}, {"Sqrt", Op::Sqrt},
        {"InverseSqrt", Op::InverseSqrt}, {"Abs", Op::Abs},
        {"Sign", Op::Sign}, {"Floor", Op::Floor}, {"Fract", Op::Fract},
        {"Sigmoid", Op::Sigmoid}};
    return m;
}

const std::map<std::string, Op>& binary_ops() {
    static const std::map<std::string, Op> m = {
        {"Atan2", Op::Atan2}, {"Mod", Op::Mod}, {"Pow", Op::Pow},
        {"Max", Op::Max}, {"Min", Op::Min}, {"Step", Op::Step},
        {"Less", Op::Less}, {"LessEqual", Op::LessEqual},
        {"Greater", Op::Greater}, {"GreaterEqual", Op::GreaterEqual}};
    return m;
}

ImgSize size_arg(const std::vector<int64_t>& ip, size_t i,
                 const std::string& name) {
    DRESSI_REQUIRE(ip.size() >= i + 2 && ip[i] >= 1 && ip[i + 1] >= 1 &&
                           ip[i] <= 1 << 30 && ip[i + 1] <= 1 << 30,
                   name + ": expects an image size (w, h) parameter");
    return {uint32_t(ip[i]), uint32_t(ip[i + 1])};
}

void nargs(const std::string& name, const Vars& xs, size_t lo, size_t hi) {
    DRESSI_REQUIRE(xs.size() >= lo && xs.size() <= hi,
                   name + ": wrong number of inputs");
}

}  // namespace

Var build_named(const std::string& name, const Vars& xs,
                const std::vector<float>& fp, const std::vector<int64_t>& ip) {
    auto fparam = [&](size_t i) {
        DRESSI_REQUIRE(fp.size() > i, name + ": missing float parameter");
        return fp[i];
    };
    auto iparam = [&](size_t i) {
        DRESSI_REQUIRE(ip.size() > i, name + ": missing integer parameter");
        return ip[i];
    };
    if (name == "Float") {
        nargs(name, xs, 0, 0);
        return F::Float(fparam(0));
    }
    if (name == "Vec2" || name == "Vec3" || name == "Vec4") {
        const size_t n = size_t(name[3] - '0');
        if (xs.empty()) {
            DRESSI_REQUIRE(fp.size() == n, name + ": expects " +
                                                   std::to_string(n) +
                                                   " float parameters");
            return F::Vec(fp);
        }
        Var v = F::Compose(xs);
        DRESSI_REQUIRE(ncomp(v->vtype) == n, name + ": component count");
        return v;
    }
    if (name == "Add" || name == "Sub" || name == "Mul" || name == "Div") {
        nargs(name, xs, 2, 2);
        if (name == "Add") return F::Add(xs[0], xs[1]);
        if (name == "Sub") return F::Sub(xs[0], xs[1]);
        if (name == "Mul") return F::Mul(xs[0], xs[1]);
        return F::Div(xs[0], xs[1]);
    }
    if (name == "Neg") {
        nargs(name, xs, 1, 1);
        return F::Neg(xs[0]);
    }
    if (auto it = unary_ops().find(name); it != unary_ops().end()) {
        nargs(name, xs, 1, 1);
        return F::Unary(it->second, xs[0]);
    }
    if (auto it = binary_ops().find(name); it != binary_ops().end()) {
        nargs(name, xs, 2, 2);
        return F::Binary(it->second, xs[0], xs[1]);
    }
    if (name == "Clamp" || name == "Mix" || name == "SmoothStep") {
        nargs(name, xs, 3, 3);
        const Op op = name == "Clamp" ? Op::Clamp
                      : name == "Mix" ? Op::Mix
                                      : Op::SmoothStep;
        return F::Ternary(op, xs[0], xs[1], xs[2]);
    }
    if (name == "GetX" || name == "GetY" || name == "GetZ" || name == "GetW") {
        nargs(name, xs, 1, 1);
        const uint32_t c = name == "GetX" ? 0 : name == "GetY" ? 1
                           : name == "GetZ" ? 2 : 3;
        return F::Extract(xs[0], c, 1);
    }
    if (name == "ExtractComps") {
        nargs(name, xs, 1, 1);
        return F::Extract(xs[0], uint32_t(iparam(0)), uint32_t(iparam(1)));
    }
    if (name == "Compose") return F::Compose(xs);
    if (name == "Dot") { nargs(name, xs, 2, 2); return F::Dot(xs[0], xs[1]); }
    if (name == "Cross") {
        nargs(name, xs, 2, 2);
        return F::Cross(xs[0], xs[1]);
    }
    if (name == "Length") { nargs(name, xs, 1, 1); return F::Length(xs[0]); }
    if (name == "Distance") {
        nargs(name, xs, 2, 2);
        return F::Length(F::Sub(xs[0], xs[1]));
    }
    if (name == "Normalize") {
        nargs(name, xs, 1, 1);
        return F::Normalize(xs[0]);
    }
    if (name == "Reflect") {
        // Sub(i, Mul(Mul(2, Dot(n, i)), n)) (f_ops.cpp:720-723)
        nargs(name, xs, 2, 2);
        return F::Sub(xs[0], F::Mul(F::Mul(F::Float(2.f),
                                           F::Dot(xs[1], xs[0])),
                                    xs[1]));
    }
    if (name == "CompSum") { nargs(name, xs, 1, 1); return F::CompSum(xs[0]); }
    if (name == "MatMul") {
        nargs(name, xs, 2, 2);
        return F::MatMul(xs[0], xs[1]);
    }
    if (name == "Transpose") {
        nargs(name, xs, 1, 1);
        return F::Transpose(xs[0]);
    }
    if (name == "OuterProduct") {
        nargs(name, xs, 2, 2);
        return F::OuterProduct(xs[0], xs[1]);
    }
    if (name == "SumPixelWise") return F::SumPixelWise(xs);
    if (name == "Sum") { nargs(name, xs, 1, 1); return F::Sum(xs[0]); }
    if (name == "Mean") { nargs(name, xs, 1, 1); return F::Mean(xs[0]); }
    if (name == "SumAll") { nargs(name, xs, 1, 1); return F::SumAll(xs[0]); }
    if (name == "Broadcast") {
        nargs(name, xs, 1, 1);
        return F::Broadcast(xs[0], size_arg(ip, 0, name));
    }
    if (name == "StopGradient") {
        nargs(name, xs, 1, 1);
        return F::StopGradient(xs[0]);
    }
    if (name == "SetFragDepth") {
        nargs(name, xs, 1, 1);
        return F::SetFragDepth(xs[0]);
    }
    if (name == "ScreenCoord") {
        nargs(name, xs, 0, 0);
        return F::ScreenCoord(size_arg(ip, 0, name));
    }
    if (name == "Rasterize") {
        nargs(name, xs, 3, 3);
        return F::Rasterize(xs[0], xs[1], xs[2], size_arg(ip, 0, name));
    }
    if (name == "RasterizeFaceId") {
        nargs(name, xs, 3, 3);
        return F::RasterizeFaceId(xs[0], xs[1], xs[2], size_arg(ip, 0, name));
    }
    if (name == "RasterizeSoft") {
        nargs(name, xs, 6, 7);
        return F::RasterizeSoft(xs[0], xs[1], xs[2], xs[3], xs[4], xs[5],
                                xs.size() == 7 ? xs[6] : nullptr,
                                size_arg(ip, 0, name), fparam(0));
    }
    if (name == "SoftClip") {
        nargs(name, xs, 2, 2);
        return F::SoftClip(xs[0], xs[1], size_arg(ip, 0, name), fparam(0));
    }
    if (name == "AntiAlias") {
        nargs(name, xs, 6, 6);
        return F::AntiAlias(xs[0], xs[1], xs[2], xs[3], xs[4], xs[5],
                            ip.empty() ? 8u : uint32_t(ip[0]));
    }
    if (name == "VertexNeighborMean") {
        nargs(name, xs, 2, 2);
        return F::VertexNeighborMean(xs[0], xs[1]);
    }
    if (name == "NormalConsistencyFaceTerm") {
        nargs(name, xs, 3, 3);
        return F::NormalConsistencyFaceTerm(xs[0], xs[1], xs[2]);
    }
    if (name == "NormalConsistencyVertexGrad") {
        nargs(name, xs, 4, 4);
        return F::NormalConsistencyVertexGrad(xs[0], xs[1], xs[2], xs[3]);
    }
    if (name == "LookupFaces") {
        nargs(name, xs, 3, 3);
        return F::LookupFaces(xs[0], xs[1], xs[2], uint32_t(iparam(0)));
    }
    if (name == "FaceFetch") {
        nargs(name, xs, 6, 6);
        return F::FaceFetch(xs[0], xs[1], xs[2], xs[3], xs[4], xs[5],
                            fparam(0), ip.empty() ? 4u : uint32_t(ip[0]));
    }
    if (name == "Texture") {
        nargs(name, xs, 3, 3);
        return F::Texture(xs[0], xs[1], xs[2]);
    }
    if (name == "TextureBilinear") {
        nargs(name, xs, 3, 3);
        return F::TextureBilinear(xs[0], xs[1], xs[2]);
    }
    if (name == "EquirectSample") {
        nargs(name, xs, 2, 2);
        return F::EquirectSample(xs[0], xs[1]);
    }
    if (name == "IrradianceConv") {
        nargs(name, xs, 1, 1);
        return F::IrradianceConv(xs[0], size_arg(ip, 0, name));
    }
    if (name == "PrefilterConv") {
        nargs(name, xs, 1, 1);
        return F::PrefilterConv(xs[0], size_arg(ip, 0, name), fparam(0));
    }
    if (name == "BrdfIntegrationLut") {
        nargs(name, xs, 0, 0);
        return F::BrdfIntegrationLut(size_arg(ip, 0, name),
                                     ip.size() > 2 ? uint32_t(ip[2]) : 512u);
    }
    if (name == "AvgPool2x2") {
        nargs(name, xs, 1, 1);
        return F::AvgPool2x2(xs[0]);
    }
    if (name == "PixelFetch") {
        nargs(name, xs, 2, 2);
        return F::PixelFetch(xs[0], uint32_t(iparam(0)), xs[1]);
    }
    if (name == "TileFetch") {
        nargs(name, xs, 2, 2);
        return F::TileFetch(xs[0], xs[1], uint32_t(iparam(0)));
    }
    throw_error(kErrInvalid, "unknown or unsupported op '" + name + "'",
                __FILE__, __LINE__);
}

// --------------------------------------------------------- backward rules

namespace {

using namespace F;

Var one() { return Float(1.f); }

// Gradient op of a special kernel (never differentiated itself).
Var grad_op(Op op, const Vars& xs, VType vt, ImgSize size,
            std::vector<float> fp = {}, std::vector<int64_t> ip = {}) {
    return make_op(op, xs, vt, size, std::move(fp), std::move(ip));
}

Var compose_replicate(const Var& s, uint32_t n) {
    return n == 1 ? s : Compose(Vars(n, s));
}

}  // namespace

Var backward_of(const Func& f, const Var& gy, uint32_t idx) {
    const Vars& xs = f->xs;
    Var y = f->y.lock();
    switch (f->op) {
    // arithmetic (f_ops.cpp:194-265)
    case Op::Add: return gy;
    case Op::Sub: return idx == 0 ? gy : Neg(gy);
    case Op::Mul: return idx == 0 ? Mul(gy, xs[1]) : Mul(gy, xs[0]);
    case Op::Div:
        if (idx == 0) return Div(gy, xs[1]);
        return Neg(Div(Mul(gy, xs[0]), Mul(xs[1], xs[1])));
    case Op::Neg: return Neg(gy);
    // UnaryMath: gy * dydx (f_ops.cpp:267-448)
    case Op::Sin: return Mul(gy, Unary(Op::Cos, xs[0]));
    case Op::Cos: return Mul(gy, Neg(Unary(Op::Sin, xs[0])));
    case Op::Tan: return Mul(gy, Add(one(), Mul(y, y)));
    case Op::Asin:
        return Mul(gy, Unary(Op::InverseSqrt, Sub(one(), Mul(xs[0], xs[0]))));
    case Op::Acos:
        return Mul(gy, Neg(Unary(Op::InverseSqrt,
                                 Sub(one(), Mul(xs[0], xs[0])))));
    case Op::Atan: return Mul(gy, Div(one(), Add(one(), Mul(xs[0], xs[0]))));
    case Op::Atan2: {
        Var denom = Add(Mul(xs[0], xs[0]), Mul(xs[1], xs[1]));
        if (idx == 0) return Div(Mul(gy, xs[1]), denom);
        return Neg(Div(Mul(gy, xs[0]), denom));
    }
    case Op::Exp: return Mul(gy, y);
    case Op::Exp2: return Mul(gy, Mul(y, Float(0.6931471805599453f)));
    case Op::Log: return Mul(gy, Div(one(), xs[0]));
    case Op::Log2: return Mul(gy, Div(Float(1.4426950408889634f), xs[0]));
    case Op::Sqrt: return Mul(gy, Div(Float(0.5f), y));
    case Op::InverseSqrt:
        return Mul(gy, Mul(Float(-0.5f), Mul(y, Mul(y, y))));
    case Op::Abs: return Mul(gy, Unary(Op::Sign, xs[0]));
    case Op::Sign: case Op::Floor: case Op::Step: case Op::Less:
    case Op::LessEqual: case Op::Greater: case Op::GreaterEqual:
    case Op::StopGradient: case Op::Const: case Op::ScreenCoord:
        return nullptr;
    case Op::Fract: return Mul(gy, one());
    case Op::Mod:
        if (idx == 0) return gy;
        return Neg(Mul(gy, Unary(Op::Floor, Div(xs[0], xs[1]))));
    case Op::Pow:
        if (idx == 0)
            return Mul(gy, Mul(xs[1], Binary(Op::Pow, xs[0],
                                             Sub(xs[1], one()))));
        return Mul(gy, Mul(y, Unary(Op::Log, xs[0])));
    // Max / Min / Clamp / Mix / SmoothStep / Sigmoid (f_ops.cpp:450-575)
    case Op::Max: {
        Var mask = Binary(Op::Step, xs[1], xs[0]);  // x0 >= x1
        return idx == 0 ? Mul(gy, mask) : Mul(gy, Sub(one(), mask));
    }
    case Op::Min: {
        Var mask = Binary(Op::Step, xs[0], xs[1]);  // x1 >= x0
        return idx == 0 ? Mul(gy, mask) : Mul(gy, Sub(one(), mask));
    }
    case Op::Clamp: {
        if (idx != 0) return nullptr;
        Var inside = Mul(Binary(Op::Step, xs[1], xs[0]),
                         Binary(Op::Step, xs[0], xs[2]));
        return Mul(gy, inside);
    }
    case Op::Mix:
        if (idx == 0) return Mul(gy, Sub(one(), xs[2]));
        if (idx == 1) return Mul(gy, xs[2]);
        return Mul(gy, Sub(xs[1], xs[0]));
    case Op::SmoothStep: {
        if (idx != 2) return nullptr;
        Var range = Sub(xs[1], xs[0]);
        Var t = Ternary(Op::Clamp, Div(Sub(xs[2], xs[0]), range), Float(0.f),
                        one());
        Var dt = Div(Mul(Float(6.f), Mul(t, Sub(one(), t))), range);
        return Mul(gy, dt);
    }
    case Op::Sigmoid: return Mul(gy, Mul(y, Sub(one(), y)));
    // vectors (f_ops.cpp:35-124, 600-760)
    case Op::Compose: {
        uint32_t ofs = 0;
        for (uint32_t i = 0; i < idx; i++) ofs += ncomp(xs[i]->vtype);
        return Extract(gy, ofs, ncomp(xs[idx]->vtype));
    }
    case Op::Extract: {
        const uint32_t ofs = uint32_t(f->ip[0]), n = uint32_t(f->ip[1]);
        const uint32_t src_n = ncomp(xs[0]->vtype);
        Vars parts;
        for (uint32_t j = 0; j < src_n; j++) {
            if (ofs <= j && j < ofs + n)
                parts.push_back(n == 1 ? gy : Extract(gy, j - ofs, 1));
            else
                parts.push_back(Float(0.f));
        }
        return Compose(parts);
    }
    case Op::Dot: return Mul(gy, xs[idx == 0 ? 1 : 0]);
    case Op::Cross: return idx == 0 ? Cross(xs[1], gy) : Cross(gy, xs[0]);
    case Op::Length: return Mul(Div(gy, y), xs[0]);
    case Op::Normalize: {
        Var len = Length(xs[0]);
        return Div(Sub(gy, Mul(y, Dot(y, gy))), len);
    }
    case Op::CompSum:
        return compose_replicate(gy, ncomp(xs[0]->vtype));
    case Op::MatMul: {
        const bool vec_rhs = is_vec(xs[1]->vtype);
        if (vec_rhs) {
            if (idx == 0) return OuterProduct(gy, xs[1]);
            return MatMul(Transpose(xs[0]), gy);
        }
        if (idx == 0) return MatMul(gy, Transpose(xs[1]));
        return MatMul(Transpose(xs[0]), gy);
    }
    case Op::Transpose: return Transpose(gy);
    case Op::OuterProduct:
        if (idx == 0) return MatMul(gy, xs[1]);
        return MatMul(Transpose(gy), xs[0]);
    case Op::SumPixelWise: case Op::SetFragDepth: return gy;
    case Op::Broadcast: return Sum(gy);
    case Op::Sum: return Broadcast(gy, xs[0]->size);
    case Op::SumPartial: case Op::SumAll: return nullptr;
    // special kernels
    case Op::RasterizeSoft:
        if (idx != 3) return nullptr;
        return grad_op(Op::RasterizeSoftGrad, {gy, y, xs[3], xs[4], xs[5]},
                       VEC4, xs[3]->size, f->fp);
    case Op::AntiAlias:
        if (idx == 0)
            return grad_op(Op::AntiAliasGradImg, {gy, xs[1], xs[2], xs[3]},
                           gy->vtype, gy->size);
        if (idx == 2)
            return grad_op(Op::AntiAliasGradVtx,
                           {gy, xs[0], xs[1], xs[2], xs[3], xs[4], xs[5]},
                           VEC4, xs[2]->size, {}, f->ip);
        return nullptr;
    case Op::LookupFaces:
        if (idx != 0) return nullptr;
        return grad_op(Op::LookupFacesGrad, {gy, xs[1], xs[2]}, gy->vtype,
                       {xs[2]->size.w, 1}, {}, f->ip);
    case Op::FaceFetch:
        if (idx != 0) return nullptr;
        return grad_op(Op::FaceFetchGrad,
                       {gy, xs[1], xs[2], xs[3], xs[4], xs[5]}, gy->vtype,
                       xs[2]->size, f->fp, f->ip);
    case Op::Texture:
        if (idx != 0) return nullptr;
        return grad_op(Op::GatherInvUV, {gy, xs[2], xs[1]}, gy->vtype,
                       xs[2]->size);
    case Op::TextureBilinear:
        if (idx != 0) return nullptr;
        return grad_op(Op::GatherInvUVBilinear, {gy, xs[2], xs[1]}, gy->vtype,
                       xs[2]->size);
    case Op::EquirectSample:
        if (idx != 0) return nullptr;
        return grad_op(Op::EquirectSampleGrad, {gy, xs[1]}, gy->vtype,
                       xs[0]->size);
    case Op::IrradianceConv:
        return grad_op(Op::IrradianceConvGrad, {gy}, gy->vtype, xs[0]->size);
    case Op::PrefilterConv:
        return grad_op(Op::PrefilterConvGrad, {gy}, gy->vtype, xs[0]->size,
                       f->fp);
    case Op::AvgPool2x2:
        return grad_op(Op::AvgPool2x2Grad, {gy}, gy->vtype, xs[0]->size);
    default:
        return nullptr;  // forward-only ops
    }
}

// ---------------------------------------------------------- BuildBackward

namespace {

// SumToShape (build_backward.cpp:13-34)
Var sum_to_shape(const Var& grad, const Var& target) {
    Var g = grad;
    const uint32_t nt = ncomp(target->vtype), ng = ncomp(g->vtype);
    if (ng != nt) {
        DRESSI_REQUIRE(nt == 1, "Gradient component count exceeds target and "
                                "target is not scalar");
        g = CompSum(g);
    }
    if (target->size.uniform() && !g->size.uniform())
        g = Sum(g);
    else if (!target->size.uniform() && g->size.uniform())
        g = Broadcast(g, target->size);
    DRESSI_REQUIRE(g->size == target->size,
                   "Gradient image size does not reduce to target size");
    return g;
}

// SumContribs (build_backward.cpp:41-58): a tree of SumPixelWise nodes of
// arity <= 4.
Var sum_contribs(Vars c) {
    while (c.size() > 1) {
        Vars next;
        for (size_t i = 0; i < c.size(); i += 4) {
            const size_t n = std::min<size_t>(4, c.size() - i);
            if (n == 1)
                next.push_back(c[i]);
            else
                next.push_back(SumPixelWise(Vars(c.begin() + i,
                                                 c.begin() + i + n)));
        }
        c = std::move(next);
    }
    return c[0];
}

}  // namespace

void build_backward(const Var& loss, Vars* inputs, Vars* grads) {
    DRESSI_REQUIRE(loss, "Null loss Variable");
    DRESSI_REQUIRE(!is_int(loss->vtype) && !is_mat(loss->vtype),
                   "Loss must be a float scalar/vector Variable");
    std::map<uint64_t, std::pair<Var, Vars>> contrib;  // by variable id
    auto by_id = [](const Func& a, const Func& b) { return a->id < b->id; };
    std::vector<Func> heap;
    std::unordered_set<uint64_t> seen;
    auto push = [&](const Func& f) {
        heap.push_back(f);
        std::push_heap(heap.begin(), heap.end(), by_id);
    };
    contrib[loss->id] = {loss, {Float(1.f)}};
    if (loss->creator) push(loss->creator);
    while (!heap.empty()) {
        std::pop_heap(heap.begin(), heap.end(), by_id);
        Func f = heap.back();
        heap.pop_back();
        if (!seen.insert(f->id).second) continue;
        Var y = f->out();
        auto it = contrib.find(y->id);
        if (it == contrib.end()) continue;  // no gradient path reached f
        Var gy = sum_contribs(it->second.second);
        contrib.erase(it);
        // materialise broadcast gradients to y's full shape
        // (build_backward.cpp:108-119)
        const uint32_t yc = ncomp(y->vtype);
        if (ncomp(gy->vtype) == 1 && yc > 1)
            gy = Mul(gy, Vec(std::vector<float>(yc, 1.f)));
        if (gy->size.uniform() && !y->size.uniform())
            gy = Broadcast(gy, y->size);
        for (uint32_t i = 0; i < f->xs.size(); i++) {
            const Var& x = f->xs[i];
            if (!x->req_grad) continue;
            Var gx = backward_of(f, gy, i);
            if (!gx) continue;
            gx = sum_to_shape(gx, x);
            auto& slot = contrib[x->id];
            slot.first = x;
            slot.second.push_back(gx);
            if (x->creator) push(x->creator);
        }
    }
    inputs->clear();
    grads->clear();
    for (auto& [id, e] : contrib) {
        if (id == loss->id) continue;
        inputs->push_back(e.first);
        grads->push_back(sum_to_shape(sum_contribs(e.second), e.first));
    }
}

std::vector<Func> traverse(const Vars& roots) {
    std::vector<Func> funcs;
    std::unordered_set<uint64_t> vf, vv;
    std::vector<Var> stack;
    for (const auto& r : roots)
        if (r) stack.push_back(r);
    while (!stack.empty()) {
        Var v = stack.back();
        stack.pop_back();
        if (!vv.insert(v->id).second) continue;
        Func c = v->creator;
        if (!c || !vf.insert(c->id).second) continue;
        funcs.push_back(c);
        for (const auto& x : c->xs) stack.push_back(x);
    }
    std::sort(funcs.begin(), funcs.end(),
              [](const Func& a, const Func& b) { return a->id < b->id; });
    return funcs;
}

}  // namespace graph
}  // namespace dressi
