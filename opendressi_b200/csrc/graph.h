// The generic graph path: Variables and Functions built by F:: ops, the
// reverse-mode graph (BuildBackward), the fusion planner that lowers a graph
// to pixel programs + reductions + special kernels, and the CUDA-graph
// executor behind DressiAD (include/dressi_b200.h, dressi_graph_* /
// dressi_ad_*).
//
// Reference counterparts (paths inside unclearness/opendressi):
//   Variable / Function nodes          include/dressi/variable.h:18-49,
//                                      include/dressi/function.h,
//                                      src/core/node.h:40-65
//   F:: ops, inference, backward rules include/dressi/f.h:12-317,
//                                      src/core/f_ops.cpp, src/core/infer.cpp
//   BuildBackward / SumToShape         src/core/build_backward.cpp:13-149
//   reactive pruning                   src/pack/reactive.cpp:10-113
//   DressiAD::execStep                 src/dressi_ad.cpp:280-530
//
// Values are float images: [h][w][ncomp], row-major, components
// interleaved; integer types hold their values as floats, as the
// reference's CpuTensor does.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "common.h"

namespace dressi {
namespace graph {

// The reference's VType numbering (include/dressi/types.h:12-25).
enum VType : int {
    FLOAT = 0, VEC2, VEC3, VEC4, MAT2, MAT3, MAT4, INT, IVEC2, IVEC3, IVEC4,
    UINT
};
uint32_t ncomp(VType t);
bool is_int(VType t);
bool is_mat(VType t);
bool is_vec(VType t);  // VEC2..VEC4 / IVEC2..IVEC4
VType vec_of(uint32_t n, bool integer = false);
uint32_t mat_dim(VType t);

struct ImgSize {
    uint32_t w = 1, h = 1;
    bool uniform() const { return w == 1 && h == 1; }
    bool operator==(const ImgSize& o) const { return w == o.w && h == o.h; }
    bool operator!=(const ImgSize& o) const { return !(*this == o); }
    size_t pixels() const { return size_t(w) * h; }
};

// Every op of the graph. Elementwise ops are evaluated per pixel (inputs of
// the output's size or uniform {1,1}); the others are kernels of their own.
enum class Op : int {
    // constants and pixel-wise maps
    Const, Add, Sub, Mul, Div, Neg, Sin, Cos, Tan, Asin, Acos, Atan, Atan2,
    Exp, Exp2, Log, Log2, Sqrt, InverseSqrt, Abs, Sign, Floor, Fract, Mod,
    Pow, Max, Min, Clamp, Mix, Step, SmoothStep, Sigmoid, Less, LessEqual,
    Greater, GreaterEqual, Compose, Extract, Dot, Cross, Length, Normalize,
    CompSum, MatMul, Transpose, OuterProduct, SumPixelWise, StopGradient,
    SetFragDepth, Broadcast, ScreenCoord,
    // reductions
    Sum, SumPartial, SumAll,
    // special kernels
    Rasterize, RasterizeFaceId, RasterizeSoft, RasterizeSoftGrad, SoftClip,
    AntiAlias, AntiAliasGradImg, AntiAliasGradVtx, VertexNeighborMean,
    NormalConsistencyFaceTerm, NormalConsistencyVertexGrad, LookupFaces,
    LookupFacesGrad, FaceFetch, FaceFetchGrad, Texture, TextureBilinear,
    GatherInvUV, GatherInvUVBilinear, EquirectSample, EquirectSampleGrad,
    IrradianceConv, IrradianceConvGrad, PrefilterConv, PrefilterConvGrad,
    BrdfLut, AvgPool2x2, AvgPool2x2Grad, PixelFetch, TileFetch,
    kCount
};
const char* op_name(Op op);
bool is_pixelwise(Op op);

struct FuncNode;

struct VarNode {
    uint64_t id = 0;
    VType vtype = FLOAT;
    ImgSize size;
    std::shared_ptr<FuncNode> creator;            // strong: creator is older
    std::vector<std::weak_ptr<FuncNode>> users;   // weak: forward edges
    bool req_grad = false;
    bool dirty = true;
    bool is_const = false;       // inline {1,1} constant (F::Float etc.)
    std::vector<float> cval;     // its components
};
using Var = std::shared_ptr<VarNode>;
using Vars = std::vector<Var>;

struct FuncNode {
    uint64_t id = 0;
    Op op = Op::Const;
    Vars xs;                     // strong: inputs are older
    std::weak_ptr<VarNode> y;    // weak: forward edge
    std::vector<float> fp;       // float parameters (radius, roughness, ...)
    std::vector<int64_t> ip;     // integer parameters (offsets, counts, ...)
    Var out() const {
        Var v = y.lock();
        DRESSI_REQUIRE(v, "function output no longer referenced");
        return v;
    }
};
using Func = std::shared_ptr<FuncNode>;

uint64_t next_node_id();

// Makes a function node over xs with an output of (vt, size).
Var make_op(Op op, const Vars& xs, VType vt, ImgSize size,
            std::vector<float> fp = {}, std::vector<int64_t> ip = {});
Var make_leaf(VType vt, ImgSize size);
void set_requires_grad_recursively(const Var& v, bool req);
void set_dirty_recursively(const Var& v, bool dirty);

// ------------------------------------------------------------ F:: ops
namespace F {
Var Float(float v);
Var Vec(const std::vector<float>& vals);  // 2..4 constants
Var Add(const Var& a, const Var& b);
Var Sub(const Var& a, const Var& b);
Var Mul(const Var& a, const Var& b);
Var Div(const Var& a, const Var& b);
Var Neg(const Var& x);
Var Unary(Op op, const Var& x);
Var Binary(Op op, const Var& a, const Var& b);
Var Ternary(Op op, const Var& a, const Var& b, const Var& c);
Var Compose(const Vars& parts);
Var Extract(const Var& v, uint32_t ofs, uint32_t n);
Var Dot(const Var& a, const Var& b);
Var Cross(const Var& a, const Var& b);
Var Length(const Var& v);
Var Normalize(const Var& v);
Var CompSum(const Var& v);
Var MatMul(const Var& a, const Var& b);
Var Transpose(const Var& m);
Var OuterProduct(const Var& c, const Var& r);
Var SumPixelWise(const Vars& xs);
Var Sum(const Var& x);
Var Mean(const Var& x);
Var SumAll(const Var& x);
Var Broadcast(const Var& x, ImgSize size);
Var StopGradient(const Var& x);
Var SetFragDepth(const Var& x);
Var ScreenCoord(ImgSize size);
Var Rasterize(const Var& clip, const Var& attr, const Var& faces,
              ImgSize screen);
Var RasterizeFaceId(const Var& clip, const Var& dummy, const Var& faces,
                    ImgSize screen);
Var RasterizeSoft(const Var& soft_clip, const Var& face_id,
                  const Var& faces_soft, const Var& clip_hard,
                  const Var& faces_tex, const Var& vtx_faces_tex,
                  const Var& prev_depth, ImgSize screen, float radius_px);
Var SoftClip(const Var& clip_hard, const Var& faces_tex, ImgSize screen,
             float radius_px);
Var AntiAlias(const Var& img, const Var& tri_id, const Var& clip,
              const Var& faces, const Var& vtx_faces_tex, const Var& seed,
              uint32_t n_samples);
Var VertexNeighborMean(const Var& pos, const Var& nbrs);
Var NormalConsistencyFaceTerm(const Var& pos, const Var& faces,
                              const Var& fadj);
Var NormalConsistencyVertexGrad(const Var& term, const Var& pos,
                                const Var& faces, const Var& vft);
Var LookupFaces(const Var& attr, const Var& faces_tex, const Var& vft,
                uint32_t corner);
Var FaceFetch(const Var& tri_attr, const Var& idx, const Var& prj0,
              const Var& prj1, const Var& prj2, const Var& seed,
              float radius_px, uint32_t n_samples);
Var Texture(const Var& tex, const Var& uv, const Var& inv_uv);
Var TextureBilinear(const Var& tex, const Var& uv, const Var& inv_uv);
Var EquirectSample(const Var& map, const Var& dir);
Var IrradianceConv(const Var& env, ImgSize out);
Var PrefilterConv(const Var& env, ImgSize out, float roughness);
Var BrdfIntegrationLut(ImgSize size, uint32_t n_samples);
Var AvgPool2x2(const Var& x);
Var PixelFetch(const Var& tex, uint32_t x_index, const Var& row_idx);
Var TileFetch(const Var& atlas, const Var& tile_idx, uint32_t tile_h);
}  // namespace F

// Builds an op from its reference name ("Add", "RasterizeSoft", ...), the
// input variables and its float / integer parameters (the C ABI's generic
// constructor).
Var build_named(const std::string& name, const Vars& xs,
                const std::vector<float>& fp, const std::vector<int64_t>& ip);

// d(sum of gy * y)/d x_idx as a graph (nullptr: no gradient).
Var backward_of(const Func& f, const Var& gy, uint32_t idx);

// BuildBackward: requires-grad leaves reachable from `loss` and their
// gradient variables.
void build_backward(const Var& loss, Vars* inputs, Vars* grads);
// Creators of `roots` and of everything they depend on, in creation order.
std::vector<Func> traverse(const Vars& roots);

// ------------------------------------------------------------ executor
class Engine;  // graph_exec.cu

}  // namespace graph
}  // namespace dressi
