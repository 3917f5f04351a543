// dressi/dressi.h -- the C++ graph API of libdressi_b200, header-only over
// its C ABI (dressi_b200.h: dressi_var_* / dressi_op / dressi_ad_*).
//
// The same classes and functions a program written against the reference's
// C++ API uses (include/dressi/{types,variable,f,dressi_ad}.h of
// unclearness/opendressi): Variable handles with value semantics, the F::
// op library and its operator overloads, and DressiAD (setLossVar,
// setOptimizer, addUpdate, markOutput, setGradOutputsEnabled, inputGrads,
// setRebuildCounts, setPackingMode, execStep, sendImg(s), recvImg(s)).
// Here execStep lowers the graph to CUDA kernels on the DressiAD's device
// and replays them as one CUDA graph; errors throw DressiError with the
// library's message.
//
// Link with -ldressi_b200 (opendressi_b200/libdressi_b200.so).
#ifndef DRESSI_B200_DRESSI_H
#define DRESSI_B200_DRESSI_H

#include <cstddef>
#include <cstdint>
#include <exception>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../dressi_b200.h"

namespace dressi {

enum VType {
    FLOAT = DRESSI_VT_FLOAT, VEC2, VEC3, VEC4, MAT2, MAT3, MAT4, INT, IVEC2,
    IVEC3, IVEC4, UINT
};

inline uint32_t NumComponents(VType t) {
    switch (t) {
    case VEC2: case IVEC2: return 2;
    case VEC3: case IVEC3: return 3;
    case VEC4: case IVEC4: case MAT2: return 4;
    case MAT3: return 9;
    case MAT4: return 16;
    default: return 1;
    }
}

struct ImgSize {
    uint32_t w = 1;
    uint32_t h = 1;
    bool operator==(const ImgSize& o) const { return w == o.w && h == o.h; }
    bool operator!=(const ImgSize& o) const { return !(*this == o); }
    bool isUniform() const { return w == 1 && h == 1; }
};

// Host image, row-major with interleaved components (no padding).
struct CpuImage {
    uint32_t width = 0, height = 0, channels = 0;
    std::vector<float> data;
    CpuImage() = default;
    CpuImage(uint32_t w, uint32_t h, uint32_t c, float fill = 0.f)
        : width(w), height(h), channels(c), data(size_t(w) * h * c, fill) {}
    ImgSize getImgSize() const { return {width, height}; }
    float& at(uint32_t x, uint32_t y, uint32_t c) {
        return data[(size_t(y) * width + x) * channels + c];
    }
    float at(uint32_t x, uint32_t y, uint32_t c) const {
        return data[(size_t(y) * width + x) * channels + c];
    }
};

struct CpuImageView {
    const float* data = nullptr;
    uint32_t width = 0, height = 0, channels = 0;
    CpuImageView() = default;
    CpuImageView(const float* d, uint32_t w, uint32_t h, uint32_t c)
        : data(d), width(w), height(h), channels(c) {}
    explicit CpuImageView(const CpuImage& img)
        : data(img.data.data()), width(img.width), height(img.height),
          channels(img.channels) {}
    size_t numElems() const { return size_t(width) * height * channels; }
};

class DressiError : public std::runtime_error {
public:
    explicit DressiError(const std::string& msg) : std::runtime_error(msg) {}
};

namespace detail {
inline void check(int rc) {
    if (rc == DRESSI_OK) return;
    std::string msg(size_t(dressi_last_error(nullptr, 0)) + 1, '\0');
    dressi_last_error(&msg[0], msg.size());
    msg.resize(msg.size() - 1);
    throw DressiError(msg);
}
}  // namespace detail

// A node of the computational graph (a 2-D image); copies share the node.
class Variable {
public:
    Variable(VType vtype = FLOAT, ImgSize size = {1, 1}) {
        detail::check(dressi_var_create(int(vtype), size.w, size.h, &h_));
    }
    Variable(std::nullptr_t) {}
    Variable(const Variable& o) {
        if (o.h_) detail::check(dressi_var_clone(o.h_, &h_));
    }
    Variable(Variable&& o) noexcept : h_(o.h_) { o.h_ = nullptr; }
    Variable& operator=(Variable o) noexcept {
        std::swap(h_, o.h_);
        return *this;
    }
    ~Variable() {
        if (h_) dressi_var_release(h_);
    }
    // Takes over a handle returned by the C ABI.
    static Variable adopt(dressi_var h) {
        Variable v(nullptr);
        v.h_ = h;
        return v;
    }
    dressi_var handle() const { return h_; }

    explicit operator bool() const { return h_ != nullptr; }
    bool operator==(const Variable& o) const {
        return (!h_ && !o.h_) || (h_ && o.h_ && id() == o.id());
    }
    bool operator!=(const Variable& o) const { return !(*this == o); }
    uint64_t id() const {
        uint64_t i = 0;
        detail::check(dressi_var_info(h_, nullptr, nullptr, nullptr, &i,
                                      nullptr));
        return i;
    }
    VType getVType() const {
        int vt = 0;
        detail::check(dressi_var_info(h_, &vt, nullptr, nullptr, nullptr,
                                      nullptr));
        return VType(vt);
    }
    ImgSize getImgSize() const {
        ImgSize s;
        detail::check(dressi_var_info(h_, nullptr, &s.w, &s.h, nullptr,
                                      nullptr));
        return s;
    }
    bool getRequiresGrad() const {
        int r = 0;
        detail::check(dressi_var_requires_grad(h_, &r));
        return r != 0;
    }
    void setRequiresGrad(bool req) {
        detail::check(dressi_var_set_requires_grad(h_, req ? 1 : 0, 0));
    }
    void setRequiresGradRecursively(bool req = true) {
        detail::check(dressi_var_set_requires_grad(h_, req ? 1 : 0, 1));
    }
    void setDirty(bool dirty) {
        detail::check(dressi_var_set_dirty(h_, dirty ? 1 : 0, 0));
    }
    void setDirtyRecursively(bool dirty) {
        detail::check(dressi_var_set_dirty(h_, dirty ? 1 : 0, 1));
    }

private:
    dressi_var h_ = nullptr;
};

using Variables = std::vector<Variable>;

namespace F {
namespace detail {
inline Variable op(const char* name, const Variables& xs,
                   const std::vector<float>& fp = {},
                   const std::vector<int64_t>& ip = {}) {
    std::vector<dressi_var> hs;
    for (const auto& x : xs) hs.push_back(x.handle());
    dressi_var out = nullptr;
    ::dressi::detail::check(dressi_op(
            name, hs.data(), uint32_t(hs.size()), fp.data(),
            uint32_t(fp.size()), ip.data(), uint32_t(ip.size()), &out));
    return Variable::adopt(out);
}
inline std::vector<int64_t> sz(ImgSize s) { return {s.w, s.h}; }
}  // namespace detail

// constants
inline Variable Float(float v) { return detail::op("Float", {}, {v}); }
inline Variable Vec2(float x, float y) { return detail::op("Vec2", {}, {x, y}); }
inline Variable Vec3(float x, float y, float z) {
    return detail::op("Vec3", {}, {x, y, z});
}
inline Variable Vec4(float x, float y, float z, float w) {
    return detail::op("Vec4", {}, {x, y, z, w});
}
// arithmetic and math
#define DRESSI_F1(N) \
    inline Variable N(const Variable& x) { return detail::op(#N, {x}); }
#define DRESSI_F2(N)                                       \
    inline Variable N(const Variable& a, const Variable& b) { \
        return detail::op(#N, {a, b});                     \
    }
#define DRESSI_F3(N)                                                       \
    inline Variable N(const Variable& a, const Variable& b, const Variable& c) { \
        return detail::op(#N, {a, b, c});                                  \
    }
DRESSI_F2(Add) DRESSI_F2(Sub) DRESSI_F2(Mul) DRESSI_F2(Div) DRESSI_F1(Neg)
DRESSI_F1(Sin) DRESSI_F1(Cos) DRESSI_F1(Tan) DRESSI_F1(Asin) DRESSI_F1(Acos)
DRESSI_F1(Atan) DRESSI_F2(Atan2) DRESSI_F1(Exp) DRESSI_F1(Exp2) DRESSI_F1(Log)
DRESSI_F1(Log2) DRESSI_F1(Sqrt) DRESSI_F1(InverseSqrt) DRESSI_F1(Abs)
DRESSI_F1(Sign) DRESSI_F1(Floor) DRESSI_F1(Fract) DRESSI_F2(Mod) DRESSI_F2(Pow)
DRESSI_F2(Max) DRESSI_F2(Min) DRESSI_F3(Clamp) DRESSI_F3(Mix) DRESSI_F2(Step)
DRESSI_F3(SmoothStep) DRESSI_F1(Sigmoid) DRESSI_F2(Less) DRESSI_F2(LessEqual)
DRESSI_F2(Greater) DRESSI_F2(GreaterEqual)
// vectors and matrices
inline Variable Vec2(const Variable& x, const Variable& y) {
    return detail::op("Vec2", {x, y});
}
inline Variable Vec3(const Variable& x, const Variable& y, const Variable& z) {
    return detail::op("Vec3", {x, y, z});
}
inline Variable Vec3(const Variable& xy, const Variable& z) {
    return detail::op("Vec3", {xy, z});
}
inline Variable Vec4(const Variable& x, const Variable& y, const Variable& z,
                     const Variable& w) {
    return detail::op("Vec4", {x, y, z, w});
}
inline Variable Vec4(const Variable& xyz, const Variable& w) {
    return detail::op("Vec4", {xyz, w});
}
DRESSI_F1(GetX) DRESSI_F1(GetY) DRESSI_F1(GetZ) DRESSI_F1(GetW)
DRESSI_F2(Dot) DRESSI_F2(Cross) DRESSI_F1(Length) DRESSI_F2(Distance)
DRESSI_F1(Normalize) DRESSI_F2(Reflect) DRESSI_F1(CompSum) DRESSI_F2(MatMul)
DRESSI_F1(Transpose) DRESSI_F2(OuterProduct)
// reductions, broadcast
inline Variable Broadcast(const Variable& x, ImgSize size) {
    return detail::op("Broadcast", {x}, {}, detail::sz(size));
}
inline Variable SumPixelWise(const Variables& xs) {
    return detail::op("SumPixelWise", xs);
}
DRESSI_F1(Sum) DRESSI_F1(Mean) DRESSI_F1(SumAll) DRESSI_F1(StopGradient)
DRESSI_F1(SetFragDepth)
// rendering
inline Variable Rasterize(const Variable& clip, const Variable& attr,
                          const Variable& faces, ImgSize screen) {
    return detail::op("Rasterize", {clip, attr, faces}, {}, detail::sz(screen));
}
inline Variable RasterizeSoft(const Variable& clip_soft, const Variable& face_id,
                              const Variable& faces_soft,
                              const Variable& clip_hard,
                              const Variable& faces_tex,
                              const Variable& vtx_faces_tex, ImgSize screen,
                              float radius_px) {
    return detail::op("RasterizeSoft",
                      {clip_soft, face_id, faces_soft, clip_hard, faces_tex,
                       vtx_faces_tex},
                      {radius_px}, detail::sz(screen));
}
inline Variable RasterizeSoft(const Variable& clip_soft, const Variable& face_id,
                              const Variable& faces_soft,
                              const Variable& clip_hard,
                              const Variable& faces_tex,
                              const Variable& vtx_faces_tex,
                              const Variable& prev_shifted_depth,
                              ImgSize screen, float radius_px) {
    return detail::op("RasterizeSoft",
                      {clip_soft, face_id, faces_soft, clip_hard, faces_tex,
                       vtx_faces_tex, prev_shifted_depth},
                      {radius_px}, detail::sz(screen));
}
inline Variable RasterizeFaceId(const Variable& clip, const Variable& dummy,
                                const Variable& faces, ImgSize screen) {
    return detail::op("RasterizeFaceId", {clip, dummy, faces}, {},
                      detail::sz(screen));
}
inline Variable AntiAlias(const Variable& img, const Variable& tri_id,
                          const Variable& vtx_clip, const Variable& faces,
                          const Variable& vtx_faces_tex, const Variable& seed,
                          uint32_t n_samples = 8) {
    return detail::op("AntiAlias",
                      {img, tri_id, vtx_clip, faces, vtx_faces_tex, seed}, {},
                      {int64_t(n_samples)});
}
inline Variable ScreenCoord(ImgSize size) {
    return detail::op("ScreenCoord", {}, {}, detail::sz(size));
}
inline Variable LookupFaces(const Variable& attr, const Variable& faces_tex,
                            const Variable& vtx_faces_tex, uint32_t corner) {
    return detail::op("LookupFaces", {attr, faces_tex, vtx_faces_tex}, {},
                      {int64_t(corner)});
}
inline Variable FaceFetch(const Variable& tri_attr, const Variable& idx_img,
                          const Variable& p0, const Variable& p1,
                          const Variable& p2, const Variable& seed,
                          float radius_px, uint32_t n_samples = 4) {
    return detail::op("FaceFetch", {tri_attr, idx_img, p0, p1, p2, seed},
                      {radius_px}, {int64_t(n_samples)});
}
inline Variable PixelFetch(const Variable& tex, uint32_t x_index,
                           const Variable& row_idx) {
    return detail::op("PixelFetch", {tex, row_idx}, {}, {int64_t(x_index)});
}
inline Variable TileFetch(const Variable& atlas, const Variable& tile_idx,
                          uint32_t tile_h) {
    return detail::op("TileFetch", {atlas, tile_idx}, {}, {int64_t(tile_h)});
}
inline Variable SoftClip(const Variable& clip_hard, const Variable& faces_tex,
                         ImgSize screen, float radius_px) {
    return detail::op("SoftClip", {clip_hard, faces_tex}, {radius_px},
                      detail::sz(screen));
}
DRESSI_F2(VertexNeighborMean) DRESSI_F3(NormalConsistencyFaceTerm)
inline Variable NormalConsistencyVertexGrad(const Variable& term,
                                            const Variable& pos,
                                            const Variable& faces,
                                            const Variable& vft) {
    return detail::op("NormalConsistencyVertexGrad", {term, pos, faces, vft});
}
DRESSI_F3(Texture) DRESSI_F3(TextureBilinear)
// split-sum IBL
DRESSI_F2(EquirectSample)
inline Variable IrradianceConv(const Variable& env, ImgSize out) {
    return detail::op("IrradianceConv", {env}, {}, detail::sz(out));
}
inline Variable PrefilterConv(const Variable& env, ImgSize out,
                              float roughness) {
    return detail::op("PrefilterConv", {env}, {roughness}, detail::sz(out));
}
inline Variable BrdfIntegrationLut(ImgSize size, uint32_t n_samples = 512) {
    return detail::op("BrdfIntegrationLut", {}, {},
                      {size.w, size.h, int64_t(n_samples)});
}
DRESSI_F1(AvgPool2x2)
#undef DRESSI_F1
#undef DRESSI_F2
#undef DRESSI_F3
}  // namespace F

// operator overloads (the reference's include/dressi/f.h:321-339)
inline Variable operator+(const Variable& a, const Variable& b) { return F::Add(a, b); }
inline Variable operator-(const Variable& a, const Variable& b) { return F::Sub(a, b); }
inline Variable operator*(const Variable& a, const Variable& b) { return F::Mul(a, b); }
inline Variable operator/(const Variable& a, const Variable& b) { return F::Div(a, b); }
inline Variable operator+(const Variable& a, float b) { return F::Add(a, F::Float(b)); }
inline Variable operator-(const Variable& a, float b) { return F::Sub(a, F::Float(b)); }
inline Variable operator*(const Variable& a, float b) { return F::Mul(a, F::Float(b)); }
inline Variable operator/(const Variable& a, float b) { return F::Div(a, F::Float(b)); }
inline Variable operator+(float a, const Variable& b) { return F::Add(F::Float(a), b); }
inline Variable operator-(float a, const Variable& b) { return F::Sub(F::Float(a), b); }
inline Variable operator*(float a, const Variable& b) { return F::Mul(F::Float(a), b); }
inline Variable operator/(float a, const Variable& b) { return F::Div(F::Float(a), b); }
inline Variable operator-(const Variable& x) { return F::Neg(x); }
inline Variable operator<(const Variable& a, const Variable& b) { return F::Less(a, b); }
inline Variable operator<(float a, const Variable& b) { return F::Less(F::Float(a), b); }
inline Variable operator<(const Variable& a, float b) { return F::Less(a, F::Float(b)); }
inline Variable operator<=(const Variable& a, const Variable& b) { return F::LessEqual(a, b); }
inline Variable operator>(const Variable& a, const Variable& b) { return F::Greater(a, b); }
inline Variable operator>=(const Variable& a, const Variable& b) { return F::GreaterEqual(a, b); }

// DR-specialised AD driver (the reference's DressiAD) on one CUDA device.
class DressiAD {
public:
    using Optimizer = std::function<Variables(Variables xs, Variables gxs)>;
    enum class PackingMode { Naive, RSP };

    explicit DressiAD(int device = 0) {
        detail::check(dressi_ad_create(device, &h_));
    }
    ~DressiAD() {
        if (h_) dressi_ad_destroy(h_);
    }
    DressiAD(const DressiAD&) = delete;
    DressiAD& operator=(const DressiAD&) = delete;

    void setLossVar(const Variable& loss) {
        detail::check(dressi_ad_set_loss(h_, loss.handle()));
    }
    void setOptimizer(const Optimizer& fn) {
        optim_ = fn;
        detail::check(dressi_ad_set_optimizer(h_, &DressiAD::trampoline, this));
    }
    void setPackingMode(PackingMode mode) {
        detail::check(dressi_ad_set_max_fusion(
                h_, mode == PackingMode::Naive ? 1u : 512u));
    }
    void setRebuildCounts(uint32_t fast, uint32_t full) {
        detail::check(dressi_ad_set_rebuild_counts(h_, fast, full));
    }
    void markOutput(const Variable& v) {
        detail::check(dressi_ad_mark_output(h_, v.handle()));
    }
    void addUpdate(const Variable& input_leaf, const Variable& updated) {
        detail::check(dressi_ad_add_update(h_, input_leaf.handle(),
                                           updated.handle()));
    }
    void setGradOutputsEnabled(bool enable) {
        detail::check(dressi_ad_set_grad_outputs(h_, enable ? 1 : 0));
    }
    std::vector<std::pair<Variable, Variable>> inputGrads() const {
        uint32_t n = 0;
        detail::check(dressi_ad_input_grads(h_, nullptr, nullptr, 0, &n));
        std::vector<dressi_var> xs(n), gs(n);
        detail::check(dressi_ad_input_grads(h_, xs.data(), gs.data(), n, &n));
        std::vector<std::pair<Variable, Variable>> out;
        for (uint32_t i = 0; i < n; i++)
            out.emplace_back(Variable::adopt(xs[i]), Variable::adopt(gs[i]));
        return out;
    }
    size_t getFuncCount() const { return stats().n_funcs; }
    size_t getStageCount() const { return stats().n_steps; }
    size_t getSubStageCount() const { return stats().n_steps; }
    dressi_ad_stats_t stats() const {
        dressi_ad_stats_t s;
        detail::check(dressi_ad_stats(h_, &s));
        return s;
    }

    // Replays the iteration on `stream` (a cudaStream_t; null = the legacy
    // default stream). Asynchronous: recvImg synchronises.
    void execStep(void* stream = nullptr) {
        const int rc = dressi_ad_exec_step(h_, stream);
        if (pending_) {
            std::exception_ptr e = pending_;
            pending_ = nullptr;
            std::rethrow_exception(e);
        }
        detail::check(rc);
    }
    void execStepWithSends(
            const std::vector<std::pair<Variable, CpuImageView>>& items) {
        sendImgs(items);
        execStep();
    }
    void sendImg(const Variable& v, const CpuImageView& img) {
        detail::check(dressi_ad_send(h_, v.handle(), img.data,
                                     img.numElems(), 0, nullptr));
    }
    void sendImg(const Variable& v, const CpuImage& img) {
        sendImg(v, CpuImageView(img));
    }
    void sendImgs(const std::vector<std::pair<Variable, CpuImageView>>& items) {
        for (const auto& [v, img] : items) sendImg(v, img);
    }
    CpuImage recvImg(const Variable& v) {
        const ImgSize s = v.getImgSize();
        CpuImage img(s.w, s.h, NumComponents(v.getVType()));
        detail::check(dressi_ad_recv(h_, v.handle(), img.data.data(),
                                     img.data.size(), 0, nullptr));
        return img;
    }
    std::vector<CpuImage> recvImgs(const Variables& vs) {
        std::vector<CpuImage> out;
        for (const auto& v : vs) out.push_back(recvImg(v));
        return out;
    }
    uint32_t status(bool clear = true) {
        uint32_t w = 0;
        detail::check(dressi_ad_status(h_, &w, clear ? 1 : 0));
        return w;
    }

private:
    static int trampoline(void* user, const dressi_var* xs,
                          const dressi_var* gxs, uint32_t n, dressi_var* out) {
        auto* self = static_cast<DressiAD*>(user);
        try {
            Variables vx, vg;
            for (uint32_t i = 0; i < n; i++) {
                dressi_var a = nullptr, b = nullptr;
                detail::check(dressi_var_clone(xs[i], &a));
                detail::check(dressi_var_clone(gxs[i], &b));
                vx.push_back(Variable::adopt(a));
                vg.push_back(Variable::adopt(b));
            }
            Variables res = self->optim_(vx, vg);
            if (res.size() != n)
                throw DressiError("Optimizer must return one output per input");
            for (uint32_t i = 0; i < n; i++)
                detail::check(dressi_var_clone(res[i].handle(), &out[i]));
            return 0;
        } catch (...) {
            self->pending_ = std::current_exception();
            return 1;
        }
    }

    dressi_ad h_ = nullptr;
    Optimizer optim_;
    std::exception_ptr pending_;
};

}  // namespace dressi

#endif  // DRESSI_B200_DRESSI_H
