// Lowering and execution of a graph (the generic path behind DressiAD).
//
// The fusion planner groups pixel-wise ops that share an output grid into
// one "pixel program" -- a scalar register program run by the templated
// interpreter kernel k_pixel_prog, one thread per pixel -- so chains of
// elementwise math, their autodiff and the optimizer's update run as few
// kernels; values consumed only inside a program never reach HBM.
// Reductions (Sum: the reference's 2x2 quad tree, walked in the same order
// so the float sums are identical; SumAll) and the rendering / texture /
// IBL ops run as their own kernels (the op-level kernels of this library).
// The resulting step list is captured once into a CUDA graph and replayed
// per iteration.
//
// Legality of fusing f into a program G (the planner's rules; the
// reference's counterpart is src/pack/greedy_packer.cpp:34-141):
//  - f is pixel-wise and its output has G's grid;
//  - every input of f is a constant, produced inside G (a same-pixel read),
//    or produced by a step that runs before G (a buffer read: same pixel,
//    or the single texel of a {1,1} value);
//  - so a value produced by a reduction or a special kernel is never
//    consumed inside the program that feeds it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <unordered_map>
#include <unordered_set>

#include "exact.cuh"
#include "graph.h"
#include "graph_exec.h"
#include "kernels.h"

namespace dressi {
namespace graph {

// ================================================================ device

namespace {

constexpr int kProgThreads = 128;

__device__ __forceinline__ float sign_f(float v) {
    return float(int(v > 0.f) - int(v < 0.f));
}

// One thread per pixel of the program's grid; the program (code and buffer
// table) and the scalar registers ([reg][thread]) live in shared memory.
__global__ void __launch_bounds__(kProgThreads)
        k_pixel_prog(const Ins* code, int n_ins, const BufRef* bufs,
                     int n_bufs, int n_regs, long long npx, int width) {
    extern __shared__ float4 sm4[];
    Ins* cs = reinterpret_cast<Ins*>(sm4);
    BufRef* bs = reinterpret_cast<BufRef*>(cs + n_ins);
    float* R = reinterpret_cast<float*>(bs + n_bufs);
    {
        const uint4* src = reinterpret_cast<const uint4*>(code);
        uint4* dst = reinterpret_cast<uint4*>(cs);
        for (int i = threadIdx.x; i < n_ins; i += blockDim.x) dst[i] = src[i];
        for (int i = threadIdx.x; i < n_bufs; i += blockDim.x) bs[i] = bufs[i];
    }
    __syncthreads();
    const int B = blockDim.x, t = threadIdx.x;
#define RG(r) R[int(r) * B + t]
    for (long long p = blockIdx.x * (long long)B + t; p < npx;
         p += (long long)gridDim.x * B) {
        for (int i = 0; i < n_ins; i++) {
            const Ins in = cs[i];
            float v;
            switch (in.op) {
            case P_LOAD: {
                const BufRef b = bs[in.buf];
                const long long q = b.uniform ? 0 : p;
                v = b.ptr[q * b.stride + in.imm];
                break;
            }
            case P_STORE: {
                const BufRef b = bs[in.buf];
                b.ptr[p * b.stride + in.imm] = RG(in.a);
                continue;
            }
            case P_CONST: v = __uint_as_float(in.imm); break;
            case P_SCRX: v = float(int(p % width)) + 0.5f; break;
            case P_SCRY: v = float(int(p / width)) + 0.5f; break;
            case P_ADD: v = RG(in.a) + RG(in.b); break;
            case P_SUB: v = RG(in.a) - RG(in.b); break;
            case P_MUL: v = RG(in.a) * RG(in.b); break;
            case P_DIV: v = RG(in.a) / RG(in.b); break;
            case P_NEG: v = -RG(in.a); break;
            case P_SIN: v = sinf(RG(in.a)); break;
            case P_COS: v = cosf(RG(in.a)); break;
            case P_TAN: v = tanf(RG(in.a)); break;
            case P_ASIN: v = asinf(RG(in.a)); break;
            case P_ACOS: v = acosf(RG(in.a)); break;
            case P_ATAN: v = atanf(RG(in.a)); break;
            case P_ATAN2: v = atan2f(RG(in.a), RG(in.b)); break;
            case P_EXP: v = expf(RG(in.a)); break;
            case P_EXP2: v = exp2f(RG(in.a)); break;
            case P_LOG: v = logf(RG(in.a)); break;
            case P_LOG2: v = log2f(RG(in.a)); break;
            case P_SQRT: v = sqrtf(RG(in.a)); break;
            case P_RSQRT: v = 1.f / sqrtf(RG(in.a)); break;
            case P_ABS: v = fabsf(RG(in.a)); break;
            case P_SIGN: v = sign_f(RG(in.a)); break;
            case P_FLOOR: v = floorf(RG(in.a)); break;
            case P_FRACT: {
                const float a = RG(in.a);
                v = a - floorf(a);
                break;
            }
            case P_MOD: {
                const float a = RG(in.a), b = RG(in.b);
                v = a - b * floorf(a / b);
                break;
            }
            case P_POW: v = powf(RG(in.a), RG(in.b)); break;
            case P_MAX: v = std_max(RG(in.a), RG(in.b)); break;
            case P_MIN: v = std_min(RG(in.a), RG(in.b)); break;
            case P_CLAMP:
                v = std_min(std_max(RG(in.a), RG(in.b)), RG(in.c));
                break;
            case P_MIX: {
                const float a = RG(in.a), b = RG(in.b), tt = RG(in.c);
                v = a + (b - a) * tt;
                break;
            }
            case P_STEP: v = RG(in.b) < RG(in.a) ? 0.f : 1.f; break;
            case P_SMOOTH: {
                const float a = RG(in.a), b = RG(in.b), x = RG(in.c);
                const float tt = std_min(std_max((x - a) / (b - a), 0.f), 1.f);
                v = tt * tt * (3.f - 2.f * tt);
                break;
            }
            case P_SIGMOID: v = 1.f / (1.f + expf(-RG(in.a))); break;
            case P_LT: v = float(RG(in.a) < RG(in.b)); break;
            case P_LE: v = float(RG(in.a) <= RG(in.b)); break;
            case P_GT: v = float(RG(in.a) > RG(in.b)); break;
            case P_GE: v = float(RG(in.a) >= RG(in.b)); break;
            default: v = 0.f; break;
            }
            RG(in.dst) = v;
        }
    }
#undef RG
}

__host__ __device__ __forceinline__ int ceil_shift(int n, int l) {
    return (n + (1 << l) - 1) >> l;
}

// L levels of the 2x2 sum tree (the reference's Reduce2x2Sum chain,
// src/core/f_ops.cpp:982-1032) over one SX x SY tile: every node starts at
// 0 and adds its existing children in row-major source order, as the
// reference's loop over source pixels does; absent children (past an odd
// extent) add nothing. in [h][w][nc] -> out [ceil(h/2^L)][ceil(w/2^L)][nc].
template <int SX, int SY, int L>
__global__ void __launch_bounds__(SX * SY)
        k_quad_sum(const float* in, int w, int h, int nc, float* out) {
    __shared__ float buf[2][SX * SY];
    const int lx = threadIdx.x % SX, ly = threadIdx.x / SX;
    const int bx = blockIdx.x, by = blockIdx.y;
    const int ow = ceil_shift(w, L);
    for (int c = 0; c < nc; c++) {
        {
            const int x = bx * SX + lx, y = by * SY + ly;
            buf[0][threadIdx.x] = (x < w && y < h)
                                          ? in[(size_t(y) * w + x) * nc + c]
                                          : 0.f;
        }
        __syncthreads();
        int cur = 0;
#pragma unroll
        for (int l = 1; l <= L; l++) {
            const int sx = SX >> l > 0 ? SX >> l : 1;
            const int sy = SY >> l > 0 ? SY >> l : 1;
            const int psx = SX >> (l - 1) > 0 ? SX >> (l - 1) : 1;
            if (lx < sx && ly < sy) {
                // level-(l-1) extents of the whole image
                const int pw = ceil_shift(w, l - 1), ph = ceil_shift(h, l - 1);
                const int gx0 = (bx * SX >> (l - 1)) + 2 * lx;
                const int gy0 = (by * SY >> (l - 1)) + 2 * ly;
                float acc = 0.f;
#pragma unroll
                for (int dy = 0; dy < 2; dy++) {
#pragma unroll
                    for (int dx = 0; dx < 2; dx++) {
                        const int cx = 2 * lx + dx, cy = 2 * ly + dy;
                        const bool in_tile =
                                cx < psx && cy < (SY >> (l - 1) > 0
                                                          ? SY >> (l - 1)
                                                          : 1);
                        if (in_tile && gx0 + dx < pw && gy0 + dy < ph)
                            acc += buf[cur][cy * psx + cx];
                    }
                }
                buf[cur ^ 1][ly * sx + lx] = acc;
            }
            cur ^= 1;
            __syncthreads();
        }
        if (threadIdx.x == 0) out[(size_t(by) * ow + bx) * nc + c] = buf[cur][0];
        __syncthreads();
    }
}

__global__ void k_extract_channel(const float* in, int stride, int ch,
                                  long long n, float* out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
         i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = in[i * stride + ch];
}

// PixelFetch (f_ops.cpp:1803-1832): out = tex(x, round(row)).
__global__ void k_pixel_fetch(const float* tex, int w, int h, int n, int x,
                              const float* row, float* out,
                              uint32_t* status) {
    const uint32_t r = x86_u32_via_i64(row[0] + 0.5f);
    const bool ok = r < uint32_t(h);
    if (!ok && threadIdx.x == 0) atomicOr(status, kStatusIndexRange);
    for (int c = threadIdx.x; c < n; c += blockDim.x)
        out[c] = ok ? tex[(size_t(r) * w + x) * n + c] : 0.f;
}

// TileFetch (f_ops.cpp:1834-1866): rows [idx tile_h, (idx + 1) tile_h).
__global__ void k_tile_fetch(const float* atlas, int w, int h, int n,
                             int tile_h, const float* idx, float* out,
                             uint32_t* status) {
    const uint32_t t = x86_u32_via_i64(idx[0] + 0.5f);
    const bool ok = (long long)(t + 1) * tile_h <= h;
    if (!ok && blockIdx.x == 0 && threadIdx.x == 0)
        atomicOr(status, kStatusIndexRange);
    const long long cnt = (long long)w * tile_h * n;
    const size_t o = size_t(t) * tile_h * w * n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
         i < cnt; i += (long long)gridDim.x * blockDim.x)
        out[i] = ok ? atlas[o + i] : 0.f;
}

void check_launch() { DRESSI_CUDA(cudaGetLastError()); }

unsigned grid_for(long long n, int threads, int cap) {
    const long long b = (n + threads - 1) / threads;
    return unsigned(std::max<long long>(1, std::min<long long>(b, cap)));
}

}  // namespace

// ================================================================ planner

namespace {

bool is_const_var(const Var& v) { return v->is_const; }

PO unary_po(Op op) {
    switch (op) {
    case Op::Neg: return P_NEG;
    case Op::Sin: return P_SIN;
    case Op::Cos: return P_COS;
    case Op::Tan: return P_TAN;
    case Op::Asin: return P_ASIN;
    case Op::Acos: return P_ACOS;
    case Op::Atan: return P_ATAN;
    case Op::Exp: return P_EXP;
    case Op::Exp2: return P_EXP2;
    case Op::Log: return P_LOG;
    case Op::Log2: return P_LOG2;
    case Op::Sqrt: return P_SQRT;
    case Op::InverseSqrt: return P_RSQRT;
    case Op::Abs: return P_ABS;
    case Op::Sign: return P_SIGN;
    case Op::Floor: return P_FLOOR;
    case Op::Fract: return P_FRACT;
    case Op::Sigmoid: return P_SIGMOID;
    default: return P_NOP;
    }
}

PO binary_po(Op op) {
    switch (op) {
    case Op::Add: return P_ADD;
    case Op::Sub: return P_SUB;
    case Op::Mul: return P_MUL;
    case Op::Div: return P_DIV;
    case Op::Atan2: return P_ATAN2;
    case Op::Mod: return P_MOD;
    case Op::Pow: return P_POW;
    case Op::Max: return P_MAX;
    case Op::Min: return P_MIN;
    case Op::Step: return P_STEP;
    case Op::Less: return P_LT;
    case Op::LessEqual: return P_LE;
    case Op::Greater: return P_GT;
    case Op::GreaterEqual: return P_GE;
    default: return P_NOP;
    }
}

// Scalar SSA instruction before register allocation.
struct SIns {
    PO op;
    int dst = -1, a = -1, b = -1, c = -1;
    int buf = 0;
    uint32_t imm = 0;
};

// Compiles one fused group into a register program.
class ProgramBuilder {
public:
    ProgramBuilder(const Step& st, const std::unordered_set<uint64_t>& mat,
                   std::vector<uint64_t>* buf_vars)
        : st_(st), mat_(mat), bufv_(buf_vars) {}

    void build(std::vector<Ins>* code, int* n_regs) {
        for (const Func& f : st_.funcs) emit(f);
        for (const Func& f : st_.funcs) {
            Var y = f->out();
            if (!mat_.count(y->id)) continue;
            const auto& v = vals_.at(y->id);
            const int slot = buf_slot(y);
            for (uint32_t c = 0; c < v.size(); c++) {
                SIns s;
                s.op = P_STORE;
                s.a = v[c];
                s.buf = slot;
                s.imm = c;
                ins_.push_back(s);
            }
        }
        allocate(code, n_regs);
    }

private:
    const Step& st_;
    const std::unordered_set<uint64_t>& mat_;
    std::vector<uint64_t>* bufv_;
    std::vector<SIns> ins_;
    int n_vals_ = 0;
    std::unordered_map<uint64_t, std::vector<int>> vals_;
    std::unordered_map<uint32_t, int> consts_;
    std::unordered_map<uint64_t, int> slots_;

    int def(SIns s) {
        s.dst = n_vals_++;
        ins_.push_back(s);
        return s.dst;
    }
    int op1(PO op, int a) { SIns s; s.op = op; s.a = a; return def(s); }
    int op2(PO op, int a, int b) {
        SIns s;
        s.op = op;
        s.a = a;
        s.b = b;
        return def(s);
    }
    int op3(PO op, int a, int b, int c) {
        SIns s;
        s.op = op;
        s.a = a;
        s.b = b;
        s.c = c;
        return def(s);
    }
    int konst(float f) {
        uint32_t bits;
        std::memcpy(&bits, &f, 4);
        auto it = consts_.find(bits);
        if (it != consts_.end()) return it->second;
        SIns s;
        s.op = P_CONST;
        s.imm = bits;
        const int v = def(s);
        consts_[bits] = v;
        return v;
    }
    int buf_slot(const Var& x) {
        auto it = slots_.find(x->id);
        if (it != slots_.end()) return it->second;
        const int slot = int(bufv_->size());
        bufv_->push_back(x->id);
        slots_[x->id] = slot;
        return slot;
    }

    const std::vector<int>& in(const Var& x) {
        auto it = vals_.find(x->id);
        if (it != vals_.end()) return it->second;
        std::vector<int> v;
        if (x->is_const) {
            for (float f : x->cval) v.push_back(konst(f));
        } else {
            const int slot = buf_slot(x);
            for (uint32_t c = 0; c < ncomp(x->vtype); c++) {
                SIns s;
                s.op = P_LOAD;
                s.buf = slot;
                s.imm = c;
                v.push_back(def(s));
            }
        }
        return vals_[x->id] = v;
    }

    // component c of x, a scalar broadcasting over components
    int comp(const Var& x, uint32_t c) {
        const auto& v = in(x);
        return v[v.size() == 1 ? 0 : c];
    }

    void emit(const Func& f) {
        Var y = f->out();
        const uint32_t ny = ncomp(y->vtype);
        std::vector<int> out;
        const Vars& xs = f->xs;
        switch (f->op) {
        case Op::Compose:
            for (const auto& p : xs)
                for (int v : in(p)) out.push_back(v);
            break;
        case Op::Extract: {
            const auto& v = in(xs[0]);
            for (int64_t c = 0; c < f->ip[1]; c++)
                out.push_back(v[size_t(f->ip[0] + c)]);
            break;
        }
        case Op::StopGradient: case Op::SetFragDepth: case Op::Broadcast:
            out = in(xs[0]);
            break;
        case Op::ScreenCoord: {
            SIns s;
            s.op = P_SCRX;
            out.push_back(def(s));
            s.op = P_SCRY;
            out.push_back(def(s));
            break;
        }
        case Op::Dot: {
            int acc = konst(0.f);
            for (uint32_t c = 0; c < ncomp(xs[0]->vtype); c++)
                acc = op2(P_ADD, acc,
                          op2(P_MUL, in(xs[0])[c], in(xs[1])[c]));
            out.push_back(acc);
            break;
        }
        case Op::Length: case Op::Normalize: {
            const auto& x = in(xs[0]);
            int acc = konst(0.f);
            for (int v : x) acc = op2(P_ADD, acc, op2(P_MUL, v, v));
            const int len = op1(P_SQRT, acc);
            if (f->op == Op::Length) {
                out.push_back(len);
            } else {
                const int inv = op2(P_DIV, konst(1.f), len);
                for (int v : x) out.push_back(op2(P_MUL, v, inv));
            }
            break;
        }
        case Op::CompSum: {
            int acc = konst(0.f);
            for (int v : in(xs[0])) acc = op2(P_ADD, acc, v);
            out.push_back(acc);
            break;
        }
        case Op::Cross: {
            const auto& a = in(xs[0]);
            const auto& b = in(xs[1]);
            auto cr = [&](int i, int j) {
                return op2(P_SUB, op2(P_MUL, a[i], b[j]),
                           op2(P_MUL, a[j], b[i]));
            };
            out = {cr(1, 2), cr(2, 0), cr(0, 1)};
            break;
        }
        case Op::MatMul: {
            const uint32_t dim = mat_dim(xs[0]->vtype);
            const auto& m = in(xs[0]);
            const auto& r = in(xs[1]);
            if (is_vec(xs[1]->vtype)) {
                for (uint32_t row = 0; row < dim; row++) {
                    int acc = konst(0.f);
                    for (uint32_t col = 0; col < dim; col++)
                        acc = op2(P_ADD, acc,
                                  op2(P_MUL, m[col * dim + row], r[col]));
                    out.push_back(acc);
                }
            } else {
                out.assign(dim * dim, -1);
                for (uint32_t col = 0; col < dim; col++)
                    for (uint32_t row = 0; row < dim; row++) {
                        int acc = konst(0.f);
                        for (uint32_t k = 0; k < dim; k++)
                            acc = op2(P_ADD, acc,
                                      op2(P_MUL, m[k * dim + row],
                                          r[col * dim + k]));
                        out[col * dim + row] = acc;
                    }
            }
            break;
        }
        case Op::Transpose: {
            const uint32_t dim = mat_dim(xs[0]->vtype);
            const auto& m = in(xs[0]);
            out.assign(dim * dim, -1);
            for (uint32_t col = 0; col < dim; col++)
                for (uint32_t row = 0; row < dim; row++)
                    out[col * dim + row] = m[row * dim + col];
            break;
        }
        case Op::OuterProduct: {
            const uint32_t dim = ncomp(xs[0]->vtype);
            const auto& a = in(xs[0]);
            const auto& b = in(xs[1]);
            out.assign(dim * dim, -1);
            for (uint32_t c = 0; c < dim; c++)
                for (uint32_t r = 0; r < dim; r++)
                    out[c * dim + r] = op2(P_MUL, a[r], b[c]);
            break;
        }
        case Op::SumPixelWise:
            for (uint32_t c = 0; c < ny; c++) {
                int acc = konst(0.f);
                for (const auto& x : xs) acc = op2(P_ADD, acc, comp(x, c));
                out.push_back(acc);
            }
            break;
        case Op::Clamp: case Op::Mix: case Op::SmoothStep: {
            const PO po = f->op == Op::Clamp ? P_CLAMP
                          : f->op == Op::Mix ? P_MIX
                                             : P_SMOOTH;
            for (uint32_t c = 0; c < ny; c++)
                out.push_back(op3(po, comp(xs[0], c), comp(xs[1], c),
                                  comp(xs[2], c)));
            break;
        }
        default: {
            const PO u = unary_po(f->op);
            const PO b = binary_po(f->op);
            if (u != P_NOP) {
                for (uint32_t c = 0; c < ny; c++)
                    out.push_back(op1(u, comp(xs[0], c)));
            } else if (b != P_NOP) {
                for (uint32_t c = 0; c < ny; c++)
                    out.push_back(op2(b, comp(xs[0], c), comp(xs[1], c)));
            } else {
                throw_error(kErrInvalid,
                            std::string("pixel program: unsupported op ") +
                                    op_name(f->op),
                            __FILE__, __LINE__);
            }
        }
        }
        DRESSI_REQUIRE(out.size() == ny, std::string("pixel program: ") +
                                                 op_name(f->op) +
                                                 " component count");
        vals_[y->id] = out;
    }

    // Linear-scan register allocation of the SSA values: a register is
    // free again after its value's last reader.
    void allocate(std::vector<Ins>* code, int* n_regs) {
        std::vector<int> last(size_t(n_vals_), -1);
        for (int i = 0; i < int(ins_.size()); i++) {
            const SIns& s = ins_[size_t(i)];
            for (int r : {s.a, s.b, s.c})
                if (r >= 0) last[size_t(r)] = i;
        }
        std::vector<int> phys(size_t(n_vals_), -1);
        std::vector<int> free_regs;
        int top = 0;
        code->clear();
        for (int i = 0; i < int(ins_.size()); i++) {
            const SIns& s = ins_[size_t(i)];
            Ins o{};
            o.op = uint16_t(s.op);
            o.buf = uint16_t(s.buf);
            o.imm = s.imm;
            o.a = uint16_t(s.a >= 0 ? phys[size_t(s.a)] : 0);
            o.b = uint16_t(s.b >= 0 ? phys[size_t(s.b)] : 0);
            o.c = uint16_t(s.c >= 0 ? phys[size_t(s.c)] : 0);
            // operands whose last reader is this instruction free their
            // registers before the result is assigned (read-before-write)
            for (int r : {s.a, s.b, s.c}) {
                if (r >= 0 && last[size_t(r)] == i && phys[size_t(r)] >= 0) {
                    free_regs.push_back(phys[size_t(r)]);
                    phys[size_t(r)] = -1;
                }
            }
            if (s.dst >= 0) {
                int reg;
                if (!free_regs.empty()) {
                    reg = free_regs.back();
                    free_regs.pop_back();
                } else {
                    reg = top++;
                }
                o.dst = uint16_t(reg);
                if (last[size_t(s.dst)] > i)
                    phys[size_t(s.dst)] = reg;
                else
                    free_regs.push_back(reg);  // dead value
            }
            code->push_back(o);
        }
        *n_regs = std::max(top, 1);
    }
};

}  // namespace

void Plan::build(const std::vector<Func>& exec_funcs, const Vars& roots,
                 size_t max_group) {
    steps.clear();
    std::unordered_map<uint64_t, int> producer;  // var id -> step
    std::unordered_set<uint64_t> lowered;        // SumPartial folded into SumAll
    for (const Func& f : exec_funcs) {
        if (f->op == Op::Const) continue;
        Var y = f->out();
        if (f->op == Op::SumPartial) {
            lowered.insert(y->id);
            producer[y->id] = producer.count(f->xs[0]->id)
                                      ? producer[f->xs[0]->id]
                                      : -1;
            continue;
        }
        if (is_pixelwise(f->op)) {
            int join = -1;
            for (int g = int(steps.size()) - 1; g >= 0; g--) {
                Step& st = steps[size_t(g)];
                if (st.kind != Step::kProgram || st.grid != y->size ||
                    st.funcs.size() >= max_group)
                    continue;
                bool ok = true;
                for (const auto& x : f->xs) {
                    if (x->is_const) continue;
                    auto it = producer.find(x->id);
                    if (it == producer.end() || it->second < 0) continue;
                    if (it->second == g) {
                        // same-pixel read inside the program
                        if (x->size != st.grid) ok = false;
                    } else if (it->second > g) {
                        ok = false;
                    }
                    if (!ok) break;
                }
                if (ok) {
                    join = g;
                    break;
                }
            }
            if (join < 0) {
                Step st;
                st.kind = Step::kProgram;
                st.grid = y->size;
                steps.push_back(st);
                join = int(steps.size()) - 1;
            }
            steps[size_t(join)].funcs.push_back(f);
            producer[y->id] = join;
            continue;
        }
        Step st;
        st.kind = (f->op == Op::Sum) ? Step::kSum
                  : (f->op == Op::SumAll) ? Step::kSumAll
                                          : Step::kSpecial;
        st.grid = y->size;
        st.funcs.push_back(f);
        steps.push_back(st);
        producer[y->id] = int(steps.size()) - 1;
    }
    // materialised values: roots, and values read by another step
    materialized.clear();
    for (const auto& r : roots)
        if (r && !r->is_const) materialized.insert(r->id);
    for (int g = 0; g < int(steps.size()); g++) {
        for (const Func& f : steps[size_t(g)].funcs) {
            for (const auto& x0 : f->xs) {
                Var x = x0;
                // SumAll reads the input of its folded SumPartial
                if (steps[size_t(g)].kind == Step::kSumAll &&
                    lowered.count(x->id))
                    x = x->creator->xs[0];
                auto it = producer.find(x->id);
                const bool inside = it != producer.end() && it->second == g &&
                                    steps[size_t(g)].kind == Step::kProgram;
                if (!inside && !(x->is_const &&
                                 steps[size_t(g)].kind == Step::kProgram))
                    materialized.insert(x->id);
            }
        }
    }
    for (const auto& id : lowered) materialized.erase(id);
    // compile the programs
    for (auto& st : steps) {
        if (st.kind != Step::kProgram) continue;
        st.buf_vars.clear();
        ProgramBuilder pb(st, materialized, &st.buf_vars);
        pb.build(&st.code, &st.n_regs);
    }
}

// =============================================================== executor

namespace {

size_t quad_levels_first_floats(ImgSize s, uint32_t nc) {
    if (s.h == 1) return size_t(ceil_shift(int(s.w), 8)) * nc;
    if (s.w == 1) return size_t(ceil_shift(int(s.h), 8)) * nc;
    return size_t(ceil_shift(int(s.w), 4)) * ceil_shift(int(s.h), 4) * nc;
}

}  // namespace

void quad_sum(const float* in, ImgSize s, uint32_t nc, float* out,
              float* scratch, cudaStream_t st) {
    // ping-pong halves of the scratch after the first level
    const size_t first = quad_levels_first_floats(s, nc);
    float* bufs[2] = {scratch, scratch + first};
    const float* src = in;
    int w = int(s.w), h = int(s.h), k = 0;
    if (w == 1 && h == 1) {
        DRESSI_CUDA(cudaMemcpyAsync(out, in, nc * 4, cudaMemcpyDeviceToDevice,
                                    st));
        return;
    }
    while (w > 1 || h > 1) {
        int ow, oh;
        float* dst;
        if (h == 1) {
            ow = ceil_shift(w, 8);
            oh = 1;
        } else if (w == 1) {
            ow = 1;
            oh = ceil_shift(h, 8);
        } else {
            ow = ceil_shift(w, 4);
            oh = ceil_shift(h, 4);
        }
        dst = (ow == 1 && oh == 1) ? out : bufs[k];
        if (h == 1)
            k_quad_sum<256, 1, 8><<<dim3(unsigned(ow), 1), 256, 0, st>>>(
                    src, w, h, int(nc), dst);
        else if (w == 1)
            k_quad_sum<1, 256, 8><<<dim3(1, unsigned(oh)), 256, 0, st>>>(
                    src, w, h, int(nc), dst);
        else
            k_quad_sum<16, 16, 4><<<dim3(unsigned(ow), unsigned(oh)), 256, 0,
                                    st>>>(src, w, h, int(nc), dst);
        check_launch();
        src = dst;
        k ^= 1;
        w = ow;
        h = oh;
    }
}

size_t quad_sum_scratch_floats(ImgSize s, uint32_t nc) {
    return 2 * quad_levels_first_floats(s, nc) + 64;
}

void launch_program(const Step& st, const Ins* code, const BufRef* bufs,
                    cudaStream_t s) {
    static bool attr_set[64] = {};
    int dev = 0;
    DRESSI_CUDA(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        DRESSI_CUDA(cudaFuncSetAttribute(
                k_pixel_prog, cudaFuncAttributeMaxDynamicSharedMemorySize,
                200 * 1024));
        attr_set[dev] = true;
    }
    const long long npx = (long long)st.grid.pixels();
    const int threads = npx <= 32 ? 32 : kProgThreads;
    const size_t smem = st.code.size() * sizeof(Ins) +
                        st.buf_vars.size() * sizeof(BufRef) +
                        size_t(st.n_regs) * threads * 4;
    DRESSI_REQUIRE(smem <= 200 * 1024,
                   "pixel program too large for shared memory");
    k_pixel_prog<<<grid_for(npx, threads, 148 * 16), threads, smem, s>>>(
            code, int(st.code.size()), bufs, int(st.buf_vars.size()),
            st.n_regs, npx, int(st.grid.w));
    check_launch();
}

// ---------------------------------------------------------- special ops

namespace {

int I(uint32_t v) { return int(v); }

AaDims aa_dims_of(uint32_t n_comp, uint32_t n_verts, uint32_t n_faces,
                  ImgSize sz) {
    AaDims d;
    d.W = I(sz.w);
    d.H = I(sz.h);
    d.views = 1;
    d.n_faces = I(n_faces);
    d.n_verts = I(n_verts);
    d.n_comp = I(n_comp);
    return d;
}

size_t aa_scratch_bytes(uint32_t n_faces) {
    return align_up(size_t(std::max<uint32_t>(n_faces, 1)) * sizeof(AaFace),
                    256) + 256;
}

SoftDims soft_dims_of(const Func& f) {
    const Var y = f->out();
    SoftDims d;
    d.W = I(y->size.w);
    d.H = I(y->size.h);
    d.views = 1;
    d.n_faces = I(f->xs[2]->size.w);
    d.n_verts = I(f->xs[3]->size.w);
    d.radius = f->fp[0];
    d.finalize();
    default_caps(&d);
    return d;
}

HardDims hard_dims_of(const Func& f, int n_comp) {
    const Var y = f->out();
    HardDims d;
    d.W = I(y->size.w);
    d.H = I(y->size.h);
    d.views = 1;
    d.n_faces = I(f->xs[2]->size.w);
    d.n_verts = I(f->xs[0]->size.w);
    d.n_comp = n_comp;
    d.finalize();
    return d;
}

}  // namespace

size_t special_scratch_bytes(const Func& f) {
    const Var y = f->out();
    switch (f->op) {
    case Op::Rasterize:
        return hard_workspace_bytes(hard_dims_of(f, I(ncomp(y->vtype))));
    case Op::RasterizeFaceId: return hard_workspace_bytes(hard_dims_of(f, 1));
    case Op::RasterizeSoft: {
        SoftDims d = soft_dims_of(f);
        Arena a;
        SoftBuffers b;
        carve_soft(a, d, &b);
        return a.used + 256;
    }
    case Op::RasterizeSoftGrad:
        return f->xs[0]->size.pixels() * 4 + 256;
    case Op::AntiAlias: return aa_scratch_bytes(f->xs[3]->size.w);
    case Op::AntiAliasGradImg: return aa_scratch_bytes(f->xs[3]->size.w);
    case Op::AntiAliasGradVtx: return aa_scratch_bytes(f->xs[4]->size.w);
    case Op::IrradianceConv: case Op::PrefilterConv:
        return env_conv_scratch_floats(I(f->xs[0]->size.w),
                                       I(f->xs[0]->size.h), I(y->size.w),
                                       I(y->size.h)) * 4 + 256;
    case Op::IrradianceConvGrad: case Op::PrefilterConvGrad:
        return env_conv_scratch_floats(I(y->size.w), I(y->size.h),
                                       I(f->xs[0]->size.w),
                                       I(f->xs[0]->size.h)) * 4 + 256;
    case Op::Sum:
        return quad_sum_scratch_floats(f->xs[0]->size,
                                       ncomp(f->xs[0]->vtype)) * 4;
    default: return 0;
    }
}

void launch_special(const Func& f, const std::vector<const float*>& in,
                    float* out, void* scratch, uint32_t* status,
                    cudaStream_t s) {
    const Var y = f->out();
    const Vars& xs = f->xs;
    const uint32_t ny = ncomp(y->vtype);
    const long long npx = (long long)y->size.pixels();
    switch (f->op) {
    case Op::Rasterize:
    case Op::RasterizeFaceId: {
        const bool ids = f->op == Op::RasterizeFaceId;
        HardDims d = hard_dims_of(f, ids ? 1 : I(ny));
        hard_raster_op(d, scratch, in[0], ids ? nullptr : in[1], in[2], out,
                       nullptr, status, s);
        break;
    }
    case Op::RasterizeSoft: {
        SoftDims d = soft_dims_of(f);
        Arena dry;
        SoftBuffers b;
        carve_soft(dry, d, &b);
        Arena a{static_cast<char*>(scratch), dry.used + 256, 0};
        carve_soft(a, d, &b);
        init_soft(d, b, s);
        b.status = status;
        SoftOpInputs si{in[0], in[1], in[2], in[3], in[4],
                        xs.size() > 6 ? in[6] : nullptr, I(xs[0]->size.w),
                        I(xs[3]->size.w)};
        soft_raster_op(d, b, si, out, s);
        break;
    }
    case Op::RasterizeSoftGrad: {
        // gy (VEC4 image): the dist channel feeds GatherDistGrad
        float* gy0 = static_cast<float*>(scratch);
        const Var g = xs[0];
        const long long n = (long long)g->size.pixels();
        k_extract_channel<<<grid_for(n, 256, 148 * 8), 256, 0, s>>>(
                in[0], I(ncomp(g->vtype)), 0, n, gy0);
        check_launch();
        DRESSI_CUDA(cudaMemsetAsync(out, 0, size_t(y->size.pixels()) * 16, s));
        dist_grad_op(gy0, in[1], in[2], in[3], 1, I(xs[2]->size.w),
                     I(xs[3]->size.w), I(g->size.w), I(g->size.h), out,
                     status, s);
        break;
    }
    case Op::SoftClip:
        soft_clip_op(in[0], in[1], 1, I(xs[0]->size.w), I(xs[1]->size.w),
                     I(uint32_t(f->fp[1])), I(uint32_t(f->fp[2])), f->fp[0],
                     out, status, s);
        break;
    case Op::AntiAlias: case Op::AntiAliasGradImg: case Op::AntiAliasGradVtx: {
        const bool vtx = f->op == Op::AntiAliasGradVtx;
        // inputs: AntiAlias (img, tri, clip, faces, vft, seed);
        // GradImg (gy, tri, clip, faces); GradVtx (gy, img, tri, clip,
        // faces, vft, seed)
        const int o = vtx ? 1 : 0;
        const float* tri = in[size_t(1 + o)];
        const float* clip = in[size_t(2 + o)];
        const float* faces = in[size_t(3 + o)];
        const Var img_v = xs[0];
        const uint32_t n_faces = xs[size_t(3 + o)]->size.w;
        const uint32_t n_verts = xs[size_t(2 + o)]->size.w;
        const AaDims d = aa_dims_of(ncomp(img_v->vtype), n_verts, n_faces,
                                    img_v->size);
        const size_t rec = align_up(size_t(std::max<uint32_t>(n_faces, 1)) *
                                            sizeof(AaFace), 256);
        AaFace* recs = static_cast<AaFace*>(scratch);
        int* vflags = reinterpret_cast<int*>(static_cast<char*>(scratch) + rec);
        aa_face_setup(d, clip, faces, recs, vflags, status, s);
        if (f->op == Op::AntiAlias) {
            aa_forward_op(d, recs, vflags, in[0], tri, out, s);
        } else if (f->op == Op::AntiAliasGradImg) {
            aa_bwd_img_op(d, recs, in[0], tri, out, s);
        } else {
            DRESSI_CUDA(cudaMemsetAsync(out, 0, size_t(n_verts) * 16, s));
            aa_bwd_vtx_op(d, recs, in[0], in[1], tri, clip, in[5],
                          I(xs[5]->size.h), 0.f, I(uint32_t(f->ip[0])), out,
                          s, in[6]);
        }
        break;
    }
    case Op::VertexNeighborMean:
        vertex_terms_op(in[0], I(xs[0]->size.w), in[1], I(xs[1]->size.h),
                        false, out, nullptr, nullptr, 0, nullptr, 0, nullptr,
                        status, s);
        break;
    case Op::NormalConsistencyFaceTerm:
        nc_face_term_op(in[0], I(xs[0]->size.w), in[1], in[2],
                        I(xs[1]->size.w), out, status, s);
        break;
    case Op::NormalConsistencyVertexGrad:
        vertex_terms_op(in[1], I(xs[1]->size.w), nullptr, 0, false, nullptr,
                        in[0], in[2], I(xs[2]->size.w), in[3],
                        I(xs[3]->size.h), out, status, s);
        break;
    case Op::LookupFaces:
        lookup_faces_op(in[0], I(xs[0]->size.w), I(ncomp(xs[0]->vtype)),
                        in[1], I(xs[1]->size.w), I(uint32_t(f->ip[0])), out,
                        status, s);
        break;
    case Op::LookupFacesGrad:
        lookup_faces_bwd_op(in[0], I(ncomp(xs[0]->vtype)), in[1],
                            I(xs[1]->size.w), in[2], I(xs[2]->size.w),
                            I(xs[2]->size.h), I(uint32_t(f->ip[0])), out,
                            status, s);
        break;
    case Op::FaceFetch:
        face_fetch_op(in[0], I(xs[0]->size.w), I(ncomp(xs[0]->vtype)), in[1],
                      npx, out, s);
        break;
    case Op::FaceFetchGrad:
        face_fetch_bwd_op(in[0], I(ncomp(xs[0]->vtype)), in[1],
                          I(xs[1]->size.w), I(xs[1]->size.h), in[2], in[3],
                          in[4], I(xs[2]->size.w), 0.f, f->fp[0],
                          I(uint32_t(f->ip[0])), out, s, in[5]);
        break;
    case Op::Texture: case Op::TextureBilinear:
        texture_sample_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h),
                          I(ncomp(xs[0]->vtype)),
                          f->op == Op::Texture ? 0 : 1, in[1], size_t(npx),
                          out, s);
        break;
    case Op::GatherInvUV: case Op::GatherInvUVBilinear:
        texture_gather_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h),
                          I(ncomp(xs[0]->vtype)),
                          f->op == Op::GatherInvUV ? 0 : 1, in[1],
                          I(xs[1]->size.w), I(xs[1]->size.h), in[2], out, s);
        break;
    case Op::EquirectSample:
        equirect_sample_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h),
                           I(ncomp(xs[0]->vtype)), in[1], npx, out, s);
        break;
    case Op::EquirectSampleGrad:
        equirect_sample_bwd_op(in[0], in[1], (long long)xs[1]->size.pixels(),
                               I(y->size.w), I(y->size.h), I(ny), out, s);
        break;
    case Op::IrradianceConv:
        irradiance_conv_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h), I(ny),
                           I(y->size.w), I(y->size.h), out,
                           static_cast<float*>(scratch), s);
        break;
    case Op::IrradianceConvGrad:
        irradiance_conv_bwd_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h),
                               I(ny), I(y->size.w), I(y->size.h), out,
                               static_cast<float*>(scratch), s);
        break;
    case Op::PrefilterConv:
        prefilter_conv_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h), I(ny),
                          I(y->size.w), I(y->size.h), f->fp[0], out,
                          static_cast<float*>(scratch), s);
        break;
    case Op::PrefilterConvGrad:
        prefilter_conv_bwd_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h),
                              I(ny), I(y->size.w), I(y->size.h), f->fp[0],
                              out, static_cast<float*>(scratch), s);
        break;
    case Op::BrdfLut:
        brdf_lut_op(I(y->size.w), I(y->size.h), I(uint32_t(f->ip[0])), out,
                    s);
        break;
    case Op::AvgPool2x2:
        avg_pool2x2_op(in[0], I(xs[0]->size.w), I(xs[0]->size.h), I(ny), out,
                       s);
        break;
    case Op::AvgPool2x2Grad:
        avg_pool2x2_bwd_op(in[0], I(y->size.w), I(y->size.h), I(ny), out, s);
        break;
    case Op::PixelFetch:
        k_pixel_fetch<<<1, 32, 0, s>>>(in[0], I(xs[0]->size.w),
                                       I(xs[0]->size.h), I(ny),
                                       I(uint32_t(f->ip[0])), in[1], out,
                                       status);
        check_launch();
        break;
    case Op::TileFetch:
        k_tile_fetch<<<grid_for(npx * ny, 256, 148 * 8), 256, 0, s>>>(
                in[0], I(xs[0]->size.w), I(xs[0]->size.h), I(ny),
                I(uint32_t(f->ip[0])), in[1], out, status);
        check_launch();
        break;
    case Op::Sum:
        quad_sum(in[0], xs[0]->size, ncomp(xs[0]->vtype), out,
                 static_cast<float*>(scratch), s);
        break;
    default:
        throw_error(kErrInvalid,
                    std::string("executor: op not supported: ") +
                            op_name(f->op),
                    __FILE__, __LINE__);
    }
}

}  // namespace graph
}  // namespace dressi
