// Internal interface of the graph executor (graph_exec.cu) to the DressiAD
// driver (graph_capi.cu): the lowered step list and the launchers.
#pragma once

#include <cuda_runtime.h>

#include <unordered_set>
#include <vector>

#include "graph.h"

namespace dressi {
namespace graph {

// Opcodes of the pixel-program interpreter (one scalar result each).
enum PO : uint16_t {
    P_NOP = 0, P_LOAD, P_STORE, P_CONST, P_SCRX, P_SCRY, P_ADD, P_SUB, P_MUL,
    P_DIV, P_NEG, P_SIN, P_COS, P_TAN, P_ASIN, P_ACOS, P_ATAN, P_ATAN2,
    P_EXP, P_EXP2, P_LOG, P_LOG2, P_SQRT, P_RSQRT, P_ABS, P_SIGN, P_FLOOR,
    P_FRACT, P_MOD, P_POW, P_MAX, P_MIN, P_CLAMP, P_MIX, P_STEP, P_SMOOTH,
    P_SIGMOID, P_LT, P_LE, P_GT, P_GE
};

// 16 bytes: registers a, b, c -> dst; LOAD / STORE use the buffer slot and
// component imm; CONST carries the float bits in imm.
struct Ins {
    uint16_t op, dst, a, b, c, buf;
    uint32_t imm;
};
static_assert(sizeof(Ins) == 16, "Ins layout");

// A program's buffer table entry: the value's device image, its component
// count (the pixel stride) and whether it is a {1,1} value read at every
// pixel.
struct BufRef {
    float* ptr;
    uint32_t stride;
    uint32_t uniform;
};
static_assert(sizeof(BufRef) == 16, "BufRef layout");

struct Step {
    enum Kind { kProgram, kSum, kSumAll, kSpecial } kind = kProgram;
    ImgSize grid;
    std::vector<Func> funcs;         // the fused ops (one for other kinds)
    // programs
    std::vector<Ins> code;
    std::vector<uint64_t> buf_vars;  // var id per buffer slot
    int n_regs = 0;
};

struct Plan {
    std::vector<Step> steps;
    std::unordered_set<uint64_t> materialized;  // values that get buffers
    // Groups exec_funcs (creation order) into steps; roots are always
    // materialised. max_group bounds the ops fused into one program.
    void build(const std::vector<Func>& exec_funcs, const Vars& roots,
               size_t max_group);
};

void launch_program(const Step& st, const Ins* code, const BufRef* bufs,
                    cudaStream_t s);
size_t special_scratch_bytes(const Func& f);
// Runs a reduction or special op: in[i] = device image of f->xs[i].
void launch_special(const Func& f, const std::vector<const float*>& in,
                    float* out, void* scratch, uint32_t* status,
                    cudaStream_t s);

}  // namespace graph
}  // namespace dressi
