// DressiAD on CUDA: the reference's staged execStep ladder
// (src/dressi_ad.cpp:280-530) over this library's graph path -- backward
// construction, optimizer wiring, traversal, reactive pruning, the fusion
// plan, and one CUDA graph per build that replays forward, backward,
// optimizer and copy-backs with no per-iteration host traffic -- and the C
// ABI of the graph (dressi_var_* / dressi_op / dressi_ad_* in
// include/dressi_b200.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <unordered_map>
#include <unordered_set>

#include "../../include/dressi_b200.h"
#include "graph.h"
#include "graph_exec.h"
#include "kernels.h"

namespace dressi {
namespace graph {
namespace {

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        DRESSI_CUDA(cudaGetDevice(&prev));
        if (prev != dev) DRESSI_CUDA(cudaSetDevice(dev));
    }
    ~DevGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && prev >= 0 && cur != prev)
            cudaSetDevice(prev);
    }
};

}  // namespace

class AdImpl {
public:
    enum Status { kBackward, kOptimizer, kTraverse, kPlan, kFinished };

    int device = 0;
    Var loss;
    dressi_optimizer_fn opt_fn = nullptr;
    void* opt_user = nullptr;
    Status status = kBackward;
    Vars input_vars, grad_vars, updated_vars;
    std::vector<std::pair<Var, Var>> extra_updates;  // (input leaf, updated)
    Vars extra_outputs;
    bool grad_outputs = false;
    std::vector<Func> all_funcs;
    Vars leaf_vars;
    std::vector<std::pair<Var, Var>> copy_backs;  // (updated, input leaf)
    uint32_t fast_rebuild = 2, full_rebuild = 8, static_cnt = 0;
    std::set<uint64_t> prev_dirty;
    bool pruning_active = false;
    size_t max_group = 512;
    uint32_t rebuilds = 0;

    struct Buf {
        float* ptr = nullptr;
        size_t floats = 0;
        bool valid = false;           // holds a computed / sent value
        std::weak_ptr<VarNode> var;   // freed when the variable dies
    };
    std::unordered_map<uint64_t, Buf> bufs;
    Plan plan;
    size_t exec_funcs = 0;
    void* prog_mem = nullptr;
    std::vector<size_t> prog_code_off, prog_buf_off;
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    uint32_t* status_dev = nullptr;
    cudaStream_t cap = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint32_t kernels_per_iter = 0;

    explicit AdImpl(int dev) : device(dev) {
        DevGuard g(device);
        DRESSI_CUDA(cudaMalloc(&status_dev, 4));
        DRESSI_CUDA(cudaMemset(status_dev, 0, 4));
        DRESSI_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    }

    ~AdImpl() {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (exec) cudaGraphExecDestroy(exec);
        for (auto& [id, b] : bufs)
            if (b.ptr) cudaFree(b.ptr);
        if (prog_mem) cudaFree(prog_mem);
        if (scratch) cudaFree(scratch);
        if (status_dev) cudaFree(status_dev);
        if (cap) cudaStreamDestroy(cap);
        if (prev >= 0) cudaSetDevice(prev);
    }

    void invalidate(Status s) {
        if (status > s) status = s;
    }

    Vars roots() const {
        Vars r = updated_vars;
        r.push_back(loss);
        for (const auto& v : extra_outputs) r.push_back(v);
        for (const auto& [inp, upd] : extra_updates) r.push_back(upd);
        if (grad_outputs)
            for (const auto& g : grad_vars) r.push_back(g);
        return r;
    }

    std::set<uint64_t> dirty_leaf_ids() const {
        std::set<uint64_t> ids;
        for (const auto& v : leaf_vars)
            if (v->dirty) ids.insert(v->id);
        return ids;
    }

    // ComputeDynamicVarIds (src/pack/reactive.cpp:10-31): the seeds are
    // the dirty leaves, the optimised parameters and the addUpdate inputs.
    std::unordered_set<uint64_t> dynamic_ids() const {
        std::unordered_set<uint64_t> dyn;
        for (const auto& v : leaf_vars)
            if (v->dirty) dyn.insert(v->id);
        if (opt_fn)
            for (const auto& v : input_vars) dyn.insert(v->id);
        for (const auto& [inp, upd] : extra_updates) dyn.insert(inp->id);
        for (const auto& f : all_funcs) {
            for (const auto& x : f->xs) {
                if (dyn.count(x->id)) {
                    dyn.insert(f->out()->id);
                    break;
                }
            }
        }
        return dyn;
    }

    bool has_cached(const Var& v) const {
        auto it = bufs.find(v->id);
        return it != bufs.end() && it->second.valid;
    }

    // FilterExecutableFuncs (src/pack/reactive.cpp:33-66): what the roots
    // need, except static values that an earlier iteration left cached.
    std::vector<Func> executable(const std::unordered_set<uint64_t>& dyn) {
        std::unordered_set<uint64_t> need, seen;
        Vars stack = roots();
        while (!stack.empty()) {
            Var v = stack.back();
            stack.pop_back();
            if (!v || !seen.insert(v->id).second) continue;
            Func c = v->creator;
            if (!c || v->is_const) continue;
            if (!dyn.count(v->id) && has_cached(v)) continue;
            if (need.insert(c->id).second)
                for (const auto& x : c->xs) stack.push_back(x);
        }
        std::vector<Func> out;
        for (const auto& f : all_funcs)
            if (need.count(f->id)) out.push_back(f);
        return out;
    }

    float* buffer(const Var& v) {
        auto it = bufs.find(v->id);
        DRESSI_REQUIRE(it != bufs.end() && it->second.ptr,
                       "DressiAD: the Variable has no device image (mark it "
                       "with markOutput before the first execStep)");
        return it->second.ptr;
    }

    Buf& ensure_buffer(const Var& v) {
        Buf& b = bufs[v->id];
        const size_t n = std::max<size_t>(1, v->size.pixels() * ncomp(v->vtype));
        if (b.ptr && b.floats == n) return b;
        if (b.ptr) cudaFree(b.ptr);
        b = Buf{};
        DRESSI_CUDA(cudaMalloc(&b.ptr, n * 4));
        DRESSI_CUDA(cudaMemset(b.ptr, 0, n * 4));
        b.floats = n;
        b.var = v;
        if (v->is_const) {
            std::vector<float> c(n);
            for (size_t i = 0; i < n; i++) c[i] = v->cval[i % v->cval.size()];
            DRESSI_CUDA(cudaMemcpy(b.ptr, c.data(), n * 4,
                                   cudaMemcpyHostToDevice));
            b.valid = true;
        }
        return b;
    }

    void build_plan() {
        const auto dyn = dynamic_ids();
        std::vector<Func> ex = executable(dyn);
        size_t packable = 0;
        for (const auto& f : all_funcs)
            if (!f->out()->is_const) packable++;
        size_t n_ex = 0;
        for (const auto& f : ex)
            if (!f->out()->is_const) n_ex++;
        pruning_active = n_ex < packable;
        exec_funcs = n_ex;
        const Vars r = roots();
        // a program whose registers would not fit shared memory is split
        // by halving the fusion bound
        for (size_t cap_ops = max_group;; cap_ops = std::max<size_t>(1, cap_ops / 2)) {
            plan.build(ex, r, cap_ops);
            bool fits = true;
            for (const auto& st : plan.steps)
                if (st.kind == Step::kProgram && st.n_regs > 192) fits = false;
            if (fits || cap_ops == 1) break;
        }
        // every value a step reads or writes gets a device image
        std::unordered_map<uint64_t, Var> by_id;
        for (const auto& f : ex) {
            by_id[f->out()->id] = f->out();
            for (const auto& x : f->xs) by_id[x->id] = x;
        }
        for (const auto& [upd, inp] : copy_backs) {
            by_id[upd->id] = upd;
            by_id[inp->id] = inp;
        }
        for (const auto& v : r) by_id[v->id] = v;
        std::unordered_set<uint64_t> needed(plan.materialized.begin(),
                                            plan.materialized.end());
        for (const auto& [upd, inp] : copy_backs) {
            needed.insert(upd->id);
            needed.insert(inp->id);
        }
        for (const auto& v : leaf_vars) needed.insert(v->id);
        for (uint64_t id : needed) {
            auto it = by_id.find(id);
            if (it != by_id.end()) ensure_buffer(it->second);
        }
        // release images of variables that no longer exist
        for (auto it = bufs.begin(); it != bufs.end();) {
            if (it->second.var.expired()) {
                cudaFree(it->second.ptr);
                it = bufs.erase(it);
            } else {
                ++it;
            }
        }
        // program code + buffer tables in one device block
        size_t bytes = 0;
        prog_code_off.assign(plan.steps.size(), 0);
        prog_buf_off.assign(plan.steps.size(), 0);
        for (size_t i = 0; i < plan.steps.size(); i++) {
            const Step& st = plan.steps[i];
            if (st.kind != Step::kProgram) continue;
            prog_code_off[i] = bytes;
            bytes += align_up(st.code.size() * sizeof(Ins), 256);
            prog_buf_off[i] = bytes;
            bytes += align_up(st.buf_vars.size() * sizeof(BufRef), 256);
        }
        std::vector<char> host(std::max<size_t>(bytes, 256));
        for (size_t i = 0; i < plan.steps.size(); i++) {
            const Step& st = plan.steps[i];
            if (st.kind != Step::kProgram) continue;
            std::memcpy(host.data() + prog_code_off[i], st.code.data(),
                        st.code.size() * sizeof(Ins));
            auto* br = reinterpret_cast<BufRef*>(host.data() + prog_buf_off[i]);
            for (size_t k = 0; k < st.buf_vars.size(); k++) {
                const Var& v = by_id.at(st.buf_vars[k]);
                br[k].ptr = buffer(v);
                br[k].stride = ncomp(v->vtype);
                br[k].uniform = v->size.uniform() && !st.grid.uniform();
            }
        }
        if (prog_mem) cudaFree(prog_mem);
        prog_mem = nullptr;
        DRESSI_CUDA(cudaMalloc(&prog_mem, host.size()));
        DRESSI_CUDA(cudaMemcpy(prog_mem, host.data(), host.size(),
                               cudaMemcpyHostToDevice));
        // shared scratch of the special kernels (they run one at a time)
        size_t need = 256;
        for (const auto& st : plan.steps)
            if (st.kind != Step::kProgram)
                need = std::max(need, special_scratch_bytes(st.funcs[0]));
        if (need > scratch_bytes) {
            if (scratch) cudaFree(scratch);
            scratch = nullptr;
            DRESSI_CUDA(cudaMalloc(&scratch, need));
            scratch_bytes = need;
        }
        sum_all_setup();
        capture(by_id);
        rebuilds++;
    }

    void record(const std::unordered_map<uint64_t, Var>& by_id,
                cudaStream_t s) {
        for (size_t i = 0; i < plan.steps.size(); i++) {
            const Step& st = plan.steps[i];
            if (st.kind == Step::kProgram) {
                const char* base = static_cast<const char*>(prog_mem);
                launch_program(st,
                               reinterpret_cast<const Ins*>(base +
                                                            prog_code_off[i]),
                               reinterpret_cast<const BufRef*>(
                                       base + prog_buf_off[i]),
                               s);
                continue;
            }
            const Func& f = st.funcs[0];
            Var y = f->out();
            if (st.kind == Step::kSumAll) {
                Var x = f->xs[0];
                if (x->creator && x->creator->op == Op::SumPartial)
                    x = x->creator->xs[0];
                DRESSI_REQUIRE(ncomp(x->vtype) <= 4,
                               "SumAll: at most 4 components");
                sum_all_op(buffer(x), int(x->size.pixels()),
                           int(ncomp(x->vtype)), buffer(y), s);
                continue;
            }
            std::vector<const float*> in;
            for (const auto& x : f->xs) in.push_back(buffer(x));
            launch_special(f, in, buffer(y), scratch, status_dev, s);
        }
        for (const auto& [upd, inp] : copy_backs) {
            const size_t n = std::max<size_t>(
                    1, inp->size.pixels() * ncomp(inp->vtype));
            DRESSI_CUDA(cudaMemcpyAsync(buffer(inp), buffer(upd), n * 4,
                                        cudaMemcpyDeviceToDevice, s));
        }
    }

    void capture(const std::unordered_map<uint64_t, Var>& by_id) {
        if (exec) {
            cudaGraphExecDestroy(exec);
            exec = nullptr;
        }
        cudaGraph_t g = nullptr;
        DRESSI_CUDA(cudaStreamBeginCapture(cap,
                                           cudaStreamCaptureModeThreadLocal));
        try {
            record(by_id, cap);
        } catch (...) {
            cudaStreamEndCapture(cap, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        DRESSI_CUDA(cudaStreamEndCapture(cap, &g));
        size_t n_nodes = 0;
        DRESSI_CUDA(cudaGraphGetNodes(g, nullptr, &n_nodes));
        std::vector<cudaGraphNode_t> nodes(n_nodes);
        DRESSI_CUDA(cudaGraphGetNodes(g, nodes.data(), &n_nodes));
        uint32_t k = 0;
        for (auto nd : nodes) {
            cudaGraphNodeType t;
            DRESSI_CUDA(cudaGraphNodeGetType(nd, &t));
            if (t == cudaGraphNodeTypeKernel) k++;
        }
        kernels_per_iter = k;
        const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        DRESSI_CUDA(e);
    }

    void exec_step(cudaStream_t s) {
        DRESSI_REQUIRE(loss, "setLossVar() must be called before execStep()");
        DevGuard dg(device);
        // reactive cache: watch the dirty pattern of the data leaves
        // (src/dressi_ad.cpp:290-308)
        if (status == kFinished) {
            const std::set<uint64_t> cur = dirty_leaf_ids();
            if (cur != prev_dirty) {
                static_cnt = 0;
                if (pruning_active) status = kPlan;
            } else {
                static_cnt++;
                if ((fast_rebuild && static_cnt == fast_rebuild) ||
                    (full_rebuild && static_cnt == full_rebuild))
                    status = kPlan;
            }
            prev_dirty = cur;
        }
        const Status entry = status;
        if (status <= kBackward) build_backward(loss, &input_vars, &grad_vars);
        if (status <= kOptimizer) {
            updated_vars.clear();
            copy_backs.clear();
            if (opt_fn) call_optimizer();
            for (const auto& [inp, upd] : extra_updates)
                copy_backs.emplace_back(upd, inp);
        }
        if (status <= kTraverse) {
            all_funcs = traverse(roots());
            leaf_vars.clear();
            std::unordered_set<uint64_t> seen;
            for (const auto& f : all_funcs)
                for (const auto& x : f->xs)
                    if (!x->creator && !x->is_const &&
                        seen.insert(x->id).second)
                        leaf_vars.push_back(x);
        }
        if (status <= kPlan) build_plan();
        DRESSI_CUDA(cudaGraphLaunch(exec, s));
        // everything the plan writes now holds this iteration's value
        for (const auto& st : plan.steps)
            for (const auto& f : st.funcs) {
                auto it = bufs.find(f->out()->id);
                if (it != bufs.end()) it->second.valid = true;
            }
        if (entry != kFinished) prev_dirty = dirty_leaf_ids();
        for (auto& v : leaf_vars) set_dirty_recursively(v, false);
        status = kFinished;
    }

    void call_optimizer() {
        const uint32_t n = uint32_t(input_vars.size());
        std::vector<dressi_var> hx(n), hg(n), ho(n, nullptr);
        for (uint32_t i = 0; i < n; i++) {
            hx[i] = reinterpret_cast<dressi_var>(new Var(input_vars[i]));
            hg[i] = reinterpret_cast<dressi_var>(new Var(grad_vars[i]));
        }
        int rc = 0;
        try {
            rc = opt_fn(opt_user, hx.data(), hg.data(), n, ho.data());
        } catch (...) {
            rc = -1;
        }
        for (uint32_t i = 0; i < n; i++) {
            delete reinterpret_cast<Var*>(hx[i]);
            delete reinterpret_cast<Var*>(hg[i]);
        }
        std::vector<Var> outs;
        for (uint32_t i = 0; i < n; i++) {
            if (ho[i]) {
                outs.push_back(*reinterpret_cast<Var*>(ho[i]));
                delete reinterpret_cast<Var*>(ho[i]);
            } else {
                outs.push_back(nullptr);
            }
        }
        DRESSI_REQUIRE(rc == 0, "optimizer callback failed");
        for (uint32_t i = 0; i < n; i++) {
            const Var& u = outs[i];
            const Var& x = input_vars[i];
            DRESSI_REQUIRE(u, "Optimizer must return one output per input");
            DRESSI_REQUIRE(u->vtype == x->vtype && u->size == x->size,
                           "Optimizer output must match its input's type "
                           "and size");
            updated_vars.push_back(u);
            copy_backs.emplace_back(u, x);
        }
    }

    void send(const Var& v, const float* data, size_t n, bool on_device,
              cudaStream_t s) {
        DevGuard dg(device);
        const size_t want = v->size.pixels() * ncomp(v->vtype);
        DRESSI_REQUIRE(n == want, "sendImg: size mismatch (" +
                                          std::to_string(n) + " floats for " +
                                          std::to_string(want) + ")");
        Buf& b = ensure_buffer(v);
        DRESSI_CUDA(cudaMemcpyAsync(b.ptr, data, n * 4,
                                    on_device ? cudaMemcpyDeviceToDevice
                                              : cudaMemcpyHostToDevice,
                                    s));
        if (!on_device) DRESSI_CUDA(cudaStreamSynchronize(s));
        b.valid = true;
        v->dirty = true;
    }

    void recv(const Var& v, float* data, size_t n, bool on_device,
              cudaStream_t s) {
        DevGuard dg(device);
        const size_t want = v->size.pixels() * ncomp(v->vtype);
        DRESSI_REQUIRE(n == want, "recvImg: size mismatch");
        DRESSI_CUDA(cudaMemcpyAsync(data, buffer(v), n * 4,
                                    on_device ? cudaMemcpyDeviceToDevice
                                              : cudaMemcpyDeviceToHost,
                                    s));
        if (!on_device) DRESSI_CUDA(cudaStreamSynchronize(s));
    }
};

}  // namespace graph
}  // namespace dressi

using namespace dressi;
using namespace dressi::graph;

struct dressi_ad_s {
    std::unique_ptr<AdImpl> impl;
};

namespace {

Var& V(dressi_var h) {
    DRESSI_REQUIRE(h, "null Variable handle");
    Var* v = reinterpret_cast<Var*>(h);
    DRESSI_REQUIRE(*v, "null Variable");
    return *v;
}

dressi_var wrap(Var v) { return reinterpret_cast<dressi_var>(new Var(std::move(v))); }

AdImpl& A(dressi_ad h) {
    DRESSI_REQUIRE(h && h->impl, "null DressiAD handle");
    return *h->impl;
}

}  // namespace

extern "C" {

int dressi_var_create(int vtype, uint32_t w, uint32_t h, dressi_var* out) {
    return guarded([&] {
        DRESSI_REQUIRE(out, "null pointer");
        DRESSI_REQUIRE(vtype >= FLOAT && vtype <= UINT, "invalid VType");
        *out = wrap(make_leaf(VType(vtype), {w, h}));
    });
}

int dressi_var_clone(dressi_var v, dressi_var* out) {
    return guarded([&] {
        DRESSI_REQUIRE(out, "null pointer");
        *out = wrap(V(v));
    });
}

int dressi_var_release(dressi_var v) {
    delete reinterpret_cast<Var*>(v);
    return 0;
}

int dressi_var_info(dressi_var v, int* vtype, uint32_t* w, uint32_t* h,
                    uint64_t* id, int* computed) {
    return guarded([&] {
        const Var& x = V(v);
        if (vtype) *vtype = int(x->vtype);
        if (w) *w = x->size.w;
        if (h) *h = x->size.h;
        if (id) *id = x->id;
        if (computed) *computed = x->creator ? 1 : 0;
    });
}

int dressi_var_set_requires_grad(dressi_var v, int req, int recursive) {
    return guarded([&] {
        if (recursive)
            set_requires_grad_recursively(V(v), req != 0);
        else
            V(v)->req_grad = req != 0;
    });
}

int dressi_var_requires_grad(dressi_var v, int* req) {
    return guarded([&] {
        DRESSI_REQUIRE(req, "null pointer");
        *req = V(v)->req_grad ? 1 : 0;
    });
}

int dressi_var_set_dirty(dressi_var v, int dirty, int recursive) {
    return guarded([&] {
        if (recursive)
            set_dirty_recursively(V(v), dirty != 0);
        else
            V(v)->dirty = dirty != 0;
    });
}

int dressi_op(const char* name, const dressi_var* xs, uint32_t n_xs,
              const float* fparams, uint32_t n_f, const int64_t* iparams,
              uint32_t n_i, dressi_var* out) {
    return guarded([&] {
        DRESSI_REQUIRE(name && out, "null pointer");
        DRESSI_REQUIRE(n_xs == 0 || xs, "null inputs");
        Vars in;
        for (uint32_t i = 0; i < n_xs; i++) in.push_back(V(xs[i]));
        std::vector<float> fp(fparams, fparams + (fparams ? n_f : 0));
        std::vector<int64_t> ip(iparams, iparams + (iparams ? n_i : 0));
        *out = wrap(build_named(name, in, fp, ip));
    });
}

int dressi_ad_create(int device, dressi_ad* out) {
    return guarded([&] {
        DRESSI_REQUIRE(out, "null pointer");
        *out = nullptr;
        auto h = std::make_unique<dressi_ad_s>();
        h->impl = std::make_unique<AdImpl>(device);
        *out = h.release();
    });
}

int dressi_ad_destroy(dressi_ad ad) {
    delete ad;
    return 0;
}

int dressi_ad_set_loss(dressi_ad ad, dressi_var loss) {
    return guarded([&] {
        AdImpl& a = A(ad);
        a.loss = V(loss);
        a.status = AdImpl::kBackward;
    });
}

int dressi_ad_set_optimizer(dressi_ad ad, dressi_optimizer_fn fn,
                            void* user) {
    return guarded([&] {
        AdImpl& a = A(ad);
        a.opt_fn = fn;
        a.opt_user = user;
        a.status = AdImpl::kBackward;
    });
}

int dressi_ad_add_update(dressi_ad ad, dressi_var input_leaf,
                         dressi_var updated) {
    return guarded([&] {
        AdImpl& a = A(ad);
        const Var& inp = V(input_leaf);
        const Var& upd = V(updated);
        DRESSI_REQUIRE(!inp->creator, "addUpdate: input must be a leaf "
                                      "Variable");
        DRESSI_REQUIRE(upd->creator, "addUpdate: updated must be a computed "
                                     "Variable");
        DRESSI_REQUIRE(inp->vtype == upd->vtype && inp->size == upd->size,
                       "addUpdate: updated must match the input's type and "
                       "size");
        a.extra_updates.emplace_back(inp, upd);
        a.invalidate(AdImpl::kOptimizer);
    });
}

int dressi_ad_mark_output(dressi_ad ad, dressi_var v) {
    return guarded([&] {
        AdImpl& a = A(ad);
        a.extra_outputs.push_back(V(v));
        a.invalidate(AdImpl::kTraverse);
    });
}

int dressi_ad_set_grad_outputs(dressi_ad ad, int enable) {
    return guarded([&] {
        AdImpl& a = A(ad);
        if (a.grad_outputs == (enable != 0)) return;
        a.grad_outputs = enable != 0;
        a.invalidate(AdImpl::kTraverse);
    });
}

int dressi_ad_set_rebuild_counts(dressi_ad ad, uint32_t fast, uint32_t full) {
    return guarded([&] {
        AdImpl& a = A(ad);
        a.fast_rebuild = fast;
        a.full_rebuild = full;
    });
}

int dressi_ad_set_max_fusion(dressi_ad ad, uint32_t max_ops) {
    return guarded([&] {
        AdImpl& a = A(ad);
        DRESSI_REQUIRE(max_ops >= 1, "max fusion must be >= 1");
        a.max_group = max_ops;
        a.invalidate(AdImpl::kPlan);
    });
}

int dressi_ad_input_grads(dressi_ad ad, dressi_var* xs, dressi_var* gxs,
                          uint32_t cap, uint32_t* n) {
    return guarded([&] {
        AdImpl& a = A(ad);
        DRESSI_REQUIRE(n, "null pointer");
        *n = uint32_t(a.input_vars.size());
        for (uint32_t i = 0; i < std::min(cap, *n); i++) {
            if (xs) xs[i] = wrap(a.input_vars[i]);
            if (gxs) gxs[i] = wrap(a.grad_vars[i]);
        }
    });
}

int dressi_ad_exec_step(dressi_ad ad, void* stream) {
    return guarded([&] {
        A(ad).exec_step(static_cast<cudaStream_t>(stream));
    });
}

int dressi_ad_send(dressi_ad ad, dressi_var v, const float* data,
                   size_t n_floats, int on_device, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(data, "null pointer");
        A(ad).send(V(v), data, n_floats, on_device != 0,
                   static_cast<cudaStream_t>(stream));
    });
}

int dressi_ad_recv(dressi_ad ad, dressi_var v, float* data, size_t n_floats,
                   int on_device, void* stream) {
    return guarded([&] {
        DRESSI_REQUIRE(data, "null pointer");
        A(ad).recv(V(v), data, n_floats, on_device != 0,
                   static_cast<cudaStream_t>(stream));
    });
}

int dressi_ad_stats(dressi_ad ad, dressi_ad_stats_t* out) {
    return guarded([&] {
        AdImpl& a = A(ad);
        DRESSI_REQUIRE(out, "null pointer");
        std::memset(out, 0, sizeof(*out));
        out->n_funcs = uint32_t(a.all_funcs.size());
        out->n_exec_funcs = uint32_t(a.exec_funcs);
        out->n_steps = uint32_t(a.plan.steps.size());
        for (const auto& st : a.plan.steps) {
            if (st.kind == Step::kProgram) {
                out->n_programs++;
                out->n_fused_ops += uint32_t(st.funcs.size());
                out->max_program_regs =
                        std::max(out->max_program_regs, uint32_t(st.n_regs));
                out->n_program_instructions += uint32_t(st.code.size());
            }
        }
        out->n_materialized = uint32_t(a.plan.materialized.size());
        out->kernels_per_iter = a.kernels_per_iter;
        out->rebuilds = a.rebuilds;
        out->pruning_active = a.pruning_active ? 1 : 0;
    });
}

int dressi_ad_status(dressi_ad ad, uint32_t* word, int clear) {
    return guarded([&] {
        AdImpl& a = A(ad);
        DRESSI_REQUIRE(word, "null pointer");
        DevGuard dg(a.device);
        DRESSI_CUDA(cudaDeviceSynchronize());
        DRESSI_CUDA(cudaMemcpy(word, a.status_dev, 4, cudaMemcpyDeviceToHost));
        if (clear) DRESSI_CUDA(cudaMemset(a.status_dev, 0, 4));
    });
}

}  // extern "C"
