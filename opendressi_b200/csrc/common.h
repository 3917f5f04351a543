// Host-side infrastructure shared by the translation units of
// libdressi_b200.so: error propagation to the C ABI and small helpers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

namespace dressi {

// Thrown inside the library, caught at the C boundary and turned into a
// status code plus dressi_last_error() text (the reference reports errors
// as DressiError with file:line, include/dressi/types.h:110-123).
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

constexpr int kOk = 0;
constexpr int kErrInvalid = 1;
constexpr int kErrCuda = 2;
constexpr int kErrOom = 3;
constexpr int kErrDevice = 4;

void set_last_error(const std::string& msg);

[[noreturn]] inline void throw_error(int code, const std::string& msg,
                                     const char* file, int line) {
    throw Error(code, msg + " (" + file + ":" + std::to_string(line) + ")");
}

#define DRESSI_REQUIRE(cond, msg)                                        \
    do {                                                                 \
        if (!(cond)) ::dressi::throw_error(::dressi::kErrInvalid, (msg), \
                                           __FILE__, __LINE__);          \
    } while (0)

#define DRESSI_CUDA(expr)                                                     \
    do {                                                                      \
        const cudaError_t e_ = (expr);                                        \
        if (e_ != cudaSuccess) {                                              \
            ::dressi::throw_error(e_ == cudaErrorMemoryAllocation             \
                                          ? ::dressi::kErrOom                 \
                                          : ::dressi::kErrCuda,               \
                                  std::string(#expr) + ": " +                 \
                                          cudaGetErrorString(e_),             \
                                  __FILE__, __LINE__);                        \
        }                                                                     \
    } while (0)

// Runs `fn`, converting exceptions into a C status code.
template <typename Fn>
int guarded(Fn&& fn) {
    try {
        fn();
        return kOk;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return kErrOom;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return kErrInvalid;
    }
}

inline size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

// Debug timing of individual kernels outside the CUDA graph: while a
// profiler is installed on the calling thread, every launch site wrapped in
// a ProfScope (the outermost of nested ones) is bracketed by a pair of CUDA
// events on its stream.
struct KernelProfiler {
    struct Rec {
        const char* name;
        cudaEvent_t a, b;
    };
    std::vector<Rec> recs;
    int depth = 0;  // open scopes; a scope nested in another is not timed
    void begin(const char* name, cudaStream_t s);
    void end(cudaStream_t s);
    // Synchronises and accumulates per-name totals (ms) and launch counts.
    void collect(std::vector<const char*>* names, std::vector<double>* ms,
                 std::vector<int>* count);
    ~KernelProfiler();
};
KernelProfiler*& current_profiler();

struct ProfScope {
    cudaStream_t s;
    KernelProfiler* p;
    ProfScope(const char* name, cudaStream_t st) : s(st), p(current_profiler()) {
        if (p && p->depth++ == 0) p->begin(name, s);
    }
    ~ProfScope() {
        if (p && --p->depth == 0) p->end(s);
    }
};

// Bump allocator over one device block (plans and op-level workspaces).
struct Arena {
    char* base = nullptr;
    size_t size = 0, used = 0;
    template <typename T>
    T* take(size_t n) {
        used = align_up(used, 256);
        T* p = reinterpret_cast<T*>(base + used);
        used += sizeof(T) * n;
        if (base && used > size) {
            throw_error(kErrInvalid, "workspace too small", __FILE__,
                        __LINE__);
        }
        return p;
    }
};

}  // namespace dressi
