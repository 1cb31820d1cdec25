// Host-side internals shared by the dot_b200 translation units: error state,
// launch accounting / optional event timing, workspace carving.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <string>

#include "../../include/dot_b200.h"

namespace dotb {

// ---- error state (thread-local text, returned through dot_last_error) -----
void set_error(const std::string& msg);
void clear_error();
int fail(int code, const std::string& msg);
// Checks cudaGetLastError() after launches; returns DOT_OK or DOT_ERR_CUDA.
int check_launch(const char* what);

// ---- launch accounting ------------------------------------------------------
// Every kernel launch goes through prof_pre/prof_post with its class.  The
// counters are always on; event timing only between dot_prof_begin/end.
// A scope may cover several launches of one class (`count`): its events then
// time the whole run of launches, gaps included.
void prof_pre(int kclass, cudaStream_t s, int count = 1);
void prof_post(int kclass, cudaStream_t s);

struct ProfScope {
    int k;
    cudaStream_t s;
    ProfScope(int kclass, cudaStream_t st, int count = 1) : k(kclass), s(st) { prof_pre(k, s, count); }
    ~ProfScope() { prof_post(k, s); }
};

// ---- workspace carving --------------------------------------------------------
// Sub-buffers are 256-byte aligned; `size()` is the total the caller must give.
struct Carve {
    char* base;
    size_t off = 0;
    explicit Carve(void* b) : base(static_cast<char*>(b)) {}
    template <typename T>
    T* take(size_t count) {
        off = (off + 255) & ~size_t(255);
        T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
    size_t size() const { return (off + 255) & ~size_t(255); }
};

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace dotb
