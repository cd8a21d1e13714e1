// Shared plumbing of libzpucuda.so: status helpers, the per-thread device /
// stream binding (the device-side mirror of zpu's threadlocal Ctx,
// src/zpu/context.zig:34-58), launch accounting and small device helpers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/zpucuda.h"

namespace zc {

struct ThreadState {
    int device = -1;
    cudaStream_t own = nullptr;   // created by the library, destroyed at thread exit
    cudaStream_t user = nullptr;  // set by zpucuda_set_stream
    bool user_set = false;
    std::string last_error;
    ~ThreadState();
};

ThreadState &ts();
// The stream a call runs on: `s` when given, else the thread's stream.
cudaStream_t resolve_stream(void *s);
// Records a CUDA failure for zpucuda_last_error and returns ZPUCUDA_ERR_CUDA.
int cuda_fail(cudaError_t e, const char *what);
int set_error(int status, const std::string &msg);
// SM count of the current device (cached per device).
int num_sms();
int current_device();

extern std::atomic<uint64_t> g_launches;
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

}  // namespace zc

#define ZC_CUDA(call)                                              \
    do {                                                           \
        cudaError_t e_ = (call);                                   \
        if (e_ != cudaSuccess) return zc::cuda_fail(e_, #call);    \
    } while (0)

// After a <<<...>>> launch: surface launch errors, count the launch.
#define ZC_LAUNCHED(what)                                          \
    do {                                                           \
        cudaError_t e_ = cudaGetLastError();                       \
        if (e_ != cudaSuccess) return zc::cuda_fail(e_, what);     \
        zc::count_launch();                                        \
    } while (0)

#define ZC_CHECK(cond, status)        \
    do {                              \
        if (!(cond)) return (status); \
    } while (0)
