// Device / thread binding, bounded sync, status strings and the refcounted
// HBM buffer (the device counterpart of src/zpu/buffer.zig:14-102).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"

namespace zc {

std::atomic<uint64_t> g_launches{0};

ThreadState::~ThreadState() {
    // The runtime may already be torn down at process exit; ignore errors.
    if (own) cudaStreamDestroy(own);
}

ThreadState &ts() {
    static thread_local ThreadState s;
    return s;
}

int set_error(int status, const std::string &msg) {
    ts().last_error = msg;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
    if (e == cudaErrorMemoryAllocation) return set_error(ZPUCUDA_ERR_OUT_OF_MEMORY, m);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver || e == cudaErrorNoKernelImageForDevice)
        return set_error(ZPUCUDA_ERR_NO_DEVICE, m);
    return set_error(ZPUCUDA_ERR_CUDA, m);
}

int current_device() {
    ThreadState &s = ts();
    if (s.device >= 0) return s.device;
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return -1;
    return d;
}

cudaStream_t resolve_stream(void *st) {
    if (st) return (cudaStream_t)st;
    ThreadState &s = ts();
    if (s.user_set) return s.user;
    if (!s.own) {
        if (s.device < 0) s.device = current_device();
        cudaStreamCreateWithFlags(&s.own, cudaStreamNonBlocking);
    }
    return s.own;
}

int num_sms() {
    static int cache[64] = {0};
    int d = current_device();
    if (d < 0 || d >= 64) return 148;
    if (!cache[d]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || v <= 0) v = 148;
        cache[d] = v;
    }
    return cache[d];
}

}  // namespace zc

using namespace zc;

extern "C" {

const char *zpucuda_status_string(int st) {
    switch (st) {
    case ZPUCUDA_OK: return "ok";
    case ZPUCUDA_ERR_OUT_OF_MEMORY: return "OutOfMemory";
    case ZPUCUDA_ERR_SHAPE_MISMATCH: return "ShapeMismatch";
    case ZPUCUDA_ERR_DTYPE_MISMATCH: return "DTypeMismatch";
    case ZPUCUDA_ERR_RANK_TOO_LARGE: return "RankTooLarge";
    case ZPUCUDA_ERR_INVALID_SHAPE: return "InvalidShape";
    case ZPUCUDA_ERR_INVALID_AXIS: return "InvalidAxis";
    case ZPUCUDA_ERR_NON_CONTIGUOUS: return "NonContiguous";
    case ZPUCUDA_ERR_INDEX_OUT_OF_RANGE: return "IndexOutOfRange";
    case ZPUCUDA_ERR_NOT_SUPPORTED: return "NotSupported";
    case ZPUCUDA_ERR_NOT_DIFFERENTIABLE: return "NotDifferentiable";
    case ZPUCUDA_ERR_NOT_POSITIVE_DEFINITE: return "NotPositiveDefinite";
    case ZPUCUDA_ERR_DEVICE_MISMATCH: return "DeviceMismatch";
    case ZPUCUDA_ERR_TIMEOUT: return "Timeout";
    case ZPUCUDA_ERR_CUDA: return "CudaError";
    case ZPUCUDA_ERR_NO_DEVICE: return "NoDevice";
    case ZPUCUDA_ERR_INVALID_ARGUMENT: return "InvalidArgument";
    default: return "unknown status";
    }
}

const char *zpucuda_last_error(void) { return ts().last_error.c_str(); }

int zpucuda_version(void) { return 100; }

uint64_t zpucuda_launch_count(void) { return g_launches.load(); }

int zpucuda_device_count(int *count) {
    ZC_CHECK(count, ZPUCUDA_ERR_INVALID_ARGUMENT);
    *count = 0;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        return ZPUCUDA_OK;
    }
    ZC_CUDA(e);
    *count = n;
    return ZPUCUDA_OK;
}

int zpucuda_thread_bind(int device) {
    int n = 0;
    int st = zpucuda_device_count(&n);
    if (st) return st;
    if (device < 0 || device >= n) return set_error(ZPUCUDA_ERR_NO_DEVICE, "no such device");
    cudaDeviceProp p;
    ZC_CUDA(cudaGetDeviceProperties(&p, device));
    if (p.major != 10) return set_error(ZPUCUDA_ERR_NO_DEVICE, "libzpucuda is built for sm_100a only");
    ZC_CUDA(cudaSetDevice(device));
    ThreadState &s = ts();
    if (s.device != device && s.own) {
        cudaStreamDestroy(s.own);
        s.own = nullptr;
    }
    s.device = device;
    if (!s.own) ZC_CUDA(cudaStreamCreateWithFlags(&s.own, cudaStreamNonBlocking));
    return ZPUCUDA_OK;
}

int zpucuda_init(int device) { return zpucuda_thread_bind(device); }

int zpucuda_get_stream(void **stream) {
    ZC_CHECK(stream, ZPUCUDA_ERR_INVALID_ARGUMENT);
    *stream = (void *)resolve_stream(nullptr);
    return ZPUCUDA_OK;
}

int zpucuda_set_stream(void *stream) {
    ThreadState &s = ts();
    s.user = (cudaStream_t)stream;
    s.user_set = stream != nullptr;
    return ZPUCUDA_OK;
}

// Bounded wait: polls the stream instead of blocking in the driver, so a
// stream that never drains turns into ZPUCUDA_ERR_TIMEOUT, not a hang.
int zpucuda_sync(int64_t timeout_ms) {
    if (timeout_ms < 0) timeout_ms = 60000;
    cudaStream_t s = resolve_stream(nullptr);
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return ZPUCUDA_OK;
        if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (ms >= timeout_ms) return set_error(ZPUCUDA_ERR_TIMEOUT, "zpucuda_sync: stream did not drain in time");
        std::this_thread::sleep_for(std::chrono::microseconds(ms < 2 ? 20 : 200));
    }
}

}  // extern "C"

// --------------------------------------------------------------------------
// Buffers
// --------------------------------------------------------------------------

struct zpucuda_buf {
    std::atomic<uint32_t> rc;
    void *ptr;
    size_t bytes;
    bool owned;
    int device;
    // residency: the host copy zpu's accessors read (Buffer.mem) when one is
    // attached, and which copies hold the current bytes
    void *host = nullptr;
    std::atomic<int> state{ZPUCUDA_RES_DEVICE};
};

// A lifetime domain for device buffers (zpu's Tracker / Scope,
// src/zpu/tensor.zig:537-664): while a scope is installed on a thread, every
// buffer that thread creates is adopted by it, and ending the scope drops
// those creation references.
struct zpucuda_scope {
    std::vector<zpucuda_buf *> list;
    bool installed = false;
};

namespace {
thread_local zpucuda_scope *t_scope = nullptr;
std::atomic<uint64_t> g_h2d_bytes{0}, g_d2h_bytes{0};

// Tracker.adopt through track() (tensor.zig:599-606): the creation reference
// goes to the thread's installed scope, if any.
void track(zpucuda_buf *b) {
    if (t_scope && t_scope->installed) t_scope->list.push_back(b);
}
// Host-side fault injection for the failure-path tests: with
// ZPUCUDA_FAULT_ALLOC_AFTER=n the (n+1)-th and later allocations fail with
// OutOfMemory before any CUDA call is made.
std::atomic<int64_t> g_alloc_count{0};
int64_t fault_alloc_after() {
    static int64_t v = [] {
        const char *e = getenv("ZPUCUDA_FAULT_ALLOC_AFTER");
        return e ? (int64_t)atoll(e) : (int64_t)-1;
    }();
    return v;
}

int alloc_impl(size_t nbytes, bool zero, zpucuda_buf **out) {
    ZC_CHECK(out, ZPUCUDA_ERR_INVALID_ARGUMENT);
    *out = nullptr;
    int64_t lim = fault_alloc_after();
    if (lim >= 0 && g_alloc_count.fetch_add(1) >= lim)
        return set_error(ZPUCUDA_ERR_OUT_OF_MEMORY, "injected allocation failure (ZPUCUDA_FAULT_ALLOC_AFTER)");
    void *p = nullptr;
    if (nbytes) {
        ZC_CUDA(cudaMalloc(&p, nbytes));  // 256-byte aligned
        if (zero) {
            cudaError_t e = cudaMemset(p, 0, nbytes);
            if (e != cudaSuccess) {
                cudaFree(p);
                return cuda_fail(e, "cudaMemset");
            }
        }
    }
    zpucuda_buf *b = new zpucuda_buf;
    b->rc.store(1);
    b->ptr = p;
    b->bytes = nbytes;
    b->owned = true;
    b->device = current_device();
    track(b);
    *out = b;
    return ZPUCUDA_OK;
}
}  // namespace

extern "C" {

int zpucuda_buf_alloc(size_t nbytes, zpucuda_buf **out) { return alloc_impl(nbytes, false, out); }
int zpucuda_buf_alloc_zeroed(size_t nbytes, zpucuda_buf **out) { return alloc_impl(nbytes, true, out); }

int zpucuda_buf_wrap(void *d_ptr, size_t nbytes, zpucuda_buf **out) {
    ZC_CHECK(out && (d_ptr || !nbytes), ZPUCUDA_ERR_INVALID_ARGUMENT);
    zpucuda_buf *b = new zpucuda_buf;
    b->rc.store(1);
    b->ptr = d_ptr;
    b->bytes = nbytes;
    b->owned = false;
    b->device = current_device();
    track(b);
    *out = b;
    return ZPUCUDA_OK;
}

zpucuda_buf *zpucuda_buf_retain(zpucuda_buf *b) {
    if (b) b->rc.fetch_add(1, std::memory_order_relaxed);
    return b;
}

void zpucuda_buf_release(zpucuda_buf *b) {
    if (!b) return;
    if (b->rc.fetch_sub(1, std::memory_order_acq_rel) == 1) {
        if (b->owned && b->ptr) cudaFree(b->ptr);
        delete b;
    }
}

uint32_t zpucuda_buf_refcount(const zpucuda_buf *b) { return b ? b->rc.load() : 0; }
void *zpucuda_buf_devptr(const zpucuda_buf *b) { return b ? b->ptr : nullptr; }
size_t zpucuda_buf_bytes(const zpucuda_buf *b) { return b ? b->bytes : 0; }

int zpucuda_buf_upload(zpucuda_buf *b, size_t off, const void *host, size_t nbytes) {
    ZC_CHECK(b && (host || !nbytes), ZPUCUDA_ERR_INVALID_ARGUMENT);
    ZC_CHECK(off <= b->bytes && nbytes <= b->bytes - off, ZPUCUDA_ERR_INDEX_OUT_OF_RANGE);
    if (!nbytes) return ZPUCUDA_OK;
    cudaStream_t s = resolve_stream(nullptr);
    ZC_CUDA(cudaMemcpyAsync((char *)b->ptr + off, host, nbytes, cudaMemcpyHostToDevice, s));
    g_h2d_bytes += nbytes;
    return zpucuda_sync(-1);
}

int zpucuda_buf_download(const zpucuda_buf *b, size_t off, void *host, size_t nbytes) {
    ZC_CHECK(b && (host || !nbytes), ZPUCUDA_ERR_INVALID_ARGUMENT);
    ZC_CHECK(off <= b->bytes && nbytes <= b->bytes - off, ZPUCUDA_ERR_INDEX_OUT_OF_RANGE);
    if (!nbytes) return ZPUCUDA_OK;
    cudaStream_t s = resolve_stream(nullptr);
    ZC_CUDA(cudaMemcpyAsync(host, (const char *)b->ptr + off, nbytes, cudaMemcpyDeviceToHost, s));
    g_d2h_bytes += nbytes;
    return zpucuda_sync(-1);
}

// ------------------------------------------------------------- residency

int zpucuda_buf_attach_host(zpucuda_buf *b, void *host, int state) {
    ZC_CHECK(b && (host || !b->bytes), ZPUCUDA_ERR_INVALID_ARGUMENT);
    ZC_CHECK(state == ZPUCUDA_RES_DEVICE || state == ZPUCUDA_RES_HOST || state == ZPUCUDA_RES_BOTH,
             ZPUCUDA_ERR_INVALID_ARGUMENT);
    b->host = host;
    b->state.store(state);
    return ZPUCUDA_OK;
}

int zpucuda_buf_residency(const zpucuda_buf *b, int *state) {
    ZC_CHECK(b && state, ZPUCUDA_ERR_INVALID_ARGUMENT);
    *state = b->state.load();
    return ZPUCUDA_OK;
}

int zpucuda_buf_mark_device_dirty(zpucuda_buf *b) {
    ZC_CHECK(b, ZPUCUDA_ERR_INVALID_ARGUMENT);
    b->state.store(ZPUCUDA_RES_DEVICE);
    return ZPUCUDA_OK;
}

int zpucuda_buf_mark_host_dirty(zpucuda_buf *b) {
    ZC_CHECK(b, ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (!b->host) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "zpucuda_buf_mark_host_dirty: no host copy attached");
    b->state.store(ZPUCUDA_RES_HOST);
    return ZPUCUDA_OK;
}

int zpucuda_buf_host_sync(zpucuda_buf *b, void *stream) {
    ZC_CHECK(b, ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (!b->host) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "zpucuda_buf_host_sync: no host copy attached");
    if (b->state.load() != ZPUCUDA_RES_DEVICE) return ZPUCUDA_OK;  // the host copy is current
    cudaStream_t s = resolve_stream(stream);
    if (b->bytes) ZC_CUDA(cudaMemcpyAsync(b->host, b->ptr, b->bytes, cudaMemcpyDeviceToHost, s));
    g_d2h_bytes += b->bytes;
    // bounded wait on that stream: the host reads the bytes right after
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60))
            return set_error(ZPUCUDA_ERR_TIMEOUT, "zpucuda_buf_host_sync: stream did not drain in time");
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    b->state.store(ZPUCUDA_RES_BOTH);
    return ZPUCUDA_OK;
}

int zpucuda_buf_device_sync(zpucuda_buf *b, void *stream) {
    ZC_CHECK(b, ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (b->state.load() != ZPUCUDA_RES_HOST) return ZPUCUDA_OK;  // the device copy is current
    cudaStream_t s = resolve_stream(stream);
    if (b->bytes) ZC_CUDA(cudaMemcpyAsync(b->ptr, b->host, b->bytes, cudaMemcpyHostToDevice, s));
    g_h2d_bytes += b->bytes;
    b->state.store(ZPUCUDA_RES_BOTH);
    return ZPUCUDA_OK;
}

int zpucuda_buf_transfer_stats(uint64_t *h2d_bytes, uint64_t *d2h_bytes) {
    ZC_CHECK(h2d_bytes && d2h_bytes, ZPUCUDA_ERR_INVALID_ARGUMENT);
    *h2d_bytes = g_h2d_bytes.load();
    *d2h_bytes = g_d2h_bytes.load();
    return ZPUCUDA_OK;
}

// ----------------------------------------------------------------- scopes

int zpucuda_scope_begin(zpucuda_scope **out) {
    ZC_CHECK(out, ZPUCUDA_ERR_INVALID_ARGUMENT);
    zpucuda_scope *sc = new zpucuda_scope;
    if (!t_scope) {  // Tracker.begin: installs only when no other scope is active
        t_scope = sc;
        sc->installed = true;
    }
    *out = sc;
    return ZPUCUDA_OK;
}

int zpucuda_scope_end(zpucuda_scope *sc) {
    ZC_CHECK(sc, ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (sc->installed) {
        if (t_scope == sc) t_scope = nullptr;
        for (zpucuda_buf *b : sc->list) zpucuda_buf_release(b);
        sc->list.clear();
        sc->installed = false;
    }
    delete sc;
    return ZPUCUDA_OK;
}

zpucuda_buf *zpucuda_scope_keep(zpucuda_scope *sc, zpucuda_buf *b) {
    (void)sc;
    return zpucuda_buf_retain(b);
}

int zpucuda_scope_forget(zpucuda_scope *sc, zpucuda_buf *b) {
    ZC_CHECK(sc && b, ZPUCUDA_ERR_INVALID_ARGUMENT);
    for (size_t i = 0; i < sc->list.size(); i++)
        if (sc->list[i] == b) {
            sc->list[i] = sc->list.back();
            sc->list.pop_back();
            return ZPUCUDA_OK;
        }
    return ZPUCUDA_OK;
}

int64_t zpucuda_scope_count(const zpucuda_scope *sc) { return sc ? (int64_t)sc->list.size() : -1; }

int zpucuda_scope_installed(const zpucuda_scope *sc) { return sc && sc->installed ? 1 : 0; }

}  // extern "C"
