// NCCL communicators for the data-parallel MLP step.
//
// The reference has no multi-device code: its MLP step runs on one CPU
// (src/zpu/transforms.zig:87-148, src/zpu/optim.zig:183-259).  Here each GPU
// is driven by its own process (or thread), the gradients of the step are
// summed across GPUs with ncclAllReduce over NVLink, and this file owns the
// one communicator per device.
//
// libnccl.so.2 is opened at run time (dlopen) on the first call, so the
// library loads and runs single-GPU work on machines without NCCL; when the
// process already holds NCCL (PyTorch loads its own copy) the loader returns
// that copy.  Communicators are created non-blocking so that a rank that never
// joins turns into ZPUCUDA_ERR_TIMEOUT after `timeout_ms` instead of a hang;
// the communicator is then aborted.
#include <dlfcn.h>
#include <string.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "common.cuh"
#include "nccl.cuh"

namespace zc {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*reduce_scatter)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                   cudaStream_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*abort)(ncclComm_t);
    ncclResult_t (*finalize)(ncclComm_t);
    ncclResult_t (*destroy)(ncclComm_t);
    const char *(*error_string)(ncclResult_t);
    ncclResult_t (*version)(int *);
};

NcclApi g_api;
int g_api_status = -1;
std::mutex g_mu;

constexpr int kMaxDevices = 64;
struct Comm {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
};
Comm g_comms[kMaxDevices];

int load_api() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_api_status >= 0) return g_api_status;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        g_api_status = set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "libnccl.so.2 could not be loaded");
        return g_api_status;
    }
    bool ok = true;
    auto sym = [&](const char *name) {
        void *p = dlsym(h, name);
        if (!p) ok = false;
        return p;
    };
    g_api.get_unique_id = (decltype(g_api.get_unique_id))sym("ncclGetUniqueId");
    g_api.init_rank_config = (decltype(g_api.init_rank_config))sym("ncclCommInitRankConfig");
    g_api.async_error = (decltype(g_api.async_error))sym("ncclCommGetAsyncError");
    g_api.all_reduce = (decltype(g_api.all_reduce))sym("ncclAllReduce");
    g_api.reduce_scatter = (decltype(g_api.reduce_scatter))sym("ncclReduceScatter");
    g_api.all_gather = (decltype(g_api.all_gather))sym("ncclAllGather");
    g_api.abort = (decltype(g_api.abort))sym("ncclCommAbort");
    g_api.finalize = (decltype(g_api.finalize))sym("ncclCommFinalize");
    g_api.destroy = (decltype(g_api.destroy))sym("ncclCommDestroy");
    g_api.error_string = (decltype(g_api.error_string))sym("ncclGetErrorString");
    g_api.version = (decltype(g_api.version))sym("ncclGetVersion");
    g_api_status = ok ? ZPUCUDA_OK : set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "libnccl.so.2 lacks a needed symbol");
    return g_api_status;
}

int nccl_fail(ncclResult_t r, const char *what) {
    std::string m = std::string(what) + ": " + (g_api.error_string ? g_api.error_string(r) : "nccl error");
    return set_error(r == ncclInvalidArgument || r == ncclInvalidUsage ? ZPUCUDA_ERR_INVALID_ARGUMENT
                                                                       : ZPUCUDA_ERR_CUDA,
                     m);
}

// Polls a non-blocking communicator until its pending operation settles.
int settle(ncclComm_t c, int64_t timeout_ms, const char *what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = g_api.async_error(c, &st);
        if (r != ncclSuccess) return nccl_fail(r, what);
        if (st == ncclSuccess) return ZPUCUDA_OK;
        if (st != ncclInProgress) return nccl_fail(st, what);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
        if (timeout_ms >= 0 && ms.count() > timeout_ms)
            return set_error(ZPUCUDA_ERR_TIMEOUT, std::string(what) + ": timed out");
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

}  // namespace

int nccl_world(int *rank) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices || !g_comms[dev].comm) {
        if (rank) *rank = 0;
        return 1;
    }
    if (rank) *rank = g_comms[dev].rank;
    return g_comms[dev].world;
}

int nccl_allreduce_sum_f32(float *d, int64_t count, cudaStream_t s) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices || !g_comms[dev].comm)
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "no NCCL communicator on this device (zpucuda_nccl_init)");
    if (count <= 0) return ZPUCUDA_OK;
    ncclComm_t c = g_comms[dev].comm;
    ncclResult_t r = g_api.all_reduce(d, d, (size_t)count, ncclFloat32, ncclSum, c, s);
    if (r == ncclInProgress) return settle(c, 60000, "ncclAllReduce");
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    return ZPUCUDA_OK;
}

// In-place reduce-scatter: d holds world * count floats; this rank's summed
// block lands at d + rank * count.
int nccl_reduce_scatter_sum_f32(float *d, int64_t count, cudaStream_t s) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices || !g_comms[dev].comm)
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "no NCCL communicator on this device (zpucuda_nccl_init)");
    if (count <= 0) return ZPUCUDA_OK;
    ncclComm_t c = g_comms[dev].comm;
    ncclResult_t r = g_api.reduce_scatter(d, d + (int64_t)g_comms[dev].rank * count, (size_t)count, ncclFloat32,
                                          ncclSum, c, s);
    if (r == ncclInProgress) return settle(c, 60000, "ncclReduceScatter");
    if (r != ncclSuccess) return nccl_fail(r, "ncclReduceScatter");
    return ZPUCUDA_OK;
}

// In-place all-gather: every rank's block d + rank * count goes to all.
int nccl_all_gather_f32(float *d, int64_t count, cudaStream_t s) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices || !g_comms[dev].comm)
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "no NCCL communicator on this device (zpucuda_nccl_init)");
    if (count <= 0) return ZPUCUDA_OK;
    ncclComm_t c = g_comms[dev].comm;
    ncclResult_t r = g_api.all_gather(d + (int64_t)g_comms[dev].rank * count, d, (size_t)count, ncclFloat32, c, s);
    if (r == ncclInProgress) return settle(c, 60000, "ncclAllGather");
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return ZPUCUDA_OK;
}

}  // namespace zc

using namespace zc;

extern "C" int zpucuda_nccl_unique_id(uint8_t *id) {
    if (!id) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "id is NULL");
    int st = load_api();
    if (st) return st;
    ncclUniqueId u;
    ncclResult_t r = g_api.get_unique_id(&u);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(u) == ZPUCUDA_NCCL_ID_BYTES, "ncclUniqueId size");
    memcpy(id, &u, sizeof u);
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_nccl_init(int rank, int world, const uint8_t *id, int64_t timeout_ms) {
    if (!id || world < 1 || rank < 0 || rank >= world)
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "nccl_init: bad rank/world/id");
    int st = load_api();
    if (st) return st;
    const int dev = current_device();
    if (dev < 0) return set_error(ZPUCUDA_ERR_NO_DEVICE, "nccl_init: no device bound");
    if (dev >= kMaxDevices) return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "nccl_init: device index too large");
    if (g_comms[dev].comm) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "nccl_init: device already has a communicator");
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t c = nullptr;
    ncclResult_t r = g_api.init_rank_config(&c, world, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclCommInitRankConfig");
    st = settle(c, timeout_ms, "ncclCommInitRankConfig");
    if (st) {
        if (c) g_api.abort(c);
        return st;
    }
    g_comms[dev].comm = c;
    g_comms[dev].rank = rank;
    g_comms[dev].world = world;
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_nccl_allreduce_f32(float *d_buf, int64_t count, void *stream) {
    if (count < 0 || (count > 0 && !d_buf)) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "allreduce: bad buffer");
    return nccl_allreduce_sum_f32(d_buf, count, resolve_stream(stream));
}

extern "C" int zpucuda_nccl_world(int *rank, int *world) {
    int r = 0;
    const int w = nccl_world(&r);
    if (rank) *rank = r;
    if (world) *world = w;
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_nccl_destroy(int64_t timeout_ms) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices || !g_comms[dev].comm) return ZPUCUDA_OK;
    ncclComm_t c = g_comms[dev].comm;
    g_comms[dev] = Comm{};
    ncclResult_t r = g_api.finalize(c);
    int st = ZPUCUDA_OK;
    if (r == ncclSuccess || r == ncclInProgress) st = settle(c, timeout_ms, "ncclCommFinalize");
    else st = nccl_fail(r, "ncclCommFinalize");
    if (st) {
        g_api.abort(c);
        return st;
    }
    r = g_api.destroy(c);
    return r == ncclSuccess ? ZPUCUDA_OK : nccl_fail(r, "ncclCommDestroy");
}
