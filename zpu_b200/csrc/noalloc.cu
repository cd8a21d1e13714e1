// A variant of the fused jit-chain reduction that allocates nothing.
//
// The regular path (zpucuda_plan_create / zpucuda_plan_run) allocates the
// reduction's scratch -- a ticket word, an error word and one f64 partial per
// block -- with cudaMalloc when the plan is built.  Some callers cannot do
// that: an application that embeds this library inside a framework whose
// caching allocator owns all device memory (a side allocation would escape
// its accounting and its memory limit), or a latency-critical loop where
// cudaMalloc's implicit device-wide synchronisation is not allowed.  For them
// this entry point keeps the scratch in a fixed file-scope __device__ array
// instead, so a call needs no allocation at all; the caller passes inputs and
// outputs as usual.
#include <string.h>

#include <mutex>
#include <string>

#include "region.cuh"
#include "regions_gen.cuh"

namespace zc {
namespace {

// The static scratch: 256 bytes of header (ticket at word 0, error word at
// word 1) and room for kNoAllocMaxBlocks f64 block partials: 16.25 KiB,
// held by every GPU that loads the library until the process exits.
constexpr int kNoAllocMaxBlocks = 2048;
constexpr size_t kNoAllocHeader = 256;
constexpr size_t kNoAllocBytes = kNoAllocHeader + sizeof(double) * kNoAllocMaxBlocks;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory: the device address is looked up once per device, with that device
// current, and cached.
std::mutex g_scratch_mu;
void *g_scratch_addr[64] = {nullptr};

int scratch_address(void **out) {
    int dev = 0;
    ZC_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(ZPUCUDA_ERR_NO_DEVICE, "device ordinal out of range");
    std::lock_guard<std::mutex> g(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "cudaGetSymbolAddress(noalloc scratch)");
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return ZPUCUDA_OK;
}

}  // namespace
}  // namespace zc

using namespace zc;

extern "C" int zpucuda_chain_tanh_sq_affine_sum_noalloc(const float *d_x, int64_t n, const float *d_a,
                                                        const float *d_b, float *d_out, void *stream) {
    ZC_CHECK(n >= 0 && d_a && d_b && d_out && (d_x || n == 0), ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (((uintptr_t)d_x & 15u) != 0)
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "zpucuda_chain_tanh_sq_affine_sum_noalloc: d_x must be 16-byte aligned");
    const int grid = fused_grid<Region_tanh_sq_affine, true>();
    if (grid > kNoAllocMaxBlocks)
        return set_error(ZPUCUDA_ERR_NOT_SUPPORTED,
                         "zpucuda_chain_tanh_sq_affine_sum_noalloc: this launch needs " + std::to_string(grid) +
                             " block partials but the static scratch holds " + std::to_string(kNoAllocMaxBlocks));
    void *ws = nullptr;
    int st = scratch_address(&ws);
    if (st) return st;
    cudaStream_t s = resolve_stream(stream);
    // the ticket and error words must start at zero; the partials are
    // written by their blocks before they are read
    ZC_CUDA(cudaMemsetAsync(ws, 0, 2 * sizeof(unsigned int), s));
    RegionIO io;
    memset(&io, 0, sizeof io);
    io.in[0] = d_x;
    io.in[1] = d_a;
    io.in[2] = d_b;
    io.red_out = d_out;
    io.ticket = (unsigned int *)ws;
    io.error = (unsigned int *)ws + 1;
    io.partials = (double *)((char *)ws + kNoAllocHeader);
    RegionProgram p;
    memset(&p, 0, sizeof p);
    p.dtype = ZPUCUDA_F32;
    p.numel = n;
    return launch_fused_f32<Region_tanh_sq_affine, true, false>(p, io, s);
}
