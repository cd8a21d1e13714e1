// Fused element-wise + reduction regions: the program format shared by the
// jit-plan lowering (plan.cu) and the kernels (region.cu), and the templated
// straight-line kernel that gen_regions.py instantiates per catalogued region.
//
// What a region computes is fixed by zpu's step semantics: every element-wise
// step rounds to the element type on its own (src/zpu/ops.zig:297-345,
// scalar.zig:262-302), a full `sum` reduces everything (ops.zig:820-869).
// What changes is where it runs: one kernel per region, every element read
// once from HBM with 128-bit loads, intermediates kept in registers, the sum
// accumulated in f64 per thread and per block, and the blocks combined by the
// last block to finish (no spin-waits, deterministic order).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace zc {

constexpr int RP_MAX_INSN = 48;
constexpr int RP_MAX_IN = 8;
constexpr int RP_MAX_OUT = 4;
constexpr int RP_MAX_REG = 32;
constexpr int RP_MAX_RANK = 8;

enum : int8_t { IN_FULL = 0, IN_SCALAR = 1, IN_ROW = 2, IN_GENERAL = 3 };
enum : int32_t { RED_NONE = 0, RED_SUM = 1, RED_PROD = 2, RED_MAX = 3, RED_MIN = 4 };
enum : uint8_t { OPC_LOAD = 250 };

struct Insn {
    uint8_t op;  // prims.Prim code, or OPC_LOAD
    uint8_t dst, a, b;
};

// One lowered region.  Loads come first (r0..r(n_in-1)), then one register
// per element-wise step, in step order.
struct RegionProgram {
    int32_t dtype;  // ZPUCUDA_F32 / ZPUCUDA_F64
    int32_t n_insn;
    Insn insn[RP_MAX_INSN];
    int32_t n_in;
    int8_t in_kind[RP_MAX_IN];
    int64_t in_numel[RP_MAX_IN];  // IN_ROW: length of the broadcast row
    int32_t rank;
    int64_t dims[RP_MAX_RANK];                  // the region's shape
    int64_t in_strides[RP_MAX_IN][RP_MAX_RANK];  // IN_GENERAL: per-axis strides (0 = broadcast)
    int64_t numel;
    int64_t outer;       // rows of a row reduction (numel / inner; set even when inner == 0)
    int32_t reduce;      // RED_*
    int32_t reduce_all;  // 1: all axes -> 1 value; 0: last axis -> numel / inner values
    int64_t inner;       // last-axis length for row reductions
    int32_t reduce_reg;
    int32_t n_out;  // element-wise outputs written to HBM
    int32_t out_reg[RP_MAX_OUT];
};

// Launch-time arguments of a region kernel.
struct RegionIO {
    const void *in[RP_MAX_IN];
    void *out[RP_MAX_OUT];  // element-wise outputs
    void *red_out;          // reduced output (numel/inner values, or 1)
    double *partials;       // one per block (full reductions)
    unsigned int *ticket;   // zero between launches
};

// Scratch a full reduction needs: a ticket word plus one double per block.
constexpr int kMaxRegionBlocks = 148 * 16;
constexpr size_t kRegionWorkspaceBytes = 256 + sizeof(double) * kMaxRegionBlocks;

typedef int (*FusedLaunch)(const RegionProgram &p, const RegionIO &io, cudaStream_t s);
struct CatalogueEntry {
    const char *signature;
    const char *name;
    FusedLaunch launch;
};

// The f32 tanh the fused kernels use: CUDA's tanhf, whose documented error
// bound (2 ulp) keeps a catalogued region within 2 ulp of zpu's
// f64-then-round tanh plus the latter's half ulp.
__device__ __forceinline__ float zc_tanhf(float x) { return tanhf(x); }

// ---------------------------------------------------------------- reduction

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide sum of `v` (all threads call); the result is valid in thread 0.
template <int THREADS>
__device__ __forceinline__ double block_sum(double v) {
    __shared__ double red[THREADS / 32];
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        v = lane < THREADS / 32 ? red[lane] : 0.0;
        v = warp_sum(v);
    }
    return v;
}

// Publishes this block's partial and lets the last block to arrive fold all
// partials in block order (deterministic) and write the result.  No block
// waits on another: the ticket only decides who finishes.
template <int THREADS>
__device__ __forceinline__ void finish_full_sum(double block_total, const RegionIO &io, bool f64_out) {
    __shared__ bool last;
    if (threadIdx.x == 0) {
        io.partials[blockIdx.x] = block_total;
        __threadfence();
        const unsigned t = atomicAdd(io.ticket, 1u);
        last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    double v = 0.0;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += THREADS) v += __ldcg(io.partials + i);
    v = block_sum<THREADS>(v);
    if (threadIdx.x == 0) {
        if (f64_out) *(double *)io.red_out = v;
        else *(float *)io.red_out = (float)v;
        *io.ticket = 0u;  // ready for the next launch
    }
}

// ------------------------------------------------- catalogued f32 regions
//
// F::call(v) is the region's straight-line code on one element; v holds the
// region's inputs (full tensors element i, scalars their single value).

constexpr int kFusedThreads = 256;
constexpr int kFusedUnroll = 4;  // 16-byte loads in flight per thread per input

template <class F, bool SUM>
__global__ void __launch_bounds__(kFusedThreads) fused_f32_kernel(const __grid_constant__ RegionIO io, int64_t n) {
    constexpr int NIN = F::NIN;
    float sv[NIN > 0 ? NIN : 1];
#pragma unroll
    for (int k = 0; k < NIN; k++)
        if (F::SCALARS & (1u << k)) sv[k] = __ldg((const float *)io.in[k]);

    const int64_t n4 = n >> 2;
    const int64_t G = (int64_t)gridDim.x * kFusedThreads;
    double acc = 0.0;
    for (int64_t base = (int64_t)blockIdx.x * kFusedThreads + threadIdx.x; base < n4; base += kFusedUnroll * G) {
        float4 v[kFusedUnroll][NIN > 0 ? NIN : 1];
#pragma unroll
        for (int u = 0; u < kFusedUnroll; u++) {
            const int64_t q = base + u * G;
#pragma unroll
            for (int k = 0; k < NIN; k++)
                if (!(F::SCALARS & (1u << k)))
                    v[u][k] = q < n4 ? __ldcs((const float4 *)io.in[k] + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kFusedUnroll; u++) {
            const int64_t q = base + u * G;
            if (q >= n4) break;
            float y[4];
#pragma unroll
            for (int l = 0; l < 4; l++) {
                float e[NIN > 0 ? NIN : 1];
#pragma unroll
                for (int k = 0; k < NIN; k++) {
                    if (F::SCALARS & (1u << k)) e[k] = sv[k];
                    else e[k] = l == 0 ? v[u][k].x : l == 1 ? v[u][k].y : l == 2 ? v[u][k].z : v[u][k].w;
                }
                y[l] = F::call(e);
            }
            if (SUM) {
                acc += (double)((y[0] + y[1]) + (y[2] + y[3]));
            } else {
                __stcs((float4 *)io.out[0] + q, make_float4(y[0], y[1], y[2], y[3]));
            }
        }
    }
    // the n % 4 leftover elements
    const int64_t t = (int64_t)blockIdx.x * kFusedThreads + threadIdx.x;
    if (t < (n & 3)) {
        const int64_t i = (n4 << 2) + t;
        float e[NIN > 0 ? NIN : 1];
#pragma unroll
        for (int k = 0; k < NIN; k++) e[k] = (F::SCALARS & (1u << k)) ? sv[k] : ((const float *)io.in[k])[i];
        const float y = F::call(e);
        if (SUM) acc += (double)y;
        else ((float *)io.out[0])[i] = y;
    }
    if (SUM) {
        const double b = block_sum<kFusedThreads>(acc);
        finish_full_sum<kFusedThreads>(b, io, false);
    }
}

// Grid of the fused kernels: every SM full, one wave (grid-stride loop).
int fused_grid(const void *kernel, int threads, size_t smem);

template <class F, bool SUM>
int launch_fused_f32(const RegionProgram &p, const RegionIO &io, cudaStream_t s) {
    auto k = fused_f32_kernel<F, SUM>;
    int grid = fused_grid((const void *)k, kFusedThreads, 0);
    if (SUM && grid > kMaxRegionBlocks) grid = kMaxRegionBlocks;
    k<<<grid, kFusedThreads, 0, s>>>(io, p.numel);
    ZC_LAUNCHED("fused region kernel");
    return ZPUCUDA_OK;
}

// The lookup the lowering uses: nullptr when `sig` is not catalogued.
const CatalogueEntry *catalogue_find(const char *sig);
// Runs a lowered region: the catalogued kernel when there is one (and the
// inputs are 16-byte aligned), the bytecode kernel otherwise.
int region_launch(const RegionProgram &p, const CatalogueEntry *cat, const RegionIO &io, cudaStream_t s);

}  // namespace zc
