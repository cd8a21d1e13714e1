// Fused element-wise + reduction regions: the program format shared by the
// jit-plan lowering (plan.cu) and the kernels (region.cu), and the templated
// straight-line kernels that gen_regions.py instantiates per catalogued region.
//
// What a region computes is fixed by zpu's step semantics: every element-wise
// step rounds to the element type on its own (src/zpu/ops.zig:297-345,
// scalar.zig:262-302), a full `sum` reduces everything (ops.zig:820-869).
// What changes is where it runs: one kernel per region, every element read
// once from HBM with 128-bit loads, intermediates kept in registers, the sum
// accumulated per thread and per block in f64, and the blocks combined by the
// last block to finish (no spin-waits between blocks, deterministic order).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace zc {

constexpr int RP_MAX_INSN = 48;
constexpr int RP_MAX_IN = 8;
constexpr int RP_MAX_OUT = 16;
constexpr int RP_MAX_REG = 32;
constexpr int RP_MAX_RANK = 8;

enum : int8_t { IN_FULL = 0, IN_SCALAR = 1, IN_ROW = 2, IN_GENERAL = 3 };
enum : int32_t {
    RED_NONE = 0, RED_SUM = 1, RED_PROD = 2, RED_MAX = 3, RED_MIN = 4, RED_ARGMAX = 5, RED_ARGMIN = 6,
    RED_ANY = 7, RED_ALL = 8,  // bool results (ops.reduceBoolKernel)
    // i64 reductions in the integer type (ops.reduceStep, ops.zig:686-700):
    // wrapping sum / product, max / min; the register holds i64 bits
    RED_ISUM = 9, RED_IPROD = 10, RED_IMAX = 11, RED_IMIN = 12
};
inline __host__ __device__ bool red_is_int(int r) { return r >= RED_ISUM && r <= RED_IMIN; }
enum : uint8_t {
    // Only in 64-bit-word regions (RegionProgram::words64), where an i64
    // value's register holds its two's-complement bits and every other
    // value's register an f64 number:
    OPC_I2F = 230,   // i64 bits -> f64 (readAtF64: @floatFromInt, round to nearest)
    OPC_F2I = 231,   // f64 -> i64 bits (scalar.fromF64: 0 for NaN, clamp, truncate)
    OPC_R32 = 232,   // f64 -> the nearest f32 (writeF64 into an f32 tensor)
    // scalar.binary / scalar.unary of i64 values (scalar.zig:262-302): the
    // integer operations zpu performs on the integers themselves
    OPC_IADD = 233, OPC_ISUB = 234, OPC_IMUL = 235, OPC_IMOD = 236, OPC_IMAX = 237, OPC_IMIN = 238,
    OPC_IABS = 239, OPC_ISIGN = 240, OPC_IRELU = 241,
    // std.math.pow(f64) step for step (zpu's pow of two i64 values)
    OPC_ZPOW = 242,
    OPC_LOAD = 250,
};
// Insn.c of a prim op in a 64-bit-word region: 1 = the step's type is f32 and
// all its operands are f32 / bool, so it computes as an f32 region does and
// the result (exact in f64) is widened back.
constexpr uint8_t kInsnF32 = 1;

struct Insn {
    uint8_t op;  // prims.Prim code, or OPC_*
    uint8_t dst, a, b, c;  // c: the third operand of `where`, else the kInsnF32 flag
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
    int32_t reduce_all;  // 1: all axes -> 1 value; 0: one axis (below)
    int64_t inner;       // last-axis length for row reductions; axes after the reduced one (reduce_mid)
    int32_t reduce_mid;  // 1: the reduced axis is not the last: [outer, red_len, inner] -> [outer, inner]
    int64_t red_len;     // length of that axis
    int32_t reduce_reg;
    int32_t n_out;  // element-wise outputs written to HBM
    int32_t out_reg[RP_MAX_OUT];
    // Bool values (predicates, zpu's one-byte DType.bool) ride in the
    // region's float registers as 0 / 1: bool inputs load a byte, bool
    // outputs store (v != 0) as a byte.
    uint8_t in_bool[RP_MAX_IN];
    uint8_t out_bool[RP_MAX_OUT];
    // A region that holds an i64 value (an argmax / argmin result, an i64
    // argument, a step of i64 values) runs on 64-bit registers: i64 values
    // as their bits (loaded, computed and stored as integers), the rest as
    // f64 numbers; f32 steps keep f32 arithmetic (kInsnF32) and f32 results
    // computed in f64 round to f32 (OPC_R32).  `dtype` is then the storage
    // type of the region's float inputs and outputs.
    int32_t words64;
    uint8_t in_i64[RP_MAX_IN];
    uint8_t out_i64[RP_MAX_OUT];
};

// Launch-time arguments of a region kernel.
struct RegionIO {
    const void *in[RP_MAX_IN];
    void *out[RP_MAX_OUT];  // element-wise outputs
    void *red_out;          // reduced output (numel/inner values, or 1)
    double *partials;       // one per block (full reductions)
    unsigned int *ticket;   // zero between launches
    unsigned int *error;    // set (never cleared by a kernel) when a bounded wait runs out
};

// Scratch a full reduction needs: a ticket word, an error word, then one
// double per block (an arg reduction uses three arrays of kMaxRegionBlocks
// 8-byte words: best value, index, leading-NaN flag).
constexpr int kMaxRegionBlocks = 148 * 16;
constexpr size_t kRegionWorkspaceBytes = 256 + 3 * sizeof(double) * kMaxRegionBlocks;

typedef int (*FusedLaunch)(const RegionProgram &p, const RegionIO &io, cudaStream_t s);
struct CatalogueEntry {
    const char *signature;
    const char *name;
    FusedLaunch launch;
};

// ------------------------------------------------------ packed f32 pairs
//
// sm_100 executes f32x2 add / sub / mul / fma as one instruction on a
// 64-bit register pair, each lane an ordinary IEEE round-to-nearest f32
// operation: the same bits as two scalar __fadd_rn / __fmul_rn / fmaf, at
// half the issue slots.  Catalogued regions evaluate two elements at a time.
typedef unsigned long long f2_t;
__device__ __forceinline__ f2_t pk2(float a, float b) {
    f2_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(f2_t r, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ f2_t add2(f2_t a, f2_t b) {
    f2_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f2_t sub2(f2_t a, f2_t b) {
    f2_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f2_t mul2(f2_t a, f2_t b) {
    f2_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f2_t fma2(f2_t a, f2_t b, f2_t c) {
    f2_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f2_t splat2(float a) { return pk2(a, a); }

// ------------------------------------------------------------------ tanh
//
// The f32 tanh of the catalogued regions, written for this library (zpu
// computes tanh in f64 and rounds, src/zpu/scalar.zig:199,262-266):
//   |x| <  0.9:  tanh(x) = x + x z P(z), z = x^2, P a degree-5 minimax
//                polynomial for (tanh(x)/x - 1)/z on [0, 0.9] (0.27 ulp;
//                coefficients from fit_tanh.py: Lawson-weighted least squares
//                on the relative error, f32-rounded coefficients);
//   |x| >= 0.9:  tanh(x) = 1 - 2 / (1 + e^(2|x|)), e^(2|x|) = 2^(2 log2(e) |x|)
//                and 1/(1 + e) from the SFU (ex2.approx, rcp.approx).  There
//                the quotient is <= 0.29, so the SFU's ~2^-22 relative errors
//                move the result by under one ulp; ex2 overflows to inf for
//                huge |x| and the result is exactly 1.
// Both branches run and a select picks one (no divergence); NaN fails the
// `< 0.9` test and propagates through ex2.  Measured exhaustively on the B200
// over every f32 in [FLT_MIN, 10] against (float)tanh((double)x): max 1 ulp.
// This form keeps the FMA pipe light; its limit is the SFU (two ops per
// element).  A polynomial exponential (one SFU op) or a polynomial for
// 2/(1 + e^-2x) trades that for more issue slots than it saves: both measured
// slower on the B200.
#define ZC_TANH_P0 -3.333321214e-01f
#define ZC_TANH_P1 1.333034933e-01f
#define ZC_TANH_P2 -5.372043326e-02f
#define ZC_TANH_P3 2.090060711e-02f
#define ZC_TANH_P4 -6.855268497e-03f
#define ZC_TANH_P5 1.301668934e-03f
#define ZC_TANH_SPLIT 0.9f
#define ZC_TWO_LOG2E 2.8853900817779268f

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// tanh of a value known to be >= 0 or NaN (e.g. a square).
__device__ __forceinline__ float zc_tanh_nonneg(float ax) {
    const float z = __fmul_rn(ax, ax);
    float p = fmaf(ZC_TANH_P5, z, ZC_TANH_P4);
    p = fmaf(p, z, ZC_TANH_P3);
    p = fmaf(p, z, ZC_TANH_P2);
    p = fmaf(p, z, ZC_TANH_P1);
    p = fmaf(p, z, ZC_TANH_P0);
    const float small = fmaf(__fmul_rn(ax, z), p, ax);
    const float e = ex2_approx(__fmul_rn(ax, ZC_TWO_LOG2E));
    const float large = fmaf(-2.0f, rcp_approx(__fadd_rn(e, 1.0f)), 1.0f);
    return ax < ZC_TANH_SPLIT ? small : large;
}
__device__ __forceinline__ float zc_tanhf(float x) { return copysignf(zc_tanh_nonneg(fabsf(x)), x); }

// The same computation on a pair; every lane gives the scalar version's bits.
__device__ __forceinline__ f2_t zc_tanh_nonneg2(f2_t ax) {
    const f2_t z = mul2(ax, ax);
    f2_t p = fma2(splat2(ZC_TANH_P5), z, splat2(ZC_TANH_P4));
    p = fma2(p, z, splat2(ZC_TANH_P3));
    p = fma2(p, z, splat2(ZC_TANH_P2));
    p = fma2(p, z, splat2(ZC_TANH_P1));
    p = fma2(p, z, splat2(ZC_TANH_P0));
    const f2_t small = fma2(mul2(ax, z), p, ax);
    float g0, g1;
    upk2(mul2(ax, splat2(ZC_TWO_LOG2E)), g0, g1);
    float d0, d1;
    upk2(add2(pk2(ex2_approx(g0), ex2_approx(g1)), splat2(1.0f)), d0, d1);
    const f2_t large = fma2(splat2(-2.0f), pk2(rcp_approx(d0), rcp_approx(d1)), splat2(1.0f));
    float a0, a1, s0, s1, l0, l1;
    upk2(ax, a0, a1);
    upk2(small, s0, s1);
    upk2(large, l0, l1);
    return pk2(a0 < ZC_TANH_SPLIT ? s0 : l0, a1 < ZC_TANH_SPLIT ? s1 : l1);
}
__device__ __forceinline__ f2_t zc_tanh2(f2_t x) {
    float x0, x1;
    upk2(x, x0, x1);
    float t0, t1;
    upk2(zc_tanh_nonneg2(pk2(fabsf(x0), fabsf(x1))), t0, t1);
    return pk2(copysignf(t0, x0), copysignf(t1, x1));
}

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
// F::call(v) / F::call2(v) are the region's straight-line code on one element
// / one pair of elements; v holds the region's inputs (full tensors: the
// element(s); scalars: their single value).

constexpr int kFusedThreads = 256;
constexpr int kFusedUnroll = 8;  // 16-byte loads in flight per thread per input

// Evaluates F on one float4 group: two packed lane pairs (f32x2).
template <class F>
__device__ __forceinline__ void eval_group(const float4 (&v)[F::NIN > 0 ? F::NIN : 1],
                                           const f2_t (&sv2)[F::NIN > 0 ? F::NIN : 1], f2_t &y01, f2_t &y23) {
    constexpr int NIN = F::NIN > 0 ? F::NIN : 1;
    f2_t lo[NIN], hi[NIN];
#pragma unroll
    for (int k = 0; k < F::NIN; k++) {
        if (F::SCALARS & (1u << k)) {
            lo[k] = sv2[k];
            hi[k] = sv2[k];
        } else {
            lo[k] = pk2(v[k].x, v[k].y);
            hi[k] = pk2(v[k].z, v[k].w);
        }
    }
    y01 = F::call2(lo);
    y23 = F::call2(hi);
}

// Register-loop kernel.  For a full sum each block streams ONE contiguous
// range of the input(s): whole chunks of THREADS * kFusedUnroll float4, the
// ranges as equal as whole chunks allow, one resident wave of blocks.  In a
// chunk, warp w reads its own 4 KiB with kFusedUnroll coalesced 512-byte
// loads per input, all in flight at once, and sums their values (the 32 of
// one chunk in f32 pairs, then one f64 add).  Measured on the 2^26-element
// tanh chain: 5695 GB/s against 5237 for the same loop over kFusedUnroll
// grid-strided streams 3 MB apart (DRAM serves a few hundred long sequential
// streams better than eight interleaved ones); under sustained load 1024-
// thread blocks (2 per SM, 128 KiB chunks) 5235 against 5040 for 256-thread
// ones; software pipelining the loads (the next chunk's issued before this
// one is evaluated) measured slower (80+ registers, 3 blocks per SM).

// Full (non-scalar) inputs of a catalogued region.
template <class F>
constexpr int full_inputs() {
    int c = 0;
    for (int k = 0; k < F::NIN; k++)
        if (!(F::SCALARS & (1u << k))) c++;
    return c;
}

template <class F, bool SUM, int THREADS>
__device__ __forceinline__ void fused_f32_body(const RegionIO &io, int64_t n) {
    constexpr int64_t kChunk4 = (int64_t)THREADS * kFusedUnroll;
    constexpr int NIN = F::NIN > 0 ? F::NIN : 1;
    float sv[NIN];
    f2_t sv2[NIN];
    const float4 *src[NIN];
#pragma unroll
    for (int k = 0; k < F::NIN; k++) {
        src[k] = (const float4 *)io.in[k];
        sv[k] = (F::SCALARS & (1u << k)) ? __ldg((const float *)io.in[k]) : 0.0f;
        sv2[k] = splat2(sv[k]);
    }
    float4 *dst = (float4 *)io.out[0];
    if constexpr (!SUM) {
        // element-wise: kFusedUnroll grid-strided streams, several waves of
        // blocks (measured at 0.92 of the HBM peak writing the tanh chain's
        // vector); the contiguous ranges below pay off for the sums
        const int64_t n4 = n >> 2;
        const int64_t G = (int64_t)gridDim.x * THREADS;
        int64_t b4 = (int64_t)blockIdx.x * THREADS + threadIdx.x;
        for (; b4 + (kFusedUnroll - 1) * G < n4; b4 += kFusedUnroll * G) {
            float4 v[kFusedUnroll][NIN];
#pragma unroll
            for (int u = 0; u < kFusedUnroll; u++)
#pragma unroll
                for (int k = 0; k < F::NIN; k++)
                    if (!(F::SCALARS & (1u << k))) v[u][k] = __ldcs(src[k] + b4 + u * G);
#pragma unroll
            for (int u = 0; u < kFusedUnroll; u++) {
                f2_t y01, y23;
                eval_group<F>(v[u], sv2, y01, y23);
                float4 o;
                upk2(y01, o.x, o.y);
                upk2(y23, o.z, o.w);
                __stcs(dst + b4 + u * G, o);
            }
        }
        for (; b4 < n4; b4 += G) {
            float4 v[NIN];
#pragma unroll
            for (int k = 0; k < F::NIN; k++)
                if (!(F::SCALARS & (1u << k))) v[k] = __ldcs(src[k] + b4);
            f2_t y01, y23;
            eval_group<F>(v, sv2, y01, y23);
            float4 o;
            upk2(y01, o.x, o.y);
            upk2(y23, o.z, o.w);
            __stcs(dst + b4, o);
        }
        const int64_t t = (int64_t)blockIdx.x * THREADS + threadIdx.x;
        if (t < (n & 3)) {
            const int64_t i = (n4 << 2) + t;
            float e[NIN];
#pragma unroll
            for (int k = 0; k < F::NIN; k++) e[k] = (F::SCALARS & (1u << k)) ? sv[k] : ((const float *)io.in[k])[i];
            ((float *)io.out[0])[i] = F::call(e);
        }
        return;
    }
    const int64_t chunks = (n >> 2) / kChunk4;
    const int64_t c0 = chunks * blockIdx.x / gridDim.x, c1 = chunks * (blockIdx.x + 1) / gridDim.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    double acc = 0.0;
    int64_t base = c0 * kChunk4 + w * (32 * kFusedUnroll) + lane;
    for (int64_t c = c0; c < c1; c++, base += kChunk4) {
        float4 v[kFusedUnroll][NIN];
#pragma unroll
        for (int u = 0; u < kFusedUnroll; u++)
#pragma unroll
            for (int k = 0; k < F::NIN; k++)
                if (!(F::SCALARS & (1u << k))) v[u][k] = __ldcs(src[k] + base + u * 32);
        f2_t s = 0ull;
#pragma unroll
        for (int u = 0; u < kFusedUnroll; u++) {
            f2_t y01, y23;
            eval_group<F>(v[u], sv2, y01, y23);
            if (SUM) {
                s = u ? add2(s, add2(y01, y23)) : add2(y01, y23);
            } else {
                float4 o;
                upk2(y01, o.x, o.y);
                upk2(y23, o.z, o.w);
                __stcs(dst + base + u * 32, o);
            }
        }
        if (SUM) {
            float s0, s1;
            upk2(s, s0, s1);
            acc += (double)(s0 + s1);
        }
    }
    // the elements past the last whole chunk (fewer than 4 * kChunk4 + 4),
    // one at a time, grid-strided
    for (int64_t i = chunks * kChunk4 * 4 + (int64_t)blockIdx.x * THREADS + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * THREADS) {
        float e[NIN];
#pragma unroll
        for (int k = 0; k < F::NIN; k++) e[k] = (F::SCALARS & (1u << k)) ? sv[k] : ((const float *)io.in[k])[i];
        const float y = F::call(e);
        if (SUM) acc += (double)y;
        else ((float *)io.out[0])[i] = y;
    }
    if (SUM) {
        const double b = block_sum<THREADS>(acc);
        finish_full_sum<THREADS>(b, io, false);
    }
}

// A one-input sum fits 32 registers without spilling, so it runs 2 blocks of
// 1024 threads per SM (64 warps); other regions keep 256-thread blocks and
// the compiler's own register choice.
template <class F, bool SUM>
constexpr bool kTightSum = SUM && full_inputs<F>() <= 1;
constexpr int kTightThreads = 1024;

template <class F, bool SUM>
__global__ void __launch_bounds__(kTightThreads, 2) fused_f32_tight_kernel(const __grid_constant__ RegionIO io, int64_t n) {
    fused_f32_body<F, SUM, kTightThreads>(io, n);
}
template <class F, bool SUM>
__global__ void __launch_bounds__(kFusedThreads) fused_f32_kernel(const __grid_constant__ RegionIO io, int64_t n) {
    fused_f32_body<F, SUM, kFusedThreads>(io, n);
}

// Threads per block of F's register-loop kernel.
template <class F, bool SUM>
constexpr int fused_threads() {
    return kTightSum<F, SUM> ? kTightThreads : kFusedThreads;
}

// The register-loop kernel launch_fused_f32 uses for F.
template <class F, bool SUM>
constexpr auto fused_kernel_of() {
    if constexpr (kTightSum<F, SUM>) return fused_f32_tight_kernel<F, SUM>;
    else return fused_f32_kernel<F, SUM>;
}

// --------------------------------------- full reductions: bulk-copy pipeline
//
// For an HBM-bound full sum the memory side runs as a bulk-async-copy
// pipeline: one thread per block streams tiles of every full input into
// kBulkStages shared-memory stages with cp.async.bulk (completion counted on
// an mbarrier per stage) while all threads evaluate the region out of shared
// memory.  Tiles go to blocks round-robin, so the grid reads one contiguous
// stretch of HBM at a time.  Every wait is bounded: a wait that runs out sets
// the error word, turns the result into NaN and drains the copies still in
// flight (again bounded) before the block leaves.

constexpr int kBulkTile = 4096;  // elements per tile per input (16 KiB)
constexpr int kBulkStages = 4;
constexpr int kBulkThreads = 256;
constexpr int kBulkPer = kBulkTile / 4 / kBulkThreads;  // float4 per thread per tile
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on one phase of a stage barrier.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

template <class F>
struct FullInputs {
    static constexpr int count() {
        int c = 0;
        for (int k = 0; k < F::NIN; k++)
            if (!(F::SCALARS & (1u << k))) c++;
        return c;
    }
    static constexpr int N = count() > 0 ? count() : 1;
};

template <class F>
__global__ void __launch_bounds__(kBulkThreads) fused_sum_bulk_kernel(const __grid_constant__ RegionIO io, int64_t n) {
    constexpr int NIN = F::NIN > 0 ? F::NIN : 1;
    constexpr int NF = FullInputs<F>::N;
    extern __shared__ __align__(128) float tiles[];  // [kBulkStages][NF][kBulkTile]
    __shared__ __align__(8) uint64_t full[kBulkStages];
    __shared__ int failed;

    float sv[NIN];
    f2_t sv2[NIN];
    const float *src[NF];
    {
        int j = 0;
#pragma unroll
        for (int k = 0; k < F::NIN; k++) {
            sv[k] = 0.0f;
            if (F::SCALARS & (1u << k)) sv[k] = __ldg((const float *)io.in[k]);
            else src[j++] = (const float *)io.in[k];
            sv2[k] = splat2(sv[k]);
        }
    }

    const int64_t ntiles = n / kBulkTile;
    const int64_t mine = ntiles > (int64_t)blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kBulkStages; s++) mbar_init(&full[s], 1);
        failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // thread 0: tile j of this block into stage j % kBulkStages
    auto issue = [&](int64_t j) {
        const int s = (int)(j % kBulkStages);
        const int64_t tile = (int64_t)blockIdx.x + j * gridDim.x;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&full[s], (uint32_t)(NF * kBulkTile * sizeof(float)));
#pragma unroll
        for (int f = 0; f < NF; f++)
            bulk_g2s(tiles + ((size_t)s * NF + f) * kBulkTile, src[f] + tile * kBulkTile,
                     (uint32_t)(kBulkTile * sizeof(float)), &full[s]);
    };
    if (threadIdx.x == 0)
        for (int64_t j = 0; j < mine && j < kBulkStages; j++) issue(j);

    double acc = 0.0;
    int64_t j = 0;
    for (; j < mine; j++) {
        const int s = (int)(j % kBulkStages);
        const uint32_t parity = (uint32_t)((j / kBulkStages) & 1);
        if (!mbar_wait(&full[s], parity)) failed = 1;
        __syncthreads();
        if (failed) break;
        f2_t part[kBulkPer];
#pragma unroll
        for (int c = 0; c < kBulkPer; c++) {
            const int e4 = c * kBulkThreads + threadIdx.x;  // float4 index within the tile
            float4 v[NIN];
            int fi = 0;
#pragma unroll
            for (int k = 0; k < F::NIN; k++)
                if (!(F::SCALARS & (1u << k)))
                    v[k] = reinterpret_cast<const float4 *>(tiles + ((size_t)s * NF + fi++) * kBulkTile)[e4];
            f2_t y01, y23;
            eval_group<F>(v, sv2, y01, y23);
            part[c] = add2(y01, y23);
        }
#pragma unroll
        for (int w = kBulkPer / 2; w >= 1; w >>= 1)
#pragma unroll
            for (int c = 0; c < w; c++) part[c] = add2(part[c], part[c + w]);
        float s0, s1;
        upk2(part[0], s0, s1);
        acc += (double)(s0 + s1);
        __syncthreads();  // stage s fully read: it may be refilled
        if (threadIdx.x == 0 && j + kBulkStages < mine) issue(j + kBulkStages);
    }
    if (failed) {
        // drain the copies this block still has in flight (bounded), then
        // report: the error word, and NaN through this block's partial.  The
        // drain starts at tile j itself: its copy is the one that stalled.
        if (threadIdx.x == 0) {
            for (int64_t q = j; q < mine && q < j + kBulkStages; q++)
                mbar_wait(&full[q % kBulkStages], (uint32_t)((q / kBulkStages) & 1));
            if (io.error) atomicOr(io.error, 1u);
        }
        acc = __int_as_float(0x7fc00000);
    }
    // the elements past the last full tile, grid-strided
    for (int64_t i = ntiles * kBulkTile + (int64_t)blockIdx.x * kBulkThreads + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * kBulkThreads) {
        float e[NIN];
        int fi = 0;
#pragma unroll
        for (int k = 0; k < F::NIN; k++) e[k] = (F::SCALARS & (1u << k)) ? sv[k] : src[fi++][i];
        acc += (double)F::call(e);
    }
    const double b = block_sum<kBulkThreads>(acc);
    finish_full_sum<kBulkThreads>(b, io, false);
}

// Grid of the fused kernels: a fixed number of blocks per SM (grid-stride
// loop); ZPUCUDA_REGION_BPS / ZPUCUDA_REGION_BULK_BPS override the defaults
// for tuning sweeps.
int fused_blocks_per_sm();
int bulk_blocks_per_sm();
// Blocks per SM of a register-loop full sum: ZPUCUDA_REGION_BPS when set,
// else the kernel's own resident blocks per SM (`occupancy`), so the grid is
// one wave (measured on the 2^26 tanh chain: 5190 GB/s at its 5 resident
// blocks per SM against 4940 at 12; element-wise regions run best at 12).
int fused_sum_blocks_per_sm(int occupancy);

// The grid launch_fused_f32 uses for the register-loop kernel of F: a sum
// runs one resident wave (the kernel's own blocks per SM), each block one
// range; element-wise regions run fused_blocks_per_sm() blocks per SM.
template <class F, bool SUM>
int fused_grid() {
    int per_sm = fused_blocks_per_sm();
    if (SUM) {
        static const int occ = [] {
            int nb = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fused_kernel_of<F, SUM>(), fused_threads<F, SUM>(), 0) !=
                cudaSuccess)
                nb = 0;
            return nb;
        }();
        per_sm = fused_sum_blocks_per_sm(occ);
    }
    int grid = num_sms() * per_sm;
    return grid > kMaxRegionBlocks ? kMaxRegionBlocks : grid;
}

// SUM: the region ends in a full sum.  BULK (full sums only): stream through
// the bulk-copy pipeline -- the generator picks it for regions with no
// transcendental step, which are HBM-bound; regions with SFU work keep the
// register loop, whose higher occupancy feeds the SFU better (measured).
template <class F, bool SUM, bool BULK>
int launch_fused_f32(const RegionProgram &p, const RegionIO &io, cudaStream_t s) {
    if (SUM && BULK) {
        auto k = fused_sum_bulk_kernel<F>;
        const size_t smem = (size_t)kBulkStages * FullInputs<F>::N * kBulkTile * sizeof(float);
        // the attribute belongs to the current device: set once per device
        static bool attr[64] = {false};
        const int dev = current_device();
        if (dev < 0 || dev >= 64 || !attr[dev]) {
            ZC_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            if (dev >= 0 && dev < 64) attr[dev] = true;
        }
        int per_sm = bulk_blocks_per_sm();
        const int fit = (int)((220u * 1024u) / (smem + 1024));
        if (per_sm > fit) per_sm = fit < 1 ? 1 : fit;
        int grid = num_sms() * per_sm;
        if (grid > kMaxRegionBlocks) grid = kMaxRegionBlocks;
        k<<<grid, kBulkThreads, smem, s>>>(io, p.numel);
        ZC_LAUNCHED("fused region kernel (bulk pipeline)");
        return ZPUCUDA_OK;
    }
    auto k = fused_kernel_of<F, SUM>();
    const int grid = fused_grid<F, SUM>();
    k<<<grid, fused_threads<F, SUM>(), 0, s>>>(io, p.numel);
    ZC_LAUNCHED("fused region kernel");
    return ZPUCUDA_OK;
}

// ops.cumsum (src/zpu/ops.zig:2032-2060) of a contiguous [outer, dim, inner]
// tensor along the middle axis into y: a running f64 sum, each prefix
// rounded to the element type; `reverse` runs from the end.
int cumsum_launch(int dtype, const void *x, void *y, int64_t outer, int64_t dim, int64_t inner, bool reverse,
                  cudaStream_t s);

// The lookup the lowering uses: nullptr when `sig` is not catalogued.
const CatalogueEntry *catalogue_find(const char *sig);
// Runs a lowered region: the catalogued kernel when there is one (and the
// inputs are 16-byte aligned), the bytecode kernel otherwise.
int region_launch(const RegionProgram &p, const CatalogueEntry *cat, const RegionIO &io, cudaStream_t s);

}  // namespace zc
