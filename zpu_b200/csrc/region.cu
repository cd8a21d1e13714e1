// Region kernels: the catalogue lookup, the grid sizing, and the generic
// one-pass bytecode kernel that runs any lowered region the build-time
// catalogue does not cover (still one read of each input, no intermediate
// HBM traffic, same reduction scheme).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "region.cuh"
#include "regions_gen.cuh"

namespace zc {

const CatalogueEntry *catalogue_find(const char *sig) {
    for (int i = 0; i < kCatalogueSize; i++)
        if (strcmp(kCatalogue[i].signature, sig) == 0) return &kCatalogue[i];
    return nullptr;
}

// Blocks per SM of the register-loop kernels (12: measured best for the
// SFU-bound tanh chain, within 2% of 8..16 for the HBM-bound ones) and of the
// bulk-copy pipeline (2 x 64 KiB of stages per SM: measured best).
int fused_blocks_per_sm() {
    static int v = [] {
        const char *e = getenv("ZPUCUDA_REGION_BPS");
        const int x = e ? atoi(e) : 0;
        return (x >= 1 && x <= 16) ? x : 12;
    }();
    return v;
}

int fused_sum_blocks_per_sm(int occupancy) {
    static const int env = [] {
        const char *e = getenv("ZPUCUDA_REGION_BPS");
        const int x = e ? atoi(e) : 0;
        return (x >= 1 && x <= 16) ? x : 0;
    }();
    if (env) return env;
    return (occupancy >= 1 && occupancy <= 16) ? occupancy : fused_blocks_per_sm();
}

int bulk_blocks_per_sm() {
    static int v = [] {
        const char *e = getenv("ZPUCUDA_REGION_BULK_BPS");
        const int x = e ? atoi(e) : 0;
        return (x >= 1 && x <= 8) ? x : 2;
    }();
    return v;
}

// ------------------------------------------------------------ per-op math
//
// f32 semantics follow zpu: + - * / are single IEEE f32 operations
// (kernels.applyBinary, src/zpu/kernels.zig:141-150); transcendental steps
// are evaluated in f64 and rounded once, which is what zpu's scalar path does
// (scalar.zig:262-266) and within one rounding of its f32 vector forms.

__device__ __forceinline__ double mod_f64(double a, double b) {
    if (b == 0.0) return nan("");
    double r = fmod(a, b);
    if (r != 0.0 && ((r < 0.0) != (b < 0.0))) r += b;
    return r;
}

__device__ double unary_f64(int op, double x) {
    switch (op) {
    case 0: return -x;
    case 1: return fabs(x);
    case 2: return exp(x);
    case 3: return expm1(x);
    case 4: return log(x);
    case 5: return log1p(x);
    case 6: return sqrt(x);
    case 7: return 1.0 / sqrt(x);
    case 8: return x * x;
    case 9: return 1.0 / x;
    case 10: return cbrt(x);
    case 11: return sin(x);
    case 12: return cos(x);
    case 13: return tan(x);
    case 14: return asin(x);
    case 15: return acos(x);
    case 16: return atan(x);
    case 17: return sinh(x);
    case 18: return cosh(x);
    case 19: return tanh(x);
    case 20: return asinh(x);
    case 21: return acosh(x);
    case 22: return atanh(x);
    case 23: return erf(x);
    case 24: return 1.0 / (1.0 + exp(-x));
    case 25: return fmax(x, 0.0) + log1p(exp(-fabs(x)));
    case 26: return x > 0.0 ? x : 0.0;
    case 27: return floor(x);
    case 28: return ceil(x);
    case 29: return round(x);
    case 30: return trunc(x);
    case 31: return x > 0.0 ? 1.0 : (x < 0.0 ? -1.0 : 0.0);
    // unary predicates (scalar.pred1F, src/zpu/scalar.zig:252-259) and
    // logical_not (ops.logicalNot: x == 0, ops.zig:516-520), as 1 / 0
    case 32: return isnan(x) ? 1.0 : 0.0;
    case 33: return isinf(x) ? 1.0 : 0.0;
    case 34: return isfinite(x) ? 1.0 : 0.0;
    case 54: return x == 0.0 ? 1.0 : 0.0;
    default: return nan("");
    }
}

__device__ float unary_f32(int op, float x) {
    switch (op) {
    case 0: return -x;
    case 1: return fabsf(x);
    case 6: return __fsqrt_rn(x);
    case 7: return __fdiv_rn(1.0f, __fsqrt_rn(x));
    case 8: return __fmul_rn(x, x);
    case 9: return __fdiv_rn(1.0f, x);
    case 24: {  // the f32 vector form 1 / (1 + exp(-x)) (kernels.zig:96)
        const float e = (float)exp(-(double)x);
        return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
    }
    case 26: return x > 0.0f ? x : 0.0f;
    case 27: return floorf(x);
    case 28: return ceilf(x);
    case 29: return roundf(x);
    case 30: return truncf(x);
    case 31: return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
    default: return (float)unary_f64(op, (double)x);
    }
}

__device__ __forceinline__ double binary_f64(int op, double a, double b) {
    switch (op) {
    case 35: return a + b;
    case 36: return a - b;
    case 37: return a * b;
    case 38: return a / b;
    case 39: return pow(a, b);
    case 40: return isnan(a) ? a : (isnan(b) ? b : (a > b ? a : b));
    case 41: return isnan(a) ? a : (isnan(b) ? b : (a < b ? a : b));
    case 42: return atan2(a, b);
    case 43: return hypot(a, b);
    case 44: return mod_f64(a, b);
    // comparisons and logical ops on f64 values (scalar.pred2F,
    // src/zpu/scalar.zig:235-249), as 1 / 0; truthiness is v != 0 (NaN is true)
    case 45: return a == b ? 1.0 : 0.0;
    case 46: return a != b ? 1.0 : 0.0;
    case 47: return a < b ? 1.0 : 0.0;
    case 48: return a <= b ? 1.0 : 0.0;
    case 49: return a > b ? 1.0 : 0.0;
    case 50: return a >= b ? 1.0 : 0.0;
    case 51: return (a != 0.0 && b != 0.0) ? 1.0 : 0.0;
    case 52: return (a != 0.0 || b != 0.0) ? 1.0 : 0.0;
    case 53: return ((a != 0.0) != (b != 0.0)) ? 1.0 : 0.0;
    default: return nan("");
    }
}

__device__ __forceinline__ float binary_f32(int op, float a, float b) {
    switch (op) {
    case 35: return __fadd_rn(a, b);
    case 36: return __fsub_rn(a, b);
    case 37: return __fmul_rn(a, b);
    case 38: return __fdiv_rn(a, b);
    default: return (float)binary_f64(op, (double)a, (double)b);
    }
}

template <class T> __device__ __forceinline__ T un(int op, T x);
template <> __device__ __forceinline__ float un<float>(int op, float x) { return unary_f32(op, x); }
template <> __device__ __forceinline__ double un<double>(int op, double x) { return unary_f64(op, x); }
template <class T> __device__ __forceinline__ T bin(int op, T a, T b);
template <> __device__ __forceinline__ float bin<float>(int op, float a, float b) { return binary_f32(op, a, b); }
template <> __device__ __forceinline__ double bin<double>(int op, double a, double b) { return binary_f64(op, a, b); }

// ------------------------------------------------------- bytecode kernel

template <class T>
__device__ __forceinline__ T load_in(const RegionProgram &p, const RegionIO &io, int k, int64_t i) {
    int64_t off;
    switch (p.in_kind[k]) {
    case IN_FULL: off = i; break;
    case IN_SCALAR: off = 0; break;
    case IN_ROW: off = i % p.in_numel[k]; break;
    default: {
        int64_t rem = i;
        off = 0;
        for (int d = p.rank - 1; d >= 0; d--) {
            const int64_t idx = rem % p.dims[d];
            rem /= p.dims[d];
            off += idx * p.in_strides[k][d];
        }
    }
    }
    if (p.in_bool[k]) return ((const uint8_t *)io.in[k])[off] ? (T)1 : (T)0;
    if (p.in_i64[k]) return (T)__ll2double_rn(((const long long *)io.in[k])[off]);
    return ((const T *)io.in[k])[off];
}

// scalar.fromF64 to i64 followed by toF64 (src/zpu/scalar.zig:7-27).
template <class T>
__device__ __forceinline__ T to_i64_value(T v) {
    if (isnan(v)) return (T)0;
    const T lim = (T)9223372036854775808.0;  // 2^63
    v = v < -lim ? -lim : (v > lim ? lim : v);
    return trunc(v);
}

template <class T>
__device__ __forceinline__ void eval(const RegionProgram &p, const RegionIO &io, int64_t i, T *r) {
    for (int k = 0; k < p.n_insn; k++) {
        const Insn in = p.insn[k];
        if (in.op == OPC_LOAD) r[in.dst] = load_in<T>(p, io, in.a, i);
        else if (in.op == OPC_TO_I64) r[in.dst] = to_i64_value<T>(r[in.a]);
        else if (in.op == 55) r[in.dst] = r[in.a] != (T)0 ? r[in.b] : r[in.c];  // where: ops.zig:572-590
        else if (in.op < 35 || in.op == 54) r[in.dst] = un<T>(in.op, r[in.a]);
        else r[in.dst] = bin<T>(in.op, r[in.a], r[in.b]);
    }
}

__device__ __forceinline__ double red_identity(int red) {
    switch (red) {
    case RED_PROD: return 1.0;
    case RED_MAX: return -INFINITY;
    case RED_MIN: return INFINITY;
    case RED_ALL: return 1.0;
    default: return 0.0;
    }
}
// NaN propagates through max/min, as reduceStep does (src/zpu/ops.zig:688-695).
__device__ __forceinline__ double red_combine(int red, double acc, double v) {
    switch (red) {
    case RED_PROD: return acc * v;
    case RED_MAX: return isnan(v) || isnan(acc) ? (isnan(acc) ? acc : v) : (v > acc ? v : acc);
    case RED_MIN: return isnan(v) || isnan(acc) ? (isnan(acc) ? acc : v) : (v < acc ? v : acc);
    // any / all of x != 0 (ops.reduceOp on a non-bool input takes ne(x, 0)
    // first, ops.zig:845-853)
    case RED_ANY: return (acc != 0.0 || v != 0.0) ? 1.0 : 0.0;
    case RED_ALL: return (acc != 0.0 && v != 0.0) ? 1.0 : 0.0;
    default: return acc + v;
    }
}
__device__ __forceinline__ double warp_reduce(int red, double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = red_combine(red, v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

constexpr int kInterpThreads = 256;

template <class T>
__device__ __forceinline__ void store_outputs(const RegionProgram &p, const RegionIO &io, int64_t i, const T *r) {
    for (int o = 0; o < p.n_out; o++) {
        if (p.out_bool[o]) ((uint8_t *)io.out[o])[i] = r[p.out_reg[o]] != (T)0;
        else if (p.out_i64[o]) ((long long *)io.out[o])[i] = __double2ll_rz((double)to_i64_value<T>(r[p.out_reg[o]]));
        else ((T *)io.out[o])[i] = r[p.out_reg[o]];
    }
}
// The reduced value at output index `i`: any / all store a bool byte.
template <class T>
__device__ __forceinline__ void store_red(const RegionProgram &p, const RegionIO &io, int64_t i, double v) {
    if (p.reduce == RED_ANY || p.reduce == RED_ALL) ((uint8_t *)io.red_out)[i] = v != 0.0;
    else ((T *)io.red_out)[i] = (T)v;
}

// MODE 0: element-wise outputs only; 1: plus a full reduction; 2: plus a
// reduction over the last axis (one warp per row); 3: plus a reduction over
// an axis that is not the last: the region is [outer, red_len, inner], one
// thread per output element walks the reduced axis in order (the row-order
// walk of ops.reduceKernel, src/zpu/ops.zig:746-752), threads of a warp on
// consecutive inner indices so every step of the walk is one coalesced load.
template <class T, int MODE>
__global__ void __launch_bounds__(kInterpThreads) interp_kernel(const __grid_constant__ RegionProgram p,
                                                                const __grid_constant__ RegionIO io) {
    T r[RP_MAX_REG];
    if (MODE == 0) {
        for (int64_t i = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; i < p.numel;
             i += (int64_t)gridDim.x * kInterpThreads) {
            eval<T>(p, io, i, r);
            store_outputs<T>(p, io, i, r);
        }
    } else if (MODE == 1) {
        double acc = red_identity(p.reduce);
        for (int64_t i = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; i < p.numel;
             i += (int64_t)gridDim.x * kInterpThreads) {
            eval<T>(p, io, i, r);
            store_outputs<T>(p, io, i, r);
            acc = red_combine(p.reduce, acc, (double)r[p.reduce_reg]);
        }
        __shared__ double part[kInterpThreads / 32];
        __shared__ bool last;
        acc = warp_reduce(p.reduce, acc);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            double b = part[0];
            for (int w = 1; w < kInterpThreads / 32; w++) b = red_combine(p.reduce, b, part[w]);
            io.partials[blockIdx.x] = b;
            __threadfence();
            last = atomicAdd(io.ticket, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (!last || threadIdx.x != 0) return;
        __threadfence();
        double v = red_identity(p.reduce);
        for (unsigned b = 0; b < gridDim.x; b++) v = red_combine(p.reduce, v, __ldcg(io.partials + b));
        store_red<T>(p, io, 0, v);
        *io.ticket = 0u;
    } else if (MODE == 3) {
        const int64_t n_out = p.outer * p.inner;
        for (int64_t o = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; o < n_out;
             o += (int64_t)gridDim.x * kInterpThreads) {
            const int64_t a = o / p.inner, c = o - a * p.inner;
            double acc = red_identity(p.reduce);
            for (int64_t k = 0; k < p.red_len; k++) {
                const int64_t i = (a * p.red_len + k) * p.inner + c;
                eval<T>(p, io, i, r);
                store_outputs<T>(p, io, i, r);
                acc = red_combine(p.reduce, acc, (double)r[p.reduce_reg]);
            }
            store_red<T>(p, io, o, acc);
        }
    } else {
        const int lane = threadIdx.x & 31;
        const int64_t warps = (int64_t)gridDim.x * (kInterpThreads / 32);
        for (int64_t row = ((int64_t)blockIdx.x * kInterpThreads + threadIdx.x) >> 5; row < p.outer; row += warps) {
            double acc = red_identity(p.reduce);
            for (int64_t j = lane; j < p.inner; j += 32) {
                const int64_t i = row * p.inner + j;
                eval<T>(p, io, i, r);
                store_outputs<T>(p, io, i, r);
                acc = red_combine(p.reduce, acc, (double)r[p.reduce_reg]);
            }
            acc = warp_reduce(p.reduce, acc);
            if (lane == 0) store_red<T>(p, io, row, acc);
        }
    }
}

// ------------------------------------------------ argmax / argmin regions
//
// ops.argReduce (src/zpu/ops.zig:931-975) scans the reduced elements in row
// order: the first seeds the best value, a later one replaces it only when
// strictly greater (argmax) or smaller (argmin).  So ties keep the first
// index, a NaN never replaces the best, and a NaN at position 0 keeps index
// 0 whatever follows.  In parallel every thread scans its positions in
// ascending order keeping the first strict best among the non-NaN values;
// partial results merge by value and, on equal values, by the smaller index
// (the order-free form of the same rule); a NaN at position 0 gives 0.
struct ArgAcc {
    double best;
    int64_t idx;   // -1: no non-NaN value seen
    int64_t nan0;  // 1: the value at position 0 is NaN
};
__device__ __forceinline__ ArgAcc arg_empty() { return ArgAcc{0.0, -1, 0}; }
__device__ __forceinline__ void arg_take(ArgAcc &a, double v, int64_t k, bool want_max) {
    if (isnan(v)) {
        if (k == 0) a.nan0 = 1;
        return;
    }
    if (a.idx < 0 || (want_max ? v > a.best : v < a.best)) {
        a.best = v;
        a.idx = k;
    }
}
__device__ __forceinline__ ArgAcc arg_merge(ArgAcc a, const ArgAcc &b, bool want_max) {
    a.nan0 |= b.nan0;
    if (b.idx < 0) return a;
    bool take_b;
    if (a.idx < 0) take_b = true;
    else if (want_max ? b.best > a.best : b.best < a.best) take_b = true;
    else if (want_max ? a.best > b.best : a.best < b.best) take_b = false;
    else take_b = b.idx < a.idx;
    if (take_b) {
        a.best = b.best;
        a.idx = b.idx;
    }
    return a;
}
__device__ __forceinline__ int64_t arg_result(const ArgAcc &a) { return (a.nan0 || a.idx < 0) ? 0 : a.idx; }
__device__ __forceinline__ ArgAcc arg_warp(ArgAcc a, bool want_max) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgAcc b;
        b.best = __shfl_xor_sync(0xffffffffu, a.best, o);
        b.idx = __shfl_xor_sync(0xffffffffu, a.idx, o);
        b.nan0 = __shfl_xor_sync(0xffffffffu, a.nan0, o);
        a = arg_merge(a, b, want_max);
    }
    return a;
}

// MODE as interp_kernel (1: all axes, 2: trailing axes, one warp per row,
// 3: an inner axis, one thread per output); the output is i64.
template <class T, int MODE>
__global__ void __launch_bounds__(kInterpThreads) interp_arg_kernel(const __grid_constant__ RegionProgram p,
                                                                    const __grid_constant__ RegionIO io) {
    T r[RP_MAX_REG];
    const bool want_max = p.reduce == RED_ARGMAX;
    int64_t *out = (int64_t *)io.red_out;
    if (MODE == 1) {
        ArgAcc acc = arg_empty();
        for (int64_t i = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; i < p.numel;
             i += (int64_t)gridDim.x * kInterpThreads) {
            eval<T>(p, io, i, r);
            store_outputs<T>(p, io, i, r);
            arg_take(acc, (double)r[p.reduce_reg], i, want_max);
        }
        __shared__ ArgAcc part[kInterpThreads / 32];
        __shared__ bool last;
        acc = arg_warp(acc, want_max);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
        __syncthreads();
        double *best = io.partials;
        int64_t *idx = (int64_t *)(io.partials + kMaxRegionBlocks);
        int64_t *nan0 = idx + kMaxRegionBlocks;
        if (threadIdx.x == 0) {
            ArgAcc b = part[0];
            for (int w = 1; w < kInterpThreads / 32; w++) b = arg_merge(b, part[w], want_max);
            best[blockIdx.x] = b.best;
            idx[blockIdx.x] = b.idx;
            nan0[blockIdx.x] = b.nan0;
            __threadfence();
            last = atomicAdd(io.ticket, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (!last || threadIdx.x != 0) return;
        __threadfence();
        ArgAcc v = arg_empty();
        for (unsigned b = 0; b < gridDim.x; b++)
            v = arg_merge(v, ArgAcc{__ldcg(best + b), __ldcg(idx + b), __ldcg(nan0 + b)}, want_max);
        out[0] = arg_result(v);
        *io.ticket = 0u;
    } else if (MODE == 3) {
        const int64_t n_out = p.outer * p.inner;
        for (int64_t o = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; o < n_out;
             o += (int64_t)gridDim.x * kInterpThreads) {
            const int64_t a = o / p.inner, c = o - a * p.inner;
            ArgAcc acc = arg_empty();
            for (int64_t k = 0; k < p.red_len; k++) {
                const int64_t i = (a * p.red_len + k) * p.inner + c;
                eval<T>(p, io, i, r);
                store_outputs<T>(p, io, i, r);
                arg_take(acc, (double)r[p.reduce_reg], k, want_max);
            }
            out[o] = arg_result(acc);
        }
    } else {
        const int lane = threadIdx.x & 31;
        const int64_t warps = (int64_t)gridDim.x * (kInterpThreads / 32);
        for (int64_t row = ((int64_t)blockIdx.x * kInterpThreads + threadIdx.x) >> 5; row < p.outer; row += warps) {
            ArgAcc acc = arg_empty();
            for (int64_t j = lane; j < p.inner; j += 32) {
                const int64_t i = row * p.inner + j;
                eval<T>(p, io, i, r);
                store_outputs<T>(p, io, i, r);
                arg_take(acc, (double)r[p.reduce_reg], j, want_max);
            }
            acc = arg_warp(acc, want_max);
            if (lane == 0) out[row] = arg_result(acc);
        }
    }
}

template <class T>
int launch_interp(const RegionProgram &p, const RegionIO &io, cudaStream_t s) {
    const int sms = num_sms();
    const bool arg = p.reduce == RED_ARGMAX || p.reduce == RED_ARGMIN;
    if (p.reduce == RED_NONE) {
        if (p.numel == 0) return ZPUCUDA_OK;
        int64_t g = (p.numel + kInterpThreads - 1) / kInterpThreads;
        if (g > sms * 8) g = sms * 8;
        interp_kernel<T, 0><<<(int)g, kInterpThreads, 0, s>>>(p, io);
    } else if (p.reduce_all) {
        int64_t g = (p.numel + kInterpThreads - 1) / kInterpThreads;
        if (g > sms * 8) g = sms * 8;
        if (g < 1) g = 1;
        if (arg) interp_arg_kernel<T, 1><<<(int)g, kInterpThreads, 0, s>>>(p, io);
        else interp_kernel<T, 1><<<(int)g, kInterpThreads, 0, s>>>(p, io);
    } else if (p.reduce_mid) {
        const int64_t n_out = p.outer * p.inner;
        if (n_out == 0) return ZPUCUDA_OK;
        int64_t g = (n_out + kInterpThreads - 1) / kInterpThreads;
        if (g > sms * 8) g = sms * 8;
        if (arg) interp_arg_kernel<T, 3><<<(int)g, kInterpThreads, 0, s>>>(p, io);
        else interp_kernel<T, 3><<<(int)g, kInterpThreads, 0, s>>>(p, io);
    } else {
        if (p.outer == 0) return ZPUCUDA_OK;
        int64_t g = (p.outer + (kInterpThreads / 32) - 1) / (kInterpThreads / 32);
        if (g > sms * 8) g = sms * 8;
        if (arg) interp_arg_kernel<T, 2><<<(int)g, kInterpThreads, 0, s>>>(p, io);
        else interp_kernel<T, 2><<<(int)g, kInterpThreads, 0, s>>>(p, io);
    }
    ZC_LAUNCHED("region bytecode kernel");
    return ZPUCUDA_OK;
}

// ------------------------------------------------------------------ cumsum
//
// One thread per (outer, inner) column walks the axis in order with zpu's f64
// accumulator, so every prefix has zpu's bits; threads of a warp take
// consecutive inner indices (coalesced when inner >= 32; for the last axis
// each thread streams its own row, sequential sectors through L1).
template <class T>
__global__ void __launch_bounds__(256) cumsum_kernel(const T *__restrict__ x, T *__restrict__ y, int64_t outer,
                                                     int64_t dim, int64_t inner, int reverse) {
    const int64_t cols = outer * inner;
    for (int64_t c = (int64_t)blockIdx.x * 256 + threadIdx.x; c < cols; c += (int64_t)gridDim.x * 256) {
        const int64_t o = c / inner, i = c - o * inner;
        const int64_t base = o * dim * inner + i;
        double acc = 0.0;
        for (int64_t d = 0; d < dim; d++) {
            const int64_t idx = base + (reverse ? dim - 1 - d : d) * inner;
            acc += (double)x[idx];
            y[idx] = (T)acc;
        }
    }
}

int cumsum_launch(int dtype, const void *x, void *y, int64_t outer, int64_t dim, int64_t inner, bool reverse,
                  cudaStream_t s) {
    const int64_t cols = outer * inner;
    if (cols == 0 || dim == 0) return ZPUCUDA_OK;
    int64_t g = (cols + 255) / 256;
    if (g > (int64_t)num_sms() * 16) g = (int64_t)num_sms() * 16;
    if (dtype == ZPUCUDA_F64)
        cumsum_kernel<double><<<(int)g, 256, 0, s>>>((const double *)x, (double *)y, outer, dim, inner, reverse);
    else
        cumsum_kernel<float><<<(int)g, 256, 0, s>>>((const float *)x, (float *)y, outer, dim, inner, reverse);
    ZC_LAUNCHED("cumsum_kernel");
    return ZPUCUDA_OK;
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int region_launch(const RegionProgram &p, const CatalogueEntry *cat, const RegionIO &io, cudaStream_t s) {
    if (cat && p.dtype == ZPUCUDA_F32) {
        bool ok = true;
        for (int k = 0; k < p.n_in; k++)
            if (p.in_kind[k] == IN_FULL && !aligned16(io.in[k])) ok = false;
        for (int o = 0; o < p.n_out; o++)
            if (!aligned16(io.out[o])) ok = false;
        if (ok) return cat->launch(p, io, s);
    }
    if (p.dtype == ZPUCUDA_F32) return launch_interp<float>(p, io, s);
    return launch_interp<double>(p, io, s);
}

}  // namespace zc
