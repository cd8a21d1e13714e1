// Region kernels: the catalogue lookup, the grid sizing, and the generic
// one-pass bytecode kernel that runs any lowered region the build-time
// catalogue does not cover (still one read of each input, no intermediate
// HBM traffic, same reduction scheme).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <type_traits>

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

// Element offset of region element i in input k.
__device__ __forceinline__ int64_t in_offset(const RegionProgram &p, int k, int64_t i) {
    switch (p.in_kind[k]) {
    case IN_FULL: return i;
    case IN_SCALAR: return 0;
    case IN_ROW: return i % p.in_numel[k];
    default: {
        int64_t rem = i, off = 0;
        for (int d = p.rank - 1; d >= 0; d--) {
            const int64_t idx = rem % p.dims[d];
            rem /= p.dims[d];
            off += idx * p.in_strides[k][d];
        }
        return off;
    }
    }
}

template <class T>
__device__ __forceinline__ T load_in(const RegionProgram &p, const RegionIO &io, int k, int64_t i) {
    const int64_t off = in_offset(p, k, i);
    if (p.in_bool[k]) return ((const uint8_t *)io.in[k])[off] ? (T)1 : (T)0;
    return ((const T *)io.in[k])[off];
}

template <class T>
__device__ __forceinline__ void eval(const RegionProgram &p, const RegionIO &io, int64_t i, T *r) {
    for (int k = 0; k < p.n_insn; k++) {
        const Insn in = p.insn[k];
        if (in.op == OPC_LOAD) r[in.dst] = load_in<T>(p, io, in.a, i);
        else if (in.op == 55) r[in.dst] = r[in.a] != (T)0 ? r[in.b] : r[in.c];  // where: ops.zig:572-590
        else if (in.op < 35 || in.op == 54) r[in.dst] = un<T>(in.op, r[in.a]);
        else r[in.dst] = bin<T>(in.op, r[in.a], r[in.b]);
    }
}

// ------------------------------------------------ 64-bit-word regions

__device__ __forceinline__ long long ibits(double r) { return __double_as_longlong(r); }
__device__ __forceinline__ double iword(long long v) { return __longlong_as_double(v); }
// scalar.fromF64(i64, v) (scalar.zig:17-27): 0 for NaN, else clamped to
// [minInt, maxInt] and truncated toward zero (cvt.rzi saturates, so 2^63,
// maxInt as an f64, gives maxInt)
__device__ __forceinline__ long long f64_to_i64(double v) { return isnan(v) ? 0 : __double2ll_rz(v); }

// std.math.pow(f64, x, y), which zpu's pow calls (scalar.zig:151-153),
// branch for branch: the special values, a half power as sqrt, then the
// integer part of |y| by repeated squaring of frexp(x)'s mantissa with the
// binary exponent kept apart, a fractional part through exp(yf * log(x)),
// and one ldexp.  With integer operands (zpu's pow of two i64 values) every
// step is an IEEE multiply or an exact scaling, so the bits are zpu's.
__device__ bool odd_integer(double x) {
    if (fabs(x) >= 9007199254740992.0) return false;  // 2^53: every such f64 is even
    double ip;
    const double fp = modf(x, &ip);
    return fp == 0.0 && (((long long)ip) & 1) == 1;
}
__device__ double zig_pow(double x, double y) {
    for (int pass = 0; pass < 2; pass++) {
        if (y == 0.0 || x == 1.0) return 1.0;
        if (isnan(x) || isnan(y)) return nan("");
        if (y == 1.0) return x;
        if (x == 0.0) {
            if (y < 0.0) return odd_integer(y) ? copysign(INFINITY, x) : INFINITY;
            return odd_integer(y) ? x : 0.0;
        }
        if (isinf(y)) {
            if (x == -1.0) return 1.0;
            return ((fabs(x) < 1.0) == (y > 0.0)) ? 0.0 : INFINITY;
        }
        if (!isinf(x)) break;
        if (x > 0.0) return y < 0.0 ? 0.0 : INFINITY;
        x = 1.0 / x;  // pow(-inf, y) = pow(-0, -y): one more pass
        y = -y;
    }
    if (y == 0.5) return sqrt(x);
    if (y == -0.5) return 1.0 / sqrt(x);
    double yi;
    double yf = modf(fabs(y), &yi);
    if (yf != 0.0 && x < 0.0) return nan("");
    if (yi >= 9223372036854775808.0) return exp(y * log(x));  // 2^63
    double a1 = 1.0;
    int ae = 0;
    if (yf != 0.0) {
        if (yf > 0.5) {
            yf -= 1.0;
            yi += 1.0;
        }
        a1 = exp(yf * log(x));
    }
    int xe;
    double x1 = frexp(x, &xe);
    for (long long i = (long long)yi; i != 0; i >>= 1) {
        if (xe < -(1 << 12) || (1 << 12) < xe) {  // far past the range: ldexp saturates
            ae += xe;
            break;
        }
        if (i & 1) {
            a1 *= x1;
            ae += xe;
        }
        x1 *= x1;
        xe <<= 1;
        if (x1 < 0.5) {
            x1 += x1;
            xe -= 1;
        }
    }
    if (y < 0.0) {
        a1 = 1.0 / a1;
        ae = -ae;
    }
    return ldexp(a1, ae);
}

// scalar.binary / scalar.unary of two i64 values (scalar.zig:262-302):
// + - * on the integers (two's-complement wrap where zpu's would overflow),
// mod with a zero divisor giving a, @mod's sign of the divisor otherwise.
__device__ __forceinline__ long long int_binary(int op, long long a, long long b) {
    const unsigned long long ua = (unsigned long long)a, ub = (unsigned long long)b;
    switch (op) {
    case OPC_IADD: return (long long)(ua + ub);
    case OPC_ISUB: return (long long)(ua - ub);
    case OPC_IMUL: return (long long)(ua * ub);
    case OPC_IMOD: {
        if (b == 0) return a;
        if (b == -1) return 0;
        long long r = a % b;
        if (r != 0 && ((r < 0) != (b < 0))) r += b;
        return r;
    }
    case OPC_IMAX: return a > b ? a : b;
    default: return a < b ? a : b;  // OPC_IMIN
    }
}
__device__ __forceinline__ long long int_unary(int op, long long x) {
    switch (op) {
    case OPC_IABS: return x < 0 ? (long long)(0ull - (unsigned long long)x) : x;
    case OPC_ISIGN: return x > 0 ? 1 : (x < 0 ? -1 : 0);
    default: return x > 0 ? x : 0;  // OPC_IRELU
    }
}

template <class T>
__device__ __forceinline__ double load_w(const RegionProgram &p, const RegionIO &io, int k, int64_t i) {
    const int64_t off = in_offset(p, k, i);
    if (p.in_bool[k]) return ((const uint8_t *)io.in[k])[off] ? 1.0 : 0.0;
    if (p.in_i64[k]) return iword(((const long long *)io.in[k])[off]);
    return (double)((const T *)io.in[k])[off];
}

template <class T>
__device__ __forceinline__ void eval_w(const RegionProgram &p, const RegionIO &io, int64_t i, double *r) {
    for (int k = 0; k < p.n_insn; k++) {
        const Insn in = p.insn[k];
        double v;
        switch (in.op) {
        case OPC_LOAD: v = load_w<T>(p, io, in.a, i); break;
        case OPC_I2F: v = __ll2double_rn(ibits(r[in.a])); break;
        case OPC_F2I: v = iword(f64_to_i64(r[in.a])); break;
        case OPC_R32: v = (double)__double2float_rn(r[in.a]); break;
        case OPC_ZPOW: v = zig_pow(r[in.a], r[in.b]); break;
        case OPC_IADD: case OPC_ISUB: case OPC_IMUL: case OPC_IMOD: case OPC_IMAX: case OPC_IMIN:
            v = iword(int_binary(in.op, ibits(r[in.a]), ibits(r[in.b])));
            break;
        case OPC_IABS: case OPC_ISIGN: case OPC_IRELU: v = iword(int_unary(in.op, ibits(r[in.a]))); break;
        case 55: v = r[in.a] != 0.0 ? r[in.b] : r[in.c]; break;
        default: {
            const bool u = in.op < 35 || in.op == 54;
            if (in.c == kInsnF32)
                v = u ? (double)unary_f32(in.op, (float)r[in.a]) : (double)binary_f32(in.op, (float)r[in.a], (float)r[in.b]);
            else
                v = u ? unary_f64(in.op, r[in.a]) : binary_f64(in.op, r[in.a], r[in.b]);
        }
        }
        r[in.dst] = v;
    }
}

// One element through either evaluator: R is the register type (T, or the
// 64-bit word of a words64 region).
template <class T, bool W>
__device__ __forceinline__ void eval_any(const RegionProgram &p, const RegionIO &io, int64_t i,
                                         typename std::conditional<W, double, T>::type *r) {
    if constexpr (W) eval_w<T>(p, io, i, r);
    else eval<T>(p, io, i, r);
}

__device__ __forceinline__ double red_identity(int red) {
    switch (red) {
    case RED_PROD: return 1.0;
    case RED_MAX: return -INFINITY;
    case RED_MIN: return INFINITY;
    case RED_ALL: return 1.0;
    // i64 identities as bits (an empty i64 max / min is zpu's -inf / +inf
    // written into an i64: minInt / maxInt); RED_ISUM's 0 is the word 0.0
    case RED_IPROD: return iword(1);
    case RED_IMAX: return iword((long long)0x8000000000000000ull);
    case RED_IMIN: return iword(0x7fffffffffffffffll);
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
    // i64 words: the order of a wrapping sum / product does not change it
    case RED_ISUM: return iword((long long)((unsigned long long)ibits(acc) + (unsigned long long)ibits(v)));
    case RED_IPROD: return iword((long long)((unsigned long long)ibits(acc) * (unsigned long long)ibits(v)));
    case RED_IMAX: return ibits(v) > ibits(acc) ? v : acc;
    case RED_IMIN: return ibits(v) < ibits(acc) ? v : acc;
    default: return acc + v;
    }
}
__device__ __forceinline__ double warp_reduce(int red, double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = red_combine(red, v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

constexpr int kInterpThreads = 256;

// R: the register type (T, or double in a words64 region, where an i64
// output's register holds its bits and a float one an exact T value).
template <class T, class R>
__device__ __forceinline__ void store_outputs(const RegionProgram &p, const RegionIO &io, int64_t i, const R *r) {
    for (int o = 0; o < p.n_out; o++) {
        if (p.out_bool[o]) ((uint8_t *)io.out[o])[i] = r[p.out_reg[o]] != (R)0;
        else if (p.out_i64[o]) ((long long *)io.out[o])[i] = __double_as_longlong((double)r[p.out_reg[o]]);
        else ((T *)io.out[o])[i] = (T)r[p.out_reg[o]];
    }
}
// The reduced value at output index `i`: any / all store a bool byte.
template <class T>
__device__ __forceinline__ void store_red(const RegionProgram &p, const RegionIO &io, int64_t i, double v) {
    if (p.reduce == RED_ANY || p.reduce == RED_ALL) ((uint8_t *)io.red_out)[i] = v != 0.0;
    else if (red_is_int(p.reduce)) ((long long *)io.red_out)[i] = ibits(v);
    else ((T *)io.red_out)[i] = (T)v;
}

// MODE 0: element-wise outputs only; 1: plus a full reduction; 2: plus a
// reduction over the last axis (one warp per row); 3: plus a reduction over
// an axis that is not the last: the region is [outer, red_len, inner], one
// thread per output element walks the reduced axis in order (the row-order
// walk of ops.reduceKernel, src/zpu/ops.zig:746-752), threads of a warp on
// consecutive inner indices so every step of the walk is one coalesced load.
template <class T, int MODE, bool W>
__global__ void __launch_bounds__(kInterpThreads) interp_kernel(const __grid_constant__ RegionProgram p,
                                                                const __grid_constant__ RegionIO io) {
    typename std::conditional<W, double, T>::type r[RP_MAX_REG];
    if (MODE == 0) {
        for (int64_t i = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; i < p.numel;
             i += (int64_t)gridDim.x * kInterpThreads) {
            eval_any<T, W>(p, io, i, r);
            store_outputs<T>(p, io, i, r);
        }
    } else if (MODE == 1) {
        double acc = red_identity(p.reduce);
        for (int64_t i = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; i < p.numel;
             i += (int64_t)gridDim.x * kInterpThreads) {
            eval_any<T, W>(p, io, i, r);
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
                eval_any<T, W>(p, io, i, r);
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
                eval_any<T, W>(p, io, i, r);
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
template <class T, int MODE, bool W>
__global__ void __launch_bounds__(kInterpThreads) interp_arg_kernel(const __grid_constant__ RegionProgram p,
                                                                    const __grid_constant__ RegionIO io) {
    typename std::conditional<W, double, T>::type r[RP_MAX_REG];
    const bool want_max = p.reduce == RED_ARGMAX;
    int64_t *out = (int64_t *)io.red_out;
    if (MODE == 1) {
        ArgAcc acc = arg_empty();
        for (int64_t i = (int64_t)blockIdx.x * kInterpThreads + threadIdx.x; i < p.numel;
             i += (int64_t)gridDim.x * kInterpThreads) {
            eval_any<T, W>(p, io, i, r);
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
                eval_any<T, W>(p, io, i, r);
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
                eval_any<T, W>(p, io, i, r);
                store_outputs<T>(p, io, i, r);
                arg_take(acc, (double)r[p.reduce_reg], j, want_max);
            }
            acc = arg_warp(acc, want_max);
            if (lane == 0) out[row] = arg_result(acc);
        }
    }
}

template <class T, bool W>
int launch_interp(const RegionProgram &p, const RegionIO &io, cudaStream_t s) {
    const int sms = num_sms();
    const bool arg = p.reduce == RED_ARGMAX || p.reduce == RED_ARGMIN;
    if (p.reduce == RED_NONE) {
        if (p.numel == 0) return ZPUCUDA_OK;
        int64_t g = (p.numel + kInterpThreads - 1) / kInterpThreads;
        if (g > sms * 8) g = sms * 8;
        interp_kernel<T, 0, W><<<(int)g, kInterpThreads, 0, s>>>(p, io);
    } else if (p.reduce_all) {
        int64_t g = (p.numel + kInterpThreads - 1) / kInterpThreads;
        if (g > sms * 8) g = sms * 8;
        if (g < 1) g = 1;
        if (arg) interp_arg_kernel<T, 1, W><<<(int)g, kInterpThreads, 0, s>>>(p, io);
        else interp_kernel<T, 1, W><<<(int)g, kInterpThreads, 0, s>>>(p, io);
    } else if (p.reduce_mid) {
        const int64_t n_out = p.outer * p.inner;
        if (n_out == 0) return ZPUCUDA_OK;
        int64_t g = (n_out + kInterpThreads - 1) / kInterpThreads;
        if (g > sms * 8) g = sms * 8;
        if (arg) interp_arg_kernel<T, 3, W><<<(int)g, kInterpThreads, 0, s>>>(p, io);
        else interp_kernel<T, 3, W><<<(int)g, kInterpThreads, 0, s>>>(p, io);
    } else {
        if (p.outer == 0) return ZPUCUDA_OK;
        int64_t g = (p.outer + (kInterpThreads / 32) - 1) / (kInterpThreads / 32);
        if (g > sms * 8) g = sms * 8;
        if (arg) interp_arg_kernel<T, 2, W><<<(int)g, kInterpThreads, 0, s>>>(p, io);
        else interp_kernel<T, 2, W><<<(int)g, kInterpThreads, 0, s>>>(p, io);
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
// readF64 / writeF64 of one element (an i64 reads as the nearest f64 and
// writes as scalar.fromF64 does)
__device__ __forceinline__ double cum_read(float v) { return (double)v; }
__device__ __forceinline__ double cum_read(double v) { return v; }
__device__ __forceinline__ double cum_read(long long v) { return __ll2double_rn(v); }
__device__ __forceinline__ void cum_write(float *y, double a) { *y = (float)a; }
__device__ __forceinline__ void cum_write(double *y, double a) { *y = a; }
__device__ __forceinline__ void cum_write(long long *y, double a) { *y = f64_to_i64(a); }

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
            acc += cum_read(x[idx]);
            cum_write(y + idx, acc);
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
    else if (dtype == ZPUCUDA_I64)
        cumsum_kernel<long long><<<(int)g, 256, 0, s>>>((const long long *)x, (long long *)y, outer, dim, inner, reverse);
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
    if (p.words64) return p.dtype == ZPUCUDA_F32 ? launch_interp<float, true>(p, io, s) : launch_interp<double, true>(p, io, s);
    if (p.dtype == ZPUCUDA_F32) return launch_interp<float, false>(p, io, s);
    return launch_interp<double, false>(p, io, s);
}

}  // namespace zc
