// ops.matmul for the element types the tensor-core GEMMs do not take: mixed
// operand types, f16, bool operands, and same-type integers.
//
// zpu routes these through two loops of its own, restated here element for
// element:
//  - ops.gemmF64 (src/zpu/ops.zig:1284-1333), for mixed types and for f16 or
//    bool operands: the output (type DType.promote of the operands,
//    src/zpu/dtype.zig:89-104) starts at 0 and, for p = 0 .. k-1 in order,
//    becomes fromF64(toF64(out) + toF64(a[i,p]) * toF64(b[p,j])) -- a
//    product and a sum in f64 (no fused multiply-add), then a rounding to
//    the output type at every step (src/zpu/scalar.zig:7-27: floats round to
//    nearest; integers take 0 for NaN, clamp and truncate);
//  - ops.gemmTyped for a same-type integer product (src/zpu/ops.zig:
//    1016-1049): the element type's own multiply and wrapping add
//    (reduceStep's +%, ops.zig:685-688).  Wrapping arithmetic is exact modulo
//    2^bits whatever the order, so the kernel sums in 64-bit integers and
//    truncates once.
// One thread per output element walks k in order out of 16 x 16 shared-memory
// tiles; the batch runs over blockIdx.z.  These products are not on the
// configurations' hot path (they are f32 / f64): the point is zpu's exact
// result on the device, not tensor-core speed.
#include <cuda_fp16.h>
#include <string.h>

#include "gemm.cuh"

namespace zc {

namespace {

constexpr int kT = 16;

struct ConvertArgs {
    const void *a;
    const void *b;
    void *c;
    int32_t adt, bdt;
    int64_t m, n, k;
    int64_t sam, sak;  // element strides of A's rows and columns
    int64_t sbk, sbn;  // of B's
    GemmBatch bt;
    int64_t batch0;    // first batch index of this launch
    int64_t stride_c;
};

// scalar.toF64 (src/zpu/scalar.zig:7-15) of element i of a typed buffer.
__device__ __forceinline__ double load_f64(const void *p, int dt, int64_t i) {
    switch (dt) {
    case ZPUCUDA_F64: return ((const double *)p)[i];
    case ZPUCUDA_F32: return (double)((const float *)p)[i];
    case ZPUCUDA_F16: return (double)__half2float(((const __half *)p)[i]);
    case ZPUCUDA_I64: return __ll2double_rn(((const long long *)p)[i]);
    case ZPUCUDA_I32: return (double)((const int *)p)[i];
    case ZPUCUDA_I16: return (double)((const short *)p)[i];
    case ZPUCUDA_I8: return (double)((const signed char *)p)[i];
    case ZPUCUDA_U8: return (double)((const unsigned char *)p)[i];
    default: return ((const unsigned char *)p)[i] ? 1.0 : 0.0;
    }
}

__device__ __forceinline__ long long load_i64(const void *p, int dt, int64_t i) {
    switch (dt) {
    case ZPUCUDA_I64: return ((const long long *)p)[i];
    case ZPUCUDA_I32: return ((const int *)p)[i];
    case ZPUCUDA_I16: return ((const short *)p)[i];
    case ZPUCUDA_I8: return ((const signed char *)p)[i];
    default: return ((const unsigned char *)p)[i];
    }
}

// The value zpu stores for v in an integer type of range [lo, hi], read back
// as f64: 0 for NaN, else clamped and truncated toward zero.
__device__ __forceinline__ double int_round(double v, double lo, double hi) {
    if (v != v) return 0.0;
    return trunc(fmin(fmax(v, lo), hi));
}

// fromF64 to the output type, read back as f64 (the `cur` of the next step).
template <int OT>
__device__ __forceinline__ double round_to(double v) {
    switch (OT) {
    case ZPUCUDA_F64: return v;
    case ZPUCUDA_F32: return (double)__double2float_rn(v);
    case ZPUCUDA_F16: return (double)__half2float(__double2half(v));
    case ZPUCUDA_I64: return int_round(v, -9223372036854775808.0, 9223372036854775808.0);
    case ZPUCUDA_I32: return int_round(v, -2147483648.0, 2147483647.0);
    case ZPUCUDA_I16: return int_round(v, -32768.0, 32767.0);
    case ZPUCUDA_I8: return int_round(v, -128.0, 127.0);
    default: return int_round(v, 0.0, 255.0);  // u8
    }
}

template <int OT>
__device__ __forceinline__ void store(void *c, int64_t i, double v) {
    switch (OT) {
    case ZPUCUDA_F64: ((double *)c)[i] = v; break;
    case ZPUCUDA_F32: ((float *)c)[i] = (float)v; break;
    case ZPUCUDA_F16: ((__half *)c)[i] = __double2half(v); break;
    case ZPUCUDA_I64: ((long long *)c)[i] = v >= 9223372036854775808.0 ? 9223372036854775807LL : (long long)v; break;
    case ZPUCUDA_I32: ((int *)c)[i] = (int)v; break;
    case ZPUCUDA_I16: ((short *)c)[i] = (short)v; break;
    case ZPUCUDA_I8: ((signed char *)c)[i] = (signed char)v; break;
    default: ((unsigned char *)c)[i] = (unsigned char)v; break;
    }
}

template <int OT>
__device__ __forceinline__ void store_wrapped(void *c, int64_t i, unsigned long long v) {
    switch (OT) {
    case ZPUCUDA_I64: ((long long *)c)[i] = (long long)v; break;
    case ZPUCUDA_I32: ((unsigned int *)c)[i] = (unsigned int)v; break;
    case ZPUCUDA_I16: ((unsigned short *)c)[i] = (unsigned short)v; break;
    case ZPUCUDA_I8:
    default: ((unsigned char *)c)[i] = (unsigned char)v; break;
    }
}

// ops.gemmF64: every step a product and a sum in f64, rounded to the output type.
template <int OT>
__global__ void __launch_bounds__(kT *kT) gemm_f64path_kernel(const __grid_constant__ ConvertArgs g) {
    __shared__ double As[kT][kT + 1], Bs[kT][kT + 1];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int64_t row = (int64_t)blockIdx.y * kT + ty, col = (int64_t)blockIdx.x * kT + tx;
    const int64_t bi = g.batch0 + blockIdx.z;
    int64_t oa, ob;
    batch_offsets(g.bt, bi, &oa, &ob);
    double acc = 0.0;
    for (int64_t p0 = 0; p0 < g.k; p0 += kT) {
        // A tile [row block][p0 ..], B tile [p0 ..][col block]
        const int64_t ar = (int64_t)blockIdx.y * kT + ty, ap = p0 + tx;
        As[ty][tx] = (ar < g.m && ap < g.k) ? load_f64(g.a, g.adt, oa + ar * g.sam + ap * g.sak) : 0.0;
        const int64_t bp = p0 + ty, bc = (int64_t)blockIdx.x * kT + tx;
        Bs[ty][tx] = (bp < g.k && bc < g.n) ? load_f64(g.b, g.bdt, ob + bp * g.sbk + bc * g.sbn) : 0.0;
        __syncthreads();
        const int kk = (int)(g.k - p0 < kT ? g.k - p0 : kT);
        for (int q = 0; q < kk; q++) acc = round_to<OT>(__dadd_rn(acc, __dmul_rn(As[ty][q], Bs[q][tx])));
        __syncthreads();
    }
    if (row < g.m && col < g.n) store<OT>(g.c, bi * g.stride_c + row * g.n + col, acc);
}

// ops.gemmTyped for integers: wrapping products and sums in the element type.
template <int OT>
__global__ void __launch_bounds__(kT *kT) gemm_int_kernel(const __grid_constant__ ConvertArgs g) {
    __shared__ long long As[kT][kT + 1], Bs[kT][kT + 1];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int64_t row = (int64_t)blockIdx.y * kT + ty, col = (int64_t)blockIdx.x * kT + tx;
    const int64_t bi = g.batch0 + blockIdx.z;
    int64_t oa, ob;
    batch_offsets(g.bt, bi, &oa, &ob);
    unsigned long long acc = 0;
    for (int64_t p0 = 0; p0 < g.k; p0 += kT) {
        const int64_t ar = (int64_t)blockIdx.y * kT + ty, ap = p0 + tx;
        As[ty][tx] = (ar < g.m && ap < g.k) ? load_i64(g.a, g.adt, oa + ar * g.sam + ap * g.sak) : 0;
        const int64_t bp = p0 + ty, bc = (int64_t)blockIdx.x * kT + tx;
        Bs[ty][tx] = (bp < g.k && bc < g.n) ? load_i64(g.b, g.bdt, ob + bp * g.sbk + bc * g.sbn) : 0;
        __syncthreads();
        const int kk = (int)(g.k - p0 < kT ? g.k - p0 : kT);
        for (int q = 0; q < kk; q++) acc += (unsigned long long)As[ty][q] * (unsigned long long)Bs[q][tx];
        __syncthreads();
    }
    if (row < g.m && col < g.n) store_wrapped<OT>(g.c, bi * g.stride_c + row * g.n + col, acc);
}

bool is_int(int dt) { return dt == ZPUCUDA_I64 || dt == ZPUCUDA_I32 || dt == ZPUCUDA_I16 || dt == ZPUCUDA_I8 || dt == ZPUCUDA_U8; }

template <int OT>
int launch_f64path(const ConvertArgs &g, dim3 grid, cudaStream_t s) {
    gemm_f64path_kernel<OT><<<grid, dim3(kT, kT), 0, s>>>(g);
    ZC_LAUNCHED("gemm_f64path_kernel");
    return ZPUCUDA_OK;
}
template <int OT>
int launch_int(const ConvertArgs &g, dim3 grid, cudaStream_t s) {
    gemm_int_kernel<OT><<<grid, dim3(kT, kT), 0, s>>>(g);
    ZC_LAUNCHED("gemm_int_kernel");
    return ZPUCUDA_OK;
}

}  // namespace

// DType.promote (src/zpu/dtype.zig:89-104): floats win over integers, the
// wider float wins, mixed signedness takes the wider type (the second on a
// tie), otherwise the wider one (the first on a tie).
int dtype_promote(int a, int b) {
    auto is_float = [](int d) { return d == ZPUCUDA_F64 || d == ZPUCUDA_F32 || d == ZPUCUDA_F16; };
    auto is_signed = [](int d) { return d == ZPUCUDA_I64 || d == ZPUCUDA_I32 || d == ZPUCUDA_I16 || d == ZPUCUDA_I8; };
    auto size = [](int d) {
        switch (d) {
        case ZPUCUDA_F64: case ZPUCUDA_I64: return 8;
        case ZPUCUDA_F32: case ZPUCUDA_I32: return 4;
        case ZPUCUDA_F16: case ZPUCUDA_I16: return 2;
        default: return 1;
        }
    };
    if (a == b) return a;
    if (is_float(a) && !is_float(b)) return a;
    if (is_float(b) && !is_float(a)) return b;
    if (is_float(a) && is_float(b)) return size(a) >= size(b) ? a : b;
    if (is_signed(a) != is_signed(b)) return size(a) > size(b) ? a : b;
    return size(a) >= size(b) ? a : b;
}

int gemm_convert_device(const void *A, int adt, const void *B, int bdt, void *C, int cdt, int64_t m, int64_t n,
                        int64_t k, int64_t lda, int64_t ldb, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                        cudaStream_t s) {
    if (cdt != dtype_promote(adt, bdt) || cdt == ZPUCUDA_BOOL) return ZPUCUDA_ERR_DTYPE_MISMATCH;
    const int64_t nb = batch_count(bt);
    if (m == 0 || n == 0 || nb == 0) return ZPUCUDA_OK;
    ConvertArgs g;
    memset(&g, 0, sizeof g);
    g.a = A;
    g.b = B;
    g.c = C;
    g.adt = adt;
    g.bdt = bdt;
    g.m = m;
    g.n = n;
    g.k = k;
    g.sam = ta ? 1 : lda;
    g.sak = ta ? lda : 1;
    g.sbk = tb ? 1 : ldb;
    g.sbn = tb ? ldb : 1;
    g.bt = bt;
    g.stride_c = stride_c;
    const int64_t gx = (n + kT - 1) / kT, gy = (m + kT - 1) / kT;
    if (gx > 0x7fffffff || gy > 65535) return ZPUCUDA_ERR_NOT_SUPPORTED;
    const bool wrap = adt == bdt && is_int(adt);
    for (int64_t b0 = 0; b0 < nb; b0 += 65535) {
        g.batch0 = b0;
        const dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(nb - b0 < 65535 ? nb - b0 : 65535));
        int st;
        if (wrap) {
            switch (cdt) {
            case ZPUCUDA_I64: st = launch_int<ZPUCUDA_I64>(g, grid, s); break;
            case ZPUCUDA_I32: st = launch_int<ZPUCUDA_I32>(g, grid, s); break;
            case ZPUCUDA_I16: st = launch_int<ZPUCUDA_I16>(g, grid, s); break;
            case ZPUCUDA_I8: st = launch_int<ZPUCUDA_I8>(g, grid, s); break;
            default: st = launch_int<ZPUCUDA_U8>(g, grid, s); break;
            }
        } else {
            switch (cdt) {
            case ZPUCUDA_F64: st = launch_f64path<ZPUCUDA_F64>(g, grid, s); break;
            case ZPUCUDA_F32: st = launch_f64path<ZPUCUDA_F32>(g, grid, s); break;
            case ZPUCUDA_F16: st = launch_f64path<ZPUCUDA_F16>(g, grid, s); break;
            case ZPUCUDA_I64: st = launch_f64path<ZPUCUDA_I64>(g, grid, s); break;
            case ZPUCUDA_I32: st = launch_f64path<ZPUCUDA_I32>(g, grid, s); break;
            case ZPUCUDA_I16: st = launch_f64path<ZPUCUDA_I16>(g, grid, s); break;
            case ZPUCUDA_I8: st = launch_f64path<ZPUCUDA_I8>(g, grid, s); break;
            default: st = launch_f64path<ZPUCUDA_U8>(g, grid, s); break;
            }
        }
        if (st) return st;
    }
    return ZPUCUDA_OK;
}

}  // namespace zc
