// Element copies of zpu tensors that live in HBM: Tensor.clone,
// Tensor.toContiguous and ops.cast (src/zpu/tensor.zig:356-361,366-404,
// src/zpu/ops.zig:2062-2071).  All three are `out.writeF64(i,
// x.readLogical(n, i))` over the logical (row-major) order: read element i of
// a strided view, widen it to f64 (scalar.toF64), narrow it to the output's
// type (scalar.fromF64, src/zpu/scalar.zig:7-27), write it at i of a
// contiguous buffer.  Here that is one kernel per (source type, output type):
//   * a plain gather, one thread per output element (coalesced writes; reads
//     coalesced when the view's last axis has unit stride);
//   * a tiled transpose for views whose unit-stride axis is the second to
//     last (the swapLastTwo views of the matmul VJP): 32 x 32 tiles through
//     shared memory so reads and writes both coalesce;
//   * cudaMemcpyAsync for a contiguous view of the same type (clone).
// HBM-bound: 1 read + 1 write per element.
#include <cuda_fp16.h>

#include <string>

#include "common.cuh"

namespace zc {
namespace {

// zpu's bool is one byte (0 / 1).
struct Bool8 {
    uint8_t v;
};

// scalar.toF64 (src/zpu/scalar.zig:7-15): floats widen, integers convert
// (round to nearest for i64 beyond 2^53), bool is 0 / 1.
template <class T> __device__ __forceinline__ double to_f64(T x) { return (double)x; }
template <> __device__ __forceinline__ double to_f64<__half>(__half x) { return (double)__half2float(x); }
template <> __device__ __forceinline__ double to_f64<int64_t>(int64_t x) { return __ll2double_rn(x); }
template <> __device__ __forceinline__ double to_f64<Bool8>(Bool8 x) { return x.v ? 1.0 : 0.0; }

// scalar.fromF64 (src/zpu/scalar.zig:17-27): floats round to nearest; an
// integer type takes 0 for NaN, else the value clamped to the type's range
// and truncated toward zero; bool is v != 0 (true for NaN).  For i64 the
// upper clamp, (f64)maxInt(i64), is 2^63, which Zig's @intFromFloat leaves
// undefined; here it saturates to maxInt(i64).
template <class T, int64_t LO, int64_t HI>
__device__ __forceinline__ T int_from_f64(double v) {
    if (isnan(v)) return (T)0;
    const double lo = (double)LO, hi = (double)HI;
    v = v < lo ? lo : (v > hi ? hi : v);
    return (T)__double2ll_rz(v);
}
template <class T> __device__ __forceinline__ T from_f64(double v);
template <> __device__ __forceinline__ double from_f64<double>(double v) { return v; }
template <> __device__ __forceinline__ float from_f64<float>(double v) { return __double2float_rn(v); }
template <> __device__ __forceinline__ __half from_f64<__half>(double v) { return __double2half(v); }
template <> __device__ __forceinline__ int64_t from_f64<int64_t>(double v) {
    return int_from_f64<int64_t, INT64_MIN, INT64_MAX>(v);
}
template <> __device__ __forceinline__ int32_t from_f64<int32_t>(double v) {
    return int_from_f64<int32_t, INT32_MIN, INT32_MAX>(v);
}
template <> __device__ __forceinline__ int16_t from_f64<int16_t>(double v) {
    return int_from_f64<int16_t, INT16_MIN, INT16_MAX>(v);
}
template <> __device__ __forceinline__ int8_t from_f64<int8_t>(double v) {
    return int_from_f64<int8_t, INT8_MIN, INT8_MAX>(v);
}
template <> __device__ __forceinline__ uint8_t from_f64<uint8_t>(double v) {
    return int_from_f64<uint8_t, 0, UINT8_MAX>(v);
}
template <> __device__ __forceinline__ Bool8 from_f64<Bool8>(double v) { return Bool8{(uint8_t)(v != 0.0)}; }

// Every element goes through f64 as in zpu, also between equal types: the
// round trip is the identity for every type except i64, whose values beyond
// 2^53 zpu's clone / toContiguous round (ops.cast returns an input of the
// requested type unchanged, ops.zig:2063: the caller does not copy then).
template <class S, class D>
__device__ __forceinline__ D convert(S x) {
    return from_f64<D>(to_f64<S>(x));
}

struct View {
    const char *data;  // element (0, .., 0)
    int32_t rank;
    int64_t dims[ZPUCUDA_MAX_RANK];
    int64_t strides[ZPUCUDA_MAX_RANK];  // elements; negative (flip) and 0 (broadcast) allowed
};

constexpr int kCopyThreads = 256;
constexpr int kTile = 64;  // transpose tile: 16 loads in flight per thread

template <class S, class D, bool CONTIG>
__global__ void __launch_bounds__(kCopyThreads) copy_gather_kernel(const __grid_constant__ View v, D *dst, int64_t n) {
    const S *src = (const S *)v.data;
    for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kCopyThreads) {
        int64_t off = i;
        if (!CONTIG) {
            int64_t rem = i;
            off = 0;
            for (int a = v.rank - 1; a >= 0; a--) {
                const int64_t d = v.dims[a];
                const int64_t q = rem / d;
                off += (rem - q * d) * v.strides[a];
                rem = q;
            }
        }
        dst[i] = convert<S, D>(src[off]);
    }
}

// View [batch..., R, C] whose axis R has unit stride and axis C stride ld:
// block (32, 8) moves one 64 x 64 tile, each warp reading 32 consecutive rows
// of a column (unit stride) and writing 32 consecutive columns of a row.
template <class S, class D>
__global__ void __launch_bounds__(256) copy_transpose_kernel(const __grid_constant__ View v, D *dst, int64_t R,
                                                                   int64_t C, int64_t ld) {
    __shared__ S tile[kTile][kTile + 1];
    const S *src = (const S *)v.data;
    for (int64_t b = blockIdx.z; true; b += gridDim.z) {
        // batch index -> offset over the leading axes
        int64_t nb = 1;
        for (int a = 0; a < v.rank - 2; a++) nb *= v.dims[a];
        if (b >= nb) break;
        int64_t rem = b, boff = 0;
        for (int a = v.rank - 3; a >= 0; a--) {
            const int64_t d = v.dims[a];
            const int64_t q = rem / d;
            boff += (rem - q * d) * v.strides[a];
            rem = q;
        }
        const int64_t r0 = (int64_t)blockIdx.y * kTile, c0 = (int64_t)blockIdx.x * kTile;
        const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
        for (int j = 0; j < kTile; j += 8)
#pragma unroll
            for (int h = 0; h < kTile; h += 32) {
                const int64_t r = r0 + tx + h, c = c0 + ty + j;
                if (r < R && c < C) tile[ty + j][tx + h] = src[boff + r + c * ld];
            }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kTile; j += 8)
#pragma unroll
            for (int h = 0; h < kTile; h += 32) {
                const int64_t r = r0 + ty + j, c = c0 + tx + h;
                if (r < R && c < C) dst[(b * R + r) * C + c] = convert<S, D>(tile[tx + h][ty + j]);
            }
        __syncthreads();
    }
}

size_t dtype_size(int dt) {
    switch (dt) {
    case 0: case 3: return 8;               // f64, i64
    case 1: case 4: return 4;               // f32, i32
    case 2: case 5: return 2;               // f16, i16
    case 6: case 7: case 8: return 1;       // i8, u8, bool
    default: return 0;
    }
}

template <class S, class D>
int launch_copy(const View &v, void *dst, int64_t n, bool contig, cudaStream_t s) {
    const int sms = num_sms();
    const int r = v.rank;
    // the tiled transpose: unit stride on the second-to-last axis, not the last
    if (r >= 2 && v.strides[r - 2] == 1 && v.strides[r - 1] != 1 && v.dims[r - 1] > 1 && v.dims[r - 2] > 1) {
        const int64_t R = v.dims[r - 2], C = v.dims[r - 1];
        int64_t nb = 1;
        for (int a = 0; a < r - 2; a++) nb *= v.dims[a];
        const int64_t gx = (C + kTile - 1) / kTile, gy = (R + kTile - 1) / kTile;
        if (gy <= 65535 && gx <= 0x7fffffff) {
            const int gz = (int)(nb < 65535 ? nb : 65535);
            copy_transpose_kernel<S, D><<<dim3((unsigned)gx, (unsigned)gy, gz), dim3(32, 8), 0, s>>>(
                v, (D *)dst, R, C, v.strides[r - 1]);
            ZC_LAUNCHED("tensor copy (tiled transpose)");
            return ZPUCUDA_OK;
        }
    }
    int64_t g = (n + kCopyThreads - 1) / kCopyThreads;
    if (g > (int64_t)sms * 16) g = (int64_t)sms * 16;
    if (contig) copy_gather_kernel<S, D, true><<<(int)g, kCopyThreads, 0, s>>>(v, (D *)dst, n);
    else copy_gather_kernel<S, D, false><<<(int)g, kCopyThreads, 0, s>>>(v, (D *)dst, n);
    ZC_LAUNCHED("tensor copy");
    return ZPUCUDA_OK;
}

template <class S>
int launch_from(const View &v, int dst_dt, void *dst, int64_t n, bool contig, cudaStream_t s) {
    switch (dst_dt) {
    case 0: return launch_copy<S, double>(v, dst, n, contig, s);
    case 1: return launch_copy<S, float>(v, dst, n, contig, s);
    case 2: return launch_copy<S, __half>(v, dst, n, contig, s);
    case 3: return launch_copy<S, int64_t>(v, dst, n, contig, s);
    case 4: return launch_copy<S, int32_t>(v, dst, n, contig, s);
    case 5: return launch_copy<S, int16_t>(v, dst, n, contig, s);
    case 6: return launch_copy<S, int8_t>(v, dst, n, contig, s);
    case 7: return launch_copy<S, uint8_t>(v, dst, n, contig, s);
    default: return launch_copy<S, Bool8>(v, dst, n, contig, s);
    }
}

}  // namespace
}  // namespace zc

using namespace zc;

extern "C" int zpucuda_tensor_copy(const zpucuda_tensor *src, zpucuda_tensor *dst, void *stream) {
    ZC_CHECK(src && dst, ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (src->rank < 0 || src->rank > ZPUCUDA_MAX_RANK) return set_error(ZPUCUDA_ERR_RANK_TOO_LARGE, "zpucuda_tensor_copy: rank");
    if (dtype_size(src->dtype) == 0 || dtype_size(dst->dtype) == 0)
        return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "zpucuda_tensor_copy: dtype code");
    if (dst->rank != src->rank) return set_error(ZPUCUDA_ERR_SHAPE_MISMATCH, "zpucuda_tensor_copy: ranks differ");
    int64_t n = 1;
    for (int a = 0; a < src->rank; a++) {
        if (src->dims[a] < 0 || dst->dims[a] != src->dims[a])
            return set_error(ZPUCUDA_ERR_SHAPE_MISMATCH, "zpucuda_tensor_copy: shapes differ");
        n *= src->dims[a];
    }
    // the output is contiguous whatever strides it came with
    int64_t st = 1;
    for (int a = src->rank - 1; a >= 0; a--) {
        dst->strides[a] = st;
        st *= src->dims[a];
    }
    if (n == 0) return ZPUCUDA_OK;
    ZC_CHECK(src->data && dst->data, ZPUCUDA_ERR_INVALID_ARGUMENT);
    View v;
    v.data = (const char *)src->data;
    v.rank = src->rank;
    bool contig = true;
    st = 1;
    for (int a = ZPUCUDA_MAX_RANK - 1; a >= 0; a--) {
        v.dims[a] = a < src->rank ? src->dims[a] : 1;
        v.strides[a] = a < src->rank ? src->strides[a] : 0;
    }
    for (int a = src->rank - 1; a >= 0; a--) {
        if (src->dims[a] != 1 && src->strides[a] != st) contig = false;
        st *= src->dims[a];
    }
    cudaStream_t s = resolve_stream(stream);
    if (contig && src->dtype == dst->dtype && src->dtype != ZPUCUDA_I64) {
        ZC_CUDA(cudaMemcpyAsync(dst->data, src->data, (size_t)n * dtype_size(src->dtype), cudaMemcpyDeviceToDevice, s));
        return ZPUCUDA_OK;
    }
    switch (src->dtype) {
    case 0: return launch_from<double>(v, dst->dtype, dst->data, n, contig, s);
    case 1: return launch_from<float>(v, dst->dtype, dst->data, n, contig, s);
    case 2: return launch_from<__half>(v, dst->dtype, dst->data, n, contig, s);
    case 3: return launch_from<int64_t>(v, dst->dtype, dst->data, n, contig, s);
    case 4: return launch_from<int32_t>(v, dst->dtype, dst->data, n, contig, s);
    case 5: return launch_from<int16_t>(v, dst->dtype, dst->data, n, contig, s);
    case 6: return launch_from<int8_t>(v, dst->dtype, dst->data, n, contig, s);
    case 7: return launch_from<uint8_t>(v, dst->dtype, dst->data, n, contig, s);
    default: return launch_from<Bool8>(v, dst->dtype, dst->data, n, contig, s);
    }
}
