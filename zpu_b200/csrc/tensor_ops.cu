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
//     last (the swapLastTwo views of the matmul VJP): tiles through shared
//     memory so reads and writes both coalesce, with 16-byte global accesses
//     when the view is 16-byte aligned (f32 at the speed of a plain copy);
//   * cudaMemcpyAsync for a contiguous view of the same type (clone).
// HBM-bound: 1 read + 1 write per element.
#include <cuda_fp16.h>
#include <type_traits>

#include <string>

#include "common.cuh"
#include "tensor_ops.cuh"

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

// Rows of a view (its last axis at least kRowMin long): each row's start
// comes from one index walk over the leading axes, then its elements stream
// with the last axis's stride -- coalesced for a unit (or -1) stride, 16-byte
// loads when every row starts 16-byte aligned and the stride is 1.
constexpr int64_t kRowMin = 64;

template <class S, class D, bool VEC>
__global__ void __launch_bounds__(kCopyThreads) copy_rows_kernel(const __grid_constant__ View v, D *dst, int64_t rows,
                                                                 int64_t C) {
    const S *src = (const S *)v.data;
    const int64_t sc = v.strides[v.rank - 1];
    constexpr int VS = 16 / sizeof(S);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        int64_t rem = r, off = 0;
        for (int a = v.rank - 2; a >= 0; a--) {
            const int64_t d = v.dims[a];
            const int64_t q = rem / d;
            off += (rem - q * d) * v.strides[a];
            rem = q;
        }
        const S *srow = src + off;
        D *drow = dst + r * C;
        if (VEC) {
            for (int64_t c = (int64_t)threadIdx.x * VS; c < C; c += (int64_t)kCopyThreads * VS) {
                const uint4 x = __ldcs((const uint4 *)(srow + c));
                const S *e = reinterpret_cast<const S *>(&x);
#pragma unroll
                for (int k = 0; k < VS; k++) drow[c + k] = convert<S, D>(e[k]);
            }
        } else {
            for (int64_t c = threadIdx.x; c < C; c += kCopyThreads) drow[c] = convert<S, D>(srow[c * sc]);
        }
    }
}

// Element offset of batch b over the axes before the last two of v.
__device__ __forceinline__ int64_t batch_offset(const View &v, int64_t b) {
    int64_t off = 0;
    for (int a = v.rank - 3; a >= 0; a--) {
        const int64_t d = v.dims[a];
        const int64_t q = b / d;
        off += (b - q * d) * v.strides[a];
        b = q;
    }
    return off;
}

// View [batch..., R, C] whose axis R has unit stride and axis C stride ld:
// block (32, 8) moves one 64 x 64 tile per batch, each warp reading 32
// consecutive rows of a column (unit stride) and writing 32 consecutive
// columns of a row.  Batch b0 + blockIdx.z; no loop inside, so that the
// offsets inside the tile, taken from block-local base pointers, are not held
// across iterations (the f32 kernel stays at 32 registers, 8 blocks per SM).
template <class S, class D>
__global__ void __launch_bounds__(256) copy_transpose_kernel(const __grid_constant__ View v, D *dst, int64_t R,
                                                                   int64_t C, int64_t ld, int64_t b0) {
    __shared__ S tile[kTile][kTile + 1];
    const int64_t r0 = (int64_t)blockIdx.y * kTile, c0 = (int64_t)blockIdx.x * kTile;
    const int rr = (int)min((int64_t)kTile, R - r0), cc = (int)min((int64_t)kTile, C - c0);
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int64_t b = b0 + blockIdx.z;
    const S *s = (const S *)v.data + batch_offset(v, b) + c0 * ld + r0;
#pragma unroll
    for (int j = 0; j < kTile; j += 8)
#pragma unroll
        for (int h = 0; h < kTile; h += 32)
            if (tx + h < rr && ty + j < cc) tile[ty + j][tx + h] = s[(int64_t)(ty + j) * ld + tx + h];
    __syncthreads();
    D *d = dst + (b * R + r0) * C + c0;
#pragma unroll
    for (int j = 0; j < kTile; j += 8)
#pragma unroll
        for (int h = 0; h < kTile; h += 32)
            if (ty + j < rr && tx + h < cc) d[(int64_t)(ty + j) * C + tx + h] = convert<S, D>(tile[tx + h][ty + j]);
}

// The same transpose with 16-byte global accesses, for views that are
// 16-byte aligned: base pointers, ld, the batch strides and R multiples of
// VS = 16 / sizeof(S) elements, C a multiple of VD = 16 / sizeof(D).  On the
// load side T / VS lanes read one column (VS rows each), on the store side
// T / VD lanes write one row (VD columns each); shared accesses stay one
// element wide (pitch T + 1).  T = 64 for 4- and 8-byte sources, 128 for 1-
// and 2-byte ones (a block then still moves 16-64 KiB: 64 x 64 tiles of
// 2-byte elements left f16 at 0.58 and the byte types at 0.47 of HBM).
template <class S>
constexpr int transpose_tile() { return sizeof(S) <= 2 ? 128 : 64; }

template <class S, class D>
__global__ void __launch_bounds__(256) copy_transpose16_kernel(const __grid_constant__ View v, D *dst, int64_t R,
                                                                     int64_t C, int64_t ld, int64_t b0) {
    constexpr int T = transpose_tile<S>();
    constexpr int VS = 16 / sizeof(S), VD = 16 / sizeof(D);
    constexpr int LS = T / VS, LD = T / VD;  // lanes per column / per row
    static_assert(VS * sizeof(S) == 16 && VD * sizeof(D) == 16, "element size divides 16");
    static_assert(256 % LS == 0 && 256 % LD == 0, "whole columns / rows per pass");
    struct alignas(16) VecS { S e[VS]; };
    struct alignas(16) VecD { D e[VD]; };
    __shared__ S tile[T][T + 1];  // [column][row]
    const int64_t r0 = (int64_t)blockIdx.y * T, c0 = (int64_t)blockIdx.x * T;
    const int rr = (int)min((int64_t)T, R - r0), cc = (int)min((int64_t)T, C - c0);
    const int t = threadIdx.x;
    const int64_t b = b0 + blockIdx.z;
    const S *s = (const S *)v.data + batch_offset(v, b) + c0 * ld + r0;
    const int ql = VS * (t % LS), wl = t / LS;
#pragma unroll
    for (int j = 0; j < T; j += 256 / LS) {
        const int c = wl + j;
        if (c < cc && ql < rr) {
            const VecS x = *(const VecS *)(s + (int64_t)c * ld + ql);
#pragma unroll
            for (int k = 0; k < VS; k++) tile[c][ql + k] = x.e[k];
        }
    }
    __syncthreads();
    D *d = dst + (b * R + r0) * C + c0;
    const int qs = VD * (t % LD), ws = t / LD;
#pragma unroll
    for (int j = 0; j < T; j += 256 / LD) {
        const int r = ws + j;
        if (r < rr && qs < cc) {
            VecD y;
#pragma unroll
            for (int k = 0; k < VD; k++) y.e[k] = convert<S, D>(tile[qs + k][r]);
            *(VecD *)(d + (int64_t)r * C + qs) = y;
        }
    }
}

// One-byte elements in and out (u8, i8, bool): moving each byte through
// shared memory on its own leaves the 128 x 128 transpose bound by the SM
// (75 %).  Here a thread loads four columns' 4-byte runs (rows 4q .. 4q+3),
// transposes the 4 x 4 bytes in registers (__byte_perm) and stores four
// words, one per row, into a word tile [row][column quad]; the store side
// reads 16-byte runs of a row.  Word w of row r sits at w ^ ((r >> 2) & 31)
// (the lanes of a warp, rows 4q + i for q = 0 .. 31, then write 32
// different banks); a 16-byte run stays in one aligned group of four words,
// permuted by the low two bits of that XOR, which the reader undoes.  Same
// preconditions as copy_transpose16_kernel.
template <class S, class D>
__global__ void __launch_bounds__(256) copy_transpose_b1_kernel(const __grid_constant__ View v, D *dst, int64_t R,
                                                                      int64_t C, int64_t ld, int64_t b0) {
    static_assert(sizeof(S) == 1 && sizeof(D) == 1, "one-byte elements");
    constexpr int T = 128;
    __shared__ uint32_t tile[T][T / 4];  // [row][column quad], swizzled
    const int64_t r0 = (int64_t)blockIdx.y * T, c0 = (int64_t)blockIdx.x * T;
    const int rr = (int)min((int64_t)T, R - r0), cc = (int)min((int64_t)T, C - c0);
    const int t = threadIdx.x;
    const int64_t b = b0 + blockIdx.z;
    const uint8_t *s = (const uint8_t *)v.data + batch_offset(v, b) + c0 * ld + r0;
    uint32_t w[4][4];
#pragma unroll
    for (int u = 0; u < 4; u++) {  // block u: row quad t % 32, column quad t / 32 + 8 u
        const int q = t & 31, cq = (t >> 5) + 8 * u;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int c = 4 * cq + j;
            w[u][j] = (c < cc && 4 * q < rr) ? *(const uint32_t *)(s + (int64_t)c * ld + 4 * q) : 0u;
        }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int q = t & 31, cq = (t >> 5) + 8 * u;
        const uint32_t lo01 = __byte_perm(w[u][0], w[u][1], 0x5140), hi01 = __byte_perm(w[u][0], w[u][1], 0x7362);
        const uint32_t lo23 = __byte_perm(w[u][2], w[u][3], 0x5140), hi23 = __byte_perm(w[u][2], w[u][3], 0x7362);
        const uint32_t o[4] = {__byte_perm(lo01, lo23, 0x5410), __byte_perm(lo01, lo23, 0x7632),
                               __byte_perm(hi01, hi23, 0x5410), __byte_perm(hi01, hi23, 0x7632)};
#pragma unroll
        for (int i = 0; i < 4; i++) tile[4 * q + i][cq ^ q] = o[i];  // (r >> 2) & 31 = q for r = 4q + i
    }
    __syncthreads();
    D *d = dst + (b * R + r0) * C + c0;
#pragma unroll
    for (int u = 0; u < 4; u++) {  // 16-byte run k = t % 8 of row t / 8 + 32 u
        const int r = (t >> 3) + 32 * u, k = t & 7;
        if (r >= rr || 16 * k >= cc) continue;
        const int x = (r >> 2) & 31;
        const uint4 g = *(const uint4 *)&tile[r][(4 * k) ^ (x & ~3)];
        const uint32_t gv[4] = {g.x, g.y, g.z, g.w};
        uint32_t ow[4];
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const int sel = m ^ (x & 3);
            ow[m] = sel == 0 ? gv[0] : sel == 1 ? gv[1] : sel == 2 ? gv[2] : gv[3];
        }
        if (!std::is_same<S, D>::value) {
#pragma unroll
            for (int m = 0; m < 4; m++) {
                uint32_t y = 0;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    S xe;
                    const uint8_t byte = (uint8_t)(ow[m] >> (8 * e));
                    memcpy(&xe, &byte, 1);
                    const D de = convert<S, D>(xe);
                    uint8_t db;
                    memcpy(&db, &de, 1);
                    y |= (uint32_t)db << (8 * e);
                }
                ow[m] = y;
            }
        }
        *(uint4 *)(d + (int64_t)r * C + 16 * k) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
}

// The same for two-byte elements in and out (f16, i16): a thread loads two
// columns' 8-byte runs (rows 4q .. 4q + 3), swaps their halves into one
// word per row (__byte_perm) and stores the four words into a word tile
// [row][column pair], word w of row r at w ^ ((r >> 2) & 31); 16-byte runs
// of a row are read back as above.
template <class S, class D>
__global__ void __launch_bounds__(256) copy_transpose_b2_kernel(const __grid_constant__ View v, D *dst, int64_t R,
                                                                      int64_t C, int64_t ld, int64_t b0) {
    static_assert(sizeof(S) == 2 && sizeof(D) == 2, "two-byte elements");
    constexpr int T = 128;
    __shared__ uint32_t tile[T][T / 2];  // [row][column pair], swizzled
    const int64_t r0 = (int64_t)blockIdx.y * T, c0 = (int64_t)blockIdx.x * T;
    const int rr = (int)min((int64_t)T, R - r0), cc = (int)min((int64_t)T, C - c0);
    const int t = threadIdx.x;
    const int64_t b = b0 + blockIdx.z;
    const uint16_t *s = (const uint16_t *)v.data + batch_offset(v, b) + c0 * ld + r0;
#pragma unroll 4
    for (int u = 0; u < 8; u++) {  // block: row quad q, column pair cp
        const int idx = t + 256 * u, q = idx & 31, cp = idx >> 5;
        uint2 w[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int c = 2 * cp + j;
            w[j] = (c < cc && 4 * q < rr) ? *(const uint2 *)(s + (int64_t)c * ld + 4 * q) : make_uint2(0u, 0u);
        }
        const int x = cp ^ q;
        tile[4 * q][x] = __byte_perm(w[0].x, w[1].x, 0x5410);
        tile[4 * q + 1][x] = __byte_perm(w[0].x, w[1].x, 0x7632);
        tile[4 * q + 2][x] = __byte_perm(w[0].y, w[1].y, 0x5410);
        tile[4 * q + 3][x] = __byte_perm(w[0].y, w[1].y, 0x7632);
    }
    __syncthreads();
    D *d = dst + (b * R + r0) * C + c0;
#pragma unroll
    for (int u = 0; u < 8; u++) {  // 16-byte run k = t % 16 of row t / 16 + 16 u
        const int idx = t + 256 * u, r = idx >> 4, k = idx & 15;
        if (r >= rr || 8 * k >= cc) continue;
        const int x = (r >> 2) & 31;
        const uint4 g = *(const uint4 *)&tile[r][(4 * k) ^ (x & ~3)];
        const uint32_t gv[4] = {g.x, g.y, g.z, g.w};
        uint32_t ow[4];
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const int sel = m ^ (x & 3);
            ow[m] = sel == 0 ? gv[0] : sel == 1 ? gv[1] : sel == 2 ? gv[2] : gv[3];
        }
        if (!std::is_same<S, D>::value) {
#pragma unroll
            for (int m = 0; m < 4; m++) {
                uint32_t y = 0;
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    S xe;
                    const uint16_t h = (uint16_t)(ow[m] >> (16 * e));
                    memcpy(&xe, &h, 2);
                    const D de = convert<S, D>(xe);
                    uint16_t dh;
                    memcpy(&dh, &de, 2);
                    y |= (uint32_t)dh << (16 * e);
                }
                ow[m] = y;
            }
        }
        *(uint4 *)(d + (int64_t)r * C + 8 * k) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
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
        const int64_t R = v.dims[r - 2], C = v.dims[r - 1], ld = v.strides[r - 1];
        constexpr int64_t VS = 16 / sizeof(S), VD = 16 / sizeof(D);
        int64_t nb = 1;
        bool aligned16 = (uintptr_t)v.data % 16 == 0 && (uintptr_t)dst % 16 == 0 && R % VS == 0 && ld % VS == 0 &&
                         C % VD == 0;
        for (int a = 0; a < r - 2; a++) {
            nb *= v.dims[a];
            aligned16 = aligned16 && v.strides[a] % VS == 0;
        }
        const int64_t T = aligned16 ? transpose_tile<S>() : kTile;
        const int64_t gx = (C + T - 1) / T, gy = (R + T - 1) / T;
        if (gy <= 65535 && gx <= 0x7fffffff) {
            // one launch per 65535 batches (the grid's z limit)
            for (int64_t b0 = 0; b0 < nb; b0 += 65535) {
                const dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(nb - b0 < 65535 ? nb - b0 : 65535));
                if constexpr (sizeof(S) == 1 && sizeof(D) == 1) {
                    if (aligned16) {
                        copy_transpose_b1_kernel<S, D><<<grid, 256, 0, s>>>(v, (D *)dst, R, C, ld, b0);
                        ZC_LAUNCHED("tensor copy (tiled transpose, one-byte words)");
                        continue;
                    }
                }
                if constexpr (sizeof(S) == 2 && sizeof(D) == 2) {
                    if (aligned16) {
                        copy_transpose_b2_kernel<S, D><<<grid, 256, 0, s>>>(v, (D *)dst, R, C, ld, b0);
                        ZC_LAUNCHED("tensor copy (tiled transpose, two-byte words)");
                        continue;
                    }
                }
                if (aligned16) {
                    copy_transpose16_kernel<S, D><<<grid, 256, 0, s>>>(v, (D *)dst, R, C, ld, b0);
                    ZC_LAUNCHED("tensor copy (tiled transpose, 16-byte)");
                } else {
                    copy_transpose_kernel<S, D><<<grid, dim3(32, 8), 0, s>>>(v, (D *)dst, R, C, ld, b0);
                    ZC_LAUNCHED("tensor copy (tiled transpose)");
                }
            }
            return ZPUCUDA_OK;
        }
    }
    if (!contig && r >= 1 && v.dims[r - 1] >= kRowMin) {
        const int64_t C = v.dims[r - 1], rows = n / C;
        constexpr int64_t VS = 16 / sizeof(S);
        bool vec = v.strides[r - 1] == 1 && (uintptr_t)v.data % 16 == 0 && C % VS == 0;
        for (int a = 0; a < r - 1; a++) vec = vec && (v.dims[a] == 1 || v.strides[a] % VS == 0);
        int64_t g = rows < (int64_t)sms * 16 ? rows : (int64_t)sms * 16;
        if (vec) copy_rows_kernel<S, D, true><<<(int)g, kCopyThreads, 0, s>>>(v, (D *)dst, rows, C);
        else copy_rows_kernel<S, D, false><<<(int)g, kCopyThreads, 0, s>>>(v, (D *)dst, rows, C);
        ZC_LAUNCHED("tensor copy (rows)");
        return ZPUCUDA_OK;
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

// dst[dst view] <- src[src view], one thread per element of the shared dims.
template <class S, class D>
__global__ void __launch_bounds__(kCopyThreads) copy_view_kernel(const __grid_constant__ View v, const __grid_constant__ View w,
                                                                 int64_t n) {
    const S *src = (const S *)v.data;
    D *dst = (D *)w.data;
    for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kCopyThreads) {
        int64_t rem = i, so = 0, dof = 0;
        for (int a = v.rank - 1; a >= 0; a--) {
            const int64_t d = v.dims[a];
            const int64_t q = rem / d, idx = rem - q * d;
            so += idx * v.strides[a];
            dof += idx * w.strides[a];
            rem = q;
        }
        dst[dof] = convert<S, D>(src[so]);
    }
}

template <class T>
__global__ void __launch_bounds__(kCopyThreads) fill_kernel(T *dst, int64_t n, double v) {
    const T x = from_f64<T>(v);
    for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kCopyThreads)
        dst[i] = x;
}

// ops.take / scatterAdd index: trunc(toF64(v)), negatives counted from the
// end once; -1 when out of range
template <class I>
__device__ __forceinline__ int64_t resolve_index(I raw, int64_t sdim) {
    const double v = to_f64<I>(raw);
    if (!(v > -9.2e18 && v < 9.2e18)) return -1;  // NaN / beyond i64
    int64_t iv = (int64_t)v;                      // toward zero, as @intFromFloat
    if (iv < 0) iv += sdim;
    return (iv < 0 || iv >= sdim) ? -1 : iv;
}

template <class T, class I>
__global__ void __launch_bounds__(kCopyThreads) take_kernel(const T *x, const I *indices, T *out, int64_t outer,
                                                            int64_t sdim, int64_t inner, int64_t k, unsigned int *err) {
    const int64_t n = outer * k * inner;
    for (int64_t j = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; j < n; j += (int64_t)gridDim.x * kCopyThreads) {
        const int64_t i = j % inner, t = (j / inner) % k, o = j / (inner * k);
        const int64_t ix = resolve_index<I>(indices[t], sdim);
        if (ix < 0) {
            atomicOr(err, 1u);
            out[j] = from_f64<T>(0.0);
        } else {
            out[j] = convert<T, T>(x[(o * sdim + ix) * inner + i]);
        }
    }
}

// take with long rows (inner >= kRowMin): one block per output row (o, t),
// the index resolved once, the row copied with coalesced (16-byte when
// aligned) accesses.
template <class T, class I, bool VEC>
__global__ void __launch_bounds__(kCopyThreads) take_rows_kernel(const T *x, const I *indices, T *out, int64_t outer,
                                                                 int64_t sdim, int64_t inner, int64_t k,
                                                                 unsigned int *err) {
    constexpr int VS = 16 / sizeof(T);
    const int64_t rows = outer * k;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const int64_t t = row % k, o = row / k;
        const int64_t ix = resolve_index<I>(indices[t], sdim);
        T *orow = out + row * inner;
        if (ix < 0) {
            if (threadIdx.x == 0) atomicOr(err, 1u);
            for (int64_t c = threadIdx.x; c < inner; c += kCopyThreads) orow[c] = from_f64<T>(0.0);
            continue;
        }
        const T *xrow = x + (o * sdim + ix) * inner;
        if (VEC) {
            for (int64_t c = (int64_t)threadIdx.x * VS; c < inner; c += (int64_t)kCopyThreads * VS)
                __stcs((uint4 *)(orow + c), __ldcs((const uint4 *)(xrow + c)));
        } else {
            for (int64_t c = threadIdx.x; c < inner; c += kCopyThreads) orow[c] = convert<T, T>(xrow[c]);
        }
    }
}

// ops.scatterAdd's indices, resolved once (zpu's rule; -1 and the error word
// for one out of range).
template <class I>
__global__ void __launch_bounds__(kCopyThreads) resolve_kernel(const I *indices, int64_t k, int64_t sdim, int64_t *ix,
                                                               unsigned int *err) {
    for (int64_t t = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; t < k; t += (int64_t)gridDim.x * kCopyThreads) {
        const int64_t r = resolve_index<I>(indices[t], sdim);
        if (r < 0) atomicOr(err, 1u);
        ix[t] = r;
    }
}

// scatter_add with the target rows split into G groups (G a power of two):
// thread (g, o, i) owns the output elements (o, r, i) with r % G == g and
// walks all k updates in order, adding those that land on its rows -- each
// output element still gets its updates in zpu's order, one thread per
// element, and G threads share a column.
template <class T>
__global__ void __launch_bounds__(kCopyThreads) scatter_add_grouped_kernel(const int64_t *ix, const T *updates, T *out,
                                                                           int64_t outer, int64_t sdim, int64_t inner,
                                                                           int64_t k, int64_t G) {
    const int64_t cols = outer * inner, total = cols * G;
    for (int64_t id = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; id < total;
         id += (int64_t)gridDim.x * kCopyThreads) {
        const int64_t i = id % inner, rest = id / inner, o = rest % outer, g = rest / outer;
        for (int64_t t = 0; t < k; t++) {
            const int64_t r = __ldg(ix + t);
            if (r < 0 || (r & (G - 1)) != g) continue;
            T *d = out + (o * sdim + r) * inner + i;
            *d = from_f64<T>(to_f64<T>(*d) + to_f64<T>(updates[(o * k + t) * inner + i]));
        }
    }
}

template <class T, class I>
__global__ void __launch_bounds__(kCopyThreads) scatter_add_kernel(const I *indices, const T *updates, T *out,
                                                                   int64_t outer, int64_t sdim, int64_t inner, int64_t k,
                                                                   unsigned int *err) {
    const int64_t cols = outer * inner;
    for (int64_t c = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; c < cols; c += (int64_t)gridDim.x * kCopyThreads) {
        const int64_t o = c / inner, i = c - o * inner;
        for (int64_t t = 0; t < k; t++) {
            const int64_t ix = resolve_index<I>(indices[t], sdim);
            if (ix < 0) {
                atomicOr(err, 1u);
                continue;
            }
            T *d = out + (o * sdim + ix) * inner + i;
            *d = from_f64<T>(to_f64<T>(*d) + to_f64<T>(updates[(o * k + t) * inner + i]));
        }
    }
}

View view_of(const zpucuda_tensor &t) {
    View v;
    v.data = (const char *)t.data;
    v.rank = t.rank;
    for (int a = 0; a < ZPUCUDA_MAX_RANK; a++) {
        v.dims[a] = a < t.rank ? t.dims[a] : 1;
        v.strides[a] = a < t.rank ? t.strides[a] : 0;
    }
    return v;
}

int grid_for(int64_t n) {
    int64_t g = (n + kCopyThreads - 1) / kCopyThreads;
    if (g > (int64_t)num_sms() * 16) g = (int64_t)num_sms() * 16;
    return g < 1 ? 1 : (int)g;
}

template <class S>
int copy_view_from(const View &v, const View &w, int dst_dtype, int64_t n, cudaStream_t s) {
    const int g = grid_for(n);
    switch (dst_dtype) {
    case 0: copy_view_kernel<S, double><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    case 1: copy_view_kernel<S, float><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    case 2: copy_view_kernel<S, __half><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    case 3: copy_view_kernel<S, int64_t><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    case 4: copy_view_kernel<S, int32_t><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    case 5: copy_view_kernel<S, int16_t><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    case 6: copy_view_kernel<S, int8_t><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    case 7: copy_view_kernel<S, uint8_t><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    default: copy_view_kernel<S, Bool8><<<g, kCopyThreads, 0, s>>>(v, w, n); break;
    }
    ZC_LAUNCHED("copy_view_kernel");
    return ZPUCUDA_OK;
}

template <class T, class I>
int take_rows(const T *x, const void *indices, T *out, int64_t outer, int64_t sdim, int64_t inner, int64_t k,
              unsigned int *err, cudaStream_t s) {
    constexpr int64_t VS = 16 / sizeof(T);
    // a plain copy of the bits for every type but i64 (zpu's round trip
    // through f64), when rows start 16-byte aligned
    const bool vec = !std::is_same<T, int64_t>::value;
    const bool aligned = vec && inner % VS == 0 && (uintptr_t)x % 16 == 0 && (uintptr_t)out % 16 == 0;
    int64_t g = outer * k;
    if (g > (int64_t)num_sms() * 16) g = (int64_t)num_sms() * 16;
    if (aligned) take_rows_kernel<T, I, true><<<(int)g, kCopyThreads, 0, s>>>(x, (const I *)indices, out, outer, sdim, inner, k, err);
    else take_rows_kernel<T, I, false><<<(int)g, kCopyThreads, 0, s>>>(x, (const I *)indices, out, outer, sdim, inner, k, err);
    ZC_LAUNCHED("take_rows_kernel");
    return ZPUCUDA_OK;
}

template <class T>
int take_typed(const void *x, int idx_dtype, const void *indices, void *out, int64_t outer, int64_t sdim,
               int64_t inner, int64_t k, unsigned int *err, cudaStream_t s) {
    const int g = grid_for(outer * k * inner);
    const T *xx = (const T *)x;
    T *oo = (T *)out;
    if (inner >= kRowMin) {
        switch (idx_dtype) {
        case ZPUCUDA_I64: return take_rows<T, int64_t>(xx, indices, oo, outer, sdim, inner, k, err, s);
        case ZPUCUDA_I32: return take_rows<T, int32_t>(xx, indices, oo, outer, sdim, inner, k, err, s);
        case ZPUCUDA_F32: return take_rows<T, float>(xx, indices, oo, outer, sdim, inner, k, err, s);
        case ZPUCUDA_F64: return take_rows<T, double>(xx, indices, oo, outer, sdim, inner, k, err, s);
        default: return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "take: index dtype");
        }
    }
    switch (idx_dtype) {
    case ZPUCUDA_I64: take_kernel<T, int64_t><<<g, kCopyThreads, 0, s>>>(xx, (const int64_t *)indices, oo, outer, sdim, inner, k, err); break;
    case ZPUCUDA_I32: take_kernel<T, int32_t><<<g, kCopyThreads, 0, s>>>(xx, (const int32_t *)indices, oo, outer, sdim, inner, k, err); break;
    case ZPUCUDA_F32: take_kernel<T, float><<<g, kCopyThreads, 0, s>>>(xx, (const float *)indices, oo, outer, sdim, inner, k, err); break;
    case ZPUCUDA_F64: take_kernel<T, double><<<g, kCopyThreads, 0, s>>>(xx, (const double *)indices, oo, outer, sdim, inner, k, err); break;
    default: return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "take: index dtype");
    }
    ZC_LAUNCHED("take_kernel");
    return ZPUCUDA_OK;
}

// Groups of target rows for the grouped scatter: enough threads to fill the
// GPU (about 2^17), a power of two no larger than the rows, 1 when the
// columns alone fill it.
int64_t scatter_groups(int64_t cols, int64_t sdim) {
    int64_t G = 1;
    while (G * 2 <= sdim && cols * G * 2 <= (int64_t)1 << 17) G *= 2;
    return G;
}

template <class T>
int scatter_typed(int idx_dtype, const void *indices, const void *updates, void *out, int64_t outer, int64_t sdim,
                  int64_t inner, int64_t k, unsigned int *err, cudaStream_t s) {
    const int g = grid_for(outer * inner);
    const T *uu = (const T *)updates;
    T *oo = (T *)out;
    const int64_t G = scatter_groups(outer * inner, sdim);
    if (G > 1) {
        int64_t *ix = nullptr;
        ZC_CUDA(cudaMallocAsync((void **)&ix, (size_t)k * sizeof(int64_t), s));
        const int gr = grid_for(k);
        switch (idx_dtype) {
        case ZPUCUDA_I64: resolve_kernel<int64_t><<<gr, kCopyThreads, 0, s>>>((const int64_t *)indices, k, sdim, ix, err); break;
        case ZPUCUDA_I32: resolve_kernel<int32_t><<<gr, kCopyThreads, 0, s>>>((const int32_t *)indices, k, sdim, ix, err); break;
        case ZPUCUDA_F32: resolve_kernel<float><<<gr, kCopyThreads, 0, s>>>((const float *)indices, k, sdim, ix, err); break;
        case ZPUCUDA_F64: resolve_kernel<double><<<gr, kCopyThreads, 0, s>>>((const double *)indices, k, sdim, ix, err); break;
        default:
            cudaFreeAsync(ix, s);
            return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "scatter_add: index dtype");
        }
        ZC_LAUNCHED("resolve_kernel");
        scatter_add_grouped_kernel<T><<<grid_for(outer * inner * G), kCopyThreads, 0, s>>>(ix, uu, oo, outer, sdim, inner,
                                                                                           k, G);
        cudaError_t e = cudaGetLastError();
        cudaFreeAsync(ix, s);
        if (e != cudaSuccess) return cuda_fail(e, "scatter_add_grouped_kernel");
        count_launch();
        return ZPUCUDA_OK;
    }
    switch (idx_dtype) {
    case ZPUCUDA_I64: scatter_add_kernel<T, int64_t><<<g, kCopyThreads, 0, s>>>((const int64_t *)indices, uu, oo, outer, sdim, inner, k, err); break;
    case ZPUCUDA_I32: scatter_add_kernel<T, int32_t><<<g, kCopyThreads, 0, s>>>((const int32_t *)indices, uu, oo, outer, sdim, inner, k, err); break;
    case ZPUCUDA_F32: scatter_add_kernel<T, float><<<g, kCopyThreads, 0, s>>>((const float *)indices, uu, oo, outer, sdim, inner, k, err); break;
    case ZPUCUDA_F64: scatter_add_kernel<T, double><<<g, kCopyThreads, 0, s>>>((const double *)indices, uu, oo, outer, sdim, inner, k, err); break;
    default: return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "scatter_add: index dtype");
    }
    ZC_LAUNCHED("scatter_add_kernel");
    return ZPUCUDA_OK;
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

namespace zc {

int copy_view(const zpucuda_tensor &src, const zpucuda_tensor &dst, cudaStream_t s) {
    int64_t n = 1;
    for (int a = 0; a < src.rank; a++) n *= src.dims[a];
    if (n == 0) return ZPUCUDA_OK;
    const View v = view_of(src), w = view_of(dst);
    switch (src.dtype) {
    case 0: return copy_view_from<double>(v, w, dst.dtype, n, s);
    case 1: return copy_view_from<float>(v, w, dst.dtype, n, s);
    case 2: return copy_view_from<__half>(v, w, dst.dtype, n, s);
    case 3: return copy_view_from<int64_t>(v, w, dst.dtype, n, s);
    case 4: return copy_view_from<int32_t>(v, w, dst.dtype, n, s);
    case 5: return copy_view_from<int16_t>(v, w, dst.dtype, n, s);
    case 6: return copy_view_from<int8_t>(v, w, dst.dtype, n, s);
    case 7: return copy_view_from<uint8_t>(v, w, dst.dtype, n, s);
    default: return copy_view_from<Bool8>(v, w, dst.dtype, n, s);
    }
}

int fill_value(int dtype, void *dst, int64_t n, double v, cudaStream_t s) {
    if (n == 0) return ZPUCUDA_OK;
    const int g = grid_for(n);
    switch (dtype) {
    case 0: fill_kernel<double><<<g, kCopyThreads, 0, s>>>((double *)dst, n, v); break;
    case 1: fill_kernel<float><<<g, kCopyThreads, 0, s>>>((float *)dst, n, v); break;
    case 2: fill_kernel<__half><<<g, kCopyThreads, 0, s>>>((__half *)dst, n, v); break;
    case 3: fill_kernel<int64_t><<<g, kCopyThreads, 0, s>>>((int64_t *)dst, n, v); break;
    case 4: fill_kernel<int32_t><<<g, kCopyThreads, 0, s>>>((int32_t *)dst, n, v); break;
    case 5: fill_kernel<int16_t><<<g, kCopyThreads, 0, s>>>((int16_t *)dst, n, v); break;
    case 6: fill_kernel<int8_t><<<g, kCopyThreads, 0, s>>>((int8_t *)dst, n, v); break;
    case 7: fill_kernel<uint8_t><<<g, kCopyThreads, 0, s>>>((uint8_t *)dst, n, v); break;
    default: fill_kernel<Bool8><<<g, kCopyThreads, 0, s>>>((Bool8 *)dst, n, v); break;
    }
    ZC_LAUNCHED("fill_kernel");
    return ZPUCUDA_OK;
}

int take_launch(int dtype, const void *x, int idx_dtype, const void *indices, void *out, int64_t outer, int64_t sdim,
                int64_t inner, int64_t k, unsigned int *err, cudaStream_t s) {
    if (outer * k * inner == 0) return ZPUCUDA_OK;
    switch (dtype) {
    case 0: return take_typed<double>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    case 1: return take_typed<float>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    case 2: return take_typed<__half>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    case 3: return take_typed<int64_t>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    case 4: return take_typed<int32_t>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    case 5: return take_typed<int16_t>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    case 6: return take_typed<int8_t>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    case 7: return take_typed<uint8_t>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    default: return take_typed<Bool8>(x, idx_dtype, indices, out, outer, sdim, inner, k, err, s);
    }
}

int scatter_add_launch(int dtype, int idx_dtype, const void *indices, const void *updates, void *out, int64_t outer,
                       int64_t sdim, int64_t inner, int64_t k, unsigned int *err, cudaStream_t s) {
    ZC_CUDA(cudaMemsetAsync(out, 0, (size_t)(outer * sdim * inner) * dtype_size(dtype), s));
    if (outer * inner == 0 || k == 0) return ZPUCUDA_OK;
    switch (dtype) {
    case 0: return scatter_typed<double>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    case 1: return scatter_typed<float>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    case 2: return scatter_typed<__half>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    case 3: return scatter_typed<int64_t>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    case 4: return scatter_typed<int32_t>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    case 5: return scatter_typed<int16_t>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    case 6: return scatter_typed<int8_t>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    case 7: return scatter_typed<uint8_t>(idx_dtype, indices, updates, out, outer, sdim, inner, k, err, s);
    default: return set_error(ZPUCUDA_ERR_DTYPE_MISMATCH, "scatter_add on bool");
    }
}

}  // namespace zc
