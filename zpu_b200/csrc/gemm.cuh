// Batched GEMM entry points shared by the matmul front end and the kernels.
#pragma once
#include "common.cuh"

namespace zc {

constexpr int kGemmMaxBatchAxes = 6;

// The flattened batch of ops.gemmBatched (src/zpu/ops.zig:1226-1282): batch
// index -> (a, b) element offsets through per-axis strides (0 = broadcast),
// walked row-major; the output is contiguous with stride_c per matrix.
struct GemmBatch {
    int32_t nax;
    int64_t dims[kGemmMaxBatchAxes];
    int64_t sa[kGemmMaxBatchAxes];
    int64_t sb[kGemmMaxBatchAxes];
};

__host__ __device__ inline int64_t batch_count(const GemmBatch &g) {
    int64_t t = 1;
    for (int i = 0; i < g.nax; i++) t *= g.dims[i];
    return t;
}

// Element offsets of batch `bi` into A and B.
__host__ __device__ inline void batch_offsets(const GemmBatch &g, int64_t bi, int64_t *oa, int64_t *ob) {
    int64_t a = 0, b = 0;
    for (int ax = g.nax - 1; ax >= 0; ax--) {
        const int64_t d = g.dims[ax];
        const int64_t i = d ? bi % d : 0;
        bi = d ? bi / d : 0;
        a += i * g.sa[ax];
        b += i * g.sb[ax];
    }
    *oa = a;
    *ob = b;
}

// What the f32 GEMM does with each result element before storing it: the
// element-wise steps that follow a matmul in nn.dense + tanh and in the tanh
// VJP (src/zpu/nn.zig:190, src/zpu/autodiff.zig:323-330), fused so the
// product never makes an extra HBM round trip.  Each step rounds to f32 on
// its own, as zpu's ops do.
enum EpiMode : int32_t {
    EPI_STORE = 0,      // c
    EPI_BIAS_TANH = 1,  // tanh(c + bias[col])
    EPI_TANH_GRAD = 2,  // c * (1 - y*y), y = aux[row, col] (a tanh output)
    EPI_BIAS = 3,       // c + bias[col]
    EPI_SCATTER = 4,    // c, stored into the inbox of the rank that owns the row
};
constexpr int kMaxPeers = 8;
struct Epilogue {
    int32_t mode = EPI_STORE;
    const float *bias = nullptr;
    const float *aux = nullptr;
    int64_t ldaux = 0;
    // EPI_SCATTER: rank r owns rows [r * rows_per_owner, (r + 1) * rows_per_owner)
    // and receives them in peer[r] (its inbox, mapped into this process),
    // slot `src` of `world`: row i of the product lands at
    // peer[r] + (src * rows_per_owner + i - r * rows_per_owner) * ldc.
    float *peer[kMaxPeers] = {};
    int64_t rows_per_owner = 0;
    int32_t src = 0, world = 0;
    // Not EPI_SCATTER: when set, the lo half of the TF32 split of every
    // stored value is also written here (same row pitch as C), for a later
    // GEMM that takes this result as an operand (gemm_f32_device_lo).
    float *lo_out = nullptr;
};

// op(A)[m,k] @ op(B)[k,n] -> C[m,n] (ldc), per batch; trans flags as in
// zpucuda_gemm_f32.
int gemm_f32_device_epi(const float *A, const float *B, float *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                        int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                        const Epilogue &epi, cudaStream_t s);
// The same with the lo halves of the operands' TF32 split supplied (nullptr:
// none): a_lo / b_lo hold lo(x) at x's own offsets (split_lo_device, or an
// Epilogue::lo_out).  Used only where gemm_f32_presplit() holds.
int gemm_f32_device_lo(const float *A, const float *B, float *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                       int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                       const Epilogue &epi, const float *a_lo, const float *b_lo, cudaStream_t s);
// Whether an m x n product (batches matrices, one A and one B matrix) reads
// the lo halves from HBM rather than making them in shared memory.
bool gemm_f32_presplit(int64_t m, int64_t n, int64_t batches);
// lo halves of n contiguous floats (16-byte aligned x and lo).
int split_lo_device(const float *x, float *lo, int64_t n, cudaStream_t s);
int gemm_f32_device(const float *A, const float *B, float *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                    int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                    cudaStream_t s);
int gemm_f64_device(const double *A, const double *B, double *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                    int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                    cudaStream_t s);
// DType.promote (src/zpu/dtype.zig:89-104) of two element types.
int dtype_promote(int a, int b);
// The products the tensor-core GEMMs do not take (mixed operand types, f16,
// bool operands, same-type integers), with zpu's own arithmetic: ops.gemmF64
// or the integer gemmTyped loop.  C is contiguous [m, n] per matrix of type
// cdt = dtype_promote(adt, bdt).
int gemm_convert_device(const void *A, int adt, const void *B, int bdt, void *C, int cdt, int64_t m, int64_t n,
                        int64_t k, int64_t lda, int64_t ldb, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                        cudaStream_t s);

}  // namespace zc
