// f64 GEMM on the FP64 DMMA path (mma.sync m16n8k4 .f64) for sm_100a.
//
// Replaces kernels.gemm / ops.gemmTyped for f64 (src/zpu/kernels.zig:339-408,
// src/zpu/ops.zig:1016-1049) and ops.gemmBatched (ops.zig:1226-1282).
// tcgen05 has no f64 kind, so the double-precision tensor path on Blackwell is
// the warp-level DMMA.  Design:
//   * 128 x 128 block tile, BK = 16, 256 threads as 2 x 4 warps of 64 x 32;
//     each warp issues 16 m16n8k4 MMAs per k-step of 4 from registers;
//   * a 4-stage cp.async pipeline (16-byte copies when every row start is
//     16-byte aligned, 8-byte otherwise) with zero-fill at the edges;
//   * shared-memory row pitches padded (20 / 136 doubles) so every fragment
//     load of a warp hits each 8-byte bank exactly twice (no conflicts);
//   * transposed operands (the matmul VJP's swapLastTwo views) are read in
//     place by swapping the tile fill, never materialised;
//   * blockIdx.z walks the broadcast batch of ops.gemmBatched.
#include <string.h>

#include "gemm.cuh"

namespace zc {

namespace {

constexpr int BM = 128, BN = 128, BK = 16, STAGES = 4, THREADS = 256;
constexpr int PAD_K = BK + 4;    // pitch of a [rows][k] tile (doubles)
constexpr int PAD_MN = BM + 8;   // pitch of a [k][rows] tile (doubles)
constexpr int TILE_DOUBLES = (BM * PAD_K > BK * PAD_MN) ? BM * PAD_K : BK * PAD_MN;
constexpr size_t SMEM_BYTES = (size_t)STAGES * 2 * TILE_DOUBLES * sizeof(double);

__device__ __forceinline__ void cp_async(double *dst, const double *src, bool valid, int bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
    const int n = valid ? bytes : 0;
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(src), "r"(n));
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void dmma(double (&c)[4], double a0, double a1, double b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
        : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
        : "d"(a0), "d"(a1), "d"(b0));
}

// Fills one [rows x k] (K_MAJOR) or [k x rows] tile of an operand.
//   K_MAJOR: element (r, kk) at src[(r0 + r) * ld + k0 + kk], smem pitch PAD_K
//   else:    element (kk, r) at src[(k0 + kk) * ld + r0 + r], smem pitch PAD_MN
template <bool K_MAJOR, int VEC>
__device__ __forceinline__ void fill_tile(double *sm, const double *src, int64_t ld, int64_t rows_total,
                                          int64_t k_total, int64_t r0, int64_t k0) {
    if (K_MAJOR) {
        constexpr int CPR = BK / VEC;  // chunks per row
        for (int c = threadIdx.x; c < BM * CPR; c += THREADS) {
            const int r = c / CPR, kc = (c % CPR) * VEC;
            const int64_t gr = r0 + r, gk = k0 + kc;
            const bool ok = gr < rows_total && gk < k_total;
            cp_async(sm + r * PAD_K + kc, ok ? src + gr * ld + gk : src, ok, VEC * 8);
        }
    } else {
        constexpr int CPR = BM / VEC;
        for (int c = threadIdx.x; c < BK * CPR; c += THREADS) {
            const int kk = c / CPR, rc = (c % CPR) * VEC;
            const int64_t gk = k0 + kk, gr = r0 + rc;
            const bool ok = gk < k_total && gr < rows_total;
            cp_async(sm + kk * PAD_MN + rc, ok ? src + gk * ld + gr : src, ok, VEC * 8);
        }
    }
}

template <bool TA, bool TB, int VEC>
__global__ void __launch_bounds__(THREADS, 1)
    dgemm_kernel(const double *__restrict__ A, const double *__restrict__ B, double *__restrict__ C, int64_t M,
                 int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc, const __grid_constant__ GemmBatch bt,
                 int64_t stride_c) {
    extern __shared__ __align__(16) double smem[];
    double *sA = smem;
    double *sB = smem + STAGES * TILE_DOUBLES;

    int64_t oa, ob;
    batch_offsets(bt, blockIdx.z, &oa, &ob);
    A += oa;
    B += ob;
    C += (int64_t)blockIdx.z * stride_c;
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;

    double acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int q = 0; q < 4; q++) acc[i][j][q] = 0.0;

    const int KT = (int)((K + BK - 1) / BK);
    auto load = [&](int stage, int kt) {
        const int64_t k0 = (int64_t)kt * BK;
        // A: op(A) is [M, K]; stored [M, K] (K-major) or, transposed, [K, M]
        fill_tile<!TA, VEC>(sA + stage * TILE_DOUBLES, A, lda, M, K, m0, k0);
        // B: op(B) is [K, N]; stored [K, N] (N-major) or, transposed, [N, K]
        fill_tile<TB, VEC>(sB + stage * TILE_DOUBLES, B, ldb, N, K, n0, k0);
    };
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < KT) load(s, s);
        cp_commit();
    }
    for (int kt = 0; kt < KT; kt++) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        {
            const int nk = kt + STAGES - 1;
            if (nk < KT) load(nk % STAGES, nk);
            cp_commit();
        }
        const double *a_s = sA + (kt % STAGES) * TILE_DOUBLES;
        const double *b_s = sB + (kt % STAGES) * TILE_DOUBLES;
#pragma unroll
        for (int kk = 0; kk < BK; kk += 4) {
            double af[4][2], bf[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = wm + i * 16 + g, c = kk + t;
                if (!TA) {
                    af[i][0] = a_s[r * PAD_K + c];
                    af[i][1] = a_s[(r + 8) * PAD_K + c];
                } else {
                    af[i][0] = a_s[c * PAD_MN + r];
                    af[i][1] = a_s[c * PAD_MN + r + 8];
                }
            }
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int cn = wn + j * 8 + g, r = kk + t;
                bf[j] = TB ? b_s[cn * PAD_K + r] : b_s[r * PAD_MN + cn];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) dmma(acc[i][j], af[i][0], af[i][1], bf[j]);
        }
    }
    cp_wait<0>();

    // epilogue: the m16n8 accumulator layout (rows g / g+8, columns 2t, 2t+1)
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t col = n0 + wn + j * 8 + 2 * t;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int64_t row = m0 + wm + i * 16 + g + h * 8;
                if (row >= M) continue;
                double *dst = C + row * ldc + col;
                if (col + 1 < N && ((((uintptr_t)dst) & 15) == 0)) {
                    *(double2 *)dst = make_double2(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
                } else {
                    if (col < N) dst[0] = acc[i][j][2 * h];
                    if (col + 1 < N) dst[1] = acc[i][j][2 * h + 1];
                }
            }
        }
}

template <bool TA, bool TB, int VEC>
int launch(const double *A, const double *B, double *C, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
           int64_t ldc, const GemmBatch &bt, int64_t stride_c, int64_t batches, cudaStream_t s) {
    auto kern = dgemm_kernel<TA, TB, VEC>;
    // the attribute belongs to the current device: set once per device
    static bool attr[64] = {false};
    const int dev = current_device();
    if (dev < 0 || dev >= 64 || !attr[dev]) {
        ZC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
        if (dev >= 0 && dev < 64) attr[dev] = true;
    }
    dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM), (unsigned)batches);
    kern<<<grid, THREADS, SMEM_BYTES, s>>>(A, B, C, m, n, k, lda, ldb, ldc, bt, stride_c);
    ZC_LAUNCHED("dgemm_kernel");
    return ZPUCUDA_OK;
}

}  // namespace

int gemm_f64_device(const double *A, const double *B, double *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                    int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                    cudaStream_t s) {
    const int64_t batches = batch_count(bt);
    if (m == 0 || n == 0 || batches == 0) return ZPUCUDA_OK;
    if (!C || ldc < n) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if (k == 0) {  // kernels.zig:346-349: an empty contraction writes zeros
        for (int64_t b = 0; b < batches; b++)
            ZC_CUDA(cudaMemset2DAsync(C + b * stride_c, ldc * sizeof(double), 0, n * sizeof(double), m, s));
        return ZPUCUDA_OK;
    }
    if (!A || !B) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if ((!ta && lda < k) || (ta && lda < m) || (!tb && ldb < n) || (tb && ldb < k))
        return ZPUCUDA_ERR_INVALID_SHAPE;
    if (batches > 65535 || (m + BM - 1) / BM > 65535) return ZPUCUDA_ERR_NOT_SUPPORTED;
    // 16-byte copies need every row start of both operands 16-byte aligned
    // and the contiguous extent even (no chunk may straddle the edge)
    bool v2 = ((uintptr_t)A % 16 == 0) && ((uintptr_t)B % 16 == 0) && lda % 2 == 0 && ldb % 2 == 0 &&
              (ta ? m : k) % 2 == 0 && (tb ? k : n) % 2 == 0;
    for (int i = 0; i < bt.nax; i++) v2 = v2 && bt.sa[i] % 2 == 0 && bt.sb[i] % 2 == 0;
#define ZC_DG(TA_, TB_)                                                                                        \
    return v2 ? launch<TA_, TB_, 2>(A, B, C, m, n, k, lda, ldb, ldc, bt, stride_c, batches, s)                 \
              : launch<TA_, TB_, 1>(A, B, C, m, n, k, lda, ldb, ldc, bt, stride_c, batches, s)
    if (!ta && !tb) ZC_DG(false, false);
    if (!ta && tb) ZC_DG(false, true);
    if (ta && !tb) ZC_DG(true, false);
    ZC_DG(true, true);
#undef ZC_DG
}

}  // namespace zc
