// f32 GEMM for sm_100a: tcgen05 tensor cores with a 3xTF32 split.
//
// Replaces kernels.gemm / ops.gemmTyped for f32 (src/zpu/kernels.zig:339-408,
// src/zpu/ops.zig:1016-1049) and ops.gemmBatched (ops.zig:1226-1282).
// zpu computes each element as an f32 FMA chain; TF32 keeps 10 mantissa
// bits, so every operand is split x = hi + lo with hi, lo exact TF32 values
// and C = A_hi B_hi + A_hi B_lo + A_lo B_hi (the lo*lo term is below f32
// resolution): three tensor-core MMAs per K step.  hi is the f32 operand as
// loaded: the tensor core reads f32 data as TF32 by ignoring the 13 low
// mantissa bits (truncation), so only lo = x - trunc(x) is computed.
//
// The tensor core's own f32 accumulation drifts with the number of MMAs it
// chains (measured: relative error growing linearly with K, 3e-5 at
// K = 4096), so the K loop is cut into chunks of KC_BLOCKS * 32: each chunk
// accumulates in one of two TMEM buffers, and folding warps add finished
// chunks into a running sum (a third TMEM region) with round-to-nearest f32
// adds while the tensor core fills the other buffer.
//
// Where lo comes from is the kernel's main limit.  Made in shared memory,
// per 32-wide K slice the TMA writes 32 KiB, making lo reads 32 and writes
// 32, and the three MMAs read 96; so every warp that is not the producer or
// the MMA issuer converts, raw tiles have a deeper ring than lo tiles, and
// the hi tiles are never rewritten.  (Feeding A from TMEM instead --
// tcgen05.mma with a TMEM A operand, hi and lo written by tcgen05.st -- cuts
// the traffic to 128 KiB but measured slower: that pipeline peaked at 180
// TFLOP/s even without conversion, against 220 for this one.)  Where every
// operand element takes part in many products, a split pass writes lo into
// HBM once per operand (split_lo_kernel, or a producing GEMM's epilogue) and
// the PRE form of the kernel TMA-loads the lo tiles beside the hi ones: no
// conversion at all (8192^3: 223 against 178 TFLOP/s, the pass included).
// Both forms give the same bits.
//
// One CTA computes a 128 x BN tile (BN = 128 or 256, chosen per problem by
// how the tiles fill the SMs; the Tile struct has the differences) with 16
// warps:
//   warp 0      TMA producer: 3-D tensor maps (inner, rows, matrix) stream
//               32-wide K slices of A and B into RAW shared-memory stages
//               (out-of-range rows/columns read as zero);
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (kind::tf32) and
//               the tcgen05.commits;
//   warps 2-15  write lo of each landed stage into one of LO lo slots at the
//               same (swizzled) position, so hi and lo tiles share their
//               descriptor layout (idle in the PRE form);
//   warps 8-15  also fold each finished chunk (tcgen05.ld / tcgen05.st
//               32x32b) whenever they wait, then store the tile (32 x 32
//               boxes through TMA stores where C has a tensor map); warp w
//               owns TMEM lanes 32 (w % 4) .. +31 and columns BN/2
//               ((w - 8) / 4) .. + BN/2 - 1.
// TMEM columns: chunk accumulators below 256, running sum from 256.
// K-major operands use the 128-byte swizzle; MN-major ones (the matmul VJP's
// swapLastTwo views, read in place) use the 128-byte swizzle with 32-byte
// atoms, the only shared-memory layout tcgen05 takes for MN-major TF32.
// Every mbarrier wait is bounded: a wait that runs out sets an error word
// (zpucuda_check_device) and its warp stops; TMEM is freed before exit.
//
// Few output tiles split K over a thread-block cluster whose CTAs add their
// partials through distributed shared memory; many tiles over a short K run
// a persistent form (tf32x3_gemm_persistent_kernel); contractions of k <= 32
// run zpu's own chain on CUDA cores (smallk_gemm_kernel).  Shapes the tensor
// maps cannot describe (row pitch not a multiple of 4 elements, base not
// 16-byte aligned, batch offsets that are not whole matrices) run a plain
// FMA-chain kernel instead.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "gemm.cuh"
#include "region.cuh"

namespace zc {

static __device__ unsigned int g_gemm_error;

namespace {

constexpr int BM = 128, BK = 32, THREADS = 512;
constexpr int NWORK = 14;   // converter warps (2-15)
constexpr int NFOLD = 256;  // folding / storing threads (warps 8-15)
constexpr uint32_t A_BYTES = BM * BK * 4;  // 16 KiB
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t SUM_COL = 256;  // the running sum starts at TMEM column 256

// The two tile shapes, 128 x BN.
//   BN = 128: two chunk accumulators (TMEM columns 0-127, 128-255), so the
//             tensor core never waits for a fold; 4 raw stages.
//   BN = 256: one chunk accumulator (columns 0-255) and 256-wide K chunks
//             (the tensor core waits for each fold, ~4% of the time); 2 raw
//             stages.  Half the shared-memory traffic per flop for A, hence
//             ~14% faster where the tile count fills the SMs.
//   PRE:      the lo halves come from HBM (split_lo_kernel wrote them once per
//             operand), so a stage holds A, B, A lo and B lo, loaded by the
//             TMA together; no converter work and no lo slots: 3 stages of
//             64 KiB (BN = 128) or 2 of 96 KiB (BN = 256).
template <int BN_, bool PRE_ = false>
struct Tile {
    static constexpr int BN = BN_;
    static constexpr int NBUF = BN_ == 128 ? 2 : 1;
    static constexpr int KC_BLOCKS = BN_ == 128 ? 4 : 8;  // K-slices per accumulation chunk
    static constexpr int RAW = PRE_ ? (BN_ == 128 ? 3 : 2) : (BN_ == 128 ? 4 : 2);  // stages
    static constexpr int LO = PRE_ ? 0 : 2;               // slots of lo tiles made in shared memory
    static constexpr uint32_t B_BYTES = BN_ * BK * 4;
    static constexpr uint32_t RAW_BYTES = A_BYTES + B_BYTES;  // A + B of one K slice
    static constexpr uint32_t STAGE_BYTES = PRE_ ? 2 * RAW_BYTES : RAW_BYTES;
    static constexpr int CONV_ITERS = (RAW_BYTES / 16 + NWORK * 32 - 1) / (NWORK * 32);
    static constexpr size_t SMEM_BYTES = (size_t)RAW * STAGE_BYTES + (size_t)LO * RAW_BYTES + 1024;  // + alignment slack
    static constexpr int FOLD_COLS = BN_ / 2;  // columns per folding thread
    // split-K: the CTA's partial tile in its own shared memory, rows padded
    // by 4 floats (a warp's float4 stores then take the minimum 4 wavefronts)
    static constexpr int XPITCH = BN_ + 4;
    static_assert(NBUF * BN_ <= (int)SUM_COL && SUM_COL + BN_ <= TMEM_COLS, "TMEM columns");
    static_assert((size_t)BM * XPITCH * 4 + 1024 <= SMEM_BYTES, "split-K partial fits the pipeline buffers");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};
constexpr uint32_t kGemmSpin = 1u << 24;

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mb_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void mb_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t parity) {
    for (uint32_t i = 0; i < kGemmSpin; i++) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(su32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    atomicOr(&g_gemm_error, 1u);
    return false;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(su32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(su32(bar))
        : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The generic address of this CTA's shared-memory object `p` in CTA `rank`
// of the cluster (plain loads through it read that CTA's shared memory).
__device__ __forceinline__ const void *cluster_map_generic(const void *p, uint32_t rank) {
    uint64_t r;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"((uint64_t)p), "r"(rank));
    return (const void *)r;
}

// TMA store of a 32 x 32 f32 box (128-byte swizzled in shared memory) at
// (x, y, z) of `map`; out-of-range rows and columns are not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
                 "r"(su32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Until at most N of this thread's committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Shared-memory matrix descriptor (sm_100, version 1).  layout: 2 = 128-byte
// swizzle, 1 = 128-byte swizzle with 32-byte atoms.
__device__ __forceinline__ uint64_t sdesc(const void *p, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return (uint64_t)((su32(p) >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Descriptor of the 8-element K step `kk` of a staged operand tile.
//   K-major tile [rows][32] (128-byte swizzle): SBO = 1024 (8 rows),
//   step = 32 bytes.
//   MN-major tile of 32-wide chunks [chunk][32 k][32] (32-byte-atom swizzle):
//   LBO = 4096 (next MN chunk), SBO = 512 (next 4 k-rows), step = 1024 bytes.
template <bool KMAJOR>
__device__ __forceinline__ uint64_t op_desc(const uint8_t *tile, int kk) {
    return KMAJOR ? sdesc(tile + kk * 32, 16, 1024, 2) : sdesc(tile + kk * 1024, 4096, 512, 1);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u));
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32p(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) { tmem_ld32p(taddr, v); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mb_test(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// One try_wait with a short suspend hint (ns): true when the phase is done.
__device__ __forceinline__ bool mb_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity), "r"(200u)
        : "memory");
    return ok != 0;
}

// The lo half of the TF32 split of four f32 values: x - trunc_tf32(x)
// (exact in f32), rounded to nearest TF32.  The hi half is x itself: the
// tensor core reads an f32 operand as TF32 by ignoring its 13 low mantissa
// bits, i.e. it truncates.  Infinities get lo = 0 (so inf * b stays inf);
// NaN gives lo = NaN.
__device__ __forceinline__ uint4 lo4(const uint4 &x) {
    uint4 out;
    const uint32_t *v = &x.x;
    uint32_t *l = &out.x;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t hi = v[i] & 0xFFFFE000u;
        const float rest = __fsub_rn(__uint_as_float(v[i]), __uint_as_float(hi));
        uint32_t r;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(rest));
        l[i] = ((v[i] & 0x7FFFFFFFu) == 0x7F800000u) ? 0u : r;
    }
    return out;
}

__device__ __forceinline__ float lo1(float x) {
    const uint4 v = lo4(make_uint4(__float_as_uint(x), 0u, 0u, 0u));
    return __uint_as_float(v.x);
}

// The lo halves of an operand stored as (inner, rows, nmats) with row pitch
// ld and matrix pitch mat, written at the same offsets of `lo`: one
// HBM-bound pass per operand, so the GEMM's tensor map for lo has the
// operand's own geometry and the GEMM makes no lo in shared memory.
__global__ void __launch_bounds__(256) split_lo_kernel(const float *__restrict__ x, float *__restrict__ lo,
                                                       int64_t inner, int64_t rows, int64_t nmats, int64_t ld,
                                                       int64_t mat) {
    const int64_t stride = (int64_t)gridDim.x * 256;
    if (ld == inner && (nmats == 1 || mat == rows * ld)) {  // one contiguous range
        const int64_t n = inner * rows * nmats, n4 = n >> 2;
        for (int64_t t = (int64_t)blockIdx.x * 256 + threadIdx.x; t < n4; t += stride)
            __stcs((uint4 *)lo + t, lo4(__ldcs((const uint4 *)x + t)));
        for (int64_t t = (n4 << 2) + (int64_t)blockIdx.x * 256 + threadIdx.x; t < n; t += stride) lo[t] = lo1(x[t]);
        return;
    }
    const int64_t v4 = (inner + 3) >> 2;  // 16-byte groups per row; the last may be partial
    const int64_t total = v4 * rows * nmats;
    for (int64_t t = (int64_t)blockIdx.x * 256 + threadIdx.x; t < total; t += stride) {
        const int64_t g = t % v4, rz = t / v4;
        const int64_t off = (rz / rows) * mat + (rz % rows) * ld + g * 4;  // ld, mat: multiples of 4
        if (g * 4 + 4 <= inner) {
            __stcs((uint4 *)(lo + off), lo4(__ldcs((const uint4 *)(x + off))));
        } else {
            for (int64_t i = g * 4; i < inner; i++) lo[off + i - g * 4] = lo1(x[off + i - g * 4]);
        }
    }
}

// Folds accumulation chunk q (TMEM buffer q % NBUF) into the running sum at
// SUM_COL with round-to-nearest f32 adds; this warp's 32 lanes, columns
// half * FOLD_COLS .. + FOLD_COLS - 1 (those inside the MMA width).
template <int BN_>
__device__ __forceinline__ void fold_chunk(uint32_t tmem, uint32_t lanes, int q, int half, int nmma, int buf = -1) {
    using T = Tile<BN_>;
    if (buf < 0) buf = q % T::NBUF;
    asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
    for (int c = 0; c < T::FOLD_COLS / 32; c++) {
        const int col = half * T::FOLD_COLS + c * 32;
        if (col >= nmma) continue;
        float v[32];
        tmem_ld32(tmem + lanes + (uint32_t)(buf * BN_ + col), v);
        if (q > 0) {
            float sum[32];
            tmem_ld32(tmem + lanes + SUM_COL + (uint32_t)col, sum);
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = __fadd_rn(sum[i], v[i]);
        }
        tmem_st32(tmem + lanes + SUM_COL + (uint32_t)col, v);
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
}

struct Maps {
    CUtensorMap a, b;
    CUtensorMap alo, blo;  // the lo halves (PRE kernels only)
    CUtensorMap c, clo;    // C and the epilogue's lo output, for the TMA tile store
};

struct Params {
    const float *A, *B;  // the operands as stored (the non-finite recompute reads them)
    int64_t lda, ldb;
    int64_t M, N, K, ldc, stride_c;
    int64_t mat_a, mat_b;  // elements between the matrices the tensor maps index
    int32_t nmma;          // MMA width: N rounded up to 16, at most BN
    int32_t group;         // row tiles per raster group (0: blockIdx order)
    uint32_t idesc;
    int32_t splits;        // K split across a cluster of this many CTAs (blockIdx.z = batch * splits + split)
    int32_t kb_per_split;  // 32-wide K slices per split
    int32_t tma_store;     // the tile leaves through maps.c (and maps.clo when epi.lo_out)
    int64_t batches;       // matrices of the flattened batch
    Epilogue epi;
    GemmBatch bt;
};

// instruction descriptor: f32 accumulate, tf32 A and B, majors, N, M
uint32_t make_idesc(bool ta, bool tb, int nmma) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((ta ? 1u : 0u) << 15) | ((tb ? 0u : 1u) << 16) |
           ((uint32_t)(nmma >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// zpu's own chain for one element (kernels.gemm, src/zpu/kernels.zig:369-400):
// c = 0, then for p = k0 .. k1-1 in order c = fma(a[row,p], b[p,col], c) --
// except for the nb % 8 columns past the last whole 8-lane vector of their
// 128-column panel, where zpu adds a separate product (row[j] += a * b).
// The tensor-core path hands an element here when its 3xTF32 result is not
// finite: an infinite operand meets a zero low TF32 half of its partner
// (inf * 0 = NaN in the hi x lo product), or the sum overflows.  zpu's chain
// then gives the exact inf / NaN it gives on the CPU.
template <bool TA, bool TB>
__device__ __noinline__ float zpu_chain_element(const float *A, const float *B, int64_t lda, int64_t ldb, int64_t row,
                                                int64_t col, int64_t N, int64_t k0, int64_t k1) {
    const int64_t jb = col & ~(int64_t)127;
    const int64_t nb = N - jb < 128 ? N - jb : 128;
    const bool fused = col - jb < (nb & ~(int64_t)7);
    float c = 0.0f;
    for (int64_t p = k0; p < k1; p++) {
        const float a = TA ? A[p * lda + row] : A[row * lda + p];
        const float b = TB ? B[col * ldb + p] : B[p * ldb + col];
        c = fused ? fmaf(a, b, c) : __fadd_rn(c, __fmul_rn(a, b));
    }
    return c;
}

// One result element through the epilogue (the element is at row, col of C).
__device__ __forceinline__ float epi_apply(const Epilogue &e, float c, int64_t row, int64_t col) {
    if (e.mode == EPI_BIAS_TANH) return zc_tanhf(__fadd_rn(c, e.bias[col]));
    if (e.mode == EPI_BIAS) return __fadd_rn(c, e.bias[col]);
    if (e.mode == EPI_TANH_GRAD) {
        const float y = e.aux[row * e.ldaux + col];
        return __fmul_rn(c, __fsub_rn(1.0f, __fmul_rn(y, y)));
    }
    return c;
}

// The epilogue on 32 consecutive columns of one row, all inside C.
__device__ __forceinline__ void epi_apply32(const Epilogue &e, float (&acc)[32], int64_t row, int64_t col0) {
    if (e.mode == EPI_STORE || e.mode == EPI_SCATTER) return;
    if (e.mode == EPI_TANH_GRAD) {
        const float *y = e.aux + row * e.ldaux + col0;
        if ((((uintptr_t)y) & 15) == 0) {
#pragma unroll
            for (int v = 0; v < 8; v++) {
                const float4 q = __ldg((const float4 *)y + v);
                acc[4 * v] = __fmul_rn(acc[4 * v], __fsub_rn(1.0f, __fmul_rn(q.x, q.x)));
                acc[4 * v + 1] = __fmul_rn(acc[4 * v + 1], __fsub_rn(1.0f, __fmul_rn(q.y, q.y)));
                acc[4 * v + 2] = __fmul_rn(acc[4 * v + 2], __fsub_rn(1.0f, __fmul_rn(q.z, q.z)));
                acc[4 * v + 3] = __fmul_rn(acc[4 * v + 3], __fsub_rn(1.0f, __fmul_rn(q.w, q.w)));
            }
        } else {
#pragma unroll
            for (int v = 0; v < 32; v++) acc[v] = __fmul_rn(acc[v], __fsub_rn(1.0f, __fmul_rn(y[v], y[v])));
        }
        return;
    }
    const float *b = e.bias + col0;
    if (e.mode == EPI_BIAS_TANH) {
#pragma unroll
        for (int v = 0; v < 32; v++) acc[v] = zc_tanhf(__fadd_rn(acc[v], __ldg(b + v)));
    } else {
#pragma unroll
        for (int v = 0; v < 32; v++) acc[v] = __fadd_rn(acc[v], __ldg(b + v));
    }
}

// Split-K inside a cluster: the `splits` CTAs of one output tile are one
// thread-block cluster, each holding its raw partial tile in its own shared
// memory.  CTA `rank` sums rows [128 rank / splits, 128 (rank + 1) / splits)
// of the tile over all partials, read through distributed shared memory and
// added in split order (deterministic, the same order for every element),
// recomputes non-finite sums with zpu's chain, applies the epilogue and
// stores.  No scratch in HBM and no second kernel.  Each thread first loads
// and adds all its elements (KR float4 per partial, loads of a partial in
// flight together), then tells the cluster it is done reading, and stores
// while the other CTAs finish; it waits for them only before it exits (its
// own partial must stay until every CTA has read it).  The caller has
// arrived on the cluster barrier once its partial was in place.
template <bool TA, bool TB, int BN_>
__device__ __forceinline__ void splitk_cluster_reduce(const uint8_t *smem, float *C, const Params &P, int64_t oa,
                                                   int64_t ob, int64_t bz, int m0, int n0) {
    constexpr int XPITCH = Tile<BN_>::XPITCH, C4 = BN_ / 4;
    constexpr int KR = (BM * C4 / 2 + THREADS - 1) / THREADS;  // float4 per thread at 2 splits (the most)
    static_assert(KR % 4 == 0, "loads go in groups of four");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // every partial is in place
    const int S = P.splits;
    const int rank = (int)cluster_rank();
    const int r0 = BM * rank / S, r1 = BM * (rank + 1) / S, n4 = (r1 - r0) * C4;
    float4 acc[KR];
    for (int sp = 0; sp < S; sp++) {
        const float *part = (const float *)cluster_map_generic(smem, (uint32_t)sp);
#pragma unroll
        for (int g = 0; g < KR; g += 4) {  // four loads in flight, then their adds
            float4 b[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = (int)threadIdx.x + (g + u) * THREADS;
                if (i < n4) b[u] = *(const float4 *)(part + (r0 + i / C4) * XPITCH + (i % C4) * 4);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (sp == 0) {
                    acc[g + u] = b[u];
                } else {
                    acc[g + u].x = __fadd_rn(acc[g + u].x, b[u].x);
                    acc[g + u].y = __fadd_rn(acc[g + u].y, b[u].y);
                    acc[g + u].z = __fadd_rn(acc[g + u].z, b[u].z);
                    acc[g + u].w = __fadd_rn(acc[g + u].w, b[u].w);
                }
            }
        }
    }
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");  // done reading the partials
    float *cm = C + bz * P.stride_c;
#pragma unroll
    for (int u = 0; u < KR; u++) {
        const int i = (int)threadIdx.x + u * THREADS;
        if (i >= n4) break;
        const int64_t row = (int64_t)m0 + r0 + i / C4, col0 = (int64_t)n0 + (i % C4) * 4;
        if (row >= P.M || col0 >= P.N) continue;
        float v[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            if (col0 + e >= P.N) break;
            if (!isfinite(v[e]))
                v[e] = zpu_chain_element<TA, TB>(P.A + oa, P.B + ob, P.lda, P.ldb, row, col0 + e, P.N, 0, P.K);
            v[e] = epi_apply(P.epi, v[e], row, col0 + e);
        }
        float *crow = cm + row * P.ldc;
        if (col0 + 4 <= P.N && (((uintptr_t)(crow + col0)) & 15) == 0) {
            *(float4 *)(crow + col0) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (col0 + e < P.N) crow[col0 + e] = v[e];
        }
        if (P.epi.lo_out) {
            float *lrow = P.epi.lo_out + row * P.ldc;
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (col0 + e < P.N) lrow[col0 + e] = lo1(v[e]);
        }
    }
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // no CTA leaves while another still reads
}

template <bool TA, bool TB, int BN_, bool PRE>
__global__ void __launch_bounds__(THREADS, 1)
    tf32x3_gemm_kernel(const __grid_constant__ Maps maps, float *__restrict__ C, const __grid_constant__ Params P) {
    using T = Tile<BN_, PRE>;
    constexpr int BN = BN_, RAW = T::RAW, LO = T::LO, NBUF = T::NBUF, KC_BLOCKS = T::KC_BLOCKS;
    constexpr uint32_t B_BYTES = T::B_BYTES, RAW_BYTES = T::RAW_BYTES, STAGE_BYTES = T::STAGE_BYTES;
    constexpr int NLO = LO > 0 ? LO : 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[RAW], empty[RAW], conv[NLO], lofree[NLO], tfull[NBUF], tfree[NBUF];
    __shared__ uint32_t tmem_base;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t oa, ob;
    const int split = (int)(blockIdx.z % (unsigned)P.splits);
    const int64_t bz = blockIdx.z / (unsigned)P.splits;
    batch_offsets(P.bt, bz, &oa, &ob);
    const int za = (int)(P.mat_a ? oa / P.mat_a : 0), zb = (int)(P.mat_b ? ob / P.mat_b : 0);
    // tile origin: with P.group > 0 the CTAs (launched x fastest) sweep
    // groups of P.group row tiles column by column, so the A and B panels a
    // wave of CTAs reads at once overlap in L2
    int mt = (int)blockIdx.y, nt = (int)blockIdx.x;
    if (P.group > 0) {
        const int gx = (int)gridDim.x, lin = (int)blockIdx.y * gx + (int)blockIdx.x;
        const int first = lin / (P.group * gx) * P.group;
        const int rows = min((int)gridDim.y - first, P.group), r = lin % (P.group * gx);
        mt = first + r % rows;
        nt = r / rows;
    }
    const int m0 = mt * BM, n0 = nt * BN;
    const int kb0 = split * P.kb_per_split;  // this CTA's first K slice
    const int KT = min((int)((P.K + BK - 1) / BK) - kb0, P.kb_per_split);
    const int NQ = (KT + KC_BLOCKS - 1) / KC_BLOCKS;

    // stage s: A then B (the hi operands as loaded), for PRE then A lo and
    // B lo; lo slot l (converted in shared memory): A then B.  For PRE the
    // lo tiles are indexed by stage.
    auto raw_a = [&](int s) { return smem + (size_t)s * STAGE_BYTES; };
    auto raw_b = [&](int s) { return smem + (size_t)s * STAGE_BYTES + A_BYTES; };
    auto lo_a = [&](int l) {
        return PRE ? smem + (size_t)l * STAGE_BYTES + RAW_BYTES : smem + (size_t)RAW * STAGE_BYTES + (size_t)l * RAW_BYTES;
    };
    auto lo_b = [&](int l) { return lo_a(l) + A_BYTES; };

    // TMA loads of K slice j into stage j % RAW (A, B; for PRE also A lo, B lo)
    auto issue = [&](int j) {
        const int s = j % RAW;
        mb_expect_tx(&full[s], STAGE_BYTES);
        const int k0 = (kb0 + j) * BK;
#pragma unroll
        for (int h = 0; h < (PRE ? 2 : 1); h++) {  // hi, then (PRE) lo
            uint8_t *da = h ? lo_a(s) : raw_a(s), *db = h ? lo_b(s) : raw_b(s);
            const CUtensorMap *ma = h ? &maps.alo : &maps.a, *mb = h ? &maps.blo : &maps.b;
            if (!TA) tma_load_3d(da, ma, k0, m0, za, &full[s]);
            else
                for (int c = 0; c < BM / 32; c++) tma_load_3d(da + c * 4096, ma, m0 + 32 * c, k0, za, &full[s]);
            if (TB) tma_load_3d(db, mb, k0, n0, zb, &full[s]);
            else
                for (int c = 0; c < BN / 32; c++) tma_load_3d(db + c * 4096, mb, n0 + 32 * c, k0, zb, &full[s]);
        }
    };
    const int first_loads = KT < RAW ? KT : RAW;

    if (threadIdx.x == 0) {
        for (int s = 0; s < RAW; s++) {
            mb_init(&full[s], 1);
            mb_init(&empty[s], 1);
        }
        for (int l = 0; l < NLO; l++) {
            mb_init(&conv[l], NWORK);
            mb_init(&lofree[l], 1);
        }
        for (int b = 0; b < NBUF; b++) {
            mb_init(&tfull[b], 1);
            mb_init(&tfree[b], NFOLD);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int j = 0; j < first_loads; j++) issue(j);  // these load while TMEM is allocated
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            for (int j = first_loads; j < KT; j++) {  // j >= RAW: wait for the stage's last MMAs
                if (!mb_wait(&empty[j % RAW], ((j / RAW) - 1) & 1)) break;
                issue(j);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t ID = P.idesc;
            for (int j = 0; j < KT; j++) {
                const int s = j % RAW, l = j % NLO, q = j / KC_BLOCKS, buf = q % NBUF;
                const bool first = (j % KC_BLOCKS) == 0;
                const bool last = (j % KC_BLOCKS) == KC_BLOCKS - 1 || j == KT - 1;
                if (first && q >= NBUF && !mb_wait(&tfree[buf], ((q / NBUF) - 1) & 1)) break;
                if (PRE ? !mb_wait(&full[s], (j / RAW) & 1) : !mb_wait(&conv[l], (j / NLO) & 1)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t d = tmem + (uint32_t)(buf * BN);
                const int lt = PRE ? s : l;  // where this slice's lo tiles are
#pragma unroll
                for (int kk = 0; kk < BK / 8; kk++) {
                    const uint64_t ah = op_desc<!TA>(raw_a(s), kk), al = op_desc<!TA>(lo_a(lt), kk);
                    const uint64_t bh = op_desc<TB>(raw_b(s), kk), bl = op_desc<TB>(lo_b(lt), kk);
                    mma_tf32(d, ah, bh, ID, (first && kk == 0) ? 0u : 1u);
                    mma_tf32(d, ah, bl, ID, 1u);
                    mma_tf32(d, al, bh, ID, 1u);
                }
                mma_commit(&empty[s]);
                if (!PRE) mma_commit(&lofree[l]);
                if (last) mma_commit(&tfull[buf]);
            }
        }
    } else {
        // workers: every landed stage -> its lo tiles; warps 8-15 also fold
        // finished chunks into the running sum and store the tile
        const int wt = threadIdx.x - 64;
        const bool folder = warp >= 8;
        const int q4 = warp & 3, half = (warp - 8) >> 2;
        const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
        int folded = 0;
        bool ok = true;
        // folds every chunk whose MMAs have completed (folder warps only)
        auto try_folds = [&]() {
            while (folded < NQ &&
                   __all_sync(0xffffffffu, mb_test(&tfull[folded % NBUF], (folded / NBUF) & 1))) {
                fold_chunk<BN_>(tmem, lanes, folded, half, P.nmma);
                mb_arrive(&tfree[folded % NBUF]);
                folded++;
            }
        };
        // a bounded wait that keeps folding while it waits
        auto wait = [&](uint64_t *bar, uint32_t parity) {
            if (!folder) return mb_wait(bar, parity);
            for (uint32_t i = 0; i < kGemmSpin; i++) {
                if (__all_sync(0xffffffffu, mb_try(bar, parity))) return true;
                try_folds();
            }
            atomicOr(&g_gemm_error, 1u);
            return false;
        };
        for (int j = 0; j < (PRE ? 0 : KT) && ok; j++) {  // PRE: nothing to convert
            const int s = j % RAW, l = j % NLO;
            if (!wait(&full[s], (j / RAW) & 1)) ok = false;
            else if (j >= NLO && !wait(&lofree[l], ((j / NLO) - 1) & 1)) ok = false;
            if (!ok) break;
            const uint4 *src = (const uint4 *)raw_a(s);  // A then B, contiguous
            uint4 *dst = (uint4 *)lo_a(l);
            uint4 x[T::CONV_ITERS];
#pragma unroll
            for (int u = 0; u < T::CONV_ITERS; u++) {
                const int i = wt + u * NWORK * 32;
                if (i < (int)(RAW_BYTES / 16)) x[u] = src[i];
            }
#pragma unroll
            for (int u = 0; u < T::CONV_ITERS; u++) {
                const int i = wt + u * NWORK * 32;
                if (i < (int)(RAW_BYTES / 16)) dst[i] = lo4(x[u]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mb_arrive(&conv[l]);
            if (folder) try_folds();
        }
        if (folder) {
            while (ok && folded < NQ) {
                if (!mb_wait(&tfull[folded % NBUF], (folded / NBUF) & 1)) {
                    ok = false;
                    break;
                }
                __syncwarp();
                fold_chunk<BN_>(tmem, lanes, folded, half, P.nmma);
                mb_arrive(&tfree[folded % NBUF]);
                folded++;
            }
            // Store: each lane holds 32 columns of its own row and writes them
            // with float4 stores.  For EPI_SCATTER (rows that live in a peer's
            // inbox) the warp first turns its 32 x 32 piece around in shared
            // memory (the pipeline's buffers are idle once the last chunk is
            // folded) and writes it a row at a time, 128 contiguous bytes per
            // instruction, so NVLink carries full-size writes.
            const int64_t row = (int64_t)m0 + q4 * 32 + lane;
            const bool staged = P.epi.mode == EPI_SCATTER;
            const int64_t row0 = (int64_t)m0 + q4 * 32;
            // per-warp staging area in the (idle) pipeline buffers: 32 rows of
            // SPITCH floats (pitch 33 for the scatter's column reads)
            constexpr int SPITCH = 36;
            float *stage = (float *)(smem + (size_t)(warp - 8) * (32 * SPITCH * sizeof(float)));
            // TMA store boxes: per warp two C boxes then two lo boxes (4 KiB
            // each, 1024-byte aligned), after the staging areas
            float *tbuf = (float *)(smem + 40960 + (size_t)(warp - 8) * 16384);
            __syncwarp();
            asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll 1
            for (int c = 0; c < T::FOLD_COLS / 32; c++) {
                const int cl = half * T::FOLD_COLS + c * 32;
                if (!ok || cl >= P.nmma) break;
                float acc[32];
                tmem_ld32(tmem + lanes + SUM_COL + (uint32_t)cl, acc);
                const int64_t col0 = (int64_t)n0 + cl;
                if (P.splits > 1) {  // split-K: the raw partial into this CTA's shared memory
                    float *xr = (float *)smem + (size_t)(q4 * 32 + lane) * T::XPITCH + cl;
#pragma unroll
                    for (int v = 0; v < 8; v++)
                        *(float4 *)(xr + 4 * v) = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
                    continue;
                }
                // non-finite results: zpu's chain instead (over the whole K)
                if (row < P.M) {
                    bool bad = false;
#pragma unroll
                    for (int v = 0; v < 32; v++) bad |= !isfinite(acc[v]);
                    if (bad) {  // through this lane's row of the (idle) staging area
                        float *mine = stage + lane * 33;
#pragma unroll
                        for (int v = 0; v < 32; v++) mine[v] = acc[v];
#pragma unroll 1
                        for (int v = 0; v < 32; v++)
                            if (!isfinite(mine[v]) && col0 + v < P.N)
                                mine[v] = zpu_chain_element<TA, TB>(P.A + oa, P.B + ob, P.lda, P.ldb, row, col0 + v,
                                                                    P.N, 0, P.K);
#pragma unroll
                        for (int v = 0; v < 32; v++) acc[v] = mine[v];
                    }
                }
                if (!staged) {
                    // the epilogue on this lane's row in registers; then the
                    // warp's 32 x 32 piece is turned around in shared memory so
                    // that each store instruction writes 128 contiguous bytes
                    // of four rows (a lane-per-row store touches 32 lines)
                    const int c4 = (lane & 7) * 4;
                    const int64_t col = col0 + c4;
                    if (P.epi.mode == EPI_TANH_GRAD) {
                        // y of the warp's 32 x 32 piece, read the same coalesced
                        // way into the staging area, then each lane takes its row
                        __syncwarp();
#pragma unroll
                        for (int it = 0; it < 8; it++) {
                            const int r = it * 4 + (lane >> 3);
                            const int64_t rr = row0 + r;
                            float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                            if (rr < P.M && col < P.N) {
                                const float *yp = P.epi.aux + rr * P.epi.ldaux + col;
                                if (col + 4 <= P.N && ((((uintptr_t)yp) & 15) == 0)) {
                                    y = __ldg((const float4 *)yp);
                                } else {
                                    y.x = yp[0];
                                    if (col + 1 < P.N) y.y = yp[1];
                                    if (col + 2 < P.N) y.z = yp[2];
                                    if (col + 3 < P.N) y.w = yp[3];
                                }
                            }
                            *(float4 *)(stage + r * SPITCH + c4) = y;
                        }
                        __syncwarp();
#pragma unroll
                        for (int v = 0; v < 8; v++) {
                            const float4 y = *(const float4 *)(stage + lane * SPITCH + 4 * v);
                            acc[4 * v] = __fmul_rn(acc[4 * v], __fsub_rn(1.0f, __fmul_rn(y.x, y.x)));
                            acc[4 * v + 1] = __fmul_rn(acc[4 * v + 1], __fsub_rn(1.0f, __fmul_rn(y.y, y.y)));
                            acc[4 * v + 2] = __fmul_rn(acc[4 * v + 2], __fsub_rn(1.0f, __fmul_rn(y.z, y.z)));
                            acc[4 * v + 3] = __fmul_rn(acc[4 * v + 3], __fsub_rn(1.0f, __fmul_rn(y.w, y.w)));
                        }
                    } else if (row < P.M) {
                        if (col0 + 32 <= P.N) {
                            epi_apply32(P.epi, acc, row, col0);
                        } else {
#pragma unroll
                            for (int v = 0; v < 32; v++)
                                if (col0 + v < P.N) acc[v] = epi_apply(P.epi, acc[v], row, col0 + v);
                        }
                    }
                    __syncwarp();
                    if (P.tma_store) {
                        // this lane's row into a 128-byte swizzled 32 x 32 box
                        // (16-byte chunk v of row r at chunk v ^ (r % 8): the
                        // warp's writes take the minimum 4 wavefronts), then
                        // one lane hands the box to the TMA; two buffers per
                        // warp, so the next piece is staged while this one leaves
                        if (c >= 2 && lane == 0) bulk_wait_read<1>();
                        __syncwarp();
                        float *bc = tbuf + (c & 1) * 1024, *bl = bc + 2048;
#pragma unroll
                        for (int v = 0; v < 8; v++)
                            *(float4 *)(bc + lane * 32 + ((v ^ (lane & 7)) * 4)) =
                                make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
                        if (P.epi.lo_out) {
#pragma unroll
                            for (int v = 0; v < 8; v++)
                                *(uint4 *)(bl + lane * 32 + ((v ^ (lane & 7)) * 4)) =
                                    lo4(make_uint4(__float_as_uint(acc[4 * v]), __float_as_uint(acc[4 * v + 1]),
                                                   __float_as_uint(acc[4 * v + 2]), __float_as_uint(acc[4 * v + 3])));
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_3d(&maps.c, bc, (int)col0, (int)row0, (int)blockIdx.z);
                            if (P.epi.lo_out) tma_store_3d(&maps.clo, bl, (int)col0, (int)row0, 0);
                            bulk_commit();
                        }
                        continue;
                    }
#pragma unroll
                    for (int v = 0; v < 8; v++)
                        *(float4 *)(stage + lane * SPITCH + 4 * v) =
                            make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
                    __syncwarp();
                    float *cm = C + (int64_t)blockIdx.z * P.stride_c;
#pragma unroll
                    for (int it = 0; it < 8; it++) {
                        const int r = it * 4 + (lane >> 3);
                        const int64_t rr = row0 + r;
                        if (rr >= P.M || col >= P.N) continue;
                        const float4 y = *(const float4 *)(stage + r * SPITCH + c4);
                        float *cp = cm + rr * P.ldc + col;
                        float *lp = P.epi.lo_out ? P.epi.lo_out + rr * P.ldc + col : nullptr;  // one matrix
                        if (col + 4 <= P.N && ((((uintptr_t)cp) & 15) == 0)) {
                            *(float4 *)cp = y;
                            if (lp && ((((uintptr_t)lp) & 15) == 0)) {
                                *(uint4 *)lp = lo4(make_uint4(__float_as_uint(y.x), __float_as_uint(y.y),
                                                              __float_as_uint(y.z), __float_as_uint(y.w)));
                            } else if (lp) {
                                lp[0] = lo1(y.x);
                                lp[1] = lo1(y.y);
                                lp[2] = lo1(y.z);
                                lp[3] = lo1(y.w);
                            }
                        } else {
                            const float yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
                            for (int e = 0; e < 4; e++)
                                if (col + e < P.N) {
                                    cp[e] = yv[e];
                                    if (lp) lp[e] = lo1(yv[e]);
                                }
                        }
                    }
                    __syncwarp();
                    continue;
                }
#pragma unroll
                for (int v = 0; v < 32; v++) stage[lane * 33 + v] = acc[v];
                __syncwarp();
                const int64_t col = col0 + lane;
#pragma unroll 4
                for (int r = 0; r < 32; r++) {
                    const int64_t rr = row0 + r;
                    if (rr >= P.M) break;
                    const int64_t owner = rr / P.epi.rows_per_owner;  // its inbox: over NVLink for a peer
                    float *dst = P.epi.peer[owner] +
                                 ((int64_t)P.epi.src * P.epi.rows_per_owner + rr - owner * P.epi.rows_per_owner) * P.ldc;
                    if (col < P.N) dst[col] = stage[r * 33 + lane];
                }
                __syncwarp();
            }
            if (P.tma_store && lane == 0) bulk_wait_read<0>();  // the boxes have left shared memory
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    // split-K: this CTA's partial is in place (the release orders the
    // folders' shared-memory stores before the other CTAs read them)
    if (P.splits > 1) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
    if (P.splits > 1) splitk_cluster_reduce<TA, TB, BN_>(smem, C, P, oa, ob, bz, m0, n0);
}

// ------------------------------------------------ persistent form
//
// For many output tiles over a short K (the vmapped 256 x 512^3 batch: 2048
// tiles of 16 K slices), a CTA's fixed costs -- barrier set-up and TMEM
// allocation, the first loads, the last fold and the tile store, ~8 of ~34
// us per tile -- leave the tensor core idle.  Here one CTA per SM walks the
// tiles blockIdx.x, blockIdx.x + gridDim.x, ...: the producer runs on into
// the next tile's K slices, the MMAs of the next tile start as soon as the
// last chunk of this one is folded, and the folding warps store a finished
// tile (TMA, one 32 x 32 box buffer per warp after the pipeline's buffers)
// while the next tile accumulates.  Stage, lo-slot and chunk phases run on
// across tiles (slice counter g, chunk counter).  Same chunks, folds and
// order per element as tf32x3_gemm_kernel: identical results.  128 x 256
// tiles, lo halves made in shared memory, epilogues without HBM inputs
// (store, bias, bias + tanh), no split-K.
template <bool TA, bool TB>
__global__ void __launch_bounds__(THREADS, 1)
    tf32x3_gemm_persistent_kernel(const __grid_constant__ Maps maps, float *__restrict__ C,
                                  const __grid_constant__ Params P) {
    using T = Tile<256, false>;
    constexpr int BN = 256, RAW = T::RAW, NLO = T::LO, NBUF = T::NBUF, KC_BLOCKS = T::KC_BLOCKS;
    constexpr uint32_t RAW_BYTES = T::RAW_BYTES, STAGE_BYTES = T::STAGE_BYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[RAW], empty[RAW], conv[NLO], lofree[NLO], tfull[NBUF], tfree[NBUF];
    __shared__ uint32_t tmem_base;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t ncols = (P.N + BN - 1) / BN, nrows = (P.M + BM - 1) / BM;
    const int64_t total = ncols * nrows * P.batches;
    const int ntiles = (int)((total - (int64_t)blockIdx.x + gridDim.x - 1) / gridDim.x);
    const int KT = (int)((P.K + BK - 1) / BK);
    const int NQ = (KT + KC_BLOCKS - 1) / KC_BLOCKS;
    struct Co {
        int m0, n0, za, zb;
        int64_t bz, oa, ob;
    };
    auto coords = [&](int it) {  // this CTA's tile `it`: columns fastest, then rows, then matrices
        Co c;
        const int64_t t = (int64_t)blockIdx.x + (int64_t)it * gridDim.x, r = t / ncols;
        c.n0 = (int)((t % ncols) * BN);
        c.m0 = (int)((r % nrows) * BM);
        c.bz = r / nrows;
        batch_offsets(P.bt, c.bz, &c.oa, &c.ob);
        c.za = (int)(P.mat_a ? c.oa / P.mat_a : 0);
        c.zb = (int)(P.mat_b ? c.ob / P.mat_b : 0);
        return c;
    };
    auto raw_a = [&](int s) { return smem + (size_t)s * STAGE_BYTES; };
    auto raw_b = [&](int s) { return smem + (size_t)s * STAGE_BYTES + A_BYTES; };
    auto lo_a = [&](int l) { return smem + (size_t)RAW * STAGE_BYTES + (size_t)l * RAW_BYTES; };
    auto lo_b = [&](int l) { return lo_a(l) + A_BYTES; };
    // K slice j of tile c into stage g % RAW (g: the slice's place in this CTA's sequence)
    auto issue = [&](int g, int j, const Co &c) {
        const int s = g % RAW;
        mb_expect_tx(&full[s], STAGE_BYTES);
        const int k0 = j * BK;
        if (!TA) tma_load_3d(raw_a(s), &maps.a, k0, c.m0, c.za, &full[s]);
        else
            for (int q = 0; q < BM / 32; q++) tma_load_3d(raw_a(s) + q * 4096, &maps.a, c.m0 + 32 * q, k0, c.za, &full[s]);
        if (TB) tma_load_3d(raw_b(s), &maps.b, k0, c.n0, c.zb, &full[s]);
        else
            for (int q = 0; q < BN / 32; q++) tma_load_3d(raw_b(s) + q * 4096, &maps.b, c.n0 + 32 * q, k0, c.zb, &full[s]);
    };
    const int first_loads = KT < RAW ? KT : RAW;

    if (threadIdx.x == 0) {
        for (int s = 0; s < RAW; s++) {
            mb_init(&full[s], 1);
            mb_init(&empty[s], 1);
        }
        for (int l = 0; l < NLO; l++) {
            mb_init(&conv[l], NWORK);
            mb_init(&lofree[l], 1);
        }
        for (int b = 0; b < NBUF; b++) {
            mb_init(&tfull[b], 1);
            mb_init(&tfree[b], NFOLD);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const Co c0 = coords(0);
        for (int j = 0; j < first_loads; j++) issue(j, j, c0);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            bool ok = true;
            for (int it = 0, g = 0; it < ntiles && ok; it++) {
                const Co c = coords(it);
                for (int j = 0; j < KT; j++, g++) {
                    if (g < first_loads) continue;  // issued before the TMEM allocation
                    if (!mb_wait(&empty[g % RAW], ((g / RAW) - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    issue(g, j, c);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t ID = P.idesc;
            bool ok = true;
            for (int it = 0, g = 0, qg = 0; it < ntiles && ok; it++) {
                for (int j = 0; j < KT; j++, g++) {
                    const int s = g % RAW, l = g % NLO, buf = qg % NBUF;
                    const bool first = (j % KC_BLOCKS) == 0;
                    const bool last = (j % KC_BLOCKS) == KC_BLOCKS - 1 || j == KT - 1;
                    if ((first && qg >= NBUF && !mb_wait(&tfree[buf], ((qg / NBUF) - 1) & 1)) ||
                        !mb_wait(&conv[l], (g / NLO) & 1)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint32_t d = tmem + (uint32_t)(buf * BN);
#pragma unroll
                    for (int kk = 0; kk < BK / 8; kk++) {
                        const uint64_t ah = op_desc<!TA>(raw_a(s), kk), al = op_desc<!TA>(lo_a(l), kk);
                        const uint64_t bh = op_desc<TB>(raw_b(s), kk), bl = op_desc<TB>(lo_b(l), kk);
                        mma_tf32(d, ah, bh, ID, (first && kk == 0) ? 0u : 1u);
                        mma_tf32(d, ah, bl, ID, 1u);
                        mma_tf32(d, al, bh, ID, 1u);
                    }
                    mma_commit(&empty[s]);
                    mma_commit(&lofree[l]);
                    if (last) {
                        mma_commit(&tfull[buf]);
                        qg++;
                    }
                }
            }
        }
    } else {
        const int wt = threadIdx.x - 64;
        const bool folder = warp >= 8;
        const int q4 = warp & 3, half = (warp - 8) >> 2;
        const uint32_t lanes = (uint32_t)(q4 * 32) << 16;
        const int total_q = ntiles * NQ;
        int folded = 0;
        bool ok = true;
        // this warp's 32 x 32 box buffer, after the stages and lo slots
        float *tb = (float *)(smem + (size_t)RAW * STAGE_BYTES + (size_t)NLO * RAW_BYTES +
                              (size_t)(warp >= 8 ? warp - 8 : 0) * 4096);
        // the finished tile `it`: running sum -> epilogue -> TMA store, one
        // 32-column piece of this warp's rows at a time
        auto store_tile = [&](int it) {
            const Co c = coords(it);
            const int64_t row = (int64_t)c.m0 + q4 * 32 + lane;
            asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll 1
            for (int pc = 0; pc < T::FOLD_COLS / 32; pc++) {
                const int cl = half * T::FOLD_COLS + pc * 32;
                if (cl >= P.nmma) break;
                if (lane == 0) bulk_wait_read<0>();  // the box buffer has left shared memory
                __syncwarp();
                float acc[32];
                tmem_ld32(tmem + lanes + SUM_COL + (uint32_t)cl, acc);
                const int64_t col0 = (int64_t)c.n0 + cl;
                if (row < P.M) {
                    bool bad = false;
#pragma unroll
                    for (int v = 0; v < 32; v++) bad |= !isfinite(acc[v]);
                    if (bad) {  // zpu's chain for the non-finite elements, through this lane's row of the buffer
                        float *mine = tb + lane * 32;
#pragma unroll
                        for (int v = 0; v < 32; v++) mine[v] = acc[v];
#pragma unroll 1
                        for (int v = 0; v < 32; v++)
                            if (!isfinite(mine[v]) && col0 + v < P.N)
                                mine[v] = zpu_chain_element<TA, TB>(P.A + c.oa, P.B + c.ob, P.lda, P.ldb, row,
                                                                    col0 + v, P.N, 0, P.K);
#pragma unroll
                        for (int v = 0; v < 32; v++) acc[v] = mine[v];
                    }
                    if (col0 + 32 <= P.N) {
                        epi_apply32(P.epi, acc, row, col0);
                    } else {
#pragma unroll
                        for (int v = 0; v < 32; v++)
                            if (col0 + v < P.N) acc[v] = epi_apply(P.epi, acc[v], row, col0 + v);
                    }
                }
                __syncwarp();
#pragma unroll
                for (int v = 0; v < 8; v++)
                    *(float4 *)(tb + lane * 32 + ((v ^ (lane & 7)) * 4)) =
                        make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&maps.c, tb, (int)col0, c.m0 + q4 * 32, (int)c.bz);
                    bulk_commit();
                }
            }
        };
        // fold chunk `folded` (its tile's first chunk starts the running
        // sum); a tile's last chunk is followed by the tile's store
        auto fold_next = [&]() {
            fold_chunk<BN>(tmem, lanes, folded % NQ, half, P.nmma, folded % NBUF);
            mb_arrive(&tfree[folded % NBUF]);
            folded++;
            if (folded % NQ == 0) store_tile(folded / NQ - 1);
        };
        auto try_folds = [&]() {
            while (folded < total_q && __all_sync(0xffffffffu, mb_test(&tfull[folded % NBUF], (folded / NBUF) & 1)))
                fold_next();
        };
        auto wait = [&](uint64_t *bar, uint32_t parity) {
            if (!folder) return mb_wait(bar, parity);
            for (uint32_t i = 0; i < kGemmSpin; i++) {
                if (__all_sync(0xffffffffu, mb_try(bar, parity))) return true;
                try_folds();
            }
            atomicOr(&g_gemm_error, 1u);
            return false;
        };
        for (int it = 0, g = 0; it < ntiles && ok; it++) {
            for (int j = 0; j < KT; j++, g++) {
                const int s = g % RAW, l = g % NLO;
                if (!wait(&full[s], (g / RAW) & 1) || (g >= NLO && !wait(&lofree[l], ((g / NLO) - 1) & 1))) {
                    ok = false;
                    break;
                }
                const uint4 *src = (const uint4 *)raw_a(s);  // A then B, contiguous
                uint4 *dst = (uint4 *)lo_a(l);
                uint4 x[T::CONV_ITERS];
#pragma unroll
                for (int u = 0; u < T::CONV_ITERS; u++) {
                    const int i = wt + u * NWORK * 32;
                    if (i < (int)(RAW_BYTES / 16)) x[u] = src[i];
                }
#pragma unroll
                for (int u = 0; u < T::CONV_ITERS; u++) {
                    const int i = wt + u * NWORK * 32;
                    if (i < (int)(RAW_BYTES / 16)) dst[i] = lo4(x[u]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mb_arrive(&conv[l]);
                if (folder) try_folds();
            }
        }
        if (folder) {
            while (ok && folded < total_q) {
                if (!mb_wait(&tfull[folded % NBUF], (folded / NBUF) & 1)) {
                    ok = false;
                    break;
                }
                __syncwarp();
                fold_next();
            }
            if (lane == 0) bulk_wait_read<0>();
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// ------------------------------------------------ plain FMA-chain fallback
//
// For shapes the tensor maps cannot take: each output element is the FMA
// chain of zpu's kernel (k ascending from 0), 16x16 tiles through shared
// memory.  Correct for any strides; not the fast path.
template <bool TA, bool TB>
__global__ void __launch_bounds__(256) fma_gemm_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                       float *__restrict__ C, int64_t M, int64_t N, int64_t K,
                                                       int64_t lda, int64_t ldb, int64_t ldc,
                                                       const __grid_constant__ GemmBatch bt, int64_t stride_c,
                                                       const __grid_constant__ Epilogue epi) {
    __shared__ float sa[16][17], sb[16][17];
    int64_t oa, ob;
    batch_offsets(bt, blockIdx.z, &oa, &ob);
    A += oa;
    B += ob;
    C += (int64_t)blockIdx.z * stride_c;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t row = (int64_t)blockIdx.y * 16 + ty, col = (int64_t)blockIdx.x * 16 + tx;
    float acc = 0.0f;
    for (int64_t k0 = 0; k0 < K; k0 += 16) {
        const int64_t ka = k0 + tx, kb = k0 + ty;
        const int64_t ar = (int64_t)blockIdx.y * 16 + ty, bc = (int64_t)blockIdx.x * 16 + tx;
        sa[ty][tx] = (ar < M && ka < K) ? (TA ? A[ka * lda + ar] : A[ar * lda + ka]) : 0.0f;
        sb[ty][tx] = (kb < K && bc < N) ? (TB ? B[bc * ldb + kb] : B[kb * ldb + bc]) : 0.0f;
        __syncthreads();
        const int kmax = (int)(K - k0 < 16 ? K - k0 : 16);
        for (int kk = 0; kk < kmax; kk++) acc = fmaf(sa[ty][kk], sb[kk][tx], acc);
        __syncthreads();
    }
    if (row < M && col < N) {
        const float y = epi_apply(epi, acc, row, col);
        C[row * ldc + col] = y;
        if (epi.lo_out) epi.lo_out[row * ldc + col] = lo1(y);
    }
}

// ------------------------------------------------ short contractions
//
// Products with k <= kSmallK (the MLP's g2 = gl W3^T has k = 16) are bound by
// writing the result (and reading the epilogue's inputs), not by flops: one
// K slice per tensor-core tile would leave every CTA in its set-up and store.
// Here CUDA cores compute zpu's own chain per element -- kernels.gemm's FMA
// order and its scalar tail (the columns past the last whole 8-lane vector of
// a 128-column panel take c + a*b), src/zpu/kernels.zig:369-400 -- so the
// bits are zpu's.  A block takes 128 columns and kSmallRowTiles tiles of 32
// rows: the B columns staged once in shared memory, each A tile in turn,
// 4 rows x 4 consecutive columns per thread, float4 stores.
constexpr int kSmallK = 32;
constexpr int kSmallRowTiles = 4;  // 32-row tiles per block (the B tile staged once)

template <bool TA, bool TB>
__global__ void __launch_bounds__(256) smallk_gemm_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                          float *__restrict__ C, int64_t M, int64_t N, int k,
                                                          int64_t lda, int64_t ldb, int64_t ldc,
                                                          const __grid_constant__ GemmBatch bt, int64_t stride_c,
                                                          const __grid_constant__ Epilogue epi) {
    __shared__ float sa[32][kSmallK + 1];
    __shared__ __align__(16) float sb[kSmallK][128];
    int64_t oa, ob;
    batch_offsets(bt, blockIdx.z, &oa, &ob);
    A += oa;
    B += ob;
    C += (int64_t)blockIdx.z * stride_c;
    const int64_t c0 = (int64_t)blockIdx.x * 128;
    // tiles zero past the matrix edges (slices p >= k are never read); a
    // thread's loads first, then its shared-memory stores, so the loads are
    // in flight together.  The B tile is staged once for kSmallRowTiles A tiles.
    constexpr int UA = 32 * kSmallK / 256, UB = kSmallK * 128 / 256;
    float vb[UB];
#pragma unroll
    for (int u = 0; u < UB; u++) {  // consecutive threads take consecutive columns
        const int i = (int)threadIdx.x + u * 256, p = i / 128, c = i % 128;
        const int64_t col = c0 + c;
        vb[u] = (p < k && col < N) ? (TB ? B[col * ldb + p] : B[(int64_t)p * ldb + col]) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < UB; u++) {
        const int i = (int)threadIdx.x + u * 256;
        sb[i / 128][i % 128] = vb[u];
    }
    const int cg = (threadIdx.x & 31) * 4, rg = (threadIdx.x >> 5) * 4;
    // the panel's vector-covered columns (c0 starts a 128-column panel)
    const int64_t nv = ((N - c0 < 128 ? N - c0 : 128) / 8) * 8;
    bool fused[4];
#pragma unroll
    for (int j = 0; j < 4; j++) fused[j] = cg + j < nv;
    const int64_t col = c0 + cg;
    for (int rt = 0; rt < kSmallRowTiles; rt++) {
        const int64_t r0 = ((int64_t)blockIdx.y * kSmallRowTiles + rt) * 32;
        if (r0 >= M) break;  // uniform over the block
        float va[UA];
#pragma unroll
        for (int u = 0; u < UA; u++) {
            const int i = (int)threadIdx.x + u * 256;
            const int r = TA ? i % 32 : i / kSmallK, p = TA ? i / 32 : i % kSmallK;
            const int64_t row = r0 + r;
            va[u] = (row < M && p < k) ? (TA ? A[(int64_t)p * lda + row] : A[row * lda + p]) : 0.0f;
        }
        __syncthreads();  // the last tile's readers are done with sa
#pragma unroll
        for (int u = 0; u < UA; u++) {
            const int i = (int)threadIdx.x + u * 256;
            sa[TA ? i % 32 : i / kSmallK][TA ? i / 32 : i % kSmallK] = va[u];
        }
        __syncthreads();
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
        if (fused[3]) {  // all four columns vector-covered (the common case): plain FMA chains
            for (int p = 0; p < k; p++) {
                const float4 b4 = *(const float4 *)&sb[p][cg];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float a = sa[rg + i][p];
                    acc[i][0] = fmaf(a, b4.x, acc[i][0]);
                    acc[i][1] = fmaf(a, b4.y, acc[i][1]);
                    acc[i][2] = fmaf(a, b4.z, acc[i][2]);
                    acc[i][3] = fmaf(a, b4.w, acc[i][3]);
                }
            }
        } else {
            for (int p = 0; p < k; p++) {
                const float4 b4 = *(const float4 *)&sb[p][cg];
                const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float a = sa[rg + i][p];
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        acc[i][j] = fused[j] ? fmaf(a, bv[j], acc[i][j]) : __fadd_rn(acc[i][j], __fmul_rn(a, bv[j]));
                }
            }
        }
        if (col >= N) continue;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int64_t row = r0 + rg + i;
            if (row >= M) break;
            float y[4];
#pragma unroll
            for (int j = 0; j < 4; j++) y[j] = col + j < N ? epi_apply(epi, acc[i][j], row, col + j) : 0.0f;
            float *cp = C + row * ldc + col;
            float *lp = epi.lo_out ? epi.lo_out + row * ldc + col : nullptr;
            if (col + 4 <= N && ((((uintptr_t)cp) & 15) == 0)) {
                *(float4 *)cp = make_float4(y[0], y[1], y[2], y[3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (col + j < N) cp[j] = y[j];
            }
            if (lp) {
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (col + j < N) lp[j] = lo1(y[j]);
            }
        }
    }
}

// ------------------------------------------------------------- host side

// Stream-ordered scratch for the lo halves of presplit operands: one memory
// pool per device that keeps what it has allocated (no release at
// synchronisation).
cudaMemPool_t splitk_pool() {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {nullptr};
    const int dev = current_device();
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!pools[dev]) {
        cudaMemPoolProps props;
        memset(&props, 0, sizeof props);
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        uint64_t keep = ~0ull;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        pools[dev] = pool;
    }
    return pools[dev];
}

// K splits for a problem of `tiles` output tiles and KT K slices: enough CTAs
// to cover the SMs when the tiles alone fill less than half of them, with at
// least two accumulation chunks per split; at most kMaxSplits (one
// portable-size cluster per tile).  ZPUCUDA_GEMM_SPLITS=<n> forces the
// split count (read at every call; still capped at kMaxSplits and KT).
constexpr int kMaxSplits = 8;
int choose_splits(int64_t tiles, int64_t KT, int kc) {
    int64_t sp;
    const char *e = getenv("ZPUCUDA_GEMM_SPLITS");
    if (e && atoi(e) >= 1) {
        sp = atoi(e);
    } else {
        const int64_t sms = num_sms();
        if (tiles * 2 > sms) return 1;
        sp = sms / tiles;
        if (sp > KT / (2 * kc)) sp = KT / (2 * kc);
    }
    if (sp > kMaxSplits) sp = kMaxSplits;
    if (sp > KT) sp = KT;
    return sp < 1 ? 1 : (int)sp;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int encode_fn() {
    static std::once_flag once;
    static int status = ZPUCUDA_OK;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            cudaGetLastError();
            status = ZPUCUDA_ERR_NO_DEVICE;
            return;
        }
        g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    });
    return status;
}

// 3-D f32 tensor map (inner, rows, matrices), box {32, box_rows, 1};
// out-of-range elements read as zero.  K-major operands: 128-byte swizzle;
// MN-major: 128-byte swizzle with 32-byte atoms.
bool make_map(CUtensorMap *map, const float *base, int64_t inner, int64_t rows, int64_t ld, int64_t nmats,
              int64_t mat_stride, int box_rows, bool kmajor) {
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)nmats};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(nmats > 1 ? mat_stride : rows * ld) * 4};
    cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          kmajor ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// The smallest positive batch stride of an operand, provided every batch
// stride is a multiple of it (so batch offsets are whole matrices); 0 when
// the operand does not move with the batch.
bool matrix_stride(const int64_t *s, int nax, int64_t *out) {
    int64_t m = 0;
    for (int i = 0; i < nax; i++)
        if (s[i] < 0) return false;
        else if (s[i] > 0 && (m == 0 || s[i] < m)) m = s[i];
    for (int i = 0; i < nax; i++)
        if (m && s[i] % m) return false;
    *out = m;
    return true;
}

int64_t max_offset(const GemmBatch &bt, const int64_t *s) {
    int64_t o = 0;
    for (int i = 0; i < bt.nax; i++) o += (bt.dims[i] > 0 ? bt.dims[i] - 1 : 0) * s[i];
    return o;
}

template <bool TA, bool TB, int BN_, bool PRE>
int launch_tf32x3(const Maps &maps, float *C, const Params &P, int64_t batches, cudaStream_t s) {
    using T = Tile<BN_, PRE>;
    auto k = tf32x3_gemm_kernel<TA, TB, BN_, PRE>;
    static bool attr[64] = {false};
    const int dev = current_device();
    if (dev < 0 || dev >= 64 || !attr[dev]) {
        ZC_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)T::SMEM_BYTES));
        if (dev >= 0 && dev < 64) attr[dev] = true;
    }
    dim3 grid((unsigned)((P.N + BN_ - 1) / BN_), (unsigned)((P.M + BM - 1) / BM), (unsigned)(batches * P.splits));
    if (P.splits == 1) {
        k<<<grid, THREADS, T::SMEM_BYTES, s>>>(maps, C, P);
        ZC_LAUNCHED("tf32x3_gemm_kernel");
        return ZPUCUDA_OK;
    }
    // split-K: the splits of one tile form a cluster along z
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = grid;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = T::SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = (unsigned)P.splits;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    ZC_CUDA(cudaLaunchKernelEx(&cfg, k, maps, C, P));
    count_launch();
    return ZPUCUDA_OK;
}

// Tile width for an m x n x batches problem: a 128 x 256 tile takes ~1.6x
// the time of a 128 x 128 one (measured 1.5-1.7 over 4096^3, the batched
// 256 x 512^3 and the MLP's products, with and without the presplit lo);
// pick the width whose whole waves of tiles over the SMs take less time.
// ZPUCUDA_GEMM_BN=128 or 256 forces the width (read at every call).
int choose_bn(int64_t m, int64_t n, int64_t batches) {
    const char *e = getenv("ZPUCUDA_GEMM_BN");
    if (e && (atoi(e) == 128 || atoi(e) == 256)) return atoi(e);
    if (n <= 128) return 128;
    const int64_t sms = num_sms();
    const int64_t rows = (m + BM - 1) / BM;
    const int64_t w128 = (rows * ((n + 127) / 128) * batches + sms - 1) / sms;
    const int64_t w256 = (rows * ((n + 255) / 256) * batches + sms - 1) / sms;
    return 1.6 * (double)w256 < (double)w128 ? 256 : 128;
}

// The persistent form: one CTA per SM (at most one per tile), each walking
// its tiles; 32 KiB more shared memory for the store boxes.
constexpr size_t kPersSmem = Tile<256, false>::SMEM_BYTES + 8 * 4096;
static_assert(kPersSmem <= 227 * 1024, "persistent form's shared memory");

template <bool TA, bool TB>
int launch_persistent(const Maps &maps, float *C, const Params &P, int64_t tiles, cudaStream_t s) {
    auto k = tf32x3_gemm_persistent_kernel<TA, TB>;
    static bool attr[64] = {false};
    const int dev = current_device();
    if (dev < 0 || dev >= 64 || !attr[dev]) {
        ZC_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPersSmem));
        if (dev >= 0 && dev < 64) attr[dev] = true;
    }
    const int64_t ctas = tiles < num_sms() ? tiles : num_sms();
    k<<<(unsigned)ctas, THREADS, kPersSmem, s>>>(maps, C, P);
    ZC_LAUNCHED("tf32x3_gemm_persistent_kernel");
    return ZPUCUDA_OK;
}

// Whether a 128 x 256 product without presplit lo runs in the persistent
// form: at least two tiles per SM over a short K (where a tile's fixed
// costs weigh), a TMA tile store, an epilogue without HBM inputs.
// ZPUCUDA_GEMM_PERSISTENT=0 or 1 forces the choice among the products the
// form can take (read at every call).
bool use_persistent(const Params &P, int64_t tiles, int64_t KT) {
    if (!P.tma_store || P.splits != 1 || P.epi.lo_out ||
        !(P.epi.mode == EPI_STORE || P.epi.mode == EPI_BIAS || P.epi.mode == EPI_BIAS_TANH))
        return false;
    const char *e = getenv("ZPUCUDA_GEMM_PERSISTENT");
    if (e && (e[0] == '0' || e[0] == '1') && e[1] == 0) return e[0] == '1';
    return tiles >= 2 * (int64_t)num_sms() && KT <= 64;
}

template <int BN_, bool PRE>
int dispatch_tf32x3(bool ta, bool tb, const Maps &maps, float *C, const Params &P, int64_t batches, cudaStream_t s) {
    if (!ta && !tb) return launch_tf32x3<false, false, BN_, PRE>(maps, C, P, batches, s);
    if (!ta && tb) return launch_tf32x3<false, true, BN_, PRE>(maps, C, P, batches, s);
    if (ta && !tb) return launch_tf32x3<true, false, BN_, PRE>(maps, C, P, batches, s);
    return launch_tf32x3<true, true, BN_, PRE>(maps, C, P, batches, s);
}

// The lo halves of one operand into stream-ordered scratch from `pool`
// (nullptr when that fails): the operand as (inner, rows, nmats).
float *split_operand(cudaMemPool_t pool, const float *x, int64_t inner, int64_t rows, int64_t nmats, int64_t ld,
                     int64_t mat, cudaStream_t s) {
    const int64_t extent = (nmats - 1) * mat + (rows - 1) * ld + inner;  // elements the map can reach
    float *lo = nullptr;
    if (!pool || cudaMallocFromPoolAsync((void **)&lo, (size_t)extent * sizeof(float), pool, s) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    const int64_t n4 = (inner + 3) / 4 * rows * nmats;
    int64_t blocks = (n4 + 255) / 256;
    if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
    split_lo_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, s>>>(x, lo, inner, rows, nmats, ld, mat);
    if (cudaGetLastError() != cudaSuccess) {
        cudaFreeAsync(lo, s);
        return nullptr;
    }
    count_launch();
    return lo;
}

// Whether the lo halves come from a split pass (PRE kernels) rather than
// from the converter warps.  The PRE kernel runs ~1.25x faster (measured:
// 8192^3 4.9 against 6.2 ms, 4096^3 0.66 against 0.87 ms), but the pass
// moves 8 bytes per operand element through HBM (read x, write lo), so it
// pays where each operand element takes part in many products: the pass's
// time 8 (na m + nb n) k / HBM below a fifth of the product's
// 2 m n k batches / (~180 TFLOP/s), i.e. na m + nb n < 0.0018 m n batches
// (4096^3 and the MLP's products yes; 1024^3 and 256 x 512^3 no: measured
// 51 -> 44 and 135 -> 117 TFLOP/s with the pass).  ZPUCUDA_GEMM_PRESPLIT=0
// or 1 forces the choice (read at every call).
// Row tiles per raster group for an rows x cols tile grid: groups of 16
// where the grid has more than 32 rows and columns of tiles (at 8192^3 a
// wave of 148 CTAs in row-major order reads every B column panel, 512 MB
// with the lo halves, so B comes from HBM again in every wave), else
// blockIdx order.  ZPUCUDA_GEMM_RASTER=<g> forces g (0: off; read at every
// call).
int raster_group(int64_t rows, int64_t cols) {
    const char *e = getenv("ZPUCUDA_GEMM_RASTER");
    if (e && e[0] >= '0' && e[0] <= '9') return atoi(e);
    return rows > 32 && cols > 32 ? 16 : 0;
}

// Whether contractions of k <= kSmallK run on CUDA cores (default);
// ZPUCUDA_GEMM_SMALLK=0 sends them to the tensor cores (read at every call).
bool use_smallk() {
    const char *e = getenv("ZPUCUDA_GEMM_SMALLK");
    return !(e && e[0] == '0' && e[1] == 0);
}

// Whether result tiles leave through TMA stores (default) rather than the
// folding warps' own stores; ZPUCUDA_GEMM_TMA_STORE=0 turns them off (read
// at every call).
bool use_tma_store() {
    const char *e = getenv("ZPUCUDA_GEMM_TMA_STORE");
    return !(e && e[0] == '0' && e[1] == 0);
}

bool use_presplit(int64_t m, int64_t n, int64_t batches, int64_t na, int64_t nb) {
    const char *e = getenv("ZPUCUDA_GEMM_PRESPLIT");
    if (e && (e[0] == '0' || e[0] == '1') && e[1] == 0) return e[0] == '1';
    return (double)(na * m + nb * n) < 0.0018 * (double)m * (double)n * (double)batches;
}

}  // namespace

int gemm_f32_device(const float *A, const float *B, float *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                    int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                    cudaStream_t s) {
    return gemm_f32_device_epi(A, B, C, m, n, k, lda, ldb, ldc, ta, tb, bt, stride_c, Epilogue{}, s);
}

bool gemm_f32_presplit(int64_t m, int64_t n, int64_t batches) { return use_presplit(m, n, batches, 1, 1); }

int split_lo_device(const float *x, float *lo, int64_t n, cudaStream_t s) {
    if (n <= 0) return ZPUCUDA_OK;
    if (!x || !lo || ((uintptr_t)x & 15) || ((uintptr_t)lo & 15)) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    int64_t blocks = (n / 4 + 255) / 256;
    if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
    split_lo_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, s>>>(x, lo, n, 1, 1, n, 0);
    ZC_LAUNCHED("split_lo_kernel");
    return ZPUCUDA_OK;
}

int gemm_f32_device_epi(const float *A, const float *B, float *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                        int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                        const Epilogue &epi, cudaStream_t s) {
    return gemm_f32_device_lo(A, B, C, m, n, k, lda, ldb, ldc, ta, tb, bt, stride_c, epi, nullptr, nullptr, s);
}

int gemm_f32_device_lo(const float *A, const float *B, float *C, int64_t m, int64_t n, int64_t k, int64_t lda,
                       int64_t ldb, int64_t ldc, bool ta, bool tb, const GemmBatch &bt, int64_t stride_c,
                       const Epilogue &epi, const float *a_lo, const float *b_lo, cudaStream_t s) {
    const int64_t batches = batch_count(bt);
    if (m == 0 || n == 0 || batches == 0) return ZPUCUDA_OK;
    if (!C || ldc < n) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if (epi.lo_out && (batches != 1 || epi.mode == EPI_SCATTER)) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)a_lo & 15) || ((uintptr_t)b_lo & 15)) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if (epi.mode != EPI_STORE) {  // the epilogue inputs belong to one matrix
        if (batches != 1 || epi.mode < 0 || epi.mode > EPI_SCATTER) return ZPUCUDA_ERR_INVALID_ARGUMENT;
        if (epi.mode == EPI_SCATTER) {
            if (epi.world < 1 || epi.world > kMaxPeers || epi.src < 0 || epi.src >= epi.world ||
                epi.rows_per_owner * epi.world != m)
                return ZPUCUDA_ERR_INVALID_ARGUMENT;
            for (int r = 0; r < epi.world; r++)
                if (!epi.peer[r]) return ZPUCUDA_ERR_INVALID_ARGUMENT;
        } else if ((epi.mode == EPI_TANH_GRAD) ? (!epi.aux || epi.ldaux < n) : !epi.bias) {
            return ZPUCUDA_ERR_INVALID_ARGUMENT;
        }
        if (k == 0) return ZPUCUDA_ERR_NOT_SUPPORTED;
    }
    if (k == 0) {  // kernels.zig:346-349: an empty contraction writes zeros
        for (int64_t b = 0; b < batches; b++)
            ZC_CUDA(cudaMemset2DAsync(C + b * stride_c, ldc * sizeof(float), 0, n * sizeof(float), m, s));
        if (epi.lo_out) ZC_CUDA(cudaMemset2DAsync(epi.lo_out, ldc * sizeof(float), 0, n * sizeof(float), m, s));
        return ZPUCUDA_OK;
    }
    if (!A || !B) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if ((!ta && lda < k) || (ta && lda < m) || (!tb && ldb < n) || (tb && ldb < k)) return ZPUCUDA_ERR_INVALID_SHAPE;
    if (batches > 65535 || (m + BM - 1) / BM > 65535) return ZPUCUDA_ERR_NOT_SUPPORTED;

    // a short contraction: zpu's chain on CUDA cores (bound by the result's bytes)
    if (k <= kSmallK && epi.mode != EPI_SCATTER && (m + 31) / 32 <= 65535 && use_smallk()) {
        dim3 grid((unsigned)((n + 127) / 128), (unsigned)((m + 32 * kSmallRowTiles - 1) / (32 * kSmallRowTiles)),
                  (unsigned)batches);
#define ZC_SK(TA_, TB_) \
    smallk_gemm_kernel<TA_, TB_><<<grid, 256, 0, s>>>(A, B, C, m, n, (int)k, lda, ldb, ldc, bt, stride_c, epi)
        if (!ta && !tb) ZC_SK(false, false);
        else if (!ta && tb) ZC_SK(false, true);
        else if (ta && !tb) ZC_SK(true, false);
        else ZC_SK(true, true);
#undef ZC_SK
        ZC_LAUNCHED("smallk_gemm_kernel");
        return ZPUCUDA_OK;
    }

    // the tensor-core path needs what a TMA tensor map can describe
    int64_t mat_a = 0, mat_b = 0;
    bool tc = encode_fn() == ZPUCUDA_OK && ((uintptr_t)A % 16 == 0) && ((uintptr_t)B % 16 == 0) && lda % 4 == 0 &&
              ldb % 4 == 0 && matrix_stride(bt.sa, bt.nax, &mat_a) && matrix_stride(bt.sb, bt.nax, &mat_b) &&
              mat_a % 4 == 0 && mat_b % 4 == 0 && m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31);
    if (tc) {
        // inner extent / rows of each operand as stored
        const int64_t a_inner = ta ? m : k, a_rows = ta ? k : m;
        const int64_t b_inner = tb ? k : n, b_rows = tb ? n : k;
        const int64_t na = mat_a ? max_offset(bt, bt.sa) / mat_a + 1 : 1;
        const int64_t nb = mat_b ? max_offset(bt, bt.sb) / mat_b + 1 : 1;
        const int bn = choose_bn(m, n, batches);
        Maps maps;
        memset(&maps, 0, sizeof maps);
        tc = make_map(&maps.a, A, a_inner, a_rows, lda, na, mat_a, ta ? 32 : BM, !ta) &&
             make_map(&maps.b, B, b_inner, b_rows, ldb, nb, mat_b, tb ? bn : 32, tb);
        if (tc) {
            Params P;
            memset(&P, 0, sizeof P);
            P.A = A;
            P.B = B;
            P.lda = lda;
            P.ldb = ldb;
            P.M = m;
            P.N = n;
            P.K = k;
            P.ldc = ldc;
            P.stride_c = stride_c;
            P.mat_a = mat_a;
            P.mat_b = mat_b;
            P.nmma = (int32_t)(n >= bn ? bn : (n + 15) / 16 * 16);
            P.idesc = make_idesc(ta, tb, P.nmma);
            P.epi = epi;
            P.bt = bt;
            const int64_t KT = (k + BK - 1) / BK;
            const int64_t tiles = ((m + BM - 1) / BM) * ((n + bn - 1) / bn) * batches;
            int splits = choose_splits(tiles, KT, bn == 256 ? Tile<256>::KC_BLOCKS : Tile<128>::KC_BLOCKS);
            if (batches * splits > 65535 || epi.mode == EPI_SCATTER) splits = 1;  // the tile store is the scatter
            P.kb_per_split = (int32_t)((KT + splits - 1) / splits);
            P.splits = (int32_t)((KT + P.kb_per_split - 1) / P.kb_per_split);  // every split has a K slice
            // the tile leaves through the TMA where C (and the lo output) can
            // be described by a tensor map: 16-byte base, pitches multiples
            // of 4 floats
            if (P.splits == 1 && epi.mode != EPI_SCATTER && use_tma_store() && ((uintptr_t)C & 15) == 0 &&
                ldc % 4 == 0 && (batches == 1 || stride_c % 4 == 0) &&
                make_map(&maps.c, C, n, m, ldc, batches, stride_c, 32, true) &&
                (!epi.lo_out || (((uintptr_t)epi.lo_out & 15) == 0 &&
                                 make_map(&maps.clo, epi.lo_out, n, m, ldc, 1, 0, 32, true))))
                P.tma_store = 1;
            // lo halves from a split pass: scratch with each operand's own
            // geometry, the same tensor maps on another base
            // (or the caller's, when it supplies them)
            float *alo = nullptr, *blo = nullptr;  // scratch made here
            bool pre = use_presplit(m, n, batches, na, nb);
            if (pre) {
                cudaMemPool_t lpool = splitk_pool();
                if (!a_lo) a_lo = alo = split_operand(lpool, A, a_inner, a_rows, na, lda, mat_a, s);
                if (a_lo && !b_lo) b_lo = blo = split_operand(lpool, B, b_inner, b_rows, nb, ldb, mat_b, s);
                pre = a_lo && b_lo && make_map(&maps.alo, a_lo, a_inner, a_rows, lda, na, mat_a, ta ? 32 : BM, !ta) &&
                      make_map(&maps.blo, b_lo, b_inner, b_rows, ldb, nb, mat_b, tb ? bn : 32, tb);
            }
            P.batches = batches;
            P.group = raster_group((m + BM - 1) / BM, (n + bn - 1) / bn);
            int st;
            if (!pre && bn == 256 && use_persistent(P, tiles, KT)) {
                if (!ta && !tb) st = launch_persistent<false, false>(maps, C, P, tiles, s);
                else if (!ta && tb) st = launch_persistent<false, true>(maps, C, P, tiles, s);
                else if (ta && !tb) st = launch_persistent<true, false>(maps, C, P, tiles, s);
                else st = launch_persistent<true, true>(maps, C, P, tiles, s);
            } else if (pre) {
                st = bn == 256 ? dispatch_tf32x3<256, true>(ta, tb, maps, C, P, batches, s)
                               : dispatch_tf32x3<128, true>(ta, tb, maps, C, P, batches, s);
            } else {
                st = bn == 256 ? dispatch_tf32x3<256, false>(ta, tb, maps, C, P, batches, s)
                               : dispatch_tf32x3<128, false>(ta, tb, maps, C, P, batches, s);
            }
            if (alo) cudaFreeAsync(alo, s);
            if (blo) cudaFreeAsync(blo, s);
            return st;
        }
    }
    if (epi.mode == EPI_SCATTER) return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "scatter epilogue needs the TMA path");
    dim3 grid((unsigned)((n + 15) / 16), (unsigned)((m + 15) / 16), (unsigned)batches);
    if ((m + 15) / 16 > 65535) return ZPUCUDA_ERR_NOT_SUPPORTED;
#define ZC_FG(TA_, TB_) \
    fma_gemm_kernel<TA_, TB_><<<grid, 256, 0, s>>>(A, B, C, m, n, k, lda, ldb, ldc, bt, stride_c, epi)
    if (!ta && !tb) ZC_FG(false, false);
    else if (!ta && tb) ZC_FG(false, true);
    else if (ta && !tb) ZC_FG(true, false);
    else ZC_FG(true, true);
#undef ZC_FG
    ZC_LAUNCHED("fma_gemm_kernel");
    return ZPUCUDA_OK;
}

}  // namespace zc

extern "C" int zpucuda_check_device(void) {
    unsigned int e = 0;
    cudaError_t r = cudaMemcpyFromSymbol(&e, zc::g_gemm_error, sizeof e);
    if (r != cudaSuccess) return zc::cuda_fail(r, "cudaMemcpyFromSymbol(device error word)");
    if (e) return zc::set_error(ZPUCUDA_ERR_TIMEOUT, "a device-side bounded wait ran out in a GEMM kernel");
    return ZPUCUDA_OK;
}
