// The MLP train step as one device-resident program.
//
// The reference computes it op by op on the CPU: valueAndGrad of
// dense -> tanh -> dense -> tanh -> dense -> sparseCrossEntropy
// (src/zpu/transforms.zig:87-148, src/zpu/nn.zig:123-134,190-194,
// src/zpu/ops.zig:998-1010), the reverse sweep's rules for matmul, tanh, sum
// and the broadcast bias (src/zpu/autodiff.zig:51,323-330,451-454,480-487),
// then Adam.step with f32 moment state (src/zpu/optim.zig:183-259).
// Here the same arithmetic is lowered to 14 kernel launches (plus the split
// passes of the presplit lo halves, below) over buffers that stay in HBM (the
// two 16-column products run split-K, the CTAs of a tile adding their
// partials inside one cluster):
//   forward   3 GEMMs; bias + tanh run in the first two GEMMs' epilogues,
//             the bias of the logits in the third's;
//   loss      one kernel per 256 rows: log-softmax, the picked NLL, the loss
//             (block partials, last block sums them in order) and the
//             gradient of the logits, restating the reverse sweep of
//             logSoftmax / mul / sum / meanAll / neg step by step;
//   backward  5 GEMMs; the tanh VJP g * (1 - y^2) runs in the epilogue of
//             the GEMM that produces g; the transposed operands (swapLastTwo
//             views in the reference, materialised there by toContiguous,
//             src/zpu/tensor.zig:395-404) are read in place as MN-major
//             tiles; bias gradients are column sums (unbroadcast);
//   update    the fused Adam kernel, once per gradient bucket (below).
// Layout in HBM: parameters, gradients and both Adam moments are one
// contiguous f32 array each, parameters in the order W1 b1 W2 b2 W3 b3, each
// starting on a 256-byte boundary.  The output layer is padded to a multiple
// of 16 columns with zeros (W3, b3 and the logits), so every GEMM operand has
// a 16-byte row pitch for the TMA tensor maps and the narrow GEMMs run 16-wide
// MMAs; the padding stays exactly zero through every step (its gradients are
// products with zero columns, and Adam maps a zero gradient and zero moments
// to a zero update).
//
// Data parallelism: with an NCCL communicator on the device
// (zpucuda_nccl_init), each rank runs the step on its slice of the global
// batch with the loss scaled by 1/global_batch, and the gradient array is
// summed across ranks in two buckets on a side stream: [W2 .. end] (plus the
// loss) as soon as dW2 is done, overlapping the last two backward GEMMs, and
// [W1, b1] at the end.  In the full train step each bucket is reduce-
// scattered instead, each rank runs Adam on its 1/world shard and the
// parameters are all-gathered (same bytes, a world-th of the optimizer work),
// all on the side stream: [W2 .. end] as soon as its sum is in and the g1 GEMM
// has read W2 (overlapping dW1), [W1, b1] last.  The same per-bucket Adam
// split runs on one GPU, without the exchange.  (After a data-parallel step
// a rank's gradient and moment arrays are final only in its own shards.)
// dW2, the bulk of the bytes, does not go through NCCL at all when the ranks
// can map each other's memory: its GEMM stores every tile into the owning
// rank's inbox over NVLink (see "dW2 over peer memory" below).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "gemm.cuh"
#include "nccl.cuh"

namespace zc {
namespace {

constexpr int kXentThreads = 256;
constexpr int kColThreads = 256;
constexpr int kColRows = 128;   // rows summed by one column-sum block
constexpr int64_t kAlign = 64;  // floats: 256-byte parameter alignment
// floats: the two gradient buckets ([W1, b1] and [W2 .. b3]) are padded to
// this, so any world size dividing 256 cuts them into float4-aligned shards
constexpr int64_t kBucketAlign = 1024;
constexpr int kTail = 64;       // floats after the gradients: [0] = loss
constexpr int kMaxOut = 64;     // widest output layer the loss kernel takes

int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// ------------------------------------------------------------------ kernels

// Column sums of X [rows, n] (pitch ld) -> out [n]: unbroadcast of the bias
// gradient (src/zpu/autodiff.zig:51, an axis-0 sum).  Block (x, y) sums rows
// y*kColRows .. +kColRows of 256 columns in row order into partials[y][col];
// the last block of each column group to finish adds the partials in order.
// The result does not depend on block timing.
__global__ void __launch_bounds__(kColThreads) colsum_kernel(const float *__restrict__ X, int64_t rows, int64_t n,
                                                             int64_t ld, float *__restrict__ partials,
                                                             unsigned int *__restrict__ tickets,
                                                             float *__restrict__ out) {
    __shared__ bool last;
    const int64_t col = (int64_t)blockIdx.x * kColThreads + threadIdx.x;
    const int64_t r0 = (int64_t)blockIdx.y * kColRows;
    const int64_t r1 = r0 + kColRows < rows ? r0 + kColRows : rows;
    if (col < n) {
        float s = 0.0f;
        const float *p = X + r0 * ld + col;
#pragma unroll 8
        for (int64_t r = r0; r < r1; r++, p += ld) s = __fadd_rn(s, __ldg(p));
        partials[(int64_t)blockIdx.y * n + col] = s;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&tickets[blockIdx.x], 1u) == gridDim.y - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (col < n) {
        float t = 0.0f;
        for (unsigned y = 0; y < gridDim.y; y++) t = __fadd_rn(t, __ldcg(partials + (int64_t)y * n + col));
        out[col] = t;
    }
    if (threadIdx.x == 0) tickets[blockIdx.x] = 0;  // ready for the next launch
}

// max over the row with NaN propagation (src/zpu/ops.zig:662-700)
__device__ __forceinline__ float nan_max(float a, float b) { return (b > a || b != b) ? b : a; }

// One row per thread: logSoftmax (ops.zig:998-1010), picked NLL through the
// one-hot mask (nn.zig:123-134, 424-440), and the reverse sweep of those
// steps for the gradient of the logits, each step rounded to f32 as zpu's
// ops do.  The loss contribution of the rows, -(sum(nll) * inv_b), goes to
// *loss.  A label outside [0, d) sets *err (reported as IndexOutOfRange by
// zpucuda_mlp_check) and that row's one-hot row stays zero.
template <int MAXD>
__global__ void __launch_bounds__(kXentThreads)
    xent_kernel(const float *__restrict__ logits, const int64_t *__restrict__ labels, int64_t rows, int d, int ldl,
                float inv_b, float *__restrict__ gl, float *__restrict__ partials, unsigned int *__restrict__ ticket,
                float *__restrict__ loss, unsigned int *__restrict__ err) {
    __shared__ float warp_sums[kXentThreads / 32];
    __shared__ bool last;
    const int64_t row = (int64_t)blockIdx.x * kXentThreads + threadIdx.x;
    float nll = 0.0f;
    if (row < rows) {
        const float *lg = logits + row * ldl;
        float x[MAXD], e[MAXD], oh[MAXD];
        int64_t lab = labels[row];
        if (lab < 0 || lab >= d) {
            atomicOr(err, 1u);
            lab = -1;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < MAXD; j++) {
            x[j] = j < d ? lg[j] : 0.0f;
            oh[j] = (j == lab) ? 1.0f : 0.0f;
            if (j < d) mx = nan_max(mx, x[j]);
        }
        float zs = 0.0f;
#pragma unroll
        for (int j = 0; j < MAXD; j++) {
            e[j] = expf(__fsub_rn(x[j], mx));
            if (j < d) zs = __fadd_rn(zs, e[j]);
        }
        const float lz = logf(zs);
#pragma unroll
        for (int j = 0; j < MAXD; j++)
            if (j < d) nll = __fadd_rn(nll, __fmul_rn(__fsub_rn(__fsub_rn(x[j], mx), lz), oh[j]));
        // reverse sweep: d(loss)/d(picked) = -inv_b; through log(z), exp, and
        // the max (split evenly over tied maxima)
        const float gmean = -inv_b;
        float sum_glp = 0.0f;
#pragma unroll
        for (int j = 0; j < MAXD; j++)
            if (j < d) sum_glp = __fadd_rn(sum_glp, __fmul_rn(gmean, oh[j]));
        const float gz = __fdiv_rn(-sum_glp, zs);
        float gs[MAXD], sum_gs = 0.0f, cnt = 0.0f;
#pragma unroll
        for (int j = 0; j < MAXD; j++) {
            gs[j] = __fadd_rn(__fmul_rn(gmean, oh[j]), __fmul_rn(gz, e[j]));
            if (j < d) {
                sum_gs = __fadd_rn(sum_gs, gs[j]);
                cnt = __fadd_rn(cnt, x[j] == mx ? 1.0f : 0.0f);
            }
        }
        const float gm = -sum_gs;
        float *g = gl + row * ldl;
#pragma unroll
        for (int j = 0; j < MAXD; j++)
            if (j < ldl) g[j] = j < d ? __fadd_rn(gs[j], __fmul_rn(gm, __fdiv_rn(x[j] == mx ? 1.0f : 0.0f, cnt))) : 0.0f;
    }
    // deterministic block sum of nll, then the last block adds the partials
    float s = nll;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, o));
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = 0.0f;
        for (int w = 0; w < kXentThreads / 32; w++) b = __fadd_rn(b, warp_sums[w]);
        partials[blockIdx.x] = b;
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        float t = 0.0f;
        for (unsigned i = 0; i < gridDim.x; i++) t = __fadd_rn(t, __ldcg(partials + i));
        *loss = -__fmul_rn(t, inv_b);
        *ticket = 0;
    }
}

struct AdamConsts {
    float b1, omb1, b2, omb2, bc1, bc2, eps, lr;
};

__device__ __forceinline__ void adam1(float &p, float g, float &m, float &v, const AdamConsts &c) {
    const float nm = __fadd_rn(__fmul_rn(m, c.b1), __fmul_rn(g, c.omb1));
    const float nv = __fadd_rn(__fmul_rn(v, c.b2), __fmul_rn(__fmul_rn(g, g), c.omb2));
    m = nm;
    v = nv;
    const float den = __fadd_rn(__fsqrt_rn(__fdiv_rn(nv, c.bc2)), c.eps);
    p = __fsub_rn(p, __fmul_rn(__fdiv_rn(__fdiv_rn(nm, c.bc1), den), c.lr));
}

// Adam.step (src/zpu/optim.zig:183-259) for f32 parameters and gradients with
// f32 moments: every step of the reference is an f32 op (its scalar constants
// rounded to f32 by mulScalar/divScalar/scalarLike, ops.zig:335-345,539;
// subInPlace's f64 subtract of two f32 values rounds to the f32 subtract,
// optim.zig:20-31), so each is one correctly rounded f32 op here, in the same
// order, with no contraction into FMAs.
__global__ void __launch_bounds__(256) adam_kernel(float4 *__restrict__ p, const float4 *__restrict__ g,
                                                   float4 *__restrict__ m, float4 *__restrict__ v, int64_t n4,
                                                   const AdamConsts c) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 pp = p[i], mm = m[i], vv = v[i];
        const float4 gg = __ldcs(g + i);
        adam1(pp.x, gg.x, mm.x, vv.x, c);
        adam1(pp.y, gg.y, mm.y, vv.y, c);
        adam1(pp.z, gg.z, mm.z, vv.z, c);
        adam1(pp.w, gg.w, mm.w, vv.w, c);
        p[i] = pp;
        m[i] = mm;
        v[i] = vv;
    }
}

// std.math.pow(f64, x, y) as the reference's Adam calls it for the bias
// corrections (optim.zig:199-200): the integer part of y by repeated squaring
// of frexp(x)'s mantissa with the binary exponent tracked apart, a
// fractional part through exp(yf * log(x)), then ldexp.  Finite x > 0 only.
double zig_pow(double x, double y) {
    if (y == 0.0 || x == 1.0) return 1.0;
    if (y == 1.0) return x;
    if (x != x || y != y) return NAN;
    if (x <= 0.0 || isinf(x) || isinf(y)) return pow(x, y);
    if (y == 0.5) return sqrt(x);
    if (y == -0.5) return 1.0 / sqrt(x);
    double yi, yf = modf(fabs(y), &yi);
    if (yi >= 9.223372036854775808e18) return pow(x, y);
    double acc = 1.0;
    long exp_acc = 0;
    if (yf != 0.0) {
        if (yf > 0.5) {
            yf -= 1.0;
            yi += 1.0;
        }
        acc = exp(yf * log(x));
    }
    int e0;
    double mant = frexp(x, &e0);
    long xe = e0;
    for (int64_t i = (int64_t)yi; i != 0; i >>= 1) {
        if (xe < -(1L << 12) || (1L << 12) < xe) {
            exp_acc += xe;
            break;
        }
        if (i & 1) {
            acc *= mant;
            exp_acc += xe;
        }
        mant *= mant;
        xe <<= 1;
        if (mant < 0.5) {
            mant += mant;
            xe--;
        }
    }
    if (y < 0) {
        acc = 1.0 / acc;
        exp_acc = -exp_acc;
    }
    return ldexp(acc, (int)exp_acc);
}

constexpr size_t kXferFlagBytes = 4096;  // flags: world x u64, error word at byte 2048
constexpr uint32_t kXferSpin = 1u << 24;  // ~256 ns each: a few seconds

struct XferFlags {
    unsigned long long *flag[kMaxPeers];  // rank r's flag array, mapped here
};

__global__ void xfer_signal_kernel(const __grid_constant__ XferFlags f, int world, int src,
                                   unsigned long long epoch) {
    __threadfence_system();
    for (int r = 0; r < world; r++)
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f.flag[r] + src), "l"(epoch) : "memory");
}

// out[i] = sum over s of inbox[s * n + i], s in rank order, once every rank's
// flag shows `epoch`; a wait that runs out (spin_limit polls ~256 ns apart)
// sets *err and writes nothing.
__global__ void __launch_bounds__(256) xfer_reduce_kernel(const float4 *__restrict__ inbox, int world, int64_t n4,
                                                          float4 *__restrict__ out,
                                                          const unsigned long long *flags,
                                                          unsigned long long epoch, unsigned int *err,
                                                          uint32_t spin_limit) {
    __shared__ int ready;
    if (threadIdx.x == 0) {
        int ok = 0;
        for (uint32_t it = 0; it < spin_limit && !ok; it++) {
            ok = 1;
            for (int r = 0; r < world; r++) {
                unsigned long long v;
                asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + r) : "memory");
                if (v < epoch) ok = 0;
            }
            if (!ok) __nanosleep(256);
        }
        if (!ok) atomicOr(err, 1u);
        ready = ok;
    }
    __syncthreads();
    if (!ready) return;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 a = __ldcg(inbox + i);
        for (int s = 1; s < world; s++) {
            const float4 b = __ldcg(inbox + (int64_t)s * n4 + i);
            a.x = __fadd_rn(a.x, b.x);
            a.y = __fadd_rn(a.y, b.y);
            a.z = __fadd_rn(a.z, b.z);
            a.w = __fadd_rn(a.w, b.w);
        }
        out[i] = a;
    }
}

}  // namespace
}  // namespace zc

using namespace zc;

// Phase boundaries the trace records, in this order: main stream -- start,
// forward GEMMs, loss, layer-3 backward + db2, dW2 GEMM, g1 GEMM, db1 + dW1
// GEMM, end (side stream joined); side stream -- bucket [W2 ..] summed,
// its Adam, bucket [W1, b1] summed, its Adam + all-gather, the all-gather of
// bucket [W2 ..] (which the next step joins before it reads W2).
constexpr int kTracePoints = 13;

struct zpucuda_mlp {
    int device = -1;
    int64_t d[4] = {0, 0, 0, 0};  // d_in, d_h1, d_h2, d_out
    int64_t d3p = 0;              // d_out padded to a multiple of 16
    int64_t max_batch = 0;
    // parameter i: rows x cols (pitch ld) at offset off[i] of each array
    int64_t rows[6], cols[6], ld[6], off[6];
    int64_t total = 0;  // floats per array (multiple of kAlign)
    float *params = nullptr, *grads = nullptr, *m = nullptr, *v = nullptr;
    float *a1 = nullptr, *a2 = nullptr, *ga2 = nullptr, *ga1 = nullptr, *logits = nullptr, *gl = nullptr;
    // lo halves of the TF32 split of the big products' operands, made once
    // per step (x, W1, W2 by a split pass; a1, ga2, ga1 by the epilogue that
    // writes them) and read by every product that takes them
    float *x_lo = nullptr, *w1_lo = nullptr, *w2_lo = nullptr, *a1_lo = nullptr, *ga2_lo = nullptr, *ga1_lo = nullptr;
    float *col_partials[3] = {nullptr, nullptr, nullptr};
    float *xent_partials = nullptr;
    unsigned int *counters = nullptr;  // colsum tickets x3 groups, xent ticket, label error
    int64_t col_groups[3] = {0, 0, 0};
    int64_t t = 0;  // Adam steps taken
    double lr = 1e-3, beta1 = 0.9, beta2 = 0.999, eps = 1e-8;
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t ev_a = nullptr, ev_b = nullptr, ev_w2 = nullptr, ev_done = nullptr, ev_w1 = nullptr;
    // a data-parallel step leaves the all-gather of bucket [W2 ..] running on
    // the side stream (ev_done); the next call that touches the arrays waits
    // for it on its own stream (join_exchange)
    bool w2_pending = false;
    // dW2 exchange over peer memory (data parallel): one allocation per rank,
    // [flags | inbox], opened on every peer through CUDA IPC
    int peer_state = 0;  // 0 not set up, 1 in use, -1 not available
    int peer_world = 0, peer_rank = 0;
    uint8_t *xfer = nullptr;                    // this rank's [flags | inbox]
    uint8_t *peer_base[kMaxPeers] = {};         // every rank's allocation, mapped here
    unsigned long long epoch = 0;               // dW2 exchanges so far
    // phase trace (zpucuda_mlp_trace): timing events at the step's phase
    // boundaries, on the main stream (kTraceMain) and the side stream
    bool trace = false;
    cudaEvent_t tev[kTracePoints] = {};
    std::mutex mu;

    float *loss_ptr() const { return grads + total; }
    unsigned int *tickets(int i) const {
        int64_t o = 0;
        for (int j = 0; j < i; j++) o += col_groups[j];
        return counters + o;
    }
    unsigned int *xent_ticket() const { return counters + col_groups[0] + col_groups[1] + col_groups[2]; }
    unsigned int *label_error() const { return xent_ticket() + 1; }
};

namespace {

void free_mlp(zpucuda_mlp *h) {
    float *bufs[] = {h->params, h->grads, h->m,   h->v,           h->a1,          h->a2,          h->ga2,
                     h->ga1,    h->logits, h->gl, h->col_partials[0], h->col_partials[1], h->col_partials[2],
                     h->xent_partials, h->x_lo, h->w1_lo, h->w2_lo, h->a1_lo, h->ga2_lo, h->ga1_lo};
    for (float *b : bufs)
        if (b) cudaFree(b);
    for (int r = 0; r < kMaxPeers; r++)
        if (h->peer_base[r] && h->peer_base[r] != h->xfer) cudaIpcCloseMemHandle(h->peer_base[r]);
    if (h->xfer) cudaFree(h->xfer);
    if (h->counters) cudaFree(h->counters);
    if (h->ev_a) cudaEventDestroy(h->ev_a);
    if (h->ev_b) cudaEventDestroy(h->ev_b);
    if (h->ev_w2) cudaEventDestroy(h->ev_w2);
    if (h->ev_done) cudaEventDestroy(h->ev_done);
    if (h->ev_w1) cudaEventDestroy(h->ev_w1);
    for (cudaEvent_t e : h->tev)
        if (e) cudaEventDestroy(e);
    if (h->comm_stream) cudaStreamDestroy(h->comm_stream);
    delete h;
}

int alloc_f32(float **p, int64_t n) {
    cudaError_t e = cudaMalloc((void **)p, (size_t)n * sizeof(float));
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return set_error(ZPUCUDA_ERR_OUT_OF_MEMORY, "cudaMalloc (mlp)");
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (mlp)");
    return ZPUCUDA_OK;
}

int colsum(zpucuda_mlp *h, int which, const float *X, int64_t rows, int64_t n, int64_t ld, float *out,
           cudaStream_t s) {
    const int64_t gy = (rows + kColRows - 1) / kColRows;
    dim3 grid((unsigned)((n + kColThreads - 1) / kColThreads), (unsigned)gy);
    colsum_kernel<<<grid, kColThreads, 0, s>>>(X, rows, n, ld, h->col_partials[which], h->tickets(which), out);
    ZC_LAUNCHED("colsum_kernel");
    return ZPUCUDA_OK;
}

int gemm(const float *A, const float *B, float *C, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
         int64_t ldc, bool ta, bool tb, const Epilogue &e, cudaStream_t s, const float *a_lo = nullptr,
         const float *b_lo = nullptr) {
    GemmBatch one;
    memset(&one, 0, sizeof one);
    return gemm_f32_device_lo(A, B, C, m, n, k, lda, ldb, ldc, ta, tb, one, 0, e, a_lo, b_lo, s);
}

// e with its lo halves written to `lo` when `want` (a later product reads them)
Epilogue with_lo(Epilogue e, bool want, float *lo) {
    e.lo_out = want ? lo : nullptr;
    return e;
}

Epilogue epi(int32_t mode, const float *bias, const float *aux = nullptr, int64_t ldaux = 0) {
    Epilogue e;
    e.mode = mode;
    e.bias = bias;
    e.aux = aux;
    e.ldaux = ldaux;
    return e;
}

#define ZC_TRY(x)              \
    do {                       \
        int st_ = (x);         \
        if (st_) return st_;   \
    } while (0)

AdamConsts adam_consts(zpucuda_mlp *h);
int adam_range(zpucuda_mlp *h, const AdamConsts &c, int64_t off, int64_t n, cudaStream_t s);

// ---------------------------------------------------- dW2 over peer memory
//
// The data-parallel step's largest gradient, dW2 [d_h1, d_h2], is
// reduce-scattered by its own GEMM: rank r owns rows [r R, (r+1) R)
// (R = d_h1 / world), and the GEMM's tile store writes every row straight into
// slot `src` of its owner's inbox -- across NVLink for a peer -- so the
// exchange overlaps the math tile by tile (gemm_f32.cu, EPI_SCATTER).  The
// GEMM is followed on the same stream by a one-thread kernel that publishes
// this step's epoch to every rank's flag for `src` (system-scope release after
// a system fence); the owner's reduction waits (bounded) until every flag
// carries the epoch, then adds the world slots in rank order.  The next
// step's GEMM cannot overwrite an inbox early: it starts only after this
// step's parameter all-gather, which needs every owner's reduced shard.
unsigned int *xfer_error(const zpucuda_mlp *h) { return (unsigned int *)(h->xfer + 2048); }
float *xfer_inbox(const zpucuda_mlp *h, int r) { return (float *)(h->peer_base[r] + kXferFlagBytes); }

// Sets up the dW2 exchange once (every rank at the same point of its first
// data-parallel step): allocate [flags | inbox], swap IPC handles with an
// NCCL all-gather, open the peers' allocations, and agree across ranks
// (an allreduce of the outcome) so that either all use it or none.
// Used by default from kPeerExchangeMinWorld ranks on: with fewer, NCCL's
// reduce-scatter of dW2 hides completely under the g1 GEMM on the side stream
// while the tile stores sit inside dW2's GEMM (measured on B200: 3 % slower at
// 2 and 4 ranks, 11 % faster at 8).  ZPUCUDA_MLP_PEER_EXCHANGE=1 / =0 (the
// same on every rank) forces it on / off.
constexpr int kPeerExchangeMinWorld = 6;

// The last bucket ([W1, b1], summed after the final GEMM with nothing left to
// overlap it) as one allreduce with Adam over the whole bucket on every rank,
// instead of reduce-scatter + Adam on a shard + all-gather: one collective's
// latency instead of two.  ZPUCUDA_MLP_LAST_BUCKET_ALLREDUCE=1 / =0 (the same
// on every rank) forces it on / off; the default is off.
bool last_bucket_allreduce(int world) {
    static const int env = [] {
        const char *e = getenv("ZPUCUDA_MLP_LAST_BUCKET_ALLREDUCE");
        return e && e[0] ? (e[0] != '0' ? 1 : 0) : -1;
    }();
    (void)world;
    return env == 1;
}

int peer_setup(zpucuda_mlp *h, int world, int rank, cudaStream_t s) {
    h->peer_state = -1;
    const char *env = getenv("ZPUCUDA_MLP_PEER_EXCHANGE");
    const bool want = env && env[0] ? env[0] != '0' : world >= kPeerExchangeMinWorld;
    if (!want || world < 2 || world > kMaxPeers || h->d[1] % world || ((h->d[1] / world) * h->d[2]) % 4)
        return ZPUCUDA_OK;
    const size_t bytes = kXferFlagBytes + (size_t)h->d[1] * (size_t)h->d[2] * sizeof(float);
    float ok = 1.0f;
    cudaIpcMemHandle_t mine;
    memset(&mine, 0, sizeof mine);
    if (cudaMalloc((void **)&h->xfer, bytes) != cudaSuccess ||
        cudaMemset(h->xfer, 0, kXferFlagBytes) != cudaSuccess || cudaIpcGetMemHandle(&mine, h->xfer) != cudaSuccess) {
        cudaGetLastError();
        ok = 0.0f;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    float *d_ex = nullptr;  // world handles (16 floats each) + the agreement word
    ZC_CUDA(cudaMalloc((void **)&d_ex, (size_t)(world * 16 + 1) * sizeof(float)));
    ZC_CUDA(cudaMemcpyAsync(d_ex + rank * 16, &mine, 64, cudaMemcpyHostToDevice, s));
    int st = nccl_all_gather_f32(d_ex, 16, s);
    std::vector<cudaIpcMemHandle_t> all(world);
    if (!st) st = cudaMemcpyAsync(all.data(), d_ex, (size_t)world * 64, cudaMemcpyDeviceToHost, s) == cudaSuccess
                      ? ZPUCUDA_OK
                      : cuda_fail(cudaGetLastError(), "copy IPC handles");
    if (!st) st = cudaStreamSynchronize(s) == cudaSuccess ? ZPUCUDA_OK : cuda_fail(cudaGetLastError(), "sync");
    h->peer_base[rank] = h->xfer;
    for (int r = 0; r < world && !st && ok != 0.0f; r++) {
        if (r == rank) continue;
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = 0.0f;
            break;
        }
        h->peer_base[r] = (uint8_t *)p;
    }
    if (!st) st = cudaMemcpyAsync(d_ex + world * 16, &ok, sizeof ok, cudaMemcpyHostToDevice, s) == cudaSuccess
                      ? ZPUCUDA_OK
                      : cuda_fail(cudaGetLastError(), "agreement word");
    if (!st) st = nccl_allreduce_sum_f32(d_ex + world * 16, 1, s);
    float agreed = 0.0f;
    if (!st) st = cudaMemcpyAsync(&agreed, d_ex + world * 16, sizeof agreed, cudaMemcpyDeviceToHost, s) == cudaSuccess
                      ? ZPUCUDA_OK
                      : cuda_fail(cudaGetLastError(), "agreement word");
    if (!st) st = cudaStreamSynchronize(s) == cudaSuccess ? ZPUCUDA_OK : cuda_fail(cudaGetLastError(), "sync");
    cudaFree(d_ex);
    if (st || agreed != (float)world) {  // someone could not map a peer: everyone keeps NCCL
        for (int r = 0; r < kMaxPeers; r++) {
            if (h->peer_base[r] && h->peer_base[r] != h->xfer) cudaIpcCloseMemHandle(h->peer_base[r]);
            h->peer_base[r] = nullptr;
        }
        if (h->xfer) cudaFree(h->xfer);
        h->xfer = nullptr;
        return st;
    }
    h->peer_world = world;
    h->peer_rank = rank;
    h->peer_state = 1;
    return ZPUCUDA_OK;
}

// Forward, loss and backward.  With `ar` set, the gradient buckets are summed
// across ranks on the side stream as they become ready; with `adam` set, the
// Adam update of each bucket follows on the side stream too: [W2 .. b3] once
// its gradients are final and the g1 GEMM has read W2, overlapping dW1, then
// [W1, b1] at the end.
// Records trace point i on stream st when the trace is on.
inline int tmark(zpucuda_mlp *h, int i, cudaStream_t st) {
    if (!h->trace) return ZPUCUDA_OK;
    ZC_CUDA(cudaEventRecord(h->tev[i], st));
    return ZPUCUDA_OK;
}

// Makes stream st wait for the all-gather of bucket [W2 ..] that the last
// data-parallel step left running on the side stream.
int join_exchange(const zpucuda_mlp *h, cudaStream_t st) {
    if (h->w2_pending) ZC_CUDA(cudaStreamWaitEvent(st, h->ev_done, 0));
    return ZPUCUDA_OK;
}

int value_and_grad(zpucuda_mlp *h, const float *x, const int64_t *labels, int64_t B, int64_t global_b, bool ar,
                   bool adam, cudaStream_t s) {
    const int64_t d0 = h->d[0], d1 = h->d[1], d2 = h->d[2], d3 = h->d[3], d3p = h->d3p;
    const float *W1 = h->params + h->off[0], *b1 = h->params + h->off[1];
    const float *W2 = h->params + h->off[2], *b2 = h->params + h->off[3];
    const float *W3 = h->params + h->off[4], *b3 = h->params + h->off[5];
    float *gW1 = h->grads + h->off[0], *gb1 = h->grads + h->off[1];
    float *gW2 = h->grads + h->off[2], *gb2 = h->grads + h->off[3];
    float *gW3 = h->grads + h->off[4], *gb3 = h->grads + h->off[5];
    int rank = 0;
    const int world = ar ? nccl_world(&rank) : 1;
    if (ar && adam && world > 1 && h->peer_state == 0) ZC_TRY(peer_setup(h, world, rank, h->comm_stream));

    // The big products that read the lo halves of their operands from HBM
    // (gemm_f32_presplit): each such operand's lo is made once, here by a
    // split pass (x and the weights) or by the epilogue of the product that
    // writes it (a1, ga2, ga1), and handed to every product that reads it.
    const bool p_f1 = gemm_f32_presplit(B, d1, 1), p_f2 = gemm_f32_presplit(B, d2, 1);
    const bool p_w2 = gemm_f32_presplit(d1, d2, 1), p_g1 = gemm_f32_presplit(B, d1, 1);
    const bool p_w1 = gemm_f32_presplit(d0, d1, 1);
    const bool x_al = ((uintptr_t)x & 15) == 0;
    const float *x_lo = nullptr, *w1_lo = nullptr, *w2_lo = nullptr;
    if ((p_f1 || p_w1) && x_al) {
        ZC_TRY(split_lo_device(x, h->x_lo, B * d0, s));
        x_lo = h->x_lo;
    }
    if (p_f1) {
        ZC_TRY(split_lo_device(W1, h->w1_lo, d0 * d1, s));
        w1_lo = h->w1_lo;
    }
    const bool a1_lo = p_f2 || p_w2, ga2_lo = p_w2 || p_g1, ga1_lo = p_w1;

    // forward: dense -> tanh -> dense -> tanh -> dense
    ZC_TRY(tmark(h, 0, s));
    ZC_TRY(gemm(x, W1, h->a1, B, d1, d0, d0, d1, d1, false, false, with_lo(epi(EPI_BIAS_TANH, b1), a1_lo, h->a1_lo),
                s, x_lo, w1_lo));
    // W2 .. b3 from here on: the last step's all-gather of them ran beside
    // the split passes and the first product
    ZC_TRY(join_exchange(h, s));
    h->w2_pending = false;
    if (p_f2 || p_g1) {
        ZC_TRY(split_lo_device(W2, h->w2_lo, d1 * d2, s));
        w2_lo = h->w2_lo;
    }
    ZC_TRY(gemm(h->a1, W2, h->a2, B, d2, d1, d1, d2, d2, false, false, epi(EPI_BIAS_TANH, b2), s,
                a1_lo ? h->a1_lo : nullptr, w2_lo));
    ZC_TRY(gemm(h->a2, W3, h->logits, B, d3p, d2, d2, d3p, d3p, false, false, epi(EPI_BIAS, b3), s));
    ZC_TRY(tmark(h, 1, s));

    // loss and d(loss)/d(logits)
    const float inv_b = (float)(1.0 / (double)global_b);
    const unsigned xb = (unsigned)((B + kXentThreads - 1) / kXentThreads);
    if (d3p <= 16)
        xent_kernel<16><<<xb, kXentThreads, 0, s>>>(h->logits, labels, B, (int)d3, (int)d3p, inv_b, h->gl,
                                                    h->xent_partials, h->xent_ticket(), h->loss_ptr(),
                                                    h->label_error());
    else
        xent_kernel<kMaxOut><<<xb, kXentThreads, 0, s>>>(h->logits, labels, B, (int)d3, (int)d3p, inv_b, h->gl,
                                                         h->xent_partials, h->xent_ticket(), h->loss_ptr(),
                                                         h->label_error());
    ZC_LAUNCHED("xent_kernel");
    ZC_TRY(tmark(h, 2, s));

    // layer 3: dW3 = a2^T gl, db3 = colsum(gl), g_a2 = (gl W3^T) * (1 - a2^2)
    ZC_TRY(gemm(h->a2, h->gl, gW3, d2, d3p, B, d2, d3p, d3p, true, false, Epilogue{}, s));
    ZC_TRY(colsum(h, 2, h->gl, B, d3p, d3p, gb3, s));
    ZC_TRY(gemm(h->gl, W3, h->ga2, B, d2, d3p, d3p, d3p, d2, false, true,
                with_lo(epi(EPI_TANH_GRAD, nullptr, h->a2, d2), ga2_lo, h->ga2_lo), s));
    // layer 2
    ZC_TRY(colsum(h, 1, h->ga2, B, d2, d2, gb2, s));
    ZC_TRY(tmark(h, 3, s));
    const int64_t nA = h->total - h->off[2], nB = h->off[2], nA3 = h->total - h->off[3];
    const bool shard = ar && adam && nA % (4 * world) == 0 && nB % (4 * world) == 0;
    const bool fused = shard && h->peer_state == 1 && h->peer_world == world && nA3 % (4 * world) == 0;
    const int64_t w2_shard = d1 / world * d2;  // floats of dW2 a rank owns (fused)
    if (fused) {  // dW2's tiles go straight into their owners' inboxes
        Epilogue se;
        se.mode = EPI_SCATTER;
        for (int r = 0; r < world; r++) se.peer[r] = xfer_inbox(h, r);
        se.rows_per_owner = d1 / world;
        se.src = rank;
        se.world = world;
        ZC_TRY(gemm(h->a1, h->ga2, gW2, d1, d2, B, d1, d2, d2, true, false, se, s, a1_lo ? h->a1_lo : nullptr,
                    ga2_lo ? h->ga2_lo : nullptr));
        XferFlags f;
        memset(&f, 0, sizeof f);
        for (int r = 0; r < world; r++) f.flag[r] = (unsigned long long *)h->peer_base[r];
        h->epoch += 1;
        xfer_signal_kernel<<<1, 1, 0, s>>>(f, world, rank, h->epoch);
        ZC_LAUNCHED("xfer_signal_kernel");
    } else {
        ZC_TRY(gemm(h->a1, h->ga2, gW2, d1, d2, B, d1, d2, d2, true, false, Epilogue{}, s, a1_lo ? h->a1_lo : nullptr,
                    ga2_lo ? h->ga2_lo : nullptr));
    }
    ZC_TRY(tmark(h, 4, s));
    cudaStream_t side = h->comm_stream;
    // With a communicator and Adam in the step, each rank updates only its
    // 1/world shard of each bucket: reduce-scatter the gradients, Adam on the
    // shard, all-gather the parameters (the same bytes as an allreduce, and a
    // world-th of the optimizer work).
    if (ar) {
        ZC_CUDA(cudaEventRecord(h->ev_a, s));
        ZC_CUDA(cudaStreamWaitEvent(side, h->ev_a, 0));
        if (fused) {
            // b2, W3, b3 and the loss (70 K floats) in one NCCL allreduce; dW2 is
            // already in the inboxes: add this rank's slots as soon as every
            // peer's flag is up, overlapping the g1 GEMM
            ZC_TRY(nccl_allreduce_sum_f32(h->grads + h->off[3], nA3 + 1, side));
            const int64_t n4 = w2_shard / 4;
            int64_t blocks = (n4 + 255) / 256;
            if (blocks > (int64_t)num_sms() * 4) blocks = (int64_t)num_sms() * 4;
            xfer_reduce_kernel<<<(unsigned)blocks, 256, 0, side>>>(
                (const float4 *)xfer_inbox(h, rank), world, n4, (float4 *)(h->grads + h->off[2] + rank * w2_shard),
                (const unsigned long long *)h->xfer, h->epoch, xfer_error(h), kXferSpin);
            ZC_LAUNCHED("xfer_reduce_kernel");
        } else if (shard) {
            ZC_TRY(nccl_reduce_scatter_sum_f32(h->grads + h->off[2], nA / world, side));
            ZC_TRY(nccl_allreduce_sum_f32(h->loss_ptr(), 1, side));
        } else {
            ZC_TRY(nccl_allreduce_sum_f32(h->grads + h->off[2], nA + 1, side));
        }
        ZC_TRY(tmark(h, 8, side));
    }
    ZC_TRY(gemm(h->ga2, W2, h->ga1, B, d1, d2, d2, d2, d1, false, true,
                with_lo(epi(EPI_TANH_GRAD, nullptr, h->a1, d1), ga1_lo, h->ga1_lo), s, ga2_lo ? h->ga2_lo : nullptr,
                w2_lo));
    ZC_TRY(tmark(h, 5, s));
    AdamConsts ac;
    if (adam) {  // every later kernel on s leaves W2, b2, W3, b3 alone
        ac = adam_consts(h);
        ZC_CUDA(cudaEventRecord(h->ev_w2, s));
        ZC_CUDA(cudaStreamWaitEvent(side, h->ev_w2, 0));
        if (fused) {  // Adam on this rank's dW2 rows; b2, W3, b3 everywhere (W2 gathered last)
            ZC_TRY(adam_range(h, ac, h->off[2] + rank * w2_shard, w2_shard, side));
            ZC_TRY(adam_range(h, ac, h->off[3], nA3, side));
        } else if (shard) {  // Adam on this rank's shard of the bucket (gathered last)
            ZC_TRY(adam_range(h, ac, h->off[2] + rank * (nA / world), nA / world, side));
        } else {
            ZC_TRY(adam_range(h, ac, h->off[2], nA, side));
        }
        ZC_TRY(tmark(h, 9, side));
    }
    // layer 1
    ZC_TRY(colsum(h, 0, h->ga1, B, d1, d1, gb1, s));
    ZC_TRY(gemm(x, h->ga1, gW1, d0, d1, B, d0, d1, d1, true, false, Epilogue{}, s, x_lo,
                ga1_lo ? h->ga1_lo : nullptr));
    ZC_TRY(tmark(h, 6, s));
    if (ar || adam) {
        ZC_CUDA(cudaEventRecord(h->ev_b, s));
        ZC_CUDA(cudaStreamWaitEvent(side, h->ev_b, 0));
        if (shard && !last_bucket_allreduce(world)) {
            ZC_TRY(nccl_reduce_scatter_sum_f32(h->grads, nB / world, side));
            ZC_TRY(tmark(h, 10, side));
            ZC_TRY(adam_range(h, ac, rank * (nB / world), nB / world, side));
            ZC_TRY(nccl_all_gather_f32(h->params, nB / world, side));
        } else {
            if (ar) ZC_TRY(nccl_allreduce_sum_f32(h->grads, nB, side));
            ZC_TRY(tmark(h, 10, side));
            if (adam) ZC_TRY(adam_range(h, ac, 0, nB, side));
        }
        ZC_TRY(tmark(h, 11, side));
        if (adam && (fused || shard)) {
            // the step ends once W1 is whole; the gather of bucket [W2 ..]
            // (the larger one) follows on the side stream and overlaps the
            // next step's split passes and first product (join_exchange)
            ZC_CUDA(cudaEventRecord(h->ev_w1, side));
            ZC_CUDA(cudaStreamWaitEvent(s, h->ev_w1, 0));
            if (fused) ZC_TRY(nccl_all_gather_f32(h->params + h->off[2], w2_shard, side));
            else ZC_TRY(nccl_all_gather_f32(h->params + h->off[2], nA / world, side));
            ZC_TRY(tmark(h, 12, side));
            ZC_CUDA(cudaEventRecord(h->ev_done, side));
            h->w2_pending = true;
        } else {
            ZC_CUDA(cudaEventRecord(h->ev_done, side));
            ZC_CUDA(cudaStreamWaitEvent(s, h->ev_done, 0));
        }
    }
    ZC_TRY(tmark(h, 7, s));
    return ZPUCUDA_OK;
}

// One Adam.step's constants (the step counter advances).
AdamConsts adam_consts(zpucuda_mlp *h) {
    h->t += 1;
    const double bc1 = 1.0 - zig_pow(h->beta1, (double)h->t);
    const double bc2 = 1.0 - zig_pow(h->beta2, (double)h->t);
    AdamConsts c;
    c.b1 = (float)h->beta1;
    c.omb1 = (float)(1.0 - h->beta1);
    c.b2 = (float)h->beta2;
    c.omb2 = (float)(1.0 - h->beta2);
    c.bc1 = (float)bc1;
    c.bc2 = (float)bc2;
    c.eps = (float)h->eps;
    c.lr = (float)h->lr;
    return c;
}

// Adam over floats [off, off + n) of the arrays (off and n multiples of 4).
int adam_range(zpucuda_mlp *h, const AdamConsts &c, int64_t off, int64_t n, cudaStream_t s) {
    const int64_t n4 = n / 4;
    int64_t blocks = (n4 + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) return ZPUCUDA_OK;
    adam_kernel<<<(unsigned)blocks, 256, 0, s>>>((float4 *)(h->params + off), (const float4 *)(h->grads + off),
                                                 (float4 *)(h->m + off), (float4 *)(h->v + off), n4, c);
    ZC_LAUNCHED("adam_kernel");
    return ZPUCUDA_OK;
}

int adam_step(zpucuda_mlp *h, cudaStream_t s) {
    const AdamConsts c = adam_consts(h);
    return adam_range(h, c, 0, h->total, s);
}

int check_step_args(zpucuda_mlp *h, const float *x, const int64_t *labels, int64_t B, int64_t global_b) {
    if (!h || !x || !labels) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp: NULL argument");
    if (B < 1 || B > h->max_batch || global_b < B)
        return set_error(ZPUCUDA_ERR_INVALID_SHAPE, "mlp: batch must be in [1, max_batch] and <= global_batch");
    if (current_device() != h->device) return set_error(ZPUCUDA_ERR_DEVICE_MISMATCH, "mlp: wrong device bound");
    if ((uintptr_t)x % 16) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp: x must be 16-byte aligned");
    return ZPUCUDA_OK;
}

// parameter / gradient / moment array selected by `what`
float *array_of(const zpucuda_mlp *h, int what) {
    switch (what) {
        case ZPUCUDA_MLP_PARAM: return h->params;
        case ZPUCUDA_MLP_GRAD: return h->grads;
        case ZPUCUDA_MLP_ADAM_M: return h->m;
        case ZPUCUDA_MLP_ADAM_V: return h->v;
        default: return nullptr;
    }
}

}  // namespace

extern "C" int zpucuda_mlp_create(int64_t d_in, int64_t d_h1, int64_t d_h2, int64_t d_out, int64_t max_batch,
                                  zpucuda_mlp **out) {
    if (!out) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_create: out is NULL");
    *out = nullptr;
    if (d_in < 1 || d_h1 < 1 || d_h2 < 1 || d_out < 1 || max_batch < 1)
        return set_error(ZPUCUDA_ERR_INVALID_SHAPE, "mlp_create: every size must be >= 1");
    if (d_out > kMaxOut) return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "mlp_create: more than 64 output classes");
    if (max_batch > (1LL << 30) || d_in > (1LL << 30) || d_h1 > (1LL << 30) || d_h2 > (1LL << 30))
        return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "mlp_create: size too large");
    const int dev = current_device();
    if (dev < 0) return set_error(ZPUCUDA_ERR_NO_DEVICE, "mlp_create: no device");
    zpucuda_mlp *h = new zpucuda_mlp();
    h->device = dev;
    h->d[0] = d_in;
    h->d[1] = d_h1;
    h->d[2] = d_h2;
    h->d[3] = d_out;
    h->d3p = round_up(d_out, 16);
    h->max_batch = max_batch;
    const int64_t r[6] = {d_in, 1, d_h1, 1, d_h2, 1};
    const int64_t c[6] = {d_h1, d_h1, d_h2, d_h2, d_out, d_out};
    const int64_t l[6] = {d_h1, d_h1, d_h2, d_h2, h->d3p, h->d3p};
    int64_t o = 0;
    for (int i = 0; i < 6; i++) {
        h->rows[i] = r[i];
        h->cols[i] = c[i];
        h->ld[i] = l[i];
        if (i == 2 || i == 3) o = round_up(o, kBucketAlign);  // buckets [W2 .. b3] and [b2 .. b3] start here
        h->off[i] = o;
        o += round_up(r[i] * l[i], kAlign);
    }
    h->total = round_up(o, kBucketAlign);
    const int64_t R = (max_batch + kColRows - 1) / kColRows;
    const int64_t widths[3] = {d_h1, d_h2, h->d3p};
    int64_t n_counters = 2;
    for (int i = 0; i < 3; i++) {
        h->col_groups[i] = (widths[i] + kColThreads - 1) / kColThreads;
        n_counters += h->col_groups[i];
    }
    int st = ZPUCUDA_OK;
    if (!st) st = alloc_f32(&h->params, h->total);
    if (!st) st = alloc_f32(&h->grads, h->total + kTail);
    if (!st) st = alloc_f32(&h->m, h->total);
    if (!st) st = alloc_f32(&h->v, h->total);
    if (!st) st = alloc_f32(&h->a1, max_batch * d_h1);
    if (!st) st = alloc_f32(&h->a2, max_batch * d_h2);
    if (!st) st = alloc_f32(&h->ga2, max_batch * d_h2);
    if (!st) st = alloc_f32(&h->ga1, max_batch * d_h1);
    if (!st) st = alloc_f32(&h->logits, max_batch * h->d3p);
    if (!st) st = alloc_f32(&h->gl, max_batch * h->d3p);
    for (int i = 0; i < 3 && !st; i++) st = alloc_f32(&h->col_partials[i], R * widths[i]);
    if (!st) st = alloc_f32(&h->xent_partials, (max_batch + kXentThreads - 1) / kXentThreads);
    if (!st) st = alloc_f32(&h->x_lo, max_batch * d_in);
    if (!st) st = alloc_f32(&h->w1_lo, d_in * d_h1);
    if (!st) st = alloc_f32(&h->w2_lo, d_h1 * d_h2);
    if (!st) st = alloc_f32(&h->a1_lo, max_batch * d_h1);
    if (!st) st = alloc_f32(&h->ga2_lo, max_batch * d_h2);
    if (!st) st = alloc_f32(&h->ga1_lo, max_batch * d_h1);
    if (!st && cudaMalloc((void **)&h->counters, (size_t)n_counters * sizeof(unsigned int)) != cudaSuccess) {
        cudaGetLastError();
        st = set_error(ZPUCUDA_ERR_OUT_OF_MEMORY, "cudaMalloc (mlp counters)");
    }
    if (!st) {
        // zero parameters (padding included), gradients, moments, counters
        const cudaError_t e[] = {cudaMemset(h->params, 0, (size_t)h->total * 4),
                                 cudaMemset(h->grads, 0, (size_t)(h->total + kTail) * 4),
                                 cudaMemset(h->m, 0, (size_t)h->total * 4), cudaMemset(h->v, 0, (size_t)h->total * 4),
                                 cudaMemset(h->counters, 0, (size_t)n_counters * sizeof(unsigned int)),
                                 cudaStreamCreateWithFlags(&h->comm_stream, cudaStreamNonBlocking),
                                 cudaEventCreateWithFlags(&h->ev_a, cudaEventDisableTiming),
                                 cudaEventCreateWithFlags(&h->ev_b, cudaEventDisableTiming),
                                 cudaEventCreateWithFlags(&h->ev_w2, cudaEventDisableTiming),
                                 cudaEventCreateWithFlags(&h->ev_done, cudaEventDisableTiming),
                                 cudaEventCreateWithFlags(&h->ev_w1, cudaEventDisableTiming)};
        for (cudaError_t x : e)
            if (x != cudaSuccess && !st) st = cuda_fail(x, "mlp_create setup");
    }
    if (st) {
        free_mlp(h);
        return st;
    }
    *out = h;
    return ZPUCUDA_OK;
}

extern "C" void zpucuda_mlp_destroy(zpucuda_mlp *h) {
    if (!h) return;
    cudaDeviceSynchronize();
    free_mlp(h);
}

extern "C" int zpucuda_mlp_param_numel(const zpucuda_mlp *h, int i, int64_t *numel) {
    if (!h || !numel || i < 0 || i > 5) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_param_numel");
    *numel = h->rows[i] * h->cols[i];
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_param_offset(const zpucuda_mlp *h, int i, int64_t *offset, int64_t *ld) {
    if (!h || !offset || !ld || i < 0 || i > 5) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_param_offset");
    *offset = h->off[i];
    *ld = h->ld[i];
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_param_count(const zpucuda_mlp *h, int64_t *count) {
    if (!h || !count) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_param_count");
    int64_t n = 0;
    for (int i = 0; i < 6; i++) n += h->rows[i] * h->cols[i];
    *count = n;
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_write(zpucuda_mlp *h, int what, int i, const float *src, int64_t numel, void *stream) {
    if (!h || !src || i < 0 || i > 5 || !array_of(h, what))
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_write: bad handle, array or index");
    if (numel != h->rows[i] * h->cols[i]) return set_error(ZPUCUDA_ERR_SHAPE_MISMATCH, "mlp_write: element count");
    float *dst = array_of(h, what) + h->off[i];
    ZC_TRY(join_exchange(h, resolve_stream(stream)));
    ZC_CUDA(cudaMemcpy2DAsync(dst, (size_t)h->ld[i] * 4, src, (size_t)h->cols[i] * 4, (size_t)h->cols[i] * 4,
                              (size_t)h->rows[i], cudaMemcpyDefault, resolve_stream(stream)));
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_read(const zpucuda_mlp *h, int what, int i, float *dst, int64_t numel, void *stream) {
    if (!h || !dst || i < 0 || i > 5 || !array_of(h, what))
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_read: bad handle, array or index");
    if (numel != h->rows[i] * h->cols[i]) return set_error(ZPUCUDA_ERR_SHAPE_MISMATCH, "mlp_read: element count");
    const float *src = array_of(h, what) + h->off[i];
    ZC_TRY(join_exchange(h, resolve_stream(stream)));
    ZC_CUDA(cudaMemcpy2DAsync(dst, (size_t)h->cols[i] * 4, src, (size_t)h->ld[i] * 4, (size_t)h->cols[i] * 4,
                              (size_t)h->rows[i], cudaMemcpyDefault, resolve_stream(stream)));
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_array(const zpucuda_mlp *h, int what, float **d_ptr, int64_t *n) {
    if (!h || !d_ptr || !n || !array_of(h, what)) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_array");
    if (h->w2_pending) ZC_CUDA(cudaEventSynchronize(h->ev_done));  // the arrays are whole when this returns
    *d_ptr = array_of(h, what);
    *n = h->total;
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_adam_config(zpucuda_mlp *h, double lr, double beta1, double beta2, double eps) {
    if (!h || !(lr >= 0) || !(beta1 >= 0 && beta1 < 1) || !(beta2 >= 0 && beta2 < 1) || !(eps > 0))
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_adam_config: lr >= 0, betas in [0,1), eps > 0");
    std::lock_guard<std::mutex> lk(h->mu);
    h->lr = lr;
    h->beta1 = beta1;
    h->beta2 = beta2;
    h->eps = eps;
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_value_and_grad(zpucuda_mlp *h, const float *d_x, const int64_t *d_labels, int64_t batch,
                                          int64_t global_batch, void *stream) {
    ZC_TRY(check_step_args(h, d_x, d_labels, batch, global_batch));
    std::lock_guard<std::mutex> lk(h->mu);
    return value_and_grad(h, d_x, d_labels, batch, global_batch, false, false, resolve_stream(stream));
}

extern "C" int zpucuda_mlp_allreduce_grads(zpucuda_mlp *h, void *stream) {
    if (!h) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_allreduce_grads: NULL handle");
    if (nccl_world(nullptr) == 1) return ZPUCUDA_OK;
    std::lock_guard<std::mutex> lk(h->mu);
    ZC_TRY(join_exchange(h, resolve_stream(stream)));
    return nccl_allreduce_sum_f32(h->grads, h->total + 1, resolve_stream(stream));
}

extern "C" int zpucuda_mlp_adam_step(zpucuda_mlp *h, void *stream) {
    if (!h) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_adam_step: NULL handle");
    std::lock_guard<std::mutex> lk(h->mu);
    ZC_TRY(join_exchange(h, resolve_stream(stream)));
    return adam_step(h, resolve_stream(stream));
}

extern "C" int zpucuda_mlp_train_step(zpucuda_mlp *h, const float *d_x, const int64_t *d_labels, int64_t batch,
                                      int64_t global_batch, void *stream) {
    ZC_TRY(check_step_args(h, d_x, d_labels, batch, global_batch));
    std::lock_guard<std::mutex> lk(h->mu);
    cudaStream_t s = resolve_stream(stream);
    return value_and_grad(h, d_x, d_labels, batch, global_batch, nccl_world(nullptr) > 1, true, s);
}

extern "C" int zpucuda_mlp_join(zpucuda_mlp *h, void *stream) {
    if (!h) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_join: NULL handle");
    std::lock_guard<std::mutex> lk(h->mu);
    return join_exchange(h, resolve_stream(stream));
}

extern "C" int zpucuda_mlp_loss(const zpucuda_mlp *h, float *dst, void *stream) {
    if (!h || !dst) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_loss: NULL argument");
    ZC_CUDA(cudaMemcpyAsync(dst, h->loss_ptr(), sizeof(float), cudaMemcpyDefault, resolve_stream(stream)));
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_check(zpucuda_mlp *h) {
    if (!h) return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT, "mlp_check: NULL handle");
    unsigned int e = 0;
    ZC_CUDA(cudaMemcpy(&e, h->label_error(), sizeof e, cudaMemcpyDeviceToHost));
    if (e) {
        ZC_CUDA(cudaMemset(h->label_error(), 0, sizeof e));
        return set_error(ZPUCUDA_ERR_INDEX_OUT_OF_RANGE, "a label was outside [0, classes) (nn.oneHot)");
    }
    if (h->xfer) {
        ZC_CUDA(cudaMemcpy(&e, xfer_error(h), sizeof e, cudaMemcpyDeviceToHost));
        if (e) {
            ZC_CUDA(cudaMemset(xfer_error(h), 0, sizeof e));
            return set_error(ZPUCUDA_ERR_TIMEOUT,
                             "a peer's dW2 tiles did not arrive in time (that step's W2 update used a stale gradient shard)");
        }
    }
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_debug_peer_reduce(const float *d_inbox, int world, int64_t n, float *d_out,
                                         const uint64_t *d_flags, uint64_t epoch, uint32_t spin_limit,
                                         uint32_t *d_err, void *stream) {
    if (!d_inbox || !d_out || !d_flags || !d_err || world < 1 || world > kMaxPeers || n < 0 || n % 4 ||
        ((uintptr_t)d_inbox & 15u) || ((uintptr_t)d_out & 15u) || spin_limit == 0)
        return set_error(ZPUCUDA_ERR_INVALID_ARGUMENT,
                         "zpucuda_debug_peer_reduce: NULL pointer, world outside [1, 8], n not a multiple of 4, "
                         "unaligned buffer or zero spin limit");
    const int64_t n4 = n / 4;
    int64_t blocks = (n4 + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > (int64_t)num_sms() * 4) blocks = (int64_t)num_sms() * 4;
    xfer_reduce_kernel<<<(unsigned)blocks, 256, 0, resolve_stream(stream)>>>(
        (const float4 *)d_inbox, world, n4, (float4 *)d_out, (const unsigned long long *)d_flags,
        (unsigned long long)epoch, d_err, spin_limit);
    ZC_LAUNCHED("xfer_reduce_kernel");
    return ZPUCUDA_OK;
}

extern "C" int64_t zpucuda_mlp_steps(const zpucuda_mlp *h) { return h ? h->t : -1; }

extern "C" int zpucuda_mlp_exchange_mode(const zpucuda_mlp *h) { return h && h->peer_state == 1 ? 1 : 0; }

extern "C" int zpucuda_mlp_trace(zpucuda_mlp *h, int on) {
    ZC_CHECK(h, ZPUCUDA_ERR_INVALID_ARGUMENT);
    std::lock_guard<std::mutex> g(h->mu);
    if (on)
        for (cudaEvent_t &e : h->tev)
            if (!e) ZC_CUDA(cudaEventCreate(&e));
    h->trace = on != 0;
    return ZPUCUDA_OK;
}

extern "C" int zpucuda_mlp_trace_read(zpucuda_mlp *h, float *ms, int n) {
    ZC_CHECK(h && ms && n >= 0, ZPUCUDA_ERR_INVALID_ARGUMENT);
    std::lock_guard<std::mutex> g(h->mu);
    ZC_CHECK(h->tev[0], ZPUCUDA_ERR_NOT_SUPPORTED);
    // bounded wait for the traced step's last points (the main stream's end
    // and the all-gather it left on the side stream)
    for (int64_t spins = 0;; spins++) {
        cudaError_t e = cudaEventQuery(h->tev[7]);
        if (e == cudaSuccess && h->w2_pending) e = cudaEventQuery(h->ev_done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(e, "cudaEventQuery");
        if (spins > 60LL * 1000 * 100) return set_error(ZPUCUDA_ERR_TIMEOUT, "zpucuda_mlp_trace_read: step did not end");
        std::this_thread::sleep_for(std::chrono::microseconds(10));
    }
    for (int i = 0; i < n && i < kTracePoints; i++) {
        float t = -1.0f;  // -1: the point was not recorded in the traced step
        if (i == 0) t = 0.0f;
        else if (cudaEventElapsedTime(&t, h->tev[0], h->tev[i]) != cudaSuccess) {
            cudaGetLastError();
            t = -1.0f;
        }
        ms[i] = t;
    }
    return ZPUCUDA_OK;
}
