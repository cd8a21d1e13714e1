/*
 * zpucuda.h -- C ABI of libzpucuda.so, the B200 (sm_100a) execution layer for
 * zpu's data-parallel hot path: ops.matmul (f32 / f64, batched / vmapped),
 * the elementwise + reduction regions of a jit plan, and the MLP train step.
 *
 * Conventions
 *  - Every entry point returns an int status (ZPUCUDA_OK == 0).  Codes 1..12
 *    are the members of zpu's tensor.Error in declaration order
 *    (src/zpu/tensor.zig:58-71); codes 13.. are device-side failures.
 *  - Pointers named `d_*` or documented as device pointers are HBM addresses
 *    (from zpucuda_buf_devptr, cudaMalloc, or any allocator on the same
 *    device).  Sizes and strides are in ELEMENTS unless named *_bytes.
 *  - `stream` is a cudaStream_t passed as void*; NULL means the calling
 *    thread's bound stream (zpucuda_thread_bind), mirroring zpu's threadlocal
 *    context (src/zpu/context.zig:34-58).  To run on the legacy default
 *    stream pass cudaStreamLegacy ((void*)0x1).  Calls are asynchronous with respect
 *    to the host unless documented otherwise; zpucuda_sync waits, bounded.
 *  - No entry point falls back to a CPU implementation: an unsupported case
 *    returns ZPUCUDA_ERR_NOT_SUPPORTED and computes nothing.
 */
#ifndef ZPUCUDA_H
#define ZPUCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
enum {
    ZPUCUDA_OK = 0,
    ZPUCUDA_ERR_OUT_OF_MEMORY = 1,       /* tensor.Error.OutOfMemory */
    ZPUCUDA_ERR_SHAPE_MISMATCH = 2,      /* tensor.Error.ShapeMismatch */
    ZPUCUDA_ERR_DTYPE_MISMATCH = 3,      /* tensor.Error.DTypeMismatch */
    ZPUCUDA_ERR_RANK_TOO_LARGE = 4,      /* tensor.Error.RankTooLarge */
    ZPUCUDA_ERR_INVALID_SHAPE = 5,       /* tensor.Error.InvalidShape */
    ZPUCUDA_ERR_INVALID_AXIS = 6,        /* tensor.Error.InvalidAxis */
    ZPUCUDA_ERR_NON_CONTIGUOUS = 7,      /* tensor.Error.NonContiguous */
    ZPUCUDA_ERR_INDEX_OUT_OF_RANGE = 8,  /* tensor.Error.IndexOutOfRange */
    ZPUCUDA_ERR_NOT_SUPPORTED = 9,       /* tensor.Error.NotSupported */
    ZPUCUDA_ERR_NOT_DIFFERENTIABLE = 10, /* tensor.Error.NotDifferentiable */
    ZPUCUDA_ERR_NOT_POSITIVE_DEFINITE = 11,
    ZPUCUDA_ERR_DEVICE_MISMATCH = 12,    /* tensor.Error.DeviceMismatch */
    ZPUCUDA_ERR_TIMEOUT = 13,            /* a bounded wait ran out */
    ZPUCUDA_ERR_CUDA = 14,               /* a CUDA runtime/driver call failed */
    ZPUCUDA_ERR_NO_DEVICE = 15,          /* no usable sm_100 device */
    ZPUCUDA_ERR_INVALID_ARGUMENT = 16    /* NULL pointer, negative size, ... */
};

/* Element types: zpu's DType enum order (src/zpu/dtype.zig:4-13).  GEMM
 * and the RNG take F64 / F32; plans take F64 / F32 / BOOL values (predicates
 * and any / all give BOOL, argmax / argmin give I64); zpucuda_tensor_copy
 * takes all nine.  BOOL is one byte, 0 or 1. */
enum {
    ZPUCUDA_F64 = 0, ZPUCUDA_F32 = 1, ZPUCUDA_F16 = 2, ZPUCUDA_I64 = 3, ZPUCUDA_I32 = 4,
    ZPUCUDA_I16 = 5, ZPUCUDA_I8 = 6, ZPUCUDA_U8 = 7, ZPUCUDA_BOOL = 8
};

/* prims.AXIS_NONE (src/zpu/prims.zig:169). */
#define ZPUCUDA_AXIS_NONE (-2)
/* shape.MAX_RANK (src/zpu/prims.zig:5). */
#define ZPUCUDA_MAX_RANK 8

const char *zpucuda_status_string(int status);
/* Text of the last CUDA error seen by this thread (for ZPUCUDA_ERR_CUDA). */
const char *zpucuda_last_error(void);
/* Library version: major * 10000 + minor * 100 + patch. */
int zpucuda_version(void);

/* ------------------------------------------------------ device / context */
/* Replaces zpu.init's per-thread context set-up (src/zpu/context.zig:74-78):
 * selects `device` for the calling thread and creates its stream. */
int zpucuda_device_count(int *count);
int zpucuda_init(int device);
int zpucuda_thread_bind(int device);
/* The calling thread's stream (cudaStream_t). */
int zpucuda_get_stream(void **stream);
/* Make `stream` (a caller-owned cudaStream_t) the thread's stream; NULL
 * restores the library-created one. */
int zpucuda_set_stream(void *stream);
/* Waits for the thread's stream for at most timeout_ms (<0: the library's
 * default of 60 s); ZPUCUDA_ERR_TIMEOUT when it does not drain in time. */
int zpucuda_sync(int64_t timeout_ms);
/* Number of kernels this library has launched from the calling process. */
uint64_t zpucuda_launch_count(void);
/* Reads the device error word the kernels' bounded waits set when they run
 * out (synchronous): ZPUCUDA_ERR_TIMEOUT if any did, else ZPUCUDA_OK.  The
 * word is sticky for the process. */
int zpucuda_check_device(void);

/* --------------------------------------------------------------- buffers */
/* Refcounted HBM storage: the device counterpart of zpu's Buffer
 * (src/zpu/buffer.zig:14-102): create / retain / release with an atomic
 * count, 256-byte aligned, freed when the count reaches zero. */
typedef struct zpucuda_buf zpucuda_buf;
int zpucuda_buf_alloc(size_t nbytes, zpucuda_buf **out);         /* Buffer.create */
int zpucuda_buf_alloc_zeroed(size_t nbytes, zpucuda_buf **out);  /* Buffer.createZeroed */
/* Non-owning wrapper of caller memory (Buffer.wrapConst): release never frees it. */
int zpucuda_buf_wrap(void *d_ptr, size_t nbytes, zpucuda_buf **out);
zpucuda_buf *zpucuda_buf_retain(zpucuda_buf *b);                 /* Buffer.retain */
void zpucuda_buf_release(zpucuda_buf *b);                        /* Buffer.release */
uint32_t zpucuda_buf_refcount(const zpucuda_buf *b);
void *zpucuda_buf_devptr(const zpucuda_buf *b);
size_t zpucuda_buf_bytes(const zpucuda_buf *b);                  /* Buffer.byteLen */
/* Host <-> HBM copies on the thread's stream; both wait for completion. */
int zpucuda_buf_upload(zpucuda_buf *b, size_t off_bytes, const void *host, size_t nbytes);
int zpucuda_buf_download(const zpucuda_buf *b, size_t off_bytes, void *host, size_t nbytes);

/* ------------------------------------------------------------ residency */
/* A zpu Buffer whose bytes also live in HBM keeps two copies: the host one
 * its accessors read and write in place (Buffer.mem and Tensor's data /
 * readF64 / writeF64, src/zpu/buffer.zig:14-24, src/zpu/tensor.zig:263-302)
 * and the zpucuda_buf.  The residency state says which copy is current, so
 * that a chain of device ops (matmul -> jit plan -> matmul) moves no bytes
 * over PCIe until the host reads a result:
 *   DEVICE: only the HBM copy is current (a device op wrote it last);
 *   HOST:   only the host copy is current (host code wrote it last);
 *   BOTH:   the two agree.
 * A buffer starts DEVICE.  attach_host: the host copy of b->bytes bytes
 * (stays owned by the caller) and the state to start in.  mark_device_dirty:
 * after a device op wrote the buffer.  mark_host_dirty: after host code wrote
 * the host copy.  host_sync: makes the host copy current before a host read
 * (a device-to-host copy when the state is DEVICE, none otherwise; waits,
 * bounded); device_sync: makes the HBM copy current before a device op
 * reads it (a host-to-device copy on `stream` when the state is HOST, none
 * otherwise).  Both leave BOTH.  transfer_stats: bytes these calls and
 * zpucuda_buf_upload / _download copied since the process started. */
enum { ZPUCUDA_RES_DEVICE = 1, ZPUCUDA_RES_HOST = 2, ZPUCUDA_RES_BOTH = 3 };
int zpucuda_buf_attach_host(zpucuda_buf *b, void *host, int state);
int zpucuda_buf_residency(const zpucuda_buf *b, int *state);
int zpucuda_buf_mark_device_dirty(zpucuda_buf *b);
int zpucuda_buf_mark_host_dirty(zpucuda_buf *b);
int zpucuda_buf_host_sync(zpucuda_buf *b, void *stream);
int zpucuda_buf_device_sync(zpucuda_buf *b, void *stream);
int zpucuda_buf_transfer_stats(uint64_t *h2d_bytes, uint64_t *d2h_bytes);

/* Scopes: zpu's Tracker / Scope (src/zpu/tensor.zig:537-664) for device
 * buffers.  scope_begin installs the scope on the calling thread when no
 * other scope is installed there (Tracker.begin; otherwise the new scope
 * stays inert and buffers go to the installed one); every buffer the thread
 * then creates (zpucuda_buf_alloc / _alloc_zeroed / _wrap) is adopted: the
 * scope owns its creation reference.  scope_keep adds a reference so the
 * buffer survives the scope (Tracker.keep); scope_forget hands the creation
 * reference back to the caller (untrack); scope_end releases every adopted
 * buffer still listed, uninstalls the scope and frees it (Scope.deinit).
 * scope_count: buffers listed; scope_installed: 1 when installed. */
typedef struct zpucuda_scope zpucuda_scope;
int zpucuda_scope_begin(zpucuda_scope **out);
int zpucuda_scope_end(zpucuda_scope *scope);
zpucuda_buf *zpucuda_scope_keep(zpucuda_scope *scope, zpucuda_buf *b);
int zpucuda_scope_forget(zpucuda_scope *scope, zpucuda_buf *b);
int64_t zpucuda_scope_count(const zpucuda_scope *scope);
int zpucuda_scope_installed(const zpucuda_scope *scope);

/* ------------------------------------------------------------------ GEMM */
/* C[b] = op(A[b]) @ op(B[b]) for b in 0..batch, row-major, written (not
 * accumulated) -- kernels.gemm / kernels.gemmBatch (src/zpu/kernels.zig:339,
 * :417) and ops.gemmTyped / ops.gemmBatched (src/zpu/ops.zig:1016, :1226).
 *   op(A) is [m,k]: transA == 0 reads A as [m,k] (lda >= k), transA != 0
 *   reads A as [k,m] (lda >= m) -- the swapLastTwo view the matmul VJP passes
 *   (src/zpu/autodiff.zig:480-487), consumed without a toContiguous copy.
 *   op(B) is [k,n]: transB == 0 reads [k,n] (ldb >= n), else [n,k] (ldb >= k).
 *   stride_a / stride_b: elements between consecutive batch matrices, 0 to
 *   broadcast one matrix over the batch (ops.zig:1143-1171); stride_c >= m*ldc.
 * f32 runs on tcgen05 tensor cores with a 3xTF32 split (relative Frobenius
 * error <= 1e-5 against zpu's f32 FMA chain); f64 on the FP64 DMMA path. */
int zpucuda_gemm_f32(const float *d_a, const float *d_b, float *d_c,
                     int64_t m, int64_t n, int64_t k,
                     int64_t lda, int64_t ldb, int64_t ldc,
                     int trans_a, int trans_b,
                     int64_t batch, int64_t stride_a, int64_t stride_b, int64_t stride_c,
                     void *stream);
int zpucuda_gemm_f64(const double *d_a, const double *d_b, double *d_c,
                     int64_t m, int64_t n, int64_t k,
                     int64_t lda, int64_t ldb, int64_t ldc,
                     int trans_a, int trans_b,
                     int64_t batch, int64_t stride_a, int64_t stride_b, int64_t stride_c,
                     void *stream);

/* A strided tensor view as zpu's Tensor holds it (src/zpu/tensor.zig:79-89),
 * with the data pointer already advanced by `offset` elements. */
typedef struct zpucuda_tensor {
    void *data;
    int32_t dtype;
    int32_t rank;
    int64_t dims[ZPUCUDA_MAX_RANK];
    int64_t strides[ZPUCUDA_MAX_RANK]; /* elements; 0 = broadcast */
    int32_t batch_depth;               /* vmap axes leading the shape */
} zpucuda_tensor;

/* ops.matmul (src/zpu/ops.zig:1062-1205): NumPy semantics on the last two
 * axes, right-aligned broadcast of payload batch axes, leading vmap axes
 * (batch_depth) carried through, 1-D promotion and squeeze.
 * zpucuda_matmul_shape fills `out` (dims, rank, batch_depth, contiguous
 * strides; data untouched).  zpucuda_matmul computes into out->data, which
 * must be a contiguous buffer of that shape.  Each operand's last two axes
 * must be row-major or transposed (unit stride on one of them); anything else
 * returns ZPUCUDA_ERR_NON_CONTIGUOUS and the caller materialises it. */
int zpucuda_matmul_shape(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out);
/* Tensor.clone, Tensor.toContiguous and ops.cast on HBM
 * (src/zpu/tensor.zig:356-361,395-404, src/zpu/ops.zig:2062-2071): writes
 * the elements of the view `src` in logical (row-major) order into the
 * contiguous buffer dst->data of type dst->dtype, each as zpu's
 * writeF64(readLogical) does -- widened to f64, then narrowed: floats round
 * to nearest; integer types take 0 for NaN, else clamp to their range and
 * truncate toward zero (i64 saturates at 2^63, where zpu is undefined);
 * BOOL is v != 0.  src may have any strides (negative from flip, 0 from
 * broadcast); dst must have src's dims and must not overlap it; its strides
 * are set to the contiguous ones.  clone: dst->dtype == src->dtype;
 * toContiguous: the same, called only for a non-contiguous src (zpu returns
 * a contiguous tensor itself); cast: another dtype (zpu returns the input
 * for an equal one). */
int zpucuda_tensor_copy(const zpucuda_tensor *src, zpucuda_tensor *dst, void *stream);
int zpucuda_matmul(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out,
                   void *stream);

/* --------------------------------------------------------------- jit plan */
/* A value of a jit trace: an argument, a folded constant or a step output,
 * identified as in zpu (Tensor.id, src/zpu/tensor.zig:88). */
typedef struct zpucuda_value {
    uint64_t id;
    int32_t dtype;
    int32_t rank;
    int64_t dims[ZPUCUDA_MAX_RANK];
    int32_t batch_depth;
} zpucuda_value;

/* jit.Step (src/zpu/jit.zig:30-36) with the Attrs fields reductions use. */
typedef struct zpucuda_step {
    int32_t prim;     /* prims.Prim code (src/zpu/prims.zig:9-109) */
    int32_t n_inputs;
    uint64_t ins[3];
    uint64_t out;
    int32_t axis;     /* Attrs.axis, ZPUCUDA_AXIS_NONE for a full reduction */
    int32_t flags;    /* Attrs.flags: bit 0 KEEP_DIMS (reductions), bit 5 REVERSE (cumsum) */
    /* reshape / broadcast: Attrs.shape[0 .. shape_len) (-1: the one dimension
     * reshape infers); transpose: Attrs.perm[0 .. nsl) */
    int64_t shape[ZPUCUDA_MAX_RANK];
    int32_t shape_len;
    int32_t nsl;
    uint8_t perm[ZPUCUDA_MAX_RANK];
    /* slice: Attrs.starts / Attrs.lens (in `shape`) / Attrs.steps [0 .. nsl),
     * the ranges sliceAttrs records (resolved: element j of axis i is
     * starts[i] + j * steps[i], j < lens[i]) */
    int64_t starts[ZPUCUDA_MAX_RANK];
    int64_t steps[ZPUCUDA_MAX_RANK];
    /* pad: Attrs.pads_lo (in `starts`) / Attrs.pads_hi [0 .. nsl) and the
     * fill value Attrs.scalar */
    int64_t pads_hi[ZPUCUDA_MAX_RANK];
    double scalar;
} zpucuda_step;

/* jit.Blob (src/zpu/jit.zig:39-42): a constant folded at build time; its
 * host data is copied into HBM when the plan is created. */
typedef struct zpucuda_blob {
    zpucuda_value value;
    const void *host_data;
} zpucuda_blob;

typedef struct zpucuda_plan zpucuda_plan;

/* Lowers a built jit plan (the output of jit.build, src/zpu/jit.zig:130-256):
 * maximal runs of element-wise steps (prims.isElementwise,
 * src/zpu/prims.zig:198) that end in at most one sum / prod / max / min over
 * all axes or over any one axis (keepdims or not), or one argmax / argmin
 * (i64 result, ops.argReduce, src/zpu/ops.zig:931-975), or one any / all
 * (BOOL result) become ONE fused
 * kernel each (no intermediate HBM traffic).  Reduction axes follow
 * ops.axesMaskOf (ops.zig:630-642): with batch_depth d, AXIS_NONE folds the
 * payload axes [d, rank) and a non-negative axis counts from axis d.  Matmul
 * steps become GEMM launches; cumsum steps (ops.cumsum, src/zpu/ops.zig:
 * 2032-2060: f64 running sum along one axis, rounded per element) a scan
 * launch each; concat / stack / pad / take / scatter_add (ops.zig:1665-1797,
 * 1995-2017) copy, fill, gather and scatter launches.  reshape / transpose /
 * broadcast / expand_dims / squeeze / slice / flip (ops.zig:1343-1635,
 * 2019-2030) are views -- new strides over the same HBM, no launch
 * -- that region loads and GEMM operands read in place; a view is copied
 * (zpucuda_tensor_copy's kernels) only where a contiguous buffer is needed:
 * a plan output, a cumsum input, a reshape of a non-contiguous view, a GEMM
 * operand whose last two axes have no unit stride.  Region kernels come from
 * a catalogue generated at build time, with a one-pass bytecode kernel for
 * regions outside it.  Steps outside that set make creation fail with
 * ZPUCUDA_ERR_NOT_SUPPORTED. */
int zpucuda_plan_create(const zpucuda_value *args, int n_args,
                        const zpucuda_blob *blobs, int n_blobs,
                        const zpucuda_step *steps, int n_steps,
                        const uint64_t *out_ids, int n_outs,
                        zpucuda_plan **out);
/* jit.Plan.runAll (src/zpu/jit.zig:99-126): `args[i]` are device pointers
 * to contiguous argument data, `outs[i]` device pointers to contiguous
 * output buffers (shapes from zpucuda_plan_output). */
int zpucuda_plan_run(zpucuda_plan *plan, const void *const *args, void *const *outs, void *stream);
/* The same call for HOST-resident tensors, i.e. Jit.call on zpu tensors
 * whose Buffer lives in host memory (src/zpu/transforms.zig:408-411): copies
 * each argument to HBM staging owned by the plan, runs, copies the outputs
 * back and waits (bounded) for the stream.  Pinned host memory gives full
 * copy bandwidth; pageable memory works at the driver's staging speed. */
int zpucuda_plan_run_host(zpucuda_plan *plan, const void *const *host_args, void *const *host_outs,
                          void *stream);
int zpucuda_plan_output(const zpucuda_plan *plan, int i, zpucuda_value *value);
/* Device-side errors of the plan's launches since the last check: waits for
 * the stream (bounded), then returns ZPUCUDA_ERR_TIMEOUT once when a fused
 * reduction's bounded wait for its input copies ran out (that result is
 * NaN), else ZPUCUDA_ERR_INDEX_OUT_OF_RANGE once for a take / scatter_add
 * index out of range (zpu's IndexOutOfRange, ops.zig:1735-1741), else
 * ZPUCUDA_OK; both flags are cleared.  zpucuda_plan_run_host checks by
 * itself. */
int zpucuda_plan_check(zpucuda_plan *plan, void *stream);
int zpucuda_plan_num_steps(const zpucuda_plan *plan);   /* jit.Plan.numSteps */
int zpucuda_plan_num_kernels(const zpucuda_plan *plan); /* launches per run */
/* Plan.describe (src/zpu/jit.zig:71-83) plus the lowering: one line per
 * kernel.  Writes at most `len` bytes including the terminating NUL. */
int zpucuda_plan_describe(const zpucuda_plan *plan, char *buf, size_t len);
void zpucuda_plan_destroy(zpucuda_plan *plan);

/* ------------------------------------------------------------------- rng */
/* rng.Rng (src/zpu/rng.zig:15-102) on the device: the same splitmix64 stream
 * as Rng.init(seed) drawn sequentially (state after i draws = seed + i*gamma,
 * so every element is generated independently).  uniform: Rng.uniformRange;
 * normal: Rng.normal (Box-Muller pairs); randint: Rng.randint (int64). */
int zpucuda_rng_uniform(uint64_t seed, int dtype, void *d_out, int64_t n, double lo, double hi, void *stream);
int zpucuda_rng_normal(uint64_t seed, int dtype, void *d_out, int64_t n, void *stream);
int zpucuda_rng_randint(uint64_t seed, int64_t *d_out, int64_t n, int64_t lo, int64_t hi, void *stream);

/* ------------------------------------------------------------ collectives */
/* No counterpart in the reference (it runs on one CPU): the gradient
 * exchange of the data-parallel MLP step, one process (or thread) per GPU,
 * NCCL over NVLink.  libnccl.so.2 is opened at run time on first use; without
 * it these calls return ZPUCUDA_ERR_NOT_SUPPORTED.  The communicator belongs
 * to the calling thread's bound device.
 *  zpucuda_nccl_unique_id: rank 0 creates the id (ncclGetUniqueId) and hands
 *    the 128 bytes to the other ranks by any host channel.
 *  zpucuda_nccl_init: joins; returns ZPUCUDA_ERR_TIMEOUT (and tears the
 *    half-made communicator down) when not every rank joined within
 *    timeout_ms (< 0: no limit).
 *  zpucuda_nccl_allreduce_f32: in-place sum of count floats on `stream`.
 *  zpucuda_nccl_world: rank and world size (0 and 1 without a communicator).
 *  zpucuda_nccl_destroy: finalizes (bounded by timeout_ms) and frees it. */
#define ZPUCUDA_NCCL_ID_BYTES 128
int zpucuda_nccl_unique_id(uint8_t *id);
int zpucuda_nccl_init(int rank, int world, const uint8_t *id, int64_t timeout_ms);
int zpucuda_nccl_allreduce_f32(float *d_buf, int64_t count, void *stream);
int zpucuda_nccl_world(int *rank, int *world);
int zpucuda_nccl_destroy(int64_t timeout_ms);

/* ---------------------------------------------------------- MLP train step */
/* The MLP step as a device-resident program: x -> tanh(x W1 + b1) ->
 * tanh(. W2 + b2) -> . W3 + b3 = logits, loss = nn.sparseCrossEntropy(logits,
 * labels) (src/zpu/nn.zig:123-134,190-194), its gradients as
 * zpu.valueAndGrad computes them (src/zpu/transforms.zig:87-148,
 * src/zpu/autodiff.zig:51,323-330,451-454,480-487), and Adam.step with f32
 * moments (src/zpu/optim.zig:149-259), lowered to 14 kernels per step
 * (2 of them, the Adam updates, on a side stream), plus one split pass per
 * large operand (x, W1, W2) where the products read presplit lo halves.
 * Parameters are numbered in the reference's argument order: 0 W1 [d_in,d_h1],
 * 1 b1 [d_h1], 2 W2 [d_h1,d_h2], 3 b2 [d_h2], 4 W3 [d_h2,d_out], 5 b3 [d_out],
 * row-major as the reference stores them; the handle owns the parameters,
 * gradients and Adam moments in HBM (all zero after create).
 *  create: max_batch bounds the rows of one call; d_out <= 64.
 *  write / read: copy parameter i of the array `what` (ZPUCUDA_MLP_*) from /
 *    to any host or device pointer (numel = the parameter's element count),
 *    asynchronously on `stream`.
 *  array: the device address and length (floats, padding included) of a
 *    whole array -- for callers that exchange it themselves; param_offset:
 *    where parameter i starts in it and its row pitch (floats).
 *  adam_config: Adam's lr, beta1, beta2, eps (defaults 1e-3, 0.9, 0.999,
 *    1e-8: optim.AdamConfig); weight decay is not supported.
 *  value_and_grad: gradients of the loss over d_x [batch, d_in] f32 (16-byte
 *    aligned) and d_labels [batch] int64, the loss averaged over
 *    global_batch rows (= batch on one GPU; the sum over ranks of each
 *    rank's slice otherwise).  Gradients land in the GRAD array, the loss in
 *    a device word read by zpucuda_mlp_loss.
 *  allreduce_grads: sums the GRAD array and the loss over the device's NCCL
 *    communicator (no-op without one).
 *  adam_step: one Adam.step with the GRAD array (step counter inside).
 *  train_step: value_and_grad, the gradient exchange when the device has a
 *    communicator (two buckets on a side stream, overlapping the last
 *    backward GEMMs), and one Adam.step.  With a communicator each bucket is
 *    reduce-scattered, every rank updates its 1/world shard and the
 *    parameters are all-gathered, so afterwards the parameters are complete
 *    on every rank but the GRAD and ADAM_M/V arrays only in the rank's own
 *    shards.
 *  loss: copies the last loss (f32) to dst (host or device) on `stream`.
 *  check: synchronous; ZPUCUDA_ERR_INDEX_OUT_OF_RANGE when a label of an
 *    earlier step was outside [0, d_out) (nn.oneHot's error; that row's
 *    one-hot row was zero), and clears the flag; ZPUCUDA_ERR_TIMEOUT when a
 *    peer's dW2 tiles did not arrive within the exchange's bounded wait
 *    (that step's W2 update then used the previous step's gradient shard:
 *    the parameters are stale and the run should be restarted from a saved
 *    state), and clears that flag too.
 *  steps: Adam steps taken. */
typedef struct zpucuda_mlp zpucuda_mlp;
enum { ZPUCUDA_MLP_PARAM = 0, ZPUCUDA_MLP_GRAD = 1, ZPUCUDA_MLP_ADAM_M = 2, ZPUCUDA_MLP_ADAM_V = 3 };
int zpucuda_mlp_create(int64_t d_in, int64_t d_h1, int64_t d_h2, int64_t d_out, int64_t max_batch,
                       zpucuda_mlp **out);
void zpucuda_mlp_destroy(zpucuda_mlp *h);
int zpucuda_mlp_param_numel(const zpucuda_mlp *h, int i, int64_t *numel);
int zpucuda_mlp_param_count(const zpucuda_mlp *h, int64_t *count);
int zpucuda_mlp_write(zpucuda_mlp *h, int what, int i, const float *src, int64_t numel, void *stream);
int zpucuda_mlp_read(const zpucuda_mlp *h, int what, int i, float *dst, int64_t numel, void *stream);
int zpucuda_mlp_array(const zpucuda_mlp *h, int what, float **d_ptr, int64_t *n);
int zpucuda_mlp_param_offset(const zpucuda_mlp *h, int i, int64_t *offset, int64_t *ld);
int zpucuda_mlp_adam_config(zpucuda_mlp *h, double lr, double beta1, double beta2, double eps);
int zpucuda_mlp_value_and_grad(zpucuda_mlp *h, const float *d_x, const int64_t *d_labels, int64_t batch,
                               int64_t global_batch, void *stream);
int zpucuda_mlp_allreduce_grads(zpucuda_mlp *h, void *stream);
int zpucuda_mlp_adam_step(zpucuda_mlp *h, void *stream);
int zpucuda_mlp_train_step(zpucuda_mlp *h, const float *d_x, const int64_t *d_labels, int64_t batch,
                           int64_t global_batch, void *stream);
int zpucuda_mlp_loss(const zpucuda_mlp *h, float *dst, void *stream);
/* A data-parallel train step returns (its stream's work ends) once W1 and b1
 * are whole; the all-gather of the larger bucket [W2 .. b3] runs on into the
 * next step, which waits for it only before it reads W2.  Every call that
 * touches the arrays (read, write, array, the next step) waits for it
 * itself; zpucuda_mlp_join makes `stream` wait for it, for callers that time
 * a sequence of steps or read the parameters by pointer.  No counterpart in
 * the reference (one CPU, no exchange). */
int zpucuda_mlp_join(zpucuda_mlp *h, void *stream);
int zpucuda_mlp_check(zpucuda_mlp *h);
int64_t zpucuda_mlp_steps(const zpucuda_mlp *h);
/* 1 when train_step exchanges dW2 over peer memory (its GEMM stores each
 * tile into the owning rank's inbox across NVLink, set up through CUDA IPC at
 * the first data-parallel step), 0 when every gradient goes through NCCL.
 * By default it is used from 6 ranks on (below that NCCL's reduce-scatter
 * hides under the next GEMM); ZPUCUDA_MLP_PEER_EXCHANGE=1 / =0, set alike on
 * every rank, forces it on / off. */
int zpucuda_mlp_exchange_mode(const zpucuda_mlp *h);
/* Phase trace of the step (diagnostics): with tracing on, each
 * value_and_grad / train_step records timing events at its phase boundaries;
 * zpucuda_mlp_trace_read waits (bounded) for the last traced step and writes
 * up to 13 times in ms from its start: [0] start, [1] forward GEMMs, [2]
 * loss, [3] layer-3 backward + db2, [4] dW2 GEMM, [5] g1 GEMM, [6] db1 + dW1
 * GEMM, [7] end (main stream); [8] bucket [W2 ..] summed, [9] its Adam,
 * [10] bucket [W1, b1] summed, [11] its Adam and all-gather, [12] the
 * all-gather of bucket [W2 ..] (side stream; -1 where a point was not
 * reached, e.g. on one rank). */
int zpucuda_mlp_trace(zpucuda_mlp *h, int on);
int zpucuda_mlp_trace_read(zpucuda_mlp *h, float *ms, int n);
/* Diagnostics, no counterpart in the reference: runs the owner-side step of
 * the peer-memory dW2 exchange -- wait until every flag d_flags[0 .. world)
 * holds at least `epoch`, then d_out[i] = sum over s in rank order of
 * d_inbox[s * n + i] -- on caller buffers (n a multiple of 4, d_inbox and
 * d_out 16-byte aligned).  The wait polls at most spin_limit times, about
 * 256 ns apart; when it runs out the kernel sets *d_err to 1, writes nothing
 * and returns, which is what zpucuda_mlp_check then reports as
 * ZPUCUDA_ERR_TIMEOUT.  Lets a test make that bounded wait run out without a
 * second GPU. */
int zpucuda_debug_peer_reduce(const float *d_inbox, int world, int64_t n, float *d_out, const uint64_t *d_flags,
                              uint64_t epoch, uint32_t spin_limit, uint32_t *d_err, void *stream);

/* ------------------------------------------------- allocation-free variant */
/* No counterpart in the reference: an addition for callers that cannot
 * allocate device memory -- an application embedding this library inside a
 * framework whose caching allocator owns the device (a side cudaMalloc would
 * escape its accounting and limits), or a latency-critical loop where
 * cudaMalloc's implicit synchronisation is not allowed.
 * *d_out = sumAll(tanh(x*x) * a + b) over the n f32 elements at d_x (16-byte
 * aligned), a = *d_a, b = *d_b (device scalars): the same fused kernel and
 * result as the plan of that jit chain, but its reduction scratch lives in a
 * static 16.25 KiB device array inside the library (held by every GPU that
 * loads it until exit), so the call allocates nothing.
 *  - The first call on a device looks the array's address up
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - Every call shares the one array: calls that overlap on the GPU (other
 *    streams, other threads) race and corrupt each other's result; order
 *    them on one stream.  Each call zeroes the counters it needs.
 *  - Launches whose grid needs more block partials than the array holds
 *    (2048) are rejected with ZPUCUDA_ERR_NOT_SUPPORTED and a message. */
int zpucuda_chain_tanh_sq_affine_sum_noalloc(const float *d_x, int64_t n, const float *d_a, const float *d_b,
                                             float *d_out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* ZPUCUDA_H */
