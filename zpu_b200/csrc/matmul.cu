// ops.matmul on the device: the shape logic of src/zpu/ops.zig:1062-1205
// (vmap depth alignment, 1-D promotion, right-aligned broadcast of payload
// batch axes, squeeze) restated over strided views, then one batched GEMM
// launch.  Transposed operands (the swapLastTwo views of the matmul VJP,
// src/zpu/autodiff.zig:480-487) are read in place, never materialised.
#include <string.h>

#include <algorithm>

#include "gemm.cuh"

namespace zc {

namespace {

struct View {
    int rank;
    int64_t dims[ZPUCUDA_MAX_RANK];
    int64_t strides[ZPUCUDA_MAX_RANK];
    int depth;
};

View view_of(const zpucuda_tensor *t) {
    View v;
    v.rank = t->rank;
    v.depth = t->batch_depth;
    bool empty = false;
    for (int i = 0; i < ZPUCUDA_MAX_RANK; i++) {
        v.dims[i] = i < t->rank ? t->dims[i] : 0;
        v.strides[i] = i < t->rank ? t->strides[i] : 0;
        if (i < t->rank && t->dims[i] == 0) empty = true;
    }
    if (empty) {  // no element is read: any strides will do, take the row-major ones
        int64_t q = 1;
        for (int i = t->rank - 1; i >= 0; i--) {
            v.strides[i] = q;
            q *= v.dims[i] > 1 ? v.dims[i] : 1;
        }
    }
    return v;
}

// withVmapDepth (ops.zig:1211-1224): lead with size-1, stride-0 axes.
int with_depth(View &v, int depth) {
    if (v.depth >= depth) return ZPUCUDA_OK;
    const int extra = depth - v.depth;
    if (v.rank + extra > ZPUCUDA_MAX_RANK) return ZPUCUDA_ERR_RANK_TOO_LARGE;
    for (int i = v.rank - 1; i >= 0; i--) {
        v.dims[i + extra] = v.dims[i];
        v.strides[i + extra] = v.strides[i];
    }
    for (int i = 0; i < extra; i++) {
        v.dims[i] = 1;
        v.strides[i] = 0;
    }
    v.rank += extra;
    v.depth = depth;
    return ZPUCUDA_OK;
}

// expandDims(t, axis): a size-1 axis with stride 0.
int expand(View &v, int axis) {
    if (v.rank + 1 > ZPUCUDA_MAX_RANK) return ZPUCUDA_ERR_RANK_TOO_LARGE;
    for (int i = v.rank; i > axis; i--) {
        v.dims[i] = v.dims[i - 1];
        v.strides[i] = v.strides[i - 1];
    }
    v.dims[axis] = 1;
    v.strides[axis] = 0;
    v.rank++;
    return ZPUCUDA_OK;
}

struct Plan {
    int32_t out_dtype;  // DType.promote of the operands
    int64_t m, n, k;
    bool ta, tb;
    int64_t lda, ldb;
    GemmBatch batch;
    int out_rank;
    int64_t out_dims[ZPUCUDA_MAX_RANK];
    int out_depth;
};

int plan_matmul(const zpucuda_tensor *ta_, const zpucuda_tensor *tb_, Plan *P) {
    if (!ta_ || !tb_ || !P) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if (ta_->rank == 0 || tb_->rank == 0) return ZPUCUDA_ERR_SHAPE_MISMATCH;
    if (ta_->rank > ZPUCUDA_MAX_RANK || tb_->rank > ZPUCUDA_MAX_RANK) return ZPUCUDA_ERR_RANK_TOO_LARGE;
    if (ta_->dtype < 0 || ta_->dtype > ZPUCUDA_BOOL || tb_->dtype < 0 || tb_->dtype > ZPUCUDA_BOOL)
        return ZPUCUDA_ERR_INVALID_ARGUMENT;
    // binaryOutDType(.mul, a, b) (ops.zig:275-285): a bool result is an error
    P->out_dtype = dtype_promote(ta_->dtype, tb_->dtype);
    if (P->out_dtype == ZPUCUDA_BOOL) return ZPUCUDA_ERR_DTYPE_MISMATCH;
    View a = view_of(ta_), b = view_of(tb_);
    const int depth = std::max(a.depth, b.depth);
    int st;
    if ((st = with_depth(a, depth)) || (st = with_depth(b, depth))) return st;
    const bool prep_a = a.rank - depth == 1;
    const bool prep_b = b.rank - depth == 1;
    if (prep_a && (st = expand(a, depth))) return st;
    if (prep_b && (st = expand(b, b.rank))) return st;
    const int ar = a.rank, br = b.rank;
    const int64_t m = a.dims[ar - 2], k = a.dims[ar - 1], k2 = b.dims[br - 2], n = b.dims[br - 1];
    if (k != k2) return ZPUCUDA_ERR_SHAPE_MISMATCH;
    const int a_nba = ar - 2 - depth, b_nba = br - 2 - depth, nb = std::max(a_nba, b_nba);
    int64_t adims[ZPUCUDA_MAX_RANK], bdims[ZPUCUDA_MAX_RANK], cdims[ZPUCUDA_MAX_RANK];
    for (int i = 0; i < nb; i++) {
        const int ia = i - (nb - a_nba), ib = i - (nb - b_nba);
        adims[i] = ia >= 0 ? a.dims[depth + ia] : 1;
        bdims[i] = ib >= 0 ? b.dims[depth + ib] : 1;
        if (adims[i] == bdims[i] || bdims[i] == 1) cdims[i] = adims[i];
        else if (adims[i] == 1) cdims[i] = bdims[i];
        else return ZPUCUDA_ERR_SHAPE_MISMATCH;
    }
    const int out_rank = nb + 2 + depth;
    if (out_rank > ZPUCUDA_MAX_RANK) return ZPUCUDA_ERR_RANK_TOO_LARGE;
    // batch axes: vmap axes first, then payload batch axes (ops.zig:1140-1171)
    GemmBatch &g = P->batch;
    memset(&g, 0, sizeof g);
    g.nax = depth + nb;
    if (g.nax > kGemmMaxBatchAxes) return ZPUCUDA_ERR_RANK_TOO_LARGE;
    // vmap axes: the lead operand carries them (ops.zig:1114-1116)
    const View &lead = ta_->batch_depth == depth ? a : b;
    for (int i = 0; i < depth; i++) {
        const int64_t dim = std::max(a.dims[i], b.dims[i]);
        (void)lead;
        g.dims[i] = dim;
        g.sa[i] = a.dims[i] == dim ? a.strides[i] : 0;
        g.sb[i] = b.dims[i] == dim ? b.strides[i] : 0;
    }
    for (int i = 0; i < nb; i++) {
        const int ia = i - (nb - a_nba), ib = i - (nb - b_nba);
        g.dims[depth + i] = cdims[i];
        g.sa[depth + i] = (ia >= 0 && adims[i] == cdims[i]) ? a.strides[depth + ia] : 0;
        g.sb[depth + i] = (ib >= 0 && bdims[i] == cdims[i]) ? b.strides[depth + ib] : 0;
    }
    // the matrix axes: row-major or transposed, never another layout
    const int64_t as0 = a.strides[ar - 2], as1 = a.strides[ar - 1];
    const int64_t bs0 = b.strides[br - 2], bs1 = b.strides[br - 1];
    if (as1 == 1 || k == 1) { P->ta = false; P->lda = (m == 1 || as0 == 0) ? std::max<int64_t>(k, 1) : as0; }
    else if (as0 == 1 || m == 1) { P->ta = true; P->lda = k == 1 ? std::max<int64_t>(m, 1) : as1; }
    else return ZPUCUDA_ERR_NON_CONTIGUOUS;
    if (bs1 == 1 || n == 1) { P->tb = false; P->ldb = (k == 1 || bs0 == 0) ? std::max<int64_t>(n, 1) : bs0; }
    else if (bs0 == 1 || k == 1) { P->tb = true; P->ldb = n == 1 ? std::max<int64_t>(k, 1) : bs1; }
    else return ZPUCUDA_ERR_NON_CONTIGUOUS;
    if (!P->ta && P->lda < k) return ZPUCUDA_ERR_NON_CONTIGUOUS;
    if (P->ta && P->lda < m) return ZPUCUDA_ERR_NON_CONTIGUOUS;
    if (!P->tb && P->ldb < n) return ZPUCUDA_ERR_NON_CONTIGUOUS;
    if (P->tb && P->ldb < k) return ZPUCUDA_ERR_NON_CONTIGUOUS;
    P->m = m;
    P->n = n;
    P->k = k;
    // output shape, then the squeezes of the 1-D promotions (ops.zig:1189-1203)
    int64_t od[ZPUCUDA_MAX_RANK];
    for (int i = 0; i < depth; i++) od[i] = g.dims[i];
    for (int i = 0; i < nb; i++) od[depth + i] = cdims[i];
    od[out_rank - 2] = m;
    od[out_rank - 1] = n;
    int r = out_rank;
    if (prep_a) {  // squeeze(-2)
        od[r - 2] = od[r - 1];
        r--;
    }
    if (prep_b) r--;  // squeeze(-1)
    P->out_rank = r;
    for (int i = 0; i < r; i++) P->out_dims[i] = od[i];
    P->out_depth = depth;
    return ZPUCUDA_OK;
}

}  // namespace

static int64_t numel_of(const zpucuda_tensor *t) {
    int64_t q = 1;
    for (int i = 0; i < t->rank; i++) q *= t->dims[i];
    return q;
}

int matmul_device(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out, cudaStream_t s) {
    Plan P;
    int st = plan_matmul(a, b, &P);
    if (st) return st;
    // empty tensors may carry a NULL data pointer (nothing is read or written)
    if (!out || (!out->data && numel_of(out)) || (!a->data && numel_of(a)) || (!b->data && numel_of(b)))
        return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if (out->rank != P.out_rank) return ZPUCUDA_ERR_SHAPE_MISMATCH;
    for (int i = 0; i < P.out_rank; i++)
        if (out->dims[i] != P.out_dims[i]) return ZPUCUDA_ERR_SHAPE_MISMATCH;
    if (out->dtype != P.out_dtype) return ZPUCUDA_ERR_DTYPE_MISMATCH;
    // the output is contiguous: batch after batch of [m, n]
    if (a->dtype != b->dtype || (a->dtype != ZPUCUDA_F32 && a->dtype != ZPUCUDA_F64))
        return gemm_convert_device(a->data, a->dtype, b->data, b->dtype, out->data, out->dtype, P.m, P.n, P.k, P.lda,
                                   P.ldb, P.ta, P.tb, P.batch, P.m * P.n, s);
    if (a->dtype == ZPUCUDA_F32)
        return gemm_f32_device((const float *)a->data, (const float *)b->data, (float *)out->data, P.m, P.n, P.k,
                               P.lda, P.ldb, P.n, P.ta, P.tb, P.batch, P.m * P.n, s);
    return gemm_f64_device((const double *)a->data, (const double *)b->data, (double *)out->data, P.m, P.n, P.k,
                           P.lda, P.ldb, P.n, P.ta, P.tb, P.batch, P.m * P.n, s);
}

// The same product with an epilogue on each element (f32, one matrix: the
// GEMM's epilogues belong to one matrix) -- the jit lowering's matmul + bias
// [+ tanh] fusion.
int matmul_device_epi(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out, const Epilogue &epi,
                      cudaStream_t s) {
    Plan P;
    int st = plan_matmul(a, b, &P);
    if (st) return st;
    if (!out || !out->data || !a->data || !b->data) return ZPUCUDA_ERR_INVALID_ARGUMENT;
    if (a->dtype != ZPUCUDA_F32 || b->dtype != ZPUCUDA_F32 || out->dtype != ZPUCUDA_F32 || batch_count(P.batch) != 1)
        return ZPUCUDA_ERR_NOT_SUPPORTED;
    if (out->rank != P.out_rank) return ZPUCUDA_ERR_SHAPE_MISMATCH;
    for (int i = 0; i < P.out_rank; i++)
        if (out->dims[i] != P.out_dims[i]) return ZPUCUDA_ERR_SHAPE_MISMATCH;
    return gemm_f32_device_epi((const float *)a->data, (const float *)b->data, (float *)out->data, P.m, P.n, P.k,
                               P.lda, P.ldb, P.n, P.ta, P.tb, P.batch, P.m * P.n, epi, s);
}

}  // namespace zc

using namespace zc;

extern "C" {

int zpucuda_matmul_shape(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out) {
    ZC_CHECK(out, ZPUCUDA_ERR_INVALID_ARGUMENT);
    Plan P;
    int st = plan_matmul(a, b, &P);
    if (st) return st;
    void *keep = out->data;
    memset(out, 0, sizeof *out);
    out->data = keep;
    out->dtype = P.out_dtype;
    out->rank = P.out_rank;
    out->batch_depth = P.out_depth;
    int64_t q = 1;
    for (int i = P.out_rank - 1; i >= 0; i--) {
        out->dims[i] = P.out_dims[i];
        out->strides[i] = q;
        q *= P.out_dims[i];
    }
    return ZPUCUDA_OK;
}

int zpucuda_matmul(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out, void *stream) {
    return matmul_device(a, b, out, resolve_stream(stream));
}

int zpucuda_gemm_f32(const float *d_a, const float *d_b, float *d_c, int64_t m, int64_t n, int64_t k, int64_t lda,
                     int64_t ldb, int64_t ldc, int trans_a, int trans_b, int64_t batch, int64_t stride_a,
                     int64_t stride_b, int64_t stride_c, void *stream) {
    ZC_CHECK(m >= 0 && n >= 0 && k >= 0 && batch >= 0, ZPUCUDA_ERR_INVALID_SHAPE);
    GemmBatch g;
    memset(&g, 0, sizeof g);
    g.nax = 1;
    g.dims[0] = batch;
    g.sa[0] = stride_a;
    g.sb[0] = stride_b;
    return gemm_f32_device(d_a, d_b, d_c, m, n, k, lda, ldb, ldc, trans_a != 0, trans_b != 0, g, stride_c,
                           resolve_stream(stream));
}

int zpucuda_gemm_f64(const double *d_a, const double *d_b, double *d_c, int64_t m, int64_t n, int64_t k, int64_t lda,
                     int64_t ldb, int64_t ldc, int trans_a, int trans_b, int64_t batch, int64_t stride_a,
                     int64_t stride_b, int64_t stride_c, void *stream) {
    ZC_CHECK(m >= 0 && n >= 0 && k >= 0 && batch >= 0, ZPUCUDA_ERR_INVALID_SHAPE);
    GemmBatch g;
    memset(&g, 0, sizeof g);
    g.nax = 1;
    g.dims[0] = batch;
    g.sa[0] = stride_a;
    g.sb[0] = stride_b;
    return gemm_f64_device(d_a, d_b, d_c, m, n, k, lda, ldb, ldc, trans_a != 0, trans_b != 0, g, stride_c,
                           resolve_stream(stream));
}

}  // extern "C"
