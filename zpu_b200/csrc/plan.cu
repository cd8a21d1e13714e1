// jit-plan lowering: turns the steps of a built jit.Plan (src/zpu/jit.zig:
// 30-36, 130-256) into a short list of launches and replays that list on
// every run (the device counterpart of Plan.runAll, jit.zig:99-126, which
// interprets one ops.applyPrim per step and materialises every
// intermediate):
//   * one fused kernel per element-wise(+reduction) region; bool values
//     (predicates, any / all) ride in the region's float registers;
//   * one GEMM per matmul step, with a following row-bias add (and tanh)
//     in its epilogue when nothing else reads the intermediates;
//   * movement prims (reshape, transpose, broadcast, expand_dims, squeeze,
//     slice, flip, copy) as views -- strides and an offset over the
//     producer's buffer -- read in place by regions and GEMMs, copied only
//     where a contiguous buffer is needed;
//   * cumsum, cast, concat / stack / pad, take and scatter_add launches.
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "gemm.cuh"
#include "region.cuh"
#include "tensor_ops.cuh"

namespace zc {
int matmul_device(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out, cudaStream_t s);
int matmul_device_epi(const zpucuda_tensor *a, const zpucuda_tensor *b, zpucuda_tensor *out, const Epilogue &epi,
                      cudaStream_t s);
}

using namespace zc;

namespace {

// prims.Prim codes the lowering knows (src/zpu/prims.zig:9-109).
enum {
    PRIM_SUM = 58,
    PRIM_PROD = 59,
    PRIM_MAX_REDUCE = 60,
    PRIM_MIN_REDUCE = 61,
    PRIM_ANY = 62,
    PRIM_ALL = 63,
    PRIM_ARGMAX = 64,
    PRIM_ARGMIN = 65,
    PRIM_LOGICAL_NOT = 54,
    PRIM_WHERE = 55,
    PRIM_RESHAPE = 66,
    PRIM_TRANSPOSE = 67,
    PRIM_BROADCAST = 68,
    PRIM_EXPAND_DIMS = 69,
    PRIM_SQUEEZE = 70,
    PRIM_SLICE = 71,
    PRIM_CONCAT = 72,
    PRIM_STACK = 73,
    PRIM_TAKE = 74,
    PRIM_SCATTER_ADD = 75,
    PRIM_PAD = 76,
    PRIM_FLIP = 77,
    PRIM_CUMSUM = 78,
    PRIM_REVERSE = 79,
    PRIM_CONSTANT = 87,
    PRIM_COPY = 88,
    PRIM_CAST = 89,
    PRIM_MATMUL = 80,
};
constexpr int32_t kFlagReverse = 1 << 5;  // prims.Attrs.REVERSE

const char *kPrimNames[] = {
    "neg", "abs", "exp", "expm1", "log", "log1p", "sqrt", "rsqrt", "square", "recip", "cbrt",
    "sin", "cos", "tan", "asin", "acos", "atan", "sinh", "cosh", "tanh", "asinh", "acosh",
    "atanh", "erf", "sigmoid", "softplus", "relu", "floor", "ceil", "round", "trunc", "sign",
    "isnan", "isinf", "isfinite", "add", "sub", "mul", "div", "pow", "maximum", "minimum",
    "atan2", "hypot", "mod_op", "eq", "ne", "lt", "le", "gt", "ge", "logical_and", "logical_or",
    "logical_xor", "logical_not", "where", "clamp", "lerp", "sum", "prod_op", "max_reduce", "min_reduce",
    "any_reduce", "all_reduce", "argmax", "argmin"};

// The element-wise prims a region kernel evaluates (prims.isElementwise,
// src/zpu/prims.zig:198): float math, the predicates (bool results:
// isnan / isinf / isfinite, comparisons, logical ops) and `where`.
bool math_unary(int p) { return p >= 0 && p <= 31; }
bool pred_unary(int p) { return (p >= 32 && p <= 34) || p == PRIM_LOGICAL_NOT; }
bool math_binary(int p) { return p >= 35 && p <= 44; }
bool pred_binary(int p) { return p >= 45 && p <= 53; }
bool region_unary(int p) { return math_unary(p) || pred_unary(p); }
bool region_binary(int p) { return math_binary(p) || pred_binary(p); }
bool arg_reduce(int p) { return p == PRIM_ARGMAX || p == PRIM_ARGMIN; }
bool bool_reduce(int p) { return p == PRIM_ANY || p == PRIM_ALL; }
bool region_reduce(int p) { return (p >= PRIM_SUM && p <= PRIM_MIN_REDUCE) || arg_reduce(p) || bool_reduce(p); }
bool float_dtype(int dt) { return dt == ZPUCUDA_F32 || dt == ZPUCUDA_F64; }
// prims.isFloatOnly (src/zpu/prims.zig:229-234): of an integer value they
// give f32 (unaryOutDType, ops.zig:268-273); div joins them for two integers
// (binaryOutDType, ops.zig:275-285)
bool float_only(int p) {
    return (p >= 2 && p <= 7) || (p >= 10 && p <= 25) || p == 42 || p == 43;
}
constexpr int PRIM_DIV = 38, PRIM_POW = 39;
// The movement prims a plan lowers as views (ops.zig:1343-1555).
// flip / reverse mirror one axis (negative stride); copy and constant replay
// as their input (ops.zig:2195-2198).
bool view_prim(int p) {
    return (p >= PRIM_RESHAPE && p <= PRIM_SLICE) || p == PRIM_FLIP || p == PRIM_REVERSE || p == PRIM_COPY ||
           p == PRIM_CONSTANT;
}
bool any_dtype(int dt) { return dt >= ZPUCUDA_F64 && dt <= ZPUCUDA_BOOL; }
// Bool values ride in a region's float registers: two values fit one region
// unless both are floats of different types.  -1: no float type required.
int carrier_of(int dt) { return float_dtype(dt) ? dt : -1; }
bool carriers_agree(int a, int b) { return a < 0 || b < 0 || a == b; }

struct Shape {
    int rank = 0;
    int64_t dims[ZPUCUDA_MAX_RANK] = {0};
    int64_t numel() const {
        int64_t n = 1;
        for (int i = 0; i < rank; i++) n *= dims[i];
        return n;
    }
    bool operator==(const Shape &o) const {
        if (rank != o.rank) return false;
        for (int i = 0; i < rank; i++)
            if (dims[i] != o.dims[i]) return false;
        return true;
    }
};

// NumPy broadcasting, right-aligned (shape.broadcastShapeRanked for
// batch_depth 0, src/zpu/shape.zig:78).
bool broadcast(const Shape &a, const Shape &b, Shape *out) {
    Shape r;
    r.rank = std::max(a.rank, b.rank);
    for (int i = 0; i < r.rank; i++) {
        const int ia = a.rank - r.rank + i, ib = b.rank - r.rank + i;
        const int64_t da = ia >= 0 ? a.dims[ia] : 1, db = ib >= 0 ? b.dims[ib] : 1;
        if (da == db || db == 1) r.dims[i] = da;
        else if (da == 1) r.dims[i] = db;
        else return false;
    }
    *out = r;
    return true;
}

enum SlotKind { SLOT_ARG, SLOT_BLOB, SLOT_TEMP, SLOT_OUT };
struct Slot {
    SlotKind kind = SLOT_TEMP;
    int index = -1;
};

struct Value {
    int32_t dtype = ZPUCUDA_F32;
    Shape shape;
    int32_t depth = 0;
    int producer = -1;  // step index, -1 for args / blobs
    bool is_arg = false, is_blob = false;
    int arg_index = -1, blob_index = -1;
    bool materialised = false;  // has a Slot
    Slot slot;
    // element (i0, i1, ...) lives at offset + sum(i_d * strides[d]) of the
    // slot: contiguous with offset 0 except for views
    int64_t strides[ZPUCUDA_MAX_RANK] = {0};
    int64_t offset = 0;
    bool view = false;          // a view step's output: the input's slot
    bool reshape_copy = false;  // a reshape of a non-contiguous view: copied first
    void set_contiguous() {
        int64_t st = 1;
        for (int d = shape.rank - 1; d >= 0; d--) {
            strides[d] = st;
            st *= shape.dims[d];
        }
    }
    bool contiguous() const {  // size-1 axes may have any stride
        int64_t st = 1;
        for (int d = shape.rank - 1; d >= 0; d--) {
            if (shape.dims[d] != 1 && strides[d] != st) return false;
            st *= shape.dims[d];
        }
        return true;
    }
};

struct Launch {
    enum { REGION, MATMUL, CUMSUM, COPY, COPYV, FILL, TAKE, SCATTER } kind = REGION;
    // COPYV: src view (ma + ma_off) into the dst view (mc + mc_off, dst's
    // strides); FILL: mc with `scalar`; TAKE / SCATTER: ma = x or updates,
    // mb = indices, mc = out, [outer, sdim, inner] and k
    zpucuda_tensor dst;
    int64_t mc_off = 0;
    double scalar = 0.0;
    int32_t idx_dtype = 0;
    int64_t k = 0;
    std::vector<int64_t> in_off;  // region inputs: byte offsets into their slots
    int64_t ma_off = 0, mb_off = 0;  // matmul / cumsum / copy source: byte offsets
    int32_t epi_mode = 0;            // matmul: EPI_BIAS / EPI_BIAS_TANH fused, 0 none
    Slot bias;                       // its bias vector
    int64_t bias_off = 0;
    zpucuda_tensor src;              // copy: the view (data set at run time)
    int32_t dst_dtype = 0;           // copy: the output's element type (a cast converts)
    RegionProgram prog;
    const CatalogueEntry *cat = nullptr;
    std::string signature;
    std::vector<Slot> ins, outs;
    Slot red;
    bool has_red = false;
    void *workspace = nullptr;
    // matmul
    Slot ma, mb, mc;
    zpucuda_tensor ta, tb, tc;
    // cumsum: [outer, dim, inner] along the middle axis
    int32_t dtype = 0;
    int64_t outer = 0, dim = 0, inner = 0;
    bool reverse = false;
    std::string text;
};

}  // namespace

struct zpucuda_plan {
    int n_args = 0;
    int n_steps = 0;
    std::vector<zpucuda_value> arg_values;
    std::vector<void *> stage_in, stage_out;  // HBM staging of zpucuda_plan_run_host
    std::vector<Launch> launches;
    std::vector<zpucuda_value> outputs;
    std::vector<void *> blobs;  // HBM copies of folded constants
    std::vector<void *> temps;  // intermediates that cross launches
    std::vector<void *> workspaces;
    unsigned int *err = nullptr;  // index errors of take / scatter_add launches
    std::string text;
    ~zpucuda_plan() {
        if (err) cudaFree(err);
        for (void *p : blobs) cudaFree(p);
        for (void *p : temps) cudaFree(p);
        for (void *p : workspaces) cudaFree(p);
        for (void *p : stage_in) cudaFree(p);
        for (void *p : stage_out) cudaFree(p);
    }
};

namespace {

// zpu's DType sizes (src/zpu/dtype.zig:4-13)
size_t itemsize(int dt) {
    switch (dt) {
    case ZPUCUDA_F64: case ZPUCUDA_I64: return 8;
    case ZPUCUDA_F32: case ZPUCUDA_I32: return 4;
    case ZPUCUDA_F16: case ZPUCUDA_I16: return 2;
    default: return 1;
    }
}

int lower_fail(zpucuda_plan *p, int st, const std::string &why) {
    delete p;
    return set_error(st, "zpucuda_plan_create: " + why);
}

std::string prim_name(int p) {
    if (p >= 0 && p < (int)(sizeof(kPrimNames) / sizeof(kPrimNames[0]))) return kPrimNames[p];
    return "prim" + std::to_string(p);
}

// The axes a reduction folds (ops.axesMaskOf, src/zpu/ops.zig:630-642):
// AXIS_NONE folds the payload axes [depth, rank); a non-negative axis counts
// from the first payload axis, a negative one from the last axis.  The folded
// axes are the contiguous range [*first, *last] (empty for a rank-0 value).
bool reduced_axes(const Shape &s, int depth, int axis, int *first, int *last) {
    if (axis == ZPUCUDA_AXIS_NONE) {
        *first = depth < s.rank ? depth : s.rank;
        *last = s.rank - 1;
        return true;
    }
    const int a = axis >= 0 ? axis + depth : axis + s.rank;
    if (a < 0 || a >= s.rank) return false;
    *first = *last = a;
    return true;
}

}  // namespace

extern "C" {

int zpucuda_plan_create(const zpucuda_value *args, int n_args, const zpucuda_blob *blobs, int n_blobs,
                        const zpucuda_step *steps, int n_steps, const uint64_t *out_ids, int n_outs,
                        zpucuda_plan **out) {
    ZC_CHECK(out && (args || !n_args) && (blobs || !n_blobs) && (steps || !n_steps) && out_ids && n_outs > 0,
             ZPUCUDA_ERR_INVALID_ARGUMENT);
    *out = nullptr;
    zpucuda_plan *plan = new zpucuda_plan;
    plan->n_args = n_args;
    plan->n_steps = n_steps;
    plan->arg_values.assign(args, args + n_args);
    std::map<uint64_t, Value> vals;

    auto add_value = [&](const zpucuda_value &v) -> Value & {
        Value &x = vals[v.id];
        x.dtype = v.dtype;
        x.shape.rank = v.rank;
        for (int i = 0; i < v.rank; i++) x.shape.dims[i] = v.dims[i];
        x.depth = v.batch_depth;
        x.set_contiguous();
        return x;
    };
    for (int i = 0; i < n_args; i++) {
        if (args[i].rank < 0 || args[i].rank > ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_RANK_TOO_LARGE, "arg rank");
        if (!any_dtype(args[i].dtype)) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "arg dtype");
        Value &v = add_value(args[i]);
        v.is_arg = true;
        v.arg_index = i;
        v.materialised = true;
        v.slot = {SLOT_ARG, i};
    }
    for (int i = 0; i < n_blobs; i++) {
        const zpucuda_value &bv = blobs[i].value;
        if (bv.rank < 0 || bv.rank > ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_RANK_TOO_LARGE, "blob rank");
        if (!float_dtype(bv.dtype) && bv.dtype != ZPUCUDA_BOOL) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "blob dtype");
        Value &v = add_value(bv);
        v.is_blob = true;
        v.blob_index = i;
        v.materialised = true;
        v.slot = {SLOT_BLOB, i};
        const size_t nb = (size_t)v.shape.numel() * itemsize(v.dtype);
        void *d = nullptr;
        if (cudaMalloc(&d, nb ? nb : 16) != cudaSuccess) {
            cudaGetLastError();
            return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "blob allocation");
        }
        plan->blobs.push_back(d);
        if (nb && cudaMemcpy(d, blobs[i].host_data, nb, cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaGetLastError();
            return lower_fail(plan, ZPUCUDA_ERR_CUDA, "blob upload");
        }
    }

    // ---- shapes of every step output, and who uses what
    std::map<uint64_t, std::vector<int>> users;
    for (int s = 0; s < n_steps; s++) {
        const zpucuda_step &st = steps[s];
        if (st.n_inputs < 0 || st.n_inputs > 3) return lower_fail(plan, ZPUCUDA_ERR_INVALID_ARGUMENT, "step arity");
        for (int k = 0; k < st.n_inputs; k++) {
            if (!vals.count(st.ins[k])) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "step input not defined before use");
            users[st.ins[k]].push_back(s);
        }
        Value o;
        o.producer = s;
        const Value &a = vals[st.ins[0]];
        o.dtype = a.dtype;
        o.depth = a.depth;
        // operand types: float math and the numeric reductions take floats;
        // predicates, `where`'s condition and any / all also take bools
        // (truthiness v != 0, ops.zig:516, 572-590, 845-853)
        const bool takes_bool = pred_unary(st.prim) || pred_binary(st.prim) || bool_reduce(st.prim) ||
                                st.prim == PRIM_WHERE;
        // i64 values (argmax / argmin results, i64 arguments) enter
        // element-wise steps and reductions, typed as zpu types them
        // (DType.promote, dtype.zig:89-104: floats win; unaryOutDType /
        // binaryOutDType, ops.zig:268-285; reduceOutDType, ops.zig:813-818):
        // against a float the float type; of i64 values alone an i64, except
        // the float-only prims and div (f32) and the predicates (bool); sum /
        // prod / max / min of i64 values an i64.
        for (int k = 0; k < st.n_inputs && (region_unary(st.prim) || region_binary(st.prim) ||
                                            region_reduce(st.prim) || st.prim == PRIM_WHERE);
             k++) {
            const int dt = vals[st.ins[k]].dtype;
            const bool ok = float_dtype(dt) || dt == ZPUCUDA_I64 ||
                            (dt == ZPUCUDA_BOOL && takes_bool && !(st.prim == PRIM_WHERE && k > 0));
            if (!ok) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "prim " + prim_name(st.prim) + " on a value of dtype " + std::to_string(dt));
        }
        if (pred_unary(st.prim) || pred_binary(st.prim) || bool_reduce(st.prim)) o.dtype = ZPUCUDA_BOOL;
        if (region_unary(st.prim) && st.n_inputs == 1) {
            o.shape = a.shape;
            if (a.dtype == ZPUCUDA_I64 && math_unary(st.prim)) o.dtype = float_only(st.prim) ? ZPUCUDA_F32 : ZPUCUDA_I64;
        } else if (region_binary(st.prim) && st.n_inputs == 2) {
            const Value &b = vals[st.ins[1]];
            const bool int_and_float = (a.dtype == ZPUCUDA_I64 && float_dtype(b.dtype)) ||
                                       (b.dtype == ZPUCUDA_I64 && float_dtype(a.dtype));
            if (!carriers_agree(carrier_of(a.dtype), carrier_of(b.dtype)) ||
                (math_binary(st.prim) && a.dtype != b.dtype && !int_and_float))
                return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "mixed dtypes in an element-wise step");
            if (math_binary(st.prim) && int_and_float) o.dtype = float_dtype(a.dtype) ? a.dtype : b.dtype;
            if (math_binary(st.prim) && a.dtype == ZPUCUDA_I64 && b.dtype == ZPUCUDA_I64)
                o.dtype = (float_only(st.prim) || st.prim == PRIM_DIV) ? ZPUCUDA_F32 : ZPUCUDA_I64;
            if (a.depth != b.depth && a.shape.rank && b.shape.rank)
                return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "vmap depth mismatch in an element-wise step");
            o.depth = std::max(a.depth, b.depth);
            if (!broadcast(a.shape, b.shape, &o.shape)) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "broadcast");
        } else if (st.prim == PRIM_WHERE && st.n_inputs == 3) {
            // where(cond, a, b): a / b broadcast, then with cond; the type
            // DType.promote(a, b) (ops.zig:572-576): i64 when both are i64,
            // else the float one; the condition is any value's v != 0
            const Value &x = vals[st.ins[1]], &y = vals[st.ins[2]];
            const bool xi = x.dtype == ZPUCUDA_I64, yi = y.dtype == ZPUCUDA_I64;
            const int odt = (xi && yi) ? ZPUCUDA_I64 : xi ? y.dtype : x.dtype;
            if ((!xi && !yi && x.dtype != y.dtype) || !carriers_agree(carrier_of(a.dtype), carrier_of(odt)))
                return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "mixed dtypes in where");
            Shape xy;
            if (!broadcast(x.shape, y.shape, &xy) || !broadcast(xy, a.shape, &o.shape))
                return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "broadcast");
            o.dtype = odt;
            o.depth = std::max(a.depth, std::max(x.depth, y.depth));
        } else if (region_reduce(st.prim) && st.n_inputs == 1) {
            // ops.reduceOutShape (src/zpu/ops.zig:644-660); argmax / argmin
            // never keep the folded axes and give i64 (ops.zig:931-934)
            int r0 = 0, r1 = -1;
            if (!reduced_axes(a.shape, a.depth, st.axis, &r0, &r1))
                return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "reduction axis");
            const bool keep = (st.flags & 1) && !arg_reduce(st.prim);
            o.shape.rank = 0;
            for (int d = 0; d < a.shape.rank; d++) {
                if (d >= r0 && d <= r1) {
                    if (keep) o.shape.dims[o.shape.rank++] = 1;
                } else {
                    o.shape.dims[o.shape.rank++] = a.shape.dims[d];
                }
            }
            if (arg_reduce(st.prim)) o.dtype = ZPUCUDA_I64;
        } else if (view_prim(st.prim) && st.n_inputs == 1) {
            o.view = true;
            o.offset = a.offset;
            const int r = a.shape.rank;
            if (st.prim == PRIM_RESHAPE) {
                // ops.reshape / reshapeTarget (ops.zig:1343-1400): a payload
                // shape under vmap keeps the batch axes; -1 is inferred
                Shape req;
                req.rank = st.shape_len;
                if (req.rank < 0 || req.rank > ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_RANK_TOO_LARGE, "reshape rank");
                for (int i = 0; i < req.rank; i++) req.dims[i] = st.shape[i];
                if (req.rank + a.depth == r && a.depth > 0) {
                    if (r > ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_RANK_TOO_LARGE, "reshape rank");
                    for (int i = req.rank - 1; i >= 0; i--) req.dims[i + a.depth] = req.dims[i];
                    for (int i = 0; i < a.depth; i++) req.dims[i] = a.shape.dims[i];
                    req.rank = r;
                }
                int64_t known = 1;
                int unknown = -1;
                for (int i = 0; i < req.rank; i++) {
                    if (req.dims[i] == 0) return lower_fail(plan, ZPUCUDA_ERR_INVALID_SHAPE, "reshape to a zero dimension");
                    if (req.dims[i] < 0) {
                        if (unknown >= 0) return lower_fail(plan, ZPUCUDA_ERR_INVALID_SHAPE, "reshape with two -1");
                        unknown = i;
                    } else {
                        known *= req.dims[i];
                    }
                }
                if (unknown >= 0) {
                    if (known == 0 || a.shape.numel() % known) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "reshape");
                    req.dims[unknown] = a.shape.numel() / known;
                }
                if (req.numel() != a.shape.numel() || req.rank < a.depth)
                    return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "reshape");
                o.shape = req;
                o.set_contiguous();
                if (!a.contiguous()) {
                    o.reshape_copy = true;
                    o.offset = 0;
                }
            } else if (st.prim == PRIM_TRANSPOSE) {
                // ops.transpose (ops.zig:1424-1449): a payload permutation
                // under vmap leaves the batch axes first
                int perm[ZPUCUDA_MAX_RANK];
                if (st.nsl == r) {
                    for (int i = 0; i < r; i++) perm[i] = st.perm[i];
                } else if (st.nsl + a.depth == r) {
                    for (int i = 0; i < a.depth; i++) perm[i] = i;
                    for (int i = 0; i < st.nsl; i++) perm[a.depth + i] = st.perm[i] + a.depth;
                } else {
                    return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "transpose permutation length");
                }
                bool seen[ZPUCUDA_MAX_RANK] = {false};
                for (int i = 0; i < r; i++) {
                    if (perm[i] < 0 || perm[i] >= r || seen[perm[i]]) return lower_fail(plan, ZPUCUDA_ERR_INVALID_SHAPE, "transpose permutation");
                    seen[perm[i]] = true;
                }
                o.shape.rank = r;
                for (int i = 0; i < r; i++) {
                    o.shape.dims[i] = a.shape.dims[perm[i]];
                    o.strides[i] = a.strides[perm[i]];
                }
            } else if (st.prim == PRIM_SLICE) {
                // ops.sliceView with the ranges sliceAttrs records
                // (ops.zig:1587-1635): element j of axis i at starts[i] +
                // j * steps[i], j < lens[i]; payload ranges under vmap leave
                // the batch axes whole.  (zpu's replay rebuilds Range(start,
                // start + len, step), which agrees for step 1.)
                int64_t st0[ZPUCUDA_MAX_RANK], ln[ZPUCUDA_MAX_RANK], sp[ZPUCUDA_MAX_RANK];
                if (st.nsl == r) {
                    for (int i = 0; i < r; i++) { st0[i] = st.starts[i]; ln[i] = st.shape[i]; sp[i] = st.steps[i]; }
                } else if (st.nsl + a.depth == r) {
                    for (int i = 0; i < a.depth; i++) { st0[i] = 0; ln[i] = a.shape.dims[i]; sp[i] = 1; }
                    for (int i = 0; i < st.nsl; i++) {
                        st0[a.depth + i] = st.starts[i];
                        ln[a.depth + i] = st.shape[i];
                        sp[a.depth + i] = st.steps[i];
                    }
                } else {
                    return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "slice ranges");
                }
                o.shape.rank = r;
                for (int i = 0; i < r; i++) {
                    const int64_t d = a.shape.dims[i];
                    if (sp[i] == 0 || ln[i] < 0) return lower_fail(plan, ZPUCUDA_ERR_INVALID_SHAPE, "slice range");
                    if (ln[i] > 0) {
                        const int64_t last = st0[i] + (ln[i] - 1) * sp[i];
                        if (st0[i] < 0 || st0[i] >= d || last < 0 || last >= d)
                            return lower_fail(plan, ZPUCUDA_ERR_INDEX_OUT_OF_RANGE, "slice range");
                        o.offset += st0[i] * a.strides[i];
                    }
                    o.shape.dims[i] = ln[i];
                    o.strides[i] = a.strides[i] * sp[i];
                }
            } else if (st.prim == PRIM_COPY || st.prim == PRIM_CONSTANT) {
                o.shape = a.shape;
                for (int i = 0; i < r; i++) o.strides[i] = a.strides[i];
            } else if (st.prim == PRIM_FLIP || st.prim == PRIM_REVERSE) {
                // ops.flip (ops.zig:2019-2030): realAxis, stride negated, the
                // offset moved to the axis's last element
                const int ax = st.axis >= 0 ? st.axis + a.depth : st.axis + r;
                if (ax < 0 || ax >= r) return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "flip axis");
                o.shape = a.shape;
                for (int i = 0; i < r; i++) o.strides[i] = a.strides[i];
                o.strides[ax] = -a.strides[ax];
                o.offset = a.offset + (a.shape.dims[ax] > 0 ? a.shape.dims[ax] - 1 : 0) * a.strides[ax];
            } else if (st.prim == PRIM_BROADCAST) {
                // ops.broadcastTo / broadcastTarget (ops.zig:1480-1522)
                Shape t;
                t.rank = st.shape_len;
                if (t.rank < r || t.rank > ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "broadcast target");
                for (int i = 0; i < t.rank; i++) t.dims[i] = st.shape[i];
                for (int i = 0; i < r; i++) {
                    const int64_t rd = t.dims[t.rank - r + i], xd = a.shape.dims[i];
                    if (rd != xd && xd != 1 && rd != 1) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "broadcast target");
                }
                // NumPy right alignment: x's axis xi = i - (t.rank - r); a
                // size-1 or missing axis gets stride 0.  (zpu's loop maps
                // axis i < r to x axis i - (t.rank - r), which is negative for
                // a rank-increasing target; for equal ranks the two agree.)
                for (int i = 0; i < t.rank; i++) {
                    const int xi = i - (t.rank - r);
                    o.strides[i] = (xi < 0 || a.shape.dims[xi] == 1) ? 0 : a.strides[xi];
                }
                o.shape = t;
            } else {
                // ops.expandDims / squeeze (ops.zig:1524-1555): payload axes
                const int payload = r - a.depth;
                int ax = st.axis;
                if (st.prim == PRIM_EXPAND_DIMS) {
                    if (ax < 0) ax += payload + 1;
                    if (ax < 0 || ax > payload || r >= ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "expand_dims axis");
                    const int pos = a.depth + ax;
                    o.shape.rank = r + 1;
                    for (int i = 0, j = 0; i < r + 1; i++) {
                        if (i == pos) {
                            o.shape.dims[i] = 1;
                            o.strides[i] = 0;
                        } else {
                            o.shape.dims[i] = a.shape.dims[j];
                            o.strides[i] = a.strides[j];
                            j++;
                        }
                    }
                } else {
                    if (ax < 0) ax += payload;
                    if (ax < 0 || ax >= payload) return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "squeeze axis");
                    const int pos = a.depth + ax;
                    if (a.shape.dims[pos] != 1) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "squeeze of an axis longer than 1");
                    o.shape.rank = r - 1;
                    for (int i = 0, j = 0; j < r; j++) {
                        if (j == pos) continue;
                        o.shape.dims[i] = a.shape.dims[j];
                        o.strides[i] = a.strides[j];
                        i++;
                    }
                }
            }
        } else if ((st.prim == PRIM_CONCAT || st.prim == PRIM_STACK) && st.n_inputs == 2) {
            // ops.concat (ops.zig:1665-1687; realAxis, equal ranks, the other
            // axes equal) and ops.stack (expand_dims of both, then concat)
            const Value &b = vals[st.ins[1]];
            if (a.dtype != b.dtype) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "concat of different dtypes");
            Shape sa = a.shape, sb = b.shape;
            if (st.prim == PRIM_STACK) {
                for (Shape *sh : {&sa, &sb}) {
                    const int payload = sh->rank - (sh == &sa ? a.depth : b.depth);
                    int ax = st.axis < 0 ? st.axis + payload + 1 : st.axis;
                    if (ax < 0 || ax > payload || sh->rank >= ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "stack axis");
                    const int pos = (sh == &sa ? a.depth : b.depth) + ax;
                    for (int d = sh->rank; d > pos; d--) sh->dims[d] = sh->dims[d - 1];
                    sh->dims[pos] = 1;
                    sh->rank += 1;
                }
            }
            if (sa.rank != sb.rank) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "concat ranks");
            const int ax = st.axis >= 0 ? st.axis + a.depth : st.axis + sa.rank;
            if (ax < 0 || ax >= sa.rank) return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "concat axis");
            for (int d = 0; d < sa.rank; d++)
                if (d != ax && sa.dims[d] != sb.dims[d]) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "concat shapes");
            o.shape = sa;
            o.shape.dims[ax] = sa.dims[ax] + sb.dims[ax];
            o.depth = std::max(a.depth, b.depth);
        } else if (st.prim == PRIM_PAD && st.n_inputs == 1) {
            // ops.pad (ops.zig:1995-2017): one (lo, hi) per axis
            if (st.nsl != a.shape.rank) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "pad widths");
            o.shape = a.shape;
            for (int d = 0; d < a.shape.rank; d++) {
                if (st.starts[d] < 0 || st.pads_hi[d] < 0) return lower_fail(plan, ZPUCUDA_ERR_INVALID_SHAPE, "pad widths");
                o.shape.dims[d] += st.starts[d] + st.pads_hi[d];
            }
        } else if ((st.prim == PRIM_TAKE && st.n_inputs == 2) || (st.prim == PRIM_SCATTER_ADD && st.n_inputs == 3)) {
            // ops.take / scatterAdd (ops.zig:1697-1797): a plain axis of x
            const Value &ix = vals[st.ins[1]];
            if (a.depth > 0 && ix.depth > 0) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "take under two vmaps");
            const int r = a.shape.rank;
            const int ax = st.axis < 0 ? st.axis + r : st.axis;
            if (ax < 0 || ax >= r) return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "take axis");
            if (ix.dtype != ZPUCUDA_I64 && ix.dtype != ZPUCUDA_I32 && !float_dtype(ix.dtype))
                return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "index dtype");
            if (st.prim == PRIM_TAKE) {
                if (r - 1 + ix.shape.rank > ZPUCUDA_MAX_RANK) return lower_fail(plan, ZPUCUDA_ERR_RANK_TOO_LARGE, "take rank");
                o.shape.rank = 0;
                for (int d = 0; d < ax; d++) o.shape.dims[o.shape.rank++] = a.shape.dims[d];
                for (int d = 0; d < ix.shape.rank; d++) o.shape.dims[o.shape.rank++] = ix.shape.dims[d];
                for (int d = ax + 1; d < r; d++) o.shape.dims[o.shape.rank++] = a.shape.dims[d];
                o.depth = std::max(a.depth, ix.depth);
            } else {
                const Value &u = vals[st.ins[2]];
                int64_t outer = 1, inner = 1;
                for (int d = 0; d < ax; d++) outer *= a.shape.dims[d];
                for (int d = ax + 1; d < r; d++) inner *= a.shape.dims[d];
                if (u.dtype != a.dtype) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "scatter_add updates dtype");
                if (u.shape.numel() != outer * ix.shape.numel() * inner)
                    return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "scatter_add updates");
                if (a.dtype == ZPUCUDA_BOOL) return lower_fail(plan, ZPUCUDA_ERR_DTYPE_MISMATCH, "scatter_add on bool");
                o.shape = a.shape;
            }
        } else if (st.prim == PRIM_CAST && st.n_inputs == 1) {
            // ops.cast (ops.zig:2062-2071; the type is Attrs.axis): the input
            // itself for its own type, else a converting copy
            if (!any_dtype(st.axis)) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "cast target dtype");
            o.shape = a.shape;
            o.dtype = st.axis;
            if (st.axis == a.dtype) {
                o.view = true;
                o.offset = a.offset;
                for (int i = 0; i < a.shape.rank; i++) o.strides[i] = a.strides[i];
            }
        } else if (st.prim == PRIM_CUMSUM && st.n_inputs == 1) {
            // ops.realAxis (src/zpu/ops.zig:1466-1471): vmap-aware, no AXIS_NONE
            // f64 accumulator, each prefix written as the element type
            // (ops.cumsum, ops.zig:2032-2057): floats and i64
            if (!float_dtype(a.dtype) && a.dtype != ZPUCUDA_I64)
                return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "cumsum of a bool or narrow integer value");
            const int ax = st.axis >= 0 ? st.axis + a.depth : st.axis + a.shape.rank;
            if (ax < 0 || ax >= a.shape.rank) return lower_fail(plan, ZPUCUDA_ERR_INVALID_AXIS, "cumsum axis");
            o.shape = a.shape;
        } else if (st.prim == PRIM_MATMUL && st.n_inputs == 2) {
            const Value &b = vals[st.ins[1]];
            zpucuda_tensor ta = {}, tb = {}, tc = {};
            ta.dtype = a.dtype;
            ta.rank = a.shape.rank;
            ta.batch_depth = a.depth;
            tb.dtype = b.dtype;
            tb.rank = b.shape.rank;
            tb.batch_depth = b.depth;
            for (int i = 0; i < a.shape.rank; i++) ta.dims[i] = a.shape.dims[i];
            for (int i = 0; i < b.shape.rank; i++) tb.dims[i] = b.shape.dims[i];
            int64_t st_ = 1;
            for (int i = ta.rank - 1; i >= 0; i--) { ta.strides[i] = st_; st_ *= ta.dims[i]; }
            st_ = 1;
            for (int i = tb.rank - 1; i >= 0; i--) { tb.strides[i] = st_; st_ *= tb.dims[i]; }
            int r = zpucuda_matmul_shape(&ta, &tb, &tc);
            if (r) return lower_fail(plan, r, "matmul shape");
            // mixed operand types run zpu's gemmF64 loop; a plan carries its
            // result when that is a float value (DType.promote: floats win)
            if (tc.dtype != ZPUCUDA_F32 && tc.dtype != ZPUCUDA_F64)
                return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "matmul with a non-float result in a plan");
            o.dtype = tc.dtype;
            o.shape.rank = tc.rank;
            for (int i = 0; i < tc.rank; i++) o.shape.dims[i] = tc.dims[i];
            o.depth = tc.batch_depth;
        } else {
            return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "prim " + prim_name(st.prim) + " is not lowered to the device");
        }
        if (vals.count(st.out)) return lower_fail(plan, ZPUCUDA_ERR_INVALID_ARGUMENT, "step output id reused");
        if (!o.view) o.set_contiguous();
        vals[st.out] = o;
    }
    std::map<uint64_t, int> out_index;
    for (int i = 0; i < n_outs; i++) {
        if (!vals.count(out_ids[i])) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "unknown output id");
        if (!out_index.count(out_ids[i])) out_index[out_ids[i]] = i;
        const Value &v = vals[out_ids[i]];
        zpucuda_value ov = {};
        ov.id = out_ids[i];
        ov.dtype = v.dtype;
        ov.rank = v.shape.rank;
        for (int d = 0; d < v.shape.rank; d++) ov.dims[d] = v.shape.dims[d];
        ov.batch_depth = v.depth;
        plan->outputs.push_back(ov);
    }

    // Where a step output lives once a launch writes it.
    auto materialise = [&](uint64_t id) -> Slot {
        Value &v = vals[id];
        if (v.materialised) return v.slot;
        auto it = out_index.find(id);
        if (it != out_index.end()) {
            v.slot = {SLOT_OUT, it->second};
        } else {
            void *d = nullptr;
            const size_t nb = (size_t)v.shape.numel() * itemsize(v.dtype);
            if (cudaMalloc(&d, nb ? nb : 16) != cudaSuccess) {
                cudaGetLastError();
                v.slot = {SLOT_TEMP, -1};
                return v.slot;
            }
            plan->temps.push_back(d);
            v.slot = {SLOT_TEMP, (int)plan->temps.size() - 1};
        }
        v.materialised = true;
        return v.slot;
    };

    // A copy launch of the view `v` (zpucuda_tensor_copy's kernels) into a
    // contiguous buffer: `dst`, or a new temp when dst.index < 0.
    auto copy_launch = [&](const Value &v, Slot dst, const std::string &why, int dst_dtype = -1) -> Slot {
        if (dst.index < 0) {
            void *d = nullptr;
            const size_t nb = (size_t)v.shape.numel() * itemsize(v.dtype);
            if (cudaMalloc(&d, nb ? nb : 16) != cudaSuccess) {
                cudaGetLastError();
                return Slot{SLOT_TEMP, -1};
            }
            plan->temps.push_back(d);
            dst = Slot{SLOT_TEMP, (int)plan->temps.size() - 1};
        }
        Launch L;
        L.kind = Launch::COPY;
        L.ma = v.slot;
        L.ma_off = v.offset * (int64_t)itemsize(v.dtype);
        memset(&L.src, 0, sizeof L.src);
        L.src.dtype = v.dtype;
        L.src.rank = v.shape.rank;
        for (int d = 0; d < v.shape.rank; d++) {
            L.src.dims[d] = v.shape.dims[d];
            L.src.strides[d] = v.strides[d];
        }
        L.mc = dst;
        L.dst_dtype = dst_dtype < 0 ? v.dtype : dst_dtype;
        L.text = "  kernel " + std::to_string(plan->launches.size()) + ": copy (" + why + ")\n";
        plan->launches.push_back(L);
        return dst;
    };
    // `v` as a contiguous value: itself, or a copy (v is left untouched)
    auto contiguous_of = [&](const Value &v, const std::string &why, Value *out) -> bool {
        *out = v;
        if (v.contiguous()) return true;
        Slot t = copy_launch(v, Slot{SLOT_TEMP, -1}, why);
        if (t.index < 0) return false;
        out->slot = t;
        out->offset = 0;
        out->set_contiguous();
        return true;
    };

    // ---- cut regions
    int s = 0;
    while (s < n_steps) {
        const zpucuda_step &st0 = steps[s];
        // descriptor of a value's view (data set at run time)
        auto desc_of = [](const Value &v) {
            zpucuda_tensor t;
            memset(&t, 0, sizeof t);
            t.dtype = v.dtype;
            t.rank = v.shape.rank;
            for (int d = 0; d < v.shape.rank; d++) {
                t.dims[d] = v.shape.dims[d];
                t.strides[d] = v.strides[d];
            }
            return t;
        };
        auto need_err = [&]() -> bool {
            if (plan->err) return true;
            if (cudaMalloc(&plan->err, sizeof(unsigned int)) != cudaSuccess ||
                cudaMemset(plan->err, 0, sizeof(unsigned int)) != cudaSuccess) {
                cudaGetLastError();
                plan->err = nullptr;
                return false;
            }
            return true;
        };
        // a COPYV launch of `src` into the part of out slot `dst` at element
        // offset `off` with out's contiguous strides `ost`
        auto copy_into = [&](const Value &src, const zpucuda_tensor &sdesc, Slot dst, const int64_t *ost, int64_t off,
                             const char *why) {
            Launch L;
            L.kind = Launch::COPYV;
            L.ma = src.slot;
            L.ma_off = src.offset * (int64_t)itemsize(src.dtype);
            L.src = sdesc;
            L.dst = sdesc;
            for (int d = 0; d < sdesc.rank; d++) L.dst.strides[d] = ost[d];
            L.mc = dst;
            L.mc_off = off * (int64_t)itemsize(src.dtype);
            L.text = "  kernel " + std::to_string(plan->launches.size()) + ": copy (" + why + ")\n";
            plan->launches.push_back(L);
        };
        if (st0.prim == PRIM_CONCAT || st0.prim == PRIM_STACK) {
            const Value &a = vals[st0.ins[0]], &b = vals[st0.ins[1]];
            Value &o = vals[st0.out];
            if (!a.materialised || !b.materialised) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "concat input not materialised");
            const Slot dst = materialise(st0.out);
            if (dst.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
            zpucuda_tensor sa = desc_of(a), sb = desc_of(b);
            if (st0.prim == PRIM_STACK)  // a length-1 axis (stride 0) at the stack position
                for (zpucuda_tensor *t : {&sa, &sb}) {
                    const int depth = t == &sa ? a.depth : b.depth, payload = t->rank - depth;
                    const int pos = depth + (st0.axis < 0 ? st0.axis + payload + 1 : st0.axis);
                    for (int d = t->rank; d > pos; d--) {
                        t->dims[d] = t->dims[d - 1];
                        t->strides[d] = t->strides[d - 1];
                    }
                    t->dims[pos] = 1;
                    t->strides[pos] = 0;
                    t->rank += 1;
                }
            const int ax = st0.axis >= 0 ? st0.axis + a.depth : st0.axis + sa.rank;
            copy_into(a, sa, dst, o.strides, 0, "concat, first part");
            copy_into(b, sb, dst, o.strides, sa.dims[ax] * o.strides[ax], "concat, second part");
            o.materialised = true;
            s++;
            continue;
        }
        if (st0.prim == PRIM_PAD) {
            const Value &a = vals[st0.ins[0]];
            Value &o = vals[st0.out];
            if (!a.materialised) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "pad input not materialised");
            const Slot dst = materialise(st0.out);
            if (dst.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
            Launch F;
            F.kind = Launch::FILL;
            F.mc = dst;
            F.dtype = o.dtype;
            F.k = o.shape.numel();
            F.scalar = st0.scalar;
            F.text = "  kernel " + std::to_string(plan->launches.size()) + ": fill (pad)\n";
            plan->launches.push_back(F);
            int64_t off = 0;
            for (int d = 0; d < o.shape.rank; d++) off += st0.starts[d] * o.strides[d];
            copy_into(a, desc_of(a), dst, o.strides, off, "pad interior");
            o.materialised = true;
            s++;
            continue;
        }
        if (st0.prim == PRIM_TAKE || st0.prim == PRIM_SCATTER_ADD) {
            const bool take = st0.prim == PRIM_TAKE;
            const Value &x0 = vals[st0.ins[0]];
            Value &o = vals[st0.out];
            Value x, ix, up;
            if (!x0.materialised || !vals[st0.ins[1]].materialised) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "take input not materialised");
            if ((take && !contiguous_of(x0, "take input", &x)) || !contiguous_of(vals[st0.ins[1]], "indices", &ix) ||
                (!take && !contiguous_of(vals[st0.ins[2]], "scatter_add updates", &up)) || !need_err())
                return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "copy buffer");
            Launch L;
            L.kind = take ? Launch::TAKE : Launch::SCATTER;
            const int r = x0.shape.rank;
            const int ax = st0.axis < 0 ? st0.axis + r : st0.axis;
            L.outer = 1;
            L.inner = 1;
            for (int d = 0; d < ax; d++) L.outer *= x0.shape.dims[d];
            for (int d = ax + 1; d < r; d++) L.inner *= x0.shape.dims[d];
            L.dim = x0.shape.dims[ax];
            L.k = ix.shape.numel();
            L.dtype = x0.dtype;
            L.idx_dtype = ix.dtype;
            L.ma = take ? x.slot : up.slot;
            L.ma_off = take ? x.offset * (int64_t)itemsize(x.dtype) : up.offset * (int64_t)itemsize(up.dtype);
            L.mb = ix.slot;
            L.mb_off = ix.offset * (int64_t)itemsize(ix.dtype);
            L.mc = materialise(st0.out);
            if (L.mc.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
            L.text = "  kernel " + std::to_string(plan->launches.size()) + (take ? ": take" : ": scatter_add") + "\n";
            plan->launches.push_back(L);
            o.materialised = true;
            s++;
            continue;
        }
        if (st0.prim == PRIM_CAST) {
            Value &a = vals[st0.ins[0]];
            Value &o = vals[st0.out];
            if (!a.materialised) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "cast of a value not materialised");
            if (o.view) {  // cast to its own type: the input itself
                o.slot = a.slot;
            } else {
                const Slot dst = materialise(st0.out);
                if (dst.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
                if (copy_launch(a, dst, "cast", o.dtype).index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "copy");
            }
            o.materialised = true;
            s++;
            continue;
        }
        if (view_prim(st0.prim)) {  // a view: the input's slot, no launch
            Value &a = vals[st0.ins[0]];
            Value &o = vals[st0.out];
            if (!a.materialised) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "view of a value not materialised");
            if (o.reshape_copy) {
                Value c;
                if (!contiguous_of(a, "reshape of a strided view", &c)) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "copy buffer");
                o.slot = c.slot;
                o.offset = 0;
            } else {
                o.slot = a.slot;
            }
            o.materialised = true;
            s++;
            continue;
        }
        if (st0.prim == PRIM_MATMUL) {
            // operands: views are read in place when one of the last two
            // axes has unit stride (row-major or transposed), else copied
            auto gemm_ok = [](const Value &v) {
                const int r = v.shape.rank;
                if (v.contiguous()) return true;
                if (r < 2) return false;
                for (int d = 0; d < r; d++)
                    if (v.strides[d] < 0) return false;
                const int64_t rows = v.shape.dims[r - 2], cols = v.shape.dims[r - 1];
                const int64_t s0 = v.strides[r - 2], s1 = v.strides[r - 1];
                if (s1 == 1 && (rows == 1 || s0 >= cols)) return true;  // row-major, leading dim s0
                if (s0 == 1 && (cols == 1 || s1 >= rows)) return true;  // transposed, leading dim s1
                return false;
            };
            Value a = vals[st0.ins[0]], b = vals[st0.ins[1]];
            if (!gemm_ok(a) && !contiguous_of(vals[st0.ins[0]], "matmul operand", &a))
                return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "copy buffer");
            if (!gemm_ok(b) && !contiguous_of(vals[st0.ins[1]], "matmul operand", &b))
                return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "copy buffer");
            Launch L;
            L.kind = Launch::MATMUL;
            L.ma = a.slot;
            L.mb = b.slot;
            L.ma_off = a.offset * (int64_t)itemsize(a.dtype);
            L.mb_off = b.offset * (int64_t)itemsize(b.dtype);
            memset(&L.ta, 0, sizeof L.ta);
            memset(&L.tb, 0, sizeof L.tb);
            L.ta.dtype = a.dtype; L.ta.rank = a.shape.rank; L.ta.batch_depth = a.depth;
            L.tb.dtype = b.dtype; L.tb.rank = b.shape.rank; L.tb.batch_depth = b.depth;
            for (int i = 0; i < a.shape.rank; i++) L.ta.dims[i] = a.shape.dims[i];
            for (int i = 0; i < b.shape.rank; i++) L.tb.dims[i] = b.shape.dims[i];
            if (a.contiguous()) {
                int64_t q = 1;
                for (int i = L.ta.rank - 1; i >= 0; i--) { L.ta.strides[i] = q; q *= L.ta.dims[i]; }
            } else {
                for (int i = 0; i < a.shape.rank; i++) L.ta.strides[i] = a.strides[i];
            }
            if (b.contiguous()) {
                int64_t q = 1;
                for (int i = L.tb.rank - 1; i >= 0; i--) { L.tb.strides[i] = q; q *= L.tb.dims[i]; }
            } else {
                for (int i = 0; i < b.shape.rank; i++) L.tb.strides[i] = b.strides[i];
            }
            zpucuda_matmul_shape(&L.ta, &L.tb, &L.tc);
            // matmul -> add(row bias) [-> tanh], each value used only by the
            // next: the f32 GEMM's bias / bias + tanh epilogue writes the last
            // one (one pass over the output instead of three)
            uint64_t final_id = st0.out;
            int fused = 0;
            const Value &mo = vals[st0.out];
            auto only_user = [&](uint64_t id, int step) {
                auto it = users.find(id);
                return !out_index.count(id) && it != users.end() && it->second.size() == 1 && it->second[0] == step;
            };
            if (a.dtype == ZPUCUDA_F32 && b.dtype == ZPUCUDA_F32 && mo.shape.rank == 2 && a.shape.rank <= 2 && b.shape.rank <= 2 &&
                s + 1 < n_steps && only_user(st0.out, s + 1)) {
                const zpucuda_step &ad = steps[s + 1];
                const uint64_t other = ad.n_inputs == 2 ? (ad.ins[0] == st0.out ? ad.ins[1] : ad.ins[0]) : 0;
                if (ad.prim == 35 && ad.n_inputs == 2 && other != st0.out && vals.count(other)) {
                    const Value &bv = vals[other];
                    const Value &ao = vals[ad.out];
                    const int64_t n = mo.shape.dims[1];
                    if (bv.dtype == ZPUCUDA_F32 && bv.materialised && bv.contiguous() && bv.shape.numel() == n &&
                        (bv.shape.rank == 1 || (bv.shape.rank == 2 && bv.shape.dims[0] == 1)) && ao.shape == mo.shape) {
                        fused = 1;
                        final_id = ad.out;
                        L.bias = bv.slot;
                        L.bias_off = bv.offset * 4;
                        if (s + 2 < n_steps && steps[s + 2].prim == 19 && steps[s + 2].n_inputs == 1 &&
                            steps[s + 2].ins[0] == ad.out && only_user(ad.out, s + 2))
                            fused = 2, final_id = steps[s + 2].out;
                    }
                }
            }
            L.epi_mode = fused == 2 ? EPI_BIAS_TANH : fused == 1 ? EPI_BIAS : 0;
            L.mc = materialise(final_id);
            if (L.mc.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
            char buf[160];
            snprintf(buf, sizeof buf, "  kernel %zu: gemm %s (%%%llu = matmul(%%%llu, %%%llu))\n", plan->launches.size(),
                     a.dtype != b.dtype ? "mixed-type (gemmF64 loop)" : a.dtype == ZPUCUDA_F64 ? "f64 dmma" : "f32 3xtf32",
                     (unsigned long long)st0.out,
                     (unsigned long long)st0.ins[0], (unsigned long long)st0.ins[1]);
            L.text = buf;
            if (fused) L.text.insert(L.text.size() - 1, fused == 2 ? " + bias + tanh epilogue" : " + bias epilogue");
            plan->launches.push_back(L);
            s += 1 + fused;
            continue;
        }
        if (st0.prim == PRIM_CUMSUM) {
            Value a;
            if (!contiguous_of(vals[st0.ins[0]], "cumsum input", &a)) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "copy buffer");
            Launch L;
            L.kind = Launch::CUMSUM;
            L.ma = a.slot;
            L.ma_off = a.offset * (int64_t)itemsize(a.dtype);
            L.dtype = a.dtype;
            const int ax = st0.axis >= 0 ? st0.axis + a.depth : st0.axis + a.shape.rank;
            L.outer = 1;
            L.inner = 1;
            for (int d = 0; d < ax; d++) L.outer *= a.shape.dims[d];
            for (int d = ax + 1; d < a.shape.rank; d++) L.inner *= a.shape.dims[d];
            L.dim = a.shape.dims[ax];
            L.reverse = (st0.flags & kFlagReverse) != 0;
            L.mc = materialise(st0.out);
            if (L.mc.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
            char buf[160];
            snprintf(buf, sizeof buf, "  kernel %zu: cumsum %s axis %d%s (%%%llu = cumsum(%%%llu))\n",
                     plan->launches.size(), a.dtype == ZPUCUDA_F64 ? "f64" : a.dtype == ZPUCUDA_I64 ? "i64" : "f32", ax, L.reverse ? " reverse" : "",
                     (unsigned long long)st0.out, (unsigned long long)st0.ins[0]);
            L.text = buf;
            plan->launches.push_back(L);
            s++;
            continue;
        }
        // a region: element-wise steps over one shape, at most one trailing reduction
        Launch L;
        RegionProgram &P = L.prog;
        memset(&P, 0, sizeof P);
        std::map<uint64_t, int> reg;  // value id -> register
        std::vector<uint64_t> loads;  // external inputs in order of first use
        std::vector<int> member;      // steps in this region
        Shape rshape;
        int32_t rdtype = -1;
        bool have_shape = false;
        int e = s;
        // first pass: which steps join
        // the float type a step computes in: its output's, else its inputs'
        // (i64 and bool values need no float type: they join any region)
        auto step_carrier = [&](const zpucuda_step &st) {
            int c = carrier_of(vals[st.out].dtype);
            for (int k = 0; k < st.n_inputs && c < 0; k++) c = carrier_of(vals[st.ins[k]].dtype);
            return c;
        };
        for (; e < n_steps; e++) {
            const zpucuda_step &st = steps[e];
            const Value &ov = vals[st.out];
            if (region_unary(st.prim) || region_binary(st.prim) || st.prim == PRIM_WHERE) {
                const int c = step_carrier(st);
                if (have_shape && (!(ov.shape == rshape) || !carriers_agree(c, rdtype))) break;
                if (!have_shape) { rshape = ov.shape; have_shape = true; }
                if (rdtype < 0) rdtype = c;
                member.push_back(e);
                continue;
            }
            if (region_reduce(st.prim)) {
                const Value &iv = vals[st.ins[0]];
                bool inside = std::find(member.begin(), member.end(), iv.producer) != member.end();
                if ((member.empty() || inside) && carriers_agree(carrier_of(iv.dtype), rdtype)) {
                    if (!have_shape) { rshape = iv.shape; have_shape = true; }
                    if (rdtype < 0) rdtype = carrier_of(iv.dtype);
                    member.push_back(e);
                    e++;
                }
            }
            break;
        }
        // an i64 value anywhere in the region (an operand, a step's result,
        // the reduced value): 64-bit registers (RegionProgram::words64)
        bool words64 = false;
        for (int m : member) {
            for (int k = 0; k < steps[m].n_inputs; k++) words64 |= vals[steps[m].ins[k]].dtype == ZPUCUDA_I64;
            if (!region_reduce(steps[m].prim)) words64 |= vals[steps[m].out].dtype == ZPUCUDA_I64;
        }
        // no float value: bools ride as f32, i64 regions store no float
        if (rdtype < 0) rdtype = words64 ? ZPUCUDA_F64 : ZPUCUDA_F32;
        if (member.empty()) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "step " + std::to_string(s) + " cannot start a region");
        P.dtype = rdtype;
        P.words64 = words64 ? 1 : 0;
        P.rank = rshape.rank;
        for (int i = 0; i < rshape.rank; i++) P.dims[i] = rshape.dims[i];
        P.numel = rshape.numel();
        std::vector<Insn> ops;
        int next_reg_after_loads = 0;
        // inputs: every operand not produced inside the region
        auto in_region = [&](uint64_t id) {
            const Value &v = vals[id];
            return v.producer >= 0 && std::find(member.begin(), member.end(), v.producer) != member.end();
        };
        for (int m : member)
            for (int k = 0; k < steps[m].n_inputs; k++) {
                uint64_t id = steps[m].ins[k];
                if (!in_region(id) && std::find(loads.begin(), loads.end(), id) == loads.end()) loads.push_back(id);
            }
        if ((int)loads.size() > RP_MAX_IN) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "region has too many inputs");
        P.n_in = (int)loads.size();
        std::string sig = std::string(rdtype == ZPUCUDA_F64 ? "f64" : "f32") + (words64 ? "w64" : "") + ";";
        std::string kinds;
        for (int k = 0; k < P.n_in; k++) {
            Value &iv = vals[loads[k]];
            if (!iv.materialised) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "region input not materialised");
            if (iv.dtype != rdtype && iv.dtype != ZPUCUDA_BOOL && iv.dtype != ZPUCUDA_I64)
                return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "mixed dtypes in a region");
            P.in_bool[k] = iv.dtype == ZPUCUDA_BOOL;
            P.in_i64[k] = iv.dtype == ZPUCUDA_I64;
            reg[loads[k]] = k;
            P.insn[k] = Insn{OPC_LOAD, (uint8_t)k, (uint8_t)k, 0};
            L.ins.push_back(iv.slot);
            L.in_off.push_back(iv.offset * (int64_t)itemsize(iv.dtype));
            const Shape &is = iv.shape;
            P.in_numel[k] = is.numel();
            if (!iv.contiguous() && is.numel() != 1) {
                // a strided view: its own strides over the region's axes
                for (int d = rshape.rank - 1; d >= 0; d--) {
                    const int id = is.rank - rshape.rank + d;
                    const int64_t dim = id >= 0 ? is.dims[id] : 1;
                    if (dim != 1 && dim != rshape.dims[d]) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "region broadcast");
                    P.in_strides[k][d] = (id < 0 || dim == 1) ? 0 : iv.strides[id];
                }
                P.in_kind[k] = IN_GENERAL;
                kinds += "G";
            } else if (is == rshape) {
                P.in_kind[k] = IN_FULL;
                kinds += "F";
            } else if (is.numel() == 1) {
                P.in_kind[k] = IN_SCALAR;
                kinds += "S";
            } else {
                // right-aligned broadcast: strides over the region's axes
                bool row = is.rank <= rshape.rank;
                int64_t stride = 1;
                for (int d = rshape.rank - 1; d >= 0; d--) {
                    const int id = is.rank - rshape.rank + d;
                    const int64_t dim = id >= 0 ? is.dims[id] : 1;
                    if (dim != 1 && dim != rshape.dims[d]) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "region broadcast");
                    P.in_strides[k][d] = dim == 1 ? 0 : stride;
                    if (id < 0 || dim == 1) { if (id >= 0) row = false; }
                    else if (dim != rshape.dims[d]) row = false;
                    stride *= dim;
                }
                // a row: the input is exactly the region's trailing axes
                int lead = rshape.rank - is.rank;
                for (int d = 0; d < is.rank && row; d++)
                    if (is.dims[d] != rshape.dims[lead + d]) row = false;
                P.in_kind[k] = row ? IN_ROW : IN_GENERAL;
                kinds += row ? "R" : "G";
            }
        }
        sig += kinds;
        next_reg_after_loads = P.n_in;
        int nreg = P.n_in;
        int n_insn = P.n_in;
        bool has_red = false;
        int red_prim = -1, red_axis = ZPUCUDA_AXIS_NONE, red_depth = 0;
        uint64_t red_in = 0, red_out_id = 0;
        // one instruction into a fresh register; -1 when the region is full
        auto push = [&](uint8_t op, int na, int a, int b, int c, uint8_t flag, const std::string &name) -> int {
            if (nreg >= RP_MAX_REG || n_insn >= RP_MAX_INSN) return -1;
            P.insn[n_insn++] = Insn{op, (uint8_t)nreg, (uint8_t)a, (uint8_t)b, (uint8_t)(na > 2 ? c : flag)};
            char buf[96];
            if (na > 2) snprintf(buf, sizeof buf, ";r%d=%s(r%d,r%d,r%d)", nreg, name.c_str(), a, b, c);
            else if (na > 1) snprintf(buf, sizeof buf, ";r%d=%s(r%d,r%d)", nreg, name.c_str(), a, b);
            else snprintf(buf, sizeof buf, ";r%d=%s(r%d)", nreg, name.c_str(), a);
            sig += buf;
            return nreg++;
        };
        // 64-bit words: the register holding i64 value `id` as an f64
        // (readAtF64), converted once at its first numeric use
        std::map<uint64_t, int> num_reg;
        auto num = [&](uint64_t id) -> int {
            if (vals[id].dtype != ZPUCUDA_I64) return reg[id];
            auto it = num_reg.find(id);
            if (it != num_reg.end()) return it->second;
            const int r = push(OPC_I2F, 1, reg[id], 0, 0, 0, "i2f");
            if (r >= 0) num_reg[id] = r;
            return r;
        };
        // scalar.binary / scalar.unary's integer operations on two i64
        // values (scalar.zig:262-302); the rest go through f64
        auto int_op = [](int prim) -> int {
            switch (prim) {
            case 35: return OPC_IADD;
            case 36: return OPC_ISUB;
            case 37: return OPC_IMUL;
            case 44: return OPC_IMOD;
            case 40: return OPC_IMAX;
            case 41: return OPC_IMIN;
            case 1: return OPC_IABS;
            case 31: return OPC_ISIGN;
            case 26: return OPC_IRELU;
            default: return -1;
            }
        };
        auto int_name = [](int op) -> const char * {
            switch (op) {
            case OPC_IADD: return "iadd";
            case OPC_ISUB: return "isub";
            case OPC_IMUL: return "imul";
            case OPC_IMOD: return "imod";
            case OPC_IMAX: return "imax";
            case OPC_IMIN: return "imin";
            case OPC_IABS: return "iabs";
            case OPC_ISIGN: return "isign";
            default: return "irelu";
            }
        };
        for (int m : member) {
            const zpucuda_step &st = steps[m];
            if (region_reduce(st.prim)) {
                has_red = true;
                red_prim = st.prim;
                red_axis = st.axis;
                red_depth = vals[st.ins[0]].depth;
                red_in = st.ins[0];
                red_out_id = st.out;
                continue;
            }
            const int n = st.n_inputs;
            int r = -1;
            if (!words64) {
                r = push((uint8_t)st.prim, n, reg[st.ins[0]], n > 1 ? reg[st.ins[1]] : 0, n > 2 ? reg[st.ins[2]] : 0, 0,
                         prim_name(st.prim));
            } else {
                const int odt = vals[st.out].dtype;
                bool all_i = true, any_i = false;
                for (int k = (st.prim == PRIM_WHERE ? 1 : 0); k < n; k++) {
                    const bool ik = vals[st.ins[k]].dtype == ZPUCUDA_I64;
                    all_i &= ik;
                    any_i |= ik;
                }
                const int iop = int_op(st.prim);
                if (odt == ZPUCUDA_I64 && all_i && iop >= 0) {
                    r = push((uint8_t)iop, n, reg[st.ins[0]], n > 1 ? reg[st.ins[1]] : 0, 0, 0, int_name(iop));
                } else {
                    // the step in f64 on f64 operands (where: ops.zig:572-590
                    // reads and writes through f64 too), or as an f32 region
                    // computes it when it is an f32 step of f32 / bool values;
                    // an f32 result of an i64 operand rounds once from f64
                    const bool f32_step = odt == ZPUCUDA_F32 && !any_i && st.prim != PRIM_WHERE;
                    int ops[3] = {0, 0, 0};
                    bool bad = false;
                    for (int k = 0; k < n; k++) bad |= (ops[k] = num(st.ins[k])) < 0;
                    if (!bad) {
                        if (st.prim == PRIM_POW && all_i) r = push(OPC_ZPOW, 2, ops[0], ops[1], 0, 0, "zpow");
                        else r = push((uint8_t)st.prim, n, ops[0], ops[1], ops[2], f32_step ? kInsnF32 : 0,
                                      prim_name(st.prim) + (f32_step ? ".f32" : ""));
                    }
                    if (r >= 0 && odt == ZPUCUDA_I64) r = push(OPC_F2I, 1, r, 0, 0, 0, "f2i");
                    else if (r >= 0 && odt == ZPUCUDA_F32 && any_i) r = push(OPC_R32, 1, r, 0, 0, 0, "r32");
                }
            }
            if (r < 0) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "region too long");
            reg[st.out] = r;
        }
        // the reduced value: i64 sum / prod / max / min on the integers,
        // anything else (argmax / argmin / any / all of i64 values) on f64
        int red_reg = -1, red_kind_int = 0;
        if (has_red) {
            const bool int_red = vals[red_in].dtype == ZPUCUDA_I64 &&
                                 (red_prim == PRIM_SUM || red_prim == PRIM_PROD || red_prim == PRIM_MAX_REDUCE ||
                                  red_prim == PRIM_MIN_REDUCE);
            red_kind_int = int_red;
            red_reg = int_red ? reg[red_in] : num(red_in);
            if (red_reg < 0) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "region too long");
        }
        (void)next_reg_after_loads;
        P.n_insn = n_insn;
        // element-wise values needed after this region
        for (int m : member) {
            const zpucuda_step &st = steps[m];
            if (region_reduce(st.prim)) continue;
            bool needed = out_index.count(st.out) > 0;
            for (int u : users[st.out])
                if (std::find(member.begin(), member.end(), u) == member.end()) needed = true;
            if (needed) {
                if (P.n_out >= RP_MAX_OUT) return lower_fail(plan, ZPUCUDA_ERR_NOT_SUPPORTED, "region has too many outputs");
                P.out_bool[P.n_out] = vals[st.out].dtype == ZPUCUDA_BOOL;
                P.out_i64[P.n_out] = vals[st.out].dtype == ZPUCUDA_I64;
                P.out_reg[P.n_out++] = reg[st.out];
                Slot sl = materialise(st.out);
                if (sl.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
                L.outs.push_back(sl);
            }
        }
        if (has_red) {
            P.reduce = red_prim == PRIM_SUM ? RED_SUM : red_prim == PRIM_PROD ? RED_PROD
                     : red_prim == PRIM_MAX_REDUCE ? RED_MAX : red_prim == PRIM_MIN_REDUCE ? RED_MIN
                     : red_prim == PRIM_ARGMAX ? RED_ARGMAX : red_prim == PRIM_ARGMIN ? RED_ARGMIN
                     : red_prim == PRIM_ANY ? RED_ANY : RED_ALL;
            if (red_kind_int) P.reduce += RED_ISUM - RED_SUM;  // the same kind on i64 words
            P.reduce_reg = red_reg;
            // the folded axes [r0, r1] split the region into [outer, red_len, inner]
            int r0 = 0, r1 = -1;
            reduced_axes(rshape, red_depth, red_axis, &r0, &r1);
            int64_t outer = 1, red_len = 1, inner = 1;
            for (int d = 0; d < rshape.rank; d++) {
                if (d < r0) outer *= rshape.dims[d];
                else if (d <= r1) red_len *= rshape.dims[d];
                else inner *= rshape.dims[d];
            }
            P.reduce_all = (outer == 1 && inner == 1) ? 1 : 0;
            if (P.reduce_all) {
                P.inner = P.numel;
                P.outer = 1;
            } else if (inner != 1) {  // an axis before the last: [outer, red_len, inner]
                P.reduce_mid = 1;
                P.red_len = red_len;
                P.outer = outer;
                P.inner = inner;
            } else {  // the trailing axes: rows of red_len
                P.inner = red_len;
                P.outer = outer;
            }
            L.has_red = true;
            L.red = materialise(red_out_id);
            if (L.red.index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "intermediate allocation");
            char buf[64];
            snprintf(buf, sizeof buf, ";out=r%d;red=%s%s%s", P.reduce_reg, red_kind_int ? "i" : "",
                     red_prim == PRIM_SUM ? "sum" : red_prim == PRIM_PROD ? "prod" : red_prim == PRIM_MAX_REDUCE ? "max"
                     : red_prim == PRIM_MIN_REDUCE ? "min" : red_prim == PRIM_ARGMAX ? "argmax"
                     : red_prim == PRIM_ARGMIN ? "argmin" : red_prim == PRIM_ANY ? "any" : "all",
                     P.reduce_all ? "" : P.reduce_mid ? "_axis" : "_rows");
            sig += buf;
            if (P.reduce_all) {
                void *w = nullptr;
                if (cudaMalloc(&w, kRegionWorkspaceBytes) != cudaSuccess || cudaMemset(w, 0, kRegionWorkspaceBytes) != cudaSuccess) {
                    cudaGetLastError();
                    return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "region workspace");
                }
                plan->workspaces.push_back(w);
                L.workspace = w;
            }
        } else {
            char buf[64];
            snprintf(buf, sizeof buf, ";out=r%d;red=none", P.n_out == 1 ? P.out_reg[0] : -1);
            sig += buf;
        }
        L.signature = sig;
        bool any_bool = false;
        for (int k = 0; k < P.n_in; k++) any_bool |= P.in_bool[k] != 0 || P.in_i64[k] != 0;
        for (int o = 0; o < P.n_out; o++) any_bool |= P.out_bool[o] != 0 || P.out_i64[o] != 0;
        const bool catalogue_shape = ((!has_red && P.n_out == 1) || (has_red && P.reduce == RED_SUM && P.reduce_all && P.n_out == 0)) &&
                                     kinds.find_first_of("RG") == std::string::npos && !any_bool;
        L.cat = catalogue_shape ? catalogue_find(sig.c_str()) : nullptr;
        L.text = "  kernel " + std::to_string(plan->launches.size()) + ": region " +
                 (L.cat ? std::string("[catalogue ") + L.cat->name + "]" : std::string("[bytecode]")) + " " + sig + "\n";
        plan->launches.push_back(L);
        s = member.back() + 1;
    }
    // outputs that are views, arguments, constants, or listed twice: copied
    // into their output buffers after everything else
    for (int i = 0; i < n_outs; i++) {
        Value &v = vals[out_ids[i]];
        if (!v.materialised) return lower_fail(plan, ZPUCUDA_ERR_SHAPE_MISMATCH, "output not computed");
        if (v.slot.kind == SLOT_OUT && v.slot.index == i && v.offset == 0 && v.contiguous()) continue;
        if (copy_launch(v, Slot{SLOT_OUT, i}, "plan output").index < 0) return lower_fail(plan, ZPUCUDA_ERR_OUT_OF_MEMORY, "copy");
    }
    char head[160];
    snprintf(head, sizeof head, "plan: %d steps -> %zu kernels\n", n_steps, plan->launches.size());
    plan->text = head;
    for (auto &L : plan->launches) plan->text += L.text;
    *out = plan;
    return ZPUCUDA_OK;
}

int zpucuda_plan_run(zpucuda_plan *plan, const void *const *args, void *const *outs, void *stream) {
    ZC_CHECK(plan && (args || !plan->n_args) && outs, ZPUCUDA_ERR_INVALID_ARGUMENT);
    cudaStream_t s = resolve_stream(stream);
    auto ptr = [&](const Slot &sl) -> void * {
        switch (sl.kind) {
        case SLOT_ARG: return (void *)args[sl.index];
        case SLOT_BLOB: return plan->blobs[sl.index];
        case SLOT_OUT: return outs[sl.index];
        default: return plan->temps[sl.index];
        }
    };
    for (auto &L : plan->launches) {
        int st;
        if (L.kind == Launch::MATMUL) {
            zpucuda_tensor a = L.ta, b = L.tb, c = L.tc;
            a.data = (char *)ptr(L.ma) + L.ma_off;
            b.data = (char *)ptr(L.mb) + L.mb_off;
            c.data = ptr(L.mc);
            if (L.epi_mode) {
                Epilogue e;
                e.mode = L.epi_mode;
                e.bias = (const float *)((char *)ptr(L.bias) + L.bias_off);
                st = matmul_device_epi(&a, &b, &c, e, s);
            } else {
                st = matmul_device(&a, &b, &c, s);
            }
        } else if (L.kind == Launch::CUMSUM) {
            st = cumsum_launch(L.dtype, (char *)ptr(L.ma) + L.ma_off, ptr(L.mc), L.outer, L.dim, L.inner, L.reverse, s);
        } else if (L.kind == Launch::COPYV) {
            zpucuda_tensor a = L.src, c = L.dst;
            a.data = (char *)ptr(L.ma) + L.ma_off;
            c.data = (char *)ptr(L.mc) + L.mc_off;
            st = copy_view(a, c, s);
        } else if (L.kind == Launch::FILL) {
            st = fill_value(L.dtype, ptr(L.mc), L.k, L.scalar, s);
        } else if (L.kind == Launch::TAKE) {
            st = take_launch(L.dtype, (char *)ptr(L.ma) + L.ma_off, L.idx_dtype, (char *)ptr(L.mb) + L.mb_off,
                             ptr(L.mc), L.outer, L.dim, L.inner, L.k, plan->err, s);
        } else if (L.kind == Launch::SCATTER) {
            st = scatter_add_launch(L.dtype, L.idx_dtype, (char *)ptr(L.mb) + L.mb_off, (char *)ptr(L.ma) + L.ma_off,
                                    ptr(L.mc), L.outer, L.dim, L.inner, L.k, plan->err, s);
        } else if (L.kind == Launch::COPY) {
            zpucuda_tensor a = L.src, c = L.src;
            a.data = (char *)ptr(L.ma) + L.ma_off;
            c.data = ptr(L.mc);
            c.dtype = L.dst_dtype;
            st = zpucuda_tensor_copy(&a, &c, s);
        } else {
            RegionIO io;
            memset(&io, 0, sizeof io);
            for (size_t k = 0; k < L.ins.size(); k++) io.in[k] = (char *)ptr(L.ins[k]) + L.in_off[k];
            for (size_t o = 0; o < L.outs.size(); o++) io.out[o] = ptr(L.outs[o]);
            if (L.has_red) io.red_out = ptr(L.red);
            if (L.workspace) {
                io.ticket = (unsigned int *)L.workspace;
                io.error = (unsigned int *)L.workspace + 1;
                io.partials = (double *)((char *)L.workspace + 256);
            }
            st = region_launch(L.prog, L.cat, io, s);
        }
        if (st) return st;
    }
    return ZPUCUDA_OK;
}

// The plan's device error words, read and cleared once the stream has
// drained: the take / scatter_add index-error word (IndexOutOfRange), and the
// error word of every full-reduction workspace, which a region kernel sets
// when one of its bounded waits runs out (its sum is then NaN): Timeout.
static int plan_device_errors(zpucuda_plan *plan) {
    bool timed_out = false;
    for (void *w : plan->workspaces) {
        unsigned int e = 0;
        ZC_CUDA(cudaMemcpy(&e, (unsigned int *)w + 1, sizeof e, cudaMemcpyDeviceToHost));
        if (e) {
            ZC_CUDA(cudaMemset((unsigned int *)w + 1, 0, sizeof e));
            timed_out = true;
        }
    }
    unsigned int idx = 0;
    if (plan->err) {
        ZC_CUDA(cudaMemcpy(&idx, plan->err, sizeof idx, cudaMemcpyDeviceToHost));
        if (idx) ZC_CUDA(cudaMemset(plan->err, 0, sizeof idx));
    }
    if (timed_out)
        return set_error(ZPUCUDA_ERR_TIMEOUT, "a fused reduction's bounded wait for its input copies ran out (its result is NaN)");
    if (idx) return set_error(ZPUCUDA_ERR_INDEX_OUT_OF_RANGE, "a take / scatter_add index was out of range (ops.take)");
    return ZPUCUDA_OK;
}

static size_t value_bytes(const zpucuda_value &v) {
    size_t n = 1;
    for (int d = 0; d < v.rank; d++) n *= (size_t)v.dims[d];
    return n * itemsize(v.dtype);
}

int zpucuda_plan_run_host(zpucuda_plan *plan, const void *const *host_args, void *const *host_outs, void *stream) {
    ZC_CHECK(plan && (host_args || !plan->n_args) && host_outs, ZPUCUDA_ERR_INVALID_ARGUMENT);
    cudaStream_t s = resolve_stream(stream);
    if (plan->stage_in.size() != plan->arg_values.size() || plan->stage_out.size() != plan->outputs.size()) {
        for (auto &v : plan->arg_values) {
            void *d = nullptr;
            ZC_CUDA(cudaMalloc(&d, value_bytes(v) ? value_bytes(v) : 16));
            plan->stage_in.push_back(d);
        }
        for (auto &v : plan->outputs) {
            void *d = nullptr;
            ZC_CUDA(cudaMalloc(&d, value_bytes(v) ? value_bytes(v) : 16));
            plan->stage_out.push_back(d);
        }
    }
    for (size_t i = 0; i < plan->arg_values.size(); i++) {
        const size_t nb = value_bytes(plan->arg_values[i]);
        if (nb) ZC_CUDA(cudaMemcpyAsync(plan->stage_in[i], host_args[i], nb, cudaMemcpyHostToDevice, s));
    }
    int st = zpucuda_plan_run(plan, (const void *const *)plan->stage_in.data(), plan->stage_out.data(), s);
    if (st) return st;
    for (size_t i = 0; i < plan->outputs.size(); i++) {
        const size_t nb = value_bytes(plan->outputs[i]);
        if (nb) ZC_CUDA(cudaMemcpyAsync(host_outs[i], plan->stage_out[i], nb, cudaMemcpyDeviceToHost, s));
    }
    // bounded wait on this stream
    for (int64_t spins = 0;; spins++) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return plan_device_errors(plan);
        if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
        if (spins > 60LL * 1000 * 100) return set_error(ZPUCUDA_ERR_TIMEOUT, "zpucuda_plan_run_host: stream did not drain");
        if (spins > 1000) usleep(10);
    }
}

int zpucuda_plan_check(zpucuda_plan *plan, void *stream) {
    ZC_CHECK(plan, ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (!plan->err && plan->workspaces.empty()) return ZPUCUDA_OK;
    cudaStream_t s = resolve_stream(stream);
    for (int64_t spins = 0;; spins++) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return plan_device_errors(plan);
        if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
        if (spins > 60LL * 1000 * 100) return set_error(ZPUCUDA_ERR_TIMEOUT, "zpucuda_plan_check: stream did not drain");
        if (spins > 1000) usleep(10);
    }
}

int zpucuda_plan_output(const zpucuda_plan *plan, int i, zpucuda_value *value) {
    ZC_CHECK(plan && value, ZPUCUDA_ERR_INVALID_ARGUMENT);
    ZC_CHECK(i >= 0 && i < (int)plan->outputs.size(), ZPUCUDA_ERR_INDEX_OUT_OF_RANGE);
    *value = plan->outputs[i];
    return ZPUCUDA_OK;
}

int zpucuda_plan_num_steps(const zpucuda_plan *plan) { return plan ? plan->n_steps : -1; }
int zpucuda_plan_num_kernels(const zpucuda_plan *plan) { return plan ? (int)plan->launches.size() : -1; }

int zpucuda_plan_describe(const zpucuda_plan *plan, char *buf, size_t len) {
    ZC_CHECK(plan && buf && len, ZPUCUDA_ERR_INVALID_ARGUMENT);
    snprintf(buf, len, "%s", plan->text.c_str());
    return ZPUCUDA_OK;
}

void zpucuda_plan_destroy(zpucuda_plan *plan) { delete plan; }

}  // extern "C"
