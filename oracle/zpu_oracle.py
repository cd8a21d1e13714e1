"""ctypes front end of the CPU oracle (liboracle.so, built from zpu_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
import this module.  The product library (zpu_b200 / libzpucuda.so) never
does, and has no CPU fallback.

Also restates the shape logic of zpu's `ops.matmul` (src/zpu/ops.zig:1062-1205)
in Python, so a batched/broadcast/vmapped matmul can be checked end to end.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

# src/zpu/prims.zig:9-109 element-wise codes (the first 32 unary, then binary)
PRIM = {
    "neg": 0, "abs": 1, "exp": 2, "expm1": 3, "log": 4, "log1p": 5, "sqrt": 6, "rsqrt": 7,
    "square": 8, "recip": 9, "cbrt": 10, "sin": 11, "cos": 12, "tan": 13, "asin": 14,
    "acos": 15, "atan": 16, "sinh": 17, "cosh": 18, "tanh": 19, "asinh": 20, "acosh": 21,
    "atanh": 22, "erf": 23, "sigmoid": 24, "softplus": 25, "relu": 26, "floor": 27,
    "ceil": 28, "round": 29, "trunc": 30, "sign": 31,
    "add": 35, "sub": 36, "mul": 37, "div": 38, "pow": 39, "maximum": 40, "minimum": 41,
    "atan2": 42, "hypot": 43, "mod_op": 44,
}

_lib = None


def build():
    """Compiles liboracle.so with the committed Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    src = os.path.join(HERE, "zpu_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        build()
    L = C.CDLL(LIB_PATH)
    P, S, D, F, I64 = C.c_void_p, C.c_size_t, C.c_double, C.c_float, C.c_int64
    sig = {
        "zo_rng_next": (C.c_uint64, [P]),
        "zo_rng_next_f64": (D, [P]),
        "zo_uniform_range_f64": (None, [C.c_uint64, P, S, D, D]),
        "zo_uniform_range_f32": (None, [C.c_uint64, P, S, D, D]),
        "zo_normal_f64": (None, [C.c_uint64, P, S]),
        "zo_normal_f32": (None, [C.c_uint64, P, S]),
        "zo_randint_i64": (C.c_int, [C.c_uint64, P, S, I64, I64]),
        "zo_gemm_f32": (None, [P, P, P, S, S, S]),
        "zo_gemm_f64": (None, [P, P, P, S, S, S]),
        "zo_gemm_batched_f32": (None, [P, P, P, S, S, S, C.c_int, P, P, P]),
        "zo_gemm_batched_f64": (None, [P, P, P, S, S, S, C.c_int, P, P, P]),
        "zo_reduce_sum_f32": (F, [P, S]),
        "zo_reduce_sum_f64": (D, [P, S]),
        "zo_reduce_maxmin_f32": (F, [P, S, C.c_int]),
        "zo_sum_f64_of_f32": (D, [P, S]),
        "zo_abssum_f64_of_f32": (D, [P, S]),
        "zo_unary_f32": (F, [C.c_int, F]),
        "zo_unary_f64": (D, [C.c_int, D]),
        "zo_binary_f32": (F, [C.c_int, F, F]),
        "zo_binary_f64": (D, [C.c_int, D, D]),
        "zo_set_cores": (None, [S]),
        "zo_worker_count": (S, [S]),
        "zo_jit_chain_tanh_sq_affine_sum": (F, [P, S, F, F, P, P]),
        "zo_pow": (D, [D, D]),
        "zo_adam_step_f32": (None, [P, P, P, P, S, C.c_long, D, D, D, D]),
        "zo_adam_step_f64": (None, [P, P, P, P, S, C.c_long, D, D, D, D]),
        "zo_mlp_loss_grad": (F, [P, P, S, S, S, S, S] + [P] * 12),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


# --------------------------------------------------------------------------- rng
def uniform_range(seed, n, lo, hi, dtype=np.float32):
    out = np.empty(n, dtype=dtype)
    f = lib().zo_uniform_range_f32 if dtype == np.float32 else lib().zo_uniform_range_f64
    f(seed, _p(out), n, lo, hi)
    return out


def normal(seed, n, dtype=np.float32):
    out = np.empty(n, dtype=dtype)
    f = lib().zo_normal_f32 if dtype == np.float32 else lib().zo_normal_f64
    f(seed, _p(out), n)
    return out


def randint(seed, n, lo, hi):
    out = np.empty(n, dtype=np.int64)
    if lib().zo_randint_i64(seed, _p(out), n, lo, hi) != 0:
        raise ValueError("randint: high <= low")
    return out


# -------------------------------------------------------------------------- gemm
def gemm(a, b):
    """kernels.gemm on contiguous row-major 2-D arrays (bit-exact with zpu)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2 and a.dtype == b.dtype
    d = np.empty((m, n), dtype=a.dtype)
    f = lib().zo_gemm_f32 if a.dtype == np.float32 else lib().zo_gemm_f64
    f(_p(a), _p(b), _p(d), m, k, n)
    return d


def gemm_batched(a, b, m, k, n, dims, acs, bcs):
    """ops.gemmBatched: flat contiguous buffers, batch axes `dims` with element
    strides `acs`/`bcs` (0 = broadcast)."""
    total = int(np.prod(dims)) if len(dims) else 1
    d = np.empty(total * m * n, dtype=a.dtype)
    dims_ = np.asarray(dims, dtype=np.int64)
    acs_ = np.asarray(acs, dtype=np.int64)
    bcs_ = np.asarray(bcs, dtype=np.int64)
    f = lib().zo_gemm_batched_f32 if a.dtype == np.float32 else lib().zo_gemm_batched_f64
    f(_p(a), _p(b), _p(d), m, k, n, len(dims), _p(dims_), _p(acs_), _p(bcs_))
    return d


def matmul(a, b, a_depth=0, b_depth=0):
    """ops.matmul (ops.zig:1062-1205) with NumPy semantics and vmap depth:
    leading `depth` axes are vmap axes; 1-D operands are promoted and the
    added axis squeezed; payload batch axes broadcast right-aligned."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    depth = max(a_depth, b_depth)
    # withVmapDepth (ops.zig:1211-1224): lead with size-1 stride-0 axes
    if a_depth < depth:
        a = a.reshape((1,) * (depth - a_depth) + a.shape)
    if b_depth < depth:
        b = b.reshape((1,) * (depth - b_depth) + b.shape)
    prep_a = a.ndim - depth == 1
    prep_b = b.ndim - depth == 1
    if prep_a:
        a = np.expand_dims(a, depth)
    if prep_b:
        b = np.expand_dims(b, b.ndim)
    m, k = a.shape[-2:]
    k2, n = b.shape[-2:]
    if k != k2:
        raise ValueError("ShapeMismatch")
    a_nba, b_nba = a.ndim - 2 - depth, b.ndim - 2 - depth
    nb = max(a_nba, b_nba)
    adims = [1] * (nb - a_nba) + list(a.shape[depth:depth + a_nba])
    bdims = [1] * (nb - b_nba) + list(b.shape[depth:depth + b_nba])
    cdims = []
    for x, y in zip(adims, bdims):
        if x == y or y == 1:
            cdims.append(x)
        elif x == 1:
            cdims.append(y)
        else:
            raise ValueError("ShapeMismatch")
    lead = [max(a.shape[i], b.shape[i]) for i in range(depth)]
    ast = [s // a.itemsize for s in a.strides]
    bst = [s // b.itemsize for s in b.strides]
    gdims, acs, bcs = [], [], []
    for i in range(depth):
        gdims.append(lead[i])
        acs.append(ast[i] if a.shape[i] == lead[i] else 0)
        bcs.append(bst[i] if b.shape[i] == lead[i] else 0)
    for i in range(nb):
        gdims.append(cdims[i])
        aj, bj = i - (nb - a_nba), i - (nb - b_nba)
        acs.append(ast[aj + depth] if aj >= 0 and adims[i] == cdims[i] else 0)
        bcs.append(bst[bj + depth] if bj >= 0 and bdims[i] == cdims[i] else 0)
    out = gemm_batched(a.ravel(), b.ravel(), m, k, n, gdims, acs, bcs)
    out = out.reshape(tuple(lead) + tuple(cdims) + (m, n))
    if prep_a:
        out = np.squeeze(out, axis=out.ndim - 2)
    if prep_b:
        out = np.squeeze(out, axis=out.ndim - 1)
    return out


def promote(a, b):
    """DType.promote (src/zpu/dtype.zig:89-104) on numpy dtypes: floats win,
    the wider float wins; mixed signedness takes the wider integer (the
    second on a tie), otherwise the wider (the first on a tie)."""
    a, b = np.dtype(a), np.dtype(b)
    if a == b:
        return a
    fa, fb = a.kind == "f", b.kind == "f"
    if fa and not fb:
        return a
    if fb and not fa:
        return b
    if fa and fb:
        return a if a.itemsize >= b.itemsize else b
    sa, sb = a.kind == "i", b.kind == "i"
    if sa != sb:
        return a if a.itemsize > b.itemsize else b
    return a if a.itemsize >= b.itemsize else b


def gemm_convert(a, b):
    """ops.matmul of two row-major [.., m, k] @ [.., k, n] arrays whose types
    are not both f32 or both f64 (same leading batch shape):
     - same-type integers: ops.gemmTyped's loop (src/zpu/ops.zig:1016-1049),
       the element type's wrapping sums (reduceStep, ops.zig:685-688);
     - otherwise ops.gemmF64 (ops.zig:1284-1333): the output, of type
       promote(a, b), starts at 0 and for p = 0 .. k-1 in order becomes
       fromF64(toF64(out) + toF64(a[.., i, p]) * toF64(b[.., p, j])), the
       product and the sum in f64 with no fused multiply-add.
    A bool result (bool @ bool) is zpu's DTypeMismatch."""
    a, b = np.asarray(a), np.asarray(b)
    out_dt = promote(a.dtype, b.dtype)
    if out_dt == np.bool_:
        raise ValueError("DTypeMismatch")
    k = a.shape[-1]
    if a.dtype == b.dtype and a.dtype.kind in "iu":
        prod = np.matmul(a.astype(np.int64), b.astype(np.int64))  # wraps modulo 2^64
        return prod.astype(out_dt)  # and modulo 2^bits
    af, bf = to_f64(a), to_f64(b)
    acc = np.zeros(a.shape[:-1] + (b.shape[-1],), dtype=out_dt)
    for p in range(k):
        step = acc.astype(np.float64) + af[..., :, p:p + 1] * bf[..., p:p + 1, :]
        acc = from_f64(step, out_dt)
    return acc


# --------------------------------------------------------------- elementwise/sum
def unary(prim, x):
    L = lib()
    code = PRIM[prim]
    x = np.asarray(x)
    if x.dtype == np.float32:
        return np.array([L.zo_unary_f32(code, float(v)) for v in x.ravel()], dtype=np.float32).reshape(x.shape)
    return np.array([L.zo_unary_f64(code, float(v)) for v in x.ravel()], dtype=np.float64).reshape(x.shape)


def binary(prim, a, b):
    L = lib()
    code = PRIM[prim]
    a, b = np.broadcast_arrays(np.asarray(a), np.asarray(b))
    if a.dtype == np.float32:
        f, dt = L.zo_binary_f32, np.float32
    else:
        f, dt = L.zo_binary_f64, np.float64
    return np.array([f(code, float(x), float(y)) for x, y in zip(a.ravel(), b.ravel())], dtype=dt).reshape(a.shape)


def reduce_sum(x):
    """kernels.reduceAll(.sum) in zpu's exact accumulation order."""
    x = np.ascontiguousarray(x).ravel()
    if x.dtype == np.float32:
        return np.float32(lib().zo_reduce_sum_f32(_p(x), x.size))
    return np.float64(lib().zo_reduce_sum_f64(_p(x), x.size))


def reduce_max(x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.float32(lib().zo_reduce_maxmin_f32(_p(x), x.size, 1))


AXIS_NONE = -2


def reduced_axes(ndim, axis, depth=0):
    """ops.axesMaskOf (src/zpu/ops.zig:630-642) as a tuple of axes: AXIS_NONE
    folds the payload axes [depth, ndim); a non-negative axis counts from the
    first payload axis, a negative one from the last."""
    if axis == AXIS_NONE:
        return tuple(range(min(depth, ndim), ndim))
    a = axis + depth if axis >= 0 else axis + ndim
    if a < 0 or a >= ndim:
        raise ValueError("InvalidAxis")
    return (a,)


def arg_reduce(x, axis=AXIS_NONE, depth=0, want_max=True):
    """ops.argReduce (src/zpu/ops.zig:931-975): the reduced elements of each
    output are visited in row order; the first seeds `best`, a later one
    replaces it only when strictly greater (argmax) / smaller (argmin), so
    ties keep the first index and a NaN never replaces (a NaN first element
    pins the answer to 0).  Values compare as f64 (readF64).  Returns i64 with
    the folded axes dropped."""
    x = np.asarray(x).astype(np.float64)
    axes = reduced_axes(x.ndim, axis, depth)
    keep = [d for d in range(x.ndim) if d not in axes]
    y = np.transpose(x, keep + list(axes))  # folded axes last, in row order
    out_shape = tuple(x.shape[d] for d in keep)
    y = y.reshape(out_shape + (-1,))
    n = y.shape[-1]
    best = np.zeros(out_shape)
    idx = np.zeros(out_shape, dtype=np.int64)
    for k in range(n):
        v = y[..., k]
        if k == 0:
            better = np.ones(out_shape, dtype=bool)
        else:
            with np.errstate(invalid="ignore"):
                better = v > best if want_max else v < best
        best = np.where(better, v, best)
        idx = np.where(better, k, idx)
    return idx


def reduce_axis(x, prim, axis=AXIS_NONE, keepdims=False, depth=0):
    """ops.reduceOp (src/zpu/ops.zig:820-869) for sum / prod / max / min over
    the axes axesMaskOf gives, as an f64 reference (order-free; the
    tolerances of the tests that use it cover the summation order)."""
    x = np.asarray(x).astype(np.float64)
    axes = reduced_axes(x.ndim, axis, depth)
    fn = {"sum": np.sum, "prod_op": np.prod, "max_reduce": np.max, "min_reduce": np.min}[prim]
    return fn(x, axis=axes, keepdims=bool(keepdims))


def mean(x, axis=AXIS_NONE, keepdims=False, depth=0):
    """ops.mean (src/zpu/ops.zig:894-908): sum, then times 1/count."""
    x = np.asarray(x).astype(np.float64)
    axes = reduced_axes(x.ndim, axis, depth)
    count = int(np.prod([x.shape[a] for a in axes])) if axes else 1
    return reduce_axis(x, "sum", axis, keepdims, depth) * (1.0 / count)


def variance(x, axis=AXIS_NONE, keepdims=False, depth=0):
    """ops.variance (src/zpu/ops.zig:914-922): mean(square(x - mean(x, keep)))."""
    m = mean(x, axis, True, depth)
    return mean(np.square(np.asarray(x, dtype=np.float64) - m), axis, keepdims, depth)


def predicate(prim, a, b=None):
    """The predicates on f64 values (scalar.pred1F / pred2F,
    src/zpu/scalar.zig:235-259; logicalNot is eq(a, 0), ops.zig:516-520):
    comparisons by IEEE rules, logical ops on truthiness v != 0 (NaN is
    true).  Returns bool with numpy broadcasting."""
    a = np.asarray(a).astype(np.float64)
    if prim == "isnan":
        return np.isnan(a)
    if prim == "isinf":
        return np.isinf(a)
    if prim == "isfinite":
        return np.isfinite(a)
    if prim == "logical_not":
        return a == 0
    b = np.asarray(b).astype(np.float64)
    with np.errstate(invalid="ignore"):
        return {"eq": np.equal, "ne": np.not_equal, "lt": np.less, "le": np.less_equal, "gt": np.greater,
                "ge": np.greater_equal,
                "logical_and": lambda x, y: (x != 0) & (y != 0),
                "logical_or": lambda x, y: (x != 0) | (y != 0),
                "logical_xor": lambda x, y: (x != 0) != (y != 0)}[prim](a, b)


def where(cond, a, b):
    """ops.where (src/zpu/ops.zig:572-590): a where cond != 0 (NaN is true),
    else b, all three broadcast."""
    return np.where(np.asarray(cond).astype(np.float64) != 0, a, b)


def reduce_bool(x, kind, axis=AXIS_NONE, keepdims=False, depth=0):
    """ops.any / ops.all (src/zpu/ops.zig:883-888, 838-853): the reduction of
    x != 0 over the axes axesMaskOf gives; empty axes give false / true."""
    t = np.asarray(x).astype(np.float64) != 0
    axes = reduced_axes(t.ndim, axis, depth)
    fn = np.any if kind == "any_reduce" else np.all
    return fn(t, axis=axes, keepdims=bool(keepdims))


def cumsum(x, axis, reverse=False, depth=0):
    """ops.cumsum (src/zpu/ops.zig:2032-2060): along ops.realAxis (a
    non-negative axis counts from the first payload axis, no AXIS_NONE), a
    running f64 sum, each prefix written into x's type as writeF64 writes it
    (rounded for floats, scalar.fromF64 for i64); `reverse` from the end."""
    x = np.asarray(x)
    ax = axis + depth if axis >= 0 else axis + x.ndim
    if ax < 0 or ax >= x.ndim:
        raise ValueError("InvalidAxis")
    v = np.moveaxis(x.astype(np.float64), ax, -1)
    if reverse:
        v = v[..., ::-1]
    acc = np.zeros(v.shape[:-1])
    out = np.empty_like(v)
    for d in range(v.shape[-1]):  # sequential, as zpu adds
        acc = acc + v[..., d]
        out[..., d] = acc
    if reverse:
        out = out[..., ::-1]
    return from_f64(np.moveaxis(out, -1, ax), x.dtype)  # writeF64


# zpu DType order (src/zpu/dtype.zig:4-13) as numpy types
DTYPES = [np.float64, np.float32, np.float16, np.int64, np.int32, np.int16, np.int8, np.uint8, np.bool_]


def to_f64(x):
    """scalar.toF64 (src/zpu/scalar.zig:7-15) element-wise."""
    return np.asarray(x).astype(np.float64)


def from_f64(v, dt):
    """scalar.fromF64 (src/zpu/scalar.zig:17-27) element-wise: floats round to
    nearest, bool is v != 0, an integer type takes 0 for NaN, else clamps to
    [minInt, maxInt] (as f64) and truncates toward zero.  For i64 the clamp
    bound (f64)maxInt = 2^63 is out of range (undefined in Zig); the device
    saturates it to maxInt, and so does this restatement."""
    v = np.asarray(v, dtype=np.float64)
    dt = np.dtype(dt)
    if dt.kind == "f":
        with np.errstate(over="ignore"):
            return v.astype(dt)
    if dt.kind == "b":
        return v != 0
    info = np.iinfo(dt)
    nan = np.isnan(v)
    c = np.clip(np.where(nan, 0.0, v), float(info.min), float(info.max))
    t = np.trunc(c)
    if dt == np.int64:
        top = t >= 2.0 ** 63
        out = np.where(top, 0.0, t).astype(np.int64)
        out[top] = info.max
        return out
    return t.astype(dt)


# ------------------------------------------------------------ i64 values
I64_INT_BINARY = ("add", "sub", "mul", "mod_op", "maximum", "minimum")
I64_INT_UNARY = ("abs", "sign", "relu")


def binary_i64(prim, a, b):
    """scalar.binary(i64, p, a, b) (src/zpu/scalar.zig:285-302) for two i64
    operands whose result type is i64: + - * on the integers (two's-complement
    wrap where zpu's own would overflow), mod with a zero divisor giving a and
    @mod's sign of the divisor otherwise, max / min; every other prim is the
    f64 computation of the operands read as f64, written back by fromF64."""
    a, b = np.broadcast_arrays(np.asarray(a, dtype=np.int64), np.asarray(b, dtype=np.int64))
    if prim in I64_INT_BINARY:
        with np.errstate(over="ignore"):
            if prim == "add":
                return a + b
            if prim == "sub":
                return a - b
            if prim == "mul":
                return a * b
            if prim == "maximum":
                return np.maximum(a, b)
            if prim == "minimum":
                return np.minimum(a, b)
        safe = np.where((b == 0) | (b == -1), 1, b)
        return np.where(b == 0, a, np.where(b == -1, 0, np.mod(a, safe)))
    return from_f64(binary(prim, to_f64(a), to_f64(b)), np.int64)


def unary_i64(prim, x):
    """scalar.unary(i64, p, x) (src/zpu/scalar.zig:262-283): relu, abs and
    sign on the integer; the rest through f64 and fromF64."""
    x = np.asarray(x, dtype=np.int64)
    if prim == "abs":
        with np.errstate(over="ignore"):
            return np.where(x < 0, -x, x)
    if prim == "sign":
        return np.sign(x).astype(np.int64)
    if prim == "relu":
        return np.where(x > 0, x, 0).astype(np.int64)
    return from_f64(unary(prim, to_f64(x)), np.int64)


def where_i64(cond, a, b):
    """ops.where with two i64 branches (src/zpu/ops.zig:572-590): both read
    as f64, the chosen one written back into an i64 by fromF64."""
    return from_f64(np.where(to_f64(cond) != 0, to_f64(a), to_f64(b)), np.int64)


def reduce_i64(x, prim, axis=AXIS_NONE, keepdims=False, depth=0):
    """ops.reduceOp of an i64 tensor (src/zpu/ops.zig:662-700, 820-869): sum
    and prod wrap in the integer type (+%, *%), max / min on the integers;
    an empty reduction gives the identity zpu writes through fromF64 (0, 1,
    minInt for -inf, maxInt for +inf)."""
    x = np.asarray(x, dtype=np.int64)
    axes = reduced_axes(x.ndim, axis, depth)
    with np.errstate(over="ignore"):
        if prim == "sum":
            return np.sum(x, axis=axes, keepdims=bool(keepdims), dtype=np.int64)
        if prim == "prod_op":
            return np.prod(x, axis=axes, keepdims=bool(keepdims), dtype=np.int64)
    info = np.iinfo(np.int64)
    if prim == "max_reduce":
        return np.max(x, axis=axes, keepdims=bool(keepdims), initial=info.min)
    return np.min(x, axis=axes, keepdims=bool(keepdims), initial=info.max)


def tensor_copy(x, dt):
    """Tensor.clone / toContiguous / ops.cast (src/zpu/tensor.zig:356-404,
    src/zpu/ops.zig:2062-2071): writeF64(i, readLogical(n, i)) for every i
    of the logical order -- a numpy view gives that order itself."""
    return from_f64(to_f64(np.ascontiguousarray(x)), dt)


def sum_f64(x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return lib().zo_sum_f64_of_f32(_p(x), x.size)


def abssum_f64(x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return lib().zo_abssum_f64_of_f32(_p(x), x.size)


def set_cores(n):
    lib().zo_set_cores(n)


def worker_count(n):
    return lib().zo_worker_count(n)


def jit_chain_tanh_sq_affine_sum(x, a, b, want_vector=False):
    """y = sumAll(tanh(x*x)*a + b) as jit.Plan.runAll runs it on the CPU.
    Returns (zpu's f32 sum, f64 sum of the same vector, vector or None)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    t = np.empty_like(x) if want_vector else None
    s64 = C.c_double(0.0)
    s = lib().zo_jit_chain_tanh_sq_affine_sum(_p(x), x.size, a, b, _p(t) if t is not None else None,
                                              C.byref(s64))
    return np.float32(s), s64.value, t


# -------------------------------------------------------------------------- adam
def pow_(x, y):
    return lib().zo_pow(x, y)


class Adam:
    """optim.Adam (optim.zig:149-259) with f32 moment state."""

    def __init__(self, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8):
        self.lr, self.beta1, self.beta2, self.eps = lr, beta1, beta2, eps
        self.t = 0
        self.m = None
        self.v = None

    def step(self, params, grads):
        if self.m is None:
            self.m = [np.zeros(p.size, dtype=np.float32) for p in params]
            self.v = [np.zeros(p.size, dtype=np.float32) for p in params]
        self.t += 1
        for p, g, m, v in zip(params, grads, self.m, self.v):
            assert p.flags.c_contiguous and g.flags.c_contiguous
            f = lib().zo_adam_step_f32 if p.dtype == np.float32 else lib().zo_adam_step_f64
            f(_p(p), _p(g), _p(m), _p(v), p.size, self.t, self.lr, self.beta1, self.beta2, self.eps)


# --------------------------------------------------------------------------- mlp
XAVIER_SEED0 = 0x5EED0010


def mlp_init(dims, seed0=XAVIER_SEED0):
    """Xavier-uniform W_l ~ U(-sqrt(6/(in+out)), +sqrt(6/(in+out))) seeded
    seed0 + l (rng.zig:46 uniformRange), zero biases."""
    params = []
    for l in range(len(dims) - 1):
        fin, fout = dims[l], dims[l + 1]
        lim = (6.0 / (fin + fout)) ** 0.5
        W = uniform_range(seed0 + l, fin * fout, -lim, lim).reshape(fin, fout)
        params += [W, np.zeros(fout, dtype=np.float32)]
    return params


def mlp_loss_grad(X, labels, params):
    """Loss and gradients of dense->tanh->dense->tanh->dense->sparseCrossEntropy."""
    W1, b1, W2, b2, W3, b3 = params
    B, d0 = X.shape
    d1, d2, d3 = W1.shape[1], W2.shape[1], W3.shape[1]
    grads = [np.empty_like(p) for p in params]
    X = np.ascontiguousarray(X, dtype=np.float32)
    labels = np.ascontiguousarray(labels, dtype=np.int64)
    loss = lib().zo_mlp_loss_grad(_p(X), _p(labels), B, d0, d1, d2, d3,
                                  *[_p(p) for p in params], *[_p(g) for g in grads])
    return np.float32(loss), grads
