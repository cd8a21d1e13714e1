"""The CPU oracle against the reference's own golden vectors (snapshots,
known answers, kernel tests) — this pins the oracle before anything is
checked against it."""
import math

import numpy as np
import pytest

from oracle import zpu_oracle as zo


def snap_close(want, got, tol):
    """tests/snapshot.zig:239-244: |w - g| <= tol * max(1, |w|, |g|)."""
    want = np.asarray(want, dtype=np.float64).ravel()
    got = np.asarray(got, dtype=np.float64).ravel()
    assert want.shape == got.shape
    bound = tol * np.maximum(1.0, np.maximum(np.abs(want), np.abs(got)))
    bad = np.abs(want - got) > bound
    assert not bad.any(), (want[bad], got[bad])


def snap(golden, name):
    s = golden["snapshots"][name]
    return np.asarray(s["values"]), s["tol"], s["shape"]


def test_rng_normal_exact(golden):
    want, tol, shape = snap(golden, "zpu/rng/normal-seed12345")
    assert tol == 0.0
    got = zo.normal(golden["inputs"]["rng_seed"], int(np.prod(shape)), np.float64)
    assert np.array_equal(want, got), (want, got)


def test_rng_uniform_exact(golden):
    want, tol, shape = snap(golden, "zpu/rng/uniform-seed12345")
    s = np.uint64(golden["inputs"]["rng_seed"])
    got = zo.uniform_range(int(s), int(np.prod(shape)), 0.0, 1.0, np.float64)
    assert np.array_equal(want, got)


def test_matmul_snapshots(golden):
    a = np.array(golden["inputs"]["spd3"]).reshape(3, 3)
    want, tol, _ = snap(golden, "zpu/linalg/matmul-3x3")
    snap_close(want, zo.matmul(a, a), tol)
    want, tol, _ = snap(golden, "zpu/linalg/matvec")
    got = zo.matmul(a, np.array(golden["inputs"]["rhs3"]))
    assert got.shape == (3,)
    snap_close(want, got, tol)


def test_vmap_and_jit_replay_snapshots(golden):
    a = np.array(golden["inputs"]["vmap_a"], dtype=np.float64).reshape(3, 2, 2)
    b = np.array(golden["inputs"]["vmap_b"], dtype=np.float64).reshape(3, 2, 2)
    got = zo.unary("tanh", zo.matmul(a, b, 1, 1))
    for name in ("zpu/transforms/vmap", "zpu/transforms/jit-replay"):
        want, tol, shape = snap(golden, name)
        assert list(got.shape) == shape
        snap_close(want, got, tol)
    assert golden["jit_steps"] == 2


@pytest.mark.parametrize("name,fn", [
    ("zpu/ops/tanh", lambda x: zo.unary("tanh", x)),
    ("zpu/ops/exp", lambda x: zo.unary("exp", x)),
    ("zpu/ops/sigmoid", lambda x: zo.unary("sigmoid", x)),
    ("zpu/ops/erf", lambda x: zo.unary("erf", x)),
    ("zpu/ops/sqrt-abs", lambda x: zo.unary("sqrt", zo.unary("abs", x))),
    ("zpu/ops/square-rsqrt", lambda x: zo.unary("rsqrt", zo.unary("square", x))),
    ("zpu/ops/mul-scalar", lambda x: zo.binary("mul", x, 2.5)),
    ("zpu/ops/add-broadcast", lambda x: zo.binary("add", x, np.array([1.0]))),
    ("zpu/ops/maximum", lambda x: zo.binary("maximum", x, zo.unary("neg", x))),
])
def test_elementwise_snapshots(golden, name, fn):
    x = np.array(golden["inputs"]["spread8"], dtype=np.float64)
    want, tol, _ = snap(golden, name)
    snap_close(want, fn(x), tol)


def test_reduction_snapshots(golden):
    x = np.array(golden["inputs"]["spread12"], dtype=np.float64).reshape(3, 4)
    want, tol, _ = snap(golden, "zpu/reduce/sum-all")
    snap_close(want, [zo.reduce_sum(x)], tol)
    # sum over axis 0 is the generic row-order walk (ops.zig:746-752)
    col = np.zeros(4)
    for r in range(3):
        col = col + x[r]
    want, tol, _ = snap(golden, "zpu/reduce/sum-axis0")
    snap_close(want, col, tol)


@pytest.mark.parametrize("name,fn", [
    ("sum-axis1-keepdims", lambda x: zo.reduce_axis(x, "sum", 1, True)),
    ("max-axis1", lambda x: zo.reduce_axis(x, "max_reduce", 1)),
    ("min-axis0", lambda x: zo.reduce_axis(x, "min_reduce", 0)),
    ("prod-axis1", lambda x: zo.reduce_axis(x, "prod_op", 1)),
    ("mean-axis1", lambda x: zo.mean(x, 1)),
    ("variance-axis1", lambda x: zo.variance(x, 1)),
    ("argmax-axis1", lambda x: zo.arg_reduce(x, 1)),
])
def test_axis_reduction_snapshots(golden, name, fn):
    """tests/snap/zpu.zig:87-93 on spread(12) as 3 x 4 (f64)."""
    x = np.array(golden["inputs"]["spread12"], dtype=np.float64).reshape(3, 4)
    want, tol, shape = snap(golden, "zpu/reduce/" + name)
    got = fn(x)
    assert list(np.shape(got)) == shape, (np.shape(got), shape)
    snap_close(want, got, tol)


def test_reduction_known_answers(golden):
    """src/zpu/tests.zig:116-124 and examples/audit_edge_cases.zig:138-144."""
    for case in golden["reduce_known"]:
        x = np.array(case["x"], dtype=np.float32 if case.get("dtype") == "f32" else np.float64)
        x = x.reshape(case["shape"])
        if case["prim"] in ("argmax", "argmin"):
            got = zo.arg_reduce(x, case["axis"], want_max=case["prim"] == "argmax")
        else:
            got = zo.reduce_axis(x, case["prim"], case["axis"], case["keepdims"])
        assert list(np.shape(got)) == case["want_shape"], case["name"]
        assert np.all(np.abs(np.asarray(got, np.float64).ravel() - case["want"]) <= case["tol"]), case["name"]


def test_arg_reduce_scan_rules():
    """ops.argReduce's sequential rules (src/zpu/ops.zig:961-969): strict
    comparison (ties keep the first), NaN never replaces, a NaN first element
    pins 0, -0.0 ties +0.0; AXIS_NONE with a vmap depth folds payload axes."""
    nan = float("nan")
    assert zo.arg_reduce(np.array([1.0, 3.0, 3.0, 2.0]), 0) == 1
    assert zo.arg_reduce(np.array([1.0, 3.0, 3.0, 2.0]), 0, want_max=False) == 0
    assert zo.arg_reduce(np.array([nan, 5.0, 7.0]), 0) == 0
    assert zo.arg_reduce(np.array([nan, 5.0, 7.0]), 0, want_max=False) == 0
    assert zo.arg_reduce(np.array([1.0, nan, 7.0, nan]), 0) == 2
    assert zo.arg_reduce(np.array([nan, nan]), 0) == 0
    assert zo.arg_reduce(np.array([-0.0, 0.0]), 0) == 0
    assert zo.arg_reduce(np.array([-np.inf, -np.inf]), 0) == 0
    assert zo.arg_reduce(np.zeros((2, 0)), 1).tolist() == [0, 0]
    x = np.array([[1.0, 9.0, 2.0, 9.0], [4.0, 1.0, 4.0, 0.0]])
    assert zo.arg_reduce(x, zo.AXIS_NONE).shape == ()
    assert zo.arg_reduce(x, zo.AXIS_NONE) == 1
    assert zo.arg_reduce(x, zo.AXIS_NONE, depth=1).tolist() == [1, 0]
    assert zo.arg_reduce(x, 0, depth=1).tolist() == [1, 0]
    assert zo.arg_reduce(x, -1, want_max=False).tolist() == [0, 3]


def _log_softmax_rows(x):
    out = np.empty_like(x)
    sm = np.empty_like(x)
    for i, row in enumerate(x):
        m = max(row)
        s = row - m
        e = zo.unary("exp", s)
        z = zo.reduce_sum(e)
        out[i] = s - math.log(z)
        sm[i] = e / z
    return out, sm


def test_softmax_snapshots(golden):
    x = np.array(golden["inputs"]["logits3x3"], dtype=np.float64).reshape(3, 3)
    lsm, sm = _log_softmax_rows(x)
    want, tol, _ = snap(golden, "zpu/nn/log-softmax")
    snap_close(want, lsm, tol)
    want, tol, _ = snap(golden, "zpu/nn/softmax")
    snap_close(want, sm, tol)


def test_linalg_and_layer_norm_snapshots(golden):
    """tests/snap/zpu.zig:124-128, 151: compositions of the path's prims as
    zpu writes them -- norm = sqrt(sum(square(a))), trace = sum(diag(a)),
    outer = expandDims(a, -1) * b, dot = sum(mul(b, b), -1)
    (linalg.zig:397-459) and layerNorm (nn.zig:202-222: mean, sub, square,
    mean, add eps, sqrt, div, mul weight, add bias) -- through the oracle's
    reductions and f64 element-wise rules."""
    inp = golden["inputs"]
    a = np.array(inp["spd3"], dtype=np.float64).reshape(3, 3)
    b = np.array(inp["rhs3"], dtype=np.float64)
    d = np.ascontiguousarray(np.diagonal(a))
    got = {
        "norm": zo.unary("sqrt", np.asarray(zo.reduce_axis(zo.unary("square", a), "sum"))),
        "trace": zo.reduce_axis(d, "sum", -1),
        "diag": d,
        "outer": zo.binary("mul", np.array(inp["outer_a"])[:, None], np.array(inp["outer_b"])),
        "dot": zo.reduce_axis(zo.binary("mul", b, b), "sum", -1),
    }
    for name, g in got.items():
        want, tol, shape = snap(golden, "zpu/linalg/" + name)
        assert list(np.shape(g)) == shape, (name, np.shape(g), shape)
        snap_close(want, g, tol)
    x = np.array(inp["ln_rows"], dtype=np.float64).reshape(2, 3)
    w, bias = np.array(inp["ln_weight"]), np.array(inp["ln_bias"])
    c = zo.binary("sub", x, zo.mean(x, -1, True))
    v = zo.mean(zo.unary("square", c), -1, True)
    den = zo.unary("sqrt", zo.binary("add", v, np.float64(inp["ln_eps"])))
    ln = zo.binary("add", zo.binary("mul", zo.binary("div", c, den), w), bias)
    want, tol, shape = snap(golden, "zpu/nn/layer-norm")
    assert list(ln.shape) == shape
    snap_close(want, ln, tol)


def test_grad_snapshots(golden):
    """tests/snap/zpu.zig:172-218: the gradient of
    sum(softmax(sigmoid(x.w) + b) * target) w.r.t. x, w and b, and its jvp
    along a tangent of x, through the reverse-sweep rules the MLP step uses:
    the matmul VJPs g.W^T and X^T.g (autodiff.zig:480-487, the oracle's
    matmul), b's broadcast undone by a sum over the rows (unbroadcast,
    autodiff.zig:51), and the element-wise and softmax VJPs."""
    inp = golden["inputs"]
    x = np.array(inp["grad_x"], dtype=np.float64).reshape(2, 3)
    w = np.array(inp["grad_w"], dtype=np.float64).reshape(3, 2)
    b = np.array(inp["grad_b"], dtype=np.float64)
    t = np.array(inp["grad_target"], dtype=np.float64).reshape(2, 2)
    tangent = np.array(inp["grad_tangent"], dtype=np.float64).reshape(2, 3)
    h = zo.unary("sigmoid", zo.matmul(x, w))
    _, p = _log_softmax_rows(zo.binary("add", h, b))
    value = zo.reduce_sum(zo.binary("mul", p, t))
    gz = p * (t - zo.reduce_axis(p * t, "sum", -1, True))  # softmax VJP of d/dp = target
    ga = gz * h * (1.0 - h)                                # sigmoid VJP
    grads = [zo.matmul(ga, np.ascontiguousarray(w.T)), zo.matmul(np.ascontiguousarray(x.T), ga),
             zo.reduce_axis(gz, "sum", 0)]
    for i, g in enumerate(grads):
        want, tol, shape = snap(golden, "zpu/grad/arg%d" % i)
        assert list(g.shape) == shape, (i, g.shape, shape)
        snap_close(want, g, tol)
    want, tol, _ = snap(golden, "zpu/grad/jvp-value")
    snap_close(want, [value], tol)
    want, tol, _ = snap(golden, "zpu/grad/jvp-tangent")
    snap_close(want, [zo.reduce_sum(grads[0] * tangent)], tol)


def test_attention_snapshot(golden):
    """tests/snap/zpu.zig:298-329: a self-attention block with one weight
    for q, k and v -- matmuls, q.k^T through a transposed operand, a scalar
    division and a row softmax."""
    inp = golden["inputs"]
    x = np.array(inp["attn_x"], dtype=np.float64).reshape(4, 3)
    w = np.array(inp["attn_w"], dtype=np.float64).reshape(3, 3)
    q = zo.matmul(x, w)
    scores = zo.binary("div", zo.matmul(q, np.ascontiguousarray(q.T)), np.float64(2.0))
    _, weights = _log_softmax_rows(scores)
    got = zo.matmul(weights, q)
    want, tol, shape = snap(golden, "zpu/nn/attention")
    assert list(got.shape) == shape
    snap_close(want, got, tol)


def test_adam_snapshots(golden):
    inp = golden["inputs"]
    p = np.array(inp["adam_params"], dtype=np.float64)
    g = np.array(inp["adam_grads"], dtype=np.float64)
    opt = zo.Adam(lr=inp["adam_lr"])
    opt.step([p], [g])
    want, tol, _ = snap(golden, "zpu/optim/adam-step1")
    snap_close(want, p, tol)
    for _ in range(9):
        opt.step([p], [g])
    want, tol, _ = snap(golden, "zpu/optim/adam-step10")
    snap_close(want, p, tol)


def test_known_answer_matmuls(golden):
    for case in golden["known_answers"]:
        a = np.array(case["a"], dtype=np.float64).reshape(case["a_shape"])
        b = np.array(case["b"], dtype=np.float64).reshape(case["b_shape"])
        got = zo.matmul(a, b)
        assert np.allclose(got.ravel(), case["want"], rtol=case["tol"], atol=0), case["name"]


def test_known_answer_matmuls_in_other_types(golden):
    """The same known answers (src/zpu/tests.zig:145-171, small integers)
    through the oracle's restatement of ops.gemmF64 and of the integer
    gemmTyped loop: every element type pair whose promotion is not bool."""
    types = [np.float64, np.float32, np.float16, np.int64, np.int32, np.int16, np.uint8]
    for case in golden["known_answers"]:
        a_shape, b_shape = case["a_shape"], case["b_shape"]
        if len(a_shape) != 2 or len(b_shape) != 2:
            continue
        for ta in types:
            for tb in types:
                if ta == tb and ta in (np.float32, np.float64):
                    continue
                a = np.array(case["a"]).reshape(a_shape).astype(ta)
                b = np.array(case["b"]).reshape(b_shape).astype(tb)
                got = zo.gemm_convert(a, b)
                assert got.dtype == zo.promote(ta, tb)
                want = np.array(case["want"], dtype=np.float64)
                if got.dtype == np.uint8:
                    want = np.minimum(want, 255.0)  # zpu clamps (mixed) or wraps (u8 @ u8)
                    if ta == tb:
                        want = np.array(case["want"], dtype=np.int64) % 256
                assert np.array_equal(got.ravel().astype(np.float64), want), (case["name"], ta, tb)
    assert zo.promote(np.uint8, np.int8) == np.int8 and zo.promote(np.int8, np.uint8) == np.uint8
    assert zo.promote(np.int16, np.uint8) == np.int16 and zo.promote(np.float16, np.int64) == np.float16
    with pytest.raises(ValueError):
        zo.gemm_convert(np.ones((2, 2), np.bool_), np.ones((2, 2), np.bool_))


def test_gemm_vs_naive_kernel_shapes(golden):
    """kernels.zig:512-543."""
    for m, k, n in golden["gemm_shapes"]:
        a = (np.arange(m * k) % 7) * 0.5 - 1.0
        b = (np.arange(k * n) % 5) * 0.25 - 0.5
        a, b = a.reshape(m, k), b.reshape(k, n)
        got = zo.gemm(a, b)
        want = np.zeros((m, n))
        for p in range(k):
            want += np.outer(a[:, p], b[p])
        assert np.allclose(got, want, rtol=1e-12, atol=1e-300)


def test_gemm_is_the_fma_chain():
    """Per element: c = 0; c = fma(a[i,p], b[p,j], c) for p ascending, with
    the non-vector tail columns as mul+add (kernels.zig:369-398)."""
    rng = np.random.default_rng(3)
    m, k, n = 5, 37, 139  # n = 128 + 11: a second panel with an 8-wide part and a tail
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    got = zo.gemm(a, b)
    want = np.zeros((m, n), dtype=np.float32)
    for j in range(n):
        pj = j % 128
        nb = min(128, n - (j - pj))
        vec = pj < (nb // 8) * 8
        for i in range(m):
            c = np.float32(0)
            for p in range(k):
                if vec:
                    c = np.float32(np.float64(a[i, p]) * np.float64(b[p, j]) + np.float64(c))
                else:
                    c = np.float32(c + np.float32(a[i, p] * b[p, j]))
            want[i, j] = c
    # fma(a,b,c) for f32 == round_f32(a*b + c in f64) except in double-rounding
    # corner cases; the products of two f32 are exact in f64, so only the final
    # sum is rounded twice -- allow a 1-ulp difference there and none elsewhere.
    assert np.max(np.abs(got.view(np.int32) - want.view(np.int32))) <= 1


def test_reduce_edges(golden):
    """kernels.zig:571-581: sums of 0..len-1 are exact at every edge length."""
    for n in golden["reduce_lengths"]:
        x = np.arange(n, dtype=np.float32)
        assert zo.reduce_sum(x) == np.float32(n * (n - 1) // 2)
    nan = np.full(8, np.nan, dtype=np.float32)
    assert np.isnan(zo.reduce_max(nan))


def test_reduce_matches_left_to_right_loosely():
    """kernels.zig:545-569: n = 1000, data[i] = sin(0.37 i) * 3."""
    data = np.sin(np.arange(1000) * 0.37) * 3.0
    want = 0.0
    for v in data:
        want += v
    assert abs(zo.reduce_sum(data) - want) <= 1e-12 * abs(want)


def test_worker_count_matches_parallel_zig():
    zo.set_cores(8)
    assert zo.worker_count(63999) == 1
    assert zo.worker_count(64000) == 4
    assert zo.worker_count(1 << 26) == 8
    zo.set_cores(0)


def test_jit_chain_small():
    x = zo.normal(0x5EED0003, 1000)
    s, s64, t = zo.jit_chain_tanh_sq_affine_sum(x, 0.5, -0.25, want_vector=True)
    ref = np.array([np.float32(np.float32(math.tanh(float(np.float32(v * v)))) * np.float32(0.5)) for v in x],
                   dtype=np.float32) + np.float32(-0.25)
    assert np.array_equal(t, ref)
    assert s == zo.reduce_sum(ref)
    assert abs(s64 - sum(float(v) for v in ref)) < 1e-9


def test_pow_integer_powers():
    for t in range(1, 30):
        # repeated squaring (Go's algorithm) sits within a few ulp of libm pow
        assert abs(zo.pow_(0.9, t) - 0.9 ** t) <= 1e-15 * 0.9 ** t


def test_mlp_gradient_finite_difference():
    """The oracle's analytic MLP gradient against central differences in f64
    arithmetic on a tiny network (a check of the restated backward pass)."""
    rng = np.random.default_rng(0)
    B, dims = 4, (6, 5, 4, 3)
    X = rng.uniform(0, 1, (B, dims[0])).astype(np.float32)
    y = rng.integers(0, dims[3], B).astype(np.int64)
    params = zo.mlp_init(list(dims))
    params[1][:] = 0.1
    loss, grads = zo.mlp_loss_grad(X, y, params)

    def f64_loss(ps):
        W1, b1, W2, b2, W3, b3 = [p.astype(np.float64) for p in ps]
        h = np.tanh(X.astype(np.float64) @ W1 + b1)
        h = np.tanh(h @ W2 + b2)
        lg = h @ W3 + b3
        lg = lg - lg.max(1, keepdims=True)
        lp = lg - np.log(np.exp(lg).sum(1, keepdims=True))
        return -lp[np.arange(B), y].mean()

    assert abs(loss - f64_loss(params)) < 1e-5
    for pi in range(6):
        for idx in [0, params[pi].size - 1]:
            ps = [p.astype(np.float64) for p in params]
            h = 1e-6
            ps[pi].ravel()[idx] += h
            up = f64_loss(ps)
            ps[pi].ravel()[idx] -= 2 * h
            dn = f64_loss(ps)
            fd = (up - dn) / (2 * h)
            assert abs(grads[pi].ravel()[idx] - fd) < 1e-4, (pi, idx, grads[pi].ravel()[idx], fd)


def test_cast_and_view_snapshots(golden):
    """tests/snap/zpu.zig:48,96-97: cast(spread(6), bool); the transpose and
    flip views of spread(12) as 3 x 4 read in logical order."""
    want, tol, shape = snap(golden, "zpu/tensor/bools")
    got = zo.tensor_copy(np.array(golden["inputs"]["spread6"]), np.bool_)
    assert got.astype(np.float64).tolist() == want.tolist()
    x = np.array(golden["inputs"]["spread12"], dtype=np.float64).reshape(3, 4)
    want, tol, shape = snap(golden, "zpu/shape/transpose")
    snap_close(want, zo.tensor_copy(x.T, np.float64), tol)
    want, tol, shape = snap(golden, "zpu/shape/flip")
    snap_close(want, zo.tensor_copy(x[:, ::-1], np.float64), tol)


def test_from_f64_rules():
    """scalar.fromF64 (src/zpu/scalar.zig:17-27) by hand."""
    v = np.array([np.nan, 2.9, -2.9, 300.0, -300.0, np.inf, -np.inf, -0.0])
    assert zo.from_f64(v, np.uint8).tolist() == [0, 2, 0, 255, 0, 255, 0, 0]
    assert zo.from_f64(v, np.int8).tolist() == [0, 2, -2, 127, -128, 127, -128, 0]
    assert zo.from_f64(v, np.bool_).tolist() == [True, True, True, True, True, True, True, False]
    assert zo.from_f64(np.array([2.0 ** 63, -2.0 ** 64]), np.int64).tolist() == [2 ** 63 - 1, -2 ** 63]


def test_selection_snapshots(golden):
    """tests/snap/zpu.zig:69-75 on spread(8): where(gt(x, 0), x, -x),
    clamp (maximum then minimum, ops.zig:593-601), lerp (a + t (b - a),
    ops.zig:604-610)."""
    x = np.array(golden["inputs"]["spread8"], dtype=np.float64)
    want, tol, _ = snap(golden, "zpu/ops/where")
    snap_close(want, zo.where(zo.predicate("gt", x, 0.0), x, -x), tol)
    want, tol, _ = snap(golden, "zpu/ops/clamp")
    snap_close(want, np.minimum(np.maximum(x, -0.5), 0.5), tol)
    want, tol, _ = snap(golden, "zpu/ops/lerp")
    snap_close(want, x + 0.25 * (-x - x), tol)


def test_predicate_known_answers(golden):
    """src/zpu/tests.zig:97-101, 873-877."""
    k = {c["name"]: c for c in golden["pred_known"]}
    a = np.array(k["gt(a, 3)"]["x"], dtype=np.float64).reshape(2, 3)
    assert zo.predicate("gt", a, 3.0).astype(np.float64).ravel().tolist() == k["gt(a, 3)"]["want"]
    w = zo.where(zo.predicate("gt", a, 3.0), a, -a)
    assert w.ravel().tolist() == k["where(gt(a, 3), a, neg(a))"]["want"]
    i = np.array(k["any(lt(i, 3))"]["x"], dtype=np.float64).reshape(2, 2)
    assert [float(zo.reduce_bool(zo.predicate("lt", i, 3.0), "any_reduce"))] == k["any(lt(i, 3))"]["want"]
    assert [float(zo.reduce_bool(zo.predicate("lt", i, 3.0), "all_reduce"))] == k["all(lt(i, 3))"]["want"]


def test_predicate_rules():
    nan = float("nan")
    x = np.array([nan, 0.0, -0.0, 1.0, np.inf])
    assert zo.predicate("eq", x, x).tolist() == [False, True, True, True, True]
    assert zo.predicate("ne", x, 0.0).tolist() == [True, False, False, True, True]
    assert zo.predicate("logical_and", x, 1.0).tolist() == [True, False, False, True, True]
    assert zo.predicate("logical_not", x).tolist() == [False, True, True, False, False]
    assert zo.where(x, 1.0, 2.0).tolist() == [1.0, 2.0, 2.0, 1.0, 1.0]
    assert bool(zo.reduce_bool(np.zeros((3, 0)), "all_reduce")) is True
    assert zo.reduce_bool(np.zeros((3, 0)), "any_reduce", 1).tolist() == [False] * 3


def test_cumsum_snapshots_and_known_answers(golden):
    """tests/snap/zpu.zig:94-95 (spread(12) as 3 x 4) and src/zpu/tests.zig:125-126."""
    x = np.array(golden["inputs"]["spread12"], dtype=np.float64).reshape(3, 4)
    want, tol, _ = snap(golden, "zpu/reduce/cumsum-axis1")
    snap_close(want, zo.cumsum(x, 1), tol)
    want, tol, _ = snap(golden, "zpu/reduce/cumsum-reverse")
    snap_close(want, zo.cumsum(x, 1, reverse=True), tol)
    for c in golden["cumsum_known"]:
        a = np.array(c["x"], dtype=np.float64).reshape(c["shape"])
        assert zo.cumsum(a, c["axis"], c["reverse"]).ravel().tolist() == c["want"]


def test_data_movement_snapshots(golden):
    """tests/snap/zpu.zig:98-101 on spread(12) as 3 x 4: pad, take, concat,
    stack (numpy's own semantics restate zpu's here)."""
    x = np.array(golden["inputs"]["spread12"], dtype=np.float64).reshape(3, 4)
    cases = {"pad": np.pad(x, ((1, 0), (0, 2)), constant_values=-1.0), "take": x[[2, 0, 2]],
             "concat": np.concatenate([x, x], 1), "stack": np.stack([x, x], 0)}
    for name, got in cases.items():
        want, tol, shape = snap(golden, "zpu/shape/" + name)
        assert list(got.shape) == shape, name
        snap_close(want, got, tol)
