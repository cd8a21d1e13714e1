"""Fused jit regions on the B200 against the oracle (zpu's CPU jit path).

Tolerances (stated, per the north star):
  * element-wise: <= 4 ulp per primitive against the oracle's f32 result;
  * the full chain tanh(x*x)*a + b: the tanh step within 4 ulp, and every
    element within |a| * 4 ulp(tanh) + 1 ulp(y) of the oracle;
  * sums: |gpu - f64 reference| <= 1e-6 * sum(|t_i|) (the GPU accumulates in
    f64; zpu's own f32 order is reported, not required).
"""
import math

import numpy as np
import pytest

from oracle import zpu_oracle as zo
from tests.helpers import ulp_diff_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SEED_X = 0x5EED0003  # the chain workload's input seed
N_FULL = 1 << 26


@pytest.fixture(scope="module")
def zc():
    import zpu_b200
    zpu_b200.check(zpu_b200.lib().zpucuda_init(0))
    return zpu_b200


def chain_plan(zc, n, reduce, a_as_blob=True):
    steps = [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0), ("mul", [11, 2], 12, -2, 0),
             ("add", [12, 3], 13, -2, 0)]
    out = 13
    if reduce:
        steps.append(("sum", [13], 14, -2, 0))
        out = 14
    if a_as_blob:
        return zc.Plan([(1, zc.F32, (n,))], [(2, np.float32(0.5)), (3, np.float32(-0.25))], steps, [out])
    return zc.Plan([(1, zc.F32, (n,)), (2, zc.F32, ()), (3, zc.F32, ())], [], steps, [out])


def test_device_rng_is_zpus_stream(zc):
    n = 4097
    for seed in (12345, SEED_X):
        u = zc.rng_uniform(seed, n, -1.0, 1.0).cpu().numpy()
        assert np.array_equal(u, zo.uniform_range(seed, n, -1.0, 1.0))
        g = zc.rng_normal(seed, n).cpu().numpy()
        assert ulp_diff_f32(g, zo.normal(seed, n)).max() <= 1
        g64 = zc.rng_normal(seed, n, dtype=torch.float64).cpu().numpy()
        # CUDA's f64 log/sin/cos are within an ulp or two of glibc's: compare
        # against the radius r (|r cos|, |r sin| <= r) rather than the value
        want64 = zo.normal(seed, n, np.float64)
        assert np.max(np.abs(g64 - want64)) <= 1e-14
        r = zc.rng_randint(seed, n, 0, 10).cpu().numpy()
        assert np.array_equal(r, zo.randint(seed, n, 0, 10))


def test_chain_lowers_to_one_catalogued_kernel(zc):
    p = chain_plan(zc, 1 << 20, True)
    assert p.num_kernels() == 1
    assert "catalogue tanh_sq_affine+sum" in p.describe()


@pytest.mark.parametrize("n", [1, 3, 4, 5, 33, 1000, (1 << 20) + 3])
def test_chain_elementwise_within_tolerance(zc, n):
    x = zo.normal(SEED_X, n)
    _, _, want = zo.jit_chain_tanh_sq_affine_sum(x, 0.5, -0.25, want_vector=True)
    p = chain_plan(zc, n, False)
    (got,) = p.run([torch.from_numpy(x).cuda()])
    got = got.cpu().numpy()
    tanh_want = np.array([zo.lib().zo_unary_f32(19, float(np.float32(v * v))) for v in x[:2000]], np.float32)
    tanh_plan = zc.Plan([(1, zc.F32, (n,))], [], [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0)], [11])
    (tg,) = tanh_plan.run([torch.from_numpy(x).cuda()])
    tg = tg.cpu().numpy()
    assert ulp_diff_f32(tg[:2000], tanh_want).max() <= 4
    ulp_t = np.spacing(np.abs(tg).astype(np.float32)).astype(np.float64)
    ulp_y = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
    bound = 0.5 * 4 * ulp_t + ulp_y
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert (err <= bound).all(), (err.max(), n)


def test_chain_tanh_ulp_full_size(zc):
    """tanh(x*x) over the whole 2^26-element workload: max ulp vs the oracle."""
    x_d = zc.rng_normal(SEED_X, N_FULL)
    p = zc.Plan([(1, zc.F32, (N_FULL,))], [], [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0)], [11])
    (t,) = p.run([x_d])
    x = x_d.cpu().numpy()
    sq = (x * x).astype(np.float32)
    want = np.tanh(sq.astype(np.float64)).astype(np.float32)  # (f32)tanh((f64)v): scalar.zig:262-266
    d = ulp_diff_f32(t.cpu().numpy(), want)
    assert d.max() <= 4, d.max()


def test_catalogue_tanh_every_float(zc):
    """The catalogued kernels' own tanh over EVERY f32 in [FLT_MIN, 10] and
    its negatives' sign rule: at most 1 ulp from (f32)tanh((f64)x) (the f64
    reference is torch's device tanh, rounded once)."""
    lo, hi = np.float32(np.finfo(np.float32).tiny).view(np.int32), np.float32(10.0).view(np.int32)
    p = None
    worst = 0
    chunk = 1 << 27
    for start in range(int(lo), int(hi), chunk):
        bits = torch.arange(start, min(start + chunk, int(hi)), dtype=torch.int32, device="cuda")
        x = bits.view(torch.float32)
        if p is None or p.outputs[0][1][0] != x.numel():
            p = zc.Plan([(1, zc.F32, (x.numel(),))], [], [("tanh", [1], 10, -2, 0)], [10])
            assert "catalogue tanh]" in p.describe()
        (t,) = p.run([x])
        want = torch.tanh(x.double()).float()
        d = (t.view(torch.int32).long() - want.view(torch.int32).long()).abs().max().item()
        worst = max(worst, d)
        (tn,) = p.run([-x])
        assert torch.equal(tn, -t)
    assert worst <= 1, worst


def test_catalogue_tanh_special_values(zc):
    x = np.array([0.0, -0.0, 1e-30, 1e-45, 0.89999, 0.9, 0.90001, 3.0, 9.0, 9.1, 9.2, 20.0, 1e30, np.inf,
                  -np.inf, np.nan], dtype=np.float32)
    p = zc.Plan([(1, zc.F32, (x.size,))], [], [("tanh", [1], 10, -2, 0)], [10])
    (t,) = p.run([torch.from_numpy(x).cuda()])
    t = t.cpu().numpy()
    assert np.isnan(t[-1])
    assert t[-3] == 1.0 and t[-2] == -1.0 and t[-4] == 1.0
    assert np.signbit(t[1]) and t[1] == 0.0
    want = np.tanh(x[:-1].astype(np.float64)).astype(np.float32)
    assert ulp_diff_f32(t[:-1], want).max() <= 1


@pytest.mark.parametrize("n", [0, 1, 7, 1000, (1 << 20) + 3, N_FULL])
def test_chain_fused_sum(zc, n):
    x_d = zc.rng_normal(SEED_X, n) if n else torch.empty(0, device="cuda")
    x = x_d.cpu().numpy()
    s32, s64, t = zo.jit_chain_tanh_sq_affine_sum(x, 0.5, -0.25, want_vector=True)
    p = chain_plan(zc, n, True)
    (got,) = p.run([x_d])
    g = float(got.cpu().numpy())
    scale = zo.abssum_f64(t) if n else 0.0
    assert abs(g - s64) <= 1e-6 * scale + 1e-30, (g, s64, s32)
    # determinism: a second run gives the same bits
    (again,) = p.run([x_d])
    assert float(again.cpu().numpy()) == g


def test_chain_scalars_as_arguments(zc):
    n = 100003
    x = zo.normal(SEED_X, n)
    s32, s64, t = zo.jit_chain_tanh_sq_affine_sum(x, 0.5, -0.25, want_vector=True)
    p = chain_plan(zc, n, True, a_as_blob=False)
    a = torch.tensor(0.5, dtype=torch.float32, device="cuda")
    b = torch.tensor(-0.25, dtype=torch.float32, device="cuda")
    (got,) = p.run([torch.from_numpy(x).cuda(), a, b])
    assert abs(float(got.cpu()) - s64) <= 1e-6 * zo.abssum_f64(t)


def test_misaligned_input_takes_the_bytecode_path(zc):
    n = 4099
    x = zo.normal(SEED_X, n + 1)
    s32, s64, t = zo.jit_chain_tanh_sq_affine_sum(x[1:], 0.5, -0.25, want_vector=True)
    base = torch.from_numpy(x).cuda()
    p = chain_plan(zc, n, True)
    (got,) = p.run([base[1:]])  # 4-byte offset: not 16-byte aligned
    assert abs(float(got.cpu()) - s64) <= 1e-6 * zo.abssum_f64(t)


UNARY = [("neg", -3, 3), ("abs", -3, 3), ("exp", -10, 10), ("expm1", -3, 3), ("log", 0.01, 100),
         ("log1p", -0.9, 10), ("sqrt", 0, 100), ("rsqrt", 0.01, 100), ("square", -10, 10),
         ("recip", 0.1, 10), ("cbrt", -8, 8), ("sin", -6, 6), ("cos", -6, 6), ("tan", -1.4, 1.4),
         ("asin", -1, 1), ("acos", -1, 1), ("atan", -10, 10), ("sinh", -5, 5), ("cosh", -5, 5),
         ("tanh", -5, 5), ("asinh", -10, 10), ("acosh", 1, 10), ("atanh", -0.99, 0.99),
         ("erf", -3, 3), ("sigmoid", -10, 10), ("softplus", -10, 10), ("relu", -3, 3),
         ("floor", -3, 3), ("ceil", -3, 3), ("round", -3, 3), ("trunc", -3, 3), ("sign", -3, 3)]


@pytest.mark.parametrize("prim,lo,hi", UNARY)
def test_bytecode_unary_within_4ulp(zc, prim, lo, hi):
    n = 3001
    x = zo.uniform_range(77, n, lo, hi)
    p = zc.Plan([(1, zc.F32, (n,))], [], [(prim, [1], 10, -2, 0), ("neg", [10], 11, -2, 0)], [11])
    assert "bytecode" in p.describe()
    (got,) = p.run([torch.from_numpy(x).cuda()])
    want = -zo.unary(prim, x)
    assert ulp_diff_f32(got.cpu().numpy(), want).max() <= 4, prim


@pytest.mark.parametrize("prim", ["add", "sub", "mul", "div", "pow", "maximum", "minimum", "atan2",
                                  "hypot", "mod_op"])
def test_bytecode_binary_within_4ulp(zc, prim):
    n = 2001
    a = zo.uniform_range(5, n, 0.1, 4.0)
    b = zo.uniform_range(6, n, -3.0, 3.0)
    if prim in ("pow", "mod_op"):
        b = zo.uniform_range(6, n, 0.5, 3.0)
    p = zc.Plan([(1, zc.F32, (n,)), (2, zc.F32, (n,))], [], [(prim, [1, 2], 10, -2, 0), ("neg", [10], 11, -2, 0)],
                [11])
    (got,) = p.run([torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    want = -zo.binary(prim, a, b)
    assert ulp_diff_f32(got.cpu().numpy(), want).max() <= 4, prim


@pytest.mark.parametrize("n", [1, 4099, (1 << 22) + 5])
@pytest.mark.parametrize("region", ["sq", "dot", "ident", "affine"])
def test_catalogue_hbm_bound_full_sums(zc, region, n):
    """Full sums of the catalogued regions without a transcendental step
    (x*x, x*y, x, x*a + b) stream through the bulk-copy pipeline kernel
    (16 KiB tiles, plain loads past the last whole tile).  Integer-valued
    inputs keep every partial sum exact, so the result is the exact sum: an
    element dropped or counted twice shows."""
    g = np.random.default_rng(n * 7 + len(region))
    x = g.integers(-2, 3, n).astype(np.float32)
    y = g.integers(-1, 2, n).astype(np.float32)
    F = zc.F32
    xd = x.astype(np.float64)
    blobs, ins = [], [x]
    if region == "sq":
        steps, want = [("mul", [1, 1], 10, -2, 0), ("sum", [10], 11, -2, 0)], np.sum(xd * xd)
    elif region == "dot":
        steps, want = [("mul", [1, 2], 10, -2, 0), ("sum", [10], 11, -2, 0)], np.sum(xd * y.astype(np.float64))
        ins = [x, y]
    elif region == "ident":
        steps, want = [("sum", [1], 11, -2, 0)], np.sum(xd)
    else:
        blobs = [(3, np.float32(2.0)), (4, np.float32(-1.0))]
        steps = [("mul", [1, 3], 10, -2, 0), ("add", [10, 4], 12, -2, 0), ("sum", [12], 11, -2, 0)]
        want = np.sum(2.0 * xd - 1.0)
    args = [(k + 1, F, (n,)) for k in range(len(ins))]
    p = zc.Plan(args, blobs, steps, [11])
    # the front end passes a scalar blob as shape (1,): at n = 1 it has the
    # region's shape and loads as a full input, which no catalogue entry
    # takes, so that plan runs in the bytecode interpreter
    if not (region == "affine" and n == 1):
        assert ("catalogue %s+sum" % region) in p.describe(), p.describe()
    (got,) = p.run([torch.from_numpy(v).cuda() for v in ins])
    assert float(got.cpu()) == want


def test_row_broadcast_and_row_reductions(zc):
    rows, cols = 37, 129
    x = zo.uniform_range(9, rows * cols, -2, 2).reshape(rows, cols)
    bias = zo.uniform_range(10, cols, -1, 1)
    for prim, fn in (("sum", np.sum), ("max_reduce", np.max), ("min_reduce", np.min)):
        p = zc.Plan([(1, zc.F32, (rows, cols)), (2, zc.F32, (cols,))], [],
                    [("add", [1, 2], 10, -2, 0), ("exp", [10], 11, -2, 0), (prim, [11], 12, -1, 0)], [12, 11])
        red, e = p.run([torch.from_numpy(x).cuda(), torch.from_numpy(bias).cuda()])
        want_e = zo.unary("exp", zo.binary("add", x, bias))
        assert ulp_diff_f32(e.cpu().numpy(), want_e).max() <= 4
        want = fn(want_e.astype(np.float64), axis=1)
        assert np.allclose(red.cpu().numpy(), want, rtol=2e-6), prim


def test_general_broadcast_and_keepdims(zc):
    x = zo.uniform_range(11, 6 * 5 * 4, -1, 1).reshape(6, 5, 4)
    col = zo.uniform_range(12, 5, -1, 1).reshape(5, 1)
    p = zc.Plan([(1, zc.F32, (6, 5, 4)), (2, zc.F32, (5, 1))], [],
                [("mul", [1, 2], 10, -2, 0), ("sum", [10], 11, -1, 1)], [11, 10])
    assert ";FG;" in p.describe()
    red, prod = p.run([torch.from_numpy(x).cuda(), torch.from_numpy(col).cuda()])
    want = (x * col).astype(np.float32)
    assert np.array_equal(prod.cpu().numpy(), want)
    assert red.shape == (6, 5, 1)
    assert np.allclose(red.cpu().numpy()[..., 0], want.astype(np.float64).sum(-1), rtol=1e-6, atol=1e-7)


def test_f64_region_and_prod_reduction(zc):
    n = 999
    x = zo.uniform_range(13, n, 0.99, 1.01, np.float64)
    p = zc.Plan([(1, zc.F64, (n,))], [(2, np.float64(1.0))],
                [("mul", [1, 2], 10, -2, 0), ("prod_op", [10], 11, -2, 0), ("sum", [1], 12, -2, 0)], [11, 12])
    assert p.num_kernels() == 2
    pr, sm = p.run([torch.from_numpy(x).cuda()])
    assert abs(float(pr.cpu()) - np.prod(x)) <= 1e-12 * abs(np.prod(x))
    assert abs(float(sm.cpu()) - zo.reduce_sum(x)) <= 1e-12 * n


def test_multi_region_plan_with_intermediates(zc):
    """softmax-like: m = max(x); e = exp(x - m); s = sum(e); y = e / s."""
    n = 50001
    x = zo.uniform_range(14, n, -5, 5)
    steps = [("max_reduce", [1], 10, -2, 0), ("sub", [1, 10], 11, -2, 0), ("exp", [11], 12, -2, 0),
             ("sum", [12], 13, -2, 0), ("div", [12, 13], 14, -2, 0)]
    p = zc.Plan([(1, zc.F32, (n,))], [], steps, [14])
    assert p.num_kernels() == 3, p.describe()
    (y,) = p.run([torch.from_numpy(x).cuda()])
    m = np.float32(x.max())
    e = zo.unary("exp", (x - m).astype(np.float32))
    want = (e / np.float32(e.astype(np.float64).sum())).astype(np.float32)
    assert ulp_diff_f32(y.cpu().numpy(), want).max() <= 8


def test_run_host_matches_device_run(zc):
    n = (1 << 20) + 5
    x_d = zc.rng_normal(SEED_X, n)
    p = chain_plan(zc, n, True)
    (dev,) = p.run([x_d])
    host = x_d.cpu().pin_memory()
    (h,) = p.run_host([host])
    assert float(h) == float(dev.cpu())


def test_launch_counter_counts_region_launches(zc):
    p = chain_plan(zc, 4096, True)
    x = zc.rng_normal(SEED_X, 4096)
    before = zc.launch_count()
    for _ in range(3):
        p.run([x])
    torch.cuda.synchronize()
    assert zc.launch_count() - before == 3


@pytest.mark.parametrize("axis,keep", [(0, 0), (1, 0), (1, 1), (-3, 1), (2, 0)])
@pytest.mark.parametrize("prim", ["sum", "max_reduce", "min_reduce", "prod_op"])
def test_reductions_over_any_axis(zc, axis, keep, prim):
    """sum / prod / max / min over one axis of a 3-D region (ops.reduceOp,
    src/zpu/ops.zig:820-869): the element-wise output and the reduction in
    one kernel; an axis other than the last walks it in row order."""
    shape = (7, 33, 65)
    x = zo.uniform_range(21, 7 * 33 * 65, 0.5, 1.5).reshape(shape)
    p = zc.Plan([(1, zc.F32, shape)], [],
                [("sqrt", [1], 10, -2, 0), (prim, [10], 11, axis, keep)], [11, 10])
    red, s = p.run([torch.from_numpy(x).cuda()])
    want_s = zo.unary("sqrt", x)
    assert ulp_diff_f32(s.cpu().numpy(), want_s).max() <= 4
    fn = {"sum": np.sum, "max_reduce": np.max, "min_reduce": np.min, "prod_op": np.prod}[prim]
    want = fn(want_s.astype(np.float64), axis=axis, keepdims=bool(keep))
    assert red.shape == want.shape, (red.shape, want.shape)
    assert np.allclose(red.cpu().numpy(), want, rtol=2e-6, atol=0), prim


def test_axis0_sum_matches_the_snapshot(zc, golden):
    """The reference's reduce/sum-axis0 snapshot (spread12 as 3 x 4, f64):
    the device walks the rows in order as zpu does, within the snapshot's
    1e-9."""
    x = np.array(golden["inputs"]["spread12"], dtype=np.float64).reshape(3, 4)
    snapv = golden["snapshots"]["zpu/reduce/sum-axis0"]
    p = zc.Plan([(1, zc.F64, (3, 4))], [], [("sum", [1], 10, 0, 0)], [10])
    (got,) = p.run([torch.from_numpy(x).cuda()])
    want = np.array(snapv["values"])
    g = got.cpu().numpy()
    assert g.shape == (4,)
    assert np.all(np.abs(g - want) <= snapv["tol"] * np.maximum(1, np.maximum(np.abs(g), np.abs(want))))


def _tanh_sum_plan(zc, region, n):
    if region == "tanh_sq_affine":
        return chain_plan(zc, n, True)
    if region == "tanh_sq":
        steps = [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0), ("sum", [11], 12, -2, 0)]
        return zc.Plan([(1, zc.F32, (n,))], [], steps, [12])
    return zc.Plan([(1, zc.F32, (n,))], [], [("tanh", [1], 10, -2, 0), ("sum", [10], 11, -2, 0)], [11])


@pytest.mark.parametrize("region", ["tanh_sq_affine", "tanh_sq", "tanh"])
@pytest.mark.parametrize("n,frac", [(N_FULL, 0.3), ((1 << 25) + 7, 1.0), ((1 << 25) + 7, 0.001),
                                    (N_FULL + 5, 0.0), ((1 << 24) + 1, 0.5), (4099, 0.5)])
def test_tanh_sums_count_every_element_once(zc, region, n, frac):
    """Full sums through tanh at sizes that reach every part of the fused
    kernel (unrolled grid-stride iterations, the float4 tail, the n % 4
    elements).  With x in {0, +-16, +-inf} every tanh value is exactly 0 or
    +-1 (tanh(16) rounds to 1 in f32) and every partial sum is exact, so the
    result must be the exactly rounded count: an element dropped or counted
    twice anywhere shows."""
    g = torch.Generator(device="cuda").manual_seed(n * 1000 + int(frac * 1000))
    r = torch.rand(n, device="cuda", generator=g)
    neg = torch.rand(n, device="cuda", generator=g) < 0.5
    inf = torch.rand(n, device="cuda", generator=g) < 0.05
    big = r < frac
    mag = torch.where(inf, torch.tensor(float("inf"), device="cuda"), torch.tensor(16.0, device="cuda"))
    x = torch.where(big, torch.where(neg, -mag, mag), torch.zeros((), device="cuda")).float().contiguous()
    k = int(big.sum())
    kneg = int((big & neg).sum())
    p = _tanh_sum_plan(zc, region, n)
    assert ("catalogue %s+sum" % region) in p.describe()
    (got,) = p.run([x])
    got = float(got.cpu())
    if region == "tanh_sq_affine":
        want = 0.5 * k - 0.25 * n  # each element: tanh * 0.5 - 0.25 with tanh 0 or 1
    elif region == "tanh_sq":
        want = float(k)
    else:
        want = float(k - 2 * kneg)
    assert got == float(np.float32(want)), (got, want, k)


def test_tanh_sum_propagates_nan(zc):
    n = N_FULL
    x = torch.zeros(n, device="cuda")
    x[12345678] = float("nan")
    x[(1 << 25) + 3] = 16.0
    for region in ("tanh_sq_affine", "tanh_sq", "tanh"):
        (got,) = _tanh_sum_plan(zc, region, n).run([x])
        assert math.isnan(float(got.cpu())), region


def _snapshot_plan(zc, name):
    """The jit plan each tests/snap/zpu.zig:87-93 case records (3 x 4 f64):
    mean and variance are their ops.zig:894-922 compositions with 1/count as
    a captured rank-0 blob."""
    c = [(2, np.float64(0.25))]
    one = {"sum-axis1-keepdims": ("sum", 1, 1), "max-axis1": ("max_reduce", 1, 0),
           "min-axis0": ("min_reduce", 0, 0), "prod-axis1": ("prod_op", 1, 0), "argmax-axis1": ("argmax", 1, 0)}
    args = [(1, zc.F64, (3, 4))]
    if name in one:
        prim, axis, keep = one[name]
        return zc.Plan(args, [], [(prim, [1], 10, axis, keep)], [10])
    if name == "mean-axis1":
        return zc.Plan(args, c, [("sum", [1], 10, 1, 0), ("mul", [10, 2], 11, -2, 0)], [11])
    steps = [("sum", [1], 10, 1, 1), ("mul", [10, 2], 11, -2, 0), ("sub", [1, 11], 12, -2, 0),
             ("square", [12], 13, -2, 0), ("sum", [13], 14, 1, 0), ("mul", [14, 2], 15, -2, 0)]
    return zc.Plan(args, c, steps, [15])


@pytest.mark.parametrize("name", ["sum-axis1-keepdims", "max-axis1", "min-axis0", "prod-axis1", "mean-axis1",
                                  "variance-axis1", "argmax-axis1"])
def test_axis_reductions_match_the_snapshots(zc, golden, name):
    x = np.array(golden["inputs"]["spread12"], dtype=np.float64).reshape(3, 4)
    snapv = golden["snapshots"]["zpu/reduce/" + name]
    (got,) = _snapshot_plan(zc, name).run([torch.from_numpy(x).cuda()])
    g = got.cpu().numpy()
    assert list(g.shape) == snapv["shape"], (g.shape, snapv["shape"])
    want = np.array(snapv["values"])
    if name == "argmax-axis1":
        assert got.dtype == torch.int64
        assert g.ravel().tolist() == want.astype(np.int64).tolist()
    else:
        g = g.ravel()
        assert np.all(np.abs(g - want) <= snapv["tol"] * np.maximum(1, np.maximum(np.abs(g), np.abs(want))))


def test_reduction_known_answers_on_device(zc, golden):
    for case in golden["reduce_known"]:
        f32 = case.get("dtype") == "f32"
        x = np.array(case["x"], dtype=np.float32 if f32 else np.float64).reshape(case["shape"])
        p = zc.Plan([(1, zc.F32 if f32 else zc.F64, tuple(case["shape"]))], [],
                    [(case["prim"], [1], 10, case["axis"], case["keepdims"])], [10])
        (got,) = p.run([torch.from_numpy(x).cuda()])
        assert list(got.shape) == case["want_shape"], case["name"]
        g = got.cpu().numpy().astype(np.float64).ravel()
        assert np.all(np.abs(g - case["want"]) <= case["tol"]), (case["name"], g)


@pytest.mark.parametrize("axis", [-2, 0, 1, 2, -1])
@pytest.mark.parametrize("prim", ["argmax", "argmin"])
@pytest.mark.parametrize("dt", ["f32", "f64"])
def test_arg_reductions_match_the_oracle(zc, axis, prim, dt):
    """argmax / argmin fused with an element-wise producer (abs, so +-v tie)
    over small integers (many ties), NaNs at scattered places and at the
    start of some rows: the index zpu's sequential scan returns."""
    rng = np.random.default_rng(7 + axis)
    shape = (9, 37, 70)
    npdt = np.float32 if dt == "f32" else np.float64
    x = rng.integers(-6, 7, size=shape).astype(npdt)
    nan_at = rng.random(shape) < 0.01
    x[nan_at] = np.nan
    x[0, 0, :] = np.nan  # position 0 of every axis-2 row of x[0, 0]
    x[:, 0, 0] = np.nan  # position 0 along axis 0 / 1 for some outputs
    p = zc.Plan([(1, zc.F32 if dt == "f32" else zc.F64, shape)], [],
                [("abs", [1], 10, -2, 0), (prim, [10], 11, axis, 0)], [11, 10])
    red, a = p.run([torch.from_numpy(x).cuda()])
    want = zo.arg_reduce(np.abs(x), axis, want_max=prim == "argmax")
    assert red.dtype == torch.int64
    assert tuple(red.shape) == want.shape
    assert np.array_equal(red.cpu().numpy(), want)
    assert np.array_equal(a.cpu().numpy(), np.abs(x), equal_nan=True)


@pytest.mark.parametrize("prim", ["argmax", "argmin"])
def test_full_arg_reduction_across_blocks(zc, prim):
    """A full argmax over 2^22 + 5 elements (many blocks): the extreme value
    planted at several places, the first of them wins; a NaN at index 0
    gives 0."""
    n = (1 << 22) + 5
    x = zo.uniform_range(33, n, -1.0, 1.0)
    v = 7.5 if prim == "argmax" else -7.5
    places = [3_000_001, 17, 4_194_300, 1_048_576]
    x[places] = v
    p = zc.Plan([(1, zc.F32, (n,))], [], [(prim, [1], 10, -2, 0)], [10])
    (got,) = p.run([torch.from_numpy(x).cuda()])
    assert int(got.cpu()) == min(places)
    x[0] = np.nan
    (got,) = p.run([torch.from_numpy(x).cuda()])
    assert int(got.cpu()) == 0


@pytest.mark.parametrize("prim,axis,keep", [("sum", -2, 0), ("sum", -2, 1), ("max_reduce", 0, 0), ("sum", -1, 1),
                                            ("argmax", -2, 0), ("argmin", 1, 0)])
def test_reductions_fold_payload_axes_under_vmap(zc, prim, axis, keep):
    """With batch_depth 1 (vmap) AXIS_NONE folds the payload axes only and a
    non-negative axis counts from the first payload axis (ops.axesMaskOf,
    src/zpu/ops.zig:630-642)."""
    shape = (4, 6, 10)
    x = zo.uniform_range(5, int(np.prod(shape)), -2.0, 2.0).reshape(shape)
    p = zc.Plan([(1, zc.F32, shape, 1)], [], [(prim, [1], 10, axis, keep)], [10])
    (got,) = p.run([torch.from_numpy(x).cuda()])
    if prim in ("argmax", "argmin"):
        want = zo.arg_reduce(x, axis, depth=1, want_max=prim == "argmax")
        assert np.array_equal(got.cpu().numpy(), want)
    else:
        want = zo.reduce_axis(x, prim, axis, keep, depth=1)
        assert tuple(got.shape) == want.shape
        assert np.allclose(got.cpu().numpy(), want, rtol=2e-6, atol=1e-6)


def test_selection_snapshots_on_device(zc, golden):
    """tests/snap/zpu.zig:69-75 as jit plans (f64 spread(8)): where(gt(x, 0),
    x, neg(x)) -- a bool value inside one region --, clamp as maximum then
    minimum with captured bounds, lerp as a + t (b - a)."""
    x = np.array(golden["inputs"]["spread8"], dtype=np.float64)
    xd = torch.from_numpy(x).cuda()
    args = [(1, zc.F64, (8,))]
    plans = {
        "where": zc.Plan(args, [(2, np.float64(0.0))],
                         [("gt", [1, 2], 10, -2, 0), ("neg", [1], 11, -2, 0), ("where", [10, 1, 11], 12, -2, 0)], [12]),
        "clamp": zc.Plan(args, [(2, np.float64(-0.5)), (3, np.float64(0.5))],
                         [("maximum", [1, 2], 10, -2, 0), ("minimum", [10, 3], 11, -2, 0)], [11]),
        "lerp": zc.Plan(args, [(2, np.float64(0.25))],
                        [("neg", [1], 10, -2, 0), ("sub", [10, 1], 11, -2, 0), ("mul", [11, 2], 12, -2, 0),
                         ("add", [1, 12], 13, -2, 0)], [13]),
    }
    for name, p in plans.items():
        assert p.num_kernels() == 1, name
        (got,) = p.run([xd])
        s = golden["snapshots"]["zpu/ops/" + name]
        g = got.cpu().numpy()
        assert np.all(np.abs(g - s["values"]) <= s["tol"] * np.maximum(1, np.abs(g))), name


def test_predicate_known_answers_on_device(zc, golden):
    k = {c["name"]: c for c in golden["pred_known"]}
    a = torch.tensor(k["gt(a, 3)"]["x"], dtype=torch.float64, device="cuda").reshape(2, 3)
    p = zc.Plan([(1, zc.F64, (2, 3))], [(2, np.float64(3.0))],
                [("gt", [1, 2], 10, -2, 0), ("neg", [1], 11, -2, 0), ("where", [10, 1, 11], 12, -2, 0)], [10, 12])
    cond, w = p.run([a])
    assert cond.dtype == torch.bool
    assert cond.cpu().numpy().astype(np.float64).ravel().tolist() == k["gt(a, 3)"]["want"]
    assert w.cpu().numpy().ravel().tolist() == k["where(gt(a, 3), a, neg(a))"]["want"]
    i = torch.tensor(k["any(lt(i, 3))"]["x"], dtype=torch.float64, device="cuda").reshape(2, 2)
    for prim, key in (("any_reduce", "any(lt(i, 3))"), ("all_reduce", "all(lt(i, 3))")):
        q = zc.Plan([(1, zc.F64, (2, 2))], [(2, np.float64(3.0))],
                    [("lt", [1, 2], 10, -2, 0), (prim, [10], 11, -2, 0)], [11])
        (r,) = q.run([i])
        assert r.dtype == torch.bool and [float(r.cpu())] == k[key]["want"]


PRED2 = ["eq", "ne", "lt", "le", "gt", "ge", "logical_and", "logical_or", "logical_xor"]


@pytest.mark.parametrize("dt", ["f32", "f64"])
def test_predicates_match_the_oracle(zc, dt):
    """Every predicate over values with NaN, +-0, +-inf and ties, broadcast
    against a row; unary predicates; where on a NaN condition."""
    npdt = np.float32 if dt == "f32" else np.float64
    code = zc.F32 if dt == "f32" else zc.F64
    rng = np.random.default_rng(3)
    x = rng.integers(-2, 3, size=(64, 33)).astype(npdt)
    x[rng.random(x.shape) < 0.05] = np.nan
    x[0, :4] = [np.inf, -np.inf, -0.0, 0.0]
    y = rng.integers(-2, 3, size=(33,)).astype(npdt)
    y[5] = np.nan
    xd, yd = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    steps = [(prim, [1, 2], 10 + i, -2, 0) for i, prim in enumerate(PRED2)]
    steps += [(prim, [1], 20 + i, -2, 0) for i, prim in enumerate(["isnan", "isinf", "isfinite", "logical_not"])]
    steps += [("where", [1, 1, 2], 30, -2, 0)]  # x itself as the condition: NaN is true
    outs = [10 + i for i in range(len(PRED2))] + [20, 21, 22, 23, 30]
    p = zc.Plan([(1, code, (64, 33)), (2, code, (33,))], [], steps, outs)
    got = p.run([xd, yd])
    for i, prim in enumerate(PRED2):
        assert got[i].dtype == torch.bool
        assert np.array_equal(got[i].cpu().numpy(), zo.predicate(prim, x, y)), prim
    for i, prim in enumerate(["isnan", "isinf", "isfinite", "logical_not"]):
        assert np.array_equal(got[len(PRED2) + i].cpu().numpy(), zo.predicate(prim, x)), prim
    w = got[-1].cpu().numpy()
    assert np.array_equal(w, zo.where(x, x, np.broadcast_to(y, x.shape)).astype(npdt), equal_nan=True)


@pytest.mark.parametrize("prim", ["any_reduce", "all_reduce"])
@pytest.mark.parametrize("axis,keep", [(-2, 0), (0, 0), (1, 1), (2, 0), (-1, 1)])
def test_any_all_match_the_oracle(zc, prim, axis, keep):
    """any / all of a comparison (bool values) and of floats (x != 0, NaN
    true), over every axis kind, with a bool argument as well."""
    rng = np.random.default_rng(11)
    shape = (5, 40, 70)
    x = (rng.random(shape) < 0.03).astype(np.float32) * rng.choice([1.0, np.nan, -2.0], size=shape).astype(np.float32)
    x[2] = 1.0  # an all-true slab
    m = rng.random(shape) < 0.5
    p = zc.Plan([(1, zc.F32, shape), (2, zc.DT_BOOL, shape)], [(3, np.float32(0.0))],
                [("ne", [1, 3], 10, -2, 0), (prim, [10], 11, axis, keep), (prim, [1], 12, axis, keep),
                 ("logical_and", [2, 10], 13, -2, 0), (prim, [13], 14, axis, keep)], [11, 12, 14])
    a, b, c = p.run([torch.from_numpy(x).cuda(), torch.from_numpy(m).cuda()])
    want = zo.reduce_bool(zo.predicate("ne", x, 0.0), prim, axis, keep)
    assert a.dtype == torch.bool and tuple(a.shape) == want.shape
    assert np.array_equal(a.cpu().numpy(), want)
    assert np.array_equal(b.cpu().numpy(), zo.reduce_bool(x, prim, axis, keep))
    assert np.array_equal(c.cpu().numpy(), zo.reduce_bool(m & (x != 0), prim, axis, keep))


def test_i64_operands_follow_zpus_promotion(zc):
    """eq(argmax(logits, 1), labels) -- a classifier's hits -- and i64
    values against floats: argmax's i64 result feeds the next region as an
    input read as zpu reads it (readAtF64), each result typed by
    DType.promote / binaryOutDType (dtype.zig:89-104, ops.zig:275-285)."""
    logits = zo.uniform_range(71, 64 * 10, -3.0, 3.0).reshape(64, 10).astype(np.float32)
    lab = (np.arange(64, dtype=np.int64) * 7) % 10
    scale = zo.uniform_range(72, 64, -2.0, 2.0).astype(np.float32)
    F = zc.F32
    steps = [("argmax", [1], 10, 1, 0), ("eq", [10, 2], 11, -2, 0), ("cast_op", [11], 12, zc.F32, 0),
             ("sum", [12], 13, -2, 0), ("mul", [10, 3], 14, -2, 0), ("ge", [10, 3], 15, -2, 0)]
    p = zc.Plan([(1, F, (64, 10)), (2, zc.DT_I64, (64,)), (3, F, (64,))], [], steps, [10, 11, 13, 14, 15])
    am, hit, nhit, prod, ge = [o.cpu().numpy() for o in p.run([torch.from_numpy(v).cuda() for v in (logits, lab, scale)])]
    want = zo.arg_reduce(logits, 1, want_max=True)
    assert np.array_equal(am, want)
    assert hit.dtype == np.bool_ and np.array_equal(hit, want == lab) and 0 < hit.sum() < 64
    assert float(nhit) == float(np.sum(want == lab))
    wide = want.astype(np.float64)
    assert prod.dtype == np.float32 and np.array_equal(prod, (wide * scale.astype(np.float64)).astype(np.float32))
    assert np.array_equal(ge, wide >= scale.astype(np.float64))
    # two i64 values: compared in f64, exact beyond 2^24
    x = np.array([2 ** 40 + 1, 2 ** 40, -(2 ** 30) - 3, 5], dtype=np.int64)
    y = np.array([2 ** 40, 2 ** 40, -(2 ** 30) - 2, 5], dtype=np.int64)
    q = zc.Plan([(1, zc.DT_I64, (4,)), (2, zc.DT_I64, (4,))], [],
                [("eq", [1, 2], 10, -2, 0), ("lt", [1, 2], 11, -2, 0)], [10, 11])
    e, l = [o.cpu().numpy() for o in q.run([torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()])]
    assert e.tolist() == [False, True, False, True] and l.tolist() == [False, False, True, False]


def test_i64_arithmetic_is_zpus_f64_compute_and_write_back(zc):
    """Steps of i64 values alone outside scalar.binary's integer set: each
    element computed from the operands read as f64 and written back as zpu
    writes an i64 (0 for NaN, clamp, truncate; scalar.zig:7-27) -- recip(2)
    is 0 before it is multiplied;
    div and the float-only prims give f32 (ops.zig:268-285); where takes
    the promoted type of its branches."""
    a = np.array([7, -7, 2 ** 40 + 3, -(2 ** 52) + 1, 0, 9], dtype=np.int64)
    b = np.array([2, 3, -5, 4, 1, -9], dtype=np.int64)
    steps = [("add", [1, 2], 10, -2, 0), ("mul", [1, 2], 11, -2, 0), ("mod_op", [1, 2], 12, -2, 0),
             ("recip", [2], 13, -2, 0), ("mul", [13, 1], 14, -2, 0), ("neg", [1], 15, -2, 0),
             ("square", [2], 16, -2, 0), ("maximum", [1, 2], 17, -2, 0), ("sign", [1], 18, -2, 0),
             ("div", [1, 2], 19, -2, 0), ("exp", [2], 20, -2, 0), ("ne", [15, 1], 21, -2, 0)]
    p = zc.Plan([(1, zc.DT_I64, (6,)), (2, zc.DT_I64, (6,))], [], steps, list(range(10, 22)))
    outs = [o.cpu().numpy() for o in p.run([torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])]
    af, bf = a.astype(np.float64), b.astype(np.float64)

    def i64(v):
        return zo.from_f64(v, np.int64)

    rec = i64(zo.unary("recip", bf))
    want = [i64(zo.binary("add", af, bf)), i64(zo.binary("mul", af, bf)), i64(zo.binary("mod_op", af, bf)), rec,
            i64(zo.binary("mul", rec.astype(np.float64), af)), i64(zo.unary("neg", af)),
            i64(zo.unary("square", bf)), i64(zo.binary("maximum", af, bf)), i64(zo.unary("sign", af))]
    for k, w in enumerate(want):
        assert outs[k].dtype == np.int64 and np.array_equal(outs[k], w), (steps[k], outs[k], w)
    assert rec.tolist() == [0, 0, 0, 0, 1, 0] and outs[4].tolist() == [0, 0, 0, 0, 0, 0]
    assert outs[9].dtype == np.float32
    np.testing.assert_allclose(outs[9], zo.from_f64(zo.binary("div", af, bf), np.float32), rtol=2.4e-7)
    np.testing.assert_allclose(outs[10], zo.from_f64(zo.unary("exp", bf), np.float32), rtol=4.8e-7)
    assert outs[11].dtype == np.bool_ and outs[11].tolist() == [True, True, True, True, False, True]
    # where: DType.promote of the branches (ops.zig:572-576)
    c = np.array([True, False, True, False, True, False])
    x = np.array([0.5, -1.5, 2.0, 3.25, -4.0, 9.5], dtype=np.float32)
    q = zc.Plan([(1, zc.DT_I64, (6,)), (2, zc.DT_I64, (6,)), (3, zc.DT_BOOL, (6,)), (4, zc.F32, (6,))], [],
                [("where", [3, 1, 2], 10, -2, 0), ("where", [3, 1, 4], 11, -2, 0)], [10, 11])
    w1, w2 = [o.cpu().numpy() for o in q.run([torch.from_numpy(v).cuda() for v in (a, b, c, x)])]
    assert w1.dtype == np.int64 and np.array_equal(w1, np.where(c, a, b))
    assert w2.dtype == np.float32 and np.array_equal(w2, np.where(c, zo.from_f64(af, np.float32), x))


def _i64_run(zc, args, steps, outs, arrays):
    p = zc.Plan(args, [], steps, outs)
    return p, [o.cpu().numpy() for o in p.run([torch.from_numpy(v).cuda() for v in arrays])]


def test_i64_steps_run_on_the_integers(zc):
    """scalar.binary / scalar.unary of two i64 values (scalar.zig:262-302):
    + - * wrap in two's complement, mod with a zero divisor gives a and
    otherwise the divisor's sign, max / min / abs / sign / relu on the
    integers -- exact beyond 2^53, where an f64 computation would round;
    neg and the rest go through f64 and fromF64 (neg(minInt) clamps)."""
    big = 2 ** 62
    a = np.array([big + 5, -big - 7, 2 ** 53 + 1, -3, 0, 9, 7, -(2 ** 63), 2 ** 63 - 1, 12345678901234567,
                  -12345678901234567, 2 ** 53 + 3], dtype=np.int64)
    b = np.array([3, -big, 1, 4, -1, -9, 0, 5, -1, 99991, 99991, -(2 ** 53) - 1], dtype=np.int64)
    names = ["add", "sub", "mul", "mod_op", "maximum", "minimum"]
    steps = [(nm, [1, 2], 10 + k, -2, 0) for k, nm in enumerate(names)]
    unames = ["abs", "sign", "relu", "neg", "square"]
    steps += [(nm, [1], 20 + k, -2, 0) for k, nm in enumerate(unames)]
    outs = [10 + k for k in range(len(names))] + [20 + k for k in range(len(unames))]
    p, got = _i64_run(zc, [(1, zc.DT_I64, a.shape), (2, zc.DT_I64, b.shape)], steps, outs, (a, b))
    assert "w64" in p.describe() and "iadd(" in p.describe()
    for k, nm in enumerate(names):
        want = zo.binary_i64(nm, a, b)
        assert got[k].dtype == np.int64 and np.array_equal(got[k], want), (nm, got[k], want)
    for k, nm in enumerate(unames):
        want = zo.unary_i64(nm, a)
        assert np.array_equal(got[len(names) + k], want), (nm, got[len(names) + k], want)
    # the integer result is not the f64 one: 2^53 + 1 + 1 and a wrapped sum
    assert got[0][2] == 2 ** 53 + 2 and got[0][0] == zo.binary_i64("add", a[:1], b[:1])[0]
    assert got[1][8] == np.int64(-(2 ** 63)) and got[3][2] == 0 and got[3][6] == 7


def test_i64_pow_is_zigs_pow_written_back(zc):
    """pow of two i64 values: std.math.pow(f64) on the operands read as f64
    (scalar.zig:151-153), written back by fromF64 -- the repeated-squaring
    product with its separate binary exponent, so odd powers above 2^53 have
    zpu's bits, negative exponents truncate to 0 (or +-1), 0^-k is +inf and
    clamps to maxInt."""
    x = np.array([-3, 2, 7, 10, -2, 3, 0, 1, 5, 2, -1, 0, 11, 2, -7, 3], dtype=np.int64)
    y = np.array([3, 10, 19, 18, 63, -1, 0, 40, 27, 62, -5, -3, 17, 64, 21, 39], dtype=np.int64)
    p, (got, f) = _i64_run(zc, [(1, zc.DT_I64, x.shape), (2, zc.DT_I64, y.shape), (3, zc.F32, x.shape)],
                           [("pow", [1, 2], 10, -2, 0), ("pow", [1, 3], 11, -2, 0)], [10, 11],
                           (x, y, y.astype(np.float32) * 0.25))
    assert "zpow(" in p.describe()
    want = zo.binary_i64("pow", x, y)
    assert got.dtype == np.int64 and np.array_equal(got, want), (got, want)
    assert got[0] == -27 and got[1] == 1024 and got[11] == 2 ** 63 - 1 and got[10] == -1
    # an i64 base against an f32 exponent: the f32 type, std.math.pow in f64
    # rounded once (binaryKernelF64, ops.zig:245-253)
    wantf = zo.from_f64(zo.binary("pow", x.astype(np.float64), (y.astype(np.float32) * 0.25).astype(np.float64)),
                        np.float32)
    assert f.dtype == np.float32
    fin = np.isfinite(wantf)
    assert np.array_equal(np.isnan(f), np.isnan(wantf))
    assert ulp_diff_f32(f[fin], wantf[fin]).max() <= 1


def test_i64_reductions_wrap_in_the_integer_type(zc):
    """sum / prod / max / min of i64 values stay i64 (reduceOutDType,
    ops.zig:813-818) and run on the integers: +% and *% wrap (reduceStep,
    ops.zig:686-700), so the result is exact where an f64 sum would round;
    every axis form, keepdims, and the empty reduction's identities written
    through fromF64 (0, 1, minInt, maxInt; ops.zig:822-838)."""
    rng = np.random.default_rng(7)
    x = rng.integers(-(2 ** 62), 2 ** 62, size=(6, 7, 5), dtype=np.int64)
    s = rng.integers(-9, 10, size=(6, 7, 5), dtype=np.int64)
    args = [(1, zc.DT_I64, x.shape), (2, zc.DT_I64, s.shape)]
    cases = [(prim, axis, keep) for prim in ("sum", "prod_op", "max_reduce", "min_reduce")
             for axis, keep in ((-2, 0), (0, 0), (1, 1), (-1, 0))]
    for prim, axis, keep in cases:
        for arr in (x, s):
            p, (got,) = _i64_run(zc, [(1, zc.DT_I64, arr.shape)], [(prim, [1], 10, axis, keep)], [10], (arr,))
            want = zo.reduce_i64(arr, prim, axis, bool(keep))
            assert got.dtype == np.int64 and got.shape == np.shape(want), (prim, axis, got.shape)
            assert np.array_equal(got, want), (prim, axis, keep)
    p = zc.Plan(args, [], [("sum", [1], 10, -2, 0)], [10])
    assert "red=isum" in p.describe()
    # fused: sum(a * b + a) of i64 values, one region on 64-bit words
    p, (got,) = _i64_run(zc, args, [("mul", [1, 2], 10, -2, 0), ("add", [10, 1], 11, -2, 0),
                                    ("sum", [11], 12, 1, 0)], [12], (x, s))
    assert p.num_kernels() == 1
    want = zo.reduce_i64(zo.binary_i64("add", zo.binary_i64("mul", x, s), x), "sum", 1)
    assert np.array_equal(got, want)
    # empty reductions: the identities as zpu writes them into an i64
    e = np.zeros((0, 4), dtype=np.int64)
    for prim, ident in (("sum", 0), ("prod_op", 1), ("max_reduce", -(2 ** 63)), ("min_reduce", 2 ** 63 - 1)):
        _, (got,) = _i64_run(zc, [(1, zc.DT_I64, e.shape)], [(prim, [1], 10, -2, 0)], [10], (e,))
        assert got.dtype == np.int64 and int(got) == ident, prim
        _, (got,) = _i64_run(zc, [(1, zc.DT_I64, e.shape)], [(prim, [1], 10, 0, 0)], [10], (e,))
        assert got.tolist() == [ident] * 4, prim


def test_i64_cumsum_and_where_as_zpu_writes_them(zc):
    """cumsum of i64 (ops.cumsum, ops.zig:2032-2057): an f64 running sum,
    each prefix written by fromF64 -- it rounds above 2^53 as zpu's does;
    where of two i64 branches reads and writes through f64 (ops.zig:572-590),
    argmax feeding i64 arithmetic in the next region."""
    x = np.array([[2 ** 53, 1, 1, 1, -5], [3, -(2 ** 62), -(2 ** 62), -(2 ** 62), 7]], dtype=np.int64)
    for axis, flags in ((1, 0), (0, 0), (1, REVERSE), (-1, 0)):
        _, (got,) = _i64_run(zc, [(1, zc.DT_I64, x.shape)], [("cumsum", [1], 10, axis, flags)], [10], (x,))
        want = zo.cumsum(x, axis, reverse=bool(flags))
        assert got.dtype == np.int64 and np.array_equal(got, want), (axis, flags, got, want)
    assert zo.cumsum(x, 1)[0, 1] == 2 ** 53  # 2^53 + 1 rounds in the f64 accumulator
    c = np.array([True, False, True, False, True])
    a = np.array([2 ** 53 + 1, 4, -(2 ** 63), 2 ** 63 - 1, 6], dtype=np.int64)
    b = np.array([1, 2 ** 60 + 1, 3, 5, -1], dtype=np.int64)
    _, (w,) = _i64_run(zc, [(1, zc.DT_BOOL, c.shape), (2, zc.DT_I64, a.shape), (3, zc.DT_I64, b.shape)],
                       [("where", [1, 2, 3], 10, -2, 0)], [10], (c, a, b))
    assert np.array_equal(w, zo.where_i64(c, a, b))
    logits = zo.uniform_range(91, 16 * 9, -1.0, 1.0).reshape(16, 9).astype(np.float32)
    off = np.arange(16, dtype=np.int64) * (2 ** 55 + 3)
    p, (am, r) = _i64_run(zc, [(1, zc.F32, logits.shape), (2, zc.DT_I64, off.shape)],
                          [("argmax", [1], 10, 1, 0), ("add", [10, 2], 11, -2, 0), ("mul", [11, 11], 12, -2, 0),
                           ("max_reduce", [12], 13, -2, 0)], [10, 13], (logits, off))
    want_am = zo.arg_reduce(logits, 1, want_max=True)
    assert np.array_equal(am, want_am)
    t = zo.binary_i64("add", want_am, off)
    assert int(r) == int(zo.reduce_i64(zo.binary_i64("mul", t, t), "max_reduce"))


REVERSE = 32  # prims.Attrs.REVERSE


def test_cumsum_snapshots_and_known_answers_on_device(zc, golden):
    x = torch.tensor(golden["inputs"]["spread12"], dtype=torch.float64, device="cuda").reshape(3, 4)
    for name, flags in (("cumsum-axis1", 0), ("cumsum-reverse", REVERSE)):
        p = zc.Plan([(1, zc.F64, (3, 4))], [], [("cumsum", [1], 10, 1, flags)], [10])
        assert "cumsum" in p.describe()
        (got,) = p.run([x])
        s = golden["snapshots"]["zpu/reduce/" + name]
        g = got.cpu().numpy().ravel()
        assert np.all(np.abs(g - s["values"]) <= s["tol"] * np.maximum(1, np.abs(g))), name
    for c in golden["cumsum_known"]:
        a = torch.tensor(c["x"], dtype=torch.float64, device="cuda").reshape(c["shape"])
        p = zc.Plan([(1, zc.F64, tuple(c["shape"]))], [], [("cumsum", [1], 10, c["axis"], REVERSE * c["reverse"])],
                    [10])
        (got,) = p.run([a])
        assert got.cpu().numpy().ravel().tolist() == c["want"]


@pytest.mark.parametrize("axis", [0, 1, 2, -1, -2])
@pytest.mark.parametrize("reverse", [0, 1])
@pytest.mark.parametrize("dt", ["f32", "f64"])
def test_cumsum_is_bit_exact(zc, axis, reverse, dt):
    """zpu's f64 running sum rounded per element, along any axis, forward and
    reverse, fed by an element-wise region and feeding one (exp of the
    prefix sums) -- every element bit-equal to the oracle."""
    npdt = np.float32 if dt == "f32" else np.float64
    shape = (6, 257, 40)
    x = zo.uniform_range(9, int(np.prod(shape)), -1.0, 1.0, npdt).reshape(shape)
    code = zc.F32 if dt == "f32" else zc.F64
    p = zc.Plan([(1, code, shape)], [],
                [("square", [1], 10, -2, 0), ("cumsum", [10], 11, axis, REVERSE * reverse),
                 ("neg", [11], 12, -2, 0)], [11, 12])
    assert p.num_kernels() == 3
    c, n = p.run([torch.from_numpy(x).cuda()])
    want = zo.cumsum((x * x).astype(npdt), axis, bool(reverse))
    assert np.array_equal(c.cpu().numpy(), want)
    assert np.array_equal(n.cpu().numpy(), -want)


def test_cumsum_under_vmap_counts_payload_axes(zc):
    shape = (3, 5, 7)
    x = zo.uniform_range(10, 105, -1.0, 1.0, np.float64).reshape(shape)
    p = zc.Plan([(1, zc.F64, shape, 1)], [], [("cumsum", [1], 10, 0, 0)], [10])  # payload axis 0 = axis 1
    (got,) = p.run([torch.from_numpy(x).cuda()])
    assert np.array_equal(got.cpu().numpy(), zo.cumsum(x, 0, depth=1))


def test_jit_mlp_loss_lowers_to_five_launches(zc):
    """The jitted function of the reference's `jit(grad MLP) f32` benchmark
    case (bench/bench.zig:137-150, 230-234; dims 64 -> 64 -> 10, batch 64):
    dense, gelu (nn.zig:39-53: x * 0.5 * (1 + erf(x / sqrt 2))), dense,
    square, mean over the last axis, sumAll -- the plan zpu's tracer records,
    scalars as captured blobs.  Lowered to gemm, one fused region, gemm, one
    fused region with the row sum, one region with the full sum; checked
    against the oracle's f32 step-by-step evaluation at 1e-5 relative (the
    device sums in f64, zpu in f32)."""
    B, I, H, O = 64, 64, 64, 10
    rng = np.random.default_rng(21)
    x = rng.standard_normal((B, I)).astype(np.float32)
    w1 = rng.standard_normal((I, H)).astype(np.float32)
    b1 = np.zeros(H, np.float32)
    w2 = rng.standard_normal((H, O)).astype(np.float32)
    b2 = np.zeros(O, np.float32)
    F = zc.F32
    args = [(1, F, (B, I)), (2, F, (I, H)), (3, F, (H,)), (4, F, (H, O)), (5, F, (O,))]
    blobs = [(6, np.float32(1.0 / np.sqrt(2.0))), (7, np.float32(1.0)), (8, np.float32(0.5)),
             (9, np.float32(1.0 / O))]
    steps = [("matmul", [1, 2], 10, -2, 0), ("add", [10, 3], 11, -2, 0),
             ("mul", [11, 6], 12, -2, 0), ("erf", [12], 13, -2, 0), ("add", [7, 13], 14, -2, 0),
             ("mul", [11, 8], 15, -2, 0), ("mul", [15, 14], 16, -2, 0),
             ("matmul", [16, 4], 17, -2, 0), ("add", [17, 5], 18, -2, 0),
             ("square", [18], 19, -2, 0), ("sum", [19], 20, -1, 0), ("mul", [20, 9], 21, -2, 0),
             ("sum", [21], 22, -2, 0)]
    p = zc.Plan(args, blobs, steps, [22])
    assert p.num_kernels() == 5, p.describe()
    (got,) = p.run([torch.from_numpy(a).cuda() for a in (x, w1, b1, w2, b2)])
    f32 = np.float32
    h = (zo.matmul(x, w1) + b1).astype(f32)
    e = zo.unary("erf", (h * f32(1.0 / np.sqrt(2.0))).astype(f32))
    act = ((h * f32(0.5)).astype(f32) * (f32(1.0) + e).astype(f32)).astype(f32)
    y = (zo.matmul(act, w2) + b2).astype(f32)
    per_row = ((y * y).astype(f32).astype(np.float64).sum(-1)).astype(f32)
    want = float(((per_row * f32(1.0 / O)).astype(f32)).astype(np.float64).sum())
    assert abs(float(got.cpu()) - want) <= 1e-5 * abs(want), (float(got.cpu()), want)


def test_views_fold_into_regions(zc):
    """transpose / reshape / broadcast / expand_dims / squeeze (ops.zig:
    1343-1555) are views over the producer's HBM; the regions after them
    read through the view's strides, and outputs that are views are copied
    out contiguous."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((6, 8, 10)).astype(np.float32)
    bias = rng.standard_normal(10).astype(np.float32)
    F = zc.F32
    steps = [("transpose", [1], 10, -2, 0, {"perm": [2, 0, 1]}),       # [10, 6, 8], strided
             ("exp", [10], 11, -2, 0),                                    # region through the view
             ("reshape", [10], 12, -2, 0, {"shape": [10, -1]}),          # strided -> copied, [10, 48]
             ("expand_dims", [2], 13, 0, 0),                              # [1, 10]
             ("broadcast", [13], 14, -2, 0, {"shape": [48, 10]}),        # stride 0 rows
             ("transpose", [12], 15, -2, 0, {"perm": [1, 0]}),           # [48, 10] view of the copy
             ("add", [15, 14], 16, -2, 0),
             ("expand_dims", [16], 17, -1, 0),                            # [48, 10, 1]
             ("squeeze", [17], 18, 2, 0),                                 # [48, 10]
             ("sum", [18], 19, 0, 0)]
    p = zc.Plan([(1, F, (6, 8, 10)), (2, F, (10,))], [], steps, [11, 12, 14, 18, 19, 10])
    outs = p.run([torch.from_numpy(x).cuda(), torch.from_numpy(bias).cuda()])
    xt = np.transpose(x, (2, 0, 1))
    want = [zo.unary("exp", np.ascontiguousarray(xt)), xt.reshape(10, 48),
            np.broadcast_to(bias[None, :], (48, 10)), None, None, xt]
    s18 = (xt.reshape(10, 48).T + bias[None, :]).astype(np.float32)
    want[3] = s18
    want[4] = s18.astype(np.float64).sum(0)
    got = [o.cpu().numpy() for o in outs]
    assert ulp_diff_f32(got[0], want[0]).max() <= 1
    for i in (1, 2, 3, 5):
        assert got[i].shape == want[i].shape and np.array_equal(got[i], want[i]), i
    assert np.allclose(got[4], want[4], rtol=1e-6, atol=1e-6)
    assert "copy (reshape of a strided view)" in p.describe()


def test_transposed_matmul_operands_are_read_in_place(zc):
    """The matmul VJP's swapLastTwo views (transpose of the last two axes)
    feed the GEMM with no copy: one launch."""
    a = zo.uniform_range(41, 96 * 64, -1.0, 1.0).reshape(96, 64)
    b = zo.uniform_range(42, 96 * 40, -1.0, 1.0).reshape(96, 40)
    F = zc.F32
    p = zc.Plan([(1, F, (96, 64)), (2, F, (96, 40))], [],
                [("transpose", [1], 10, -2, 0, {"perm": [1, 0]}), ("matmul", [10, 2], 11, -2, 0)], [11])
    assert p.num_kernels() == 1, p.describe()
    (c,) = p.run([torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    want = a.T.astype(np.float64) @ b.astype(np.float64)
    assert np.linalg.norm(c.cpu().numpy() - want) <= 1e-5 * np.linalg.norm(want)


def test_broadcast_matmul_operand_is_copied(zc):
    """A view with a zero stride inside the matrix axes has no leading
    dimension a GEMM can take: the plan copies it first."""
    v = zo.uniform_range(43, 32, -1.0, 1.0)
    b = zo.uniform_range(44, 32 * 16, -1.0, 1.0).reshape(32, 16)
    F = zc.F32
    p = zc.Plan([(1, F, (32,)), (2, F, (32, 16))], [],
                [("broadcast", [1], 10, -2, 0, {"shape": [24, 32]}), ("matmul", [10, 2], 11, -2, 0)], [11])
    assert "copy (matmul operand)" in p.describe()
    (c,) = p.run([torch.from_numpy(v).cuda(), torch.from_numpy(b).cuda()])
    want = np.broadcast_to(v, (24, 32)).astype(np.float64) @ b.astype(np.float64)
    assert np.linalg.norm(c.cpu().numpy() - want) <= 1e-5 * np.linalg.norm(want)


def test_views_under_vmap_use_payload_axes(zc):
    """batch_depth 1: transpose, reshape, expand_dims and squeeze take
    payload-relative arguments and keep the batch axis first.  A reshape
    target gets the batch axes in front only when it has the payload's rank
    (ops.zig:1345-1350); another rank is zpu's ShapeMismatch here too."""
    x = zo.uniform_range(45, 3 * 4 * 5, -1.0, 1.0).reshape(3, 4, 5)
    F = zc.F32
    steps = [("transpose", [1], 10, -2, 0, {"perm": [1, 0]}),   # payload perm -> (0, 2, 1)
             ("reshape", [10], 11, -2, 0, {"shape": [2, 10]}),   # payload shape -> [3, 2, 10]
             ("expand_dims", [1], 12, 0, 0),                      # -> [3, 1, 4, 5]
             ("squeeze", [12], 13, 0, 0),                         # -> [3, 4, 5]
             ("neg", [11], 14, -2, 0)]
    p = zc.Plan([(1, F, (3, 4, 5), 1)], [], steps, [10, 11, 12, 13, 14])
    t, r, e, q, n = [o.cpu().numpy() for o in p.run([torch.from_numpy(x).cuda()])]
    xt = np.transpose(x, (0, 2, 1))
    assert np.array_equal(t, xt) and np.array_equal(r, xt.reshape(3, 2, 10))
    assert np.array_equal(e, x[:, None]) and np.array_equal(q, x) and np.array_equal(n, -xt.reshape(3, 2, 10))
    with pytest.raises(zc.ZpuCudaError) as err:
        zc.Plan([(1, F, (3, 4, 5), 1)], [], [("reshape", [1], 10, -2, 0, {"shape": [20]})], [10])
    assert err.value.status == 2  # ShapeMismatch


def test_argument_output_is_copied(zc):
    x = torch.randn(7, 9, device="cuda")
    p = zc.Plan([(1, zc.F32, (7, 9))], [], [("neg", [1], 10, -2, 0)], [1, 10, 1])
    a, n, b = p.run([x])
    assert torch.equal(a, x) and torch.equal(b, x) and torch.equal(n, -x)


def test_flip_copy_and_cast_steps(zc):
    """flip / reverse (negative-stride views, ops.zig:2019-2030, 2198), copy
    (the input itself) and cast_op (a converting copy, ops.zig:2062-2071 --
    Attrs.axis is the type): an i64 argument cast to f32 feeds a region, and
    a flipped view feeds a region, a GEMM (copied: negative strides) and an
    output."""
    x = zo.uniform_range(51, 12 * 7, -3.0, 3.0).reshape(12, 7)
    lab = np.arange(12, dtype=np.int64) * 3 - 5
    w = zo.uniform_range(52, 7 * 5, -1.0, 1.0).reshape(7, 5)
    F = zc.F32
    steps = [("flip", [1], 10, 0, 0), ("abs", [10], 11, -2, 0), ("reverse", [10], 12, -1, 0),
             ("copy", [12], 13, -2, 0), ("cast_op", [2], 14, zc.F32, 0), ("mul", [14, 14], 15, -2, 0),
             ("matmul", [10, 3], 16, -2, 0), ("cast_op", [1], 17, zc.F32, 0), ("cast_op", [1], 18, zc.DT_BOOL, 0)]
    p = zc.Plan([(1, F, (12, 7)), (2, zc.DT_I64, (12,)), (3, F, (7, 5))], [], steps, [10, 11, 13, 15, 16, 17, 18])
    outs = [o.cpu().numpy() for o in p.run([torch.from_numpy(a).cuda() for a in (x, lab, w)])]
    xf = x[::-1]
    assert np.array_equal(outs[0], xf) and np.array_equal(outs[1], np.abs(xf))
    assert np.array_equal(outs[2], xf[:, ::-1])
    lf = lab.astype(np.float32)
    assert np.array_equal(outs[3], lf * lf)
    want = xf.astype(np.float64) @ w.astype(np.float64)
    assert np.linalg.norm(outs[4] - want) <= 1e-5 * np.linalg.norm(want)
    assert np.array_equal(outs[5], x) and outs[6].dtype == np.bool_ and np.array_equal(outs[6], x != 0)


def test_slice_views(zc):
    """slice from its recorded ranges (ops.zig:1587-1635): element j of axis
    i at starts[i] + j * steps[i]; positive and negative steps, feeding a
    region and copied out; payload ranges under vmap."""
    x = zo.uniform_range(61, 10 * 12, -2.0, 2.0).reshape(10, 12)
    F = zc.F32
    steps = [("slice", [1], 10, -2, 0, {"starts": [2, 1], "shape": [4, 5], "steps": [2, 2]}),
             ("slice", [1], 11, -2, 0, {"starts": [9, 11], "shape": [3, 4], "steps": [-3, -2]}),
             ("neg", [10], 12, -2, 0), ("abs", [11], 13, -2, 0)]
    p = zc.Plan([(1, F, (10, 12))], [], steps, [10, 11, 12, 13])
    a, b, c, d = [o.cpu().numpy() for o in p.run([torch.from_numpy(x).cuda()])]
    sa, sb = x[2:10:2, 1:11:2], x[9:0:-3, 11:3:-2]
    assert np.array_equal(a, sa) and np.array_equal(b, sb)
    assert np.array_equal(c, -sa) and np.array_equal(d, np.abs(sb))
    y = zo.uniform_range(62, 3 * 6 * 4, -1.0, 1.0).reshape(3, 6, 4)
    q = zc.Plan([(1, F, (3, 6, 4), 1)], [],
                [("slice", [1], 10, -2, 0, {"starts": [1, 3], "shape": [2, 1], "steps": [3, 1]})], [10])
    (r,) = q.run([torch.from_numpy(y).cuda()])
    assert np.array_equal(r.cpu().numpy(), y[:, 1:6:3, 3:4])
    with pytest.raises(zc.ZpuCudaError) as err:
        zc.Plan([(1, F, (10, 12))], [], [("slice", [1], 10, -2, 0, {"starts": [8, 0], "shape": [2, 1], "steps": [2, 1]})], [10])
    assert err.value.status == 8  # IndexOutOfRange: 8 + 2 is past the axis


def test_concat_stack_and_pad(zc):
    """ops.concat / stack / pad (ops.zig:1665-1695, 1995-2017): copies into
    parts of a new buffer, reading strided views as they are."""
    rng = np.random.default_rng(71)
    a = rng.standard_normal((4, 5)).astype(np.float32)
    b = rng.standard_normal((3, 5)).astype(np.float32)
    c = rng.standard_normal((5, 4)).astype(np.float32)
    F = zc.F32
    steps = [("concat_op", [1, 2], 10, 0, 0),
             ("transpose", [3], 11, -2, 0, {"perm": [1, 0]}),          # [4, 5], strided
             ("concat_op", [1, 11], 12, 1, 0),                           # [4, 10]
             ("stack_op", [1, 11], 13, 1, 0),                            # [4, 2, 5]
             ("stack_op", [1, 11], 14, -1, 0),                           # [4, 5, 2]
             ("pad", [1], 15, -2, 0, {"pads": [(1, 2), (0, 3)], "scalar": -7.0}),
             ("neg", [12], 16, -2, 0)]
    p = zc.Plan([(1, F, (4, 5)), (2, F, (3, 5)), (3, F, (5, 4))], [], steps, [10, 12, 13, 14, 15, 16])
    got = [o.cpu().numpy() for o in p.run([torch.from_numpy(v).cuda() for v in (a, b, c)])]
    ct = c.T
    want = [np.concatenate([a, b], 0), np.concatenate([a, ct], 1), np.stack([a, ct], 1), np.stack([a, ct], -1),
            np.pad(a, ((1, 2), (0, 3)), constant_values=-7.0), -np.concatenate([a, ct], 1)]
    for g, w in zip(got, want):
        assert g.shape == w.shape and np.array_equal(g, w)


def test_take_and_scatter_add(zc):
    """ops.take / scatterAdd (ops.zig:1697-1797): indices of any numeric type
    truncated toward zero, negatives counted from the end once; scatter_add
    starts from zeros and adds repeated indices in order, each sum in f64
    rounded to f32; a bad index is IndexOutOfRange through plan.check()."""
    rng = np.random.default_rng(72)
    x = rng.standard_normal((6, 8)).astype(np.float32)
    idx = np.array([[0, -1], [5, 2], [3, 3]], dtype=np.int64)
    fidx = np.array([2.7, -1.2], dtype=np.float32)
    sidx = np.array([0, 2, 0, 5, 2], dtype=np.int32)  # plan arg dtype 4 = DType.i32
    upd = rng.standard_normal((5, 8)).astype(np.float32)
    F = zc.F32
    p = zc.Plan([(1, F, (6, 8)), (2, zc.DT_I64, (3, 2)), (3, F, (2,)), (4, 4, (5,)), (5, F, (5, 8))], [],
                [("take", [1, 2], 10, 0, 0), ("take", [1, 3], 11, 1, 0), ("scatter_add", [1, 4, 5], 12, 0, 0)],
                [10, 11, 12])
    t0, t1, sc = [o.cpu().numpy() for o in p.run([torch.from_numpy(v).cuda() for v in (x, idx, fidx, sidx, upd)])]
    assert np.array_equal(t0, x[np.where(idx < 0, idx + 6, idx)])
    assert np.array_equal(t1, x[:, [2, 7]])
    want = np.zeros((6, 8), np.float32)
    for t, j in enumerate(sidx):
        want[j] = (want[j].astype(np.float64) + upd[t].astype(np.float64)).astype(np.float32)
    assert np.array_equal(sc, want)
    p.check()  # no bad index so far
    bad = zc.Plan([(1, F, (6, 8)), (2, zc.DT_I64, (2,))], [], [("take", [1, 2], 10, 0, 0)], [10])
    bad.run([torch.from_numpy(x).cuda(), torch.tensor([1, 6], device="cuda")])
    with pytest.raises(zc.ZpuCudaError) as err:
        bad.check()
    assert err.value.status == 8  # IndexOutOfRange
    bad.check()  # reported once


def test_value_and_grad_trace_of_an_mlp(zc):
    """A jit(valueAndGrad) trace of dense -> tanh -> dense -> meanAll(square)
    as zpu's autodiff records it (autodiff.zig: matmul VJP through
    swapLastTwo views, add's VJP as unbroadcast sums, tanh's VJP as
    g * (1 - a^2), meanAll's as a broadcast scalar): nine launches -- the
    transposes are views read by the GEMMs in place, the forward bias + tanh
    and bias run in the GEMM epilogues -- and the loss and all four gradients
    within 1e-4 of torch's f64 autograd."""
    B, I, H, O = 48, 20, 32, 6
    rng = np.random.default_rng(81)
    x, w1, b1 = (rng.standard_normal(s).astype(np.float32) for s in ((B, I), (I, H), (H,)))
    w2, b2 = (rng.standard_normal(s).astype(np.float32) * 0.3 for s in ((H, O), (O,)))
    F = zc.F32
    args = [(1, F, (B, I)), (2, F, (I, H)), (3, F, (H,)), (4, F, (H, O)), (5, F, (O,))]
    blobs = [(6, np.float32(1.0 / (B * O))), (7, np.float32(2.0)), (8, np.float32(1.0))]
    T = {"perm": [1, 0]}
    steps = [("matmul", [1, 2], 10, -2, 0), ("add", [10, 3], 11, -2, 0), ("tanh", [11], 12, -2, 0),
             ("matmul", [12, 4], 13, -2, 0), ("add", [13, 5], 14, -2, 0), ("square", [14], 15, -2, 0),
             ("sum", [15], 16, -2, 0), ("mul", [16, 6], 17, -2, 0),
             # backward
             ("broadcast", [6], 20, -2, 0, {"shape": [B, O]}), ("mul", [14, 7], 21, -2, 0),
             ("mul", [20, 21], 22, -2, 0), ("sum", [22], 23, 0, 0),
             ("transpose", [4], 24, -2, 0, T), ("matmul", [22, 24], 25, -2, 0),
             ("transpose", [12], 26, -2, 0, T), ("matmul", [26, 22], 27, -2, 0),
             ("square", [12], 28, -2, 0), ("sub", [8, 28], 29, -2, 0), ("mul", [25, 29], 30, -2, 0),
             ("sum", [30], 31, 0, 0), ("transpose", [1], 32, -2, 0, T), ("matmul", [32, 30], 33, -2, 0)]
    p = zc.Plan(args, blobs, steps, [17, 33, 31, 27, 23])
    assert p.num_kernels() == 9, p.describe()
    d = p.describe()
    assert "copy" not in d and "bias + tanh epilogue" in d and "+ bias epilogue" in d, d
    loss, gw1, gb1, gw2, gb2 = [o.cpu().numpy().astype(np.float64)
                                for o in p.run([torch.from_numpy(v).cuda() for v in (x, w1, b1, w2, b2)])]
    ts = [torch.tensor(v, dtype=torch.float64, requires_grad=True) for v in (x, w1, b1, w2, b2)]
    y = torch.tanh(ts[0] @ ts[1] + ts[2]) @ ts[3] + ts[4]
    ref = (y * y).mean()
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 1e-4 * abs(ref.item())
    for g, t in zip((gw1, gb1, gw2, gb2), ts[1:]):
        w = t.grad.numpy()
        assert np.linalg.norm(g - w) <= 1e-4 * np.linalg.norm(w)


def test_matmul_bias_tanh_fuse_into_the_gemm_epilogue(zc):
    """matmul -> add(row bias) -> tanh with each value used only by the next
    runs as one GEMM whose epilogue adds the bias and takes tanh; when the
    sum is needed elsewhere only the bias fuses, and a product used twice
    keeps its own region."""
    rng = np.random.default_rng(91)
    x = rng.standard_normal((40, 24)).astype(np.float32)
    w = rng.standard_normal((24, 36)).astype(np.float32) * 0.3
    b = rng.standard_normal(36).astype(np.float32)
    F = zc.F32
    args = [(1, F, (40, 24)), (2, F, (24, 36)), (3, F, (36,))]
    mm = [("matmul", [1, 2], 10, -2, 0), ("add", [10, 3], 11, -2, 0), ("tanh", [11], 12, -2, 0)]
    ref_h = x.astype(np.float64) @ w.astype(np.float64) + b
    cases = [([12], 1, "bias + tanh epilogue"), ([11, 12], 2, "+ bias epilogue"),
             ([12, 10], 2, None)]  # the product is an output: no fusion
    for outs, kernels, tag in cases:
        p = zc.Plan(args, [], mm, outs)
        d = p.describe()
        assert p.num_kernels() == kernels, d
        if tag:
            assert tag in d, d
        else:
            assert "epilogue" not in d, d
        got = dict(zip(outs, [o.cpu().numpy().astype(np.float64)
                              for o in p.run([torch.from_numpy(v).cuda() for v in (x, w, b)])]))
        assert np.max(np.abs(got[12] - np.tanh(ref_h))) <= 2e-5
        if 11 in got:
            assert np.linalg.norm(got[11] - ref_h) <= 1e-5 * np.linalg.norm(ref_h)


def test_split_k_gemm_epilogues(zc):
    """A product with one output tile and a long K runs split-K (the tile's
    CTAs add their partials in a cluster): the bias + tanh and the bias
    epilogues are applied after that sum."""
    rng = np.random.default_rng(93)
    x = rng.standard_normal((64, 4096)).astype(np.float32) * 0.05
    w = rng.standard_normal((4096, 36)).astype(np.float32) * 0.05
    b = rng.standard_normal(36).astype(np.float32)
    F = zc.F32
    args = [(1, F, (64, 4096)), (2, F, (4096, 36)), (3, F, (36,))]
    mm = [("matmul", [1, 2], 10, -2, 0), ("add", [10, 3], 11, -2, 0), ("tanh", [11], 12, -2, 0)]
    ref_h = x.astype(np.float64) @ w.astype(np.float64) + b
    for outs in ([12], [11, 12]):
        p = zc.Plan(args, [], mm, outs)
        got = dict(zip(outs, [o.cpu().numpy().astype(np.float64)
                              for o in p.run([torch.from_numpy(v).cuda() for v in (x, w, b)])]))
        torch.cuda.synchronize()
        zc.check(zc.lib().zpucuda_check_device())
        assert np.max(np.abs(got[12] - np.tanh(ref_h))) <= 2e-5
        if 11 in got:
            assert np.linalg.norm(got[11] - ref_h) <= 1e-5 * np.linalg.norm(ref_h)


def test_short_contraction_epilogues(zc):
    """matmul (k = 16) -> add(row bias) -> tanh as one short-contraction
    launch: zpu's chain for the product, then the bias and tanh epilogue."""
    rng = np.random.default_rng(97)
    x = rng.standard_normal((300, 16)).astype(np.float32)
    w = rng.standard_normal((16, 77)).astype(np.float32) * 0.3
    b = rng.standard_normal(77).astype(np.float32)
    F = zc.F32
    args = [(1, F, (300, 16)), (2, F, (16, 77)), (3, F, (77,))]
    mm = [("matmul", [1, 2], 10, -2, 0), ("add", [10, 3], 11, -2, 0), ("tanh", [11], 12, -2, 0)]
    ins = [torch.from_numpy(v).cuda() for v in (x, w, b)]
    want11 = (zo.gemm(x, w) + b).astype(np.float32)  # f32 add after zpu's chain
    p = zc.Plan(args, [], mm[:2], [11])  # bias epilogue
    assert p.num_kernels() == 1, p.describe()
    (got11,) = [o.cpu().numpy() for o in p.run(ins)]
    assert np.array_equal(got11, want11)
    p = zc.Plan(args, [], mm, [12])  # bias + tanh epilogue
    assert p.num_kernels() == 1, p.describe()
    (got12,) = [o.cpu().numpy() for o in p.run(ins)]
    assert np.max(np.abs(got12.astype(np.float64) - np.tanh(want11.astype(np.float64)))) <= 2e-7


def test_persistent_gemm_epilogues(zc, monkeypatch):
    """The bias + tanh and bias epilogues in the persistent GEMM form (one CTA
    per SM walking its tiles) give the one-tile-per-CTA kernel's bits."""
    monkeypatch.setenv("ZPUCUDA_GEMM_BN", "256")
    monkeypatch.setenv("ZPUCUDA_GEMM_PRESPLIT", "0")
    rng = np.random.default_rng(95)
    x = rng.standard_normal((700, 96)).astype(np.float32)
    w = rng.standard_normal((96, 600)).astype(np.float32) * 0.1
    b = rng.standard_normal(600).astype(np.float32)
    F = zc.F32
    args = [(1, F, (700, 96)), (2, F, (96, 600)), (3, F, (600,))]
    mm = [("matmul", [1, 2], 10, -2, 0), ("add", [10, 3], 11, -2, 0), ("tanh", [11], 12, -2, 0)]
    ins = [torch.from_numpy(v).cuda() for v in (x, w, b)]
    for outs in ([12], [11, 12]):
        res = []
        for mode in ("1", "0"):
            monkeypatch.setenv("ZPUCUDA_GEMM_PERSISTENT", mode)
            p = zc.Plan(args, [], mm, outs)
            res.append([o.cpu().numpy() for o in p.run(ins)])
            torch.cuda.synchronize()
            zc.check(zc.lib().zpucuda_check_device())
        for g, w_ in zip(*res):
            assert np.array_equal(g, w_)
    h = x.astype(np.float64) @ w.astype(np.float64) + b
    assert np.max(np.abs(res[0][-1] - np.tanh(h))) <= 2e-5
    assert np.linalg.norm(res[0][0] - h) <= 1e-5 * np.linalg.norm(h)


def test_data_movement_snapshots_on_device(zc, golden):
    """The reference's shape/{pad,take,concat,stack} snapshots as plan steps."""
    x = torch.tensor(golden["inputs"]["spread12"], dtype=torch.float64, device="cuda").reshape(3, 4)
    idx = torch.tensor([2, 0, 2], dtype=torch.int32, device="cuda")
    D = zc.F64
    p = zc.Plan([(1, D, (3, 4)), (2, 4, (3,))], [],
                [("pad", [1], 10, -2, 0, {"pads": [(1, 0), (0, 2)], "scalar": -1.0}), ("take", [1, 2], 11, 0, 0),
                 ("concat_op", [1, 1], 12, 1, 0), ("stack_op", [1, 1], 13, 0, 0)], [10, 11, 12, 13])
    for name, o in zip(("pad", "take", "concat", "stack"), p.run([x, idx])):
        s = golden["snapshots"]["zpu/shape/" + name]
        g = o.cpu().numpy()
        assert list(g.shape) == s["shape"], name
        assert np.all(np.abs(g.ravel() - s["values"]) <= s["tol"] * np.maximum(1, np.abs(g.ravel()))), name
