"""f32 GEMM (tcgen05 3xTF32) and ops.matmul on the B200 against the oracle.

Tolerance: relative Frobenius error <= 1e-5 against zpu's f32 FMA-chain
gemm (the north star's bound for f32).

Every test runs twice: with the lo halves of the TF32 split made in shared
memory by the kernel's converter warps (ZPUCUDA_GEMM_PRESPLIT=0) and made
by a split pass in HBM and loaded beside the operands (=1); by default the
library picks per problem.
"""
import os

import numpy as np
import pytest

from oracle import zpu_oracle as zo
from tests.helpers import rel_fro

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-5


@pytest.fixture(scope="module", params=["0", "1"], ids=["lo-in-smem", "lo-presplit"], autouse=True)
def lo_mode(request):
    old = os.environ.get("ZPUCUDA_GEMM_PRESPLIT")
    os.environ["ZPUCUDA_GEMM_PRESPLIT"] = request.param
    yield request.param
    if old is None:
        del os.environ["ZPUCUDA_GEMM_PRESPLIT"]
    else:
        os.environ["ZPUCUDA_GEMM_PRESPLIT"] = old


@pytest.fixture(scope="module")
def zc():
    import zpu_b200
    zpu_b200.check(zpu_b200.lib().zpucuda_init(0))
    return zpu_b200


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check_no_device_error(zc):
    torch.cuda.synchronize()
    zc.check(zc.lib().zpucuda_check_device())


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("m,k,n", [(128, 32, 128), (256, 64, 256), (129, 100, 136), (300, 516, 260),
                                   (1, 8, 4), (513, 33, 1000)])
def test_layouts_and_edges(zc, monkeypatch, ta, tb, m, k, n):
    # the tensor-core path also for the short contractions (k <= 32), which
    # otherwise run zpu's chain on CUDA cores (test_short_contractions_exact)
    monkeypatch.setenv("ZPUCUDA_GEMM_SMALLK", "0")
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    want = zo.gemm(a, b)
    A = dev(a.T.copy()) if ta else dev(a)
    B = dev(b.T.copy()) if tb else dev(b)
    got = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
    check_no_device_error(zc)
    assert rel_fro(got, want) <= TOL, (m, k, n, ta, tb, rel_fro(got, want))


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_lo_in_hbm_and_in_shared_memory_give_the_same_bits(zc, ta, tb):
    """The two sources of the lo halves feed the tensor core identical
    operands in the same order, so the products agree bit for bit (split-K,
    a broadcast batch and the FMA-chain shapes included)."""
    keep = os.environ["ZPUCUDA_GEMM_PRESPLIT"]
    try:
        _same_bits_both_ways(zc, ta, tb)
    finally:
        os.environ["ZPUCUDA_GEMM_PRESPLIT"] = keep


def _same_bits_both_ways(zc, ta, tb):
    rng = np.random.default_rng(11)
    cases = [(512, 1024, 640), (256, 8192, 16), (129, 100, 136)]
    for m, k, n in cases:
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        A = dev(a.T.copy()) if ta else dev(a)
        B = dev(b.T.copy()) if tb else dev(b)
        outs = []
        for mode in ("0", "1"):
            os.environ["ZPUCUDA_GEMM_PRESPLIT"] = mode
            outs.append(zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy())
        check_no_device_error(zc)
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), (m, k, n, ta, tb)
    A3 = dev(rng.standard_normal((6, 96, 160)).astype(np.float32))
    B1 = dev(rng.standard_normal((160, 72)).astype(np.float32))
    outs = []
    for mode in ("0", "1"):
        os.environ["ZPUCUDA_GEMM_PRESPLIT"] = mode
        outs.append(zc.matmul(A3, B1, a_depth=1).cpu().numpy())
    assert np.array_equal(outs[0], outs[1])


def test_kernel_test_shapes_take_the_fma_path(zc, golden):
    """kernels.zig:512-543 shapes (odd pitches run the FMA-chain kernel)."""
    for m, k, n in golden["gemm_shapes"]:
        a = ((np.arange(m * k) % 7) * 0.5 - 1.0).astype(np.float32).reshape(m, k)
        b = ((np.arange(k * n) % 5) * 0.25 - 0.5).astype(np.float32).reshape(k, n)
        got = zc.gemm(dev(a), dev(b)).cpu().numpy()
        assert rel_fro(got, zo.gemm(a, b)) <= TOL


def test_config1_1024_cubed(zc):
    """zpu.matmul f32 1024^3, A, B ~ U[-1, 1] (seeds 0x5EED0001/2)."""
    n = 1024
    A = zc.rng_uniform(0x5EED0001, n * n, -1.0, 1.0).view(n, n)
    B = zc.rng_uniform(0x5EED0002, n * n, -1.0, 1.0).view(n, n)
    got = zc.matmul(A, B).cpu().numpy()
    check_no_device_error(zc)
    want = zo.gemm(A.cpu().numpy(), B.cpu().numpy())
    assert rel_fro(got, want) <= TOL


def test_config3_vmap_batched(zc):
    """The vmap-batched configuration at its full size: 256 products of
    512 x 512 matrices, N(0, 1/512) inputs (seeds 0x5EED0004/5), as bench
    times it; 8 matrices spread over the batch are checked against the
    oracle's FMA chain (on all host cores)."""
    import concurrent.futures as cf
    bsz, n = 256, 512
    s = 1.0 / np.sqrt(512.0)
    A = (zc.rng_normal(0x5EED0004, bsz * n * n) * s).view(bsz, n, n)
    B = (zc.rng_normal(0x5EED0005, bsz * n * n) * s).view(bsz, n, n)
    got = zc.matmul(A, B, a_depth=1, b_depth=1).cpu().numpy()
    check_no_device_error(zc)
    a, b = A.cpu().numpy(), B.cpu().numpy()
    picks = (0, 37, 73, 110, 146, 183, 219, 255)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        wants = list(ex.map(lambda i: zo.gemm(a[i], b[i]), picks))
    for i, want in zip(picks, wants):
        assert rel_fro(got[i], want) <= TOL, i


def test_batch_broadcast_and_transposed_views(zc):
    rng = np.random.default_rng(9)
    a = rng.standard_normal((6, 64, 96)).astype(np.float32)
    w = rng.standard_normal((96, 128)).astype(np.float32)
    got = zc.matmul(dev(a), dev(w)).cpu().numpy()
    assert rel_fro(got, zo.matmul(a, w)) <= TOL
    # the matmul VJP's a^T g and g w^T, read in place
    x = rng.standard_normal((256, 96)).astype(np.float32)
    g = rng.standard_normal((256, 128)).astype(np.float32)
    X, G, W = dev(x), dev(g), dev(w)
    got = zc.matmul(X.transpose(0, 1), G).cpu().numpy()
    assert rel_fro(got, zo.gemm(x.T.copy(), g)) <= TOL
    got = zc.matmul(G, W.transpose(0, 1)).cpu().numpy()
    assert rel_fro(got, zo.gemm(g, w.T.copy())) <= TOL
    check_no_device_error(zc)


def test_empty_contraction_writes_zeros(zc):
    a = torch.zeros((4, 0), dtype=torch.float32, device="cuda")
    b = torch.zeros((0, 3), dtype=torch.float32, device="cuda")
    c = torch.full((4, 3), 7.0, dtype=torch.float32, device="cuda")
    zc.gemm(a, b, out=c)
    assert float(c.abs().sum()) == 0.0


def test_nan_propagates_like_the_fma_chain(zc):
    """A NaN in row i of A makes row i of C NaN (zpu's FMA chain); every
    other element stays finite and within tolerance."""
    rng = np.random.default_rng(7)
    m, k, n = 256, 96, 200
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    a[5, 17] = np.nan
    a[130, 0] = np.nan
    want = zo.gemm(a, b)
    got = zc.gemm(dev(a), dev(b)).cpu().numpy()
    check_no_device_error(zc)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = ~np.isnan(want)
    assert rel_fro(got[fin], want[fin]) <= TOL


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("m,k,n", [(256, 8192, 16), (1024, 1024, 1024), (300, 3000, 40), (128, 100000 // 8, 8)])
def test_split_k_shapes(zc, ta, tb, m, k, n):
    """Few output tiles and a long K: the K range is split across CTAs and the
    partials added in split order."""
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    want = zo.gemm(a, b)
    A = dev(a.T.copy()) if ta else dev(a)
    B = dev(b.T.copy()) if tb else dev(b)
    got = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
    check_no_device_error(zc)
    assert rel_fro(got, want) <= TOL, (m, k, n, ta, tb, rel_fro(got, want))
    again = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
    assert np.array_equal(got, again)  # deterministic


@pytest.mark.parametrize("splits", ["2", "3", "4", "5", "8"])
@pytest.mark.parametrize("bn", ["128", "256"])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, True)])
def test_split_k_cluster_counts(zc, monkeypatch, splits, bn, ta, tb):
    """Split counts forced to 2..8 (the CTAs of a tile form one cluster and
    add their partials through distributed shared memory): ragged rows and
    columns, rows of a tile shared unevenly among the splits (128 / 3, / 5),
    both tile widths; deterministic from call to call."""
    monkeypatch.setenv("ZPUCUDA_GEMM_SPLITS", splits)
    monkeypatch.setenv("ZPUCUDA_GEMM_BN", bn)
    rng = np.random.default_rng(int(splits) * 10 + int(bn))
    for m, k, n in ((200, 2048, 10), (131, 1000, 300)):
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        want = zo.gemm(a, b)
        A = dev(a.T.copy()) if ta else dev(a)
        B = dev(b.T.copy()) if tb else dev(b)
        got = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
        check_no_device_error(zc)
        assert rel_fro(got, want) <= TOL, (m, k, n, rel_fro(got, want))
        again = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
        assert np.array_equal(got, again)


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
def test_persistent_form_matches(zc, monkeypatch, ta, tb):
    """The persistent form (one CTA per SM walking its tiles, the next tile's
    loads and MMAs overlapping this tile's last fold and its store) gives
    the bits of the one-tile-per-CTA kernel: ragged rows and columns, a
    batch, fewer tiles than SMs and many tiles per SM, K up to the form's 64
    slices; both agree with zpu's chain."""
    monkeypatch.setenv("ZPUCUDA_GEMM_BN", "256")
    monkeypatch.setenv("ZPUCUDA_GEMM_PRESPLIT", "0")
    rng = np.random.default_rng(7 + 2 * ta + tb)
    for bs, m, k, n in ((1, 200, 300, 520), (40, 130, 96, 300), (300, 128, 64, 256), (3, 256, 2048, 512)):
        a = rng.uniform(-1, 1, (bs, m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (bs, k, n)).astype(np.float32)
        A = dev(np.swapaxes(a, 1, 2).copy()) if ta else dev(a)
        B = dev(np.swapaxes(b, 1, 2).copy()) if tb else dev(b)
        if bs == 1:
            A, B = A[0], B[0]
        monkeypatch.setenv("ZPUCUDA_GEMM_PERSISTENT", "1")
        got = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
        check_no_device_error(zc)
        monkeypatch.setenv("ZPUCUDA_GEMM_PERSISTENT", "0")
        want = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
        assert np.array_equal(got, want), (bs, m, k, n)
        got = got.reshape(bs, m, n)
        for i in sorted({0, bs // 2, bs - 1}):
            assert rel_fro(got[i], zo.gemm(a[i], b[i])) <= TOL, (bs, m, k, n, i)


@pytest.mark.parametrize("group", ["1", "3", "16"])
def test_raster_groups_cover_every_tile(zc, monkeypatch, group):
    """Grouped tile order (CTAs sweep `group` row tiles column by column):
    every tile computed once, ragged last group, the same bits as blockIdx
    order."""
    rng = np.random.default_rng(int(group))
    a = rng.uniform(-1, 1, (1000, 96)).astype(np.float32)
    b = rng.uniform(-1, 1, (96, 1100)).astype(np.float32)
    A, B = dev(a), dev(b)
    monkeypatch.setenv("ZPUCUDA_GEMM_RASTER", "0")
    want = zc.gemm(A, B).cpu().numpy()
    monkeypatch.setenv("ZPUCUDA_GEMM_RASTER", group)
    got = zc.gemm(A, B).cpu().numpy()
    check_no_device_error(zc)
    assert np.array_equal(got, want)
    assert rel_fro(got, zo.gemm(a, b)) <= TOL


def test_persistent_form_infinities(zc, monkeypatch):
    """zpu's infinities and NaNs (the non-finite recompute) in the persistent form."""
    monkeypatch.setenv("ZPUCUDA_GEMM_BN", "256")
    monkeypatch.setenv("ZPUCUDA_GEMM_PRESPLIT", "0")
    monkeypatch.setenv("ZPUCUDA_GEMM_PERSISTENT", "1")
    rng = np.random.default_rng(17)
    a = (rng.integers(-8, 9, (300, 160)) / 8.0).astype(np.float32)
    b = (rng.integers(-8, 9, (160, 600)) / 8.0).astype(np.float32)
    a[3, 5] = np.inf
    a[250, 9] = -np.inf
    a[11, 2] = np.nan
    b[4, 517] = np.inf
    want = zo.gemm(a, b)
    got = zc.gemm(dev(a), dev(b)).cpu().numpy()
    check_no_device_error(zc)
    _exact_nonfinite(got, want)


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (300, 16, 4096), (77, 7, 133), (257, 32, 263), (64, 5, 8)])
def test_short_contractions_exact(zc, ta, tb, m, k, n):
    """k <= 32: zpu's own chain on CUDA cores, bit for bit the oracle's
    kernels.gemm (FMA order and the scalar tail of each 128-column panel:
    n = 133 and 263 leave 5 and 7 tail columns)."""
    rng = np.random.default_rng(m * 31 + k * 7 + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    A = dev(a.T.copy()) if ta else dev(a)
    B = dev(b.T.copy()) if tb else dev(b)
    got = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
    check_no_device_error(zc)
    assert np.array_equal(got, zo.gemm(a, b)), (m, k, n, ta, tb)


def test_short_contractions_batched_exact(zc):
    rng = np.random.default_rng(12)
    a = rng.standard_normal((5, 70, 12)).astype(np.float32)
    b = rng.standard_normal((5, 12, 300)).astype(np.float32)
    got = zc.gemm(dev(a), dev(b)).cpu().numpy()
    check_no_device_error(zc)
    for i in range(5):
        assert np.array_equal(got[i], zo.gemm(a[i], b[i])), i


def test_split_k_batched(zc):
    rng = np.random.default_rng(11)
    a = rng.uniform(-1, 1, (3, 128, 4096)).astype(np.float32)
    b = rng.uniform(-1, 1, (3, 4096, 64)).astype(np.float32)
    got = zc.gemm(dev(a), dev(b)).cpu().numpy()
    check_no_device_error(zc)
    for i in range(3):
        assert rel_fro(got[i], zo.gemm(a[i], b[i])) <= TOL


def _exact_nonfinite(got, want):
    """Non-finite elements equal bit for bit in kind (inf sign, NaN), the
    finite ones within the GEMM tolerance."""
    bad_w = ~np.isfinite(want)
    assert np.array_equal(~np.isfinite(got), bad_w)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[np.isinf(want)], want[np.isinf(want)])
    fin = ~bad_w
    assert rel_fro(got[fin], want[fin]) <= TOL


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("m,k,n", [(256, 128, 192), (128, 8192, 128)])
def test_infinities_give_zpus_infinities(zc, ta, tb, m, k, n):
    """An infinite operand against partners whose low TF32 halves are zero
    (values exact in TF32): the 3xTF32 hi x lo product is inf * 0 = NaN, but
    zpu's FMA chain gives +-inf.  Such elements are recomputed with zpu's
    chain (kernels.zig:388-398), so C matches the oracle's inf / NaN pattern
    exactly; the second shape runs split-K (the recompute is then in the
    reduction)."""
    rng = np.random.default_rng(5 + m)
    a = (rng.integers(-8, 9, (m, k)) / 8.0).astype(np.float32)  # exact in TF32: lo = 0
    b = (rng.integers(-8, 9, (k, n)) / 8.0).astype(np.float32)
    a[3, 5] = np.inf
    a[7, 9] = -np.inf
    a[11, 2] = np.nan
    b[4, 17] = np.inf
    b[min(k - 1, 5000), 40] = -np.inf
    want = zo.gemm(a, b)
    assert np.isinf(want).any() and np.isnan(want).any()
    A = dev(a.T.copy()) if ta else dev(a)
    B = dev(b.T.copy()) if tb else dev(b)
    got = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
    check_no_device_error(zc)
    _exact_nonfinite(got, want)


def test_infinities_batched_and_through_matmul(zc):
    rng = np.random.default_rng(21)
    a = (rng.integers(-4, 5, (4, 64, 96)) / 4.0).astype(np.float32)
    b = (rng.integers(-4, 5, (4, 96, 80)) / 4.0).astype(np.float32)
    a[2, 10, 3] = np.inf
    b[1, 7, 66] = -np.inf
    got = zc.matmul(dev(a), dev(b)).cpu().numpy()
    check_no_device_error(zc)
    for i in range(4):
        _exact_nonfinite(got[i], zo.gemm(a[i], b[i]))
