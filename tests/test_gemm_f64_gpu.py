"""f64 GEMM (FP64 DMMA) and ops.matmul on the B200 against the oracle.

Tolerance: relative Frobenius error <= 1e-12 against zpu's f64 FMA-chain
gemm (the north star's bound); the reference's known answers at 1e-12.
"""
import os

import numpy as np
import pytest

from oracle import zpu_oracle as zo
from tests.helpers import rel_fro

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def zc():
    import zpu_b200
    zpu_b200.check(zpu_b200.lib().zpucuda_init(0))
    return zpu_b200


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_known_answers(zc, golden):
    """src/zpu/tests.zig:145-171 through the device ops.matmul."""
    for case in golden["known_answers"]:
        a = np.array(case["a"], dtype=np.float64).reshape(case["a_shape"])
        b = np.array(case["b"], dtype=np.float64).reshape(case["b_shape"])
        got = zc.matmul(dev(a), dev(b)).cpu().numpy()
        assert np.allclose(got.ravel(), case["want"], rtol=case["tol"], atol=0), case["name"]


def test_matmul_snapshots(zc, golden):
    a = np.array(golden["inputs"]["spd3"]).reshape(3, 3)
    s = golden["snapshots"]["zpu/linalg/matmul-3x3"]
    assert np.allclose(zc.matmul(dev(a), dev(a)).cpu().numpy().ravel(), s["values"], rtol=s["tol"])
    s = golden["snapshots"]["zpu/linalg/matvec"]
    got = zc.matmul(dev(a), dev(np.array(golden["inputs"]["rhs3"]))).cpu().numpy()
    assert got.shape == (3,)
    assert np.allclose(got, s["values"], rtol=s["tol"])


def test_jit_replay_and_vmap_snapshots(zc, golden):
    """tanh(matmul(a, b)) on [3,2,2] f64, as a lowered jit plan (2 steps ->
    a GEMM + a region) and as a vmapped matmul (depth 1)."""
    a = np.array(golden["inputs"]["vmap_a"], dtype=np.float64).reshape(3, 2, 2)
    b = np.array(golden["inputs"]["vmap_b"], dtype=np.float64).reshape(3, 2, 2)
    p = zc.Plan([(1, zc.F64, (3, 2, 2)), (2, zc.F64, (3, 2, 2))], [],
                [("matmul", [1, 2], 10, -2, 0), ("tanh", [10], 11, -2, 0)], [11])
    assert p.num_steps() == golden["jit_steps"]
    (got,) = p.run([dev(a), dev(b)])
    for name in ("zpu/transforms/jit-replay", "zpu/transforms/vmap"):
        s = golden["snapshots"][name]
        w = np.array(s["values"])
        g = got.cpu().numpy().ravel()
        assert np.all(np.abs(w - g) <= s["tol"] * np.maximum(1, np.maximum(np.abs(w), np.abs(g))))
    m = zc.matmul(dev(a), dev(b), a_depth=1, b_depth=1)
    assert np.allclose(np.tanh(m.cpu().numpy()).ravel(), golden["snapshots"]["zpu/transforms/vmap"]["values"],
                       rtol=1e-9)


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
def test_kernel_shapes_all_layouts(zc, golden, ta, tb):
    """kernels.zig:512-543 shapes plus tile-straddling ones, every layout."""
    shapes = golden["gemm_shapes"] + [[129, 17, 131], [256, 64, 128], [1, 300, 7], [200, 1, 3]]
    rng = np.random.default_rng(1)
    for m, k, n in shapes:
        a = rng.standard_normal((m, k))
        b = rng.standard_normal((k, n))
        want = zo.gemm(a, b)
        A = dev(a.T.copy()) if ta else dev(a)
        B = dev(b.T.copy()) if tb else dev(b)
        got = zc.gemm(A, B, trans_a=ta, trans_b=tb).cpu().numpy()
        assert rel_fro(got, want) <= 1e-12, (m, k, n, ta, tb)


def test_odd_leading_dimensions_take_8_byte_copies(zc):
    m, k, n = 67, 44, 33
    rng = np.random.default_rng(2)
    a = rng.standard_normal((m, k + 1))[:, :k]  # lda = k + 1 (odd pitch)
    b = rng.standard_normal((k, n))
    want = zo.gemm(np.ascontiguousarray(a), b)
    A = dev(rng.standard_normal((m, k + 1)))
    A[:, :k] = dev(a)
    got = zc.gemm(A[:, :k], dev(b)).cpu().numpy()
    assert rel_fro(got, want) <= 1e-12


def test_batched_and_broadcast(zc):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((5, 40, 24))
    b = rng.standard_normal((24, 56))
    got = zc.matmul(dev(a), dev(b)).cpu().numpy()
    want = zo.matmul(a, b)
    assert rel_fro(got, want) <= 1e-12
    b3 = rng.standard_normal((5, 24, 56))
    got = zc.matmul(dev(a), dev(b3)).cpu().numpy()
    assert rel_fro(got, zo.matmul(a, b3)) <= 1e-12
    # broadcast over a leading axis of size 1 on a, 4-D
    a4 = rng.standard_normal((1, 3, 8, 16))
    b4 = rng.standard_normal((2, 1, 16, 8))
    got = zc.matmul(dev(a4), dev(b4)).cpu().numpy()
    assert got.shape == (2, 3, 8, 8)
    assert rel_fro(got, zo.matmul(a4, b4)) <= 1e-12


def test_transposed_views_are_read_in_place(zc):
    """The matmul VJP's swapLastTwo views (autodiff.zig:480-487)."""
    rng = np.random.default_rng(4)
    a = rng.standard_normal((96, 64))
    g = rng.standard_normal((96, 80))
    A, G = dev(a), dev(g)
    got = zc.matmul(A.transpose(0, 1), G).cpu().numpy()  # a^T g
    assert rel_fro(got, zo.gemm(a.T.copy(), g)) <= 1e-12
    w = rng.standard_normal((64, 80))
    got = zc.matmul(G, dev(w).transpose(0, 1)).cpu().numpy()  # g w^T
    assert rel_fro(got, zo.gemm(g, w.T.copy())) <= 1e-12


def test_config5_slice_8192(zc):
    """8192^3 f64 with A, B ~ N(0,1) (seeds 0x5EED0008/9), checked on the
    1024-row slice against the oracle's FMA chain (rows are independent, so
    the oracle runs 64-row pieces on all host cores)."""
    import concurrent.futures as cf
    n = 8192
    A = zc.rng_normal(0x5EED0008, n * n, dtype=torch.float64).view(n, n)
    B = zc.rng_normal(0x5EED0009, n * n, dtype=torch.float64).view(n, n)
    C = zc.gemm(A, B)
    rows = 1024
    a, b = A[:rows].cpu().numpy(), B.cpu().numpy()
    got = C[:rows].cpu().numpy()
    del A, C
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as ex:
        parts = list(ex.map(lambda r: zo.gemm(np.ascontiguousarray(a[r:r + 64]), b), range(0, rows, 64)))
    assert rel_fro(got, np.concatenate(parts)) <= 1e-12


def test_empty_and_degenerate(zc):
    a = torch.zeros((4, 0), dtype=torch.float64, device="cuda")
    b = torch.zeros((0, 3), dtype=torch.float64, device="cuda")
    c = torch.full((4, 3), 7.0, dtype=torch.float64, device="cuda")
    zc.gemm(a, b, out=c)
    assert float(c.abs().sum()) == 0.0  # k == 0 writes zeros (kernels.zig:346-349)
    with pytest.raises(zc.ZpuCudaError) as e:
        zc.matmul(dev(np.ones((2, 3))), dev(np.ones((4, 5))))
    assert e.value.name == "ShapeMismatch"
