"""The allocation-free variant of the fused jit-chain reduction.

Some callers cannot allocate device memory: an application that embeds the
library inside a framework whose caching allocator owns the device, or a
latency-critical loop where cudaMalloc's implicit synchronisation is not
allowed.  zpucuda_chain_tanh_sq_affine_sum_noalloc serves them with a static
scratch array inside the library.  This file checks, through the C ABI, that
two calls in a row give the existing entry point's result (the lowered jit
plan of the same chain) within the suite's sum tolerance.  It is named to run
last, and passes both alone in a fresh process and after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import zpu_oracle as zo

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SEED_X = 0x5EED0003


def test_no_alloc_matches_plan_twice_in_a_row():
    import zpu_b200 as zc
    zc.check(zc.lib().zpucuda_init(0))
    L = zc.lib()
    n = (1 << 22) + 3
    x = zc.rng_normal(SEED_X, n)
    a = torch.tensor(0.5, dtype=torch.float32, device="cuda")
    b = torch.tensor(-0.25, dtype=torch.float32, device="cuda")
    # the existing entry point: the jit plan of sumAll(tanh(x*x)*a + b)
    steps = [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0), ("mul", [11, 2], 12, -2, 0),
             ("add", [12, 3], 13, -2, 0), ("sum", [13], 14, -2, 0)]
    plan = zc.Plan([(1, zc.F32, (n,)), (2, zc.F32, ()), (3, zc.F32, ())], [], steps, [14])
    (want,) = plan.run([x, a, b])
    want = float(want.cpu())
    # the suite's sum tolerance: 1e-6 * sum|t_i| (t from the oracle)
    _, s64, t = zo.jit_chain_tanh_sq_affine_sum(x.cpu().numpy(), 0.5, -0.25, want_vector=True)
    tol = 1e-6 * zo.abssum_f64(t)
    assert abs(want - s64) <= tol
    stream = zc.stream_of()
    for call in range(2):
        out = torch.full((), float("nan"), dtype=torch.float32, device="cuda")
        zc.check(L.zpucuda_chain_tanh_sq_affine_sum_noalloc(x.data_ptr(), n, a.data_ptr(), b.data_ptr(),
                                                            out.data_ptr(), stream))
        got = float(out.cpu())
        assert abs(got - want) <= tol, (call, got, want)


def test_no_alloc_rejects_bad_arguments():
    import zpu_b200 as zc
    zc.check(zc.lib().zpucuda_init(0))
    L = zc.lib()
    x = torch.zeros(9, dtype=torch.float32, device="cuda")
    s = torch.zeros((), dtype=torch.float32, device="cuda")
    # a 4-byte offset breaks the 16-byte alignment the 128-bit loads need
    st = L.zpucuda_chain_tanh_sq_affine_sum_noalloc(x.data_ptr() + 4, 8, s.data_ptr(), s.data_ptr(),
                                                    s.data_ptr(), zc.stream_of())
    assert zc._capi.STATUS[st] == "InvalidArgument"
    assert b"16-byte" in L.zpucuda_last_error()
    st = L.zpucuda_chain_tanh_sq_affine_sum_noalloc(x.data_ptr(), -1, s.data_ptr(), s.data_ptr(),
                                                    s.data_ptr(), zc.stream_of())
    assert zc._capi.STATUS[st] == "InvalidArgument"
