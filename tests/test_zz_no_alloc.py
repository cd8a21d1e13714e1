"""The allocation-free variant of the fused jit-chain reduction.

Some callers cannot allocate device memory: an application that embeds the
library inside a framework whose caching allocator owns the device, or a
latency-critical loop where cudaMalloc's implicit synchronisation is not
allowed.  zpucuda_chain_tanh_sq_affine_sum_noalloc serves them with a static
scratch array inside the library.  This file checks, through the C ABI, that
two calls in a row give the existing entry point's result (the lowered jit
plan of the same chain): the same kernel on the same grid, so the two agree
bit for bit, and both lie within the suite's sum tolerance of the f64 sum.
It is named to run last, and passes both alone in a fresh process and after
the other tests.
"""
import os
import struct
import subprocess
import sys

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
    bits = lambda v: struct.pack("<f", v)
    for call in range(2):
        out = torch.full((), float("nan"), dtype=torch.float32, device="cuda")
        zc.check(L.zpucuda_chain_tanh_sq_affine_sum_noalloc(x.data_ptr(), n, a.data_ptr(), b.data_ptr(),
                                                            out.data_ptr(), stream))
        got = float(out.cpu())
        assert bits(got) == bits(want), (call, got, want)
        assert abs(got - s64) <= tol


_OVERSIZE = r"""
import torch, zpu_b200 as zc
zc.check(zc.lib().zpucuda_init(0))
L = zc.lib()
x = torch.zeros(1 << 20, dtype=torch.float32, device="cuda")
s = torch.zeros((), dtype=torch.float32, device="cuda")
st = L.zpucuda_chain_tanh_sq_affine_sum_noalloc(x.data_ptr(), x.numel(), s.data_ptr(), s.data_ptr(),
                                                s.data_ptr(), zc.stream_of())
print(zc._capi.STATUS[st])
print(L.zpucuda_last_error().decode())
"""


def test_no_alloc_rejects_a_grid_beyond_its_scratch():
    # 16 blocks per SM on 148 SMs needs 2368 block partials; the static
    # scratch holds 2048, so the call must refuse instead of overrunning it
    env = dict(os.environ, ZPUCUDA_REGION_BPS="16")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _OVERSIZE], env=env, cwd=root, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.strip().splitlines()
    assert lines[-2] == "NotSupported", r.stdout
    assert "block partials" in lines[-1] and "2048" in lines[-1], r.stdout


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
