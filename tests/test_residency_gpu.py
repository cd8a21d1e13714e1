"""A chain of device ops on device-resident buffers, on the B200.

zpu's ops read and write Buffer.mem on the host (src/zpu/tensor.zig:263-302).
With the residency protocol a zpu op that runs on the device makes its
operands' HBM copies current (zpucuda_buf_device_sync: a copy only when the
host copy is newer), writes its result on the device and marks it
(zpucuda_buf_mark_device_dirty); a host read makes the host copy current
first (zpucuda_buf_host_sync).  Here matmul -> jit plan (tanh(.) * 0.5) ->
matmul runs under a scope: only the three inputs cross PCIe before the chain,
nothing inside it, one result after it, and the scope releases every buffer
it adopted except the one kept.
"""
import ctypes as C

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


def stats(L):
    h, d = C.c_uint64(), C.c_uint64()
    assert L.zpucuda_buf_transfer_stats(C.byref(h), C.byref(d)) == 0
    return h.value, d.value


def alloc(zc, nbytes):
    b = C.c_void_p()
    zc.check(zc.lib().zpucuda_buf_alloc(nbytes, C.byref(b)))
    return b


def desc(zc, ptr, shape):
    from zpu_b200._capi import Tensor
    d = Tensor()
    d.data = ptr
    d.dtype = zc.F32
    d.rank = len(shape)
    q = 1
    for i in range(len(shape) - 1, -1, -1):
        d.dims[i] = shape[i]
        d.strides[i] = q
        q *= shape[i]
    return d


def test_matmul_plan_matmul_chain_stays_on_the_device(zc):
    L = zc.lib()
    stream = zc.stream_of()
    A = zo.normal(0x5EED0A01, 64 * 48).reshape(64, 48)
    B = zo.normal(0x5EED0A02, 48 * 32).reshape(48, 32)
    W = zo.normal(0x5EED0A03, 32 * 16).reshape(32, 16)
    plan = zc.Plan([(1, zc.F32, (64, 32))], [(2, np.float32(0.5))],
                   [("tanh", [1], 10, -2, 0), ("mul", [10, 2], 11, -2, 0)], [11])
    sc = C.c_void_p()
    zc.check(L.zpucuda_scope_begin(C.byref(sc)))
    bufs = {}
    for name, arr in (("A", A), ("B", B), ("W", W)):
        bufs[name] = alloc(zc, arr.nbytes)
        zc.check(L.zpucuda_buf_attach_host(bufs[name], arr.ctypes.data, zc._capi.RES_HOST))
    for name in ("C", "D"):
        bufs[name] = alloc(zc, 64 * 32 * 4)
    bufs["E"] = alloc(zc, 64 * 16 * 4)
    assert L.zpucuda_scope_count(sc) == 6
    h0, d0 = stats(L)
    # the operands' HBM copies are made current once
    for name in ("A", "B", "W"):
        zc.check(L.zpucuda_buf_device_sync(bufs[name], stream))
    h1, d1 = stats(L)
    assert (h1 - h0, d1 - d0) == (A.nbytes + B.nbytes + W.nbytes, 0)
    dev = {k: L.zpucuda_buf_devptr(v) for k, v in bufs.items()}
    # matmul -> plan -> matmul, each result marked as written on the device
    dc = desc(zc, dev["C"], (64, 32))
    zc.check(L.zpucuda_matmul(C.byref(desc(zc, dev["A"], (64, 48))), C.byref(desc(zc, dev["B"], (48, 32))),
                              C.byref(dc), stream))
    zc.check(L.zpucuda_buf_mark_device_dirty(bufs["C"]))
    zc.check(L.zpucuda_plan_run(plan.handle, (C.c_void_p * 1)(dev["C"]), (C.c_void_p * 1)(dev["D"]), stream))
    zc.check(L.zpucuda_buf_mark_device_dirty(bufs["D"]))
    de = desc(zc, dev["E"], (64, 16))
    zc.check(L.zpucuda_matmul(C.byref(desc(zc, dev["D"], (64, 32))), C.byref(desc(zc, dev["W"], (32, 16))),
                              C.byref(de), stream))
    zc.check(L.zpucuda_buf_mark_device_dirty(bufs["E"]))
    # a device sync of an operand that is already current copies nothing
    zc.check(L.zpucuda_buf_device_sync(bufs["A"], stream))
    assert stats(L) == (h1, d1)
    # the host reads the result: one copy back, then none
    E = np.full((64, 16), np.nan, dtype=np.float32)
    zc.check(L.zpucuda_buf_attach_host(bufs["E"], E.ctypes.data, zc._capi.RES_DEVICE))
    zc.check(L.zpucuda_buf_host_sync(bufs["E"], stream))
    zc.check(L.zpucuda_buf_host_sync(bufs["E"], stream))
    h2, d2 = stats(L)
    assert (h2 - h1, d2 - d1) == (0, E.nbytes)
    st = C.c_int()
    zc.check(L.zpucuda_buf_residency(bufs["E"], C.byref(st)))
    assert st.value == zc._capi.RES_BOTH
    # the oracle: zpu's FMA-chain matmuls and f64-then-round tanh
    Cw = zo.matmul(A, B)
    Dw = (zo.unary("tanh", Cw) * np.float32(0.5)).astype(np.float32)
    Ew = zo.matmul(Dw, W)
    assert rel_fro(E, Ew) <= 1e-5
    # the scope: E survives with the reference keep added, the rest go
    kept = L.zpucuda_scope_keep(sc, bufs["E"])
    assert kept == bufs["E"].value
    L.zpucuda_buf_retain(bufs["A"])  # an outside owner of A
    zc.check(L.zpucuda_scope_end(sc))
    assert L.zpucuda_buf_refcount(bufs["E"]) == 1
    assert L.zpucuda_buf_refcount(bufs["A"]) == 1
    E2 = np.zeros_like(E)
    zc.check(L.zpucuda_buf_download(bufs["E"], 0, E2.ctypes.data, E2.nbytes))
    assert np.array_equal(E, E2)
    L.zpucuda_buf_release(bufs["E"])
    L.zpucuda_buf_release(bufs["A"])


def test_host_write_then_device_read_copies_once(zc):
    L = zc.lib()
    stream = zc.stream_of()
    x = np.arange(256, dtype=np.float32)
    b = alloc(zc, x.nbytes)
    zc.check(L.zpucuda_buf_attach_host(b, x.ctypes.data, zc._capi.RES_HOST))
    h0, d0 = stats(L)
    zc.check(L.zpucuda_buf_device_sync(b, stream))
    zc.check(L.zpucuda_buf_device_sync(b, stream))
    torch.cuda.synchronize()
    assert stats(L) == (h0 + x.nbytes, d0)
    # host code writes the host copy (writeF64): the next device read copies again
    x[:] = -x
    zc.check(L.zpucuda_buf_mark_host_dirty(b))
    zc.check(L.zpucuda_buf_device_sync(b, stream))
    y = np.zeros_like(x)
    zc.check(L.zpucuda_buf_download(b, 0, y.ctypes.data, y.nbytes))
    assert np.array_equal(y, x)
    L.zpucuda_buf_release(b)
