"""Residency state and scopes of device buffers, on the CPU.

A zpu Buffer that also lives in HBM has a host copy (what zpu's accessors
read, src/zpu/tensor.zig:263-302) and a device copy; the state says which is
current.  Scopes mirror zpu's Tracker / Scope (src/zpu/tensor.zig:537-664):
buffers created while a scope is installed are adopted and released when it
ends; keep adds a reference, forget hands the creation reference back.
Wrapped buffers (zpucuda_buf_wrap) make no CUDA call, so all of this runs
here; the copies themselves are covered by tests/test_residency_gpu.py.
"""
import ctypes as C

import pytest


@pytest.fixture(scope="module")
def capi():
    from zpu_b200 import build
    build.build()
    from zpu_b200 import _capi
    return _capi


def wrap(L, nbytes=64):
    mem = (C.c_char * nbytes)()
    b = C.c_void_p()
    assert L.zpucuda_buf_wrap(C.cast(mem, C.c_void_p), nbytes, C.byref(b)) == 0
    return b, mem


def state(L, b):
    s = C.c_int(0)
    assert L.zpucuda_buf_residency(b, C.byref(s)) == 0
    return s.value


def test_residency_transitions_without_copies(capi):
    L = capi.lib()
    b, _ = wrap(L)
    host = (C.c_char * 64)()
    assert state(L, b) == capi.RES_DEVICE
    # no host copy attached: host-side marks and syncs are refused
    assert capi.STATUS[L.zpucuda_buf_mark_host_dirty(b)] == "InvalidArgument"
    assert capi.STATUS[L.zpucuda_buf_host_sync(b, None)] == "InvalidArgument"
    assert L.zpucuda_buf_attach_host(b, C.cast(host, C.c_void_p), capi.RES_BOTH) == 0
    assert capi.STATUS[L.zpucuda_buf_attach_host(b, C.cast(host, C.c_void_p), 7)] == "InvalidArgument"
    h0, d0 = C.c_uint64(), C.c_uint64()
    assert L.zpucuda_buf_transfer_stats(C.byref(h0), C.byref(d0)) == 0
    # both copies current: neither sync copies anything
    assert L.zpucuda_buf_host_sync(b, None) == 0 and L.zpucuda_buf_device_sync(b, None) == 0
    assert state(L, b) == capi.RES_BOTH
    assert L.zpucuda_buf_mark_device_dirty(b) == 0 and state(L, b) == capi.RES_DEVICE
    assert L.zpucuda_buf_mark_host_dirty(b) == 0 and state(L, b) == capi.RES_HOST
    # a device sync of a HOST buffer must copy: that needs the GPU, so only
    # the already-current cases are exercised here
    assert L.zpucuda_buf_mark_device_dirty(b) == 0
    assert L.zpucuda_buf_device_sync(b, None) == 0 and state(L, b) == capi.RES_DEVICE
    h1, d1 = C.c_uint64(), C.c_uint64()
    assert L.zpucuda_buf_transfer_stats(C.byref(h1), C.byref(d1)) == 0
    assert (h1.value, d1.value) == (h0.value, d0.value)
    L.zpucuda_buf_release(b)


def test_scope_adopts_and_releases(capi):
    L = capi.lib()
    sc = C.c_void_p()
    assert L.zpucuda_scope_begin(C.byref(sc)) == 0
    assert L.zpucuda_scope_installed(sc) == 1
    a, ma = wrap(L)
    b, mb = wrap(L)
    c, mc = wrap(L)
    assert L.zpucuda_scope_count(sc) == 3
    # keep: b survives the scope with a reference of its own
    assert L.zpucuda_scope_keep(sc, b) == b.value
    assert L.zpucuda_buf_refcount(b) == 2
    # forget: c's creation reference goes back to the caller
    assert L.zpucuda_scope_forget(sc, c) == 0
    assert L.zpucuda_scope_count(sc) == 2
    L.zpucuda_buf_retain(a)  # a second owner of a, outside the scope
    assert L.zpucuda_scope_end(sc) == 0
    assert L.zpucuda_buf_refcount(a) == 1  # the scope dropped its reference
    assert L.zpucuda_buf_refcount(b) == 1
    assert L.zpucuda_buf_refcount(c) == 1
    for x in (a, b, c):
        L.zpucuda_buf_release(x)


def test_nested_scope_is_inert_like_trackers(capi):
    """Tracker.begin installs only when no other tracker is active: buffers
    made under an inner scope go to the outer one."""
    L = capi.lib()
    outer, inner = C.c_void_p(), C.c_void_p()
    assert L.zpucuda_scope_begin(C.byref(outer)) == 0
    assert L.zpucuda_scope_begin(C.byref(inner)) == 0
    assert L.zpucuda_scope_installed(outer) == 1 and L.zpucuda_scope_installed(inner) == 0
    b, _ = wrap(L)
    assert L.zpucuda_scope_count(outer) == 1 and L.zpucuda_scope_count(inner) == 0
    L.zpucuda_buf_retain(b)
    assert L.zpucuda_scope_end(inner) == 0
    assert L.zpucuda_buf_refcount(b) == 2  # the inert scope released nothing
    assert L.zpucuda_scope_end(outer) == 0
    assert L.zpucuda_buf_refcount(b) == 1
    L.zpucuda_buf_release(b)
    # with no scope installed, new buffers are owned by their creator alone
    b2, _ = wrap(L)
    assert L.zpucuda_buf_refcount(b2) == 1
    L.zpucuda_buf_release(b2)
