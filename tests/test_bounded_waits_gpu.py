"""Bounded device waits that run out, on one GPU, without a fault.

The data-parallel MLP step's dW2 exchange ends in a kernel that waits for
every rank's flag before it adds the ranks' slots of its inbox.  Here the
same kernel runs through zpucuda_debug_peer_reduce on buffers of the test's
own: flags that nothing ever sets make its wait run out after a short spin
limit, and the kernel must return, set the error word and leave the output
untouched; flags that are set give the in-order sum.  Nothing waits on
another process or GPU.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def zc():
    import zpu_b200
    zpu_b200.check(zpu_b200.lib().zpucuda_init(0))
    return zpu_b200


def _run(zc, inbox, world, n, out, flags, epoch, spin, err):
    L = zc.lib()
    zc.check(L.zpucuda_debug_peer_reduce(inbox.data_ptr(), world, n, out.data_ptr(), flags.data_ptr(), epoch,
                                         spin, err.data_ptr(), zc.stream_of()))
    torch.cuda.synchronize()


def test_peer_reduce_wait_runs_out_and_reports(zc):
    world, n = 4, 4096
    inbox = torch.randn(world * n, device="cuda")
    flags = torch.zeros(world, dtype=torch.int64, device="cuda")  # no rank ever publishes
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((n,), 7.0, device="cuda")
    _run(zc, inbox, world, n, out, flags, 1, 2000, err)
    assert int(err.item()) == 1
    assert torch.all(out == 7.0)


def test_peer_reduce_sums_in_rank_order_when_flags_are_up(zc):
    world, n = 3, 1 << 16
    inbox = torch.randn(world * n, device="cuda")
    flags = torch.tensor([5, 6, 5], dtype=torch.int64, device="cuda")  # every rank at epoch >= 5
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros(n, device="cuda")
    _run(zc, inbox, world, n, out, flags, 5, 2000, err)
    assert int(err.item()) == 0
    s = inbox.view(world, n).cpu().numpy()
    want = (s[0] + s[1]).astype(np.float32) + s[2]  # rank order, each add rounded to f32
    assert np.array_equal(out.cpu().numpy(), want.astype(np.float32))


def test_peer_reduce_one_missing_rank_still_times_out(zc):
    world, n = 2, 1024
    inbox = torch.ones(world * n, device="cuda")
    flags = torch.tensor([3, 2], dtype=torch.int64, device="cuda")  # rank 1 is an epoch behind
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((n,), -1.0, device="cuda")
    _run(zc, inbox, world, n, out, flags, 3, 1000, err)
    assert int(err.item()) == 1
    assert torch.all(out == -1.0)


def test_peer_reduce_rejects_bad_arguments(zc):
    L = zc.lib()
    x = torch.zeros(16, device="cuda")
    f = torch.zeros(2, dtype=torch.int64, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    for args in [(x.data_ptr(), 2, 6, x.data_ptr(), f.data_ptr(), 1, 100, e.data_ptr()),     # n % 4
                 (x.data_ptr(), 9, 4, x.data_ptr(), f.data_ptr(), 1, 100, e.data_ptr()),     # world > 8
                 (x.data_ptr() + 4, 2, 4, x.data_ptr(), f.data_ptr(), 1, 100, e.data_ptr()),  # unaligned
                 (x.data_ptr(), 2, 4, x.data_ptr(), f.data_ptr(), 1, 0, e.data_ptr())]:      # no spin limit
        st = L.zpucuda_debug_peer_reduce(*args, zc.stream_of())
        assert zc._capi.STATUS[st] == "InvalidArgument"
