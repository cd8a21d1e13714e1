"""MLP train step on the B200 (zpucuda_mlp_*) against the oracle.

The oracle restates zpu's valueAndGrad of dense->tanh->dense->tanh->dense->
sparseCrossEntropy and Adam.step with f32 moments on the CPU.  Tolerance:
relative error <= 1e-4 for the loss, every gradient and the parameters after
Adam steps (the GEMMs are 3xTF32 and the sums re-associate); at the full
784->4096->4096->10, batch 8192 size the reference is PyTorch fp32 autograd
with TF32 off (the oracle needs hours there), at the same 1e-4.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import zpu_oracle as zo
from tests.helpers import rel_fro

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-4


@pytest.fixture(scope="module", params=[None, "1"], ids=["lo-by-rule", "lo-presplit"], autouse=True)
def lo_mode(request):
    """Each test runs with the library's own choice of where the GEMMs' TF32
    lo halves come from, and with every product forced onto lo halves made
    in HBM (split passes and the epilogues' lo outputs, handed on from the
    product that writes an operand to the ones that read it)."""
    import os
    old = os.environ.pop("ZPUCUDA_GEMM_PRESPLIT", None)
    if request.param is not None:
        os.environ["ZPUCUDA_GEMM_PRESPLIT"] = request.param
    yield request.param
    os.environ.pop("ZPUCUDA_GEMM_PRESPLIT", None)
    if old is not None:
        os.environ["ZPUCUDA_GEMM_PRESPLIT"] = old


@pytest.fixture(scope="module")
def zc():
    import zpu_b200
    zpu_b200.check(zpu_b200.lib().zpucuda_init(0))
    return zpu_b200


def problem(dims, B, seed):
    X = zo.uniform_range(seed, B * dims[0], 0.0, 1.0).reshape(B, dims[0])
    labels = zo.randint(seed + 1, B, 0, dims[3])
    return X, labels, zo.mlp_init(dims)


def make(zc, dims, max_batch, params):
    from zpu_b200.mlp import MLP
    m = MLP(*dims, max_batch=max_batch)
    m.set_params(params)
    return m


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check_grads(got, want, tol=TOL):
    for name, g, w in zip(("W1", "b1", "W2", "b2", "W3", "b3"), got, want):
        assert g.shape == w.shape
        e = rel_fro(g, w)
        assert e <= tol, (name, e)


@pytest.mark.parametrize("dims,B", [((64, 96, 80, 10), 300), ((128, 256, 128, 10), 1024),
                                    ((30, 50, 42, 10), 77), ((16, 32, 32, 3), 5), ((64, 64, 64, 33), 129)])
def test_value_and_grad_matches_oracle(zc, dims, B):
    """Loss and all six gradients; the odd sizes (row pitch not a multiple of
    4) run the FMA-chain GEMM with the same epilogues, 33 classes the wide
    loss kernel."""
    X, labels, params = problem(dims, B, 0x5EED0100 + B)
    loss_ref, grads_ref = zo.mlp_loss_grad(X, labels, params)
    m = make(zc, dims, max(B, 64), params)
    m.value_and_grad(dev(X), dev(labels))
    loss = m.loss()
    m.check()
    assert abs(loss - loss_ref) <= TOL * abs(loss_ref), (loss, loss_ref)
    check_grads(m.grads(), grads_ref)
    zc.check(zc.lib().zpucuda_check_device())


def test_adam_steps_match_oracle(zc):
    """Three train steps (valueAndGrad + Adam.step) against the oracle's loop;
    parameters, losses and both moments after every step."""
    dims, B = (64, 96, 80, 10), 256
    X, labels, params = problem(dims, B, 0x5EED0200)
    m = make(zc, dims, B, params)
    adam = zo.Adam(lr=1e-3)
    p_ref = [p.copy() for p in params]
    xd, ld = dev(X), dev(labels)
    for step in range(3):
        loss_ref, g_ref = zo.mlp_loss_grad(X, labels, p_ref)
        adam.step(p_ref, g_ref)
        m.train_step(xd, ld)
        loss = m.loss()
        assert abs(loss - loss_ref) <= TOL * abs(loss_ref), (step, loss, loss_ref)
        got = m.params()
        for i, (g, w) in enumerate(zip(got, p_ref)):
            assert rel_fro(g, w) <= TOL, (step, i, rel_fro(g, w))
    mm, vv = m.adam_state()
    for i in (0, 2, 4):
        assert rel_fro(mm[i], adam.m[i].reshape(mm[i].shape)) <= 1e-3
        assert rel_fro(vv[i], adam.v[i].reshape(vv[i].shape)) <= 1e-3
    assert m.steps() == 3


def test_train_step_is_value_and_grad_then_adam_and_deterministic(zc):
    dims, B = (64, 96, 80, 10), 200
    X, labels, params = problem(dims, B, 0x5EED0300)
    xd, ld = dev(X), dev(labels)
    a, b = make(zc, dims, B, params), make(zc, dims, B, params)
    for _ in range(2):
        a.train_step(xd, ld)
        b.value_and_grad(xd, ld)
        b.allreduce_grads()  # no communicator: nothing to do
        b.adam_step()
    for x, y in zip(a.params(), b.params()):
        assert np.array_equal(x, y)
    # the same input twice gives the same bits
    a.value_and_grad(xd, ld)
    g1 = a.grads()
    a.value_and_grad(xd, ld)
    for x, y in zip(g1, a.grads()):
        assert np.array_equal(x, y)


def test_global_batch_split_sums_to_full_batch(zc):
    """The data-parallel decomposition on one GPU: two halves, each scaled by
    1/global_batch, add up to the full-batch gradient."""
    dims, B = (64, 96, 80, 10), 512
    X, labels, params = problem(dims, B, 0x5EED0400)
    m = make(zc, dims, B, params)
    m.value_and_grad(dev(X), dev(labels))
    full, full_loss = m.grads(), m.loss()
    h = B // 2
    parts, loss = [], 0.0
    for s in (slice(0, h), slice(h, B)):
        m.value_and_grad(dev(X[s]), dev(labels[s]), global_batch=B)
        parts.append(m.grads())
        loss += m.loss()
    for i in range(6):
        assert rel_fro(parts[0][i] + parts[1][i], full[i]) <= 1e-5, i
    assert abs(loss - full_loss) <= 1e-5 * abs(full_loss)


def test_padding_stays_zero(zc):
    """W3 and b3 are stored 16 columns wide; the 6 pad columns stay 0."""
    dims, B = (64, 96, 80, 10), 128
    X, labels, params = problem(dims, B, 0x5EED0500)
    m = make(zc, dims, B, params)
    for _ in range(3):
        m.train_step(dev(X), dev(labels))
    torch.cuda.synchronize()
    L = zc.lib()
    for what in (0, 1, 2, 3):
        ptr, n = m.array(what)
        buf = C.c_void_p()
        zc.check(L.zpucuda_buf_wrap(ptr, n * 4, C.byref(buf)))
        host = np.empty(n, dtype=np.float32)
        zc.check(L.zpucuda_buf_download(buf, 0, host.ctypes.data, n * 4))
        L.zpucuda_buf_release(buf)
        off, ld = m.param_offset(4)
        boff, _ = m.param_offset(5)
        assert ld == 16 and boff >= off + 80 * 16
        w3 = host[off:off + 80 * 16].reshape(80, 16)
        b3 = host[boff:boff + 16]
        assert not w3[:, 10:].any() and not b3[10:].any(), what
        if what in (0, 1):
            assert w3[:, :10].any()


def test_bad_label_reports_index_out_of_range(zc):
    dims, B = (16, 32, 32, 3), 40
    X, labels, params = problem(dims, B, 0x5EED0600)
    labels[7] = 3
    m = make(zc, dims, B, params)
    m.value_and_grad(dev(X), dev(labels))
    with pytest.raises(zc.ZpuCudaError) as e:
        m.check()
    assert e.value.status == 8  # IndexOutOfRange, as nn.oneHot returns
    m.check()  # the flag is cleared


def test_argument_errors(zc):
    from zpu_b200.mlp import MLP
    m = MLP(16, 32, 32, 3, max_batch=8)
    x = torch.zeros(9, 16, device="cuda")
    y = torch.zeros(9, dtype=torch.int64, device="cuda")
    with pytest.raises(zc.ZpuCudaError) as e:
        m.value_and_grad(x, y)
    assert e.value.status == 5  # InvalidShape: batch > max_batch
    with pytest.raises(zc.ZpuCudaError):
        MLP(16, 32, 32, 65, max_batch=8)  # more than 64 classes: NotSupported
    with pytest.raises(zc.ZpuCudaError):
        m.set_params([np.zeros(3, np.float32)] * 6)


def torch_reference(X, labels, params):
    tp = [torch.from_numpy(p).cuda().requires_grad_(True) for p in params]
    W1, b1, W2, b2, W3, b3 = tp
    x = torch.from_numpy(X).cuda()
    a1 = torch.tanh(x @ W1 + b1)
    a2 = torch.tanh(a1 @ W2 + b2)
    logits = a2 @ W3 + b3
    loss = torch.nn.functional.cross_entropy(logits, torch.from_numpy(labels).cuda())
    loss.backward()
    return float(loss), [p.grad.cpu().numpy() for p in tp]


def test_full_size_step_against_torch_fp32(zc):
    """784->4096->4096->10, batch 8192, X ~ U[0,1] (seed 0x5EED0006), labels
    randint(0,10) (seed 0x5EED0007), Xavier-uniform init (seeds 0x5EED0010+l):
    one valueAndGrad against PyTorch fp32 autograd (TF32 off)."""
    from zpu_b200.mlp import MLP
    dims, B = (784, 4096, 4096, 10), 8192
    xd = zc.rng_uniform(0x5EED0006, B * 784, 0.0, 1.0).view(B, 784)
    ld = zc.rng_randint(0x5EED0007, B, 0, 10)
    m = MLP(*dims, max_batch=B)
    m.init_xavier()
    params = m.params()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        loss_ref, grads_ref = torch_reference(xd.cpu().numpy(), ld.cpu().numpy(), params)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    m.value_and_grad(xd, ld)
    loss = m.loss()
    m.check()
    assert abs(loss - loss_ref) <= TOL * abs(loss_ref), (loss, loss_ref)
    check_grads(m.grads(), grads_ref)
    # the inputs match the oracle's generators
    assert np.array_equal(xd[:2].cpu().numpy().ravel(), zo.uniform_range(0x5EED0006, 2 * 784, 0.0, 1.0))
    m.close()
    torch.cuda.empty_cache()


def test_phase_trace_orders_the_step(zc):
    """zpucuda_mlp_trace: one GPU, so no gradient exchange (point 8 is never
    reached); the main-stream points come in step order, the step's end waits
    for the side stream's Adam, and tracing leaves the results unchanged."""
    dims, B = (128, 256, 128, 10), 512
    X, labels, params = problem(dims, B, 0x5EED0900)
    xd, ld = dev(X), dev(labels)
    a, b = make(zc, dims, B, params), make(zc, dims, B, params)
    b.trace(True)
    for _ in range(2):
        a.train_step(xd, ld)
        b.train_step(xd, ld)
    t = b.trace_read()
    assert t[0] == 0.0
    assert all(t[i] > 0 for i in range(1, 8)) and all(t[i] <= t[i + 1] for i in range(0, 7)), t
    assert t[8] == -1.0 and t[12] == -1.0  # no exchange, no deferred all-gather
    assert 0 < t[9] <= t[11] <= t[7] and t[10] <= t[11], t
    for x, y in zip(a.params(), b.params()):
        assert np.array_equal(x, y)
    b.trace(False)
