"""The MLP train step on the device (zpucuda_mlp_* and zpucuda_nccl_*).

Mirrors what the reference's MLP training loop does with
`zpu.valueAndGrad(alloc, loss, null, &args, &wrt)` followed by
`adam.step(&params, r.grads)` (examples/train_mlp.zig, src/zpu/optim.zig):
the model is dense -> tanh -> dense -> tanh -> dense, the loss
nn.sparseCrossEntropy of the logits against integer labels, the optimiser
Adam with f32 moments (AdamConfig defaults lr 1e-3, betas 0.9 / 0.999,
eps 1e-8).  Parameters, gradients and moments live in HBM inside the
library's handle; `params()` / `grads()` copy them out in the reference's
shapes.

Data parallelism: `init_process_group_nccl(rank, world)` joins this
process's GPU to an NCCL communicator (the 128-byte id travels through
torch.distributed's store); `train_step` then sums gradients across ranks.
"""
import ctypes as C

import numpy as np

from . import _capi
from ._capi import check, lib

PARAM, GRAD, ADAM_M, ADAM_V = 0, 1, 2, 3
NAMES = ("W1", "b1", "W2", "b2", "W3", "b3")
XAVIER_SEED0 = 0x5EED0010


class AdamConfig:
    """optim.AdamConfig (src/zpu/optim.zig:149-157) without weight decay."""

    def __init__(self, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8):
        self.lr, self.beta1, self.beta2, self.eps = lr, beta1, beta2, eps


def _stream(stream):
    from . import stream_of
    return stream_of(stream)


class MLP:
    """dense(d_in->d_h1) tanh dense(->d_h2) tanh dense(->d_out), with its
    gradients and Adam state on the current CUDA device."""

    def __init__(self, d_in, d_h1, d_h2, d_out, max_batch, adam=None):
        self.dims = (d_in, d_h1, d_h2, d_out)
        self.max_batch = max_batch
        h = C.c_void_p()
        check(lib().zpucuda_mlp_create(d_in, d_h1, d_h2, d_out, max_batch, C.byref(h)))
        self._h = h
        a = adam or AdamConfig()
        check(lib().zpucuda_mlp_adam_config(h, a.lr, a.beta1, a.beta2, a.eps))

    # ------------------------------------------------------------ parameters
    def shapes(self):
        d0, d1, d2, d3 = self.dims
        return [(d0, d1), (d1,), (d1, d2), (d2,), (d2, d3), (d3,)]

    def numel(self):
        n = C.c_int64()
        check(lib().zpucuda_mlp_param_count(self._h, C.byref(n)))
        return n.value

    def _write(self, what, arrays, stream=None):
        assert len(arrays) == 6
        for i, (a, shp) in enumerate(zip(arrays, self.shapes())):
            if hasattr(a, "data_ptr"):  # a torch tensor (host or device)
                if str(a.dtype) != "torch.float32":
                    raise _capi.ZpuCudaError(3, "%s must be float32" % NAMES[i])
                if not a.is_contiguous():
                    raise _capi.ZpuCudaError(7, "%s must be contiguous" % NAMES[i])
                got, ptr, n = tuple(a.shape), a.data_ptr(), a.numel()
            else:
                a = np.ascontiguousarray(a, dtype=np.float32)
                got, ptr, n = a.shape, a.ctypes.data, a.size
            if got != shp:
                raise _capi.ZpuCudaError(2, "%s has shape %s, the model wants %s" % (NAMES[i], got, shp))
            check(lib().zpucuda_mlp_write(self._h, what, i, ptr, n, _stream(stream)))
            if not hasattr(a, "data_ptr"):
                self.sync()  # the numpy buffer must outlive the copy

    def _read(self, what, stream=None):
        out = []
        for i, shp in enumerate(self.shapes()):
            a = np.empty(shp, dtype=np.float32)
            check(lib().zpucuda_mlp_read(self._h, what, i, a.ctypes.data, a.size, _stream(stream)))
            out.append(a)
        self.sync()
        return out

    def set_params(self, params, stream=None):
        self._write(PARAM, params, stream)

    def params(self):
        return self._read(PARAM)

    def grads(self):
        return self._read(GRAD)

    def adam_state(self):
        return self._read(ADAM_M), self._read(ADAM_V)

    def array(self, what):
        """(device address, floats) of a whole padded array."""
        p, n = C.c_void_p(), C.c_int64()
        check(lib().zpucuda_mlp_array(self._h, what, C.byref(p), C.byref(n)))
        return p.value, n.value

    def param_offset(self, i):
        """(offset, row pitch) of parameter i inside the arrays, in floats."""
        o, ld = C.c_int64(), C.c_int64()
        check(lib().zpucuda_mlp_param_offset(self._h, i, C.byref(o), C.byref(ld)))
        return o.value, ld.value

    def init_xavier(self, seed0=XAVIER_SEED0, stream=None):
        """Xavier-uniform weights W_l ~ U(-sqrt(6/(in+out)), +sqrt(6/(in+out)))
        from rng.Rng(seed0 + l).uniformRange on the device, zero biases."""
        import torch
        from . import rng_uniform
        d = self.dims
        arrays = []
        for l in range(3):
            lim = (6.0 / (d[l] + d[l + 1])) ** 0.5
            w = rng_uniform(seed0 + l, d[l] * d[l + 1], -lim, lim, stream=stream).view(d[l], d[l + 1])
            arrays += [w, torch.zeros(d[l + 1], dtype=torch.float32, device=w.device)]
        self._write(PARAM, arrays, stream)
        self.sync()

    # ------------------------------------------------------------------ step
    def _args(self, x, labels, global_batch):
        B = x.shape[0]
        if tuple(x.shape) != (B, self.dims[0]) or tuple(labels.shape) != (B,):
            raise _capi.ZpuCudaError(2, "x must be [batch, %d] and labels [batch]" % self.dims[0])
        if str(x.dtype) != "torch.float32" or str(labels.dtype) != "torch.int64":
            raise _capi.ZpuCudaError(3, "x must be float32 and labels int64")
        if not (x.is_contiguous() and labels.is_contiguous()):
            raise _capi.ZpuCudaError(7, "x and labels must be contiguous")
        if not (x.is_cuda and labels.is_cuda):
            raise _capi.ZpuCudaError(12, "x and labels must be device tensors")
        return x.data_ptr(), labels.data_ptr(), B, global_batch or B

    def value_and_grad(self, x, labels, global_batch=None, stream=None):
        xp, lp, B, G = self._args(x, labels, global_batch)
        check(lib().zpucuda_mlp_value_and_grad(self._h, xp, lp, B, G, _stream(stream)))

    def allreduce_grads(self, stream=None):
        check(lib().zpucuda_mlp_allreduce_grads(self._h, _stream(stream)))

    def adam_step(self, stream=None):
        check(lib().zpucuda_mlp_adam_step(self._h, _stream(stream)))

    def train_step(self, x, labels, global_batch=None, stream=None):
        xp, lp, B, G = self._args(x, labels, global_batch)
        check(lib().zpucuda_mlp_train_step(self._h, xp, lp, B, G, _stream(stream)))

    def join(self, stream=None):
        """Makes `stream` wait for the exchange a data-parallel step leaves
        running (the all-gather of W2 .. b3): call it before timing ends."""
        check(lib().zpucuda_mlp_join(self._h, _stream(stream)))

    def loss_to(self, dst_ptr, stream=None):
        check(lib().zpucuda_mlp_loss(self._h, dst_ptr, _stream(stream)))

    def loss(self):
        v = np.zeros(1, dtype=np.float32)
        self.loss_to(v.ctypes.data)
        self.sync()
        return float(v[0])

    def check(self):
        check(lib().zpucuda_mlp_check(self._h))

    def steps(self):
        return lib().zpucuda_mlp_steps(self._h)

    def trace(self, on=True):
        """Record the step's phase boundaries (zpucuda_mlp_trace)."""
        check(lib().zpucuda_mlp_trace(self._h, int(on)))

    def trace_read(self):
        """Times (ms from the step's start) of the last traced step's phase
        boundaries, in zpucuda_mlp_trace_read's order (-1: not reached)."""
        buf = (C.c_float * 13)()
        check(lib().zpucuda_mlp_trace_read(self._h, buf, 13))
        return [float(v) for v in buf]

    def exchange_mode(self):
        """1 when dW2 travels over peer memory from its GEMM, 0 when all
        gradients go through NCCL."""
        return lib().zpucuda_mlp_exchange_mode(self._h)

    def sync(self):
        import torch
        torch.cuda.synchronize()

    def close(self):
        if getattr(self, "_h", None):
            lib().zpucuda_mlp_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ NCCL
def nccl_unique_id():
    buf = (C.c_uint8 * 128)()
    check(lib().zpucuda_nccl_unique_id(buf))
    return bytes(buf)


def exchange_id(rank, make_id, broadcast):
    """Rank 0 makes the communicator id, every rank gets it.  `broadcast`
    takes a list [obj] and fills it from rank 0 (torch.distributed's
    broadcast_object_list over any backend)."""
    box = [make_id() if rank == 0 else None]
    broadcast(box)
    uid = box[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise _capi.ZpuCudaError(16, "NCCL id must be 128 bytes")
    return bytes(uid)


def nccl_init(rank, world, uid, timeout_ms=60000):
    buf = (C.c_uint8 * 128).from_buffer_copy(uid)
    check(lib().zpucuda_nccl_init(rank, world, buf, timeout_ms))


def init_process_group_nccl(rank, world, timeout_ms=60000):
    """Joins this process's GPU to a communicator of `world` ranks; the id
    travels through the already-initialised torch.distributed group."""
    import torch.distributed as dist
    uid = exchange_id(rank, nccl_unique_id, lambda box: dist.broadcast_object_list(box, src=0))
    nccl_init(rank, world, uid, timeout_ms)


def nccl_world():
    r, w = C.c_int(), C.c_int()
    check(lib().zpucuda_nccl_world(C.byref(r), C.byref(w)))
    return r.value, w.value


def nccl_destroy(timeout_ms=30000):
    check(lib().zpucuda_nccl_destroy(timeout_ms))
