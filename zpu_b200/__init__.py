"""zpu_b200: the B200 (sm_100a) execution layer for zpu's data-parallel hot path.

The product is libzpucuda.so (C ABI in include/zpucuda.h).  This package is
its Python front end: torch tensors provide device memory and streams, every
computation runs in the library's own CUDA kernels, and nothing falls back to
a CPU path when the library is missing -- importing the operations raises.
"""
import ctypes as C

from ._capi import (AXIS_NONE, DT_BOOL, DT_I64, F32, F64, PRIM, Blob, Step, Tensor, Value, ZpuCudaError, check,
                    exported_names, lib)

__all__ = ["lib", "check", "ZpuCudaError", "Plan", "gemm", "matmul", "matmul_shape", "stream_of",
           "launch_count", "AXIS_NONE", "F32", "F64", "PRIM"]


CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy


def _torch():
    import torch
    return torch


def stream_of(stream=None):
    """cudaStream_t (as int) of a torch stream, default the current one."""
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    h = s.cuda_stream
    # torch's default stream is the legacy NULL stream; NULL means "the
    # thread's own stream" to the C ABI, so name it as cudaStreamLegacy.
    return h if h else CUDA_STREAM_LEGACY


def dtype_code(t):
    torch = _torch()
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.float64:
        return F64
    raise ZpuCudaError(9, "dtype %s" % t.dtype)


def torch_dtype(code):
    """torch dtype of a zpu DType code (src/zpu/dtype.zig:4-13)."""
    torch = _torch()
    return [torch.float64, torch.float32, torch.float16, torch.int64, torch.int32, torch.int16, torch.int8,
            torch.uint8, torch.bool][code]


def rng_normal(seed, n, dtype=None, device="cuda", out=None, stream=None):
    """rng.Rng(seed).normal on the device (the same stream as zpu's)."""
    torch = _torch()
    out = out if out is not None else torch.empty(n, dtype=dtype or torch.float32, device=device)
    check(lib().zpucuda_rng_normal(seed, dtype_code(out), out.data_ptr(), out.numel(), stream_of(stream)))
    return out


def rng_uniform(seed, n, lo=0.0, hi=1.0, dtype=None, device="cuda", out=None, stream=None):
    """rng.Rng(seed).uniformRange(lo, hi) on the device."""
    torch = _torch()
    out = out if out is not None else torch.empty(n, dtype=dtype or torch.float32, device=device)
    check(lib().zpucuda_rng_uniform(seed, dtype_code(out), out.data_ptr(), out.numel(), lo, hi,
                                    stream_of(stream)))
    return out


def rng_randint(seed, n, lo, hi, device="cuda", out=None, stream=None):
    """rng.Rng(seed).randint(lo, hi) on the device (int64)."""
    torch = _torch()
    out = out if out is not None else torch.empty(n, dtype=torch.int64, device=device)
    check(lib().zpucuda_rng_randint(seed, out.data_ptr(), out.numel(), lo, hi, stream_of(stream)))
    return out


def launch_count():
    return int(lib().zpucuda_launch_count())


def tensor_desc(t, batch_depth=0):
    """zpucuda_tensor for a torch tensor view (strides in elements)."""
    d = Tensor()
    d.data = t.data_ptr()
    d.dtype = storage_code(t)
    d.rank = t.dim()
    for i in range(t.dim()):
        d.dims[i] = t.shape[i]
        d.strides[i] = t.stride(i)
    d.batch_depth = batch_depth
    return d


def storage_code(t):
    """zpu DType code (src/zpu/dtype.zig:4-13) of a torch tensor's element type."""
    torch = _torch()
    codes = {torch.float64: 0, torch.float32: 1, torch.float16: 2, torch.int64: 3, torch.int32: 4,
             torch.int16: 5, torch.int8: 6, torch.uint8: 7, torch.bool: 8}
    if t.dtype not in codes:
        raise ZpuCudaError(9, "dtype %s" % t.dtype)
    return codes[t.dtype]


def tensor_copy(src, out, stream=None):
    """Tensor.clone / toContiguous / ops.cast on device: the elements of the
    view `src` (a torch tensor, or a zpucuda_tensor descriptor for views torch
    cannot express, e.g. negative strides) in logical order into the
    contiguous torch tensor `out`, converted to out's type as zpu converts."""
    if isinstance(src, Tensor):
        d = src
    else:
        d = tensor_desc(src)
        d.dtype = storage_code(src)
    o = tensor_desc(out)
    o.dtype = storage_code(out)
    check(lib().zpucuda_tensor_copy(C.byref(d), C.byref(o), stream_of(stream)))
    return out


def matmul_shape(a, b, a_depth=0, b_depth=0, with_dtype=False):
    """Output shape and vmap depth of ops.matmul (and its zpu DType code,
    DType.promote of the operands, when with_dtype)."""
    out = Tensor()
    check(lib().zpucuda_matmul_shape(C.byref(tensor_desc(a, a_depth)), C.byref(tensor_desc(b, b_depth)),
                                     C.byref(out)))
    shape = tuple(out.dims[i] for i in range(out.rank))
    return (shape, out.batch_depth, out.dtype) if with_dtype else (shape, out.batch_depth)


def matmul(a, b, a_depth=0, b_depth=0, out=None, stream=None):
    """ops.matmul on device tensors (NumPy semantics, vmap depth); any of
    zpu's element types, the result of type DType.promote(a, b)."""
    torch = _torch()
    shape, depth, code = matmul_shape(a, b, a_depth, b_depth, with_dtype=True)
    if out is None:
        out = torch.empty(shape, dtype=torch_dtype(code), device=a.device)
    da, db, dc = tensor_desc(a, a_depth), tensor_desc(b, b_depth), tensor_desc(out, depth)
    check(lib().zpucuda_matmul(C.byref(da), C.byref(db), C.byref(dc), stream_of(stream)))
    return out


def gemm(a, b, out=None, trans_a=False, trans_b=False, stream=None):
    """C = op(A) @ op(B) for 2-D or batched 3-D device tensors (row-major,
    contiguous innermost axis).  op(A) = A^T when trans_a (A stored [k, m])."""
    torch = _torch()
    batched = a.dim() == 3 or b.dim() == 3
    A = a if a.dim() == 3 else a.unsqueeze(0)
    B = b if b.dim() == 3 else b.unsqueeze(0)
    m = A.shape[2] if trans_a else A.shape[1]
    k = A.shape[1] if trans_a else A.shape[2]
    n = B.shape[1] if trans_b else B.shape[2]
    batch = max(A.shape[0], B.shape[0])
    if out is None:
        out = torch.empty((batch, m, n) if batched else (m, n), dtype=a.dtype, device=a.device)
    O = out if out.dim() == 3 else out.unsqueeze(0)
    sa = A.stride(0) if A.shape[0] > 1 else 0
    sb = B.stride(0) if B.shape[0] > 1 else 0
    f = lib().zpucuda_gemm_f32 if a.dtype == torch.float32 else lib().zpucuda_gemm_f64
    check(f(A.data_ptr(), B.data_ptr(), O.data_ptr(), m, n, k, A.stride(1), B.stride(1), O.stride(1),
            int(trans_a), int(trans_b), batch, sa, sb, O.stride(0) if O.shape[0] > 1 else m * n,
            stream_of(stream)))
    return out


class Plan:
    """A lowered jit plan (zpucuda_plan_*)."""

    def __init__(self, args, blobs, steps, out_ids):
        """args: [(id, dtype_code, shape[, batch_depth])], blobs: [(id, numpy
        array)], steps: [(prim, [input ids], out id, axis, flags[, {"shape":
        dims, "perm": axes}])] (flags: Attrs.flags, 1 = KEEP_DIMS, 32 =
        REVERSE; shape / perm: reshape, broadcast, transpose), out_ids: [id].
        batch_depth is Tensor.batch_depth (vmap's leading axes,
        src/zpu/tensor.zig:79-89): reductions fold payload axes only."""
        import numpy as np
        L = lib()
        self._keep = []
        va = (Value * max(1, len(args)))()
        for i, a in enumerate(args):
            _fill_value(va[i], a[0], a[1], a[2], a[3] if len(a) > 3 else 0)
        bl = (Blob * max(1, len(blobs)))()
        for i, (vid, arr) in enumerate(blobs):
            arr = np.ascontiguousarray(arr)
            self._keep.append(arr)
            code = F64 if arr.dtype == np.float64 else DT_BOOL if arr.dtype == np.bool_ else F32
            _fill_value(bl[i].value, vid, code, arr.shape)
            bl[i].host_data = arr.ctypes.data
        st = (Step * max(1, len(steps)))()
        for i, step in enumerate(steps):
            prim, ins, out, axis, keepdims = step[:5]
            extra = step[5] if len(step) > 5 else {}
            st[i].prim = PRIM[prim] if isinstance(prim, str) else prim
            st[i].n_inputs = len(ins)
            for k, x in enumerate(ins):
                st[i].ins[k] = x
            st[i].out = out
            st[i].axis = axis
            st[i].flags = int(keepdims)  # Attrs.flags: 1 = KEEP_DIMS, 32 = REVERSE
            shape = extra.get("shape", ())
            st[i].shape_len = len(shape)
            for k, d in enumerate(shape):
                st[i].shape[k] = d
            perm = extra.get("perm", ())
            st[i].nsl = len(perm)
            for k, d in enumerate(perm):
                st[i].perm[k] = d
            if "starts" in extra:  # slice: starts, lens (as "shape"), steps
                st[i].nsl = len(extra["starts"])
                for k in range(len(extra["starts"])):
                    st[i].starts[k] = extra["starts"][k]
                    st[i].steps[k] = extra["steps"][k]
            if "pads" in extra:  # pad: [(lo, hi)] per axis and the fill value
                st[i].nsl = len(extra["pads"])
                for k, (lo, hi) in enumerate(extra["pads"]):
                    st[i].starts[k] = lo
                    st[i].pads_hi[k] = hi
                st[i].scalar = float(extra.get("scalar", 0.0))
        oi = (C.c_uint64 * len(out_ids))(*out_ids)
        h = C.c_void_p()
        check(L.zpucuda_plan_create(va, len(args), bl, len(blobs), st, len(steps), oi, len(out_ids),
                                    C.byref(h)))
        self.handle = h
        self.n_args = len(args)
        self.outputs = []
        for i in range(len(out_ids)):
            v = Value()
            check(L.zpucuda_plan_output(h, i, C.byref(v)))
            self.outputs.append((v.dtype, tuple(v.dims[d] for d in range(v.rank))))

    def num_steps(self):
        return lib().zpucuda_plan_num_steps(self.handle)

    def check(self, stream=None):
        """zpucuda_plan_check: raises IndexOutOfRange for a bad take /
        scatter_add index since the last check."""
        check(lib().zpucuda_plan_check(self.handle, stream_of(stream)))

    def num_kernels(self):
        return lib().zpucuda_plan_num_kernels(self.handle)

    def describe(self):
        buf = C.create_string_buffer(8192)
        check(lib().zpucuda_plan_describe(self.handle, buf, len(buf)))
        return buf.value.decode()

    def run(self, args, outs=None, stream=None):
        torch = _torch()
        if outs is None:
            dev = args[0].device if args else torch.device("cuda")
            outs = [torch.empty(shape, dtype=torch_dtype(dt), device=dev) for dt, shape in self.outputs]
        pa = (C.c_void_p * max(1, len(args)))(*[a.data_ptr() for a in args])
        po = (C.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
        check(lib().zpucuda_plan_run(self.handle, pa, po, stream_of(stream)))
        return outs

    def run_host(self, args, outs=None, stream=None):
        """zpucuda_plan_run_host on host (CPU, ideally pinned) torch tensors."""
        torch = _torch()
        if outs is None:
            outs = [torch.empty(shape, dtype=torch_dtype(dt)) for dt, shape in self.outputs]
        pa = (C.c_void_p * max(1, len(args)))(*[a.data_ptr() for a in args])
        po = (C.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
        check(lib().zpucuda_plan_run_host(self.handle, pa, po, stream_of(stream)))
        return outs

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                lib().zpucuda_plan_destroy(h)
            except Exception:
                pass
            self.handle = None


def _fill_value(v, vid, dt, shape, depth=0):
    v.id = vid
    v.dtype = dt
    v.rank = len(shape)
    for i, s in enumerate(shape):
        v.dims[i] = s
    v.batch_depth = depth
