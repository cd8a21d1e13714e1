"""The C ABI library on the CPU: it loads, exports every function the header
declares, reports no device here, and lowers jit plans (lowering is host
code; running them needs the GPU)."""
import ctypes as C
import os
import subprocess
import sys

import pytest

from tests.helpers import ROOT, header_functions


@pytest.fixture(scope="module")
def capi():
    from zpu_b200 import build
    build.build()
    from zpu_b200 import _capi
    return _capi


def test_every_header_function_is_exported(capi):
    lib = C.CDLL(capi.LIB_PATH)
    names = header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes binding covers the whole header as well
    assert set(names) <= set(capi.exported_names()), set(names) - set(capi.exported_names())


def test_status_strings_follow_zpu_error_set(capi):
    L = capi.lib()
    assert L.zpucuda_status_string(0) == b"ok"
    # src/zpu/tensor.zig:58-71 in declaration order
    order = [b"OutOfMemory", b"ShapeMismatch", b"DTypeMismatch", b"RankTooLarge", b"InvalidShape",
             b"InvalidAxis", b"NonContiguous", b"IndexOutOfRange", b"NotSupported",
             b"NotDifferentiable", b"NotPositiveDefinite", b"DeviceMismatch"]
    for i, name in enumerate(order, start=1):
        assert L.zpucuda_status_string(i) == name
    assert L.zpucuda_version() >= 100


def test_no_device_here_is_reported_not_crashed(capi):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = capi.lib()
    n = C.c_int(-1)
    assert L.zpucuda_device_count(C.byref(n)) == 0
    assert n.value == 0
    assert L.zpucuda_init(0) == 15  # NoDevice


def test_allocation_fault_injection_is_host_side(capi):
    """ZPUCUDA_FAULT_ALLOC_AFTER makes allocations fail with OutOfMemory
    before any CUDA call (no GPU is touched)."""
    code = ("import ctypes as C; from zpu_b200 import _capi; L=_capi.lib(); p=C.c_void_p(); "
            "print(L.zpucuda_buf_alloc(1024, C.byref(p)))")
    env = dict(os.environ, ZPUCUDA_FAULT_ALLOC_AFTER="0", PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, cwd=ROOT)
    assert out.stdout.strip() == "1", out.stderr


def test_buffer_refcount_with_wrapped_memory(capi):
    """Buffer.retain/release semantics on a non-owning wrapper (no CUDA call)."""
    L = capi.lib()
    mem = (C.c_char * 64)()
    b = C.c_void_p()
    assert L.zpucuda_buf_wrap(C.cast(mem, C.c_void_p), 64, C.byref(b)) == 0
    assert L.zpucuda_buf_refcount(b) == 1
    L.zpucuda_buf_retain(b)
    assert L.zpucuda_buf_refcount(b) == 2
    L.zpucuda_buf_release(b)
    assert L.zpucuda_buf_refcount(b) == 1
    assert L.zpucuda_buf_bytes(b) == 64
    L.zpucuda_buf_release(b)


def _chain_steps(reduce):
    # jit trace of sumAll(tanh(x*x)*a + b): ids as zpu would hand them out
    steps = [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0), ("mul", [11, 2], 12, -2, 0),
             ("add", [12, 3], 13, -2, 0)]
    if reduce:
        steps.append(("sum", [13], 14, -2, 0))
    return steps


def test_lowering_fuses_the_chain_into_one_catalogued_kernel(capi):
    import zpu_b200 as zc
    args = [(1, zc.F32, (1024,)), (2, zc.F32, ()), (3, zc.F32, ())]
    p = zc.Plan(args, [], _chain_steps(False), [13])
    assert p.num_steps() == 4
    assert p.num_kernels() == 1
    d = p.describe()
    assert "catalogue tanh_sq_affine" in d, d
    assert p.outputs == [(zc.F32, (1024,))]


def test_lowering_keeps_needed_intermediates_and_splits_on_shape(capi):
    import zpu_b200 as zc
    # y = exp(x) ; z = y + row ; both outputs; then a [4,8] -> [8] broadcast row
    args = [(1, zc.F32, (4, 8)), (2, zc.F32, (8,))]
    steps = [("exp", [1], 10, -2, 0), ("add", [10, 2], 11, -2, 0), ("neg", [11], 12, -2, 0)]
    p = zc.Plan(args, [], steps, [10, 12])
    assert p.num_kernels() == 1
    d = p.describe()
    assert "bytecode" in d and ";FR;" in d, d


def test_lowering_rejects_unsupported_prims(capi):
    """solve / inv / det / cholesky / triangular_solve / conv: zpu's own jit
    replay refuses them (ops.zig:2197-2199), and so does the lowering."""
    import zpu_b200 as zc
    args = [(1, zc.F32, (4, 4)), (2, zc.F32, (4,))]
    for prim in (81, 82, 83, 84, 86):
        with pytest.raises(zc.ZpuCudaError) as e:
            zc.Plan(args, [], [(prim, [1, 2], 10, -2, 0)], [10])
        assert e.value.name == "NotSupported"


def test_lowering_types_i64_operands_as_zpu_promotes(capi):
    """argmax / argmin give i64 (ops.zig:931-934); an i64 operand against a
    float gives the float type; i64 operands alone give i64, f32 for the
    float-only prims and div, bool for predicates (DType.promote,
    dtype.zig:89-104; unaryOutDType / binaryOutDType, ops.zig:268-285); sum /
    prod / max / min of i64 give i64 (reduceOutDType, ops.zig:813-818).  The
    region holding them runs on 64-bit words: + - * max min mod abs sign relu
    of two i64 values on the integers, the rest through f64 (i2f / f2i), f32
    results of an i64 operand rounded once (r32)."""
    import zpu_b200 as zc
    F, I, B = zc.F32, zc.DT_I64, zc.DT_BOOL
    args = [(1, F, (8, 10)), (2, I, (8,)), (3, F, (8,))]
    p = zc.Plan(args, [], [("argmax", [1], 10, 1, 0), ("eq", [10, 2], 11, -2, 0), ("mul", [10, 3], 12, -2, 0),
                           ("gt", [12, 3], 13, -2, 0), ("add", [10, 2], 14, -2, 0), ("neg", [14], 15, -2, 0),
                           ("exp", [10], 16, -2, 0), ("div", [10, 2], 17, -2, 0), ("sign", [2], 18, -2, 0)],
                [10, 11, 12, 13, 14, 15, 16, 17, 18])
    shp = (8,)
    assert p.outputs == [(I, shp), (B, shp), (F, shp), (B, shp), (I, shp), (I, shp), (F, shp), (F, shp), (I, shp)]
    d = p.describe()
    assert "bytecode" in d and "catalogue" not in d, d
    for word in ("w64", "iadd(", "isign(", "f2i(", "i2f(", "r32("):
        assert word in d, (word, d)
    w = zc.Plan(args + [(4, B, (8,))], [], [("argmax", [1], 10, 1, 0), ("where", [4, 2, 10], 11, -2, 0),
                                            ("where", [4, 2, 3], 12, -2, 0)], [10, 11, 12])
    assert w.outputs == [(I, shp), (I, shp), (F, shp)]
    # (a reduction's plan needs a device workspace: its typing is checked in
    # the GPU tests)
    for step, want in [(("pow", [10, 2], 11, -2, 0), (I, shp)), (("where", [2, 10, 10], 11, -2, 0), (I, shp)),
                       (("where", [3, 10, 2], 11, -2, 0), (I, shp)), (("cumsum", [2], 11, 0, 0), (I, shp))]:
        # the argmax result is an output too: a plan made without a GPU
        # cannot allocate an intermediate
        q = zc.Plan(args, [], [("argmax", [1], 10, 1, 0), step], [10, 11])
        assert q.outputs[1] == want, step
    assert "zpow(" in zc.Plan(args, [], [("argmax", [1], 10, 1, 0), ("pow", [10, 2], 11, -2, 0)], [10, 11]).describe()
    for bad in [("add", [10, 4], 11, -2, 0), ("sum", [4], 11, -2, 0)]:  # i64 + bool; a sum of bools
        with pytest.raises(zc.ZpuCudaError) as e:
            zc.Plan(args + [(4, B, (8,))], [], [("argmax", [1], 10, 1, 0), bad], [10, 11])
        assert e.value.name == "NotSupported", bad


def test_abi_struct_layouts_match_the_header(capi, tmp_path):
    """Every struct the ctypes binding mirrors has the header's size and
    field offsets (a C probe compiled here with gcc)."""
    from zpu_b200 import _capi
    structs = {"zpucuda_step": _capi.Step, "zpucuda_value": _capi.Value, "zpucuda_tensor": _capi.Tensor,
               "zpucuda_blob": _capi.Blob}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "zpucuda.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append('printf("%s %%zu\\n", sizeof(%s));' % (cname, cname))
        for fname, _ in cls._fields_:
            lines.append('printf("%s.%s %%zu\\n", offsetof(%s, %s));' % (cname, fname, cname, fname))
    lines.append("return 0; }")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines())
    for cname, cls in structs.items():
        assert int(got[cname]) == C.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert int(got["%s.%s" % (cname, fname)]) == getattr(cls, fname).offset, (cname, fname)


def test_lowering_of_views_is_host_logic(capi):
    """A transposed GEMM operand is read in place (one launch, no copy), and
    a transpose under vmap permutes the payload axes only."""
    import zpu_b200 as zc
    T = {"perm": [1, 0]}
    p = zc.Plan([(1, zc.F32, (16, 8)), (2, zc.F32, (16, 4))], [],
                [("transpose", [1], 10, -2, 0, T), ("matmul", [10, 2], 11, -2, 0)], [11])
    assert p.num_kernels() == 1 and "copy" not in p.describe()
    assert p.outputs == [(zc.F32, (8, 4))]
    q = zc.Plan([(1, zc.F32, (3, 4, 5), 1)], [],
                [("transpose", [1], 10, -2, 0, T), ("neg", [10], 11, -2, 0)], [11])
    assert q.outputs == [(zc.F32, (3, 5, 4))]


def test_matmul_shape_logic_matches_ops_matmul(capi):
    """ops.matmul shapes (src/zpu/ops.zig:1062-1205) through the C ABI."""
    import numpy as np
    from oracle import zpu_oracle as zo
    L = capi.lib()

    def desc(shape, depth=0):
        d = capi.Tensor()
        d.dtype = capi.F32
        d.rank = len(shape)
        st = 1
        for i in reversed(range(len(shape))):
            d.dims[i] = shape[i]
            d.strides[i] = st
            st *= shape[i]
        d.batch_depth = depth
        return d

    cases = [((2, 3), (3, 4), 0, 0), ((3,), (3, 4), 0, 0), ((2, 3), (3,), 0, 0), ((3,), (3,), 0, 0),
             ((5, 2, 3), (3, 4), 0, 0), ((5, 2, 3), (5, 3, 4), 0, 0), ((1, 2, 3), (6, 3, 4), 0, 0),
             ((7, 2, 3), (7, 3, 4), 1, 1), ((7, 2, 3), (3, 4), 1, 0), ((7, 4, 2, 3), (4, 3, 5), 1, 0)]
    for sa, sb, da, db in cases:
        out = capi.Tensor()
        st = L.zpucuda_matmul_shape(C.byref(desc(sa, da)), C.byref(desc(sb, db)), C.byref(out))
        assert st == 0, (sa, sb)
        got = tuple(out.dims[i] for i in range(out.rank))
        want = zo.matmul(np.ones(sa, np.float32), np.ones(sb, np.float32), da, db).shape
        assert got == want, (sa, sb, got, want)
    out = capi.Tensor()
    assert L.zpucuda_matmul_shape(C.byref(desc((2, 3))), C.byref(desc((4, 5))), C.byref(out)) == 2
