"""Tensor.clone / toContiguous / ops.cast on HBM (zpucuda_tensor_copy)
against the oracle's writeF64(readLogical) restatement: bit-exact for every
pair of zpu's nine element types, for contiguous, transposed, sliced,
flipped (negative strides) and broadcast (zero strides) views."""
import ctypes as C

import numpy as np
import pytest

from oracle import zpu_oracle as zo

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TORCH = [torch.float64, torch.float32, torch.float16, torch.int64, torch.int32, torch.int16, torch.int8,
         torch.uint8, torch.bool]
NAMES = ["f64", "f32", "f16", "i64", "i32", "i16", "i8", "u8", "bool"]


@pytest.fixture(scope="module")
def zc():
    import zpu_b200
    zpu_b200.check(zpu_b200.lib().zpucuda_init(0))
    return zpu_b200


def special_values(k):
    """Values of zpu type k that exercise every conversion rule."""
    dt = zo.DTYPES[k]
    if np.dtype(dt).kind == "f":
        v = [0.0, -0.0, 1.5, -1.5, 2.5, -2.7, 0.49, 127.9, 128.0, -128.6, -129.0, 255.9, 256.0, 32767.5,
             65504.0, 65520.0, 70000.0, 2.0 ** 31, -2.0 ** 31 - 1, 1e10, -1e10, 2.0 ** 53 + 2, 2.0 ** 63,
             -2.0 ** 63, 1e30, 3.4e38, 1e-8, 6e-8, np.inf, -np.inf, np.nan]
        with np.errstate(over="ignore"):
            return np.array(v, dtype=np.float64).astype(dt)
    if np.dtype(dt).kind == "b":
        return np.array([True, False, True, True, False])
    info = np.iinfo(dt)
    v = [0, 1, -1, 2, 127, -128, 255, info.max, info.min, info.max - 1, info.min + 1]
    if dt == np.int64:
        v += [2 ** 53 + 1, 2 ** 53 - 1, -(2 ** 53) - 1, 2 ** 62 + 3, 1 << 40]
    return np.array([x for x in v if info.min <= x <= info.max], dtype=dt)


def same_bits(got, want):
    if got.dtype.kind == "f":
        return np.array_equal(got, want, equal_nan=True) and np.array_equal(np.signbit(got), np.signbit(want))
    return np.array_equal(got, want)


@pytest.mark.parametrize("src", range(9), ids=NAMES)
@pytest.mark.parametrize("dst", range(9), ids=NAMES)
def test_cast_every_type_pair(zc, src, dst):
    x = special_values(src)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(x.shape, dtype=TORCH[dst], device="cuda")
    zc.tensor_copy(xd, out)
    want = zo.tensor_copy(x, zo.DTYPES[dst])
    got = out.cpu().numpy()
    assert same_bits(got, want), (NAMES[src], NAMES[dst], x, got, want)


@pytest.mark.parametrize("dst", [torch.float32, torch.float64, torch.int32, torch.float16])
def test_transposed_views_take_the_tiled_path(zc, dst):
    """swapLastTwo views ([R, C] with unit stride on R), batched and ragged."""
    for shape in [(300, 257), (3, 65, 129), (2, 2, 31, 33), (1, 1)]:
        x = zo.uniform_range(11, int(np.prod(shape)), -300.0, 300.0).reshape(shape)
        xd = torch.from_numpy(x).cuda().transpose(-1, -2)
        out = torch.empty(xd.shape, dtype=dst, device="cuda")
        zc.tensor_copy(xd, out)
        want = zo.tensor_copy(np.swapaxes(x, -1, -2), zo.DTYPES[TORCH.index(dst)])
        assert same_bits(out.cpu().numpy(), want), shape


def spread_values(k, n):
    """n values of zpu type k spread over most of its range."""
    dt = zo.DTYPES[k]
    u = zo.uniform_range(21, n, -1.0, 1.0)
    kind = np.dtype(dt).kind
    if kind == "f":
        return (u * (3.0e4 if dt == np.float16 else 3.0e7)).astype(dt)  # f32 of i32 beyond 2^24 rounds
    if kind == "b":
        return u > 0
    info = np.iinfo(dt)
    if info.min == 0:
        return ((u + 1.0) * 0.5 * info.max).astype(dt)
    return (u * min(info.max, 2 ** 40)).astype(dt)


@pytest.mark.parametrize("dst", [torch.float64, torch.float32, torch.float16, torch.int8, torch.bool],
                         ids=["f64", "f32", "f16", "i8", "bool"])
@pytest.mark.parametrize("src", range(9), ids=NAMES)
def test_transposed_aligned_views(zc, src, dst):
    """16-byte aligned views (every dim a multiple of 16 elements, ragged
    64- and 128-tiles) take the 16-byte transpose for every element size; a
    one-element offset with an odd ld takes the 1-element kernel; a flipped
    column axis (negative ld) and a broadcast batch axis (stride 0) cover the
    addressing of both."""
    cases = []
    for shape in [(144, 80), (3, 48, 32), (272, 256), (2, 2, 16, 32), (400, 272)]:
        x = spread_values(src, int(np.prod(shape))).reshape(shape)
        cases.append((torch.from_numpy(x).cuda().transpose(-1, -2), np.swapaxes(x, -1, -2)))
    x = spread_values(src, 67 * 131).reshape(67, 131)  # offset 1 element, ld 131
    cases.append((torch.from_numpy(x).cuda()[:, 1:].transpose(0, 1), x[:, 1:].T))
    x = spread_values(src, 96 * 128).reshape(96, 128)  # [R=128, C=96] view with ld = -128
    xd = torch.from_numpy(x).cuda()
    d = zc.Tensor()
    d.data = xd.data_ptr() + (95 * 128) * x.itemsize
    d.dtype = src
    d.rank = 2
    d.dims[0], d.dims[1] = 128, 96
    d.strides[0], d.strides[1] = 1, -128
    cases.append((d, x[::-1].T))
    x = spread_values(src, 64 * 80).reshape(64, 80)  # batch axis of stride 0
    cases.append((torch.from_numpy(x).cuda().expand(3, 64, 80).transpose(-1, -2),
                  np.broadcast_to(x, (3, 64, 80)).swapaxes(-1, -2)))
    for view, npv in cases:
        out = torch.empty(npv.shape, dtype=dst, device="cuda")
        zc.tensor_copy(view, out)
        want = zo.tensor_copy(np.ascontiguousarray(npv), zo.DTYPES[TORCH.index(dst)])
        assert same_bits(out.cpu().numpy(), want), npv.shape


@pytest.mark.parametrize("inner", [2, 4])
def test_transpose_of_more_batches_than_one_grid_holds(zc, inner):
    """65537 batches: the grid's z axis holds 65535, the rest is a second
    launch (scalar kernel at 2 x 2, 16-byte kernel at 4 x 4)."""
    nb = 65537
    x = np.arange(nb * inner * inner, dtype=np.float32).reshape(nb, inner, inner)
    out = torch.empty((nb, inner, inner), dtype=torch.float32, device="cuda")
    zc.tensor_copy(torch.from_numpy(x).cuda().transpose(-1, -2), out)
    assert np.array_equal(out.cpu().numpy(), np.swapaxes(x, -1, -2))


def test_sliced_and_broadcast_views(zc):
    x = zo.uniform_range(12, 40 * 50, -5.0, 5.0).reshape(40, 50).astype(np.float64)
    xd = torch.from_numpy(x).cuda()
    for view, npv in [(xd[3:37:3, 1::2], x[3:37:3, 1::2]), (xd[:, 7], x[:, 7]),
                      (xd[5].expand(6, 50), np.broadcast_to(x[5], (6, 50))),
                      (xd.T[10:20, ::5], x.T[10:20, ::5])]:
        out = torch.empty(view.shape, dtype=torch.float32, device="cuda")
        zc.tensor_copy(view, out)
        assert same_bits(out.cpu().numpy(), zo.tensor_copy(npv, np.float32))


def test_flipped_view_with_negative_strides(zc):
    """ops.flip gives negative strides (tensor.zig:376-381): the descriptor
    points at element (0, 0) of the view, the last row of the buffer."""
    x = np.arange(7 * 9, dtype=np.float32).reshape(7, 9)
    xd = torch.from_numpy(x).cuda()
    d = zc.Tensor()
    d.data = xd.data_ptr() + (6 * 9) * 4  # row 6, column 0
    d.dtype = zc.F32
    d.rank = 2
    d.dims[0], d.dims[1] = 7, 9
    d.strides[0], d.strides[1] = -9, 1
    out = torch.empty((7, 9), dtype=torch.int16, device="cuda")
    zc.tensor_copy(d, out)
    assert np.array_equal(out.cpu().numpy(), x[::-1].astype(np.int16))
    # both axes flipped: element (0, 0) is the buffer's last element
    d.data = xd.data_ptr() + (7 * 9 - 1) * 4
    d.strides[0], d.strides[1] = -9, -1
    out64 = torch.empty((7, 9), dtype=torch.float64, device="cuda")
    zc.tensor_copy(d, out64)
    assert np.array_equal(out64.cpu().numpy(), x[::-1, ::-1].astype(np.float64))


def test_clone_of_large_i64_rounds_through_f64_as_zpu_does(zc):
    x = np.array([2 ** 53 + 1, 2 ** 62 + 3, -(2 ** 53) - 1, 7], dtype=np.int64)
    out = torch.empty(4, dtype=torch.int64, device="cuda")
    zc.tensor_copy(torch.from_numpy(x).cuda(), out)
    assert np.array_equal(out.cpu().numpy(), zo.tensor_copy(x, np.int64))
    assert out.cpu().numpy()[0] == 2 ** 53  # round to nearest even


def test_clone_of_a_contiguous_float_tensor_is_a_copy(zc):
    x = torch.randn(1000, 33, device="cuda")
    out = torch.empty_like(x)
    zc.tensor_copy(x, out)
    assert torch.equal(out, x) and out.data_ptr() != x.data_ptr()


def test_shape_and_type_errors(zc):
    x = torch.zeros(4, 5, device="cuda")
    with pytest.raises(zc.ZpuCudaError) as e:
        zc.tensor_copy(x, torch.empty(5, 4, device="cuda"))
    assert e.value.status == 2  # ShapeMismatch
    d = zc.tensor_desc(x)
    d.dtype = 12
    with pytest.raises(zc.ZpuCudaError) as e:
        zc.tensor_copy(d, torch.empty(4, 5, device="cuda"))
    assert e.value.status == 9  # NotSupported
    zc.tensor_copy(torch.zeros(0, 3, device="cuda"), torch.empty(0, 3, dtype=torch.int8, device="cuda"))


def test_transpose_bandwidth(zc):
    """toContiguous of an 8192 x 4096 f32 swapLastTwo view (the matmul VJP's
    transposed activations): both directions coalesced, HBM-bound."""
    x = torch.randn(4096, 8192, device="cuda").T
    out = torch.empty(8192, 4096, device="cuda")
    for _ in range(3):
        zc.tensor_copy(x, out)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(10):
        zc.tensor_copy(x, out)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / 10
    gbs = 2 * 8192 * 4096 * 4 / ms / 1e6
    print("transpose 8192x4096 f32: %.3f ms, %.0f GB/s" % (ms, gbs))
    assert torch.equal(out, x.contiguous())
    assert gbs > 2500


def test_cast_and_view_snapshots_on_device(zc, golden):
    """tests/snap/zpu.zig:48,96-97 through zpucuda_tensor_copy."""
    s6 = torch.tensor(golden["inputs"]["spread6"], dtype=torch.float64, device="cuda")
    out = torch.empty(6, dtype=torch.bool, device="cuda")
    zc.tensor_copy(s6, out)
    assert out.cpu().numpy().astype(np.float64).tolist() == golden["snapshots"]["zpu/tensor/bools"]["values"]
    x = torch.tensor(golden["inputs"]["spread12"], dtype=torch.float64, device="cuda").reshape(3, 4)
    t = torch.empty(4, 3, dtype=torch.float64, device="cuda")
    zc.tensor_copy(x.T, t)
    snapv = golden["snapshots"]["zpu/shape/transpose"]
    assert np.allclose(t.cpu().numpy().ravel(), snapv["values"], rtol=snapv["tol"], atol=snapv["tol"])
    d = zc.tensor_desc(x)
    d.data = x.data_ptr() + 3 * 8  # flip(x, 1): element (0, 0) is x[0, 3]
    d.strides[1] = -1
    f = torch.empty(3, 4, dtype=torch.float64, device="cuda")
    zc.tensor_copy(d, f)
    snapv = golden["snapshots"]["zpu/shape/flip"]
    assert np.allclose(f.cpu().numpy().ravel(), snapv["values"], rtol=snapv["tol"], atol=snapv["tol"])
