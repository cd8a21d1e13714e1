"""ops.matmul for the element types outside the tensor-core GEMMs, on the B200.

zpu computes mixed-type, f16 and bool-operand products with ops.gemmF64 (an
f64 product and sum per step, rounded to the promoted output type at every
step, src/zpu/ops.zig:1284-1333) and same-type integer products with the
element type's wrapping arithmetic (ops.gemmTyped, ops.zig:1016-1049).  The
device restates both loops, so the results are compared bit for bit with the
oracle's restatement (oracle.zpu_oracle.gemm_convert).
"""
import zlib

import numpy as np
import pytest

from oracle import zpu_oracle as zo

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

NP = {"f64": np.float64, "f32": np.float32, "f16": np.float16, "i64": np.int64, "i32": np.int32,
      "i16": np.int16, "i8": np.int8, "u8": np.uint8, "bool": np.bool_}


@pytest.fixture(scope="module")
def zc():
    import zpu_b200
    zpu_b200.check(zpu_b200.lib().zpucuda_init(0))
    return zpu_b200


def sample(rng, dt, shape):
    dt = np.dtype(NP[dt])
    if dt.kind == "f":
        return (rng.standard_normal(shape) * 3).astype(dt)
    if dt.kind == "b":
        return rng.integers(0, 2, shape).astype(dt)
    info = np.iinfo(dt)
    lo, hi = max(int(info.min), -100), min(int(info.max), 100)
    return rng.integers(lo, hi + 1, shape).astype(dt)


def run(zc, a, b):
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    C = zc.matmul(A, B)
    torch.cuda.synchronize()
    return C.cpu().numpy()


PAIRS = [("f16", "f16"), ("f32", "f64"), ("f64", "f32"), ("f16", "f32"), ("f32", "f16"), ("i32", "f32"),
         ("bool", "f32"), ("f64", "i64"), ("i32", "i32"), ("i8", "i8"), ("i64", "i64"), ("u8", "u8"),
         ("u8", "i8"), ("i8", "u8"), ("i16", "i32"), ("bool", "i16"), ("f16", "i64")]


@pytest.mark.parametrize("ta,tb", PAIRS)
@pytest.mark.parametrize("shape", [((5, 7), (7, 3)), ((3, 20, 33), (3, 33, 17)), ((1, 1), (1, 1)), ((4, 0), (0, 6))])
def test_matches_zpu_loops_bit_for_bit(zc, ta, tb, shape):
    rng = np.random.default_rng(zlib.crc32(repr((ta, tb, shape[0])).encode()))
    a, b = sample(rng, ta, shape[0]), sample(rng, tb, shape[1])
    got = run(zc, a, b)
    want = zo.gemm_convert(a, b)
    assert got.dtype == want.dtype
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (ta, tb)


def test_integer_products_wrap_in_the_element_type(zc):
    # 100 * 2 + 100 * 1 = 300 wraps to 300 - 256 = 44 in i8 (reduceStep's +%)
    a = np.array([[100, 100]], dtype=np.int8)
    b = np.array([[2], [1]], dtype=np.int8)
    got = run(zc, a, b)
    assert got.dtype == np.int8 and int(got[0, 0]) == 44
    assert np.array_equal(got, zo.gemm_convert(a, b))


def test_mixed_integers_clamp_at_every_step(zc):
    # u8 @ i8 promotes to i8 (mixed signedness, equal size: the second type),
    # and zpu's gemmF64 loop clamps each partial sum to [-128, 127]
    a = np.array([[200, 200, 1]], dtype=np.uint8)
    b = np.array([[1], [1], [-100]], dtype=np.int8)
    got = run(zc, a, b)
    want = zo.gemm_convert(a, b)
    assert got.dtype == np.int8 and np.array_equal(got, want) and int(want[0, 0]) == 27


def test_f16_rounds_every_partial_sum(zc):
    # 2048 + 1 + 1 in f16: each partial sum rounds (ulp 2 at 2048), so zpu gets
    # 2048 where an f32 accumulator would give 2050
    a = np.array([[2048.0, 1.0, 1.0]], dtype=np.float16)
    b = np.ones((3, 1), dtype=np.float16)
    got = run(zc, a, b)
    assert got.dtype == np.float16 and float(got[0, 0]) == 2048.0
    assert np.array_equal(got, zo.gemm_convert(a, b))


def test_transposed_and_broadcast_operands(zc):
    rng = np.random.default_rng(7)
    a = sample(rng, "f16", (6, 9))
    b = sample(rng, "f32", (4, 9))  # used as b^T: a (6,9) @ (9,4)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda().t()
    got = zc.matmul(A, B).cpu().numpy()
    assert np.array_equal(got, zo.gemm_convert(a, np.ascontiguousarray(b.T)))
    # one f64 matrix against a batch of f32 ones (batch broadcast)
    a3 = sample(rng, "f32", (5, 3, 8))
    b2 = sample(rng, "f64", (8, 2))
    got = zc.matmul(torch.from_numpy(a3).cuda(), torch.from_numpy(b2).cuda()).cpu().numpy()
    want = zo.gemm_convert(a3, np.broadcast_to(b2, (5, 8, 2)))
    assert np.array_equal(got, want)


def test_bool_at_bool_is_a_dtype_mismatch(zc):
    a = torch.ones(2, 2, dtype=torch.bool, device="cuda")
    with pytest.raises(zc.ZpuCudaError) as e:
        zc.matmul(a, a)
    assert e.value.name == "DTypeMismatch"


def test_plan_matmul_of_f32_and_f64_values(zc):
    rng = np.random.default_rng(3)
    a = sample(rng, "f32", (8, 5))
    b = sample(rng, "f64", (5, 6))
    plan = zc.Plan([(1, zc.F32, (8, 5)), (2, zc.F64, (5, 6))], [], [("matmul", [1, 2], 3, -2, 0)], [3])
    (got,) = plan.run([torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    got = got.cpu().numpy()
    assert got.dtype == np.float64
    assert np.array_equal(got, zo.gemm_convert(a, b))
