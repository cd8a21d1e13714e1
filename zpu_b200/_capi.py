"""ctypes binding of libzpucuda.so (the C ABI declared in include/zpucuda.h).

This is the same binding a Zig, Go or Python caller writes against the
header; the Python package uses it for the tests and the benchmark.  The
library must exist: there is no fallback of any kind when it is missing.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# ZPUCUDA_LIB names another build of the library (same ABI) to load instead.
LIB_PATH = os.environ.get("ZPUCUDA_LIB") or os.path.join(HERE, "libzpucuda.so")

MAX_RANK = 8
AXIS_NONE = -2
F64, F32 = 0, 1
DT_I64 = 3  # zpu DType.i64: argmax / argmin results
DT_BOOL = 8  # zpu DType.bool (one byte): predicates, any / all
# residency states of a buffer (zpucuda_buf_residency)
RES_DEVICE, RES_HOST, RES_BOTH = 1, 2, 3

STATUS = {
    0: "ok", 1: "OutOfMemory", 2: "ShapeMismatch", 3: "DTypeMismatch", 4: "RankTooLarge",
    5: "InvalidShape", 6: "InvalidAxis", 7: "NonContiguous", 8: "IndexOutOfRange",
    9: "NotSupported", 10: "NotDifferentiable", 11: "NotPositiveDefinite", 12: "DeviceMismatch",
    13: "Timeout", 14: "CudaError", 15: "NoDevice", 16: "InvalidArgument",
}

# src/zpu/prims.zig:9-109
PRIM = {
    "neg": 0, "abs": 1, "exp": 2, "expm1": 3, "log": 4, "log1p": 5, "sqrt": 6, "rsqrt": 7,
    "square": 8, "recip": 9, "cbrt": 10, "sin": 11, "cos": 12, "tan": 13, "asin": 14,
    "acos": 15, "atan": 16, "sinh": 17, "cosh": 18, "tanh": 19, "asinh": 20, "acosh": 21,
    "atanh": 22, "erf": 23, "sigmoid": 24, "softplus": 25, "relu": 26, "floor": 27,
    "ceil": 28, "round": 29, "trunc": 30, "sign": 31, "isnan": 32, "isinf": 33,
    "isfinite": 34, "add": 35, "sub": 36, "mul": 37, "div": 38, "pow": 39, "maximum": 40,
    "minimum": 41, "atan2": 42, "hypot": 43, "mod_op": 44, "eq": 45, "ne": 46, "lt": 47, "le": 48,
    "gt": 49, "ge": 50, "logical_and": 51, "logical_or": 52, "logical_xor": 53, "logical_not": 54,
    "where": 55, "sum": 58, "prod_op": 59, "max_reduce": 60, "min_reduce": 61, "any_reduce": 62,
    "all_reduce": 63, "argmax": 64, "argmin": 65, "reshape": 66, "transpose": 67, "broadcast": 68, "expand_dims": 69,
    "squeeze": 70, "slice": 71, "concat_op": 72, "stack_op": 73, "take": 74, "scatter_add": 75,
    "pad": 76, "flip": 77, "cumsum": 78, "reverse": 79, "matmul": 80,
    "constant": 87, "copy": 88, "cast_op": 89,
}


class ZpuCudaError(RuntimeError):
    def __init__(self, status, message=""):
        self.status = status
        self.name = STATUS.get(status, "status %d" % status)
        super().__init__("%s%s" % (self.name, (": " + message) if message else ""))


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int32), ("rank", C.c_int32),
                ("dims", C.c_int64 * MAX_RANK), ("strides", C.c_int64 * MAX_RANK),
                ("batch_depth", C.c_int32)]


class Value(C.Structure):
    _fields_ = [("id", C.c_uint64), ("dtype", C.c_int32), ("rank", C.c_int32),
                ("dims", C.c_int64 * MAX_RANK), ("batch_depth", C.c_int32)]


class Step(C.Structure):
    _fields_ = [("prim", C.c_int32), ("n_inputs", C.c_int32), ("ins", C.c_uint64 * 3),
                ("out", C.c_uint64), ("axis", C.c_int32), ("flags", C.c_int32),
                ("shape", C.c_int64 * MAX_RANK), ("shape_len", C.c_int32), ("nsl", C.c_int32),
                ("perm", C.c_uint8 * MAX_RANK), ("starts", C.c_int64 * MAX_RANK),
                ("steps", C.c_int64 * MAX_RANK), ("pads_hi", C.c_int64 * MAX_RANK), ("scalar", C.c_double)]


class Blob(C.Structure):
    _fields_ = [("value", Value), ("host_data", C.c_void_p)]


_lib = None

P, I32, I64, U64, S = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_size_t
SIGNATURES = {
    "zpucuda_status_string": (C.c_char_p, [I32]),
    "zpucuda_last_error": (C.c_char_p, []),
    "zpucuda_version": (I32, []),
    "zpucuda_device_count": (I32, [C.POINTER(I32)]),
    "zpucuda_init": (I32, [I32]),
    "zpucuda_thread_bind": (I32, [I32]),
    "zpucuda_get_stream": (I32, [C.POINTER(P)]),
    "zpucuda_set_stream": (I32, [P]),
    "zpucuda_sync": (I32, [I64]),
    "zpucuda_launch_count": (U64, []),
    "zpucuda_check_device": (I32, []),
    "zpucuda_buf_alloc": (I32, [S, C.POINTER(P)]),
    "zpucuda_buf_alloc_zeroed": (I32, [S, C.POINTER(P)]),
    "zpucuda_buf_wrap": (I32, [P, S, C.POINTER(P)]),
    "zpucuda_buf_retain": (P, [P]),
    "zpucuda_buf_release": (None, [P]),
    "zpucuda_buf_refcount": (C.c_uint32, [P]),
    "zpucuda_buf_devptr": (P, [P]),
    "zpucuda_buf_bytes": (S, [P]),
    "zpucuda_buf_upload": (I32, [P, S, P, S]),
    "zpucuda_buf_download": (I32, [P, S, P, S]),
    "zpucuda_buf_attach_host": (I32, [P, P, I32]),
    "zpucuda_buf_residency": (I32, [P, C.POINTER(I32)]),
    "zpucuda_buf_mark_device_dirty": (I32, [P]),
    "zpucuda_buf_mark_host_dirty": (I32, [P]),
    "zpucuda_buf_host_sync": (I32, [P, P]),
    "zpucuda_buf_device_sync": (I32, [P, P]),
    "zpucuda_buf_transfer_stats": (I32, [C.POINTER(U64), C.POINTER(U64)]),
    "zpucuda_scope_begin": (I32, [C.POINTER(P)]),
    "zpucuda_scope_end": (I32, [P]),
    "zpucuda_scope_keep": (P, [P, P]),
    "zpucuda_scope_forget": (I32, [P, P]),
    "zpucuda_scope_count": (I64, [P]),
    "zpucuda_scope_installed": (I32, [P]),
    "zpucuda_gemm_f32": (I32, [P, P, P, I64, I64, I64, I64, I64, I64, I32, I32, I64, I64, I64, I64, P]),
    "zpucuda_gemm_f64": (I32, [P, P, P, I64, I64, I64, I64, I64, I64, I32, I32, I64, I64, I64, I64, P]),
    "zpucuda_matmul_shape": (I32, [C.POINTER(Tensor), C.POINTER(Tensor), C.POINTER(Tensor)]),
    "zpucuda_matmul": (I32, [C.POINTER(Tensor), C.POINTER(Tensor), C.POINTER(Tensor), P]),
    "zpucuda_plan_create": (I32, [C.POINTER(Value), I32, C.POINTER(Blob), I32, C.POINTER(Step), I32,
                                  C.POINTER(U64), I32, C.POINTER(P)]),
    "zpucuda_plan_run": (I32, [P, C.POINTER(P), C.POINTER(P), P]),
    "zpucuda_plan_run_host": (I32, [P, C.POINTER(P), C.POINTER(P), P]),
    "zpucuda_plan_output": (I32, [P, I32, C.POINTER(Value)]),
    "zpucuda_plan_num_steps": (I32, [P]),
    "zpucuda_plan_num_kernels": (I32, [P]),
    "zpucuda_plan_describe": (I32, [P, C.c_char_p, S]),
    "zpucuda_plan_destroy": (None, [P]),
    "zpucuda_rng_uniform": (I32, [U64, I32, P, I64, C.c_double, C.c_double, P]),
    "zpucuda_rng_normal": (I32, [U64, I32, P, I64, P]),
    "zpucuda_rng_randint": (I32, [U64, P, I64, I64, I64, P]),
    "zpucuda_chain_tanh_sq_affine_sum_noalloc": (I32, [P, I64, P, P, P, P]),
    "zpucuda_tensor_copy": (I32, [P, P, P]),
    "zpucuda_plan_check": (I32, [P, P]),
    "zpucuda_nccl_unique_id": (I32, [P]),
    "zpucuda_nccl_init": (I32, [I32, I32, P, I64]),
    "zpucuda_nccl_allreduce_f32": (I32, [P, I64, P]),
    "zpucuda_nccl_world": (I32, [C.POINTER(I32), C.POINTER(I32)]),
    "zpucuda_nccl_destroy": (I32, [I64]),
    "zpucuda_mlp_create": (I32, [I64, I64, I64, I64, I64, C.POINTER(P)]),
    "zpucuda_mlp_destroy": (None, [P]),
    "zpucuda_mlp_param_numel": (I32, [P, I32, C.POINTER(I64)]),
    "zpucuda_mlp_param_count": (I32, [P, C.POINTER(I64)]),
    "zpucuda_mlp_write": (I32, [P, I32, I32, P, I64, P]),
    "zpucuda_mlp_read": (I32, [P, I32, I32, P, I64, P]),
    "zpucuda_mlp_array": (I32, [P, I32, C.POINTER(P), C.POINTER(I64)]),
    "zpucuda_mlp_param_offset": (I32, [P, I32, C.POINTER(I64), C.POINTER(I64)]),
    "zpucuda_mlp_adam_config": (I32, [P, C.c_double, C.c_double, C.c_double, C.c_double]),
    "zpucuda_mlp_value_and_grad": (I32, [P, P, P, I64, I64, P]),
    "zpucuda_mlp_allreduce_grads": (I32, [P, P]),
    "zpucuda_mlp_adam_step": (I32, [P, P]),
    "zpucuda_mlp_train_step": (I32, [P, P, P, I64, I64, P]),
    "zpucuda_mlp_loss": (I32, [P, P, P]),
    "zpucuda_mlp_join": (I32, [P, P]),
    "zpucuda_mlp_check": (I32, [P]),
    "zpucuda_mlp_steps": (I64, [P]),
    "zpucuda_mlp_exchange_mode": (I32, [P]),
    "zpucuda_mlp_trace": (I32, [P, I32]),
    "zpucuda_mlp_trace_read": (I32, [P, P, I32]),
    "zpucuda_debug_peer_reduce": (I32, [P, I32, I64, P, P, U64, C.c_uint32, P, P]),
}


def exported_names():
    return list(SIGNATURES)


def lib():
    """The loaded library; raises when the in-tree build is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError("libzpucuda.so is not built (run `python -m zpu_b200.build`); "
                           "zpu_b200 has no CPU fallback")
    L = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status):
    if status != 0:
        msg = lib().zpucuda_last_error()
        raise ZpuCudaError(status, msg.decode() if msg else "")
    return status
