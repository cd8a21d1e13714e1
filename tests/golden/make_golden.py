"""Extracts the golden vectors for the hot path from the reference checkout.

Run once, in a container that has the reference mounted:

    python tests/golden/make_golden.py <path of the zpu checkout>

It reads the reference's own snapshot files (snapshots/zpu/**.snap, written by
`zig build test -Dupdate-snapshots`) and pairs each with the inputs that
tests/snap/zpu.zig feeds it, plus the known answers of src/zpu/tests.zig and
the kernel tests of src/zpu/kernels.zig.  The result, zpu_golden.json, is
committed; the tests read only that file, never the reference.
"""
import json
import math
import os
import sys

CASES = {
    # name -> (snapshot path, tolerance from tests/snap/zpu.zig)
    "linalg/matmul-3x3": 1e-9,     # tests/snap/zpu.zig:118
    "linalg/matvec": 1e-9,         # tests/snap/zpu.zig:119
    "linalg/norm": 1e-9,           # tests/snap/zpu.zig:124 (sqrt(sum(square(a))))
    "linalg/trace": 1e-9,          # tests/snap/zpu.zig:125 (sum of the diagonal)
    "linalg/diag": 1e-9,           # tests/snap/zpu.zig:126
    "linalg/outer": 1e-9,          # tests/snap/zpu.zig:127 (expandDims(a, -1) * b)
    "linalg/dot": 1e-9,            # tests/snap/zpu.zig:128 (sum(mul(b, b), -1))
    "nn/layer-norm": 1e-9,         # tests/snap/zpu.zig:151 (nn.zig:202-222)
    "grad/arg0": 1e-9,             # tests/snap/zpu.zig:196-202: grad of
    "grad/arg1": 1e-9,             #   sum(softmax(sigmoid(x.w) + b) * target)
    "grad/arg2": 1e-9,             #   w.r.t. x, w, b
    "grad/jvp-value": 1e-9,        # tests/snap/zpu.zig:217 (the function's value)
    "grad/jvp-tangent": 1e-9,      # tests/snap/zpu.zig:218 (J.v along a tangent of x)
    "nn/attention": 1e-9,          # tests/snap/zpu.zig:298-329 (softmax(q.k^T / 2).v, wq = wk = wv)
    "transforms/vmap": 1e-9,       # tests/snap/zpu.zig:279
    "transforms/jit-replay": 1e-9, # tests/snap/zpu.zig:288
    "reduce/sum-all": 1e-9,        # tests/snap/zpu.zig:85
    "reduce/sum-axis0": 1e-9,      # tests/snap/zpu.zig:86
    "reduce/sum-axis1-keepdims": 1e-9,  # tests/snap/zpu.zig:87
    "reduce/max-axis1": 1e-9,      # tests/snap/zpu.zig:88
    "reduce/min-axis0": 1e-9,      # tests/snap/zpu.zig:89
    "reduce/mean-axis1": 1e-9,     # tests/snap/zpu.zig:90
    "reduce/variance-axis1": 1e-9, # tests/snap/zpu.zig:91
    "reduce/prod-axis1": 1e-9,     # tests/snap/zpu.zig:92
    "reduce/argmax-axis1": 0.0,    # tests/snap/zpu.zig:93
    "reduce/cumsum-axis1": 1e-9,   # tests/snap/zpu.zig:94
    "reduce/cumsum-reverse": 1e-9, # tests/snap/zpu.zig:95
    "ops/tanh": 1e-9,              # tests/snap/zpu.zig:62
    "ops/exp": 1e-9,               # tests/snap/zpu.zig:60
    "ops/sigmoid": 1e-9,           # tests/snap/zpu.zig:61
    "ops/erf": 1e-9,               # tests/snap/zpu.zig:63
    "ops/mul-scalar": 1e-9,        # tests/snap/zpu.zig:67
    "ops/add-broadcast": 1e-9,     # tests/snap/zpu.zig:66
    "ops/square-rsqrt": 1e-9,      # tests/snap/zpu.zig:65
    "ops/sqrt-abs": 1e-9,          # tests/snap/zpu.zig:64
    "ops/maximum": 1e-9,           # tests/snap/zpu.zig:68
    "ops/where": 1e-9,             # tests/snap/zpu.zig:69-73 (where(gt(x, 0), x, neg(x)))
    "ops/clamp": 1e-9,             # tests/snap/zpu.zig:74
    "ops/lerp": 1e-9,              # tests/snap/zpu.zig:75
    "nn/log-softmax": 1e-9,        # tests/snap/zpu.zig:143
    "nn/softmax": 1e-9,            # tests/snap/zpu.zig:142
    "optim/adam-step1": 1e-9,      # tests/snap/zpu.zig:340
    "optim/adam-step10": 1e-9,     # tests/snap/zpu.zig:342
    "tensor/bools": 0.0,           # tests/snap/zpu.zig:48 (cast of spread(6) to bool)
    "shape/transpose": 1e-9,       # tests/snap/zpu.zig:96
    "shape/flip": 1e-9,            # tests/snap/zpu.zig:97
    "shape/pad": 1e-9,             # tests/snap/zpu.zig:98 (pads (1,0),(0,2), value -1)
    "shape/take": 1e-9,            # tests/snap/zpu.zig:99 (i32 indices [2,0,2], axis 0)
    "shape/concat": 1e-9,          # tests/snap/zpu.zig:100 (x with itself, axis 1)
    "shape/stack": 1e-9,           # tests/snap/zpu.zig:101 (x with itself, axis 0)
    "rng/normal-seed12345": 0.0,   # tests/snap/zpu.zig:355
    "rng/uniform-seed12345": 0.0,  # tests/snap/zpu.zig:358
}


def parse_snap(path):
    shape, dtype, values = None, None, []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            if line.startswith("#"):
                parts = line[1:].split()
                if parts and parts[0] == "shape":
                    i = parts.index("dtype")
                    dims = parts[1:i]
                    shape = [] if dims == ["()"] else [int(d) for d in dims]
                    dtype = parts[i + 1]
                continue
            values.extend(float(v) for v in line.split())
    return {"shape": shape, "dtype": dtype, "values": values}


def spread(n):
    """tests/snap/zpu.zig:28-36: sin(0.7 i) * 1.5 + 0.01 i - 0.25."""
    return [math.sin(i * 0.7) * 1.5 + i * 0.01 - 0.25 for i in range(n)]


def main(ref):
    snaps = {}
    for name, tol in CASES.items():
        snap = parse_snap(os.path.join(ref, "snapshots", "zpu", name + ".snap"))
        snap["tol"] = tol
        snaps["zpu/" + name] = snap
    with open(os.path.join(ref, "snapshots", "zpu", "transforms", "jit-steps.snap")) as f:
        jit_steps = int(f.read().split()[1])

    inputs = {
        # tests/snap/zpu.zig:111-119
        "spd3": [4.0, 1.0, 0.5, 1.0, 3.0, 0.25, 0.5, 0.25, 2.0],
        "rhs3": [1.0, 2.0, 3.0],
        # tests/snap/zpu.zig:28-36 (x = spread(8) for ops, spread(12) as 3x4 for reductions)
        "spread6": spread(6),
        "spread8": spread(8),
        "spread12": spread(12),
        # tests/snap/zpu.zig:137-141
        "logits3x3": [1.0, 2.0, 3.0, -1.0, 0.0, 0.5, 2.5, -2.5, 0.0],
        # tests/snap/zpu.zig:127 (outer of [1, 2] and [3, 4, 5])
        "outer_a": [1.0, 2.0],
        "outer_b": [3.0, 4.0, 5.0],
        # tests/snap/zpu.zig:145-151: layerNorm(rows [2, 3], ones(3), bias, 1e-5, -1)
        "ln_rows": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0],
        "ln_weight": [1.0, 1.0, 1.0],
        "ln_bias": [0.5, -0.5, 1.0],
        "ln_eps": 1e-5,
        # tests/snap/zpu.zig:190-193, 209: x [2, 3], w [3, 2], b [2], target [2, 2], tangent of x
        "grad_x": [0.5, -1.0, 2.0, 0.25, -0.5, 1.5],
        "grad_w": [1.0, -1.0, 0.5, 0.25, 2.0, -0.5],
        "grad_b": [0.1, -0.2],
        "grad_target": [1.0, 0.0, 0.25, 0.75],
        "grad_tangent": [0.3, -0.7, 0.2, 0.4, -0.1, 0.6],
        # tests/snap/zpu.zig:317-327: x [4, 3] and the one weight [3, 3]
        "attn_x": [0.5, -1.0, 2.0, 1.0, 0.5, -0.5, -1.0, 2.0, 0.25, 0.0, 1.0, 1.0],
        "attn_w": [1.0, 0.0, 0.5, 0.0, 1.0, -0.5, 0.5, 0.5, 1.0],
        # tests/snap/zpu.zig:267-276 (shape [3,2,2] each); f = tanh(matmul(a, b))
        "vmap_a": [1, 2, 3, 4, 0.5, -1, 2, 0.25, 2, 0, -1, 1],
        "vmap_b": [1, 0, 0, 1, 2, -1, 0.5, 1, -1, 1, 1, 0],
        # tests/snap/zpu.zig:333-342: Adam(lr=0.01) on f64 params
        "adam_params": [1.0, -2.0, 0.5],
        "adam_grads": [0.1, -0.25, 0.05],
        "adam_lr": 0.01,
        "rng_seed": 12345,
    }

    known = [
        # src/zpu/tests.zig:145-171
        {"name": "matmul 2x3 @ 3x2", "a": [1, 2, 3, 4, 5, 6], "a_shape": [2, 3],
         "b": [7, 8, 9, 10, 11, 12], "b_shape": [3, 2], "want": [58, 64, 139, 154], "tol": 1e-12},
        {"name": "matmul vector @ matrix", "a": [1, 1, 1], "a_shape": [3],
         "b": [7, 8, 9, 10, 11, 12], "b_shape": [3, 2], "want": [27, 30], "tol": 1e-12},
        {"name": "matmul matrix @ vector", "a": [1, 2, 3, 4, 5, 6], "a_shape": [2, 3],
         "b": [1, 1, 1], "b_shape": [3], "want": [6, 15], "tol": 1e-12},
        {"name": "matmul batched", "a": [1, 2, 3, 4, 1, 0, 0, 1], "a_shape": [2, 2, 2],
         "b": [5, 6, 7, 8, 1, 2, 3, 4], "b_shape": [2, 2, 2], "want": [19, 22, 43, 50, 1, 2, 3, 4],
         "tol": 1e-12},
        {"name": "matmul batch broadcast", "a": [1, 2, 3, 4, 1, 0, 0, 1], "a_shape": [2, 2, 2],
         "b": [1, 2, 3, 4], "b_shape": [2, 2], "want": [7, 10, 15, 22, 1, 2, 3, 4], "tol": 1e-12},
    ]

    # src/zpu/tests.zig:116-124: reductions of [[1,2,3],[4,5,6]] (f64);
    # examples/audit_edge_cases.zig:138-144: argmax of a length-5 f32 vector
    reduce_known = [
        {"name": "sum axis 0", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "prim": "sum", "axis": 0,
         "keepdims": 0, "want": [5, 7, 9], "want_shape": [3], "tol": 1e-12},
        {"name": "sum axis -1", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "prim": "sum", "axis": -1,
         "keepdims": 0, "want": [6, 15], "want_shape": [2], "tol": 1e-12},
        {"name": "sum axis 1 keepdims", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "prim": "sum", "axis": 1,
         "keepdims": 1, "want": [6, 15], "want_shape": [2, 1], "tol": 1e-12},
        {"name": "max axis 0", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "prim": "max_reduce", "axis": 0,
         "keepdims": 0, "want": [4, 5, 6], "want_shape": [3], "tol": 1e-12},
        {"name": "min axis 1", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "prim": "min_reduce", "axis": 1,
         "keepdims": 0, "want": [1, 4], "want_shape": [2], "tol": 1e-12},
        {"name": "argmax axis -1", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "prim": "argmax", "axis": -1,
         "keepdims": 0, "want": [2, 2], "want_shape": [2], "tol": 0.0},
        {"name": "argmax of a vector (f32)", "x": [1.0, 5.0, 3.0, 2.0, 4.0], "shape": [5], "dtype": "f32",
         "prim": "argmax", "axis": 0, "keepdims": 0, "want": [1], "want_shape": [], "tol": 0.0},
    ]

    # src/zpu/tests.zig:97-101 (a = 1..6 as 2 x 3) and :873-877 (lt of the
    # i64 [1, 2, 3, 4] against 3, any / all; the f64 values compare alike)
    # src/zpu/tests.zig:125-126: cumsum of [[1,2,3],[4,5,6]] along axis 1
    cumsum_known = [
        {"x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "axis": 1, "reverse": False, "want": [1, 3, 6, 4, 9, 15]},
        {"x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "axis": 1, "reverse": True, "want": [6, 5, 3, 15, 11, 6]},
    ]
    pred_known = [
        {"name": "gt(a, 3)", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3], "want": [0, 0, 0, 1, 1, 1]},
        {"name": "where(gt(a, 3), a, neg(a))", "x": [1, 2, 3, 4, 5, 6], "shape": [2, 3],
         "want": [-1, -2, -3, 4, 5, 6]},
        {"name": "any(lt(i, 3))", "x": [1, 2, 3, 4], "shape": [2, 2], "want": [1]},
        {"name": "all(lt(i, 3))", "x": [1, 2, 3, 4], "shape": [2, 2], "want": [0]},
    ]

    # src/zpu/kernels.zig:512-543: gemm vs the naive triple loop at 1e-12 on
    # these shapes, inputs a[i] = (i % 7) * 0.5 - 1, b[i] = (i % 5) * 0.25 - 0.5.
    gemm_shapes = [[1, 1, 1], [3, 4, 5], [32, 7, 128], [35, 9, 133], [2, 33, 2]]
    # src/zpu/kernels.zig:545-581: reduction edges (lengths 0, 1, L, L+1, 4L+3
    # of 0..len-1 sum exactly) and data[i] = sin(0.37 i) * 3 for n = 1000.
    reduce_lengths = [0, 1, 8, 9, 35]

    out = {
        "generated_by": "tests/golden/make_golden.py",
        "reference_files": ["snapshots/zpu/**/*.snap", "tests/snap/zpu.zig",
                            "src/zpu/tests.zig", "src/zpu/kernels.zig"],
        "snapshot_tolerance_rule": "|w - g| <= tol * max(1, |w|, |g|)  (tests/snapshot.zig:239-244)",
        "snapshots": snaps,
        "jit_steps": jit_steps,
        "inputs": inputs,
        "known_answers": known,
        "reduce_known": reduce_known,
        "pred_known": pred_known,
        "cumsum_known": cumsum_known,
        "gemm_shapes": gemm_shapes,
        "reduce_lengths": reduce_lengths,
    }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "zpu_golden.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the zpu checkout>")
    main(sys.argv[1])
