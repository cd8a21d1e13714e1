#!/usr/bin/env python
"""Benchmark of the zpu B200 execution layer: prints ONE JSON line.

Workload (the headline): the jit-fused chain y = sumAll(tanh(x*x)*a + b) on
x of 2^26 f32 ~ N(0,1) (rng.Rng(0x5EED0003).normal, generated on the device
by the library's own splitmix64/Box-Muller kernel), a = 0.5, b = -0.25 as
folded f32 constants.  One step = one run of the lowered jit plan = one fused
kernel reading the 256 MiB input once (inputs larger than L2, so no flush).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs one process per GPU (torchrun); every rank evaluates its own
2^26-element shard (weak scaling, no data-path collective); the time is the
max over ranks of the CUDA-event time of exactly K steps.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEED_X = 0x5EED0003
N_ELEM = 1 << 26
BYTES_PER_STEP = N_ELEM * 4 + 4  # read x once, write the f32 sum
A, B = 0.5, -0.25
METRIC = "fused-elementwise HBM GB/s: jit chain y = sumAll(tanh(x*x)*a + b), x = 2^26 f32"
WORKLOAD = "jit_chain_tanh_sq_affine_sum_2^26_f32"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--only", default=None, choices=sorted(ONLY_CASES),
                    help="run one workload alone (for profiling) and print its timing")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic(workload):
    """DRAM bytes per launch of the workload's kernel (dram__bytes_read.sum +
    dram__bytes_write.sum from one ncu capture), kept in
    profiles/traffic.json; None when no capture is recorded."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return int(json.load(f)[workload]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


class Clocks:
    """nvidia-smi samples (clocks, throttle reasons) while the GPU is loaded."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        import tempfile
        self.path = tempfile.mktemp(prefix="zpu_clocks_", suffix=".csv")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
            os.unlink(self.path)
        except OSError:
            return None
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def cpu_chain_baseline(seconds=12.0, steps=None, warmup=0):
    """zpu's CPU jit path (the oracle restatement with zpu's threading model)
    on the same workload.  Returns (GB/s, cores, sample text, per-step list)."""
    import numpy as np
    from oracle import zpu_oracle as zo
    cores = os.cpu_count() or 1
    zo.set_cores(cores)
    x = zo.normal(SEED_X, N_ELEM)
    t0 = time.perf_counter()
    zo.jit_chain_tanh_sq_affine_sum(x, A, B)
    one = time.perf_counter() - t0
    n = N_ELEM
    if steps is not None:
        # keep the whole reference run within ~2 minutes
        budget = 120.0 / max(1, steps + warmup)
        if one > budget:
            n = max(1 << 20, int(N_ELEM * budget / one) & ~1023)
        xs = np.ascontiguousarray(x[:n])
        for _ in range(warmup):
            zo.jit_chain_tanh_sq_affine_sum(xs, A, B)
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            zo.jit_chain_tanh_sq_affine_sum(xs, A, B)
            times.append(time.perf_counter() - t0)
        per = sum(times) / len(times)
        sample = "%d of the 2^26 elements per step (%s), %d steps" % (n, "full" if n == N_ELEM else "prefix", steps)
        return (n * 4 + 4) / per / 1e9, zo.worker_count(n), sample, per
    reps, total = 1, one
    while total < seconds:
        t0 = time.perf_counter()
        zo.jit_chain_tanh_sq_affine_sum(x, A, B)
        total += time.perf_counter() - t0
        reps += 1
    per = total / reps
    return BYTES_PER_STEP / per / 1e9, zo.worker_count(N_ELEM), "full 2^26-element workload, %d passes" % reps, per


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    gbs, cores, sample, per = cpu_chain_baseline(steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (rng.Rng(0x5EED0003).normal)",
        "config": {"workload": WORKLOAD, "n_elements": N_ELEM, "a": A, "b": B,
                   "parallelism": "CPU, zpu's threading model (parallel.zig)"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample + "; zpu's jit.Plan.runAll step by step (mul threaded "
                                   "min(cores, n/16000) ways, tanh/scalar ops/sum single-threaded)"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _peak_tflops():
    """TF32 and FP64 denominators: TF32 dense is half the measured bf16
    rate (MEASURED_PEAKS.json), 3xTF32's algorithmic ceiling a third of
    that; FP64 is the nominal 40 TFLOP/s (no measured FP64 peak exists)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16 = float(json.load(f)["bf16_tflops"])
        src = "measured bf16 / 2"
    except Exception:
        bf16, src = 1590.0, "fallback bf16 / 2"
    return bf16 / 2.0, 40.0, src


def _time_events(fn, reps, warm=2):
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _time_graph(fn, calls=20, reps=5):
    """Device time of one fn() call: `calls` calls captured in a CUDA graph,
    replayed `reps` times between CUDA events (host launch cost excluded).
    None when the calls cannot be captured."""
    import torch
    try:
        fn()
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(calls):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * calls)
        del g
        return ms
    except Exception:
        torch.cuda.synchronize()
        return None


def _max_over_ranks(ms, world, dev):
    if world == 1:
        return ms
    import torch
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch
        torch.distributed.barrier()


# 2-D output-tile grids for the f64 GEMM at 1, 2, 4, 8 ranks
F64_GRIDS = {1: (1, 1), 2: (1, 2), 4: (2, 2), 8: (2, 4)}


def gemm_configs(rank=0, world=1, dev="cuda"):
    """The GEMM workloads of the hot path, each timed with CUDA events on
    device-resident inputs (zpu's RNG streams, seeds per config), max over
    ranks, no data-path collective:
    1: f32 1024^3 U[-1,1], replicas (too small to split);
    3: vmap-batched 256 x 512^3 N(0, 1/512), rank r computes matrices
       [256 r / N, 256 (r+1) / N);
    5: f64 8192^3 N(0,1), 2-D output tiles on a 1x1 / 1x2 / 2x2 / 2x4 grid,
       each rank's A row panel and B column panel staged in its own HBM."""
    import torch
    import zpu_b200 as zc
    tf32, fp64, src = _peak_tflops()
    out = {}
    n = 1024
    A = zc.rng_uniform(0x5EED0001, n * n, -1.0, 1.0, device=dev).view(n, n)
    B = zc.rng_uniform(0x5EED0002, n * n, -1.0, 1.0, device=dev).view(n, n)
    C = torch.empty(n, n, device=dev)
    _barrier(world)
    host_ms = _max_over_ranks(_time_events(lambda: zc.matmul(A, B, out=C), 20), world, dev)
    # at ~10 us of device time per product, the Python call that launches it
    # costs as much: the device time comes from a CUDA graph of 20 calls
    g_ms = _time_graph(lambda: zc.matmul(A, B, out=C))
    ms = _max_over_ranks(g_ms if g_ms is not None else host_ms, world, dev)
    t = 2 * n ** 3 / ms / 1e9
    out["config1_f32_gemm_1024"] = {"tflops_per_replica": t, "ms": ms, "frac_of_3xtf32_ceiling": t / (tf32 / 3),
                                    "ceiling_tflops": tf32 / 3, "ceiling_source": src,
                                    "timing": "CUDA graph of 20 calls" if g_ms is not None else "host loop",
                                    "host_loop_ms": host_ms, "tflops_host_loop": 2 * n ** 3 / host_ms / 1e9,
                                    "parallelism": "replicas (%d)" % world}
    bsz, n = 256, 512
    s = 1.0 / (512.0 ** 0.5)
    A = (zc.rng_normal(0x5EED0004, bsz * n * n, device=dev) * s).view(bsz, n, n)
    B = (zc.rng_normal(0x5EED0005, bsz * n * n, device=dev) * s).view(bsz, n, n)
    per = bsz // world
    A, B = A[rank * per:(rank + 1) * per].contiguous(), B[rank * per:(rank + 1) * per].contiguous()
    C = torch.empty(per, n, n, device=dev)
    _barrier(world)
    ms = _max_over_ranks(_time_events(lambda: zc.matmul(A, B, a_depth=1, b_depth=1, out=C), 10), world, dev)
    t = bsz * 2 * n ** 3 / ms / 1e9
    out["config3_vmap_batched_f32_256x512"] = {"tflops": t, "ms": ms, "tflops_per_gpu": t / world,
                                               "frac_of_3xtf32_ceiling_per_gpu": t / world / (tf32 / 3),
                                               "parallelism": "batch axis over %d GPUs, %d matrices each" % (world, per)}
    del A, B, C
    n = 8192
    gr, gc = F64_GRIDS.get(world, (1, world))
    i, j = rank // gc, rank % gc
    rows, cols = n // gr, n // gc
    A = zc.rng_normal(0x5EED0008, n * n, dtype=torch.float64, device=dev).view(n, n)[i * rows:(i + 1) * rows].contiguous()
    B = zc.rng_normal(0x5EED0009, n * n, dtype=torch.float64, device=dev).view(n, n)[:, j * cols:(j + 1) * cols].contiguous()
    C = torch.empty(rows, cols, dtype=torch.float64, device=dev)
    torch.cuda.empty_cache()
    _barrier(world)
    ms = _max_over_ranks(_time_events(lambda: zc.matmul(A, B, out=C), 3, warm=1), world, dev)
    t = 2 * n ** 3 / ms / 1e9
    out["config5_f64_gemm_8192"] = {"tflops": t, "ms": ms, "tflops_per_gpu": t / world,
                                    "frac_of_fp64_nominal_per_gpu": t / world / fp64, "fp64_peak_tflops": fp64,
                                    "fp64_peak_source": "nominal B200",
                                    "parallelism": "2-D output tiles %dx%d" % (gr, gc)}
    del A, B, C
    torch.cuda.empty_cache()
    return out


def chain_sharded_config(rank, world, steps, dev):
    """The jit chain sumAll(tanh(x*x)*a + b) on ONE 2^26-element input
    range-sharded over the N GPUs: rank r reduces elements
    [r 2^26 / N, (r+1) 2^26 / N) with the fused kernel, then one
    1-element NCCL all-reduce sums the N partials (zpu's single reduction,
    ops.sumAll, done as partial sums plus one exchange).  At 8 GPUs a shard
    is 32 MiB and would stay in the 126 MB L2 between steps, so L2 is
    flushed (a 256 MiB write) before every step, outside the timed span;
    each step's span (kernel + all-reduce) is timed with CUDA events and the
    spans summed, max over ranks.  The all-reduce alone is timed the same
    way for its share."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import zpu_b200 as zc
    n = N_ELEM // world
    x = zc.rng_normal(SEED_X, N_ELEM, device=dev)[rank * n:(rank + 1) * n].contiguous()
    torch.cuda.empty_cache()
    steps_def = [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0), ("mul", [11, 2], 12, -2, 0),
                 ("add", [12, 3], 13, -2, 0), ("sum", [13], 14, -2, 0)]
    plan = zc.Plan([(1, zc.F32, (n,))], [(2, np.float32(A)), (3, np.float32(B))], steps_def, [14])
    part = torch.empty((), dtype=torch.float32, device=dev)
    flush = torch.empty(1 << 26, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        plan.run([x], [part])
        if world > 1:
            dist.all_reduce(part)

    def timed(fn, k):
        total = 0.0
        for _ in range(k):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        return total / k

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    ms = _max_over_ranks(timed(step, steps), world, dev)
    result = float(part.item())
    ar_ms = _max_over_ranks(timed(lambda: dist.all_reduce(part), steps), world, dev) if world > 1 else 0.0
    del flush
    torch.cuda.empty_cache()
    return {"metric": "fused-elementwise HBM GB/s, one 2^26 input range-sharded (whole job)",
            "gbs": BYTES_PER_STEP / ms / 1e6, "ms_per_step": ms, "n_gpus": world,
            "elements_per_gpu": n, "allreduce_ms": ar_ms, "allreduce_share": ar_ms / ms if world > 1 else 0.0,
            "sum": result, "l2": "flushed before every step (a shard of %d MiB%s)" % (
                n * 4 >> 20, " fits in L2" if n * 4 < 126 * 10 ** 6 else ""),
            "scaling": "strong (one input, fixed size)"}


MLP_DIMS = (784, 4096, 4096, 10)
MLP_BATCH = 8192
# GEMM flops of one step: forward 2*B*(784*4096 + 4096^2 + 4096*10), backward
# the weight gradients (the same again) plus the activation gradients of
# layers 3 and 2, 2*B*(4096*10 + 4096^2)
MLP_FLOPS = 2 * MLP_BATCH * (784 * 4096 + 4096 * 4096 + 4096 * 10) * 2 + 2 * MLP_BATCH * (4096 * 10 + 4096 * 4096)
MLP_PARAMS = 784 * 4096 + 4096 + 4096 * 4096 + 4096 + 4096 * 10 + 10


PARITY_DIMS, PARITY_BATCH, PARITY_STEPS = (64, 96, 80, 10), 512, 3


def mlp_parity(rank, world, dev):
    """The data-parallel step's parity, outside the timed region: every rank
    trains the 64->96->80->10 net for 3 steps on its 1/N of a 512-row batch
    from the same initial parameters, once with dW2 exchanged over peer
    memory by its GEMM and once with every gradient through NCCL's
    reduce-scatter.  The ranks' parameters must be bit-identical (an
    all-reduce of their bits, max against min) and rank 0's must match a
    one-GPU full-batch run (value_and_grad + Adam on rank 0's GPU) within
    1e-5 relative Frobenius per parameter, the loss within 1e-5 relative."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from zpu_b200 import mlp as zm
    from oracle import zpu_oracle as zo
    dims, B, steps = PARITY_DIMS, PARITY_BATCH, PARITY_STEPS
    X = zo.uniform_range(0x5EED0800, B * dims[0], 0.0, 1.0).reshape(B, dims[0])
    y = zo.randint(0x5EED0801, B, 0, dims[3])
    init = zo.mlp_init(dims)
    per = B // world
    xs = torch.from_numpy(np.ascontiguousarray(X[rank * per:(rank + 1) * per])).to(dev)
    ys = torch.from_numpy(np.ascontiguousarray(y[rank * per:(rank + 1) * per])).to(dev)
    want = want_loss = split = split_loss = None
    if rank == 0:
        xd, yd = torch.from_numpy(X).to(dev), torch.from_numpy(y).to(dev)
        m1 = zm.MLP(*dims, max_batch=B)
        m1.set_params(init)
        for _ in range(steps):
            m1.value_and_grad(xd, yd)
            m1.adam_step()
        want, want_loss = m1.params(), m1.loss()
        # the same N-way split of every sum on this one GPU: value_and_grad
        # on each rank's rows, gradients and losses added in rank order in
        # f32, one Adam step
        m2 = zm.MLP(*dims, max_batch=B)
        m2.set_params(init)
        for _ in range(steps):
            gsum = lsum = None
            for r in range(world):
                m2.value_and_grad(xd[r * per:(r + 1) * per].contiguous(), yd[r * per:(r + 1) * per].contiguous(),
                                  global_batch=B)
                g, l = m2.grads(), np.float32(m2.loss())
                gsum = g if gsum is None else [a + b for a, b in zip(gsum, g)]
                lsum = l if lsum is None else np.float32(lsum + l)
            m2._write(zm.GRAD, gsum)
            m2.adam_step()
        split, split_loss = m2.params(), float(lsum)
        m1.close()
        m2.close()
    out = {"net": "%d->%d->%d->%d" % dims, "global_batch": B, "adam_steps": steps,
           "tolerance": "ranks bit-identical; rel. Frobenius <= 1e-5 per parameter and loss vs one GPU",
           "split_emulation": "one GPU, value_and_grad on each rank's rows, sums in rank order (NCCL's ring "
                              "order differs from rank order beyond 2 ranks)"}
    saved = os.environ.get("ZPUCUDA_MLP_PEER_EXCHANGE")
    try:
        for mode in ("1", "0"):
            os.environ["ZPUCUDA_MLP_PEER_EXCHANGE"] = mode
            m = zm.MLP(*dims, max_batch=per)
            m.set_params(init)
            for _ in range(steps):
                m.train_step(xs, ys, global_batch=B)
            got, loss, ex = m.params(), m.loss(), m.exchange_mode()
            m.close()
            bits = torch.from_numpy(np.concatenate([g.ravel() for g in got]).view(np.int32)).to(dev)
            hi, lo = bits.clone(), bits.clone()
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            entry = {"exchange": "peer memory (dW2 stored by its GEMM)" if ex == 1 else "NCCL reduce-scatter",
                     "ranks_bit_identical": bool(torch.equal(hi, lo))}
            if rank == 0:
                rel = max(float(np.linalg.norm(g.astype(np.float64) - w) / np.linalg.norm(w.astype(np.float64)))
                          for g, w in zip(got, want))
                lrel = abs(loss - want_loss) / abs(want_loss)
                same = all(np.array_equal(g, w) for g, w in zip(got, split)) and loss == split_loss
                srel = max(float(np.linalg.norm(g.astype(np.float64) - w) / np.linalg.norm(w.astype(np.float64)))
                           for g, w in zip(got, split))
                entry.update({"max_rel_fro_vs_1gpu": rel, "loss": loss, "loss_1gpu": want_loss,
                              "loss_rel_diff": lrel,
                              "bit_identical_to_1gpu_split_emulation": same,
                              "max_rel_fro_vs_1gpu_split_emulation": srel,
                              "within": entry["ranks_bit_identical"] and rel <= 1e-5 and lrel <= 1e-5})
            out["peer_exchange" if mode == "1" else "nccl"] = entry
    finally:
        if saved is None:
            os.environ.pop("ZPUCUDA_MLP_PEER_EXCHANGE", None)
        else:
            os.environ["ZPUCUDA_MLP_PEER_EXCHANGE"] = saved
    return out


def mlp_drift(dev, adam_steps, loss_at_n):
    """How far the loss after `adam_steps` Adam steps moves when only the
    summation order changes: the full 784->4096->4096->10 step on one GPU over
    the whole batch, with the rows in order and with the rows permuted (the
    same mean loss and gradients in exact arithmetic), against the loss the
    N-GPU run reached after as many steps."""
    import torch
    import zpu_b200 as zc
    from zpu_b200 import mlp as zm
    xs = zc.rng_uniform(0x5EED0006, MLP_BATCH * 784, 0.0, 1.0, device=dev).view(MLP_BATCH, 784)
    ys = zc.rng_randint(0x5EED0007, MLP_BATCH, 0, 10, device=dev)
    perm = torch.randperm(MLP_BATCH, generator=torch.Generator().manual_seed(1234)).to(dev)
    losses = {}
    for name, (x, y) in (("rows_in_order", (xs, ys)), ("rows_permuted", (xs[perm].contiguous(), ys[perm].contiguous()))):
        m = zm.MLP(*MLP_DIMS, max_batch=MLP_BATCH)
        m.init_xavier()
        for _ in range(adam_steps):
            m.value_and_grad(x, y)
            m.adam_step()
        losses[name] = m.loss()
        m.close()
    a, b = losses["rows_in_order"], losses["rows_permuted"]
    del xs, ys
    torch.cuda.empty_cache()
    return {"adam_steps": adam_steps, "loss_1gpu_rows_in_order": a, "loss_1gpu_rows_permuted": b,
            "rel_diff_permuted_vs_in_order": abs(a - b) / abs(a), "loss_at_n_gpus": loss_at_n,
            "rel_diff_n_gpus_vs_1gpu": abs(loss_at_n - a) / abs(a)}


def mlp_config(rank, world, steps, warmup, dev):
    """The data-parallel MLP train step (784->4096->4096->10, tanh, softmax
    cross-entropy, global batch 8192, Adam lr 1e-3): each rank takes 8192/N
    rows of X ~ U[0,1] (seed 0x5EED0006) and labels randint(0,10) (seed
    0x5EED0007), Xavier-uniform init (seeds 0x5EED0010 + l), gradients summed
    over NCCL in two buckets overlapping the backward pass.  Device-timed
    steps (max over ranks) and an end-to-end run with X and labels copied
    from pinned host memory and the loss copied back every step."""
    import torch
    import zpu_b200 as zc
    from zpu_b200 import mlp as zm
    tf32, _, src = _peak_tflops()
    bl = MLP_BATCH // world
    xs = zc.rng_uniform(0x5EED0006, MLP_BATCH * 784, 0.0, 1.0, device=dev).view(MLP_BATCH, 784)
    ys = zc.rng_randint(0x5EED0007, MLP_BATCH, 0, 10, device=dev)
    x = xs[rank * bl:(rank + 1) * bl].contiguous()
    y = ys[rank * bl:(rank + 1) * bl].contiguous()
    del xs, ys
    if world > 1:
        zm.init_process_group_nccl(rank, world)
    m = zm.MLP(*MLP_DIMS, max_batch=bl)
    m.init_xavier()
    stream = torch.cuda.current_stream()
    for _ in range(max(3, warmup)):
        m.train_step(x, y, global_batch=MLP_BATCH)
    loss0 = m.loss()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    l0 = zc.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        m.train_step(x, y, global_batch=MLP_BATCH)
    m.join(stream)  # the last step's gather of W2 .. b3 inside the timed span
    e1.record(stream)
    torch.cuda.synchronize()
    launches = zc.launch_count() - l0
    ms = e0.elapsed_time(e1) / steps
    # end to end: every step copies its X / labels from pinned host memory
    # into HBM and its loss back to the host.  The copies run on a side stream
    # into two alternating device buffers, so step i+1's input crosses PCIe
    # while step i computes.
    xh, yh = x.cpu().pin_memory(), y.cpu().pin_memory()
    lh = torch.empty(1, dtype=torch.float32).pin_memory()
    xs_, ys_ = [x, torch.empty_like(x)], [y, torch.empty_like(y)]
    copy_stream = torch.cuda.Stream(device=dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    used = [torch.cuda.Event(), torch.cuda.Event()]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    copy_stream.wait_event(e2)

    def issue_copy(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(used[b])
            xs_[b].copy_(xh, non_blocking=True)
            ys_[b].copy_(yh, non_blocking=True)
            copied[b].record(copy_stream)

    issue_copy(0)
    for i in range(steps):
        if i + 1 < steps:
            issue_copy(i + 1)
        b = i % 2
        stream.wait_event(copied[b])
        m.train_step(xs_[b], ys_[b], global_batch=MLP_BATCH)
        used[b].record(stream)
        m.loss_to(lh.data_ptr())
    m.join(stream)
    e3.record(stream)
    torch.cuda.synchronize()
    e_ms = e2.elapsed_time(e3) / steps
    loss1 = float(lh[0])
    adam_steps = m.steps()
    # one more step with the phase trace on (outside every timed span): where
    # the step's time goes on this rank, in ms from the step's start
    m.trace(True)
    m.train_step(x, y, global_batch=MLP_BATCH)
    trace = m.trace_read()
    m.trace(False)
    names = ["start", "forward_gemms", "loss", "layer3_bwd_db2", "dW2_gemm", "g1_gemm", "db1_dW1_gemm",
             "main_stream_end", "bucket_W2_summed", "bucket_W2_adam", "bucket_W1_summed",
             "bucket_W1_adam_gather", "bucket_W2_gather"]
    trace = {k: round(v, 4) for k, v in zip(names, trace)}
    if world > 1:
        t = torch.tensor([ms, e_ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e_ms = float(t[0]), float(t[1])
    m.close()
    del x, y
    torch.cuda.empty_cache()
    parity = mlp_parity(rank, world, dev) if world > 1 else None
    drift = mlp_drift(dev, adam_steps, loss1) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
        zm.nccl_destroy()
    tflops = MLP_FLOPS / (ms / 1e3) / 1e12
    return {"metric": "MLP train steps/s (global batch 8192)", "steps_per_s": 1e3 / ms, "ms_per_step": ms,
            "n_gpus": world, "batch_per_gpu": bl, "gemm_tflops_whole_job": tflops,
            "gemm_tflops_per_gpu": tflops / world, "frac_of_3xtf32_ceiling_per_gpu": tflops / world / (tf32 / 3),
            "flops_per_step": MLP_FLOPS, "params": MLP_PARAMS, "allreduce_bytes_per_step": MLP_PARAMS * 4,
            "kernel_launches_per_step": launches / steps, "loss_after_warmup": loss0, "loss_last": loss1,
            "e2e": {"steps_per_s": 1e3 / e_ms, "ms_per_step": e_ms, "h2d_bytes_per_step": bl * (784 * 4 + 8),
                    "d2h_bytes_per_step": 4},
            "scaling": "strong (global batch fixed)", "dtype": "f32 (3xTF32 GEMMs)",
            "parity": parity, "drift": drift, "phase_trace_rank0_ms": trace}


def run_ours(args):
    import torch
    import zpu_b200 as zc
    import numpy as np

    rank, local, world = dist_env()
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    zc.check(zc.lib().zpucuda_init(local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    x = zc.rng_normal(SEED_X + rank, N_ELEM, device=dev)
    steps_def = [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0), ("mul", [11, 2], 12, -2, 0),
                 ("add", [12, 3], 13, -2, 0), ("sum", [13], 14, -2, 0)]
    plan = zc.Plan([(1, zc.F32, (N_ELEM,))], [(2, np.float32(A)), (3, np.float32(B))], steps_def, [14])
    out = torch.empty((), dtype=torch.float32, device=dev)
    for _ in range(max(3, args.warmup)):
        plan.run([x], [out])
    torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    # keep the GPU loaded with the same kernel while the sampler comes up
    t0 = time.perf_counter()
    soak = 0
    while time.perf_counter() - t0 < 1.0:
        for _ in range(200):
            plan.run([x], [out])
        torch.cuda.synchronize()
        soak += 200
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = zc.launch_count()
    ev0.record(stream)
    for _ in range(args.steps):
        plan.run([x], [out])
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = zc.launch_count() - launches0
    barrier()
    ms = ev0.elapsed_time(ev1)
    # the timed region is short: keep sampling over another ~1 s of the same load
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 1.0:
        for _ in range(200):
            plan.run([x], [out])
        torch.cuda.synchronize()
    clk = clocks.stop()
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_max = float(t.item())
    per_step_s = ms_max / args.steps / 1e3
    value = world * BYTES_PER_STEP / per_step_s / 1e9

    # end to end through the C ABI with host buffers: H2D of x, the fused
    # kernel, D2H of the scalar, every step
    x_h = x.cpu().pin_memory()
    out_h = torch.empty((), dtype=torch.float32).pin_memory()
    for _ in range(2):
        plan.run_host([x_h], [out_h])
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(3, min(args.steps, 20))
    e0.record(stream)
    for _ in range(e_steps):
        plan.run_host([x_h], [out_h])
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e_ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_value = world * BYTES_PER_STEP / (e_ms / e_steps / 1e3) / 1e9

    peak, peak_kind = peaks()
    kernel_ms = ms / args.steps  # one fused kernel per step on this stream
    achieved = BYTES_PER_STEP / (kernel_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (rng.Rng(0x5EED0003 + rank).normal on the device; same stream as zpu's)",
        "config": {"workload": WORKLOAD, "n_elements_per_gpu": N_ELEM, "a": A, "b": B,
                   "l2": "inputs larger than L2 (256 MiB per step > 126 MB), no flush",
                   "parallelism": "replicas: each GPU runs the plan on its own 2^26 shard",
                   "kernel": "catalogue region tanh_sq_affine+sum (1 launch/step)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": ncu_traffic("tanh_sq_affine+sum 2^26 f32"),
                     "peak_source": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": N_ELEM * 4, "d2h_bytes_per_step": 4,
                "path": "zpucuda_plan_run_host (pinned host x -> HBM, fused kernel, scalar -> host)"},
        "gpu_launches": launches,
        "clocks": clk,
        "warmup_soak_steps": soak,
    }
    line["other_configs"] = gemm_configs(rank, world, dev)
    line["other_configs"]["config2_chain_range_sharded"] = chain_sharded_config(rank, world, min(args.steps, 20), dev)
    line["other_configs"]["config4_mlp_train_step"] = mlp_config(rank, world, min(args.steps, 20), args.warmup, dev)
    if rank == 0 and world == 1:
        gbs, cores, sample, per = cpu_chain_baseline()
        line["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                                "sample": sample + " (oracle restatement of zpu's jit.Plan.runAll)"}
        # the checker on the timed input: the device's sum against zpu's own
        # f32 summation order and the f64 sum of the same element values
        from oracle import zpu_oracle as zo
        s32, s64, t = zo.jit_chain_tanh_sq_affine_sum(x.cpu().numpy(), A, B, want_vector=True)
        got = float(out.cpu())
        scale = zo.abssum_f64(t)
        line["cpu_baseline"]["parity"] = {
            "device_sum": got, "zpu_f32_order_sum": float(s32), "f64_sum": s64,
            "abs_diff_vs_f64": abs(got - s64), "abs_diff_vs_zpu_f32_order": abs(got - float(s32)),
            "tolerance": "|device - f64| <= 1e-6 * sum|t_i|", "bound": 1e-6 * scale,
            "within": abs(got - s64) <= 1e-6 * scale}
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def _only_gemm(kind, steps, warmup):
    import torch
    import zpu_b200 as zc
    if kind == "f32_1024":
        n, bsz = 1024, 0
        A = zc.rng_uniform(0x5EED0001, n * n, -1.0, 1.0).view(n, n)
        B = zc.rng_uniform(0x5EED0002, n * n, -1.0, 1.0).view(n, n)
    elif kind in ("f32_4096", "f32_8192"):
        n, bsz = int(kind[4:]), 0
        A = zc.rng_uniform(0x5EED0001, n * n, -1.0, 1.0).view(n, n)
        B = zc.rng_uniform(0x5EED0002, n * n, -1.0, 1.0).view(n, n)
    elif kind == "f32_batched":
        n, bsz = 512, 256
        s = 1.0 / (512.0 ** 0.5)
        A = (zc.rng_normal(0x5EED0004, bsz * n * n) * s).view(bsz, n, n)
        B = (zc.rng_normal(0x5EED0005, bsz * n * n) * s).view(bsz, n, n)
    else:
        n, bsz = 4096, 0
        A = zc.rng_normal(0x5EED0008, n * n, dtype=torch.float64).view(n, n)
        B = zc.rng_normal(0x5EED0009, n * n, dtype=torch.float64).view(n, n)
    C = torch.empty_like(A)
    d = 1 if bsz else 0
    ms = _time_events(lambda: zc.matmul(A, B, a_depth=d, b_depth=d, out=C), steps, warm=warmup)
    return {"ms": ms, "tflops": max(1, bsz) * 2 * n ** 3 / ms / 1e9, "n": n, "batch": max(1, bsz)}


def _only_kernel(kind, steps, warmup):
    """One of the library's other kernels alone, on inputs larger than L2, for
    its ncu summary: returns its CUDA-event time per call and the algorithmic
    bytes per call (reads + writes of the kernel's own data)."""
    import ctypes as C
    import numpy as np
    import torch
    import zpu_b200 as zc
    F = zc.F32
    if kind in ("region_bytecode", "sum_sq_bulk"):
        n = 1 << 26
        x = zc.rng_normal(SEED_X, n)
        if kind == "sum_sq_bulk":  # catalogue "sq+sum": the bulk-copy pipeline
            plan = zc.Plan([(1, F, (n,))], [], [("mul", [1, 1], 10, -2, 0), ("sum", [10], 11, -2, 0)], [11])
            out = [torch.empty((), device="cuda")]
            nbytes = n * 4 + 4
        else:  # outside the catalogue: the one-pass bytecode kernel
            plan = zc.Plan([(1, F, (n,))], [], [("sin", [1], 10, -2, 0), ("mul", [1, 1], 11, -2, 0),
                                                 ("add", [10, 11], 12, -2, 0)], [12])
            out = [torch.empty(n, device="cuda")]
            nbytes = n * 8
        fn = lambda: plan.run([x], out)
    elif kind == "cumsum":
        r, c = 8192, 4096
        x = zc.rng_normal(SEED_X, r * c).view(r, c)
        plan = zc.Plan([(1, F, (r, c))], [], [("cumsum", [1], 10, 0, 0)], [10])
        out = [torch.empty(r, c, device="cuda")]
        fn = lambda: plan.run([x], out)
        nbytes = r * c * 8
    elif kind in ("take", "scatter_add"):
        r, c, k = 16384, 1024, 16384
        x = zc.rng_normal(SEED_X, r * c).view(r, c)
        idx = zc.rng_randint(SEED_X + 1, k, 0, r)
        if kind == "take":
            plan = zc.Plan([(1, F, (r, c)), (2, zc.DT_I64, (k,))], [], [("take", [1, 2], 10, 0, 0)], [10])
            out = [torch.empty(k, c, device="cuda")]
            fn = lambda: plan.run([x, idx], out)
            nbytes = k * c * 8 + k * 8
        else:
            upd = zc.rng_normal(SEED_X + 2, k * c).view(k, c)
            plan = zc.Plan([(1, F, (r, c)), (2, zc.DT_I64, (k,)), (3, F, (k, c))], [],
                           [("scatter_add", [1, 2, 3], 10, 0, 0)], [10])
            out = [torch.empty(r, c, device="cuda")]
            fn = lambda: plan.run([x, idx, upd], out)
            nbytes = r * c * 8 + k * c * 4 + k * 8
    elif kind == "rng_normal":
        n = 1 << 26
        buf = torch.empty(n, device="cuda")
        fn = lambda: zc.rng_normal(SEED_X, n, out=buf)
        nbytes = n * 4
    elif kind == "peer_reduce":  # the owner-side sum of the dW2 exchange, 8 slots
        world, n = 8, 1 << 23
        inbox = zc.rng_normal(SEED_X, world * n)
        flags = torch.ones(world, dtype=torch.int64, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        outv = torch.empty(n, device="cuda")
        L = zc.lib()
        fn = lambda: zc.check(L.zpucuda_debug_peer_reduce(inbox.data_ptr(), world, n, outv.data_ptr(),
                                                          flags.data_ptr(), 1, 1 << 20, err.data_ptr(), zc.stream_of()))
        nbytes = world * n * 4 + n * 4
    elif kind == "gather_copy":  # a flipped (negative-stride) view made contiguous
        r, c = 8192, 4096
        x = zc.rng_normal(SEED_X, r * c).view(r, c)
        d = zc.tensor_desc(x)
        d.data = x.data_ptr() + (r - 1) * c * 4
        d.strides[0] = -c
        out = torch.empty(r, c, device="cuda")
        fn = lambda: zc.tensor_copy(d, out)
        nbytes = r * c * 8
    elif kind == "gemm_fma_fallback":  # a row pitch the tensor maps cannot take
        n, ld = 2048, 2049
        a = zc.rng_uniform(SEED_X, n * ld, -1.0, 1.0).view(n, ld)[:, :n]
        b = zc.rng_uniform(SEED_X + 1, n * ld, -1.0, 1.0).view(n, ld)[:, :n]
        o = torch.empty(n, n, device="cuda")
        fn = lambda: zc.matmul(a, b, out=o)
        nbytes = None
        flops = 2 * n ** 3
    elif kind == "gemm_smallk":  # a short contraction (k = 16, like the MLP's g2): zpu's chain, CUDA cores
        m, n, k = 8192, 4096, 16
        a = zc.rng_uniform(SEED_X, m * k, -1.0, 1.0).view(m, k)
        b = zc.rng_uniform(SEED_X + 1, n * k, -1.0, 1.0).view(n, k)
        o = torch.empty(m, n, device="cuda")
        fn = lambda: zc.gemm(a, b, out=o, trans_b=True)
        nbytes = m * n * 4 + (m + n) * k * 4
    elif kind in ("transpose_f16", "transpose_u8"):  # toContiguous of a transposed view, 256 MiB (> L2)
        dt = torch.float16 if kind == "transpose_f16" else torch.uint8
        r, c = (16384, 8192) if dt == torch.float16 else (16384, 16384)
        x = (zc.rng_uniform(SEED_X, r * c, 0.0, 100.0).view(r, c)).to(dt)
        out = torch.empty(c, r, dtype=dt, device="cuda")
        fn = lambda: zc.tensor_copy(x.transpose(0, 1), out)
        nbytes = 2 * r * c * x.element_size()
    elif kind == "gemm_convert":  # f16 @ f32: zpu's gemmF64 loop
        n = 1024
        a = zc.rng_uniform(SEED_X, n * n, -1.0, 1.0).view(n, n).half()
        b = zc.rng_uniform(SEED_X + 1, n * n, -1.0, 1.0).view(n, n)
        o = torch.empty(n, n, device="cuda")
        fn = lambda: zc.matmul(a, b, out=o)
        nbytes = None
        flops = 2 * n ** 3
    else:
        raise ValueError(kind)
    ms = _time_events(fn, steps, warm=warmup)
    res = {"ms": ms}
    if nbytes:
        res.update({"gbs": nbytes / ms / 1e6, "algorithmic_bytes": nbytes})
    else:
        res.update({"tflops": flops / ms / 1e9})
    return res


KERNEL_CASES = ("region_bytecode", "sum_sq_bulk", "cumsum", "take", "scatter_add", "rng_normal", "peer_reduce",
                "gather_copy", "gemm_fma_fallback", "gemm_convert", "gemm_smallk", "transpose_f16", "transpose_u8")

ONLY_CASES = {
    "chain": None, "mlp": None, "chain_sharded": None,
    "gemm_f32_1024": "f32_1024", "gemm_f32_4096": "f32_4096", "gemm_f32_8192": "f32_8192",
    "gemm_f32_batched": "f32_batched",
    "gemm_f64_4096": "f64_4096",
}
ONLY_CASES.update({k: None for k in KERNEL_CASES})


def run_only(args):
    """One workload alone, for ncu captures: the same kernels and inputs as
    the full run, none of the others."""
    import torch
    import numpy as np
    import zpu_b200 as zc
    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    zc.check(zc.lib().zpucuda_init(local))
    if args.only in ("mlp", "chain_sharded"):  # the cases that run under torchrun (data parallel)
        if world > 1:
            import datetime
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                                 device_id=torch.device("cuda", local))
        if args.only == "mlp":
            out = mlp_config(rank, world, args.steps, args.warmup, torch.device("cuda", local))
        else:
            out = chain_sharded_config(rank, world, args.steps, torch.device("cuda", local))
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        if rank != 0:
            return 0
    elif args.only == "chain":
        x = zc.rng_normal(SEED_X, N_ELEM)
        steps_def = [("mul", [1, 1], 10, -2, 0), ("tanh", [10], 11, -2, 0), ("mul", [11, 2], 12, -2, 0),
                     ("add", [12, 3], 13, -2, 0), ("sum", [13], 14, -2, 0)]
        plan = zc.Plan([(1, zc.F32, (N_ELEM,))], [(2, np.float32(A)), (3, np.float32(B))], steps_def, [14])
        y = torch.empty((), dtype=torch.float32, device="cuda")
        ms = _time_events(lambda: plan.run([x], [y]), args.steps, warm=args.warmup)
        out = {"ms": ms, "gbs": BYTES_PER_STEP / ms / 1e6}
    elif args.only in KERNEL_CASES:
        out = _only_kernel(args.only, args.steps, args.warmup)
    else:
        out = _only_gemm(ONLY_CASES[args.only], args.steps, args.warmup)
    print(json.dumps({"only": args.only, **out}), flush=True)
    return 0


def main():
    args = parse()
    if args.only:
        return run_only(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
