"""Data-parallel MLP step over NCCL on 2 GPUs, and the communicator's bounded
join on one.

Each rank is a child process bound to its own GPU; the 128-byte NCCL id
travels through a gloo process group.  Run once with dW2 exchanged over peer
memory by its GEMM and once with NCCL alone.  After two train steps on halves of
the batch (gradients summed over NCCL in the library's two buckets) every
rank's parameters must equal each other bit for bit, match a one-GPU
full-batch run within 1e-5 (the halves' partial sums re-associate), and
equal bit for bit a one-GPU run of the same split (each half's gradients
added in f32 in rank order before Adam).
"""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

DIMS, B, STEPS = (64, 96, 80, 10), 512, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


RANK_SCRIPT = textwrap.dedent("""
    import datetime, os, sys
    import numpy as np, torch, torch.distributed as dist
    sys.path.insert(0, {root!r})
    rank, world, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
    torch.cuda.set_device(rank)
    import zpu_b200 as zc
    from zpu_b200 import mlp as zm
    from oracle import zpu_oracle as zo
    zc.check(zc.lib().zpucuda_init(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    zm.init_process_group_nccl(rank, world, timeout_ms=60000)
    assert zm.nccl_world() == (rank, world)
    dims, B, steps = {dims!r}, {B}, {steps}
    X = zo.uniform_range(0x5EED0800, B * dims[0], 0.0, 1.0).reshape(B, dims[0])
    y = zo.randint(0x5EED0801, B, 0, dims[3])
    per = B // world
    xs = torch.from_numpy(np.ascontiguousarray(X[rank * per:(rank + 1) * per])).cuda()
    ys = torch.from_numpy(np.ascontiguousarray(y[rank * per:(rank + 1) * per])).cuda()
    m = zm.MLP(*dims, max_batch=per)
    m.set_params(zo.mlp_init(dims))
    for _ in range(steps):
        m.train_step(xs, ys, global_batch=B)
    loss = m.loss()
    np.savez(out, loss=np.float32(loss), mode=np.int32(m.exchange_mode()), *m.params())
    m.close()
    zm.nccl_destroy()
    dist.barrier()
    dist.destroy_process_group()
""")


@pytest.mark.parametrize("peer,last_ar", [("1", "0"), ("0", "0"), ("1", "1")])
def test_two_gpu_train_steps_match_one_gpu(tmp_path, peer, last_ar):
    """peer "1": dW2 goes from its GEMM's tile stores into the owner's inbox
    over NVLink (the exchange must be active); "0": every gradient through
    NCCL's reduce-scatter.  last_ar "1": the last bucket [W1, b1] as one
    allreduce with Adam on every rank instead of reduce-scatter + all-gather."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import zpu_b200 as zc
    from zpu_b200 import mlp as zm
    from oracle import zpu_oracle as zo
    script = tmp_path / "rank.py"
    script.write_text(RANK_SCRIPT.format(root=ROOT, dims=DIMS, B=B, steps=STEPS))
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), NCCL_NVLS_ENABLE="0",
               ZPUCUDA_MLP_PEER_EXCHANGE=peer, ZPUCUDA_MLP_LAST_BUCKET_ALLREDUCE=last_ar)
    procs = [subprocess.Popen([sys.executable, str(script), str(r), "2", str(tmp_path / ("r%d.npz" % r))], env=env)
             for r in range(2)]
    try:
        rcs = [p.wait(timeout=240) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert rcs == [0, 0]
    r0, r1 = np.load(tmp_path / "r0.npz"), np.load(tmp_path / "r1.npz")
    assert int(r0["mode"]) == int(r1["mode"]) == int(peer)
    # one GPU, the whole batch
    zc.check(zc.lib().zpucuda_init(0))
    X = zo.uniform_range(0x5EED0800, B * DIMS[0], 0.0, 1.0).reshape(B, DIMS[0])
    y = zo.randint(0x5EED0801, B, 0, DIMS[3])
    m = zm.MLP(*DIMS, max_batch=B)
    m.set_params(zo.mlp_init(DIMS))
    xd, yd = torch.from_numpy(X).cuda(), torch.from_numpy(y).cuda()
    for _ in range(STEPS):
        m.train_step(xd, yd)
    want = m.params()
    for i in range(6):
        a, b = r0["arr_%d" % i], r1["arr_%d" % i]
        assert np.array_equal(a, b), i
        assert np.linalg.norm(a - want[i]) <= 1e-5 * np.linalg.norm(want[i]), i
    assert abs(float(r0["loss"]) - m.loss()) <= 1e-5 * abs(m.loss())
    # exactly the arithmetic of the split: one GPU, value_and_grad on each
    # rank's half (loss averaged over the global batch), gradients and losses
    # added in f32 in rank order, then Adam -- bit for bit the 2-GPU result
    per = B // 2
    e = zm.MLP(*DIMS, max_batch=B)
    e.set_params(zo.mlp_init(DIMS))
    for _ in range(STEPS):
        gsum = lsum = None
        for r in range(2):
            e.value_and_grad(xd[r * per:(r + 1) * per].contiguous(), yd[r * per:(r + 1) * per].contiguous(),
                             global_batch=B)
            g, l = e.grads(), np.float32(e.loss())
            gsum = g if gsum is None else [a + b for a, b in zip(gsum, g)]
            lsum = l if lsum is None else np.float32(lsum + l)
        e._write(zm.GRAD, gsum)
        e.adam_step()
    split = e.params()
    for i in range(6):
        assert np.array_equal(r0["arr_%d" % i], split[i]), i
    assert np.float32(r0["loss"]) == lsum


JOIN_SCRIPT = textwrap.dedent("""
    import sys, time
    sys.path.insert(0, {root!r})
    import torch
    torch.cuda.set_device(0)
    import zpu_b200 as zc
    from zpu_b200 import mlp as zm
    zc.check(zc.lib().zpucuda_init(0))
    uid = zm.nccl_unique_id()
    t0 = time.time()
    try:
        zm.nccl_init(0, 2, uid, timeout_ms=2000)   # rank 1 never joins
        print("JOINED")
    except zc.ZpuCudaError as e:
        print("STATUS", e.status, round(time.time() - t0, 1))
    assert zm.nccl_world() == (0, 1)
""")


def test_nccl_join_times_out_when_a_rank_never_joins(tmp_path):
    """A rank that never joins: the host-side wait ends with Timeout (13)
    after the given limit and the half-made communicator is torn down; no
    kernel is in flight on the GPU."""
    script = tmp_path / "join.py"
    script.write_text(JOIN_SCRIPT.format(root=ROOT))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, str(script)], env=env, capture_output=True, text=True, timeout=180)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [l for l in r.stdout.splitlines() if l.startswith(("STATUS", "JOINED"))][-1]
    parts = line.split()
    assert parts[0] == "STATUS" and parts[1] == "13", line
    assert 1.5 <= float(parts[2]) <= 30, line
