"""Host side of the data-parallel MLP step, as world_size-2 gloo ranks on CPU.

What the GPU ranks do per step is: the loss of the local rows scaled by
1/global_batch, its gradients, an allreduce (sum) of the gradient array and
the loss, then the same Adam update everywhere.  Here each rank runs the
oracle's valueAndGrad on its half of the batch, the gloo allreduce sums them,
and the result must equal the full-batch gradient; the NCCL id exchange runs
over the same group.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from oracle import zpu_oracle as zo
        from zpu_b200.mlp import exchange_id

        # the communicator id: made on rank 0, the same 128 bytes everywhere
        uid = exchange_id(rank, lambda: bytes(range(128)), lambda box: dist.broadcast_object_list(box, src=0))
        assert uid == bytes(range(128))
        if rank == 0:
            bad = None
            try:
                exchange_id(0, lambda: b"short", lambda box: None)
            except Exception as e:  # a malformed id is refused before NCCL sees it
                bad = type(e).__name__
            assert bad == "ZpuCudaError"

        dims, B = (32, 48, 40, 10), 64
        X = zo.uniform_range(0x5EED0700, B * dims[0], 0.0, 1.0).reshape(B, dims[0])
        labels = zo.randint(0x5EED0701, B, 0, dims[3])
        params = zo.mlp_init(dims)
        per = B // world
        sl = slice(rank * per, (rank + 1) * per)
        loss, grads = zo.mlp_loss_grad(np.ascontiguousarray(X[sl]), np.ascontiguousarray(labels[sl]), params)
        # the oracle averages over its own rows; the device kernel scales by
        # 1/global_batch instead: the same thing for equal shards
        flat = np.concatenate([g.ravel() for g in grads] + [np.array([loss], np.float32)]) * (per / B)
        t = torch.from_numpy(flat.astype(np.float32))
        dist.all_reduce(t)
        if rank == 0:
            full_loss, full = zo.mlp_loss_grad(X, labels, params)
            want = np.concatenate([g.ravel() for g in full] + [np.array([full_loss], np.float32)])
            got = t.numpy()
            err = np.linalg.norm(got - want) / np.linalg.norm(want)
            assert err <= 1e-5, err
            assert abs(got[-1] - full_loss) <= 1e-5 * abs(full_loss)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as e:  # report, never hang the parent
        q.put((rank, "%s: %s" % (type(e).__name__, e)))


def test_two_rank_gradient_sum_equals_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            r, msg = q.get(timeout=120)
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert results == {0: "ok", 1: "ok"}, results
