"""bench.py's multi-GPU correctness check (gather_check) on CPU with gloo
ranks: the ranks' C slices — of unequal widths, so the all-gather pads — are
assembled and compared with rank 0's expected whole-problem result; a wrong element in
one rank's slice is caught."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvfp4_b200 import inputs, shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _pattern(shape):
    m, n, l = shape
    i = torch.arange(m).view(m, 1, 1) * 7 + torch.arange(n).view(1, n, 1) * 3 + torch.arange(l).view(1, 1, l)
    return (i % 997).to(torch.float16)


def _worker(rank, world, port, problem, m, n, k, corrupt, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        data = inputs.baseline_input(problem, m, k, 1, 5, n=None if problem == "gemv" else n, device="cpu")
        c = data[-1]
        shape = tuple(c.shape)
        sl = shard.output_slice(problem, shape, world, rank)
        mine = _pattern(shape)[sl].clone()  # this rank's shard result
        if corrupt and rank == world - 1:
            mine[0, 0, 0] += 1
        res = bench.gather_check(problem, shape, mine, lambda: _pattern(shape), world, rank, dist)
        if rank == 0:
            q.put(("ok", res))
    except Exception as e:
        q.put(("err", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("corrupt", [False, True])
@pytest.mark.parametrize("problem,m,n,k", [("gemv", 384, 1, 256), ("gemm", 128, 384, 256), ("dual", 128, 384, 256)])
def test_gather_check(problem, m, n, k, corrupt):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, problem, m, n, k, corrupt, q)) for r in range(2)]
    for p in procs:
        p.start()
    status, res = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
    assert status == "ok", res
    assert res["elements"] == m * n
    assert res["ok"] is (not corrupt)
    assert res["mismatches"] == (1 if corrupt else 0)
