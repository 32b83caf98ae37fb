"""The N>1 host path on CPU: world_size-2 gloo ranks each take their shard of
one problem (nvfp4_b200.shard), compute it with the CPU oracle (no GPU here),
all_gather the C shards and compare with the single-rank result.  Also checks
the shard views keep the strides the drop-in kernels require."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvfp4_b200 import inputs, shard
from tests.refcheck import oracle_ref

CASES = [("gemv", 512, 1, 256, 2), ("gemm", 128, 512, 256, 1), ("dual", 128, 256, 256, 1)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, problem, m, n, k, l, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        data = inputs.reference_input(problem, m, k, l, 1111, n=None if problem == "gemv" else n, device="cpu")
        part = shard.shard_tuple(problem, data, world, rank)
        out = torch.from_numpy(oracle_ref(problem, part).astype(np.float32))
        sizes = [None] * world
        dist.all_gather_object(sizes, tuple(out.shape))
        gathered = [torch.empty(s) for s in sizes]
        dist.all_gather(gathered, out.contiguous())
        if rank == 0:
            axis = 0 if problem == "gemv" else 1
            full = torch.cat(gathered, dim=axis).numpy()
            q.put(("ok", full))
    except Exception as e:  # report to the parent instead of hanging it
        q.put(("err", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("problem,m,n,k,l", CASES)
def test_two_rank_shards_reassemble_single_rank_result(problem, m, n, k, l):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, problem, m, n, k, l, q)) for r in range(2)]
    for p in procs:
        p.start()
    status, payload = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert status == "ok", payload
    data = inputs.reference_input(problem, m, k, l, 1111, n=None if problem == "gemv" else n, device="cpu")
    np.testing.assert_array_equal(payload.astype(np.float16), oracle_ref(problem, data))


@pytest.mark.parametrize("problem,m,n,k,l", CASES)
@pytest.mark.parametrize("world", [2, 4])
def test_shard_views_keep_kernel_strides(problem, m, n, k, l, world):
    if problem == "gemv" and m // 128 < world or problem != "gemv" and n // 128 < world:
        pytest.skip("fewer 128-blocks than ranks")
    data = inputs.reference_input(problem, m, k, l, 3, n=None if problem == "gemv" else n, device="cpu")
    covered = 0
    for r in range(world):
        part = shard.shard_tuple(problem, data, world, r)
        a, c = part[0], part[-1]
        assert a.stride(1) == 1 and a.stride(0) == a.shape[1]
        assert c.stride(1) == 1 or problem == "gemv"
        if problem == "gemv":
            sfa_p = part[4]
            assert sfa_p.stride()[:5] == (16, 4, (k // 64) * 512, 1, 512)
            covered += a.shape[0]
        else:
            b, sfb_p = part[1], part[5] if problem == "gemm" else part[7]
            assert b.stride(1) == 1 and b.stride(0) == b.shape[1]
            assert sfb_p.stride()[:5] == (16, 4, (k // 64) * 512, 1, 512)
            assert sfb_p.shape[2] * 128 == b.shape[0]
            covered += b.shape[0]
    assert covered == (m if problem == "gemv" else n)


def test_shard_bounds_balanced():
    b = [shard.shard_bounds(7168, 8, r) for r in range(8)]
    assert b[0] == (0, 896) and b[-1] == (7168 - 896, 7168)
    assert all(hi - lo in (0, 896) for lo, hi in b)


@pytest.mark.parametrize("problem,m,n,k,l", CASES)
def test_dense_shards_match_views_and_are_dense(problem, m, n, k, l):
    """dense_shard_tuple: equal values to the shard views, each tensor one
    dense run in the reference's storage order (so a pinned host buffer of
    the same strides copies in one DMA)."""
    world = 2
    if problem == "gemv" and m // 128 < world or problem != "gemv" and n // 128 < world:
        pytest.skip("fewer 128-blocks than ranks")
    data = inputs.reference_input(problem, m, k, l, 3, n=None if problem == "gemv" else n, device="cpu")
    for r in range(world):
        views = shard.shard_tuple(problem, data, world, r)
        dense = shard.dense_shard_tuple(problem, data, world, r)
        for v, d in zip(views, dense):
            assert v.shape == d.shape
            assert torch.equal(v.view(torch.uint8) if v.element_size() == 1 else v,
                               d.view(torch.uint8) if d.element_size() == 1 else d)
            # dense: the strides are a permutation of a contiguous layout
            assert d.is_contiguous() or d.permute(*sorted(range(d.dim()), key=lambda i: -d.stride(i))).is_contiguous()
        a = dense[0]
        assert a.stride() == (a.shape[1], 1, a.shape[0] * a.shape[1])
