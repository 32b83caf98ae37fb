"""Failure detection without faulting a GPU.

GPU: a test hook (NVFP4_FAULT_INJECT=1) makes CTA 0 of the GEMM withhold one
TMA load, so the full barrier it expects never completes.  Every pipeline
wait in the kernels is bounded (1 s, %globaltimer); the waits run out, the
kernel records a status code, drains its tensor-core work, frees TMEM and
exits.  The host reads the status, and the next call on the same context is
correct.

CPU (gloo): a rank that disappears before a collective makes the surviving
rank's barrier fail within the process-group timeout instead of hanging
(the pattern bench.py uses for its multi-GPU timing)."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvfp4_b200 import _lib, inputs, ops
from tests.refcheck import assert_match, oracle_ref


@pytest.mark.gpu
def test_gemm_wait_timeout_reports_status_and_context_survives(monkeypatch):
    monkeypatch.setenv("NVFP4_SPLITS", "1")
    monkeypatch.setenv("NVFP4_PAIR", "0")
    data = inputs.baseline_input("gemm", 512, 1024, 1, 4, n=512)
    assert _lib.device_status(True) == 0
    monkeypatch.setenv("NVFP4_FAULT_INJECT", "1")
    t0 = time.time()
    ops._CACHE.clear()
    ops.gemm(data)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    status = _lib.device_status(True)
    assert status in (1, 2, 3, 4), status  # a pipeline wait ran out
    assert elapsed < 15, elapsed
    monkeypatch.delenv("NVFP4_FAULT_INJECT")
    ops._CACHE.clear()
    out = ops.gemm(data)
    torch.cuda.synchronize()
    assert _lib.device_status(True) == 0
    assert_match(out, oracle_ref("gemm", data), "gemm after a timed-out launch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the next collective
    t0 = time.time()
    try:
        dist.barrier()
        q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((type(e).__name__, time.time() - t0))


def test_lost_rank_fails_the_barrier_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, waited = q.get(timeout=90)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert kind != "no error"
    assert waited < 60
