"""Failure detection without faulting a GPU.

GPU: a test hook (NVFP4_FAULT_INJECT=1) makes CTA 0 of a tensor-core kernel
(GEMV, GEMM in each of its forms, dual GEMM) withhold one TMA load, so the
full barrier it expects never completes.  Every pipeline
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


def _timeout_then_recover(monkeypatch, problem, data, fn, env, check):
    """Injects a withheld load under `env`, expects a recorded timeout within
    a few seconds, clears the status (which also re-zeroes the library's
    workspaces), then expects correct results from the same context on two
    further calls without injection."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    assert _lib.device_status(True) == 0
    monkeypatch.setenv("NVFP4_FAULT_INJECT", "1")
    ops._CACHE.clear()
    t0 = time.time()
    fn(data)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    status = _lib.device_status(True)
    assert status in (1, 2, 3, 4, 5), status  # a pipeline wait ran out
    assert elapsed < 20, elapsed
    monkeypatch.delenv("NVFP4_FAULT_INJECT")
    ops._CACHE.clear()
    for _ in range(2):
        out = fn(data)
        torch.cuda.synchronize()
        assert _lib.device_status(True) == 0
        check(out)


@pytest.mark.gpu
@pytest.mark.parametrize("kernel,env,shape", [
    ("single", {"NVFP4_SPLITS": "1", "NVFP4_PAIR": "0"}, (512, 512, 2048)),
    ("pair", {"NVFP4_SPLITS": "1", "NVFP4_PAIR": "1"}, (512, 512, 2048)),
    ("split_k_cluster", {"NVFP4_SPLITS": "4", "NVFP4_PAIR": "0"}, (512, 512, 2048)),
    # 156 tiles of 128x256 on 148 SMs: the stream-K ranges cut tiles
    ("stream_k", {"NVFP4_SPLITS": "1", "NVFP4_PAIR": "0", "NVFP4_STREAMK": "2"}, (1664, 3072, 512)),
    ("pair_stream_k", {"NVFP4_SPLITS": "1", "NVFP4_PAIR": "1", "NVFP4_STREAMK": "2"}, (512, 512, 2048)),
])
def test_gemm_wait_timeout_reports_status_and_context_survives(monkeypatch, kernel, env, shape):
    """Every GEMM kernel form: the 1-CTA kernel, the 2-CTA pair kernel (the
    default for BASELINE config 2), K split across a thread-block cluster,
    and stream-K (whose flags and partial slots in the workspace a timed-out
    launch leaves behind: the status clear re-zeroes them)."""
    m, n, k = shape
    data = inputs.baseline_input("gemm", m, k, 1, 4, n=n)
    exp = oracle_ref("gemm", data)
    _timeout_then_recover(monkeypatch, "gemm", data, ops.gemm, env,
                          lambda out: assert_match(out, exp, f"gemm ({kernel}) after a timed-out launch"))


@pytest.mark.gpu
@pytest.mark.parametrize("kernel,env", [
    ("single_split", {"NVFP4_PAIR": "0"}),
    ("pair", {"NVFP4_PAIR": "1"}),
])
def test_dual_gemm_wait_timeout(monkeypatch, kernel, env):
    data = inputs.baseline_input("dual", 256, 2048, 1, 4, n=256)
    exp = oracle_ref("dual", data)
    _timeout_then_recover(monkeypatch, "dual", data, ops.dual_gemm, env,
                          lambda out: assert_match(out, exp, f"dual ({kernel}) after a timed-out launch"))


@pytest.mark.gpu
def test_gemv_tensor_core_wait_timeout(monkeypatch):
    """The tensor-core GEMV: CTA 0 withholds a load, so it never adds its
    partial sums for its row blocks and their arrival counters stay short;
    after the status clear (which re-zeroes the counters) the next calls are
    correct."""
    monkeypatch.delenv("NVFP4_GEMV_PATH", raising=False)
    data = inputs.baseline_input("gemv", 512, 16384, 2, 4)
    exp = oracle_ref("gemv", data)
    _timeout_then_recover(monkeypatch, "gemv", data, ops.gemv, {},
                          lambda out: assert_match(out, exp, "gemv after a timed-out launch"))


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
