"""Benchmark of the NVFP4 hot path (GEMV / GEMM / dual GEMM) on 1..N B200s.

python bench.py [--gpus N] [--steps K] [--warmup W] [--config gemv|gemm|dual|gemm_square]
                [--impl ours|reference]

One "step" is one call of the problem's custom_kernel over one batch of
synthetic inputs of the chosen BASELINE.json configuration (default: configs[1],
the M=7168 K=16384 L=4 GEMV).  Multi-GPU runs (torchrun, one process per GPU)
split the configuration along its natural axis (GEMV rows M, GEMM / dual-GEMM
columns N) with no collective on the data path; every rank times its own
launches with CUDA events and the job time is the max over ranks.

Rank 0 prints one JSON line.  `value` is the whole-job throughput with inputs
resident in HBM; `e2e` is the same metric through the public custom_kernel
API with the inputs copied from pinned host memory and the output copied back
inside the timed region; `roofline` relates the kernel's algorithmic bytes (or
flops) per launch to the measured peak; `cpu_baseline` times the CPU port of
the reference's dequantise-and-matmul path on a bounded sample.
`--impl reference` times that CPU port alone (rank 0; other ranks exit).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "reference-kernels_b200"))

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024

CONFIGS = {
    # name: problem, shape, shard axis, BASELINE.json index
    "gemv": dict(problem="gemv", m=7168, n=1, k=16384, l=4, shard="m", index=1),
    "gemm": dict(problem="gemm", m=1024, n=7168, k=16384, l=1, shard="n", index=2),
    "dual": dict(problem="dual", m=256, n=4096, k=7168, l=1, shard="n", index=3),
    "gemm_square": dict(problem="gemm", m=16384, n=16384, k=16384, l=1, shard="n", index=4),
}


# committed ncu summaries (profiles/<name>.txt) of each workload's kernel
PROFILE_NAMES = {
    "gemv": "gemv_tc_kernel_M7168_K16384_L4",
    "gemm": "gemm_pair_kernel_M1024_N7168_K16384",
    "dual": "dual_gemm_kernel_M256_N4096_K7168",
}


def algo_bytes(problem, m, n, k, l):
    """Algorithmic bytes per call: packed operands, their scales and C (GEMV b unpadded)."""
    nb = 2 if problem == "dual" else 1
    return l * (m * k // 2 + nb * n * k // 2 + m * k // 16 + nb * n * k // 16 + m * n * 2)


def algo_flops(problem, m, n, k, l):
    nb = 2 if problem == "dual" else 1
    return 2 * m * n * k * l * nb


def load_peaks(long_run=False):
    """(HBM GB/s, dense bf16 TFLOP/s, source).  The bf16 figure is the burst
    one for short timed regions and the sustained (power-capped) one when the
    timed region runs long."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        if long_run and "bf16_tflops_sustained" in p:
            return float(p["hbm_gbs"]), float(p["bf16_tflops_sustained"]), "measured sustained"
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured burst"
    except Exception:
        return 6650.0, (1400.0 if long_run else 1590.0), "fallback"


def profile_traffic(name):
    """dram bytes per launch recorded in the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"{name}.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index):
        self.samples = []
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self, t0, t1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        inside = [s for s in self.samples if t0 <= s[0] <= t1] or \
                 sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
        mhz = sorted(s[1] for s in inside)
        mask = 0
        for s in inside:
            mask |= s[2]
        reasons = [v for b, v in self.REASONS.items() if mask & b and v != "gpu_idle"]
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside)}


def make_inputs(cfg, shape, seed, device):
    from nvfp4_b200 import inputs
    m, n, k, l = shape
    if cfg["problem"] == "gemv":
        return inputs.baseline_input("gemv", m, k, l, seed, device=device)
    return inputs.baseline_input(cfg["problem"], m, k, l, seed, n=n, device=device)


def kernel_fn(problem):
    from nvfp4_b200 import ops
    return {"gemv": ops.gemv, "gemm": ops.gemm, "dual": ops.dual_gemm}[problem]


def used_tensors(problem, data):
    """The tuple members the kernel reads (copied host->device for e2e) and the output."""
    if problem == "gemv":
        a, b, _, _, sfa_p, sfb_p, c = data
        return [a, b, sfa_p, sfb_p], c
    if problem == "gemm":
        a, b, _, _, sfa_p, sfb_p, c = data
        return [a, b, sfa_p, sfb_p], c
    a, b1, b2, _, _, _, sfa_p, sfb1_p, sfb2_p, c = data
    return [a, b1, b2, sfa_p, sfb1_p, sfb2_p], c


class CpuSample:
    """A bounded sample of the workload for the CPU port of ref_kernel
    (dequantise to fp32 through lookup tables, fp32 torch matmul, fp16 cast),
    run on all host threads."""

    def __init__(self, cfg, seed=99):
        from nvfp4_b200 import inputs
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.problem, k = cfg["problem"], cfg["k"]
        if self.problem == "gemv":
            m, n = min(cfg["m"], 1024), 1
        elif self.problem == "gemm":
            m, n = min(cfg["m"], 256), min(cfg["n"], 1024)
        else:
            m, n = min(cfg["m"], 256), min(cfg["n"], 512)
        d = inputs.baseline_input(self.problem, m, k, 1, seed, n=None if self.problem == "gemv" else n,
                                  device="cpu")
        u = lambda t: t[:, :, 0].view(torch.uint8)  # noqa: E731
        if self.problem == "dual":
            self.args = (u(d[0]), u(d[1]), u(d[3]), u(d[4]), u(d[2]), u(d[5]))
        else:
            self.args = (u(d[0]), u(d[1]), u(d[2]), u(d[3]))
        if self.problem == "gemv":
            self.work = algo_bytes("gemv", m, 1, k, 1) / 1e9
        else:
            self.work = algo_flops(self.problem, m, n, k, 1) / 1e12
        self.desc = (f"{self.problem} M={m} N={n} K={k} L=1 slice of the {cfg_name(cfg)} workload; "
                     f"dequantise (byte->pair table, e4m3 table) + fp32 torch matmul on {self.threads} threads")

    def run(self):
        """One pass; returns throughput in the metric's unit (GB/s or TFLOP/s)."""
        from oracle import oracle
        t0 = time.perf_counter()
        oracle.cpu_port(self.problem, *self.args)
        return self.work / (time.perf_counter() - t0)


def cpu_sample(cfg, seconds):
    """Median CPU-port throughput over ~`seconds` of repetitions (at least 3)."""
    s = CpuSample(cfg)
    s.run()
    vals = []
    t_end = time.perf_counter() + seconds
    while (time.perf_counter() < t_end or len(vals) < 3) and len(vals) < 500:
        vals.append(s.run())
    return sorted(vals)[len(vals) // 2], s.desc + f"; median of {len(vals)} runs", s.threads


def cfg_name(cfg):
    return next(k for k, v in CONFIGS.items() if v is cfg)


def metric_of(cfg):
    if cfg["problem"] == "gemv":
        return "nvfp4_gemv_hbm_throughput", "GB/s"
    return f"nvfp4_{cfg['problem']}_tflops", "TFLOP/s"


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    metric, unit = metric_of(cfg)
    sample = CpuSample(cfg)
    for _ in range(args.warmup):
        sample.run()
    t0 = time.perf_counter()
    per_step = [sample.run() for _ in range(args.steps)]
    val = sorted(per_step)[len(per_step) // 2]
    threads, desc = sample.threads, sample.desc + f"; median of {args.steps} steps"
    wall = time.perf_counter() - t0
    line = {
        "impl": "reference", "metric": metric, "value": val, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall / max(1, args.steps),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (dequantised nvfp4)",
        "data": "synthetic", "config": {"workload": cfg_name(cfg), "baseline_config_index": cfg["index"],
                                        "M": cfg["m"], "N": cfg["n"], "K": cfg["k"], "L": cfg["l"]},
        "cpu_baseline": {"value": val, "unit": unit, "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": val, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# The reference's task.yml `benchmarks:` shapes and their published
# speed-of-light times (problems/nvidia/nvfp4_*/task.yml descriptions).
SUITE = [
    ("gemv", 7168, 1, 16384, 1, 8.622), ("gemv", 4096, 1, 7168, 8, 17.275), ("gemv", 7168, 1, 2048, 4, 4.317),
    ("gemm", 128, 7168, 16384, 1, 8.994), ("gemm", 128, 4096, 7168, 1, 2.354), ("gemm", 128, 7168, 2048, 1, 1.333),
    ("dual", 256, 4096, 7168, 1, 4.708), ("dual", 512, 4096, 7168, 1, 8.714), ("dual", 256, 3072, 4096, 1, 2.125),
    ("dual", 512, 3072, 7168, 1, 6.535),
]


def run_suite(repeats=20):
    """Times the reference's benchmark shapes the way its harnesses do:
    GEMM / dual GEMM: 50 distinct seeded inputs per event pair after an L2
    flush, time / 50 (eval_better_bench.py:252-268); GEMV: one call per event
    pair after an L2 flush (eval.py:238-245).  Inputs: the reference's own
    distributions (generate_input restated in nvfp4_b200.inputs)."""
    from nvfp4_b200 import inputs
    flush = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    logs = []
    for prob, m, n, k, l, sol in SUITE:
        fn = kernel_fn(prob)
        count = 1 if prob == "gemv" else 50
        datas = [inputs.reference_input(prob, m, k, l, 1111 + 42 * (i + 1), n=None if prob == "gemv" else n)
                 for i in range(count)]
        for d in datas:
            fn(d)
        torch.cuda.synchronize()
        times = []
        for _ in range(repeats if prob != "gemv" else 5 * repeats):
            flush.fill_(1)
            e0.record()
            for d in datas:
                fn(d)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3 / count)
        mean = sum(times) / len(times)
        line = {"suite": "reference_benchmarks", "problem": prob, "m": m, "n": n, "k": k, "l": l,
                "us_mean": mean, "us_best": min(times), "sol_us": sol, "sol_over_time": sol / mean}
        logs.append(mean / sol)
        print(json.dumps(line), flush=True)
    geo = math.exp(sum(math.log(x) for x in logs) / len(logs))
    print(json.dumps({"suite": "reference_benchmarks", "geomean_time_over_sol": geo}), flush=True)


def gather_check(problem, full_data, fn, world, rank, dist):
    """Multi-GPU correctness evidence, outside the timed region: every rank's
    slice of C (written by its shard's custom_kernel calls) is assembled with an
    NCCL all-gather, and rank 0 compares it with the whole problem run on its
    one GPU (rtol = atol = 1e-3, infinities equal — the reference's check; the
    two runs tile and split K differently, so bit equality is not expected)."""
    from nvfp4_b200 import shard
    c = full_data[-1]
    shape = tuple(c.shape)
    axis = 0 if problem == "gemv" else 1
    bounds = [shard.shard_bounds(shape[axis], world, r) for r in range(world)]
    width = max(hi - lo for lo, hi in bounds)
    mine = c[shard.output_slice(problem, shape, world, rank)]
    pad_shape = list(shape)
    pad_shape[axis] = width
    send = torch.zeros(pad_shape, dtype=c.dtype, device=c.device)
    send.narrow(axis, 0, mine.shape[axis]).copy_(mine)
    recv = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(recv, send)
    if rank != 0:
        return None
    assembled = torch.cat([r.narrow(axis, 0, hi - lo) for r, (lo, hi) in zip(recv, bounds)], dim=axis)
    fn(full_data)  # the whole problem on rank 0's GPU, into the same C buffer
    if c.is_cuda:
        torch.cuda.synchronize()
    close = torch.isclose(assembled.float(), c.float(), rtol=1e-3, atol=1e-3, equal_nan=True)
    bad = int((~close).sum())
    return {"kind": "NCCL all_gather of the ranks' C slices vs the whole problem on rank 0's GPU",
            "elements": int(close.numel()), "mismatches": bad, "ok": bad == 0}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="gemv", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--eager", action="store_true",
                    help="time the K steps as eager calls instead of one CUDA-graph replay")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--suite", action="store_true",
                    help="time the reference's task.yml benchmark shapes (one JSON line each) and exit")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    for d in "mnkl":
        ap.add_argument(f"--{d}", type=int, default=None, help=f"override {d.upper()} (small profiling cases)")
    args = ap.parse_args()
    if args.suite:
        return run_suite()
    cfg = CONFIGS[args.config]
    if any(getattr(args, d) is not None for d in "mnkl"):
        cfg = dict(cfg, **{d: getattr(args, d) for d in "mnkl" if getattr(args, d) is not None})
        CONFIGS[f"{args.config}_custom"] = cfg
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        return run_reference(args, cfg)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    from nvfp4_b200 import shard
    problem = cfg["problem"]
    fn = kernel_fn(problem)
    full_shape = (cfg["m"], cfg["n"], cfg["k"], cfg["l"])
    # Every rank draws the full problem from the same seed and runs its shard
    # (GEMV rows / GEMM columns) through views of it.
    one_full = make_inputs(cfg, full_shape, 1111 + cfg["index"], dev)
    one = shard.shard_tuple(problem, one_full, world, rank)
    m, k2, l = one[0].shape
    k = 2 * k2
    n = 1 if problem == "gemv" else one[1].shape[0]
    shape = (m, n, k, l)
    bytes_step = algo_bytes(problem, m, n, k, l)
    flops_step = algo_flops(problem, m, n, k, l)

    # Rotating input sets so that every step reads operands that are not in L2.
    read_bytes = sum(t.numel() * t.element_size() for t in used_tensors(problem, one)[0])
    nsets = max(1, min(8, math.ceil(2 * L2_BYTES / read_bytes) + (1 if read_bytes < L2_BYTES else 0)))
    sets = [one] + [shard.shard_tuple(problem, make_inputs(cfg, full_shape, 2000 + 17 * i, dev), world, rank)
                    for i in range(1, nsets)]
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        fn(sets[i % nsets])
    torch.cuda.synchronize()

    # ---- device-resident timed region.  The K steps are captured into one
    # CUDA graph (PDL edges between the launches are kept) and replayed once,
    # so the host's per-call dispatch (~8 us) does not pace short shards; the
    # per-launch kernel durations come from a separate eager pass with an
    # event pair around every launch.
    use_graph = not args.eager
    graph = None
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                fn(sets[i % nsets])
        for _ in range(max(1, args.warmup // max(1, args.steps))):
            graph.replay()
        torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler:
        time.sleep(0.01)
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        start.record(stream)
        if use_graph:
            graph.replay()
        else:
            for i in range(args.steps):
                fn(sets[i % nsets])
        end.record(stream)
        torch.cuda.synchronize()
        w1 = time.perf_counter()
        # per-launch durations (eager, one event pair per launch)
        for i in range(args.steps):
            ev[i][0].record(stream)
            fn(sets[i % nsets])
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        w2 = time.perf_counter()
        if dist:
            dist.barrier()
    # clocks under load: the graph replay and the eager pass right after it
    clocks = sampler.summary(w0, w2)
    clocks["timed_region_s"] = w1 - w0
    t_ms = start.elapsed_time(end)
    launch_ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    t_all = torch.tensor([t_ms, launch_ms], device=dev)
    if dist:
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    t_ms, iso_ms = float(t_all[0]), float(t_all[1])
    # Average launch duration over the timed region: only this kernel runs
    # there, one launch per step, consecutive launches overlapping their
    # prologues through programmatic dependent launch.  The isolated figure
    # (one event pair around each launch, no overlap) is reported beside it.
    launch_ms = t_ms / args.steps

    # ---- end to end: pinned host inputs -> device, custom_kernel, output -> host
    ins, out = used_tensors(problem, sets[0])
    host_in = [t.cpu().pin_memory() for t in ins]
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out.numel() * host_out.element_size()
    e2e_steps = max(3, min(args.e2e_steps, args.steps))
    for _ in range(2):
        for hd, t in zip(host_in, ins):
            t.copy_(hd, non_blocking=True)
        fn(sets[0])
        host_out.copy_(out, non_blocking=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        for hd, t in zip(host_in, ins):
            t.copy_(hd, non_blocking=True)
        fn(sets[0])
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev)
    if dist:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        dist.barrier()
    e_ms = float(e_ms)

    check = gather_check(problem, one_full, fn, world, rank, dist) if dist else None

    # whole-job totals
    tot_bytes = bytes_step * world
    tot_flops = flops_step * world
    ms_step = t_ms / args.steps
    metric, unit = metric_of(cfg)
    # A timed region over 100 ms is a long, power-capped run: sustained peak.
    hbm_peak, bf16_peak, peak_kind = load_peaks(long_run=t_ms > 100.0)
    if problem == "gemv":
        value = tot_bytes / (ms_step * 1e-3) / 1e9
        e2e_value = tot_bytes / (e_ms * 1e-3) / 1e9
        achieved = bytes_step / (launch_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_source": f"{peak_kind} hbm_gbs (copy bandwidth)"}
    else:
        value = tot_flops / (ms_step * 1e-3) / 1e12
        e2e_value = tot_flops / (e_ms * 1e-3) / 1e12
        achieved = flops_step / (launch_ms * 1e-3) / 1e12
        fp4_peak = 4.0 * bf16_peak
        t_mem = bytes_step / (hbm_peak * 1e9)
        t_fp4 = flops_step / (fp4_peak * 1e12)
        roof = {"bound": "tensor", "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s",
                "frac": achieved / fp4_peak,
                "peak_source": f"4 x {peak_kind} dense bf16 (B200 dense fp4 = 4x bf16)",
                "frac_of_max_mem_fp4_roofline": (max(t_mem, t_fp4) * 1e3) / launch_ms}
    roof["traffic"] = profile_traffic(PROFILE_NAMES.get(cfg_name(cfg), "")) if world == 1 else None
    roof["kernel_ms_per_launch"] = launch_ms
    roof["kernel_ms_per_launch_isolated"] = iso_ms
    roof["frac_isolated"] = roof["frac"] * launch_ms / iso_ms
    roof["algorithmic_bytes_per_launch"] = bytes_step
    if problem != "gemv":
        roof["algorithmic_flops_per_launch"] = flops_step

    line = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "nvfp4 e2m1 x e4m3/16 -> fp32 acc -> fp16", "data": "synthetic",
        "config": {"workload": cfg_name(cfg), "baseline_config_index": cfg["index"], "M": cfg["m"], "N": cfg["n"],
                   "K": cfg["k"], "L": cfg["l"], "shard": f"{cfg['shard']}/{world}", "per_rank_shape": list(shape),
                   "l2": f"{nsets} rotating input sets of {read_bytes / 1e6:.1f} MB (L2 126 MB)",
                   "distribution": "bytes uniform 0..255, scales uniform [0.25, 2] -> e4m3",
                   "launch": "eager custom_kernel calls" if args.eager else
                   "K custom_kernel calls captured in one CUDA graph, replayed once"},
        "roofline": roof,
        "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                "steps": e2e_steps, "ms_per_step": e_ms,
                "path": "pinned host -> device copies of the tensors the kernel reads, custom_kernel, output -> host"},
        "gpu_launches": args.steps,
        **({"check": check} if check else {}),
        "clocks": clocks,
    }
    if rank == 0 and world == 1:
        v, desc, threads = cpu_sample(cfg, args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": unit, "cores": threads, "kind": "port", "sample": desc}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
