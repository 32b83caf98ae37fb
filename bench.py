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
    "gemm_square": "gemm_pair_kernel_M16384_N16384_K16384",
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
    """The CPU port of ref_kernel (dequantise to fp32 through lookup tables,
    fp32 torch matmul, fp16 cast; oracle.cpu_port) on all host threads.  It
    runs the whole configuration (every batch index) except for the 16384^3
    GEMM, where one pass would take minutes and a 1024-column slice of N
    stands in (`same_config` says which)."""

    SLICE_N = {"gemm_square": 1024}

    def __init__(self, cfg, seed=99):
        from nvfp4_b200 import inputs
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.problem, m, n, k, l = cfg["problem"], cfg["m"], cfg["n"], cfg["k"], cfg["l"]
        n = min(n, self.SLICE_N.get(cfg_name(cfg), n))
        self.same_config = n == cfg["n"]
        d = inputs.baseline_input(self.problem, m, k, l, seed, n=None if self.problem == "gemv" else n,
                                  device="cpu")
        u = lambda t, i: t[:, :, i].view(torch.uint8)  # noqa: E731
        if self.problem == "dual":
            self.args = [(u(d[0], i), u(d[1], i), u(d[3], i), u(d[4], i), u(d[2], i), u(d[5], i)) for i in range(l)]
        else:
            self.args = [(u(d[0], i), u(d[1], i), u(d[2], i), u(d[3], i)) for i in range(l)]
        if self.problem == "gemv":
            self.work = algo_bytes("gemv", m, 1, k, l) / 1e9
        else:
            self.work = algo_flops(self.problem, m, n, k, l) / 1e12
        what = "the whole" if self.same_config else f"an N={n} column slice of the"
        self.desc = (f"{self.problem} M={m} N={n} K={k} L={l}: {what} {cfg_name(cfg)} workload; "
                     f"dequantise (byte->pair table, e4m3 table) + fp32 torch matmul on {self.threads} threads")

    def run(self):
        """One pass; returns throughput in the metric's unit (GB/s or TFLOP/s)."""
        from oracle import oracle
        t0 = time.perf_counter()
        for args in self.args:
            oracle.cpu_port(self.problem, *args)
        return self.work / (time.perf_counter() - t0)


def cpu_sample(cfg, seconds):
    """Median CPU-port throughput over ~`seconds` of repetitions (at least 2)."""
    s = CpuSample(cfg)
    s.run()
    vals = []
    t_end = time.perf_counter() + seconds
    while (time.perf_counter() < t_end or len(vals) < 2) and len(vals) < 500:
        vals.append(s.run())
    return sorted(vals)[len(vals) // 2], s.desc + f"; median of {len(vals)} runs", s.threads, s.same_config


def cfg_name(cfg):
    return next(k for k, v in CONFIGS.items() if v is cfg)


def metric_of(cfg):
    if cfg["problem"] == "gemv":
        return "nvfp4_gemv_hbm_throughput", "GB/s"
    return f"nvfp4_{cfg['problem']}_tflops", "TFLOP/s"


def _reference_leg(cfg, steps, warmup, budget_s):
    """The CPU port on `cfg`: `warmup` untimed passes (at most 1), then up to
    `steps` timed passes, stopping early once `budget_s` seconds have run."""
    sample = CpuSample(cfg)
    for _ in range(min(warmup, 1)):
        sample.run()
    t0 = time.perf_counter()
    per_step = []
    while len(per_step) < max(1, steps) and (not per_step or time.perf_counter() - t0 < budget_s):
        per_step.append(sample.run())
    wall = time.perf_counter() - t0
    val = sorted(per_step)[len(per_step) // 2]
    desc = sample.desc + f"; median of {len(per_step)} passes"
    return val, wall / len(per_step), len(per_step), sample, desc


def run_reference(args, cfg):
    """The reference arm: the reference's dequantise-and-matmul path on the
    host cores (the reference has no CPU implementation of its own, so its
    ref_kernel is restated as oracle.cpu_port).  Rank 0 alone runs it; the
    default run adds the other configurations under `per_config`."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    metric, unit = metric_of(cfg)
    val, sec, ran, sample, desc = _reference_leg(cfg, args.steps, args.warmup, args.ref_seconds)
    line = {
        "impl": "reference", "metric": metric, "value": val, "unit": unit, "n_gpus": args.gpus,
        "steps": ran, "steps_requested": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sec,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (dequantised nvfp4)",
        "data": "synthetic", "config": {"workload": cfg_name(cfg), "baseline_config_index": cfg["index"],
                                        "M": cfg["m"], "N": cfg["n"], "K": cfg["k"], "L": cfg["l"]},
        "cpu_baseline": {"value": val, "unit": unit, "cores": sample.threads, "kind": "port", "sample": desc,
                         "same_config": sample.same_config},
        "e2e": {"value": val, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.all_configs:
        per = {}
        for name in PER_CONFIG:
            c = CONFIGS[name]
            m2, u2 = metric_of(c)
            v2, s2, r2, smp, d2 = _reference_leg(c, 3, 1, args.ref_seconds / 4)
            per[name] = {"metric": m2, "value": v2, "unit": u2, "ms_per_step": 1e3 * s2, "steps": r2,
                         "config": {"workload": name, "baseline_config_index": c["index"], "M": c["m"],
                                    "N": c["n"], "K": c["k"], "L": c["l"]},
                         "cpu_baseline": {"value": v2, "unit": u2, "cores": smp.threads, "kind": "port",
                                          "sample": d2, "same_config": smp.same_config},
                         "e2e": {"value": v2, "unit": u2, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        line["per_config"] = per
    print(json.dumps(line), flush=True)


# Speed-of-light times (us) the reference publishes for its task.yml
# `benchmarks:` shapes (problems/nvidia/nvfp4_*/task.yml descriptions).
SOL_US = {
    ("gemv", 7168, 1, 16384, 1): 8.622, ("gemv", 4096, 1, 7168, 8): 17.275, ("gemv", 7168, 1, 2048, 4): 4.317,
    ("gemm", 128, 7168, 16384, 1): 8.994, ("gemm", 128, 4096, 7168, 1): 2.354, ("gemm", 128, 7168, 2048, 1): 1.333,
    ("dual", 256, 4096, 7168, 1): 4.708, ("dual", 512, 4096, 7168, 1): 8.714, ("dual", 256, 3072, 4096, 1): 2.125,
    ("dual", 512, 3072, 7168, 1): 6.535,
}


def suite_cases():
    """(problem, m, n, k, l, source) for every task.yml benchmark shape of the
    three problems and BASELINE.json configs 1-4."""
    cases = [(p, m, n, k, l, "task.yml benchmarks") for (p, m, n, k, l) in SOL_US]
    for name in ("gemv", "gemm", "dual", "gemm_square"):
        c = CONFIGS[name]
        cases.append((c["problem"], c["m"], c["n"], c["k"], c["l"], f"BASELINE configs[{c['index']}]"))
    return cases


def _suite_inputs(ref, prob, m, n, k, l, source, count, seed0):
    """Inputs for one suite case: the reference's own generate_input for the
    task.yml shapes (seed 1111 + 42 i, as eval_better_bench.py:180-183 does),
    the BASELINE distributions for BASELINE configs."""
    from nvfp4_b200 import inputs
    out = []
    for i in range(count):
        seed = seed0 + 42 * (i + 1)
        if source.startswith("task.yml"):
            kw = dict(m=m, k=k, l=l, seed=seed) if prob == "gemv" else dict(m=m, n=n, k=k, l=l, seed=seed)
            out.append(ref.generate_input(**kw))
        else:
            out.append(inputs.baseline_input(prob, m, k, l, seed, n=None if prob == "gemv" else n, device="cuda"))
    return out


def _clone(data):
    return tuple(t.clone() if isinstance(t, torch.Tensor) else t for t in data)


def _time_impl(fn, datas, flush, budget_s=1.5, max_repeats=50):
    """Mean us per call: all of `datas` between one event pair after an L2
    flush, repeated until `budget_s` (the timing of eval_better_bench.py:252-268)."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for d in datas:
        fn(d)
    torch.cuda.synchronize()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < max_repeats):
        flush.fill_(1)
        e0.record()
        for d in datas:
            fn(d)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3 / len(datas))
    return sum(times) / len(times), min(times)


def run_suite(only=None):
    """Same-box comparison with the reference's own implementations of the path.

    For every task.yml benchmark shape and BASELINE config 1-4, three
    implementations are run on identical inputs and timed the way the
    reference's harness times them (50 distinct inputs per event pair after an
    L2 flush, fewer when 50 would not fit in a few GB):
      ours       this build's custom_kernel (libnvfp4_b200.so);
      ref_cute   the reference's CuTe-DSL sm_100 custom_kernel, unmodified
                 (nvfp4_gemm/submission.py:708-761, nvfp4_dual_gemm/submission.py:894-957,
                 nvfp4_gemv/template_cute.py:199-247);
      scaled_mm  the reference's ref_kernel (torch._scaled_mm -> cuBLASLt,
                 nvfp4_*/reference.py), as written.
    Each implementation's output on the first input is checked with the
    reference's check_implementation (rtol = atol = 1e-3).  The reference is
    imported from the baseline/_ref install (baseline/refload.py)."""
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import refload
    if not refload.available():
        print(json.dumps({"suite": "same_box", "unavailable": "reference not installed in baseline/_ref"}))
        return
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ratios = {"ref_cute": [], "scaled_mm": []}
    for prob, m, n, k, l, source in suite_cases():
        if only and prob not in only:
            continue
        ref = refload.load(prob)
        cute_mod = refload.load(prob, "template_cute" if prob == "gemv" else "submission")
        impls = {"ours": kernel_fn(prob), "ref_cute": cute_mod.custom_kernel, "scaled_mm": ref.ref_kernel}
        per_set = algo_bytes(prob, m, n, k, l) + (m * n * l * 2 if prob != "gemv" else 0)
        count = 1 if prob == "gemv" else max(2, min(50, int(4e9 // per_set)))
        datas = _suite_inputs(ref, prob, m, n, k, l, source, count, 1111)
        line = {"suite": "same_box", "problem": prob, "m": m, "n": n, "k": k, "l": l, "source": source,
                "inputs_per_timing": count}
        sol = SOL_US.get((prob, m, n, k, l))
        for name, fn in impls.items():
            try:
                first = _clone(datas[0])
                out = fn(first)
                torch.cuda.synchronize()
                ok, msg = ref.check_implementation(_clone(datas[0]), out)
                mean, best = _time_impl(fn, datas, flush)
                line[f"{name}_us"] = mean
                line[f"{name}_us_best"] = best
                line[f"{name}_check"] = "pass" if ok else f"fail: {msg[:200]}"
            except Exception as e:  # noqa: BLE001 - one implementation failing must not hide the others
                line[f"{name}_us"] = None
                line[f"{name}_error"] = f"{type(e).__name__}: {str(e)[:300]}"
            torch.cuda.synchronize()
        for other in ("ref_cute", "scaled_mm"):
            if line.get("ours_us") and line.get(f"{other}_us"):
                line[f"speedup_vs_{other}"] = line[f"{other}_us"] / line["ours_us"]
                ratios[other].append(line[f"speedup_vs_{other}"])
        if prob == "gemv":
            line["ours_gbs"] = algo_bytes(prob, m, n, k, l) / (line["ours_us"] * 1e3) if line.get("ours_us") else None
        else:
            line["ours_tflops"] = algo_flops(prob, m, n, k, l) / (line["ours_us"] * 1e6) if line.get("ours_us") else None
        if sol:
            line["sol_us"] = sol
        print(json.dumps(line), flush=True)
        del datas
        torch.cuda.empty_cache()
    summary = {"suite": "same_box"}
    for other, xs in ratios.items():
        if xs:
            summary[f"geomean_speedup_vs_{other}"] = math.exp(sum(math.log(x) for x in xs) / len(xs))
            summary[f"min_speedup_vs_{other}"] = min(xs)
    print(json.dumps(summary), flush=True)


def scaled_mm_reference(problem, data):
    """The reference's ref_kernel arithmetic (nvfp4_*/reference.py): one
    torch._scaled_mm per batch index on the plain scales put in the blocked
    order, fp16 out (the dual GEMM: two fp32 products, silu(x)*y in fp32)."""
    from nvfp4_b200.inputs import to_blocked
    c = data[-1]
    m, n, l = c.shape
    out = torch.empty((m, n, l), dtype=torch.float16, device=c.device)
    for i in range(l):
        if problem == "dual":
            a, b1, b2, sfa, sfb1, sfb2 = data[:6]
            sa = to_blocked(sfa[:, :, i].contiguous())
            r1 = torch._scaled_mm(a[:, :, i], b1[:, :, i].transpose(0, 1), sa,
                                  to_blocked(sfb1[:, :, i].contiguous()), bias=None, out_dtype=torch.float32)
            r2 = torch._scaled_mm(a[:, :, i], b2[:, :, i].transpose(0, 1), sa,
                                  to_blocked(sfb2[:, :, i].contiguous()), bias=None, out_dtype=torch.float32)
            out[:, :, i] = (torch.nn.functional.silu(r1) * r2).to(torch.float16)
            continue
        a, b, sfa, sfb = data[:4]
        res = torch._scaled_mm(a[:, :, i], b[:, :, i].transpose(0, 1), to_blocked(sfa[:, :, i].contiguous()),
                               to_blocked(sfb[:, :, i].contiguous()), bias=None, out_dtype=torch.float16)
        out[:, :, i] = res[:, :1] if problem == "gemv" else res
    return out


def gather_check(problem, c_shape, mine, expected_fn, world, rank, dist):
    """Multi-GPU correctness evidence, outside the timed region: every rank's
    slice of C (its shard's output, `mine`) is assembled with an NCCL
    all-gather, and rank 0 compares it with `expected_fn()` — the reference's
    own arithmetic (torch._scaled_mm, as ref_kernel calls it) on the whole
    problem — with the reference's tolerance (rtol = atol = 1e-3, infinities
    equal)."""
    from nvfp4_b200 import shard
    axis = 0 if problem == "gemv" else 1
    bounds = [shard.shard_bounds(c_shape[axis], world, r) for r in range(world)]
    width = max(hi - lo for lo, hi in bounds)
    pad_shape = list(c_shape)
    pad_shape[axis] = width
    send = torch.zeros(pad_shape, dtype=mine.dtype, device=mine.device)
    send.narrow(axis, 0, mine.shape[axis]).copy_(mine)
    recv = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(recv, send)
    if rank != 0:
        return None
    assembled = torch.cat([r.narrow(axis, 0, hi - lo) for r, (lo, hi) in zip(recv, bounds)], dim=axis)
    expected = expected_fn()
    if expected.is_cuda:
        torch.cuda.synchronize()
    close = torch.isclose(assembled.float(), expected.float(), rtol=1e-3, atol=1e-3, equal_nan=True)
    bad = int((~close).sum())
    return {"kind": "NCCL all_gather of the ranks' C slices vs torch._scaled_mm (ref_kernel) on the whole problem",
            "elements": int(close.numel()), "mismatches": bad, "ok": bad == 0}


# configurations reported under `per_config` in the default run, besides the headline
PER_CONFIG = ("gemm", "dual", "gemm_square")


class Ctx:
    def __init__(self, world, rank, local, dev, dist):
        self.world, self.rank, self.local, self.dev, self.dist = world, rank, local, dev, dist

    def max_over_ranks(self, *vals):
        t = torch.tensor(vals, dtype=torch.float64, device=self.dev)
        if self.dist:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(x) for x in t]

    def barrier(self):
        if self.dist:
            self.dist.barrier()


def measure(cfg, args, ctx, steps, with_cpu):
    """One configuration: device-resident throughput (`value`), the kernel's
    roofline, end-to-end throughput through custom_kernel with host buffers,
    and (N > 1) the gathered-output check.  Returns the JSON fields."""
    from nvfp4_b200 import shard
    name = cfg_name(cfg)
    world, rank, dev = ctx.world, ctx.rank, ctx.dev
    problem = cfg["problem"]
    fn = kernel_fn(problem)
    full_shape = (cfg["m"], cfg["n"], cfg["k"], cfg["l"])
    # Every rank draws the full problem from the same seed and keeps a dense
    # copy of its shard (GEMV rows / GEMM columns) in the reference's layout.
    full = make_inputs(cfg, full_shape, 1111 + cfg["index"], dev)
    one = shard.dense_shard_tuple(problem, full, world, rank)
    keep_full = world > 1 and rank == 0
    if not keep_full:
        del full
    m, k2, l = one[0].shape
    k = 2 * k2
    n = 1 if problem == "gemv" else one[1].shape[0]
    shape = (m, n, k, l)
    bytes_step = algo_bytes(problem, m, n, k, l)
    flops_step = algo_flops(problem, m, n, k, l)

    # Rotating input sets so that every step reads operands that are not in L2
    # (at least two sets, so that no two consecutive steps read the same one).
    read_bytes = sum(t.numel() * t.element_size() for t in used_tensors(problem, one)[0])
    nsets = max(2, min(8, math.ceil(2 * L2_BYTES / read_bytes) + (1 if read_bytes < L2_BYTES else 0)))
    sets = [one]
    for i in range(1, nsets):
        other = make_inputs(cfg, full_shape, 2000 + 17 * i, dev)
        sets.append(shard.dense_shard_tuple(problem, other, world, rank))
        del other
    torch.cuda.synchronize()

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
            for i in range(steps):
                fn(sets[i % nsets])
        graph.replay()
        torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(ctx.local)
    with sampler:
        time.sleep(0.01)
        ctx.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        start.record(stream)
        if use_graph:
            graph.replay()
        else:
            for i in range(steps):
                fn(sets[i % nsets])
        end.record(stream)
        torch.cuda.synchronize()
        w1 = time.perf_counter()
        for i in range(steps):
            ev[i][0].record(stream)
            fn(sets[i % nsets])
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        w2 = time.perf_counter()
        ctx.barrier()
    clocks = sampler.summary(w0, w2)
    clocks["timed_region_s"] = w1 - w0
    iso_ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    t_ms, iso_ms = ctx.max_over_ranks(start.elapsed_time(end), iso_ms)
    del graph
    # Average launch duration over the timed region: only this kernel runs
    # there, one launch per step, consecutive launches overlapping their
    # prologues through programmatic dependent launch.  The isolated figure
    # (one event pair around each launch, no overlap) is reported beside it.
    launch_ms = t_ms / steps

    # ---- end to end: pinned host buffers with the device tensors' layout ->
    # device, custom_kernel, output -> host.  Dense shards make each copy one DMA.
    ins, out = used_tensors(problem, sets[0])
    host_in = [torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, pin_memory=True) for t in ins]
    for h, t in zip(host_in, ins):
        h.copy_(t)
    host_out = torch.empty_strided(out.shape, out.stride(), dtype=out.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out.numel() * host_out.element_size()
    e2e_steps = max(3, min(args.e2e_steps, steps))

    def e2e_step():
        for hd, t in zip(host_in, ins):
            t.copy_(hd, non_blocking=True)
        fn(sets[0])
        host_out.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    (e_ms,) = ctx.max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    ctx.barrier()

    check = None
    if world > 1:
        check = gather_check(problem, tuple(cfg[d] for d in ("m", "n", "l")) if problem != "gemv"
                             else (cfg["m"], 1, cfg["l"]), sets[0][-1],
                             (lambda: scaled_mm_reference(problem, full)) if keep_full else None,
                             world, rank, ctx.dist)
    if keep_full:
        del full
    del sets, one, host_in, host_out, ins, out
    torch.cuda.empty_cache()

    tot_bytes, tot_flops = bytes_step * world, flops_step * world
    ms_step = t_ms / steps
    metric, unit = metric_of(cfg)
    # A timed region over 100 ms, or one the power cap throttled, is judged
    # against the sustained (power-capped) peak.
    hbm_peak, bf16_peak, peak_kind = load_peaks(long_run=t_ms > 100.0 or "sw_power_cap" in clocks["reasons"])
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
    roof["traffic"] = profile_traffic(PROFILE_NAMES.get(name, "")) if world == 1 else None
    roof["kernel_ms_per_launch"] = launch_ms
    roof["kernel_ms_per_launch_isolated"] = iso_ms
    roof["frac_isolated"] = roof["frac"] * launch_ms / iso_ms
    roof["algorithmic_bytes_per_launch"] = bytes_step
    if problem != "gemv":
        roof["algorithmic_flops_per_launch"] = flops_step

    res = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "nvfp4 e2m1 x e4m3/16 -> fp32 acc -> fp16", "data": "synthetic",
        "config": {"workload": name, "baseline_config_index": cfg["index"], "M": cfg["m"], "N": cfg["n"],
                   "K": cfg["k"], "L": cfg["l"], "shard": f"{cfg['shard']}/{world}", "per_rank_shape": list(shape),
                   "l2": f"{nsets} rotating input sets of {read_bytes / 1e6:.1f} MB (L2 126 MB)",
                   "distribution": "bytes uniform 0..255, scales uniform [0.25, 2] -> e4m3",
                   "launch": "eager custom_kernel calls" if args.eager else
                   "K custom_kernel calls captured in one CUDA graph, replayed once"},
        "roofline": roof,
        "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": h2d * world,
                "d2h_bytes_per_step": d2h * world, "steps": e2e_steps, "ms_per_step": e_ms,
                "path": "pinned host -> device copies of the tensors the kernel reads, custom_kernel, "
                        "output -> host"},
        "gpu_launches": steps,
        **({"check": check} if check else {}),
        "clocks": clocks,
    }
    if with_cpu and rank == 0 and world == 1:
        v, desc, threads, same = cpu_sample(cfg, args.cpu_seconds)
        res["cpu_baseline"] = {"value": v, "unit": unit, "cores": threads, "kind": "port", "sample": desc,
                               "same_config": same}
    return res


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
    ap.add_argument("--headline-only", dest="all_configs", action="store_false",
                    help="measure only --config (default: also GEMM, dual GEMM and 16384^3 under per_config)")
    ap.add_argument("--suite", action="store_true",
                    help="same-box comparison with the reference's CuTe kernels and ref_kernel (one JSON line "
                         "per shape) and exit")
    ap.add_argument("--suite-only", default=None, help="comma-separated problems for --suite")
    ap.add_argument("--cpu-seconds", type=float, default=5.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg (tuning runs)")
    ap.add_argument("--ref-seconds", type=float, default=60.0,
                    help="time budget of the reference arm's timed passes")
    for d in "mnkl":
        ap.add_argument(f"--{d}", type=int, default=None, help=f"override {d.upper()} (small profiling cases)")
    args = ap.parse_args()
    if args.suite:
        return run_suite(args.suite_only.split(",") if args.suite_only else None)
    cfg = CONFIGS[args.config]
    if any(getattr(args, d) is not None for d in "mnkl"):
        cfg = dict(cfg, **{d: getattr(args, d) for d in "mnkl" if getattr(args, d) is not None})
        CONFIGS[f"{args.config}_custom"] = cfg
        args.all_configs = False
    if args.config != "gemv":
        args.all_configs = False
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
    ctx = Ctx(world, rank, local, dev, dist)

    line = measure(cfg, args, ctx, args.steps, with_cpu=not args.no_cpu)
    if args.all_configs:
        per = {}
        for name in PER_CONFIG:
            c = CONFIGS[name]
            # the 16384^3 GEMM runs ~2 ms per step on one GPU: fewer steps keep
            # its timed region near a second
            steps = min(args.steps, 50) if name == "gemm_square" else args.steps
            per[name] = measure(c, args, ctx, steps, with_cpu=not args.no_cpu)
        line["per_config"] = per
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
