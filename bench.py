"""Benchmark of the fused dense-operator path on B200.

One step = one call of the headline operator over one batch of synthetic input:
BASELINE configs[1], plain GEMM M=N=K=4096, bf16 A (row-major) and B (column-major),
fp32 accumulate, bf16 out, seed 1.  `value` is device time (CUDA events on the launching
stream, L2 flushed between steps by a 256 MiB write outside the events), `e2e` is the
same metric through the public API (icpp_tuning_b200.gemm.gemm.build_kernel) with the
step's inputs copied from pinned host memory and the result read back inside the timed
region.  At N>1 (torchrun, NCCL) every rank owns one 4096-row shard of a global
M = 4096*N problem (weak scaling, no collective on the data path); times are the max
over ranks.  Rank 0 prints one JSON line.  At N=1 it also carries `per_op` (all five
BASELINE workloads, device time, each beside the reference's CPU program on a row
sample); at N>1 `strong` (each fixed global workload split into row / image shards over
the ranks, global FLOPs over the max per-rank time, plus the NCCL all-gather of the
output timed separately).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "TFLOP/s per fused op (GEMM+bias+act/LN, conv) and % of B200 BF16 peak"
UNIT = "TFLOP/s"
WORKLOAD = ("gemm M=N=K=4096 bf16: A row-major, B column-major, fp32 accumulate, bf16 out, "
            "A,B ~ N(0,1)/sqrt(K), seed 1 (BASELINE configs[1])")
M0 = N0 = K0 = 4096
FLUSH_BYTES = 256 << 20
# ~100 us of GPU spin queued ahead of every start event, so the host-side launch cost of
# the timed call is hidden and the events bracket device execution only.
QUEUE_PAD_CYCLES = 200_000


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d.get("bf16_tflops_sustained"), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        return ws, rank, local, dist
    torch.cuda.set_device(local)
    return 1, 0, local, None


def _barrier(dist):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(x: float, dist) -> float:
    if dist is None:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of one GPU, sampled every 50 ms."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except OSError:
            self.proc = None
        time.sleep(0.2)
        return self

    def _read(self):
        for line in self.proc.stdout:
            f = [x.strip() for x in line.split(",")]
            if len(f) == 8:
                self.rows.append(f)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        load = [r for r in self.rows if (num(r[3]) or 0) >= 50] or self.rows
        sm = [num(r[0]) for r in load if num(r[0]) is not None]
        mx = [num(r[1]) for r in self.rows if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in load for i in range(4) if r[4 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(load)}


def _inputs(seed: int, rank: int):
    g = torch.Generator().manual_seed(seed + 1000 * rank)
    a = (torch.randn(M0, K0, generator=g) * K0 ** -0.5).to(torch.bfloat16)
    bt = (torch.randn(N0, K0, generator=g) * K0 ** -0.5).to(torch.bfloat16)  # B column-major
    return a, bt


def e2e_pipelined(kern, a_h, bt_h, out_like, dev, steps: int, dist) -> float:
    """Mean ms per step of `steps` host-to-host calls of kern (see run_ours), max over ranks."""
    a_p, bt_p = a_h.pin_memory(), bt_h.pin_memory()
    outs_p = [torch.empty_like(out_like, device="cpu").pin_memory() for _ in range(2)]
    a_d = [torch.empty_like(a_p, device=dev) for _ in range(2)]
    bt_d = [torch.empty_like(bt_p, device=dev) for _ in range(2)]
    out_d = [torch.empty_like(out_like) for _ in range(2)]
    s_in, s_mm, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_done = [ev(), ev()]
    mm_done = [ev(), ev()]
    out_done = [ev(), ev()]

    def run(n):
        for i in range(n):
            k = i & 1
            with torch.cuda.stream(s_in):
                s_in.wait_event(mm_done[k]) if i >= 2 else None  # buffer k's last reader finished
                a_d[k].copy_(a_p, non_blocking=True)
                bt_d[k].copy_(bt_p, non_blocking=True)
                in_done[k].record(s_in)
            with torch.cuda.stream(s_mm):
                s_mm.wait_event(in_done[k])
                if i >= 2:
                    s_mm.wait_event(out_done[k])  # out_d[k] downloaded
                kern(a_d[k], bt_d[k], out=out_d[k])
                mm_done[k].record(s_mm)
            with torch.cuda.stream(s_out):
                s_out.wait_event(mm_done[k])
                outs_p[k].copy_(out_d[k], non_blocking=True)
                out_done[k].record(s_out)

    run(4)
    torch.cuda.synchronize(dev)
    _barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    run(steps)
    s_in.wait_stream(s_out)
    e1.record(s_in)
    torch.cuda.synchronize(dev)
    _barrier(dist)
    return _max_over_ranks(e0.elapsed_time(e1) / steps, dist)


def run_ours(args):
    from icpp_tuning_b200 import _native as N
    from icpp_tuning_b200.autotuner.gpu_spec import get_gpu_spec
    from icpp_tuning_b200.gemm import gemm

    ws, rank, local, dist = _dist()
    dev = torch.device("cuda", local)
    a_h, bt_h = _inputs(1, rank)
    a, bt = a_h.to(dev), bt_h.to(dev)
    kern = gemm.build_kernel(M0, N0, K0, out_dtype=torch.bfloat16, b_layout="nk")
    out = torch.empty(M0, N0, dtype=torch.bfloat16, device=dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    flops = 2.0 * M0 * N0 * K0

    for _ in range(args.warmup):
        kern(a, bt, out=out)
    _barrier(dist)

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    launches0 = N.launch_count()
    with ClockSampler(local) as clk:
        _barrier(dist)
        for s, e in ev:
            flush.zero_()
            torch.cuda._sleep(QUEUE_PAD_CYCLES)
            s.record(stream)
            kern(a, bt, out=out)
            e.record(stream)
        _barrier(dist)
        launches = N.launch_count() - launches0
        dev_ms = sum(s.elapsed_time(e) for s, e in ev)
        # Keep the GPU busy a little longer if the timed region was too short for clock samples.
        t_end = time.time() + (0.0 if args.profile else max(0.0, 0.6 - dev_ms / 1e3))
        while time.time() < t_end:
            kern(a, bt, out=out)
        torch.cuda.synchronize()
    dev_ms_max = _max_over_ranks(dev_ms, dist)
    ms_step = dev_ms_max / args.steps
    value = flops * ws / (ms_step / 1e3) / 1e12

    if args.profile:
        if rank == 0:
            print(json.dumps({"profile_run": True, "ms_per_step": dev_ms / args.steps, "launches": launches}))
        return
    # End to end through the public callable with host buffers.  Every step copies its
    # inputs from pinned host memory and reads its result back inside the timed region;
    # steps are pipelined over three streams (copy-in, compute, copy-out) with two device
    # buffer sets, so step i+1's upload overlaps step i's multiply and download.
    e2e_ms = e2e_pipelined(kern, a_h, bt_h, out, dev, max(3, min(args.steps, 50)), dist)
    e2e = {"value": round(flops * ws / (e2e_ms / 1e3) / 1e12, 2), "unit": UNIT,
           "h2d_bytes_per_step": a_h.numel() * 2 + bt_h.numel() * 2, "d2h_bytes_per_step": out.numel() * 2,
           "ms_per_step": round(e2e_ms, 4), "pipelined": "h2d / compute / d2h on three streams, 2 buffer sets"}
    # host<->device traffic each rank sustains in that run (the 1 -> N e2e limit: all
    # ranks' copies share the host's memory system and PCIe root)
    e2e["host_copy_gbs_per_rank"] = round((e2e["h2d_bytes_per_step"] + e2e["d2h_bytes_per_step"]) / (e2e_ms / 1e3) / 1e9, 2)
    strong = strong_table(args, ws, rank, dist) if ws > 1 and not args.no_ops else None

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    peak, peak_sus, hbm, kind = _peaks()
    per_launch_ms = dev_ms / args.steps
    achieved = flops / (per_launch_ms / 1e3) / 1e12
    traffic = None
    prof = ROOT / "profiles" / "gemm_4096_bf16.md"  # committed ncu summary of this kernel
    if prof.exists():
        for line in prof.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                traffic = int(line.split(":", 1)[1])
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded randn, BASELINE configs[1] shapes)",
        "config": _config(ws),
        "tile": "BM%d_BN%d_BK%d_S%d_G%d" % (kern.config["block_M"], kern.config["block_N"],
                                             kern.config.get("block_K", 64), kern.config["num_stages"],
                                             kern.config.get("group_m", 0)),
        "e2e": e2e,
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": UNIT,
                     "frac": round(achieved / peak, 4), "peak_kind": f"{kind} bf16 burst (cuBLAS 8192^3)",
                     "traffic": traffic, "algorithmic_bytes": 3 * M0 * N0 * 2,
                     "frac_of_nominal_2250": round(achieved / 2250.0, 4)},
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "gpu": get_gpu_spec().name,
    }
    if ws == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(args, budget_s=args.cpu_budget)
    if ws == 1 and not args.no_ops:
        line["per_op"] = per_op_table(args)
    if strong is not None:
        line["strong"] = strong
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def cpu_rate(run, rows_total: int, flops_per_row: float, budget_s: float, steps: int, warmup: int):
    """TFLOP/s of `run(rows)` (the reference's CPU program on the first `rows` rows of a
    workload) on all host threads: one calibration call, then `warmup` untimed and `steps`
    timed calls on a row sample sized so that all of them fit `budget_s`; the median step.
    Both bench arms time the CPU path with this one function."""
    torch.set_num_threads(os.cpu_count() or 1)
    probe = max(1, min(rows_total, 64))
    t0 = time.perf_counter()
    run(probe)
    t_row = (time.perf_counter() - t0) / probe
    rows = int(max(probe, min(rows_total, budget_s / max(1, steps + warmup) / max(t_row, 1e-9))))
    for _ in range(warmup):
        run(rows)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run(rows)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    return flops_per_row * rows / dt / 1e12, rows, dt


def _cpu_config2(budget_s: float, steps: int, warmup: int) -> dict:
    """The reference's CPU program for the headline workload (oracle port of gemm.py:20-21
    with the bf16 output of configs[1])."""
    from oracle import ref_ops as R

    a, bt = _inputs(1, 0)
    v, rows, dt = cpu_rate(lambda r: R.gemm(a[:r], bt, "nk").to(torch.bfloat16), M0, 2.0 * N0 * K0,
                           budget_s, steps, warmup)
    return {"value": round(v, 4), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{rows} of {M0} rows of the 4096^3 bf16 GEMM per step, median of {steps} steps "
                      f"after {warmup} warm-up", "ms_per_step": round(dt * 1e3, 3), "cpu": _cpu_name()}


def cpu_baseline(args, budget_s: float = 20.0) -> dict:
    return _cpu_config2(budget_s, 3, 1)


def _cpu_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _g(seed):
    return torch.Generator().manual_seed(seed)


def host_inputs(key: str):
    """Seeded CPU inputs of one BASELINE workload, drawn in BASELINE.json's order."""
    if key == "config1":
        g = _g(0)
        a = (torch.rand(1024, 1024, generator=g) * 2 - 1).half()
        b = (torch.rand(1024, 1024, generator=g) * 2 - 1).half()
        return {"a": a, "b": b, "bias": (torch.randn(1024, generator=g) * 0.1).half()}
    if key == "config2":
        a, bt = _inputs(1, 0)
        return {"a": a, "b": bt}
    if key == "config3":
        g = _g(2)
        return {"a": torch.randn(8192, 4096, generator=g).bfloat16(),
                "b": (torch.randn(16384, 4096, generator=g) * 0.02).bfloat16(),
                "bias": (torch.randn(16384, generator=g) * 0.02).bfloat16()}
    if key == "config4":
        g = _g(3)
        return {"a": torch.randn(16384, 4096, generator=g).bfloat16(),
                "b": (torch.randn(4096, 4096, generator=g) / 64).bfloat16(),
                "bias": (torch.randn(4096, generator=g) * 0.02).bfloat16(),
                "gamma": (1 + torch.randn(4096, generator=g) * 0.02).bfloat16(),
                "beta": (torch.randn(4096, generator=g) * 0.02).bfloat16()}
    g = _g(4)
    return {"x": torch.randn(256, 28, 28, 128, generator=g).bfloat16(),
            "w": (torch.randn(3, 3, 128, 128, generator=g) / (9 * 128) ** 0.5).bfloat16(),
            "bias": (torch.randn(128, generator=g) * 0.1).bfloat16()}


# name, rows (GEMM M, or conv batch) of the global problem, FLOPs per row, shard alignment
WORKLOADS = {
    "config1": ("gemm_bias_relu 1024^3 fp16", 1024, 2.0 * 1024 * 1024, 128),
    "config2": ("gemm 4096^3 bf16", 4096, 2.0 * 4096 * 4096, 256),
    "config3": ("gemm_bias_gelu_tanh 8192x16384x4096 bf16", 8192, 2.0 * 16384 * 4096, 256),
    "config4": ("gemm_bias_layernorm 16384x4096x4096 bf16", 16384, 2.0 * 4096 * 4096, 256),
    "config5": ("conv2d_bias_relu 256x28x28x128->128 3x3 bf16", 256, 2.0 * 28 * 28 * 128 * 128 * 9, 1),
}


def build_workload(key: str, dev, lo: int = 0, hi: int = None, inputs=None, config=None):
    """Rows [lo, hi) of workload `key` on `dev` through the public operator modules:
    returns (step, out) where step() runs one call and writes out.  `config`: a raw tile
    config replacing the autotuner's pick (profiling runs)."""
    from icpp_tuning_b200.conv import conv2d_relu
    from icpp_tuning_b200.gemm import gemm, gemm_bias_act, gemm_bias_layernorm

    t = inputs if inputs is not None else host_inputs(key)
    hi = WORKLOADS[key][1] if hi is None else hi
    m = hi - lo
    if key == "config5":
        x = t["x"][lo:hi].contiguous().to(dev)
        wt, bias = t["w"].to(dev), t["bias"].to(dev)
        y = torch.empty(m, 28, 28, 128, dtype=torch.bfloat16, device=dev)
        k = conv2d_relu.build_conv2d_relu_kernel(m, 128, 28, 28, 128, 3, 3, 1, 1, 1, config=config)
        return (lambda: k(x, wt, y, bias=bias)), y
    a = t["a"][lo:hi].contiguous().to(dev)
    b = t["b"].to(dev)
    n, kk = (b.shape[1], b.shape[0]) if key == "config1" else (b.shape[0], b.shape[1])
    if key == "config1":
        bias = t["bias"].to(dev)
        k = gemm_bias_act.build_kernel(m, n, kk, config=config, act="relu", out_dtype=torch.float16)
        out = torch.empty(m, n, dtype=torch.float16, device=dev)
        return (lambda: k(a, b, bias, out=out)), out
    out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    if key == "config2":
        k = gemm.build_kernel(m, n, kk, config=config, out_dtype=torch.bfloat16, b_layout="nk")
        return (lambda: k(a, b, out=out)), out
    if key == "config3":
        bias = t["bias"].to(dev)
        k = gemm_bias_act.build_kernel(m, n, kk, config=config, act="gelu_tanh", out_dtype=torch.bfloat16, b_layout="nk")
        return (lambda: k(a, b, bias, out=out)), out
    bias, gam, bet = (t[x].to(dev) for x in ("bias", "gamma", "beta"))
    k = gemm_bias_layernorm.build_fused_kernel(m, n, kk, gemm_config=config, out_dtype=torch.bfloat16, b_layout="nk")
    return (lambda: k(a, b, bias, gam, bet, out=out)), out


def cpu_program(key: str, t: dict):
    """run(rows): the reference's CPU program (restated in oracle/ref_ops.py) on the first
    `rows` rows of workload `key`: gemm.py:20-21, gemm_bias_act.py:44-47 (+ GELU-tanh,
    end2end.py:37-38), gemm_bias_layernorm.py:44-50, conv2d_relu.py:29-60 (+ bias)."""
    from oracle import ref_ops as R

    if key == "config1":
        return lambda r: R.gemm_bias_act(t["a"][:r], t["b"], t["bias"], "relu").to(torch.float16)
    if key == "config2":
        return lambda r: R.gemm(t["a"][:r], t["b"], "nk").to(torch.bfloat16)
    if key == "config3":
        return lambda r: R.gemm_bias_act(t["a"][:r], t["b"], t["bias"], "gelu_tanh", b_layout="nk").to(torch.bfloat16)
    if key == "config4":
        return lambda r: R.gemm_bias_layernorm(t["a"][:r], t["b"], t["bias"], t["gamma"], t["beta"],
                                               b_layout="nk", out_dtype=torch.bfloat16)
    return lambda r: R.conv2d_bias_relu(t["x"][:r], t["w"], t["bias"], out_dtype=torch.bfloat16)


def time_steps(fn, steps: int, flush) -> float:
    """Mean device ms of fn over `steps`, L2 flushed and the queue padded before each."""
    tot = 0.0
    for _ in range(steps):
        flush.zero_()
        torch.cuda._sleep(QUEUE_PAD_CYCLES)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        tot += s.elapsed_time(e)
    return tot / steps


def per_op_table(args) -> list:
    """Device-timed TFLOP/s of all five BASELINE workloads (config2 is the headline), each
    beside the reference's CPU program on the same inputs (bounded row sample)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    peak = _peaks()[0]
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    steps = max(5, min(args.steps, 20))
    res = []
    for key, (name, rows, fpr, _) in WORKLOADS.items():
        t = host_inputs(key)
        fn, _out = build_workload(key, dev, inputs=t)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ms = time_steps(fn, steps, flush)
        tf = fpr * rows / (ms / 1e3) / 1e12
        row = {"op": f"{key} {name}", "ms": round(ms, 5), "tflops": round(tf, 2),
               "frac_measured": round(tf / peak, 4), "frac_nominal": round(tf / 2250.0, 4)}
        if not args.no_cpu:
            cv, crows, _ = cpu_rate(cpu_program(key, t), rows, fpr, args.cpu_budget / 5, 3, 1)
            row.update({"cpu_tflops": round(cv, 4), "cpu_sample_rows": crows, "gpu_over_cpu": round(tf / cv, 1)})
        res.append(row)
        del fn, _out
        torch.cuda.empty_cache()
    return res


def strong_table(args, ws: int, rank: int, dist) -> list:
    """Strong scaling (N > 1): each fixed global workload split into contiguous row (or
    image) shards, one per rank, weights replicated, no collective on the data path.
    Throughput = global FLOPs / the max over ranks of the per-shard device time.  The
    NCCL all-gather that assembles the whole output on every rank (shard.gather_rows) is
    timed separately."""
    from icpp_tuning_b200 import shard

    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    steps = max(5, min(args.steps, 20))
    res = []
    for key, (name, rows, fpr, align) in WORKLOADS.items():
        lo, hi = shard.row_shard(rows, ws, rank, align)
        fn, out = build_workload(key, dev, lo, hi)
        for _ in range(3):
            fn()
        _barrier(dist)
        ms = _max_over_ranks(time_steps(fn, steps, flush), dist)
        tf = fpr * rows / (ms / 1e3) / 1e12
        entry = {"op": f"{key} {name}", "global_rows": rows, "rows_per_rank": hi - lo, "ms": round(ms, 5),
                 "tflops": round(tf, 2)}
        flat = out.reshape(out.shape[0], -1)
        whole = torch.empty((rows, flat.shape[1]), dtype=flat.dtype, device=dev)
        shard.gather_rows(flat, rows, out=whole)  # NCCL communicator set-up outside the timing
        _barrier(dist)
        g_ms = _max_over_ranks(time_steps(lambda: shard.gather_rows(flat, rows, out=whole), 5, flush), dist)
        entry["allgather_ms"] = round(g_ms, 4)
        entry["allgather_bytes"] = rows * flat.shape[1] * flat.element_size()
        entry["allgather_gbs"] = round(entry["allgather_bytes"] / (g_ms / 1e3) / 1e9, 1)
        res.append(entry)
        del fn, out, flat, whole
        torch.cuda.empty_cache()
    return res


def _tile_arg(args):
    """--tile BM,BN,BK,STAGES,GROUP[,key=value...] -> a raw config dict (None: autotuner)."""
    if not args.tile:
        return None
    f = args.tile.split(",")
    c = {"block_M": int(f[0]), "block_N": int(f[1]), "block_K": int(f[2]), "num_stages": int(f[3]),
         "group_m": int(f[4]), "thread_num": 320}
    for kv in f[5:]:
        k, v = kv.split("=")
        c[k] = int(v)
    return c


def profile_op(args):
    """--profile --op configN: W warm-up steps then K timed steps of one workload, for ncu."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    name, rows, fpr, _ = WORKLOADS[args.op]
    fn, _out = build_workload(args.op, dev, config=_tile_arg(args))
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    ms = time_steps(fn, args.steps, flush)
    print(json.dumps({"profile_run": args.op, "workload": name, "ms": ms, "tflops": fpr * rows / (ms / 1e3) / 1e12}))


def _config(ws: int) -> dict:
    """The workload description both arms print (the driver compares them)."""
    return {"workload": WORKLOAD, "parallelism": f"M-shard x{ws} (weak: 4096 rows per GPU)",
            "l2": "flushed between timed steps (256 MiB write outside the events)"}


def run_reference(args):
    """The reference's CPU implementation of the path (its PyTorch program, restated in
    oracle/ref_ops.py) on the host cores, same metric and workload, bounded samples."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cb = _cpu_config2(min(120.0, 3.0 * (args.steps + args.warmup)), args.steps, args.warmup)
    v = cb["value"]
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded randn, BASELINE configs[1] shapes)", "impl": "reference",
            "config": _config(ws), "cpu_baseline": cb,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-op table of all five workloads")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--op", default="config2", choices=["config1", "config2", "config3", "config4", "config5"],
                    help="with --profile: the workload to run")
    ap.add_argument("--tile", default="", help="with --profile: BM,BN,BK,STAGES,GROUP[,ln_mode=1,swap_ab=2,...]")
    ap.add_argument("--profile", action="store_true",
                    help="timed steps only (no e2e, CPU baseline, per-op table or clock hold): for ncu")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.profile and args.op != "config2":
        profile_op(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
