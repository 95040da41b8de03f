"""Benchmark of the fused dense-operator path on B200.

One step = one call of the headline operator over one batch of synthetic input:
BASELINE configs[1], plain GEMM M=N=K=4096, bf16 A (row-major) and B (column-major),
fp32 accumulate, bf16 out, seed 1.  `value` is device time (CUDA events on the launching
stream, L2 flushed between steps by a 256 MiB write outside the events), `e2e` is the
same metric through the public API (icpp_tuning_b200.gemm.gemm.build_kernel) with the
step's inputs copied from pinned host memory and the result read back inside the timed
region.  At N>1 (torchrun, NCCL) every rank owns one 4096-row shard of a global
M = 4096*N problem (weak scaling, no collective on the data path); times are the max
over ranks.  Rank 0 prints one JSON line.

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
        "config": {"workload": WORKLOAD, "parallelism": f"M-shard x{ws} (weak: 4096 rows per GPU)",
                   "tile": "BM%d_BN%d_BK%d_S%d_G%d" % (kern.config["block_M"], kern.config["block_N"],
                                                        kern.config.get("block_K", 64), kern.config["num_stages"],
                                                        kern.config.get("group_m", 0)),
                   "l2": "flushed between timed steps (256 MiB write outside the events)"},
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
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def cpu_baseline(args, budget_s: float = 20.0) -> dict:
    """The reference's CPU program for the workload (oracle port of gemm.py:20-21 with the
    bf16 output of configs[1]) on all host cores, on a bounded row sample."""
    from oracle import ref_ops as R

    torch.set_num_threads(os.cpu_count() or 1)
    a, bt = _inputs(1, 0)
    t0 = time.perf_counter()
    R.gemm(a[:512], bt, "nk").to(torch.bfloat16)
    t_full = (time.perf_counter() - t0) * M0 / 512
    rows = M0 if 3 * t_full <= budget_s else 512
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        R.gemm(a[:rows], bt, "nk").to(torch.bfloat16)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    return {"value": round(2.0 * rows * N0 * K0 / dt / 1e12, 4), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{rows} of {M0} rows of the 4096^3 bf16 GEMM, median of {len(times)}",
            "cpu": _cpu_name()}


def _cpu_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def workloads(dev) -> dict:
    """The five BASELINE workloads: name -> (builder, FLOPs).  A builder allocates the
    seeded inputs on `dev` and returns a zero-argument callable running one step."""
    from icpp_tuning_b200.conv import conv2d_relu
    from icpp_tuning_b200.gemm import gemm, gemm_bias_act, gemm_bias_layernorm

    def c1():
        g = torch.Generator().manual_seed(0)
        a = (torch.rand(1024, 1024, generator=g) * 2 - 1).half().to(dev)
        b = (torch.rand(1024, 1024, generator=g) * 2 - 1).half().to(dev)
        bias = (torch.randn(1024, generator=g) * 0.1).half().to(dev)
        k = gemm_bias_act.build_kernel(1024, 1024, 1024, act="relu", out_dtype=torch.float16)
        return lambda: k(a, b, bias)

    def c2():
        a, bt = (t.to(dev) for t in _inputs(1, 0))
        k = gemm.build_kernel(4096, 4096, 4096, out_dtype=torch.bfloat16, b_layout="nk")
        return lambda: k(a, bt)

    def c3():
        g = torch.Generator().manual_seed(2)
        x = torch.randn(8192, 4096, generator=g).bfloat16().to(dev)
        w = (torch.randn(16384, 4096, generator=g) * 0.02).bfloat16().to(dev)
        bias = (torch.randn(16384, generator=g) * 0.02).bfloat16().to(dev)
        k = gemm_bias_act.build_kernel(8192, 16384, 4096, act="gelu_tanh", out_dtype=torch.bfloat16, b_layout="nk")
        return lambda: k(x, w, bias)

    def c4():
        g = torch.Generator().manual_seed(3)
        x = torch.randn(16384, 4096, generator=g).bfloat16().to(dev)
        w = (torch.randn(4096, 4096, generator=g) / 64).bfloat16().to(dev)
        bias = (torch.randn(4096, generator=g) * 0.02).bfloat16().to(dev)
        gam = (1 + torch.randn(4096, generator=g) * 0.02).bfloat16().to(dev)
        bet = (torch.randn(4096, generator=g) * 0.02).bfloat16().to(dev)
        k = gemm_bias_layernorm.build_fused_kernel(16384, 4096, 4096, out_dtype=torch.bfloat16, b_layout="nk")
        return lambda: k(x, w, bias, gam, bet)

    def c5():
        g = torch.Generator().manual_seed(4)
        x = torch.randn(256, 28, 28, 128, generator=g).bfloat16().to(dev)
        wt = (torch.randn(3, 3, 128, 128, generator=g) / (9 * 128) ** 0.5).bfloat16().to(dev)
        bias = (torch.randn(128, generator=g) * 0.1).bfloat16().to(dev)
        y = torch.empty(256, 28, 28, 128, dtype=torch.bfloat16, device=dev)
        k = conv2d_relu.build_conv2d_relu_kernel(256, 128, 28, 28, 128, 3, 3, 1, 1, 1)
        return lambda: k(x, wt, y, bias=bias)

    return {
        "config1": ("gemm_bias_relu 1024^3 fp16", c1, 2.0 * 1024 ** 3),
        "config2": ("gemm 4096^3 bf16", c2, 2.0 * 4096 ** 3),
        "config3": ("gemm_bias_gelu_tanh 8192x16384x4096 bf16", c3, 2.0 * 8192 * 16384 * 4096),
        "config4": ("gemm_bias_layernorm 16384x4096x4096 bf16", c4, 2.0 * 16384 * 4096 * 4096),
        "config5": ("conv2d_bias_relu 256x28x28x128->128 3x3 bf16", c5, 2.0 * 256 * 28 * 28 * 128 * 128 * 9),
    }


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
    """Device-timed TFLOP/s of all five BASELINE workloads (config2 is the headline)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    peak = _peaks()[0]
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    steps = max(5, min(args.steps, 20))
    res = []
    for key, (name, build, flops) in workloads(dev).items():
        fn = build()
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ms = time_steps(fn, steps, flush)
        tf = flops / (ms / 1e3) / 1e12
        res.append({"op": f"{key} {name}", "ms": round(ms, 5), "tflops": round(tf, 2),
                    "frac_measured": round(tf / peak, 4), "frac_nominal": round(tf / 2250.0, 4)})
        del fn
        torch.cuda.empty_cache()
    return res


def profile_op(args):
    """--profile --op configN: W warm-up steps then K timed steps of one workload, for ncu."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    name, build, flops = workloads(dev)[args.op]
    fn = build()
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    ms = time_steps(fn, args.steps, flush)
    print(json.dumps({"profile_run": args.op, "workload": name, "ms": ms, "tflops": flops / (ms / 1e3) / 1e12}))


def run_reference(args):
    """The reference's CPU implementation of the path (its PyTorch program, restated in
    oracle/ref_ops.py) on the host cores, same metric and workload, bounded samples."""
    from oracle import ref_ops as R

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    a, bt = _inputs(1, 0)
    t0 = time.perf_counter()
    R.gemm(a[:256], bt, "nk").to(torch.bfloat16)
    t_row = (time.perf_counter() - t0) / 256
    budget = 120.0
    rows = int(max(64, min(M0, budget / max(1, args.steps + args.warmup) / max(t_row, 1e-9))))
    for _ in range(args.warmup):
        R.gemm(a[:rows], bt, "nk").to(torch.bfloat16)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        R.gemm(a[:rows], bt, "nk").to(torch.bfloat16)
    dt = (time.perf_counter() - t0) / args.steps
    v = round(2.0 * rows * N0 * K0 / dt / 1e12, 4)
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded randn, BASELINE configs[1] shapes)", "impl": "reference",
            "config": {"workload": WORKLOAD, "parallelism": "host CPU, rank 0 only"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"{rows} of {M0} rows per step", "cpu": _cpu_name()},
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
