"""Formula-selected kernels against PyTorch over the reference's evaluation sweeps.

The reference keeps the outputs of these runs (evaluation/gemm_formula_full.csv,
gemm_bias_act_formula_full.csv, gemm_bias_layernorm_formula_full.csv,
gemm_three_ops_formula_summary.csv, gemm_three_ops_formula_report.md,
conv2d_formula_changed_after_costmodel.csv) but not the scripts that wrote them.  This
module rewrites them for the B200 operators with the same CSV columns:

  op,M,N,K,config,runtime_config,score,formula_ms,torch_ms,speedup
  Index,N,C,H,W,F_out,Kernel_H,Kernel_W,Stride,Pad,Formula_Config,Formula_Score,
      Formula_Latency_ms,Torch_Latency_ms,Speedup_vs_Torch,Is_Correct

For each shape the formula's top-1 config (`select_best`) is built and timed; `config` is
the formula's choice, `runtime_config` the config the launched kernel ran with (the
same: no runtime re-tuning happens here).  GEMM sweep: M = 1..126 step 5, N = 2304,
K = 768, fp16 (the reference's sweep, gemm_three_ops_formula_report.md:3-4).  Conv: the
nine shapes of the reference's conv CSV.

Torch baselines are each reference script's own (`--torch-baseline reference`):
gemm -> torch.mm(a.float(), b.float()) with TF32 off (gemm.py:146-149), gemm_bias_act
-> relu((A@B).float() + bias) (gemm_bias_act.py:44-47, eager here), gemm_bias_layernorm
-> torch_baseline (gemm_bias_layernorm.py:44-50), conv -> F.conv2d on permuted NHWC
tensors (conv2d.py:35-62).  `--torch-baseline native` times the same results computed
the fast way in PyTorch (fp16 cuBLAS matmul, fused addmm, F.layer_norm), the stronger
comparison.

Timing follows triton.testing.do_bench, which the reference scripts used: before every
repetition a 256 MiB buffer is zeroed (flushing the 126 MB L2, and keeping the GPU busy
while the host enqueues the timed call), then CUDA events bracket the call on the
current stream.  The reported figure is the median (do_bench defaults to the mean; one
preempted repetition can double a mean of 10-us kernels).

    python -m icpp_tuning_b200.formula_bench --op all --csv-dir out/ --report out/report.md
"""
from __future__ import annotations

import argparse
import csv
import statistics
from pathlib import Path
from typing import Callable, Dict, List, Sequence

import torch
import torch.nn.functional as F

from .autotuner.interface import select_best
from .conv import conv2d as conv_mod
from .gemm import gemm as gemm_mod
from .gemm import gemm_bias_act, gemm_bias_layernorm

GEMM_FIELDS = ["op", "M", "N", "K", "config", "runtime_config", "score", "formula_ms", "torch_ms", "speedup"]
CONV_FIELDS = ["Index", "N", "C", "H", "W", "F_out", "Kernel_H", "Kernel_W", "Stride", "Pad", "Formula_Config",
               "Formula_Score", "Formula_Latency_ms", "Torch_Latency_ms", "Speedup_vs_Torch", "Is_Correct"]
GEMM_OPS = ("gemm", "gemm_bias_act", "gemm_bias_layernorm")
# (N, C, H, W, F_out, KH, KW, stride, pad): the shapes of the reference's conv evaluation
CONV_SHAPES = [(4, 64, 224, 224, 64, 3, 3, 1, 1), (8, 64, 224, 224, 64, 3, 3, 1, 1),
               (12, 64, 112, 112, 64, 3, 3, 1, 1), (20, 64, 224, 224, 64, 3, 3, 1, 1),
               (20, 512, 14, 14, 512, 3, 3, 1, 1), (24, 256, 28, 28, 512, 3, 3, 1, 1),
               (32, 64, 56, 56, 192, 3, 3, 1, 1), (36, 512, 28, 28, 512, 3, 3, 1, 1),
               (60, 64, 112, 112, 64, 3, 3, 1, 1)]


def do_bench(fn: Callable[[], object], warmup: int = 25, rep: int = 100) -> float:
    """Median device time of fn() in ms, L2 flushed before each repetition."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(rep)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(rep)]
    for i in range(rep):
        flush.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return statistics.median(s.elapsed_time(e) for s, e in zip(starts, ends))


def _gemm_case(op: str, M: int, N: int, K: int, baseline: str, g: torch.Generator):
    """(formula callable, torch callable, descriptor, config, score, check) for one shape."""
    dev = "cuda"
    a = torch.randn(M, K, generator=g).half().to(dev)
    b = torch.randn(K, N, generator=g).half().to(dev)
    bias = torch.randn(N, generator=g).half().to(dev)
    if op == "gemm":
        desc = gemm_mod.DESCRIPTOR
        cfg, score = select_best(desc, M=M, N=N, K=K, out_bytes=4)
        kern = gemm_mod.build_kernel(M, N, K, config=cfg)
        ours = lambda: kern(a, b)
        if baseline == "reference":
            theirs = lambda: torch.mm(a.float(), b.float())
        else:
            theirs = lambda: torch.mm(a, b).float()
    elif op == "gemm_bias_act":
        desc = gemm_bias_act.DESCRIPTOR
        cfg, score = select_best(desc, M=M, N=N, K=K, out_bytes=4)
        kern = gemm_bias_act.build_kernel(M, N, K, config=cfg)
        ours = lambda: kern(a, b, bias)
        if baseline == "reference":
            theirs = lambda: gemm_bias_act.ref_program(a, b, bias)
        else:
            theirs = lambda: torch.relu(torch.addmm(bias, a, b)).float()
    elif op == "gemm_bias_layernorm":
        gamma = torch.randn(N, generator=g).half().to(dev)
        beta = torch.randn(N, generator=g).half().to(dev)
        desc = gemm_bias_layernorm.DESCRIPTOR
        cfg, score = select_best(desc, M=M, N=N, K=K)
        kern = gemm_bias_layernorm.build_fused_kernel(M, N, K, gemm_config=cfg)
        ours = lambda: kern(a, b, bias, gamma, beta)
        if baseline == "reference":
            theirs = lambda: gemm_bias_layernorm.torch_baseline(a, b, bias, gamma, beta)
        else:
            theirs = lambda: F.layer_norm(torch.addmm(bias, a, b), (N,), gamma, beta)
    else:
        raise ValueError(op)
    # A baseline computed in the input dtype can round differently; the reference's
    # own check is allclose(rtol=atol=1e-2) against its fp32-accumulated function.
    check = lambda: torch.allclose(ours().float(), theirs().float(), rtol=1e-2, atol=5e-2)
    return ours, theirs, desc, cfg, score, check


def run_gemm_sweep(op: str, Ms: Sequence[int], N: int = 2304, K: int = 768, baseline: str = "reference",
                   warmup: int = 25, rep: int = 100, log=print) -> List[Dict[str, object]]:
    rows = []
    g = torch.Generator().manual_seed(0)
    for M in Ms:
        ours, theirs, desc, cfg, score, check = _gemm_case(op, M, N, K, baseline, g)
        cfg_str = desc.format_config(cfg)
        t_ours = do_bench(ours, warmup, rep)
        t_torch = do_bench(theirs, warmup, rep)
        ok = check()
        log(f"{op} M={M} N={N} K={K}  {cfg_str} score={score:.6f}  formula {t_ours:.4f} ms  "
            f"torch {t_torch:.4f} ms  speedup {t_torch / t_ours:.4f}x  correct={ok}")
        if not ok:
            raise RuntimeError(f"{op} M={M}: formula kernel disagrees with the torch baseline")
        rows.append({"op": op, "M": M, "N": N, "K": K, "config": cfg_str, "runtime_config": cfg_str,
                     "score": f"{score:.6f}", "formula_ms": f"{t_ours:.4f}", "torch_ms": f"{t_torch:.4f}",
                     "speedup": f"{t_torch / t_ours:.4f}"})
    return rows


CONV_OPS = ("conv2d", "conv2d_bn_relu", "conv_bn_add_relu")


def _conv_case(op, N, C, H, W, Fo, KH, KW, S, P, baseline, g):
    """(ours, theirs, check, descriptor, config, score) for one conv shape of `op`.  The
    BatchNorm ops follow their reference checks (conv2d_bn_relu.py:293-316,
    conv_bn_add_relu.py:188-216): randn gamma / beta / mean, var = rand + 0.5."""
    from .conv import conv2d_bn_relu, conv_bn_add_relu

    X = torch.randn(N, H, W, C, generator=g).half().cuda()
    Wt = (torch.randn(KH, KW, C, Fo, generator=g) / (KH * KW * C) ** 0.5).half().cuda()
    mod = {"conv2d": conv_mod, "conv2d_bn_relu": conv2d_bn_relu, "conv_bn_add_relu": conv_bn_add_relu}[op]
    cfg, score = select_best(mod.DESCRIPTOR, N=N, C=C, H=H, W=W, OC=Fo, KH=KH, KW=KW, stride=S, padding=P)
    OH, OW = conv_mod.calc_oh_ow(H, W, KH, KW, S, P, 1)
    Y = torch.empty(N, OH, OW, Fo, dtype=torch.float16, device="cuda")
    Yr = torch.empty_like(Y)
    ref = mod.get_ref_program(S, P, 1)
    Xc = X.permute(0, 3, 1, 2)
    Wc = Wt.permute(3, 2, 0, 1).contiguous(memory_format=torch.channels_last)
    if op == "conv2d":
        kern = conv_mod.build_conv2d_kernel(N, C, H, W, Fo, KH, KW, S, P, config=cfg)
        ours, run_ref = (lambda: kern(X, Wt, Y)), (lambda: ref(X, Wt, Yr))
        native = lambda: F.conv2d(Xc, Wc, stride=S, padding=P)
    else:
        gamma, beta, mean = (torch.randn(Fo, generator=g).half().cuda() for _ in range(3))
        var = (torch.rand(Fo, generator=g) + 0.5).half().cuda()
        eps = mod.EPS
        scale = (gamma.float() * torch.rsqrt(var.float() + eps)).view(1, -1, 1, 1)
        shift = (beta.float() - mean.float() * scale.view(-1)).view(1, -1, 1, 1)
        if op == "conv2d_bn_relu":
            kern = conv2d_bn_relu.build_conv2d_bn_relu_kernel(N, C, H, W, Fo, KH, KW, S, P, config=cfg)
            ours = lambda: kern(X, Wt, gamma, beta, mean, var, Y)
            run_ref = lambda: ref(X, Wt, gamma, beta, mean, var, Yr)
            native = lambda: torch.relu(F.conv2d(Xc, Wc, stride=S, padding=P) * scale + shift)
        else:
            res = torch.randn(N, OH, OW, Fo, generator=g).half().cuda()
            resc = res.permute(0, 3, 1, 2)
            kern = conv_bn_add_relu.build_conv2d_bn_add_relu_kernel(N, C, H, W, Fo, KH, KW, S, P, config=cfg)
            ours = lambda: kern(X, Wt, res, gamma, beta, mean, var, Y)
            run_ref = lambda: ref(X, Wt, res, gamma, beta, mean, var, Yr)
            native = lambda: torch.relu(F.conv2d(Xc, Wc, stride=S, padding=P) * scale + shift + resc)

    def check():
        ours()
        run_ref()
        return bool(torch.allclose(Y.float(), Yr.float(), rtol=1e-2, atol=1e-2))

    return ours, (run_ref if baseline == "reference" else native), check, mod.DESCRIPTOR, cfg, score


def run_conv_sweep(shapes=CONV_SHAPES, baseline: str = "reference", warmup: int = 10, rep: int = 50,
                   log=print, op: str = "conv2d") -> List[Dict[str, object]]:
    """`native` baselines: cuDNN on channels-last views (no permute copies) plus the
    BatchNorm / residual / ReLU as PyTorch elementwise ops."""
    rows = []
    g = torch.Generator().manual_seed(0)
    for idx, (N, C, H, W, Fo, KH, KW, S, P) in enumerate(shapes, 1):
        ours, theirs, check, desc, cfg, score = _conv_case(op, N, C, H, W, Fo, KH, KW, S, P, baseline, g)
        t_ours = do_bench(ours, warmup, rep)
        t_torch = do_bench(theirs, warmup, rep)
        ok = check()
        cfg_str = desc.format_config(cfg)
        log(f"{op} [{idx}] N={N} C={C} H={H} W={W} F={Fo} {KH}x{KW} s{S} p{P}  {cfg_str}  formula {t_ours:.4f} ms  "
            f"torch {t_torch:.4f} ms  speedup {t_torch / t_ours:.4f}x  correct={ok}")
        rows.append({"Index": idx, "N": N, "C": C, "H": H, "W": W, "F_out": Fo, "Kernel_H": KH, "Kernel_W": KW,
                     "Stride": S, "Pad": P, "Formula_Config": cfg_str, "Formula_Score": f"{score:.6f}",
                     "Formula_Latency_ms": f"{t_ours:.4f}", "Torch_Latency_ms": f"{t_torch:.4f}",
                     "Speedup_vs_Torch": f"{t_torch / t_ours:.4f}", "Is_Correct": str(ok)})
    return rows


def write_csv(path: Path, fields: Sequence[str], rows: Sequence[Dict[str, object]]) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(fields))
        w.writeheader()
        w.writerows(rows)


def summarize(rows: Sequence[Dict[str, object]], worst: int = 5) -> str:
    """Markdown summary in the layout of the reference's gemm_three_ops_formula_report.md:
    per-op speedup statistics, then the slowest shapes of each op."""
    out = ["| op | shapes | min speedup | median | mean | max | slower than torch | near baseline (<1.1x) |",
           "|---|---:|---:|---:|---:|---:|---:|---:|"]
    ops = sorted({str(r["op"]) for r in rows}, key=lambda o: GEMM_OPS.index(o) if o in GEMM_OPS else 99)
    for op in ops:
        sp = [float(r["speedup"]) for r in rows if r["op"] == op]
        out.append(f"| `{op}` | {len(sp)} | {min(sp):.4f} | {statistics.median(sp):.4f} | {statistics.fmean(sp):.4f} "
                   f"| {max(sp):.4f} | {sum(s < 1 for s in sp)} | {sum(1 <= s < 1.1 for s in sp)} |")
    for op in ops:
        sel = sorted((r for r in rows if r["op"] == op), key=lambda r: float(r["speedup"]))[:worst]
        out += ["", f"### {op}", "", "| M | config | formula ms | torch ms | speedup |", "|---:|---|---:|---:|---:|"]
        out += [f"| {r['M']} | `{r['config']}` | {r['formula_ms']} | {r['torch_ms']} | {r['speedup']} |" for r in sel]
    return "\n".join(out) + "\n"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="formula top-1 kernels vs torch over the reference's sweeps")
    ap.add_argument("--op", default="all", choices=("all",) + CONV_OPS + GEMM_OPS)
    ap.add_argument("--m-start", type=int, default=1)
    ap.add_argument("--m-stop", type=int, default=128)
    ap.add_argument("--m-step", type=int, default=5)
    ap.add_argument("--N", type=int, default=2304)
    ap.add_argument("--K", type=int, default=768)
    ap.add_argument("--torch-baseline", default="reference", choices=("reference", "native"))
    ap.add_argument("--warmup", type=int, default=25)
    ap.add_argument("--rep", type=int, default=100)
    ap.add_argument("--csv-dir", default="formula_results")
    ap.add_argument("--report", default=None, help="write a markdown summary of the GEMM sweeps here")
    args = ap.parse_args(argv)
    torch.backends.cuda.matmul.allow_tf32 = False  # as the reference scripts (gemm_bias_act.py:17)
    out = Path(args.csv_dir)
    Ms = list(range(args.m_start, args.m_stop, args.m_step))
    print(f"GPU: {torch.cuda.get_device_name(0)}  torch baseline: {args.torch_baseline}")
    all_rows = []
    for op in GEMM_OPS:
        if args.op in ("all", op):
            rows = run_gemm_sweep(op, Ms, args.N, args.K, args.torch_baseline, args.warmup, args.rep)
            write_csv(out / f"{op}_formula_full.csv", GEMM_FIELDS, rows)
            all_rows += rows
    if all_rows:
        write_csv(out / "gemm_three_ops_formula_summary.csv", GEMM_FIELDS, all_rows)
        if args.report:
            Path(args.report).write_text(summarize(all_rows))
    for op in CONV_OPS:
        if args.op in ("all", op):
            write_csv(out / f"{op}_formula.csv", CONV_FIELDS, run_conv_sweep(baseline=args.torch_baseline, op=op))


if __name__ == "__main__":
    main()
