"""Decision table: the measured level of the two-level config selector.

The reference's design (docs/autotuner_design.md:472-525) describes, but never
implements, an offline profiling pass whose results become a decision table, and an
online `AdaptiveTuner.select` that looks the shape up in the table (level "table") and
falls back to the analytical formula (level "formula") for shapes the table does not
cover.  This module implements both:

  build_sampling_plan  shapes to profile (wave-stratified M for GEMMs, batch for conv)
  profile              times every (shape, config) pair with a timer callable
  build_decision_table groups measurements by the non-M shape keys ((N, K) for GEMMs),
                       keeps the fastest config per profiled M and merges neighbouring
                       M points with the same winner into intervals
  DecisionTable        lookup(shape) -> config for an M inside a group's profiled range
                       (the nearest profiled M decides), JSON save / load
  AdaptiveTuner        select(**shape) -> SelectResult(config, level, score)
  gpu_timer            the timer that runs this package's kernels (needs a GPU)

    python -m icpp_tuning_b200.autotuner.decision_table --op gemm --out gemm_table.json
"""
from __future__ import annotations

import argparse
import bisect
import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

from .interface import TileLangKernelBase, rank_all

GEMM_GROUP = ("N", "K")
CONV_GROUP = ("C", "H", "W", "OC", "KH", "KW", "stride", "padding")


def _is_conv(shape: Dict[str, Any]) -> bool:
    return "M" not in shape


def _axis(shape: Dict[str, Any]) -> str:
    """The profiled axis: GEMM rows M, or the conv batch N."""
    return "N" if _is_conv(shape) else "M"


def _group(shape: Dict[str, Any]) -> Tuple:
    keys = CONV_GROUP if _is_conv(shape) else GEMM_GROUP
    return tuple(int(shape[k]) for k in keys)


def _cfg_key(cfg: Dict[str, Any]) -> str:
    return json.dumps(cfg, sort_keys=True)


@dataclass
class Measurement:
    shape: Dict[str, Any]
    config: Dict[str, Any]
    ms: float


@dataclass
class SelectResult:
    config: Dict[str, Any]
    level: str            # "table" or "formula"
    score: Optional[float]  # formula score of the chosen config (None for table hits)


class DecisionTable:
    """Per shape group, the profiled axis points (sorted) and the fastest config at each;
    `intervals(group)` shows the merged [lo, hi] -> config runs."""

    def __init__(self, op: str, groups: Dict[Tuple, List[Tuple[int, Dict[str, Any], float]]]):
        self.op = op
        self.groups = {g: sorted(pts, key=lambda t: t[0]) for g, pts in groups.items()}

    def lookup(self, **shape) -> Optional[Dict[str, Any]]:
        pts = self.groups.get(_group(shape))
        if not pts:
            return None
        m = int(shape[_axis(shape)])
        ms = [p[0] for p in pts]
        if m < ms[0] or m > ms[-1]:
            return None  # outside the profiled range: the formula decides
        i = bisect.bisect_left(ms, m)
        if i < len(ms) and ms[i] == m:
            return dict(pts[i][1])
        lo, hi = pts[i - 1], pts[i]
        return dict(lo[1] if m - lo[0] <= hi[0] - m else hi[1])

    def intervals(self, group: Tuple) -> List[Tuple[int, int, Dict[str, Any]]]:
        out: List[Tuple[int, int, Dict[str, Any]]] = []
        for m, cfg, _ in self.groups.get(group, []):
            if out and _cfg_key(out[-1][2]) == _cfg_key(cfg):
                out[-1] = (out[-1][0], m, out[-1][2])
            else:
                out.append((m, m, cfg))
        return out

    def to_json(self) -> str:
        return json.dumps({"op": self.op, "groups": [
            {"group": list(g), "points": [{"m": m, "config": c, "ms": t} for m, c, t in pts]}
            for g, pts in sorted(self.groups.items())]}, indent=1)

    @classmethod
    def from_json(cls, text: str) -> "DecisionTable":
        d = json.loads(text)
        return cls(d["op"], {tuple(e["group"]): [(p["m"], p["config"], p["ms"]) for p in e["points"]]
                             for e in d["groups"]})

    def save(self, path) -> None:
        Path(path).write_text(self.to_json())

    @classmethod
    def load(cls, path) -> "DecisionTable":
        return cls.from_json(Path(path).read_text())


def build_decision_table(op: str, measurements: Sequence[Measurement]) -> DecisionTable:
    """The fastest measured config per (group, axis point); failed timings (ms None or
    not finite) are skipped."""
    best: Dict[Tuple, Dict[int, Tuple[Dict[str, Any], float]]] = {}
    for r in measurements:
        if r.ms is None or not (r.ms == r.ms) or r.ms == float("inf"):
            continue
        g, m = _group(r.shape), int(r.shape[_axis(r.shape)])
        cur = best.setdefault(g, {}).get(m)
        if cur is None or r.ms < cur[1]:
            best[g][m] = (dict(r.config), float(r.ms))
    return DecisionTable(op, {g: [(m, c, t) for m, (c, t) in pts.items()] for g, pts in best.items()})


def build_sampling_plan(op: str, m_points: Optional[Sequence[int]] = None,
                        nk: Sequence[Tuple[int, int]] = ((2304, 768), (768, 768), (4096, 4096))) -> List[Dict]:
    """GEMM shapes: M stratified by how the tile grid fills the 148 SMs (dense where the
    wave count changes fastest, at small M), for each (N, K).  Conv: batch 1..64 over a
    few layer geometries."""
    if op.startswith("conv"):
        geoms = [(64, 56, 56, 64), (128, 28, 28, 128), (256, 14, 14, 256), (512, 7, 7, 512)]
        return [{"N": n, "C": c, "H": h, "W": w, "OC": f, "KH": 3, "KW": 3, "stride": 1, "padding": 1}
                for c, h, w, f in geoms for n in (m_points or (1, 2, 4, 8, 16, 32, 64))]
    ms = list(m_points or (1, 16, 64, 128, 256, 512, 1024, 2048, 4096, 8192))
    return [{"M": m, "N": n, "K": k} for n, k in nk for m in ms]


def candidate_configs(descriptor: TileLangKernelBase, shapes: Sequence[Dict], top_k: int = 6) -> List[Dict]:
    """Union over the shapes of the formula's top_k configs: the profiled pool (the
    formula prunes, the measurement decides)."""
    seen, out = set(), []
    for sh in shapes:
        for r in rank_all(descriptor, **sh)[:top_k]:
            k = _cfg_key(r["raw_config"])
            if k not in seen:
                seen.add(k)
                out.append(dict(r["raw_config"]))
    return out


def profile(shapes: Sequence[Dict], configs: Sequence[Dict],
            timer: Callable[[Dict, Dict], Optional[float]], log: Optional[Callable[[str], None]] = None
            ) -> List[Measurement]:
    out = []
    for sh in shapes:
        for cfg in configs:
            ms = timer(sh, cfg)
            out.append(Measurement(dict(sh), dict(cfg), ms))
            if log is not None:
                log(f"{sh} {cfg} -> {ms}")
    return out


TABLE_DIR = Path(__file__).resolve().parent / "tables"


def shipped_table(op: str) -> Optional[DecisionTable]:
    """The table profiled on B200 for `op` that ships with the package
    (tables/<op>_b200.json: gemm, gemm_bias_layernorm, conv2d_relu), or None."""
    path = TABLE_DIR / f"{op}_b200.json"
    return DecisionTable.load(path) if path.exists() else None


class AdaptiveTuner:
    """Table first, formula second (docs/autotuner_design.md:478-506).  table="shipped"
    loads the package's B200 table for the descriptor's op, when there is one."""

    def __init__(self, descriptor: TileLangKernelBase, table=None, hw=None):
        self.descriptor = descriptor
        self.table = shipped_table(descriptor.name) if table == "shipped" else table
        self.hw = hw

    def select(self, **shape) -> SelectResult:
        if self.table is not None:
            cfg = self.table.lookup(**shape)
            if cfg is not None:
                return SelectResult(cfg, "table", None)
        ranked = rank_all(self.descriptor, hw=self.hw, **shape)
        if not ranked:
            raise RuntimeError(f"No valid configs for {self.descriptor.name} at {shape}")
        return SelectResult(dict(ranked[0]["raw_config"]), "formula", ranked[0]["score"])


def gpu_timer(op: str, warmup: int = 5, rep: int = 25) -> Callable[[Dict, Dict], Optional[float]]:
    """Timer running this package's kernel for `op` (gemm, gemm_bias_act,
    gemm_bias_layernorm, conv2d) on the current GPU: fp16 inputs, L2 flushed before each
    repetition, median CUDA-event time in ms; None when the library rejects the config."""
    import torch

    from .. import _native as N
    from .. import fused
    from ..formula_bench import do_bench

    cache: Dict[str, Any] = {}

    def inputs(shape):
        key = json.dumps(shape, sort_keys=True)
        if key not in cache:
            cache.clear()  # one shape's tensors at a time
            g = torch.Generator().manual_seed(0)
            if _is_conv(shape):
                x = torch.randn(shape["N"], shape["H"], shape["W"], shape["C"], generator=g).half().cuda()
                w = (torch.randn(shape["KH"], shape["KW"], shape["C"], shape["OC"], generator=g) * 0.05).half().cuda()
                cache[key] = (x, w)
            else:
                a = torch.randn(shape["M"], shape["K"], generator=g).half().cuda()
                b = (torch.randn(shape["K"], shape["N"], generator=g) * 0.05).half().cuda()
                v = [torch.randn(shape["N"], generator=g).half().cuda() for _ in range(3)]
                cache[key] = (a, b, v)
        return cache[key]

    def timer(shape, cfg):
        tile = fused.as_tile_cfg(cfg)
        try:
            if _is_conv(shape):
                x, w = inputs(shape)
                ws_n = fused.conv_workspace_bytes(shape["N"], shape["H"], shape["W"], shape["C"], shape["OC"],
                                                  shape["KH"], shape["KW"], shape["stride"], shape["padding"], 1,
                                                  config=tile)
                ws = torch.zeros(max(16, ws_n), dtype=torch.uint8, device="cuda")
                fn = lambda: fused.conv2d_nhwc(x, w, relu=op.endswith("relu"), stride=shape["stride"],
                                               padding=shape["padding"], workspace=ws, config=tile)
            else:
                a, b, (bias, gamma, beta) = inputs(shape)
                epi = {"gemm": "none", "gemm_bias_act": "bias_relu", "gemm_bias_layernorm": "bias_layernorm"}[op]
                ws_n = fused.workspace_bytes(shape["M"], shape["N"], shape["K"], epi, tile)
                ws = torch.zeros(max(16, ws_n), dtype=torch.uint8, device="cuda")
                kw = {} if epi == "none" else {"bias": bias}
                if epi == "bias_layernorm":
                    kw.update(gamma=gamma, beta=beta)
                fn = lambda: fused.gemm(a, b, epilogue=epi, workspace=ws, config=tile, **kw)
            fn()
            return do_bench(fn, warmup, rep)
        except N.FoError:
            return None

    return timer


def evaluate(descriptor: TileLangKernelBase, shapes: Sequence[Dict], measurements: Sequence[Measurement]) -> Dict:
    """The formula's pick against the measured best over the profiled shapes: top-1
    accuracy and the time ratio best / formula (the design doc's accuracy table)."""
    by_shape: Dict[str, Dict[str, float]] = {}
    for r in measurements:
        if r.ms is not None:
            by_shape.setdefault(json.dumps(r.shape, sort_keys=True), {})[_cfg_key(r.config)] = r.ms
    hits, ratios, rows = 0, [], []
    for sh in shapes:
        times = by_shape.get(json.dumps(sh, sort_keys=True))
        if not times:
            continue
        pick = _cfg_key(rank_all(descriptor, **sh)[0]["raw_config"])
        best = min(times.values())
        t_pick = times.get(pick)
        if t_pick is None:
            continue
        hits += int(t_pick <= best * 1.0001)
        ratios.append(best / t_pick)
        rows.append({**sh, "formula_ms": t_pick, "best_ms": best, "ratio": best / t_pick})
    n = len(ratios)
    return {"shapes": n, "top1": hits / n if n else 0.0, "mean_ratio": sum(ratios) / n if n else 0.0,
            "min_ratio": min(ratios) if ratios else 0.0, "rows": rows}


def main(argv=None) -> None:
    from ..conv import conv2d_relu
    from ..gemm import gemm, gemm_bias_act, gemm_bias_layernorm

    descs = {"gemm": gemm.DESCRIPTOR, "gemm_bias_act": gemm_bias_act.DESCRIPTOR,
             "gemm_bias_layernorm": gemm_bias_layernorm.DESCRIPTOR, "conv2d_relu": conv2d_relu.DESCRIPTOR}
    ap = argparse.ArgumentParser(description="profile shapes x configs and build a decision table")
    ap.add_argument("--op", default="gemm", choices=sorted(descs))
    ap.add_argument("--m", type=int, nargs="*", help="profiled M (GEMM) or batch (conv) points")
    ap.add_argument("--top-k", type=int, default=6, help="formula top-k configs per shape to profile")
    ap.add_argument("--out", default=None, help="write the table as JSON")
    ap.add_argument("--report", default=None, help="write the formula-vs-measured summary as JSON")
    ap.add_argument("--measurements", default=None, help="write every (shape, config, ms) as JSON")
    args = ap.parse_args(argv)
    desc = descs[args.op]
    shapes = build_sampling_plan(args.op, args.m)
    configs = candidate_configs(desc, shapes, args.top_k)
    print(f"{args.op}: {len(shapes)} shapes x {len(configs)} configs")
    meas = profile(shapes, configs, gpu_timer(args.op))
    table = build_decision_table(args.op, meas)
    ev = evaluate(desc, shapes, meas)
    print(f"formula top-1 {ev['top1']:.2f}, time ratio best/formula mean {ev['mean_ratio']:.3f} "
          f"min {ev['min_ratio']:.3f} over {ev['shapes']} shapes")
    for g in sorted(table.groups):
        print(g, [(lo, hi, desc.format_config(c)) for lo, hi, c in table.intervals(g)])
    if args.out:
        table.save(args.out)
    if args.report:
        Path(args.report).write_text(json.dumps(ev, indent=1))
    if args.measurements:
        Path(args.measurements).write_text(json.dumps([r.__dict__ for r in meas]))


if __name__ == "__main__":
    main()
