"""Descriptor / autotuner API.

Mirrors kernel/autotuner/interface.py of the reference: every operator module exposes a
`DESCRIPTOR` (a `TileLangKernelBase` subclass, :50-128) and the generic `select_best`
(:136-178) / `rank_all` (:181-241) score its raw configs with `score_formula`.  The class
keeps the reference's name so callers switch by changing one import; in this package the
descriptors enumerate configs of the sm_100a kernels (`TuneConfig.kind == "tcgen05"`),
which `score_formula` scores with the B200 model.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

from .cost_model import OpSpec, TuneConfig, score_formula, score_formula_detailed
from .gpu_spec import GPUSpec, get_gpu_spec


class TileLangKernelBase:
    """Base descriptor (reference interface.py:50-128).

    Subclasses override `name`, `make_op_spec` and `get_raw_configs`; the defaults of
    the other methods handle the reference's (block_M, block_N, block_K, num_stages,
    thread_num) dicts.
    """

    @property
    def name(self) -> str:
        raise NotImplementedError

    def make_op_spec(self, raw_config: Optional[Dict[str, Any]] = None, **shape: Any) -> OpSpec:
        raise NotImplementedError

    def get_raw_configs(self, **shape: Any) -> List[Dict[str, Any]]:
        raise NotImplementedError

    def raw_config_to_tune_config(self, raw: Dict[str, Any]) -> TuneConfig:
        return TuneConfig(block_M=raw["block_M"], block_N=raw["block_N"], block_K=raw["block_K"],
                          num_stages=raw["num_stages"], num_warps=raw["thread_num"] // 32)

    def score_adjustment(self, raw: Dict[str, Any], base_score: float, **shape: Any) -> float:
        return base_score

    def format_config(self, raw: Dict[str, Any]) -> str:
        parts = [f"BM{raw['block_M']}", f"BN{raw['block_N']}", f"BK{raw['block_K']}"]
        if "split_k" in raw:
            parts.append(f"SK{raw['split_k']}")
        parts.append(f"S{raw['num_stages']}")
        parts.append(f"T{raw['thread_num']}")
        if "group_m" in raw:
            parts.append(f"G{raw['group_m']}")
        return "_".join(parts)


def _scored(descriptor: TileLangKernelBase, hw: GPUSpec, detailed: bool, shape: Dict[str, Any]):
    for raw in descriptor.get_raw_configs(**shape):
        op = descriptor.make_op_spec(raw_config=raw, **shape)
        cfg = descriptor.raw_config_to_tune_config(raw)
        if detailed:
            detail = score_formula_detailed(op, cfg, hw)
            base = detail["score"]
        else:
            detail, base = None, score_formula(op, cfg, hw)
        yield raw, descriptor.score_adjustment(raw, base, **shape), detail


def select_best(descriptor: TileLangKernelBase, hw: Optional[GPUSpec] = None,
                **shape_kwargs: Any) -> Tuple[Dict[str, Any], float]:
    """Highest-scoring raw config and its score (first one wins ties).

    Raises RuntimeError when the descriptor yields no configs (reference :174-177).
    """
    hw = hw or get_gpu_spec()
    best, best_score = None, -1.0
    for raw, score, _ in _scored(descriptor, hw, False, shape_kwargs):
        if score > best_score:
            best, best_score = raw, score
    if best is None:
        raise RuntimeError(f"No configs generated for {descriptor.name} with {shape_kwargs}")
    return best, best_score


def rank_all(descriptor: TileLangKernelBase, hw: Optional[GPUSpec] = None, detailed: bool = False,
             **shape_kwargs: Any) -> List[Dict[str, Any]]:
    """Every config with score and formatted name, best first (stable for ties)."""
    hw = hw or get_gpu_spec()
    out = []
    for raw, score, detail in _scored(descriptor, hw, detailed, shape_kwargs):
        e = {"raw_config": raw, "score": score, "formatted": descriptor.format_config(raw)}
        if detailed:
            e["detail"] = detail
        out.append(e)
    out.sort(key=lambda e: e["score"], reverse=True)
    return out


_CACHE_DIR: Optional[Path] = None


def configure_autotuner_cache(cache_dir: str = ".tilelang_cache") -> None:
    """Kept for callers of the reference API (interface.py:249-261), which pointed
    TileLang's JIT cache at `cache_dir`.  The kernels here are compiled ahead of time
    into libb200fo.so, so there is no JIT cache: this only creates the directory and
    remembers it for tools that store measurement logs there."""
    global _CACHE_DIR
    root = Path(cache_dir).expanduser().resolve()
    root.mkdir(parents=True, exist_ok=True)
    _CACHE_DIR = root


def autotuner_cache_dir() -> Optional[Path]:
    return _CACHE_DIR


__all__ = ["TileLangKernelBase", "autotuner_cache_dir", "configure_autotuner_cache", "rank_all",
           "select_best"]
