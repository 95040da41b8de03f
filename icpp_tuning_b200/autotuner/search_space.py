"""Config search space: parameter pools, LCM marginal sampling, hardware pruning and the
cold / structure / warm initialisation modes.

Mirrors kernel/autotuner/search_space.py of the reference (pools :32-66, LCM sampling
:97-156, exhaustive enumeration :174-196, occupancy :208-232, three-level pruning
:239-286, stratified sampling :293-411, modes :413-596, shape samplers :603-664,
summary :671-706) and adds the "tcgen05" backend for this package's sm_100a kernels.
For that backend the pruning levels are the kernel's real limits: L1 dynamic shared
memory <= the opt-in per-block maximum (227 KB), L2 TMEM columns of the two fp32
accumulators <= 512, L3 a pipeline at least 2 stages deep (3 for the conv gather).
Register pressure and warp occupancy do not bound this design: the accumulator is in
TMEM and one CTA owns an SM.

The reference's enumeration calls TuneConfig.is_valid_for_backend, which it never
defines, so its generate_search_space raises AttributeError; here the method exists.
"""
from __future__ import annotations

import math
import random
from collections import defaultdict
from typing import Dict, List, Optional

from .cost_model import TuneConfig
from .gpu_spec import GPUSpec

_TRITON_MATMUL_PARAMS = {"block_M": [32, 64, 128], "block_N": [32, 64, 128, 256], "block_K": [32, 64],
                         "num_stages": [2, 3, 4, 5], "num_warps": [2, 4, 8]}
_TILELANG_MATMUL_PARAMS = {"block_M": [32, 48, 64, 80, 96, 112, 128], "block_N": [64, 128, 256],
                           "block_K": [32, 64], "num_stages": [2, 3, 4], "num_warps": [4, 8]}
_TRITON_CONV2D_PARAMS = {"block_M": [32, 64, 128], "block_N": [32, 64, 128], "block_K": [16, 32, 64],
                         "num_stages": [2, 3, 4, 5], "num_warps": [2, 4, 8]}
_TILELANG_CONV2D_PARAMS = {"block_M": [32, 48, 64, 96, 128], "block_N": [32, 64, 128],
                           "block_K": [16, 32, 64], "num_stages": [2, 3, 4], "num_warps": [4, 8]}
# sm_100a kernels: tcgen05 M = 128 (one CTA) or 256 (a CTA pair, cta_group::2), one
# 128-byte swizzle row of K, fixed role split.
_TCGEN05_MATMUL_PARAMS = {"block_M": [128, 256], "block_N": [64, 128, 256], "block_K": [64],
                          "num_stages": [2, 3, 4, 5, 6, 7, 8], "num_warps": [10], "group_size_m": [0, 8, 16]}
_TCGEN05_CONV2D_PARAMS = {"block_M": [128, 256], "block_N": [64, 128, 256], "block_K": [64],
                          "num_stages": [3, 4, 5, 6, 7, 8], "num_warps": [13], "group_size_m": [0]}

MIN_OCCUPANCY_THRESHOLD = 0.2
_KEYS = ("block_M", "block_N", "block_K", "num_stages", "num_warps", "group_size_m")


def _get_param_pools(op_type: str, backend: str) -> Dict[str, List[int]]:
    table = {
        ("matmul", "triton"): _TRITON_MATMUL_PARAMS, ("matmul", "tilelang"): _TILELANG_MATMUL_PARAMS,
        ("matmul", "tcgen05"): _TCGEN05_MATMUL_PARAMS, ("conv2d", "triton"): _TRITON_CONV2D_PARAMS,
        ("conv2d", "tilelang"): _TILELANG_CONV2D_PARAMS, ("conv2d", "tcgen05"): _TCGEN05_CONV2D_PARAMS,
    }
    if (op_type, backend) not in table:
        raise ValueError(f"Unsupported op_type/backend: {op_type}/{backend}")
    return {k: list(v) for k, v in table[(op_type, backend)].items()}


def _multi_lcm(values: List[int]) -> int:
    out = values[0]
    for v in values[1:]:
        out = out * v // math.gcd(out, v)
    return out


def lcm_marginal_sample(param_pools: Dict[str, List[int]], n_samples: Optional[int] = None,
                        seed: Optional[int] = None) -> List[Dict[str, int]]:
    """Samples in which every value of every pool appears equally often: replicate each
    pool to the LCM of the pool sizes (or n_samples), shuffle each independently, zip."""
    rng = random.Random(seed)
    names = list(param_pools)
    L = _multi_lcm([len(param_pools[n]) for n in names])
    n_samples = L if n_samples is None else n_samples
    length = max(L, n_samples)
    cols = {}
    for n in names:
        pool = param_pools[n]
        col = (pool * math.ceil(length / len(pool)))[:length]
        rng.shuffle(col)
        cols[n] = col
    return [{n: cols[n][i] for n in names} for i in range(n_samples)]


def _to_tune_config(d: Dict[str, int], backend: str = "tilelang") -> TuneConfig:
    kw = dict(block_M=d["block_M"], block_N=d["block_N"], block_K=d["block_K"],
              num_stages=d["num_stages"], num_warps=d["num_warps"])
    if backend == "tcgen05":
        kw.update(group_size_m=d.get("group_size_m", 0), kind="tcgen05")
    return TuneConfig(**kw)


def generate_exhaustive_configs(op_type: str = "matmul", backend: str = "tilelang") -> List[TuneConfig]:
    """Cartesian product of the backend's pools, statically legal tiles only."""
    pools = _get_param_pools(op_type, backend)
    names = list(pools)
    out: List[TuneConfig] = []

    def rec(i, cur):
        if i == len(names):
            c = _to_tune_config(cur, backend)
            # tcgen05: shape legality here; the shared-memory budget is pruning level L1
            shape_ok = c.kind == "tcgen05" and not (c.block_M == 256 and c.block_N < 128)
            if c.is_valid_for_backend(backend) or (backend == "tcgen05" and shape_ok):
                out.append(c)
            return
        for v in pools[names[i]]:
            cur[names[i]] = v
            rec(i + 1, cur)

    rec(0, {})
    return out


def estimate_occupancy(config: TuneConfig, hw: GPUSpec) -> float:
    """Resident warps / max warps per SM from thread, shared-memory and register limits."""
    by_threads = hw.max_warps_per_sm // config.num_warps
    smem = config.shared_mem_bytes
    by_smem = hw.shared_mem_per_sm // smem if smem > 0 else hw.max_blocks_per_sm
    regs = config.regs_per_thread_estimate * config.threads
    by_regs = hw.max_regs_per_sm // regs if regs > 0 else hw.max_blocks_per_sm
    blocks = max(0, min(by_threads, by_smem, by_regs, hw.max_blocks_per_sm))
    return min(1.0, blocks * config.num_warps / hw.max_warps_per_sm) if hw.max_warps_per_sm else 0.0


def prune_shared_memory(configs: List[TuneConfig], hw: GPUSpec) -> List[TuneConfig]:
    """L1: dynamic shared memory within the per-block maximum."""
    return [c for c in configs if c.shared_mem_bytes <= hw.shared_mem_per_block]


def prune_register_pressure(configs: List[TuneConfig], hw: GPUSpec) -> List[TuneConfig]:
    """L2: registers (SIMT tiles) or TMEM columns (tcgen05 tiles)."""
    out = []
    for c in configs:
        if c.kind == "tcgen05":
            if hw.tmem_cols_per_sm and c.tmem_columns <= hw.tmem_cols_per_sm:
                out.append(c)
        elif c.regs_per_thread_estimate * c.threads <= hw.max_regs_per_block:
            out.append(c)
    return out


def prune_minimum_occupancy(configs: List[TuneConfig], hw: GPUSpec,
                            min_occupancy: float = MIN_OCCUPANCY_THRESHOLD) -> List[TuneConfig]:
    """L3: SIMT tiles need occupancy >= min_occupancy; tcgen05 tiles (one persistent CTA
    per SM by design) need a pipeline deep enough to overlap loads with MMAs."""
    out = []
    for c in configs:
        if c.threads > hw.max_threads_per_block or c.threads > hw.max_threads_per_sm:
            continue
        if c.shared_mem_bytes > hw.shared_mem_per_sm:
            continue
        if c.kind == "tcgen05":
            if c.num_stages >= (3 if c.num_warps == 9 else 2):
                out.append(c)
        elif estimate_occupancy(c, hw) >= min_occupancy:
            out.append(c)
    return out


def prune_configs(configs: List[TuneConfig], hw: GPUSpec) -> List[TuneConfig]:
    return prune_minimum_occupancy(prune_register_pressure(prune_shared_memory(configs, hw), hw), hw)


def _key(c: TuneConfig):
    return tuple(getattr(c, k) for k in _KEYS)


def _stratified_sample_from_valid(valid: List[TuneConfig], n_samples: Optional[int] = None,
                                  seed: int = 42) -> List[TuneConfig]:
    """Round-robin over block_N buckets (block_M for SIMT tiles) so every tile width is
    equally represented, then fill from the rest (reference :293-411)."""
    if not valid:
        return []
    rng = random.Random(seed)
    strat = "block_N" if all(c.kind == "tcgen05" for c in valid) else "block_M"
    pools = [sorted({getattr(c, k) for c in valid}) for k in _KEYS]
    lcm = _multi_lcm([len(p) for p in pools])
    want = min(max(2 * lcm, 30) if n_samples is None else n_samples, len(valid))
    if want >= len(valid):
        out = list(valid)
        rng.shuffle(out)
        return out
    buckets: Dict[int, List[TuneConfig]] = defaultdict(list)
    for c in valid:
        buckets[getattr(c, strat)].append(c)
    for b in buckets.values():
        rng.shuffle(b)
    order = sorted(buckets)
    cursor = {k: 0 for k in order}
    picked, seen = [], set()
    while len(picked) < want:
        progress = False
        for k in order:
            if len(picked) >= want:
                break
            b = buckets[k]
            while cursor[k] < len(b):
                c = b[cursor[k]]
                cursor[k] += 1
                if _key(c) not in seen:
                    picked.append(c)
                    seen.add(_key(c))
                    progress = True
                    break
        if not progress:
            break
    if len(picked) < want:
        rest = [c for c in valid if _key(c) not in seen]
        rng.shuffle(rest)
        picked += rest[:want - len(picked)]
    return picked


def cold_start_configs(op_type: str, backend: str, hw: GPUSpec, n_samples: Optional[int] = None,
                       seed: int = 42) -> List[TuneConfig]:
    """Prune first, then sample with uniform marginals inside the valid set."""
    valid = prune_configs(generate_exhaustive_configs(op_type, backend), hw)
    return _stratified_sample_from_valid(valid, n_samples, seed)


def structure_aware_cold_start_configs(valid_configs: List[TuneConfig], hw: GPUSpec,
                                       n_samples: Optional[int] = None, seed: int = 42) -> List[TuneConfig]:
    """Stratified sample of a known-valid list (re-pruned for this GPU)."""
    pruned = prune_configs(valid_configs, hw) if valid_configs else []
    return _stratified_sample_from_valid(pruned, n_samples, seed)


def warm_start_configs(top_k_configs: List[TuneConfig], op_type: str, backend: str, hw: GPUSpec,
                       n_explore: Optional[int] = None, seed: int = 42) -> List[TuneConfig]:
    """Known-good configs first, then unbiased exploration configs not already present."""
    n_explore = max(len(top_k_configs), 10) if n_explore is None else n_explore
    exploit = prune_configs(top_k_configs, hw)
    explore = cold_start_configs(op_type, backend, hw, n_samples=n_explore * 2, seed=seed)
    seen = {_key(c) for c in exploit}
    merged = list(exploit)
    for c in explore:
        if _key(c) not in seen:
            seen.add(_key(c))
            merged.append(c)
            if len(merged) >= len(exploit) + n_explore:
                break
    return merged


def generate_search_space(op_type: str, hw: GPUSpec, backend: str = "tilelang", mode: str = "exhaustive",
                          n_samples: Optional[int] = None, valid_configs: Optional[List[TuneConfig]] = None,
                          top_k_configs: Optional[List[TuneConfig]] = None, seed: int = 42) -> List[TuneConfig]:
    if mode == "exhaustive":
        return prune_configs(generate_exhaustive_configs(op_type, backend), hw)
    if mode == "cold":
        return cold_start_configs(op_type, backend, hw, n_samples, seed)
    if mode == "structure":
        if valid_configs is None:
            raise ValueError("mode='structure' requires valid_configs")
        return structure_aware_cold_start_configs(valid_configs, hw, n_samples, seed)
    if mode == "warm":
        if top_k_configs is None:
            raise ValueError("mode='warm' requires top_k_configs")
        return warm_start_configs(top_k_configs, op_type, backend, hw, n_samples, seed)
    raise ValueError(f"Unsupported mode: {mode}")


def generate_matmul_sample_shapes(M_range: tuple = (1, 4096), N_values: Optional[List[int]] = None,
                                  K_values: Optional[List[int]] = None) -> List[dict]:
    """M dense where wave counts change fast (small M), sparse at large M."""
    N_values = N_values or [768, 2304, 4096]
    K_values = K_values or [768, 2304, 4096]
    ms = set(range(1, 17)) | set(range(16, 129, 16)) | set(range(128, 1025, 64)) \
        | set(range(1024, min(M_range[1] + 1, 4097), 256))
    ms = sorted(m for m in ms if M_range[0] <= m <= M_range[1])
    return [{"M": m, "N": n, "K": k} for m in ms for n in N_values for k in K_values]


def generate_conv2d_sample_shapes(N_values=None, HW_values=None, C_values=None, OC_values=None) -> List[dict]:
    N_values = N_values or [1, 2, 4, 8, 16, 32]
    HW_values = HW_values or [7, 14, 28, 56, 112, 224]
    C_values = C_values or [64, 128, 256, 512]
    OC_values = OC_values or [64, 128, 256, 512]
    return [{"N": n, "C": c, "H": hw, "W": hw, "OC": oc, "KH": 3, "KW": 3, "stride": 1, "padding": 1}
            for n in N_values for hw in HW_values for c in C_values for oc in OC_values]


def search_space_summary(op_type: str, hw: GPUSpec, backend: str = "tilelang", mode: str = "exhaustive",
                         **kwargs) -> dict:
    full = generate_exhaustive_configs(op_type, backend)
    l1 = prune_shared_memory(full, hw)
    l2 = prune_register_pressure(l1, hw)
    l3 = prune_minimum_occupancy(l2, hw)
    mode_cfgs = generate_search_space(op_type, hw, backend, mode=mode, **kwargs)
    occ = [estimate_occupancy(c, hw) for c in l3]
    return {"op_type": op_type, "backend": backend, "mode": mode, "exhaustive_full": len(full),
            "after_smem_prune": len(l1), "after_reg_prune": len(l2), "after_occupancy_prune": len(l3),
            "min_occupancy_threshold": MIN_OCCUPANCY_THRESHOLD,
            "avg_occupancy": round(sum(occ) / len(occ), 3) if occ else 0, "mode_output_size": len(mode_cfgs),
            "pruning_ratio": round(1 - len(l3) / len(full), 3) if full else 0}
