"""Raw config spaces of the sm_100a kernels and their descriptor base class.

A raw config is the dict the operator modules pass to the kernel (and that
`select_best` returns): block_M (tcgen05 M = 128, or 256 for a CTA pair), block_N (64 /
128 / 256), block_K (64 = one 128-byte swizzle row of 16-bit elements per stage, or 128 =
two; 192 = three filter taps per stage in the direct conv), num_stages, thread_num (10
warps for GEMMs: producer / MMA / 8 epilogue; 13 for conv: 4 producer warps; 11 for the
direct conv: weight producer / MMA / 8 epilogue / pixel-slot producer), group_m (tile
raster) and swap_ab (conv: 1 = operand-swapped im2col kernel, 2 = direct conv).  Legality
is the C ABI's (fo_query_config_legal): shared memory <= 227 KB, TMEM <= 512 columns; the
direct conv's shared memory depends on the image width and is checked per shape.
"""
from __future__ import annotations

from typing import Any, Dict, List, Sequence

from .cost_model import TuneConfig
from .interface import TileLangKernelBase

GEMM_THREADS = 320
CONV_THREADS = 416
DIRECT_THREADS = 352  # direct conv: weight producer, MMA, 8 epilogue, slot producer
SMEM_LIMIT = 232448


def smem_bytes(block_n: int, stages: int, block_m: int = 128, block_k: int = 64) -> int:
    """Dynamic shared memory of one CTA (= fo_config_smem_bytes of the C ABI).  block_m
    256 is a CTA pair: each CTA holds 128 rows of A and half of the B tile."""
    b_cols = block_n // 2 if block_m == 256 else block_n
    return 1024 + stages * (128 + b_cols) * block_k * 2 + 32768 + 1536


def max_stages(block_n: int, block_m: int = 128, block_k: int = 64) -> int:
    s = 8
    while s > 2 and smem_bytes(block_n, s, block_m, block_k) > SMEM_LIMIT:
        s -= 1
    return s


def tcgen05_configs(block_ns: Sequence[int] = (64, 128, 256), group_ms: Sequence[int] = (8, 16, 0),
                    conv: bool = False, stages: Sequence[int] = (),
                    block_ms: Sequence[int] = (128, 256)) -> List[Dict[str, Any]]:
    out = []
    for bm in block_ms:
        for bn in block_ns:
            if bm == 256 and bn < 128:
                continue
            top = max_stages(bn, bm)
            # deepest pipeline first: rank_all keeps generation order among equal scores,
            # and measured ties (S5 / S6 pairs) never favour the shallower ring
            st = sorted({s for s in (stages or (3, 4, top)) if (3 if conv else 2) <= s <= top}, reverse=True)
            for s in st:
                for g in group_ms:
                    out.append({"block_M": bm, "block_N": bn, "block_K": 64, "num_stages": s,
                                "thread_num": CONV_THREADS if conv else GEMM_THREADS, "group_m": g})
    # block_K 128 (two K slices per stage: half the waits and commits per MMA for the one
    # issuing thread) measured +5-7% on 128- and 64-column single-CTA tiles, +1-20% on
    # CTA pairs (whose issuing thread has no slack at block_K 64), and a loss on 256-column
    # single-CTA tiles, which it leaves with two stages
    for bm, bn in ((128, 64), (128, 128), (256, 128), (256, 256)):
        if conv or bn not in block_ns or bm not in block_ms:  # the conv kernels stage one K slice
            continue
        top = max_stages(bn, bm, 128)
        if top >= 3 or (top >= 2 and not conv and bm == 128):
            for g in group_ms:
                out.append({"block_M": bm, "block_N": bn, "block_K": 128, "num_stages": top,
                            "thread_num": CONV_THREADS if conv else GEMM_THREADS, "group_m": g})
    if conv:  # operand-swapped conv: 128 output channels x block_N pixels per tile
        for bn in (128, 256):
            for s in sorted({x for x in (stages or (3, 4)) if 3 <= x <= max_stages(bn)}, reverse=True):
                out.append({"block_M": 128, "block_N": bn, "block_K": 64, "num_stages": s,
                            "thread_num": CONV_THREADS, "group_m": 0, "swap_ab": 1})
        # direct conv (stride 1, C % 64 == 0, padded row <= 256 positions; the model scores
        # other shapes 0): up to 256 positions x 128 channels per tile, one to three filter
        # taps per weight stage, as many stages as fit beside two 224-position pixel slots
        for bk, s in ((64, 6), (128, 3), (192, 2)):
            out.append({"block_M": 128, "block_N": 256, "block_K": bk, "num_stages": s,
                        "thread_num": DIRECT_THREADS, "group_m": 0, "swap_ab": 2})
    return out


class Tcgen05Descriptor(TileLangKernelBase):
    """Descriptor base for the sm_100a kernels: raw configs map to kind="tcgen05"."""

    def raw_config_to_tune_config(self, raw: Dict[str, Any]) -> TuneConfig:
        return TuneConfig(block_M=raw["block_M"], block_N=raw["block_N"], block_K=raw["block_K"],
                          num_stages=raw["num_stages"], num_warps=raw["thread_num"] // 32,
                          group_size_m=raw.get("group_m", 0), kind="tcgen05",
                          max_ctas=raw.get("max_ctas", 0), swap_ab=raw.get("swap_ab", 0))

    def format_config(self, raw: Dict[str, Any]) -> str:
        base = super().format_config(raw)
        sw = raw.get("swap_ab", 0)
        return base + ("_DC" if sw == 2 else "_SW" if sw else "")
