"""The reference's own TileLang config spaces and descriptors.

These reproduce which config the reference's autotuner picks for its register-tiled
TileLang kernels (kernel/tilelang/gemm/gemm.py:24-48 and :97-114,
gemm_bias_act.py:20-41 and :103-116, gemm_bias_layernorm.py:19-40 and :196-208,
conv/conv2d.py:186-205 and :467-479).  They are kept so the published A100 decisions in
the reference's evaluation/*.csv can be replayed as golden tests of the cost model, and
so a caller can ask what the reference would have chosen for a shape.  The sm_100a
kernels of this package use the descriptors in icpp_tuning_b200.gemm / .conv instead.
"""
from __future__ import annotations

import itertools
import math
from typing import Any, Dict, List

from .cost_model import make_conv2d_spec, make_matmul_spec
from .interface import TileLangKernelBase


def _product(keys, pools, keep=lambda d: True) -> List[Dict[str, Any]]:
    out = []
    for vals in itertools.product(*pools):
        d = dict(zip(keys, vals))
        if keep(d):
            out.append(d)
    return out


def gemm_splitk_configs(M: int, K: int, split_k_values=(2,)) -> List[Dict[str, Any]]:
    """gemm.py:24-48: split-K TileLang configs with K/split_k divisible by block_K."""
    keys = ("block_M", "block_N", "block_K", "split_k", "num_stages", "thread_num")
    pools = ([16, 32, 64], [128, 256], [32, 64, 128], list(split_k_values), [1, 2, 4, 8],
             [64, 128, 256])
    return _product(keys, pools,
                    lambda d: K % d["split_k"] == 0 and (K // d["split_k"]) % d["block_K"] == 0)


def tilelang_fused_configs(K: int) -> List[Dict[str, Any]]:
    """gemm_bias_act.py:20-41 / gemm_bias_layernorm.py:19-40: 72 configs, K % block_K == 0."""
    keys = ("block_M", "block_N", "block_K", "num_stages", "thread_num")
    pools = ([16, 32, 64], [64, 128, 256], [32, 64], [1, 2], [128, 256])
    return _product(keys, pools, lambda d: K % d["block_K"] == 0)


def tilelang_conv_configs() -> List[Dict[str, Any]]:
    """conv/conv2d.py:186-205: 72 configs, no shape filter."""
    keys = ("block_M", "block_N", "block_K", "num_stages", "thread_num")
    pools = ([16, 32, 64], [64, 128, 256], [32, 64], [1, 2], [128, 256])
    return _product(keys, pools)


class LegacyGemmSplitK(TileLangKernelBase):
    name = "gemm_splitk"

    def make_op_spec(self, raw_config=None, M=0, N=0, K=0, **kw):
        sk = raw_config.get("split_k", 2) if raw_config else 2
        return make_matmul_spec(M=M, N=N, K=K // sk)

    def get_raw_configs(self, M, K, **kw):
        return gemm_splitk_configs(M, K)

    def score_adjustment(self, raw, base_score, **kw):
        sk = raw.get("split_k", 2)
        return base_score * math.sqrt(sk) / sk


class LegacyGemmBiasRelu(TileLangKernelBase):
    name = "gemm_bias_relu"

    def make_op_spec(self, raw_config=None, M=0, N=0, K=0, **kw):
        return make_matmul_spec(M=M, N=N, K=K, primitives=["bias_add", "relu"])

    def get_raw_configs(self, M=0, K=0, **kw):
        return tilelang_fused_configs(K)


class LegacyGemmBiasLayerNorm(TileLangKernelBase):
    name = "gemm_bias_layernorm"

    def make_op_spec(self, raw_config=None, M=0, N=0, K=0, **kw):
        return make_matmul_spec(M=M, N=N, K=K, primitives=["bias_add", "row_layernorm"])

    def get_raw_configs(self, K=0, **kw):
        return tilelang_fused_configs(K)


class LegacyConv2d(TileLangKernelBase):
    name = "conv2d"

    def make_op_spec(self, raw_config=None, N=1, C=1, H=1, W=1, OC=1, KH=1, KW=1, stride=1,
                     padding=0, **kw):
        return make_conv2d_spec(N, C, H, W, OC, KH, KW, stride=stride, padding=padding)

    def get_raw_configs(self, **kw):
        return tilelang_conv_configs()


LEGACY_DESCRIPTORS = {
    "gemm": LegacyGemmSplitK(),
    "gemm_bias_act": LegacyGemmBiasRelu(),
    "gemm_bias_layernorm": LegacyGemmBiasLayerNorm(),
    "conv2d": LegacyConv2d(),
}
