"""C = act(A @ B + bias), act in {relu, gelu_tanh, gelu_erf, none}
(reference kernel/tilelang/gemm/gemm_bias_act.py).

Reference surface kept: get_configs(M, K), ref_program(A, B, bias), build_kernel(M, N,
K, config=None) -> kernel(a, b, bias) -> C, DESCRIPTOR (name "gemm_bias_relu",
primitives bias_add + relu, :103-116).  The reference implements ReLU only and writes
fp32 (:50-88); here the activation is a build argument (GELU-tanh follows
evaluation/end2end.py:37-38, GELU-erf :83) and the output dtype is selectable.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch

from .. import fused
from ..autotuner.cost_model import make_matmul_spec
from ..autotuner.interface import select_best
from ..autotuner.tcgen05_space import Tcgen05Descriptor, tcgen05_configs
from .gemm import _check_shape

_EPI = {"relu": "bias_relu", "gelu_tanh": "bias_gelu_tanh", "gelu_erf": "bias_gelu_erf", "none": "bias"}
_PRIM = {"relu": ["bias_add", "relu"], "gelu_tanh": ["bias_add", "gelu"], "gelu_erf": ["bias_add", "gelu"],
         "none": ["bias_add"]}


def ref_program(A: torch.Tensor, B: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """The reference's expected result (gemm_bias_act.py:44-47), eager PyTorch."""
    return torch.relu((A @ B).to(torch.float32) + bias.unsqueeze(0))


def get_configs(M: int = 0, K: int = 0) -> List[Dict[str, Any]]:
    return tcgen05_configs()


class GemmBiasActDescriptor(Tcgen05Descriptor):
    def __init__(self, act: str = "relu"):
        self.act = act

    @property
    def name(self) -> str:
        return "gemm_bias_relu" if self.act == "relu" else f"gemm_bias_{self.act}"

    def make_op_spec(self, raw_config=None, M=0, N=0, K=0, out_bytes: int = 2, **kw):
        return make_matmul_spec(M=M, N=N, K=K, primitives=_PRIM[self.act], output_element_bytes=out_bytes)

    def get_raw_configs(self, M=0, K=0, **kw):
        return get_configs(M, K)


DESCRIPTOR = GemmBiasActDescriptor("relu")
DESCRIPTORS = {a: GemmBiasActDescriptor(a) for a in _EPI}


def build_kernel(M: int, N: int, K: int, config: Optional[Dict[str, Any]] = None, act: str = "relu",
                 out_dtype: torch.dtype = torch.float32, b_layout: str = "kn"):
    """Returns kernel(a, b, bias) -> C[M, N]."""
    if act not in _EPI:
        raise ValueError(f"act must be one of {sorted(_EPI)}")
    if config is None:
        config, _ = select_best(DESCRIPTORS[act], M=M, N=N, K=K,
                                out_bytes=torch.empty((), dtype=out_dtype).element_size())
    cfg = fused.as_tile_cfg(config)
    ws_bytes = fused.workspace_bytes(M, N, K, "none", cfg)
    # zero-filled once per stream; the kernel leaves its split-K counters zeroed after every call
    wss = fused.StreamWorkspaces(ws_bytes)
    epi = _EPI[act]

    def kernel(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        _check_shape(a, b, M, N, K, b_layout)
        return fused.gemm(a, b, b_layout=b_layout, epilogue=epi, bias=bias, out=out, out_dtype=out_dtype,
                          workspace=wss.get(), config=cfg)

    kernel.config = config
    kernel.workspace = wss.default
    return kernel
