"""Plain GEMM C = A @ B (reference kernel/tilelang/gemm/gemm.py).

Reference surface kept: get_configs(M, K), ref_program(A, B, C), build_kernel(M, N, K,
config=None) -> kernel(a, b) -> C, DESCRIPTOR.  The reference launches a split-K
TileLang kernel that atomically adds fp32 partial tiles (gemm.py:51-81); here one
persistent tcgen05 kernel computes each 128 x BN tile over the whole K in TMEM, so no
zero-initialised output or atomics are needed and the output may be f16 / bf16 / fp32.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch

from .. import fused
from ..autotuner.cost_model import make_matmul_spec
from ..autotuner.interface import select_best
from ..autotuner.tcgen05_space import Tcgen05Descriptor, tcgen05_configs


def ref_program(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor) -> None:
    """The reference's expected result (gemm.py:20-21): C[...] = (A @ B) in fp32.  Eager
    PyTorch, used by callers as a check; build_kernel never calls it."""
    C[...] = (A @ B).to(torch.float32)


def get_configs(M: int = 0, K: int = 0) -> List[Dict[str, Any]]:
    return tcgen05_configs()


class GemmDescriptor(Tcgen05Descriptor):
    @property
    def name(self) -> str:
        return "gemm"

    def make_op_spec(self, raw_config=None, M=0, N=0, K=0, out_bytes: int = 4, **kw):
        return make_matmul_spec(M=M, N=N, K=K, output_element_bytes=out_bytes)

    def get_raw_configs(self, M=0, K=0, **kw):
        return get_configs(M, K)


DESCRIPTOR = GemmDescriptor()


def build_kernel(M: int, N: int, K: int, config: Optional[Dict[str, Any]] = None,
                 out_dtype: torch.dtype = torch.float32, b_layout: str = "kn"):
    """Returns kernel(a, b) -> C[M, N] (out_dtype).  a: [M, K]; b: [K, N] ("kn", the
    reference layout) or [N, K] ("nk").  Shapes are fixed at build time as in the
    reference (its prim_func closes over M, N, K)."""
    if config is None:
        config, _ = select_best(DESCRIPTOR, M=M, N=N, K=K, out_bytes=torch.empty((), dtype=out_dtype).element_size())
    cfg = fused.as_tile_cfg(config)
    # split-K workspace: zero-filled once per stream, left zeroed by every call
    wss = fused.StreamWorkspaces(fused.workspace_bytes(M, N, K, "none", cfg))

    def kernel(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        _check_shape(a, b, M, N, K, b_layout)
        return fused.gemm(a, b, b_layout=b_layout, out=out, out_dtype=out_dtype, workspace=wss.get(), config=cfg)

    kernel.config = config
    kernel.workspace = wss.default
    return kernel


def _check_shape(a, b, M, N, K, b_layout):
    want_b = (K, N) if b_layout == "kn" else (N, K)
    if tuple(a.shape) != (M, K) or tuple(b.shape) != want_b:
        raise ValueError(f"kernel built for a[{M},{K}], b{list(want_b)}; got a{list(a.shape)}, b{list(b.shape)}")
