"""CPU restatement of the reference's expected-result programs (test infrastructure only).

Each function follows one PyTorch program of leon062112/icpp-tuning and keeps its
rounding points, so the result is what the reference checks its kernels against:

  gemm                kernel/tilelang/gemm/gemm.py:20-21        C = (A @ B).to(fp32)
  gemm_bias_act       kernel/tilelang/gemm/gemm_bias_act.py:44-47
                      relu((A @ B).to(fp32) + bias); GELU variants follow
                      evaluation/end2end.py:37-38 (tanh) and :83 (erf)
  gemm_bias_layernorm kernel/tilelang/gemm/gemm_bias_layernorm.py:44-50
                      layer_norm((A @ B).to(fp32) + bias, gamma, beta, eps).to(out)
  conv2d              kernel/tilelang/conv/conv2d.py:35-62      NHWC<->NCHW permutes
  conv2d_relu         kernel/tilelang/conv/conv2d_relu.py:29-60 relu in fp32

A @ B is evaluated in the inputs' dtype, as the reference does, so the product is rounded
to fp16/bf16 before the fp32 epilogue.  The `upcast=True` variants accumulate and keep
fp32 throughout (A.float() @ B.float()), the tighter check of an fp32-accumulating kernel.
All functions run on CPU tensors.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


def _cpu(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu")


def _b_kn(B: torch.Tensor, b_layout: str) -> torch.Tensor:
    return B if b_layout == "kn" else B.t()


def product(A: torch.Tensor, B: torch.Tensor, b_layout: str = "kn", upcast: bool = False) -> torch.Tensor:
    """fp32 [M, N] of A[M,K] @ B (gemm.py:20-21): rounded to A's dtype unless upcast."""
    A, B = _cpu(A), _b_kn(_cpu(B), b_layout)
    if upcast:
        return A.float() @ B.float()
    return (A @ B).to(torch.float32)


def activation(x: torch.Tensor, act: Optional[str]) -> torch.Tensor:
    if act in (None, "none"):
        return x
    if act == "relu":
        return torch.relu(x)
    if act == "gelu_tanh":  # end2end.py:37-38 new_gelu
        return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * torch.pow(x, 3.0))))
    if act == "gelu_erf":  # end2end.py:83 F.gelu
        return F.gelu(x)
    raise ValueError(f"unknown activation {act!r}")


def gemm(A, B, b_layout: str = "kn", upcast: bool = False) -> torch.Tensor:
    return product(A, B, b_layout, upcast)


def gemm_bias_act(A, B, bias, act: str = "relu", b_layout: str = "kn", upcast: bool = False) -> torch.Tensor:
    """act((A @ B).to(fp32) + bias) in fp32 (gemm_bias_act.py:44-47)."""
    x = product(A, B, b_layout, upcast) + _cpu(bias).float().unsqueeze(0)
    return activation(x, act)


def gemm_bias_layernorm(A, B, bias, gamma, beta, eps: float = 1e-5, b_layout: str = "kn",
                        out_dtype: torch.dtype = torch.float16, upcast: bool = False) -> torch.Tensor:
    """layer_norm over N of (A @ B).to(fp32) + bias, cast to out_dtype
    (gemm_bias_layernorm.py:44-50; that function returns fp16)."""
    x = product(A, B, b_layout, upcast) + _cpu(bias).float().unsqueeze(0)
    n = x.shape[1]
    y = F.layer_norm(x, (n,), weight=_cpu(gamma).float(), bias=_cpu(beta).float(), eps=eps)
    return y.to(out_dtype)


def _conv_nchw(X, W, stride, padding, dilation, upcast):
    Xn = _cpu(X).permute(0, 3, 1, 2)
    Wn = _cpu(W).permute(3, 2, 0, 1)
    if upcast:
        Xn, Wn = Xn.float(), Wn.float()
    return F.conv2d(Xn, Wn, stride=stride, padding=padding, dilation=dilation)


def conv2d(X, W, stride: int = 1, padding: int = 1, dilation: int = 1,
           out_dtype: torch.dtype = torch.float16, upcast: bool = False) -> torch.Tensor:
    """NHWC conv, weights [KH,KW,C,F] (conv2d.py:35-62); Y cast to out_dtype."""
    return _conv_nchw(X, W, stride, padding, dilation, upcast).permute(0, 2, 3, 1).to(out_dtype)


def conv2d_bias_relu(X, W, bias=None, relu: bool = True, stride: int = 1, padding: int = 1,
                     dilation: int = 1, out_dtype: torch.dtype = torch.float16,
                     upcast: bool = False) -> torch.Tensor:
    """conv2d_relu.py:29-60: conv in the input dtype, .to(fp32), relu, cast.  The optional
    bias (added in fp32 before the relu) is the fused bias of this package's conv op; the
    reference's conv kernels have none."""
    y = _conv_nchw(X, W, stride, padding, dilation, upcast).to(torch.float32)
    if bias is not None:
        y = y + _cpu(bias).float().view(1, -1, 1, 1)
    if relu:
        y = torch.relu(y)
    return y.permute(0, 2, 3, 1).to(out_dtype)


def conv2d_bn(X, W, gamma, beta, mean, var, eps: float = 1e-5, relu: bool = False, residual=None,
              clamp_var: bool = False, stride: int = 1, padding: int = 1, dilation: int = 1,
              out_dtype: torch.dtype = torch.float16, upcast: bool = False) -> torch.Tensor:
    """Conv + BatchNorm (inference form) [+ residual] [+ ReLU], the reference's
    conv2d_bn.py:29-45 (eps 1e-3 there), conv2d_bn_relu.py:123-137 and
    conv_bn_add_relu.py:29-46 (var clamped at 0, residual added before the ReLU): the
    conv in the input dtype, .to(fp32), (y - mean) * rsqrt(var + eps) * gamma + beta."""
    y = _conv_nchw(X, W, stride, padding, dilation, upcast).to(torch.float32)
    g, b, m, v = (_cpu(t).float().view(1, -1, 1, 1) for t in (gamma, beta, mean, var))
    if clamp_var:
        v = torch.clamp(v, min=0.0)
    y = (y - m) * torch.rsqrt(v + eps) * g + b
    if residual is not None:
        y = y + _cpu(residual).permute(0, 3, 1, 2).float()
    if relu:
        y = torch.relu(y)
    return y.permute(0, 2, 3, 1).to(out_dtype)


def conv_flops(n: int, c: int, oh: int, ow: int, f: int, kh: int, kw: int) -> int:
    """2 * N * OH * OW * F * C * KH * KW (conv2d.py:71-72)."""
    return 2 * n * oh * ow * f * c * kh * kw
