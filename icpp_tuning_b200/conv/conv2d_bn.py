"""NHWC conv2d + BatchNorm (inference form) as implicit GEMM (reference
kernel/tilelang/conv/conv2d_bn.py).

The reference applies bn(y) = (y - mean) / sqrt(var + eps) * gamma + beta to the fp16
conv tile in its epilogue (:141-154, eps 1e-3).  Here the epilogue folds the four
vectors into one per-channel (scale, shift) in fp32 and applies it to the fp32
accumulator.  Reference surface kept: get_ref_program, build_conv2d_bn_kernel(N, C, H, W,
F_out, KH, KW, S=1, P=1, D=1, config=None) -> kernel(X, W, BN_Gamma, BN_Beta, BN_Mean,
BN_Var, Y), estimate_total_flops, verify_correctness, Conv2dBnDescriptor / DESCRIPTOR.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import fused
from .conv2d import Conv2dDescriptor, _select, calc_oh_ow

EPS = 1e-3


def bn_reference(stride=1, padding=1, dilation=1, eps=EPS, relu=False, clamp_var=False):
    """ref(X, W, gamma, beta, mean, var, Y[, residual]): the reference functions' math
    (conv in the input dtype, then fp32 BatchNorm), eager PyTorch on the tensors' device."""

    def ref_program(X, W, BN_Gamma, BN_Beta, BN_Mean, BN_Var, Y, residual=None):
        y = F.conv2d(X.permute(0, 3, 1, 2), W.permute(3, 2, 0, 1), stride=stride, padding=padding,
                     dilation=dilation).to(torch.float32)
        g, b, m, v = (t.to(torch.float32).view(1, -1, 1, 1) for t in (BN_Gamma, BN_Beta, BN_Mean, BN_Var))
        if clamp_var:
            v = torch.clamp(v, min=0.0)
        y = (y - m) * torch.rsqrt(v + eps) * g + b
        if residual is not None:
            y = y + residual.permute(0, 3, 1, 2).to(torch.float32)
        if relu:
            y = torch.relu(y)
        Y.copy_(y.permute(0, 2, 3, 1).to(Y.dtype))

    return ref_program


def get_ref_program(stride=1, padding=1, dilation=1, eps=EPS):
    """The reference's expected result (conv2d_bn.py:29-64)."""
    return bn_reference(stride, padding, dilation, eps)


class Conv2dBnDescriptor(Conv2dDescriptor):
    primitives = ("batchnorm",)

    @property
    def name(self) -> str:
        return "conv2d_bn"


DESCRIPTOR = Conv2dBnDescriptor()


def estimate_total_flops(N, OH, OW, F_out, C, KH, KW):
    """Conv FLOPs plus ~6 per output for the BatchNorm (conv2d_bn.py:169-175)."""
    return 2 * N * OH * OW * F_out * C * KH * KW + 6 * N * OH * OW * F_out


def build_bn_kernel(desc, N, C, H, W, F_out, KH, KW, S, P, D, config, eps, relu, with_residual):
    """Shared builder of the three BatchNorm conv operators."""
    config = _select(desc, N, C, H, W, F_out, KH, KW, S, P, config)
    cfg = fused.as_tile_cfg(config)
    OH, OW = calc_oh_ow(H, W, KH, KW, S, P, D)
    ws_bytes = fused.conv_workspace_bytes(N, H, W, C, F_out, KH, KW, S, P, D, config=cfg)
    # zero-filled once per stream; the kernel leaves its split-K counters zeroed after every call
    wss = fused.StreamWorkspaces(ws_bytes)

    def run(X, Wt, bn, Y, residual=None):
        if tuple(X.shape) != (N, H, W, C) or tuple(Wt.shape) != (KH, KW, C, F_out):
            raise ValueError("input shapes differ from the built shape")
        fused.conv2d_nhwc(X, Wt, bn=bn, bn_eps=eps, relu=relu, residual=residual, stride=S, padding=P, dilation=D,
                          out=Y, workspace=wss.get(), config=cfg)
        return Y

    if with_residual:
        def kernel(X, Wt, residual, BN_Gamma, BN_Beta, BN_Mean, BN_Var, Y):
            return run(X, Wt, (BN_Gamma, BN_Beta, BN_Mean, BN_Var), Y, residual)
    else:
        def kernel(X, Wt, BN_Gamma, BN_Beta, BN_Mean, BN_Var, Y):
            return run(X, Wt, (BN_Gamma, BN_Beta, BN_Mean, BN_Var), Y)

    kernel.config = config
    kernel.out_shape = (N, OH, OW, F_out)
    kernel.workspace = wss.default
    return kernel


def build_conv2d_bn_kernel(N, C, H, W, F_out, KH, KW, S=1, P=1, D=1, config=None):
    """Returns kernel(X, W, BN_Gamma, BN_Beta, BN_Mean, BN_Var, Y): Y = bn(conv(X, W)), in place."""
    return build_bn_kernel(DESCRIPTOR, N, C, H, W, F_out, KH, KW, S, P, D, config, EPS, False, False)


def verify_correctness(kernel, ref_prog, N, C, H, W, F_out, KH, KW, S, P, D, seed=None):
    """The reference's check (conv2d_bn.py:177-205): randn fp16 inputs, mean / var the
    per-channel batch statistics of the conv output, assert_close(rtol = atol = 1e-2)."""
    g = torch.Generator(device="cuda")
    if seed is not None:
        g.manual_seed(seed)
    OH, OW = calc_oh_ow(H, W, KH, KW, S, P, D)
    X = torch.randn(N, H, W, C, dtype=torch.float16, device="cuda", generator=g)
    Wt = torch.randn(KH, KW, C, F_out, dtype=torch.float16, device="cuda", generator=g)
    gamma = torch.randn(F_out, dtype=torch.float16, device="cuda", generator=g)
    beta = torch.randn(F_out, dtype=torch.float16, device="cuda", generator=g)
    y = F.conv2d(X.permute(0, 3, 1, 2), Wt.permute(3, 2, 0, 1), stride=S, padding=P, dilation=D).float()
    mean = y.mean(dim=(0, 2, 3)).half()
    var = y.var(dim=(0, 2, 3), unbiased=False).half()
    Y_ref = torch.zeros(N, OH, OW, F_out, dtype=torch.float16, device="cuda")
    Y = torch.zeros_like(Y_ref)
    ref_prog(X, Wt, gamma, beta, mean, var, Y_ref)
    kernel(X, Wt, gamma, beta, mean, var, Y)
    try:
        torch.testing.assert_close(Y, Y_ref, rtol=1e-2, atol=1e-2)
        return True
    except AssertionError:
        return False
