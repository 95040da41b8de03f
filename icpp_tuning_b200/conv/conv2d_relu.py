"""NHWC conv2d + (bias) + ReLU as implicit GEMM (reference
kernel/tilelang/conv/conv2d_relu.py).

The reference fuses ReLU in fp32 after the conv (:133-139) and has no bias; here the
bias (fp32, before the ReLU) is an optional call argument, which the BASELINE conv
workload uses.  Reference surface kept: get_ref_program, build_conv2d_relu_kernel(N, C,
H, W, F_out, KH, KW, S=1, P=1, D=1, config=None) -> kernel(X, W, Y), estimate_total_flops,
Conv2dReluDescriptor / DESCRIPTOR.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import fused
from .conv2d import Conv2dDescriptor, _select, calc_oh_ow


def get_ref_program(stride=1, padding=1, dilation=1):
    """The reference's expected result (conv2d_relu.py:29-60): relu(conv(X, W)) in fp32,
    cast to Y's dtype.  Eager PyTorch."""

    def ref_program(X, W, Y, bias=None):
        y = F.conv2d(X.permute(0, 3, 1, 2), W.permute(3, 2, 0, 1), stride=stride, padding=padding,
                     dilation=dilation).to(torch.float32)
        if bias is not None:
            y = y + bias.float().view(1, -1, 1, 1)
        Y.copy_(torch.relu(y).permute(0, 2, 3, 1).to(Y.dtype))

    return ref_program


class Conv2dReluDescriptor(Conv2dDescriptor):
    primitives = ("relu",)

    @property
    def name(self) -> str:
        return "conv2d_relu"


DESCRIPTOR = Conv2dReluDescriptor()


def estimate_total_flops(N, OH, OW, F_out, C, KH, KW):
    """Conv FLOPs plus one per output for the ReLU (conv2d_relu.py:158-163)."""
    return 2 * N * OH * OW * F_out * C * KH * KW + N * OH * OW * F_out


def build_conv2d_relu_kernel(N, C, H, W, F_out, KH, KW, S=1, P=1, D=1, config=None):
    """Returns kernel(X, W, Y, bias=None): Y = relu(conv(X, W) + bias), in place."""
    config = _select(DESCRIPTOR, N, C, H, W, F_out, KH, KW, S, P, config)
    cfg = fused.as_tile_cfg(config)
    OH, OW = calc_oh_ow(H, W, KH, KW, S, P, D)
    ws_bytes = fused.conv_workspace_bytes(N, H, W, C, F_out, KH, KW, S, P, D, config=cfg)
    # zero-filled once per stream; the kernel leaves its split-K counters zeroed after every call
    wss = fused.StreamWorkspaces(ws_bytes)

    def kernel(X, Wt, Y, bias=None):
        if tuple(X.shape) != (N, H, W, C) or tuple(Wt.shape) != (KH, KW, C, F_out):
            raise ValueError("input shapes differ from the built shape")
        fused.conv2d_nhwc(X, Wt, bias=bias, relu=True, stride=S, padding=P, dilation=D, out=Y, workspace=wss.get(), config=cfg)
        return Y

    kernel.config = config
    kernel.out_shape = (N, OH, OW, F_out)
    kernel.workspace = wss.default
    return kernel
