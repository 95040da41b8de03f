"""NHWC conv2d + BatchNorm (inference form) + residual add + ReLU as implicit GEMM
(reference kernel/tilelang/conv/conv_bn_add_relu.py; eps 1e-5, var clamped at 0).  The
residual [n, oh, ow, f] is read in the epilogue next to the accumulator tile.  Reference
surface kept: get_ref_program, build_conv2d_bn_add_relu_kernel(n, c, h, w, f_out, kh, kw,
s=1, p=1, d=1, config=None) -> kernel(x, w, residual, bn_gamma, bn_beta, bn_mean, bn_var,
y), estimate_total_flops, verify_correctness, ConvBnAddReluDescriptor / DESCRIPTOR.
"""
from __future__ import annotations

import torch

from ..autotuner.cost_model import FusionPrimitive
from .conv2d import Conv2dDescriptor, calc_oh_ow
from .conv2d_bn import bn_reference, build_bn_kernel

EPS = 1e-5


def get_ref_program(stride=1, padding=1, dilation=1, eps=EPS):
    """The reference's expected result (conv_bn_add_relu.py:29-70):
    ref(x, w, residual, gamma, beta, mean, var, y)."""
    inner = bn_reference(stride, padding, dilation, eps, relu=True, clamp_var=True)

    def ref_program(x, w, residual, bn_gamma, bn_beta, bn_mean, bn_var, y):
        inner(x, w, bn_gamma, bn_beta, bn_mean, bn_var, y, residual=residual)

    return ref_program


# The residual tile read next to the accumulator (2 bytes per output); the B200 cost
# model charges its load time to each tile.
RESIDUAL_ADD = FusionPrimitive("residual_add", 1.0, 2.0)


class ConvBnAddReluDescriptor(Conv2dDescriptor):
    primitives = ("batchnorm", RESIDUAL_ADD, "relu")

    @property
    def name(self) -> str:
        return "conv_bn_add_relu"


DESCRIPTOR = ConvBnAddReluDescriptor()


def estimate_total_flops(n, oh, ow, f_out, c, kh, kw):
    """Conv FLOPs plus ~8 per output for BatchNorm + add + ReLU (conv_bn_add_relu.py:179-186)."""
    return 2 * n * oh * ow * f_out * c * kh * kw + 8 * n * oh * ow * f_out


def build_conv2d_bn_add_relu_kernel(n, c, h, w, f_out, kh, kw, s=1, p=1, d=1, config=None):
    """Returns kernel(x, w, residual, bn_gamma, bn_beta, bn_mean, bn_var, y):
    y = relu(bn(conv(x, w)) + residual), in place."""
    return build_bn_kernel(DESCRIPTOR, n, c, h, w, f_out, kh, kw, s, p, d, config, EPS, True, True)


def verify_correctness(kernel, ref_prog, n, c, h, w, f_out, kh, kw, s, p, d, seed=None):
    """The reference's check (conv_bn_add_relu.py:188-216): randn fp16 inputs and residual,
    var = rand + 0.5, assert_close(rtol = atol = 1e-2)."""
    g = torch.Generator(device="cuda")
    if seed is not None:
        g.manual_seed(seed)
    oh, ow = calc_oh_ow(h, w, kh, kw, s, p, d)
    x = torch.randn(n, h, w, c, dtype=torch.float16, device="cuda", generator=g)
    wt = torch.randn(kh, kw, c, f_out, dtype=torch.float16, device="cuda", generator=g)
    residual = torch.randn(n, oh, ow, f_out, dtype=torch.float16, device="cuda", generator=g)
    gamma, beta, mean = (torch.randn(f_out, dtype=torch.float16, device="cuda", generator=g) for _ in range(3))
    var = torch.rand(f_out, dtype=torch.float16, device="cuda", generator=g) + 0.5
    y_ref = torch.zeros(n, oh, ow, f_out, dtype=torch.float16, device="cuda")
    y = torch.zeros_like(y_ref)
    ref_prog(x, wt, residual, gamma, beta, mean, var, y_ref)
    kernel(x, wt, residual, gamma, beta, mean, var, y)
    try:
        torch.testing.assert_close(y, y_ref, rtol=1e-2, atol=1e-2)
        return True
    except AssertionError:
        return False
