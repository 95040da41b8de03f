"""NHWC conv2d + BatchNorm (inference form) + ReLU as implicit GEMM (reference
kernel/tilelang/conv/conv2d_bn_relu.py; eps 1e-5).  Reference surface kept:
get_ref_program, build_conv2d_bn_relu_kernel(N, C, H, W, F_out, KH, KW, S=1, P=1, D=1,
config=None) -> kernel(X, W, BN_Gamma, BN_Beta, BN_Mean, BN_Var, Y), estimate_total_flops,
verify_correctness, Conv2dBnReluDescriptor / DESCRIPTOR.
"""
from __future__ import annotations

import torch

from .conv2d import Conv2dDescriptor, calc_oh_ow
from .conv2d_bn import bn_reference, build_bn_kernel

EPS = 1e-5


def get_ref_program(stride=1, padding=1, dilation=1, eps=EPS):
    """The reference's expected result (conv2d_bn_relu.py:123-160)."""
    return bn_reference(stride, padding, dilation, eps, relu=True)


class Conv2dBnReluDescriptor(Conv2dDescriptor):
    primitives = ("batchnorm", "relu")

    @property
    def name(self) -> str:
        return "conv2d_bn_relu"


DESCRIPTOR = Conv2dBnReluDescriptor()


def estimate_total_flops(N, OH, OW, F_out, C, KH, KW):
    """Conv FLOPs plus ~7 per output for BatchNorm + ReLU (conv2d_bn_relu.py:282-290)."""
    return 2 * N * OH * OW * F_out * C * KH * KW + 7 * N * OH * OW * F_out


def build_conv2d_bn_relu_kernel(N, C, H, W, F_out, KH, KW, S=1, P=1, D=1, config=None):
    """Returns kernel(X, W, BN_Gamma, BN_Beta, BN_Mean, BN_Var, Y): Y = relu(bn(conv)), in place."""
    return build_bn_kernel(DESCRIPTOR, N, C, H, W, F_out, KH, KW, S, P, D, config, EPS, True, False)


def verify_correctness(kernel, ref_prog, N, C, H, W, F_out, KH, KW, S, P, D, seed=None):
    """The reference's check (conv2d_bn_relu.py:293-316): randn fp16 inputs, var = rand + 0.5,
    assert_close(rtol = atol = 1e-2)."""
    g = torch.Generator(device="cuda")
    if seed is not None:
        g.manual_seed(seed)
    OH, OW = calc_oh_ow(H, W, KH, KW, S, P, D)
    X = torch.randn(N, H, W, C, dtype=torch.float16, device="cuda", generator=g)
    Wt = torch.randn(KH, KW, C, F_out, dtype=torch.float16, device="cuda", generator=g)
    gamma, beta, mean = (torch.randn(F_out, dtype=torch.float16, device="cuda", generator=g) for _ in range(3))
    var = torch.rand(F_out, dtype=torch.float16, device="cuda", generator=g) + 0.5
    Y_ref = torch.zeros(N, OH, OW, F_out, dtype=torch.float16, device="cuda")
    Y = torch.zeros_like(Y_ref)
    ref_prog(X, Wt, gamma, beta, mean, var, Y_ref)
    kernel(X, Wt, gamma, beta, mean, var, Y)
    try:
        torch.testing.assert_close(Y, Y_ref, rtol=1e-2, atol=1e-2)
        return True
    except AssertionError:
        return False
