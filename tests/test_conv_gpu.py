"""Implicit-GEMM conv2d against the oracle, through the C ABI."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from icpp_tuning_b200.conv import conv2d, conv2d_relu
from oracle import ref_ops as R
from tests.gpu_util import TOL, assert_close, cuda, gen, randn, status_clean

pytestmark = pytest.mark.gpu

SHAPES = [  # n, h, w, c, f, k, stride, pad, dil
    (2, 8, 8, 64, 64, 3, 1, 1, 1),
    (3, 13, 11, 24, 72, 3, 2, 1, 1),
    (1, 17, 9, 136, 128, 3, 1, 1, 1),  # C not a multiple of 64
    (2, 10, 10, 16, 32, 5, 1, 2, 1),
    (2, 12, 12, 32, 64, 3, 1, 2, 2),   # dilation
    (4, 7, 7, 64, 256, 1, 1, 0, 1),    # 1x1
    (1, 9, 7, 8, 16, 3, 2, 0, 1),
]


@pytest.mark.parametrize("shape", SHAPES, ids=str)
@pytest.mark.parametrize("bn", [64, 128, 256])
def test_conv_bias_relu(shape, bn):
    n, h, w, c, f, k, s, p, d = shape
    g = gen(20)
    x = randn(g, n, h, w, c)
    wt = randn(g, k, k, c, f, scale=(k * k * c) ** -0.5)
    bias = randn(g, f, scale=0.1)
    cfg = N.tile_cfg(bn, {256: 4, 128: 6, 64: 8}[bn], 0)
    out = fused.conv2d_nhwc(*cuda(x, wt), bias=bias.cuda(), relu=True, stride=s, padding=p, dilation=d, config=cfg)
    assert_close(out, R.conv2d_bias_relu(x, wt, bias, True, s, p, d, out_dtype=torch.bfloat16), TOL)
    status_clean()


@pytest.mark.parametrize("odt", [torch.float16, torch.float32])
def test_conv_plain_reference_api(odt):
    n, c, h, w, f, k = 2, 32, 9, 9, 48, 3
    g = gen(21)
    x = randn(g, n, h, w, c, dtype=torch.float16)
    wt = randn(g, k, k, c, f, dtype=torch.float16, scale=(k * k * c) ** -0.5)
    kern = conv2d.build_conv2d_kernel(n, c, h, w, f, k, k, 1, 1, 1)
    y = torch.zeros(n, h, w, f, dtype=odt, device="cuda")
    kern(*cuda(x, wt), y)
    assert_close(y, R.conv2d(x, wt, out_dtype=odt), TOL)


def test_verify_correctness_helper():
    kern = conv2d.build_conv2d_kernel(2, 16, 8, 8, 32, 3, 3)
    assert conv2d.verify_correctness(kern, conv2d.get_ref_program(1, 1, 1), 2, 16, 8, 8, 32, 3, 3, 1, 1, 1, seed=0)


def test_config5_conv_full():
    """Config 5: batch 256, 28x28, 128 -> 128, 3x3 s1 p1, bias + ReLU, bf16, seed 4."""
    g = gen(4)
    x = randn(g, 256, 28, 28, 128)
    wt = randn(g, 3, 3, 128, 128, scale=(9 * 128) ** -0.5)
    bias = randn(g, 128, scale=0.1)
    kern = conv2d_relu.build_conv2d_relu_kernel(256, 128, 28, 28, 128, 3, 3, 1, 1, 1)
    y = torch.empty(256, 28, 28, 128, dtype=torch.bfloat16, device="cuda")
    kern(*cuda(x, wt), y, bias=bias.cuda())
    # every image (the CPU oracle takes well under a second for all 256)
    ref = R.conv2d_bias_relu(x, wt, bias, True, 1, 1, 1, out_dtype=torch.bfloat16)
    assert_close(y, ref, TOL)
    status_clean()


@pytest.mark.parametrize("shape", SHAPES, ids=str)
@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("odt", [torch.bfloat16, torch.float32])
def test_conv_swapped_operands(shape, bn, odt):
    """swap_ab: Y^T = W^T X^T (M = output channels, N = pixels), transposing epilogue."""
    n, h, w, c, f, k, s, p, d = shape
    g = gen(22)
    x = randn(g, n, h, w, c)
    wt = randn(g, k, k, c, f, scale=(k * k * c) ** -0.5)
    bias = randn(g, f, scale=0.1)
    cfg = N.tile_cfg(bn, 4 if bn == 256 else 6, 0, swap_ab=1)
    out = fused.conv2d_nhwc(*cuda(x, wt), bias=bias.cuda(), relu=True, stride=s, padding=p, dilation=d,
                            out_dtype=odt, config=cfg)
    assert_close(out, R.conv2d_bias_relu(x, wt, bias, True, s, p, d, out_dtype=odt), TOL)
    status_clean()


@pytest.mark.parametrize("swap", [0, 1])
def test_conv_split_tail(swap):
    """A partial last wave split along K (workspace given) matches the whole-tile result."""
    n, h, w, c, f = 56, 28, 28, 256, 128  # a partial last wave for both tilings, K = 36 k-blocks
    g = gen(23)
    x = randn(g, n, h, w, c)
    wt = randn(g, 3, 3, c, f, scale=(9 * c) ** -0.5)
    bias = randn(g, f, scale=0.1)
    cfg = N.tile_cfg(256 if swap else 128, 4, 0, swap_ab=swap)
    nbytes = fused.conv_workspace_bytes(n, h, w, c, f, 3, 3, config=cfg)
    assert nbytes > 0
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    xd, wd_, bd = cuda(x, wt, bias)
    whole = fused.conv2d_nhwc(xd, wd_, bias=bd, relu=True, config=cfg)
    for _ in range(2):
        split = fused.conv2d_nhwc(xd, wd_, bias=bd, relu=True, workspace=ws, config=cfg)
        torch.testing.assert_close(split.float(), whole.float(), atol=1e-2, rtol=1e-2)
    assert_close(split[:4], R.conv2d_bias_relu(x[:4], wt, bias, True, 1, 1, 1, out_dtype=torch.bfloat16), TOL)
    assert int(ws[:256].view(torch.int32).abs().sum()) == 0
    status_clean()
