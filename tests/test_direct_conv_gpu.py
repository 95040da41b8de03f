"""Direct (padded-pitch) conv kernel, swap_ab = 2, against the oracle through the C ABI:
each input row loaded once per channel block, filter taps as shifted shared-memory views."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from oracle import ref_ops as R
from tests.gpu_util import TOL, assert_close, cuda, gen, randn, status_clean

pytestmark = pytest.mark.gpu


def dcfg(stages=4, block_k=64, block_n=256):
    """block_n caps the tile's positions (rows of P padded positions); the host picks the
    rows per tile."""
    return N.tile_cfg(block_n=block_n, stages=stages, group_m=0, swap_ab=2, block_k=block_k)


SHAPES = [  # n, h, w, c, f, k, pad
    (2, 28, 28, 128, 128, 3, 1),   # P = 32: 7-row tiles, 4 per image
    (3, 30, 30, 64, 192, 3, 1),    # W + 2 pad = 32 exactly; two channel tiles
    (2, 56, 56, 64, 72, 3, 1),     # P = 64; a partial channel tile (72)
    (1, 28, 28, 64, 64, 5, 2),     # 5x5
    (4, 32, 32, 128, 256, 1, 0),   # 1x1, no padding
    (1, 17, 13, 192, 128, 3, 1),   # ragged image inside one padded row
    (2, 112, 112, 64, 64, 3, 1),   # P = 128
]


@pytest.mark.parametrize("shape", SHAPES, ids=str)
@pytest.mark.parametrize("odt,bk", [(torch.bfloat16, 64), (torch.float32, 64), (torch.bfloat16, 128), (torch.bfloat16, 192)])
def test_direct_conv_bias_relu(shape, odt, bk):
    """block_k 128 / 192: two / three filter taps per weight stage (5x5: a tap count that
    neither divides, 1x1: one)."""
    n, h, w, c, f, k, p = shape
    g = gen(70)
    x = randn(g, n, h, w, c)
    wt = randn(g, k, k, c, f, scale=(k * k * c) ** -0.5)
    bias = randn(g, f, scale=0.1)
    out = fused.conv2d_nhwc(*cuda(x, wt), bias=bias.cuda(), relu=True, padding=p, out_dtype=odt,
                            config=dcfg({64: 4, 128: 3, 192: 2}[bk], bk))
    ref = R.conv2d_bias_relu(x, wt, bias, True, 1, p, 1, out_dtype=odt)
    assert_close(out, ref, TOL)
    status_clean()


@pytest.mark.parametrize("shape", [(2, 28, 28, 128, 128, 3, 1), (1, 17, 13, 192, 128, 3, 1), (3, 30, 30, 64, 64, 5, 2),
                                   (2, 9, 20, 64, 96, 3, 1)], ids=str)
def test_direct_conv_narrow_tiles(shape):
    """block_n 128: at most 128 positions (4 rows of 32) per tile, half of the epilogue
    warps idle; 9 x 20: P = 32 with OH = 9 (tiles of 3 rows, or 4 + 4 + 1)."""
    n, h, w, c, f, k, p = shape
    g = gen(74)
    x = randn(g, n, h, w, c)
    wt = randn(g, k, k, c, f, scale=(k * k * c) ** -0.5)
    bias = randn(g, f, scale=0.1)
    for bn in (128, 256):
        out = fused.conv2d_nhwc(*cuda(x, wt), bias=bias.cuda(), relu=True, padding=p, config=dcfg(4, 64, bn))
        ref = R.conv2d_bias_relu(x, wt, bias, True, 1, p, 1, out_dtype=torch.bfloat16)
        assert_close(out, ref, TOL)
    status_clean()


def test_direct_conv_matches_im2col_kernel_fp16():
    g = gen(71)
    x = randn(g, 3, 28, 28, 128, dtype=torch.float16)
    wt = randn(g, 3, 3, 128, 128, dtype=torch.float16, scale=(9 * 128) ** -0.5)
    a = fused.conv2d_nhwc(*cuda(x, wt), out_dtype=torch.float32, config=dcfg())
    b = fused.conv2d_nhwc(*cuda(x, wt), out_dtype=torch.float32, config=N.tile_cfg(256, 4, 0, swap_ab=1))
    assert_close(a, b, dict(atol=1e-4, rtol=1e-4))


@pytest.mark.parametrize("mode", ["bn", "bn_relu", "bn_add_relu"])
def test_direct_conv_batchnorm(mode):
    g = gen(72)
    n, h, w, c, f = 2, 28, 28, 64, 136
    x, wt = randn(g, n, h, w, c), randn(g, 3, 3, c, f, scale=(9 * c) ** -0.5)
    gamma, beta, mean = randn(g, f), randn(g, f, scale=0.5), randn(g, f, scale=0.5)
    var = (torch.rand(f, generator=g) + 0.5).to(torch.bfloat16)
    res = randn(g, n, h, w, f) if mode == "bn_add_relu" else None
    eps = 1e-3 if mode == "bn" else 1e-5
    out = fused.conv2d_nhwc(*cuda(x, wt), bn=tuple(v.cuda() for v in (gamma, beta, mean, var)), bn_eps=eps,
                            relu=mode != "bn", residual=res.cuda() if res is not None else None, config=dcfg())
    ref = R.conv2d_bn(x, wt, gamma, beta, mean, var, eps=eps, relu=mode != "bn", residual=res,
                      clamp_var=mode == "bn_add_relu", out_dtype=torch.bfloat16)
    assert_close(out, ref, dict(atol=3e-2, rtol=2e-2))
    status_clean()


@pytest.mark.parametrize("kw,msg", [(dict(stride=2), "stride 1"), (dict(c=48), "C % 64"), (dict(w=300), "<= 256")])
def test_direct_conv_rejects(kw, msg):
    geo = dict(n=1, h=16, w=16, c=64, f=64, k=3, stride=1)
    geo.update(kw)
    x = torch.zeros(geo["n"], geo["h"], geo["w"], geo["c"], dtype=torch.bfloat16, device="cuda")
    wt = torch.zeros(3, 3, geo["c"], geo["f"], dtype=torch.bfloat16, device="cuda")
    with pytest.raises(N.FoError, match=msg):
        fused.conv2d_nhwc(x, wt, stride=geo["stride"], config=dcfg())
