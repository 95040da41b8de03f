"""Conv + BatchNorm epilogues (reference conv2d_bn / conv2d_bn_relu / conv_bn_add_relu)
against the oracle, through the C ABI, on every conv kernel variant."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from icpp_tuning_b200.conv import conv2d_bn, conv2d_bn_relu, conv_bn_add_relu
from oracle import ref_ops as R
from tests.gpu_util import assert_close, cuda, gen, randn, status_clean

pytestmark = pytest.mark.gpu
TOL_BN = dict(atol=3e-2, rtol=2e-2)  # BatchNorm scales reach ~|gamma| / sqrt(0.5); bf16 output

CFGS = {  # name -> tile config
    "bn64": N.tile_cfg(64, 8, 0), "bn128": N.tile_cfg(128, 6, 0), "bn256": N.tile_cfg(256, 4, 0),
    "swap128": N.tile_cfg(128, 4, 0, swap_ab=1), "swap256": N.tile_cfg(256, 4, 0, swap_ab=1),
    "pair256": N.tile_cfg(256, 6, 0, block_m=256),
}
SHAPES = [(2, 12, 12, 64, 72, 3, 1, 1), (3, 13, 11, 24, 136, 3, 2, 1), (4, 14, 14, 128, 256, 1, 1, 0)]
MODES = {"bn": (1e-3, False, False), "bn_relu": (1e-5, True, False), "bn_add_relu": (1e-5, True, True)}


def _bn_vectors(g, f, dt):
    gamma, beta, mean = randn(g, f, dtype=dt), randn(g, f, dtype=dt, scale=0.5), randn(g, f, dtype=dt, scale=0.5)
    var = (torch.rand(f, generator=g) + 0.5).to(dt)
    return gamma, beta, mean, var


@pytest.mark.parametrize("cfg", list(CFGS), ids=str)
@pytest.mark.parametrize("shape", SHAPES, ids=str)
@pytest.mark.parametrize("mode", list(MODES))
def test_conv_bn_epilogues(cfg, shape, mode):
    n, h, w, c, f, k, s, p = shape
    eps, relu, add = MODES[mode]
    g = gen(50)
    x = randn(g, n, h, w, c)
    wt = randn(g, k, k, c, f, scale=(k * k * c) ** -0.5)
    bn = _bn_vectors(g, f, torch.bfloat16)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    res = randn(g, n, oh, ow, f) if add else None
    tile = CFGS[cfg]
    ws_bytes = fused.conv_workspace_bytes(n, h, w, c, f, k, k, s, p, 1, config=tile)
    ws = torch.zeros(max(16, ws_bytes), dtype=torch.uint8, device="cuda")
    out = fused.conv2d_nhwc(*cuda(x, wt), bn=tuple(v.cuda() for v in bn), bn_eps=eps, relu=relu,
                            residual=res.cuda() if add else None, stride=s, padding=p, workspace=ws, config=tile)
    # the conv in bf16 (rounded before the BatchNorm), as the reference computes it
    ref = R.conv2d_bn(x, wt, *bn, eps=eps, relu=relu, residual=res, clamp_var=add, stride=s, padding=p,
                      out_dtype=torch.bfloat16)
    assert_close(out, ref, TOL_BN)
    status_clean()


def test_bn_add_relu_clamps_negative_variance():
    """conv_bn_add_relu clamps var at 0 (conv_bn_add_relu.py:40); a negative var with eps
    1e-5 gives the same finite result as var = 0."""
    g = gen(51)
    n, h, w, c, f = 2, 8, 8, 32, 64
    x, wt = randn(g, n, h, w, c), randn(g, 3, 3, c, f, scale=(9 * c) ** -0.5)
    gamma, beta, mean, var = _bn_vectors(g, f, torch.bfloat16)
    var[::3] = -0.25
    res = randn(g, n, h, w, f)
    out = fused.conv2d_nhwc(*cuda(x, wt), bn=tuple(v.cuda() for v in (gamma, beta, mean, var)), relu=True,
                            residual=res.cuda())
    ref = R.conv2d_bn(x, wt, gamma, beta, mean, var, eps=1e-5, relu=True, residual=res, clamp_var=True,
                      out_dtype=torch.bfloat16)
    assert torch.isfinite(out.float()).all()
    # var = 0: the scale is gamma * rsqrt(1e-5) ~ 316 |gamma|, so compare relative to it
    assert_close(out, ref, dict(atol=0.5, rtol=2e-2))


@pytest.mark.parametrize("mod,builder,shape", [
    (conv2d_bn, "build_conv2d_bn_kernel", (2, 64, 14, 14, 64, 3, 3, 1, 1)),
    (conv2d_bn_relu, "build_conv2d_bn_relu_kernel", (2, 32, 16, 16, 128, 3, 3, 1, 1)),
    (conv_bn_add_relu, "build_conv2d_bn_add_relu_kernel", (2, 64, 14, 14, 192, 3, 3, 2, 1)),
], ids=["conv2d_bn", "conv2d_bn_relu", "conv_bn_add_relu"])
def test_reference_api_verify_correctness(mod, builder, shape):
    """Each module's build_*_kernel passes its reference-style verify_correctness (fp16)."""
    N_, C, H, W, F_out, KH, KW, S, P = shape
    kernel = getattr(mod, builder)(N_, C, H, W, F_out, KH, KW, S, P, 1)
    assert mod.verify_correctness(kernel, mod.get_ref_program(S, P, 1), N_, C, H, W, F_out, KH, KW, S, P, 1, seed=7)
    status_clean()
