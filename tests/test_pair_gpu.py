"""CTA-pair kernels (block_m 256: tcgen05 cta_group::2, each CTA loads half of B) against
the oracle and against the single-CTA kernels, through the C ABI."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from oracle import ref_ops as R
from tests.gpu_util import TOL, TOL_LN, assert_close, cuda, gen, randn, status_clean

pytestmark = pytest.mark.gpu


def pcfg(bn, group_m=8, max_ctas=0):
    return N.tile_cfg(block_n=bn, stages=6 if bn == 256 else 7, group_m=group_m, max_ctas=max_ctas, block_m=256)


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("M,Nn,K", [(512, 512, 256), (333, 264, 200), (1000, 1304, 520)])
def test_pair_gemm(bn, layout, M, Nn, K):
    g = gen(31)
    a = randn(g, M, K, scale=K ** -0.25)
    b = randn(g, *((K, Nn) if layout == "kn" else (Nn, K)), scale=K ** -0.25)
    out = fused.gemm(*cuda(a, b), b_layout=layout, out_dtype=torch.float32, config=pcfg(bn))
    assert_close(out, R.gemm(a, b, layout, upcast=True), dict(atol=1e-4, rtol=1e-4))
    single = fused.gemm(*cuda(a, b), b_layout=layout, out_dtype=torch.float32, config=N.tile_cfg(bn, 4, 8))
    assert torch.equal(out, single)  # same K order per output element
    status_clean()


@pytest.mark.parametrize("M,Nn,K,max_ctas,split_k", [(512, 512, 2048, 0, 0), (1280, 512, 1000, 8, 3),
                                                    (300, 1304, 520, 0, 4), (2304, 2304, 4096, 0, 0)])
def test_pair_split_tail(M, Nn, K, max_ctas, split_k):
    """Pairs whose last partial wave is split along K (each CTA of a pair reduces its own
    128 rows); repeated calls check the self-resetting arrival counters."""
    g = gen(35)
    a, b = randn(g, M, K, scale=K ** -0.25), randn(g, Nn, K, scale=K ** -0.25)
    cfg = N.tile_cfg(block_n=256, stages=6, group_m=8, max_ctas=max_ctas, block_m=256, split_k=split_k)
    nbytes = fused.workspace_bytes(M, Nn, K, "none", cfg)
    assert nbytes > 0
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    ref = R.gemm(a, b, "nk", upcast=True)
    for _ in range(3):
        out = fused.gemm(*cuda(a, b), b_layout="nk", out_dtype=torch.float32, workspace=ws, config=cfg)
        assert_close(out, ref, dict(atol=1e-4, rtol=1e-4))
    assert int(ws[:32].view(torch.int32).abs().sum()) == 0  # first split tile's counters left zeroed
    status_clean()


@pytest.mark.parametrize("act", ["relu", "gelu_tanh"])
def test_pair_bias_act_f16(act):
    g = gen(32)
    a, b = randn(g, 700, 384, dtype=torch.float16, scale=0.3), randn(g, 384, 640, dtype=torch.float16, scale=0.1)
    bias = randn(g, 640, dtype=torch.float16, scale=0.1)
    out = fused.gemm(*cuda(a, b), epilogue=f"bias_{act}", bias=bias.cuda(), config=pcfg(128, max_ctas=20))
    assert_close(out, R.gemm_bias_act(a, b, bias, act), TOL)


def test_pair_layernorm():
    g = gen(33)
    M, Nn, K = 600, 1024, 256
    x, w = randn(g, M, K), randn(g, Nn, K, scale=K ** -0.5)
    bias, gamma, beta = randn(g, Nn, scale=0.02), randn(g, Nn, scale=0.02, shift=1.0), randn(g, Nn, scale=0.02)
    cfg = pcfg(256, group_m=0)
    ws = torch.zeros(fused.ln_workspace_bytes(M, Nn, cfg), dtype=torch.uint8, device="cuda")
    out = fused.gemm(*cuda(x, w), b_layout="nk", epilogue="bias_layernorm", bias=bias.cuda(), gamma=gamma.cuda(),
                     beta=beta.cuda(), workspace=ws, config=cfg)
    assert_close(out, R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=torch.bfloat16), TOL_LN)


@pytest.mark.parametrize("shape", [(4, 28, 28, 128, 128, 3, 1, 1), (3, 13, 11, 24, 256, 3, 2, 1)], ids=str)
def test_pair_conv(shape):
    n, h, w, c, f, k, s, p = shape
    g = gen(34)
    x = randn(g, n, h, w, c)
    wt = randn(g, k, k, c, f, scale=(k * k * c) ** -0.5)
    bias = randn(g, f, scale=0.1)
    out = fused.conv2d_nhwc(*cuda(x, wt), bias=bias.cuda(), relu=True, stride=s, padding=p,
                            config=N.tile_cfg(128 if f <= 128 else 256, 6, 0, block_m=256))
    assert_close(out, R.conv2d_bias_relu(x, wt, bias, True, s, p, 1, out_dtype=torch.bfloat16), TOL)
    status_clean()
