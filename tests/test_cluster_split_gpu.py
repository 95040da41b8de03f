"""Cluster split-K (split_mode 2, and the automatic choice): the parts of a tile run as one
thread-block cluster and reduce-scatter their fp32 partials through distributed shared
memory.  Against the oracle through the C ABI, bitwise reproducible, and rejected with
FO_EINVAL where it cannot run."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from oracle import ref_ops as R
from tests.gpu_util import TOL, assert_close, cuda, gen, randn, status_clean

pytestmark = pytest.mark.gpu


def _inputs(seed, M, Nn, K, dt=torch.bfloat16, layout="kn"):
    g = gen(seed)
    a = randn(g, M, K, dtype=dt, scale=K ** -0.25)
    b = randn(g, *((K, Nn) if layout == "kn" else (Nn, K)), dtype=dt, scale=K ** -0.25)
    return a, b, randn(g, Nn, dtype=dt, scale=0.1)


def _cfg(bn, s, stages=4, bk=64, mode=N.SPLIT_CLUSTER):
    return N.tile_cfg(bn, stages, 0, block_k=bk, split_k=s, split_mode=mode)


@pytest.mark.parametrize("bn,bk,s", [(64, 128, 2), (64, 128, 3), (64, 64, 4), (64, 64, 8), (128, 64, 2),
                                     (128, 128, 4), (128, 64, 6), (256, 64, 2)])
def test_cluster_split_gelu(bn, bk, s):
    M, Nn, K = 128, 512, 768  # 8 tiles of 64 columns: every part count fits the GPU
    a, b, bias = _inputs(80 + s, M, Nn, K)
    stages = 3 if bn == 256 or (bn == 128 and bk == 128) else 4
    out = fused.gemm(*cuda(a, b), epilogue="bias_gelu_erf", bias=bias.cuda(), config=_cfg(bn, s, stages, bk))
    assert_close(out, R.gemm_bias_act(a, b, bias, "gelu_erf"), TOL)
    status_clean()


@pytest.mark.parametrize("odt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_cluster_split_ragged(odt, layout):
    """M, N and K off the tile grid: a partial 32-column chunk, rows past M, a short last part."""
    M, Nn, K = 200, 1000, 1000
    dt = torch.float16 if odt == torch.float16 else torch.bfloat16
    a, b, bias = _inputs(90, M, Nn, K, dt, layout)
    out = fused.gemm(*cuda(a, b), b_layout=layout, epilogue="bias_relu", bias=bias.cuda(), out_dtype=odt,
                     config=_cfg(64, 3))
    assert out.dtype == odt
    assert_close(out, R.gemm_bias_act(a, b, bias, "relu", layout), TOL)
    status_clean()


def test_cluster_split_fp32_matches_upcast_product():
    M, Nn, K = 256, 512, 2048
    a, b, _ = _inputs(91, M, Nn, K)
    out = fused.gemm(*cuda(a, b), out_dtype=torch.float32, config=_cfg(128, 4))
    assert_close(out, R.gemm(a, b, upcast=True), dict(atol=1e-4, rtol=1e-4))


def test_cluster_split_is_bitwise_reproducible():
    M, Nn, K = 128, 768, 768  # 12 tiles x 6 parts
    a, b, bias = (t.cuda() for t in _inputs(92, M, Nn, K))
    outs = [fused.gemm(a, b, epilogue="bias_gelu_tanh", bias=bias, out_dtype=torch.float32, config=_cfg(64, 6))
            for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_cluster_split_residual_layernorm():
    """The residual LayerNorm path's GEMM (bias store, then the row pass) split by clusters."""
    M, Nn, K = 128, 768, 3072
    g = gen(93)
    dt = torch.float16
    a, b = randn(g, M, K, dtype=dt, scale=0.5), randn(g, K, Nn, dtype=dt, scale=K ** -0.5)
    bias, res = randn(g, Nn, dtype=dt, scale=0.1), randn(g, M, Nn, dtype=dt)
    gamma, beta = randn(g, Nn, dtype=dt, scale=0.1, shift=1.0), randn(g, Nn, dtype=dt, scale=0.1)
    a, b, bias, res, gamma, beta = (t.cuda() for t in (a, b, bias, res, gamma, beta))
    out = fused.gemm(a, b, epilogue="bias_residual_layernorm", bias=bias, gamma=gamma, beta=beta, residual=res,
                     config=_cfg(64, 4, bk=128))
    y = (a.float() @ b.float() + bias.float()).to(dt)
    ref = F.layer_norm((y + res).float(), (Nn,), gamma.float(), beta.float(), 1e-5)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    status_clean()


@pytest.mark.parametrize("M,Nn,K", [(128, 768, 3072), (64, 4096, 1024), (1024, 1024, 1024)])
def test_automatic_split_without_workspace(M, Nn, K):
    """split_mode 0 without a workspace: small problems take the cluster split."""
    a, b, bias = _inputs(94, M, Nn, K)
    out = fused.gemm(*cuda(a, b), epilogue="bias_relu", bias=bias.cuda(), config=N.tile_cfg(128, 6, 8))
    assert_close(out, R.gemm_bias_act(a, b, bias, "relu"), TOL)
    status_clean()


def _call(M, Nn, K, cfg, epilogue=N.FO_EPI_NONE, ws=None):
    a = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(K, Nn, dtype=torch.bfloat16, device="cuda")
    o = torch.zeros(M, Nn, dtype=torch.bfloat16, device="cuda")
    v = torch.ones(Nn, dtype=torch.bfloat16, device="cuda")
    d = N.FoGemmDesc()
    d.M, d.N, d.K = M, Nn, K
    d.a, d.b, d.out, d.bias, d.gamma, d.beta = a.data_ptr(), b.data_ptr(), o.data_ptr(), v.data_ptr(), v.data_ptr(), v.data_ptr()
    d.lda, d.ldb, d.ldo = K, Nn, Nn
    d.in_dtype = d.out_dtype = d.vec_dtype = N.FO_DT_BF16
    d.b_layout, d.epilogue, d.eps = N.FO_B_KN, epilogue, 1e-5
    if ws is not None:
        d.workspace, d.workspace_bytes = ws.data_ptr(), ws.numel()
    rc = N.lib().fo_gemm(ctypes.byref(d), ctypes.byref(cfg), None)
    torch.cuda.synchronize()
    return rc


def test_cluster_split_rejections():
    assert _call(128, 512, 512, _cfg(64, 9)) == N.FO_EINVAL           # more than 8 parts
    assert "cluster split" in N.last_error()
    assert _call(4096, 4096, 512, _cfg(128, 2)) == N.FO_EINVAL        # a whole wave of tiles
    assert _call(128, 512, 128, _cfg(64, 4, bk=128)) == N.FO_EINVAL   # empty parts
    assert _call(128, 512, 512, _cfg(64, 2, mode=3)) == N.FO_EINVAL   # bad split_mode
    assert "split_mode" in N.last_error()
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    assert _call(128, 512, 512, _cfg(64, 2), N.FO_EPI_BIAS_LN, ws) == N.FO_EINVAL  # in-kernel LayerNorm
    assert _call(128, 512, 512, _cfg(64, 2)) == N.FO_OK


@pytest.mark.parametrize("bm,bn,st,s,max_ctas", [(128, 128, 6, 2, 0), (128, 64, 8, 3, 0), (256, 256, 4, 2, 0),
                                                 (256, 128, 6, 3, 0), (128, 128, 6, 3, 16), (128, 256, 4, 4, 8)])
def test_workspace_split_staged_and_fallback(bm, bn, st, s, max_ctas):
    """Workspace split-K: the last-arriving part stages the other parts' blocks in the idle
    pipeline ring with bulk copies (a CTA's only split unit), or reads them from L2 (a small
    max_ctas gives CTAs several split units); both sum the parts in part order."""
    M, Nn, K = 600, 1000, 2048
    a, b, bias = _inputs(95, M, Nn, K, layout="nk")
    cfg = N.tile_cfg(bn, st, 8, block_m=bm, max_ctas=max_ctas, split_k=s, split_mode=N.SPLIT_WORKSPACE)
    ws = torch.zeros(fused.workspace_bytes(M, Nn, K, "bias_gelu_tanh", cfg), dtype=torch.uint8, device="cuda")
    assert ws.numel() > 0
    a, b, bias = a.cuda(), b.cuda(), bias.cuda()
    outs = [fused.gemm(a, b, b_layout="nk", epilogue="bias_gelu_tanh", bias=bias, out_dtype=torch.float32,
                       workspace=ws, config=cfg) for _ in range(3)]
    assert_close(outs[0], R.gemm_bias_act(a.cpu(), b.cpu(), bias.cpu(), "gelu_tanh", "nk", upcast=True),
                 dict(atol=2e-3, rtol=2e-3))
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    status_clean()


@pytest.mark.parametrize("parts", [2, 3])
def test_swapped_conv_split_is_reproducible(parts):
    """2 parts: own + other (staged); 3 parts: every part in part order."""
    g = gen(96)
    x = randn(g, 2, 14, 14, 256).cuda()
    w = randn(g, 3, 3, 256, 128, scale=(9 * 256) ** -0.5).cuda()
    cfg = N.tile_cfg(256, 4, 0, swap_ab=1, split_k=parts)
    ws = torch.zeros(fused.conv_workspace_bytes(2, 14, 14, 256, 128, 3, 3, 1, 1, 1, config=cfg), dtype=torch.uint8,
                     device="cuda")
    assert ws.numel() > 0
    outs = [fused.conv2d_nhwc(x, w, relu=True, stride=1, padding=1, workspace=ws, config=cfg, out_dtype=torch.float32)
            for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = R.conv2d_bias_relu(x.cpu(), w.cpu(), None, True, out_dtype=torch.float32, upcast=True)  # NHWC
    assert_close(outs[0], ref, dict(atol=2e-3, rtol=2e-3))
    status_clean()
