"""gemm + bias + LayerNorm fused kernel against the oracle, through the C ABI."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from icpp_tuning_b200.gemm import gemm_bias_layernorm as gbln
from oracle import ref_ops as R
from tests.gpu_util import TOL_LN, assert_close, cuda, gen, randn, status_clean

pytestmark = pytest.mark.gpu


def _inputs(seed, M, Nn, K, dt=torch.bfloat16, layout="nk", shift=0.0):
    g = gen(seed)
    x = randn(g, M, K, dtype=dt)
    w = randn(g, *((Nn, K) if layout == "nk" else (K, Nn)), dtype=dt, scale=K ** -0.5)
    bias = randn(g, Nn, dtype=dt, scale=0.02, shift=shift)
    gamma = randn(g, Nn, dtype=dt, scale=0.02, shift=1.0)
    beta = randn(g, Nn, dtype=dt, scale=0.02)
    return x, w, bias, gamma, beta


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("odt", [torch.bfloat16, torch.float16])
def test_ln_ragged(bn, odt):
    M, Nn, K = 300, 1000, 192  # N not a multiple of BN, M not of 128
    dt = odt
    x, w, bias, gamma, beta = _inputs(10, M, Nn, K, dt)
    cfg = N.tile_cfg(bn, {256: 4, 128: 6, 64: 8}[bn], 0)
    # zero counters, arbitrary statistics: every call writes each statistic before reading it
    ws = torch.full((fused.ln_workspace_bytes(M, Nn, cfg),), 0x7F, dtype=torch.uint8, device="cuda")
    hdr = _header_bytes(M)
    ws[:hdr] = 0
    for _ in range(3):
        out = fused.gemm(*cuda(x, w), b_layout="nk", epilogue="bias_layernorm", bias=bias.cuda(),
                         gamma=gamma.cuda(), beta=beta.cuda(), workspace=ws, out_dtype=odt, config=cfg)
        assert_close(out, R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=odt), TOL_LN)
    assert int(ws[:hdr].count_nonzero()) == 0  # the counters are left zeroed
    status_clean()


def _header_bytes(M):
    """Bytes of arrival counters at the head of the LayerNorm workspace."""
    return (((M + 31) // 32) * 8 + 255) // 256 * 256


def _ln_call(x, w, bias, gamma, beta, cfg, ws=None, odt=torch.bfloat16):
    M, Nn = x.shape[0], w.shape[0]
    if ws is None:
        ws = torch.zeros(fused.ln_workspace_bytes(M, Nn, cfg), dtype=torch.uint8, device="cuda")
    out = fused.gemm(*cuda(x, w), b_layout="nk", epilogue="bias_layernorm", bias=bias.cuda(), gamma=gamma.cuda(),
                     beta=beta.cuda(), workspace=ws, out_dtype=odt, config=cfg)
    return out, ws


@pytest.mark.parametrize("bm,bn,bk,st,gm", [(128, 128, 64, 6, 0), (128, 256, 64, 4, 0), (128, 256, 64, 4, 8),
                                           (256, 256, 128, 3, 0), (256, 256, 128, 3, 8), (256, 128, 128, 4, 16)])
def test_ln_one_kernel(bm, bn, bk, st, gm):
    """ln_mode 2 (each epilogue warp normalises its own stored slice once its rows'
    statistics are all published) against the oracle and against the two-kernel path,
    on single CTAs and CTA pairs, row-major and grouped rasters (the grouped ones defer
    a slice by more than one unit), ragged M and N; the counters are left zeroed and a
    repeated call gives the same bits."""
    M, Nn, K = 1500, 3000, 320
    x, w, bias, gamma, beta = _inputs(14, M, Nn, K)
    one = N.tile_cfg(bn, st, gm, block_m=bm, block_k=bk, ln_mode=N.LN_ONE_KERNEL)
    two = N.tile_cfg(bn, st, gm, block_m=bm, block_k=bk, ln_mode=N.LN_TWO_KERNELS)
    n0 = N.launch_count()
    out1, ws = _ln_call(x, w, bias, gamma, beta, one)
    assert N.launch_count() - n0 == 1  # one kernel, no row pass
    ref = R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=torch.bfloat16)
    assert_close(out1, ref, TOL_LN)
    assert int(ws[:_header_bytes(M)].count_nonzero()) == 0
    again, _ = _ln_call(x, w, bias, gamma, beta, one, ws=ws)
    assert torch.equal(again, out1)
    out2, _ = _ln_call(x, w, bias, gamma, beta, two)
    # same statistics and centring: the two paths differ by at most one output rounding
    assert_close(out1, out2, dict(atol=1e-2, rtol=1e-2))
    status_clean()


def test_ln_one_kernel_rejections():
    x, w, bias, gamma, beta = _inputs(15, 256, 512, 64)
    with pytest.raises(N.FoError, match="block_n >= 128"):
        _ln_call(x, w, bias, gamma, beta, N.tile_cfg(64, 8, 0, ln_mode=N.LN_ONE_KERNEL))
    # automatic mode takes the two-kernel path for block_n 64
    out, _ = _ln_call(x, w, bias, gamma, beta, N.tile_cfg(64, 8, 0))
    assert_close(out, R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=torch.bfloat16), TOL_LN)


@pytest.mark.parametrize("bm,bn,bk,st", [(128, 128, 64, 6), (128, 256, 64, 4), (256, 256, 128, 3), (256, 128, 128, 4)])
def test_ln_held(bm, bn, bk, st):
    """ln_mode 3 (each epilogue warp keeps its slice in the TMEM accumulator until its
    rows' statistics are merged, then normalises and stores it once) against the oracle
    and the stored-slice one-kernel path, single CTAs and CTA pairs, ragged M and N; the
    counters are left zeroed and a repeated call gives the same bits."""
    M, Nn, K = 1500, 3000, 320
    x, w, bias, gamma, beta = _inputs(16, M, Nn, K)
    held = N.tile_cfg(bn, st, 0, block_m=bm, block_k=bk, ln_mode=N.LN_HELD)
    n0 = N.launch_count()
    out, ws = _ln_call(x, w, bias, gamma, beta, held)
    assert N.launch_count() - n0 == 1
    ref = R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=torch.bfloat16)
    assert_close(out, ref, TOL_LN)
    assert int(ws[:_header_bytes(M)].count_nonzero()) == 0
    again, _ = _ln_call(x, w, bias, gamma, beta, held, ws=ws)
    assert torch.equal(again, out)
    one, _ = _ln_call(x, w, bias, gamma, beta, N.tile_cfg(bn, st, 0, block_m=bm, block_k=bk, ln_mode=N.LN_ONE_KERNEL))
    # the stored path rounds the centred slice to 16 bits once more: two output roundings apart
    assert_close(out, one, TOL_LN)
    status_clean()


def test_ln_held_fp16_ragged_rows():
    """Held slices with fp16 output and M not a multiple of 32: the last row group's
    partial warps still release their accumulators and the counters end at zero."""
    M, Nn, K = 1000, 1536, 256
    x, w, bias, gamma, beta = _inputs(19, M, Nn, K, dt=torch.float16)
    cfg = N.tile_cfg(256, 3, 0, block_m=256, block_k=128, ln_mode=N.LN_HELD)
    out, ws = _ln_call(x, w, bias, gamma, beta, cfg, odt=torch.float16)
    ref = R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=torch.float16)
    assert_close(out, ref, TOL_LN)
    assert int(ws[:_header_bytes(M)].count_nonzero()) == 0
    status_clean()


def test_ln_auto_takes_held_slices():
    """Automatic mode holds the slices in TMEM for a problem of at most 4 waves with
    K >= 2048 and >= 4M outputs: same bits as ln_mode 3, one launch, oracle on sampled rows."""
    M, Nn, K = 4096, 1024, 2048
    x, w, bias, gamma, beta = _inputs(18, M, Nn, K)
    auto = N.tile_cfg(256, 3, 0, block_m=256, block_k=128)
    n0 = N.launch_count()
    out, _ = _ln_call(x, w, bias, gamma, beta, auto)
    assert N.launch_count() - n0 == 1
    held, _ = _ln_call(x, w, bias, gamma, beta, N.tile_cfg(256, 3, 0, block_m=256, block_k=128, ln_mode=N.LN_HELD))
    assert torch.equal(out, held)
    rows = torch.arange(0, M, 61)
    ref = R.gemm_bias_layernorm(x[rows], w, bias, gamma, beta, b_layout="nk", out_dtype=torch.bfloat16)
    assert_close(out[rows.cuda()], ref, TOL_LN)
    status_clean()


def test_ln_held_rejections():
    """Held slices need block_n >= 128 and a raster whose row blocks span fewer units than
    a wave (group_m 8 here spreads a row block over 8 x 23 units)."""
    x, w, bias, gamma, beta = _inputs(17, 1500, 3000, 64)
    with pytest.raises(N.FoError, match="held slices"):
        _ln_call(x, w, bias, gamma, beta, N.tile_cfg(64, 8, 0, ln_mode=N.LN_HELD))
    with pytest.raises(N.FoError, match="held slices"):
        _ln_call(x, w, bias, gamma, beta, N.tile_cfg(128, 6, 8, ln_mode=N.LN_HELD))


@pytest.mark.parametrize("M,Nn,bn", [(2000, 1000, 64), (1100, 2304, 256), (3000, 4096, 128), (100, 5000, 256),
                                     (1500, 6144, 128), (1, 768, 64)])
def test_ln_row_pass_variants(M, Nn, bn):
    """Each row-pass kernel: block per row (M <= 1024), warp per row (larger M), and the
    batched pass for N > 4096; ragged N against the slab / chunk widths."""
    K = 128
    x, w, bias, gamma, beta = _inputs(13, M, Nn, K)
    cfg = N.tile_cfg(bn, {256: 4, 128: 6, 64: 8}[bn], 0)
    ws = torch.zeros(fused.ln_workspace_bytes(M, Nn, cfg), dtype=torch.uint8, device="cuda")
    out = fused.gemm(*cuda(x, w), b_layout="nk", epilogue="bias_layernorm", bias=bias.cuda(), gamma=gamma.cuda(),
                     beta=beta.cuda(), workspace=ws, out_dtype=torch.bfloat16, config=cfg)
    rows = torch.arange(0, M, max(1, M // 64))
    ref = R.gemm_bias_layernorm(x[rows], w, bias, gamma, beta, b_layout="nk", out_dtype=torch.bfloat16)
    assert_close(out[rows.cuda()], ref, TOL_LN)
    status_clean()


def test_ln_large_mean_offset():
    """Rows whose mean is far from zero: the centred (Chan) statistics stay accurate
    where E[x^2] - E[x]^2 (the reference LN kernel, gemm_bias_layernorm.py:143) loses bits."""
    M, Nn, K = 256, 2048, 256
    x, w, bias, gamma, beta = _inputs(11, M, Nn, K, shift=30.0)
    k = gbln.build_fused_kernel(M, Nn, K, out_dtype=torch.bfloat16, b_layout="nk")
    out = k(*cuda(x, w, bias, gamma, beta))
    ref = R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=torch.float32, upcast=True)
    assert_close(out, ref, TOL_LN)


def test_reference_api_shape_and_assert():
    with pytest.raises(AssertionError):
        gbln.build_fused_kernel(128, 1000, 64, block_N_ln=128)
    M, Nn, K = 64, 256, 128
    g = gen(12)
    A, B = randn(g, M, K, dtype=torch.float16), randn(g, K, Nn, dtype=torch.float16, scale=K ** -0.5)
    bias, gamma, beta = (randn(g, Nn, dtype=torch.float16, scale=0.02),
                         randn(g, Nn, dtype=torch.float16, scale=0.02, shift=1.0),
                         randn(g, Nn, dtype=torch.float16, scale=0.02))
    k = gbln.build_fused_kernel(M, Nn, K)  # reference defaults: fp16 out, B [K, N]
    out = k(*cuda(A, B, bias, gamma, beta))
    assert out.dtype == torch.float16
    assert_close(out, R.gemm_bias_layernorm(A, B, bias, gamma, beta), TOL_LN)


def test_config4_ln_full():
    """Config 4: M=16384, K=4096, N=4096 bf16, X ~ N(0,1), W ~ N(0,1)/sqrt(K), seed 3."""
    M, Nn, K = 16384, 4096, 4096
    x, w, bias, gamma, beta = _inputs(3, M, Nn, K)
    k = gbln.build_fused_kernel(M, Nn, K, out_dtype=torch.bfloat16, b_layout="nk")
    n0 = N.launch_count()
    out = k(*cuda(x, w, bias, gamma, beta))
    assert N.launch_count() - n0 == 1  # the tuned config runs the one-kernel LayerNorm
    # every row (the CPU oracle takes ~2 s)
    ref = R.gemm_bias_layernorm(x, w, bias, gamma, beta, b_layout="nk", out_dtype=torch.bfloat16)
    assert_close(out, ref, TOL_LN)
    # every row normalised: mean ~ beta-mean, unit variance before the affine transform
    y = (out.float() - beta.cuda().float()) / gamma.cuda().float()
    assert y.mean(dim=1).abs().max() < 0.05 and (y.var(dim=1, unbiased=False) - 1).abs().max() < 0.05
    status_clean()
