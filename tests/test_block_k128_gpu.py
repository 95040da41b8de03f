"""block_k = 128: two 64-wide K slices per pipeline stage (one barrier wait and one commit
per 8 MMAs).  Odd k-block counts leave the last stage half full."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from oracle import ref_ops as R
from tests.gpu_util import TOL, assert_close, cuda, gen, randn, status_clean

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", [dict(block_n=256, stages=2), dict(block_n=128, stages=3), dict(block_n=64, stages=4),
                                 dict(block_n=256, stages=3, block_m=256), dict(block_n=128, stages=3, block_m=256)],
                         ids=str)
@pytest.mark.parametrize("M,Nn,K", [(300, 520, 520), (1000, 1304, 200), (128, 256, 64), (256, 512, 1088)], ids=str)
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_gemm_block_k128(cfg, M, Nn, K, layout):
    g = gen(80)
    a = randn(g, M, K, scale=K ** -0.25)
    b = randn(g, *((K, Nn) if layout == "kn" else (Nn, K)), scale=K ** -0.25)
    # whole tiles in both (a split would sum its parts in a different order)
    tile = N.tile_cfg(group_m=8, block_k=128, split_k=1, **cfg)
    out = fused.gemm(*cuda(a, b), b_layout=layout, out_dtype=torch.float32, config=tile)
    ref_cfg = N.tile_cfg(cfg["block_n"], 4 if cfg["block_n"] == 256 else 6, 8, split_k=1)
    same = fused.gemm(*cuda(a, b), b_layout=layout, out_dtype=torch.float32, config=ref_cfg)
    assert torch.equal(out, same)  # same K order per output element as block_k 64
    assert_close(out, R.gemm(a, b, layout, upcast=True), dict(atol=1e-4, rtol=1e-4))
    status_clean()


@pytest.mark.parametrize("block_m", [128, 256])
def test_split_tail_block_k128(block_m):
    g = gen(81)
    M, Nn, K = 2304, 2304, 2240  # 35 k-blocks: odd parts
    a, b = randn(g, M, K, scale=K ** -0.25), randn(g, Nn, K, scale=K ** -0.25)
    tile = N.tile_cfg(256, 3 if block_m == 256 else 2, 8, block_m=block_m, block_k=128, split_k=3)
    ws = torch.zeros(fused.workspace_bytes(M, Nn, K, "none", tile), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        out = fused.gemm(*cuda(a, b), b_layout="nk", out_dtype=torch.float32, workspace=ws, config=tile)
        assert_close(out, R.gemm(a, b, "nk", upcast=True), dict(atol=1e-4, rtol=1e-4))
    status_clean()


def test_conv_rejects_block_k128():
    """The conv kernels stage one 64-wide K slice; block_k 128 is a GEMM-family option."""
    x = torch.zeros(2, 8, 8, 64, dtype=torch.bfloat16, device="cuda")
    wt = torch.zeros(3, 3, 64, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(N.FoError, match="block_k must be 64"):
        fused.conv2d_nhwc(x, wt, config=N.tile_cfg(128, 3, 0, block_k=128))
