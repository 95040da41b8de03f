"""fo_gemm_bias_layernorm_noalloc: the fused GEMM + bias + LayerNorm for callers that
cannot allocate device memory (for example a serving process that fixes its memory
budget at start-up, or a plugin interface that hands over inputs and outputs but no
allocator).  It takes its LayerNorm scratch from a static per-GPU array instead of a
caller workspace.  Here it is called through the C ABI twice in a row and compared with
fo_gemm on a caller-allocated workspace; the second call checks that state the first
call left in the shared array does not leak into the result.  This file is collected
last so that a run stopping at the first failure has already run every other test."""
import ctypes

import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused

pytestmark = pytest.mark.gpu

TOL_LN = dict(atol=2e-2, rtol=2e-2)  # the LayerNorm tolerance of the other tests


def _desc(x, w, bias, gamma, beta, out, M, Nn, K, layout):
    d = N.FoGemmDesc()
    d.M, d.N, d.K = M, Nn, K
    d.a, d.b, d.out = x.data_ptr(), w.data_ptr(), out.data_ptr()
    d.lda, d.ldb, d.ldo = x.stride(0), w.stride(0), out.stride(0)
    d.bias, d.gamma, d.beta = bias.data_ptr(), gamma.data_ptr(), beta.data_ptr()
    d.in_dtype = d.vec_dtype = d.out_dtype = N.FO_DT_BF16
    d.b_layout = N.FO_B_NK if layout == "nk" else N.FO_B_KN
    d.epilogue = N.FO_EPI_BIAS_LN
    d.eps = 1e-5
    return d


@pytest.mark.parametrize("M,Nn,K,layout,bn", [(300, 1000, 192, "nk", 128), (1024, 2048, 512, "kn", 256)])
def test_noalloc_matches_fo_gemm_twice(M, Nn, K, layout, bn):
    g = torch.Generator().manual_seed(77)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (torch.randn(*((Nn, K) if layout == "nk" else (K, Nn)), generator=g) * K ** -0.5).bfloat16().cuda()
    bias = (torch.randn(Nn, generator=g) * 0.02).bfloat16().cuda()
    gamma = (1 + torch.randn(Nn, generator=g) * 0.02).bfloat16().cuda()
    beta = (torch.randn(Nn, generator=g) * 0.02).bfloat16().cuda()
    cfg = N.tile_cfg(bn, {256: 4, 128: 6}[bn], 0)

    ws = torch.zeros(fused.ln_workspace_bytes(M, Nn, cfg), dtype=torch.uint8, device="cuda")
    expect = fused.gemm(x, w, b_layout=layout, epilogue="bias_layernorm", bias=bias, gamma=gamma, beta=beta,
                        workspace=ws, config=cfg)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((M, Nn), float("nan"), dtype=torch.bfloat16, device="cuda")
        d = _desc(x, w, bias, gamma, beta, out, M, Nn, K, layout)
        rc = N.lib().fo_gemm_bias_layernorm_noalloc(ctypes.byref(d), ctypes.byref(cfg), stream)
        assert rc == N.FO_OK, N.last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), expect.float(), **TOL_LN, msg=f"call {call}")


def test_noalloc_rejects_oversized_problems():
    cfg = N.tile_cfg(64, 8, 0)
    d = N.FoGemmDesc()
    d.M, d.N, d.K = 1 << 20, 4096, 64  # 64 N-tiles x 1M rows of statistics >> 8 MiB
    d.a = d.b = d.out = d.bias = d.gamma = d.beta = 1 << 20
    d.lda, d.ldb, d.ldo = 64, 64, 4096
    d.in_dtype = d.vec_dtype = d.out_dtype = N.FO_DT_BF16
    d.b_layout, d.epilogue, d.eps = N.FO_B_NK, N.FO_EPI_BIAS_LN, 1e-5
    rc = N.lib().fo_gemm_bias_layernorm_noalloc(ctypes.byref(d), ctypes.byref(cfg), None)
    assert rc == N.FO_EINVAL
    assert "static scratch holds" in N.last_error()
