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
from oracle import ref_ops as R

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
    # the reference's own program on sampled rows (the oracle of the other LayerNorm tests)
    rows = torch.arange(0, M, 37)
    ref = R.gemm_bias_layernorm(x.cpu()[rows], w.cpu(), bias.cpu(), gamma.cpu(), beta.cpu(), b_layout=layout,
                                out_dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((M, Nn), float("nan"), dtype=torch.bfloat16, device="cuda")
        d = _desc(x, w, bias, gamma, beta, out, M, Nn, K, layout)
        n0 = N.launch_count()
        rc = N.lib().fo_gemm_bias_layernorm_noalloc(ctypes.byref(d), ctypes.byref(cfg), stream)
        assert rc == N.FO_OK, N.last_error()
        assert N.launch_count() > n0  # counted like fo_gemm
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), expect.float(), **TOL_LN, msg=f"call {call}")
        torch.testing.assert_close(out[rows.cuda()].float().cpu(), ref.float(), **TOL_LN, msg=f"call {call}")
    # a bounded wait that ran out would show here, in fo_device_status's word
    rc, where = N.device_status(torch.cuda.current_device())
    assert rc == 0, f"device status {rc} at {where:#x}"


def test_noalloc_rejects_oversized_problems():
    """The size rule rejects the call before anything is enqueued.  The call is made
    while a side stream is being captured and the capture is discarded unlaunched, so
    even if the check regressed nothing would run on the (tiny, real) buffers."""
    cfg = N.tile_cfg(64, 8, 0)
    t = torch.zeros(4096, dtype=torch.bfloat16, device="cuda")
    d = N.FoGemmDesc()
    d.M, d.N, d.K = 1 << 20, 4096, 64  # 64 N-tiles x 1M rows of statistics >> 8 MiB
    d.a = d.b = d.out = d.bias = d.gamma = d.beta = t.data_ptr()
    d.lda, d.ldb, d.ldo = 64, 64, 4096
    d.in_dtype = d.vec_dtype = d.out_dtype = N.FO_DT_BF16
    d.b_layout, d.epilogue, d.eps = N.FO_B_NK, N.FO_EPI_BIAS_LN, 1e-5
    side = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        g.capture_begin()
        rc = N.lib().fo_gemm_bias_layernorm_noalloc(ctypes.byref(d), ctypes.byref(cfg), side.cuda_stream)
        msg = N.last_error()
        g.capture_end()
    del g  # never replayed
    assert rc == N.FO_EINVAL
    assert "static scratch holds" in msg
