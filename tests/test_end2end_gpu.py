"""The BERT forward of the reference's evaluation/end2end.py with the fused operators,
against the reference's PyTorch formulation (oracle/end2end_ref.py), and the residual
LayerNorm epilogue against its PyTorch definition."""
import pytest
import torch
import torch.nn.functional as F

from icpp_tuning_b200 import fused
from icpp_tuning_b200.end2end import HEAD_SIZE, FusedBert, make_weights
from oracle.end2end_ref import bert_forward
from tests.gpu_util import gen, randn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,dt", [(300, 768, 768, torch.float16), (257, 1024, 4096, torch.bfloat16),
                                      (128, 4096, 512, torch.float16), (3000, 2304, 256, torch.float16),
                                      (1500, 4096, 128, torch.bfloat16), (2049, 512, 192, torch.float16)])
def test_residual_layernorm_epilogue(M, N, K, dt):
    g = gen(40)
    a, b = randn(g, M, K, dtype=dt, scale=0.5), randn(g, K, N, dtype=dt, scale=K ** -0.5)
    bias, res = randn(g, N, dtype=dt, scale=0.1), randn(g, M, N, dtype=dt)
    gamma, beta = randn(g, N, dtype=dt, scale=0.1, shift=1.0), randn(g, N, dtype=dt, scale=0.1)
    a, b, bias, res, gamma, beta = (t.cuda() for t in (a, b, bias, res, gamma, beta))
    out = fused.gemm(a, b, epilogue="bias_residual_layernorm", bias=bias, gamma=gamma, beta=beta, residual=res)
    y = (a.float() @ b.float() + bias.float()).to(dt)  # the GEMM result rounded first
    ref = F.layer_norm((y + res).float(), (N,), gamma.float(), beta.float(), 1e-5)  # 16-bit add, end2end.py:78
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("model,layers,heads,batch,seq", [("bert_small", 2, 8, 2, 128), ("bert_base", 1, 12, 4, 96)])
def test_bert_forward_matches_reference(model, layers, heads, batch, seq):
    hidden = heads * HEAD_SIZE
    w = make_weights(layers, hidden, batch, seq)
    x = (torch.rand(batch, seq, hidden, generator=torch.Generator().manual_seed(1)) * 0.8 - 0.4).half().cuda()
    with torch.no_grad():
        ours = FusedBert(w, heads, batch * seq)(x)
        ref = bert_forward(w, x, heads, HEAD_SIZE)
    # the LayerNorm tolerance of the other parity tests
    torch.testing.assert_close(ours.float(), ref.float(), atol=2e-2, rtol=2e-2)
