"""CUDA-graph capture of the fused operators: a captured call replayed on new inputs gives
the same bits as the eager call (the split-K counters reset themselves, tensor maps are
kernel parameters), a process whose very first library call is made under a global-mode
capture works, and the captured BERT forward equals the eager one."""
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from icpp_tuning_b200.end2end import HEAD_SIZE, FusedBert, make_weights, torch_native_bert
from icpp_tuning_b200.graphs import CapturedStep
from oracle.end2end_ref import bert_forward
from tests.gpu_util import gen, randn, status_clean

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _gemm_case(epilogue, M, N_, K, cfg, dt=torch.bfloat16, split=False):
    g = gen(70)
    b = randn(g, K, N_, dtype=dt, scale=K ** -0.5).cuda()
    bias = randn(g, N_, dtype=dt, scale=0.1).cuda()
    gamma, beta = randn(g, N_, dtype=dt, scale=0.1, shift=1.0).cuda(), randn(g, N_, dtype=dt, scale=0.1).cuda()
    ws = None
    if epilogue == "bias_layernorm":
        ws = torch.zeros(fused.ln_workspace_bytes(M, N_, cfg), dtype=torch.uint8, device="cuda")
    elif split:
        ws = torch.zeros(max(fused.workspace_bytes(M, N_, K, epilogue, cfg), 16), dtype=torch.uint8, device="cuda")
    ln = "layernorm" in epilogue

    def fn(a, res):
        return fused.gemm(a, b, epilogue=epilogue, bias=bias if epilogue != "none" else None,
                          gamma=gamma if ln else None, beta=beta if ln else None, workspace=ws,
                          residual=res if epilogue == "bias_residual_layernorm" else None, config=cfg)

    def inputs(seed):
        g2 = gen(seed)
        return [randn(g2, M, K, dtype=dt).cuda(), randn(g2, M, N_, dtype=dt).cuda()]

    return fn, inputs


def _conv_case(cfg, relu, add):
    n, h, w, c, f = 2, 14, 14, 64, 128
    g = gen(71)
    wt = randn(g, 3, 3, c, f, scale=(9 * c) ** -0.5).cuda()
    bn = tuple(t.cuda() for t in (randn(g, f), randn(g, f, scale=0.5), randn(g, f, scale=0.5),
                                  (torch.rand(f, generator=g) + 0.5).bfloat16()))

    def fn(x, res):
        return fused.conv2d_nhwc(x, wt, stride=1, padding=1, bn=bn, config=cfg, relu=relu,
                                 residual=res if add else None)

    def inputs(seed):
        g2 = gen(seed)
        return [randn(g2, n, h, w, c).cuda(), randn(g2, n, h, w, f).cuda()]

    return fn, inputs


CASES = {
    "gemm_split": lambda: _gemm_case("none", 1000, 768, 3072, N.tile_cfg(128, 6, 8), split=True),
    "gemm_pair_gelu": lambda: _gemm_case("bias_gelu_erf", 2048, 3072, 768, N.tile_cfg(256, 4, 8, block_m=256)),
    "gemm_bk128_relu": lambda: _gemm_case("bias_relu", 1536, 1024, 1024, N.tile_cfg(128, 3, 8, block_k=128)),
    "bias_layernorm": lambda: _gemm_case("bias_layernorm", 700, 1024, 512, N.tile_cfg(128, 6, 8)),
    # the one-kernel LayerNorm: a cooperative launch inside the captured graph
    "bias_layernorm_one_kernel": lambda: _gemm_case("bias_layernorm", 1500, 2048, 256,
                                                    N.tile_cfg(256, 3, 0, block_m=256, block_k=128,
                                                               ln_mode=N.LN_ONE_KERNEL)),
    "residual_layernorm": lambda: _gemm_case("bias_residual_layernorm", 384, 768, 768, N.tile_cfg(128, 6, 8),
                                             dt=torch.float16),
    "conv_bn_add_relu": lambda: _conv_case(N.tile_cfg(128, 6, 0), True, True),
    "conv_direct_bn": lambda: _conv_case(N.tile_cfg(256, 6, 0, swap_ab=2), False, False),
}


@pytest.mark.parametrize("case", list(CASES))
def test_captured_call_replays_bit_exact(case):
    fn, inputs = CASES[case]()
    step = CapturedStep(fn, inputs(1))
    launches = N.launch_count()
    for seed in (2, 3, 4):
        x = inputs(seed)
        got = step(*x).clone()
        want = fn(*x)
        torch.cuda.synchronize()
        assert torch.equal(got, want), case
    status_clean()
    # The eager calls above add launches on the host; the replays add none.
    before = N.launch_count()
    step.replay()
    torch.cuda.synchronize()
    assert N.launch_count() == before and before > launches


def test_first_library_call_under_global_capture():
    """A fresh process makes its first calls (device setup, kernel attributes, tensor-map
    encoder lookup) inside torch.cuda.graph's default global-mode capture."""
    script = textwrap.dedent("""
        import torch
        from icpp_tuning_b200 import _native as N, fused
        g = torch.Generator().manual_seed(5)
        a = torch.randn(512, 1024, generator=g).bfloat16().cuda()
        b = (torch.randn(1024, 1536, generator=g) * 0.03).bfloat16().cuda()
        bias = torch.randn(1536, generator=g).bfloat16().cuda()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            out = fused.gemm(a, b, epilogue="bias_gelu_tanh", bias=bias, config=N.tile_cfg(256, 4, 8, block_m=256))
        graph.replay()
        torch.cuda.synchronize()
        ref = fused.gemm(a, b, epilogue="bias_gelu_tanh", bias=bias, config=N.tile_cfg(256, 4, 8, block_m=256))
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert N.device_status(0)[0] == 0
        print("captured-first-call-ok")
    """)
    r = subprocess.run([sys.executable, "-c", script], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "captured-first-call-ok" in r.stdout, r.stdout + r.stderr


def test_captured_bert_forward_equals_eager():
    heads, layers, batch, seq = 12, 2, 2, 128
    w = make_weights(layers, heads * HEAD_SIZE, batch, seq)
    x = (torch.rand(batch, seq, heads * HEAD_SIZE, generator=gen(6)) * 0.8 - 0.4).half().cuda()
    with torch.no_grad():
        model = FusedBert(w, heads, batch * seq)
        step = CapturedStep(model, [x])
        got = step(x).clone()
        want = model(x)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_torch_native_arm_matches_reference_formulation():
    heads, layers, batch, seq = 8, 2, 2, 64
    w = make_weights(layers, heads * HEAD_SIZE, batch, seq)
    x = (torch.rand(batch, seq, heads * HEAD_SIZE, generator=gen(7)) * 0.8 - 0.4).half().cuda()
    with torch.no_grad():
        got = torch_native_bert(w, heads)(x)
        ref = bert_forward(w, x, heads, HEAD_SIZE)
    err = (got.float() - ref.float()).abs()
    assert err.mean() < 5e-3 and err.max() < 0.1, (err.mean().item(), err.max().item())
