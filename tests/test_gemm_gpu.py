"""GEMM-family kernels (gemm, gemm + bias + act) against the oracle, through the C ABI."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from oracle import ref_ops as R
from tests.gpu_util import TOL, assert_close, cuda, gen, randn, status_clean, uniform

pytestmark = pytest.mark.gpu

CFGS = {bn: N.tile_cfg(block_n=bn, stages={256: 4, 128: 6, 64: 8}[bn], group_m=8) for bn in (64, 128, 256)}


def _inputs(seed, M, Nn, K, dt, layout, bias=True):
    g = gen(seed)
    a = randn(g, M, K, dtype=dt, scale=K ** -0.25)
    b = randn(g, *((K, Nn) if layout == "kn" else (Nn, K)), dtype=dt, scale=K ** -0.25)
    bv = randn(g, Nn, dtype=dt, scale=0.1) if bias else None
    return a, b, bv


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_plain_ragged(bn, layout, dt):
    M, Nn, K = 333, 264, 200  # none a multiple of the tile
    a, b, _ = _inputs(1, M, Nn, K, dt, layout, bias=False)
    out = fused.gemm(*cuda(a, b), b_layout=layout, out_dtype=torch.float32, config=CFGS[bn])
    assert_close(out, R.gemm(a, b, layout, upcast=True), dict(atol=1e-4, rtol=1e-4))
    assert_close(out, R.gemm(a, b, layout), TOL)
    status_clean()


@pytest.mark.parametrize("act", ["relu", "gelu_tanh", "gelu_erf", "none"])
@pytest.mark.parametrize("odt", [torch.float16, torch.bfloat16, torch.float32])
def test_gemm_bias_act(act, odt):
    M, Nn, K = 517, 776, 320
    dt = torch.float16 if odt == torch.float16 else torch.bfloat16
    a, b, bias = _inputs(2, M, Nn, K, dt, "kn")
    epi = "bias" if act == "none" else f"bias_{act}"
    out = fused.gemm(*cuda(a, b), b_layout="kn", epilogue=epi, bias=bias.cuda(), out_dtype=odt, config=CFGS[128])
    ref = R.gemm_bias_act(a, b, bias, act)
    assert out.dtype == odt
    assert_close(out, ref, TOL)
    status_clean()


@pytest.mark.parametrize("act", ["gelu_erf", "gelu_tanh"])
def test_gelu_fp32_accuracy(act):
    """GELU epilogues into fp32 against the fp32-upcast oracle over pre-activations of
    about +-10 (the erf is Abramowitz & Stegun 7.1.28, |error| ~3e-6 in fp32, GELU within
    ~1e-6; tanh uses tanh.approx)."""
    g = gen(60)
    M, Nn, K = 300, 520, 256
    a, b = randn(g, M, K, scale=0.6), randn(g, K, Nn, scale=K ** -0.5 * 5)
    bias = randn(g, Nn, scale=1.0)
    out = fused.gemm(*cuda(a, b), epilogue=f"bias_{act}", bias=bias.cuda(), out_dtype=torch.float32,
                     config=N.tile_cfg(256, 4, 0))
    ref = R.gemm_bias_act(a, b, bias, act, upcast=True)
    assert ref.abs().max() > 5
    tol = dict(atol=2e-5, rtol=2e-5) if act == "gelu_erf" else dict(atol=2e-3, rtol=2e-3)
    assert_close(out, ref, tol)


def test_misaligned_bias_vector():
    """A bias view that is not 16-byte aligned takes the per-lane load path."""
    g = gen(61)
    M, Nn, K = 200, 512, 128
    a, b = randn(g, M, K), randn(g, K, Nn, scale=K ** -0.5)
    store = randn(g, Nn + 1, scale=0.5).cuda()
    bias = store[1:]  # 2-byte offset
    out = fused.gemm(*cuda(a, b), epilogue="bias_relu", bias=bias, out_dtype=torch.float32, config=N.tile_cfg(128, 6, 0))
    assert_close(out, R.gemm_bias_act(a, b, bias.cpu(), "relu"), TOL)


@pytest.mark.parametrize("M", [1, 2, 127, 128, 129])
def test_small_m(M):
    a, b, bias = _inputs(3, M, 2304, 768, torch.float16, "kn")
    out = fused.gemm(*cuda(a, b), epilogue="bias_relu", bias=bias.cuda(), out_dtype=torch.float32, config=CFGS[64])
    assert_close(out, R.gemm_bias_act(a, b, bias, "relu"), TOL)


def test_k_zero_gives_bias():
    g = gen(4)
    a = torch.empty(130, 0, dtype=torch.bfloat16)
    b = torch.empty(0, 72, dtype=torch.bfloat16)
    bias = randn(g, 72)
    out = fused.gemm(*cuda(a, b), epilogue="bias_relu", bias=bias.cuda(), out_dtype=torch.float32)
    assert_close(out, torch.relu(bias.float()).expand(130, 72), dict(atol=0, rtol=0))


def test_empty_m():
    a, b, _ = _inputs(5, 0, 64, 64, torch.bfloat16, "nk", bias=False)
    out = fused.gemm(*cuda(a, b), b_layout="nk")
    assert out.shape == (0, 64)


def test_strided_rows():
    # row strides larger than the logical width (views into wider buffers)
    g = gen(6)
    A = randn(g, 200, 256)
    B = randn(g, 160, 256)
    a, b = A[:, :192], B[:, :192]
    out_buf = torch.zeros(200, 256, dtype=torch.bfloat16, device="cuda")
    out = fused.gemm(a.cuda(), b.cuda(), b_layout="nk", out=out_buf[:, :160], config=CFGS[128])
    assert_close(out, R.gemm(a, b, "nk"), TOL)
    assert (out_buf[:, 160:] == 0).all()


@pytest.mark.parametrize("group_m", [0, 1, 3, 8, 64])
def test_raster_orders_bitwise_identical(group_m):
    a, b, _ = _inputs(7, 1100, 1304, 256, torch.bfloat16, "nk", bias=False)
    a, b = cuda(a, b)
    base = fused.gemm(a, b, b_layout="nk", config=N.tile_cfg(256, 4, 0))
    out = fused.gemm(a, b, b_layout="nk", config=N.tile_cfg(256, 4, group_m, max_ctas=37))
    assert torch.equal(base, out)


def test_row_shards_bitwise_identical():
    """Each output element's K loop is independent of the tile schedule, so a row shard
    computed alone equals the same rows of the full product (the multi-GPU property)."""
    a, b, bias = _inputs(8, 1000, 512, 384, torch.bfloat16, "kn")
    a, b, bias = cuda(a, b, bias)
    full = fused.gemm(a, b, epilogue="bias_gelu_tanh", bias=bias)
    for lo, hi in [(0, 384), (384, 1000), (512, 640)]:
        part = fused.gemm(a[lo:hi], b, epilogue="bias_gelu_tanh", bias=bias)
        assert torch.equal(part, full[lo:hi])


def test_bad_shapes_raise():
    a = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        fused.gemm(a, torch.zeros(32, 64, dtype=torch.bfloat16, device="cuda"), b_layout="kn")
    with pytest.raises(N.FoError, match="lda"):
        fused.gemm(torch.zeros(64, 12, dtype=torch.bfloat16, device="cuda"),
                   torch.zeros(12, 64, dtype=torch.bfloat16, device="cuda"))


# ---- BASELINE workloads at full size ---------------------------------------------

def test_config1_gemm_bias_relu_1024():
    """Config 1: fp16, M=N=K=1024, A,B ~ U(-1,1), bias ~ N(0,0.1), fp16 out, seed 0."""
    g = gen(0)
    a, b = uniform(g, 1024, 1024), uniform(g, 1024, 1024)
    bias = randn(g, 1024, dtype=torch.float16, scale=0.1)
    from icpp_tuning_b200.gemm import gemm_bias_act
    k = gemm_bias_act.build_kernel(1024, 1024, 1024, act="relu", out_dtype=torch.float16)
    out = k(*cuda(a, b, bias))
    assert_close(out, R.gemm_bias_act(a, b, bias, "relu"), TOL)
    status_clean()


def test_config2_gemm_4096():
    """Config 2: bf16 4096^3, A, B ~ N(0,1)/sqrt(K), A row-major, B column-major, seed 1."""
    g = gen(1)
    a = randn(g, 4096, 4096, scale=4096 ** -0.5)
    bt = randn(g, 4096, 4096, scale=4096 ** -0.5)  # B[K,N] column-major == B^T [N,K] row-major
    from icpp_tuning_b200.gemm import gemm
    k = gemm.build_kernel(4096, 4096, 4096, out_dtype=torch.bfloat16, b_layout="nk")
    out = k(*cuda(a, bt))
    assert_close(out, R.gemm(a, bt, "nk"), TOL)
    status_clean()


def test_config3_gemm_bias_gelu_mlp():
    """Config 3: bf16, M=8192, K=4096, N=16384, X ~ N(0,1), W ~ N(0,0.02), bias ~ N(0,0.02), GELU-tanh."""
    g = gen(2)
    x = randn(g, 8192, 4096)
    w = randn(g, 16384, 4096, scale=0.02)  # nn.Linear layout [N, K]
    bias = randn(g, 16384, scale=0.02)
    from icpp_tuning_b200.gemm import gemm_bias_act
    k = gemm_bias_act.build_kernel(8192, 16384, 4096, act="gelu_tanh", out_dtype=torch.bfloat16, b_layout="nk")
    out = k(*cuda(x, w, bias))
    # every row (the CPU oracle takes ~10 s on a 16-core host)
    assert_close(out, R.gemm_bias_act(x, w, bias, "gelu_tanh", "nk"), TOL)
    status_clean()


@pytest.mark.parametrize("M,Nn,K,bn,layout", [
    (126, 2304, 2048, 64, "kn"),      # 36 tiles on 148 SMs: split 4 ways along K
    (4096, 4096, 4096, 256, "nk"),    # 512 tiles: the 68-tile last wave split 2 ways
    (300, 520, 2056, 128, "kn"),      # K of 33 k-blocks: uneven parts (17 + 16)
])
def test_split_k_tail(M, Nn, K, bn, layout):
    a, b, bias = _inputs(9, M, Nn, K, torch.bfloat16, layout)
    cfg = N.tile_cfg(bn, {256: 4, 128: 6, 64: 8}[bn], 8)
    nbytes = fused.workspace_bytes(M, Nn, K, "bias_gelu_tanh", cfg)
    assert nbytes > 0
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    a_d, b_d, bias_d = cuda(a, b, bias)
    whole = fused.gemm(a_d, b_d, b_layout=layout, epilogue="bias_gelu_tanh", bias=bias_d, config=cfg)
    for _ in range(2):
        split = fused.gemm(a_d, b_d, b_layout=layout, epilogue="bias_gelu_tanh", bias=bias_d, workspace=ws,
                           config=cfg)
        torch.testing.assert_close(split.float(), whole.float(), atol=1e-2, rtol=1e-2)
    rows = slice(0, M, max(1, M // 64))
    assert_close(split[rows], R.gemm_bias_act(a[rows], b, bias, "gelu_tanh", layout), TOL)
    # the arrival counters at the start of the workspace come back zeroed
    assert int(ws[:256].view(torch.int32).abs().sum()) == 0
    status_clean()


def test_built_kernel_workspace_per_stream():
    """A built operator gives each CUDA stream its own zero-filled split-K workspace, so
    calls overlapping on two streams do not share counters or partials."""
    from icpp_tuning_b200.gemm import gemm as gm

    M, Nn, K = 512, 768, 4096  # 24 tiles: a split-K tail on idle SMs
    g = gen(77)
    a, b = randn(g, M, K), randn(g, K, Nn, scale=K ** -0.5)
    k = gm.build_kernel(M, Nn, K, out_dtype=torch.float32)
    ref = R.gemm(a, b)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    ad, bd = cuda(a, b)
    outs = []
    torch.cuda.synchronize()
    for s in (s1, s2, s1, s2):
        with torch.cuda.stream(s):
            outs.append(k(ad, bd))
    torch.cuda.synchronize()
    for o in outs:
        assert_close(o, ref)
    status_clean()
