"""The C ABI without a GPU: the library loads, exports every symbol include/b200fo.h
declares, and rejects bad arguments before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

from icpp_tuning_b200 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200fo.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_0-9]+\s*\*?\s*(fo_[a-z0-9_]+)\(", text, re.M)))


def test_header_declarations_match_binding_list():
    assert declared_functions() == sorted(N.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version():
    assert N.version().startswith("b200fo ") and "sm_100a" in N.version()


def _desc(**kw):
    d = N.FoGemmDesc()
    d.M, d.N, d.K = 256, 256, 64
    d.a = d.b = d.out = 1 << 20  # aligned fake addresses: validation never dereferences
    d.lda, d.ldb, d.ldo = 64, 64, 256
    d.in_dtype, d.out_dtype, d.vec_dtype = N.FO_DT_BF16, N.FO_DT_BF16, N.FO_DT_BF16
    d.b_layout, d.epilogue = N.FO_B_NK, N.FO_EPI_NONE
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def _call(d, cfg=None):
    cfg = cfg or N.tile_cfg(256, 4, 8)
    return N.lib().fo_gemm(ctypes.byref(d), ctypes.byref(cfg), None)


@pytest.mark.parametrize("kw,msg", [
    (dict(in_dtype=N.FO_DT_F32), "in_dtype"),
    (dict(out_dtype=7), "output dtype"),
    (dict(b_layout=5), "b_layout"),
    (dict(epilogue=42), "epilogue"),
    (dict(epilogue=N.FO_EPI_BIAS_RELU), "bias"),
    (dict(lda=60), "lda"),
    (dict(lda=63), "lda"),
    (dict(ldo=100), "ldo"),
    (dict(out=(1 << 20) + 8), "16-byte"),
    (dict(M=-1), "negative"),
    (dict(epilogue=N.FO_EPI_BIAS_LN, bias=1 << 20), "gamma"),
    (dict(epilogue=N.FO_EPI_BN_RELU), "gemm epilogue"),  # BatchNorm epilogues are conv-only
    (dict(epilogue=N.FO_EPI_BIAS_RESIDUAL_LN, bias=1 << 20, gamma=1 << 20, beta=1 << 20), "residual"),
    (dict(epilogue=N.FO_EPI_BIAS_RESIDUAL_LN, bias=1 << 20, gamma=1 << 20, beta=1 << 20, residual=1 << 20, ldr=256,
          N=5000, ldo=5000), "N <= 4096"),
])
def test_gemm_rejects(kw, msg):
    rc = _call(_desc(**kw))
    assert rc == N.FO_EINVAL
    assert msg in N.last_error()


def test_gemm_layernorm_needs_workspace():
    d = _desc(epilogue=N.FO_EPI_BIAS_LN, bias=1 << 20, gamma=1 << 20, beta=1 << 20)
    assert _call(d) == N.FO_EINVAL and "workspace" in N.last_error()
    need = N.lib().fo_gemm_workspace_size(ctypes.byref(d), ctypes.byref(N.tile_cfg(256, 4, 0)))
    # counters for 2 row blocks padded to 256 B + (mean, M2, shift, pad) per row per slice
    # (a slice is half of a 256-column N tile: one epilogue warp's columns)
    assert need == 256 + 256 * 2 * 16


def test_gemm_bad_config():
    assert _call(_desc(), N.tile_cfg(96, 4)) == N.FO_EINVAL
    assert "config" in N.last_error()


def test_empty_output_is_a_no_op():
    assert _call(_desc(M=0)) == N.FO_OK
    assert _call(_desc(N=0)) == N.FO_OK


def test_valid_call_without_gpu_reports_no_device():
    import torch

    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    assert _call(_desc()) == N.FO_ENODEVICE


def test_conv_rejects():
    d = N.FoConvDesc()
    for k, v in dict(n=1, h=8, w=8, c=12, f=64, kh=3, kw=3, stride=1, pad=1, dil=1).items():
        setattr(d, k, v)
    d.x = d.wgt = d.out = 1 << 20
    d.in_dtype = d.out_dtype = N.FO_DT_BF16
    d.epilogue = N.FO_EPI_BIAS_GELU_TANH
    cfg = N.tile_cfg(128, 4, 0)
    assert N.lib().fo_conv2d(ctypes.byref(d), ctypes.byref(cfg), None) == N.FO_EINVAL
    assert "epilogue" in N.last_error()
    d.epilogue = N.FO_EPI_RELU
    assert N.lib().fo_conv2d(ctypes.byref(d), ctypes.byref(cfg), None) == N.FO_EINVAL
    assert "C % 8" in N.last_error()


def _conv_desc(**kw):
    d = N.FoConvDesc()
    for k, v in dict(n=1, h=8, w=8, c=16, f=64, kh=3, kw=3, stride=1, pad=1, dil=1).items():
        setattr(d, k, v)
    d.x = d.wgt = d.out = 1 << 20
    d.in_dtype = d.out_dtype = d.vec_dtype = N.FO_DT_BF16
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,msg", [
    (dict(epilogue=N.FO_EPI_BN), "bn_gamma"),
    (dict(epilogue=N.FO_EPI_BN_RELU, bn_gamma=1 << 20, bn_beta=1 << 20, bn_mean=1 << 20), "bn_var"),
    (dict(epilogue=N.FO_EPI_BN, bn_gamma=1 << 20, bn_beta=1 << 20, bn_mean=1 << 20, bn_var=1 << 20, bn_eps=-1.0),
     "bn_eps"),
    (dict(epilogue=N.FO_EPI_BN_ADD_RELU, bn_gamma=1 << 20, bn_beta=1 << 20, bn_mean=1 << 20, bn_var=1 << 20),
     "residual"),
    (dict(epilogue=N.FO_EPI_BN_ADD_RELU, bn_gamma=1 << 20, bn_beta=1 << 20, bn_mean=1 << 20, bn_var=1 << 20,
          residual=(1 << 20) + 2), "residual"),
    (dict(epilogue=N.FO_EPI_BN_ADD_RELU, bn_gamma=1 << 20, bn_beta=1 << 20, bn_mean=1 << 20, bn_var=1 << 20,
          residual=1 << 20, out_dtype=N.FO_DT_F32), "f16 or bf16"),
    (dict(epilogue=N.FO_EPI_BIAS_LN), "epilogue"),
])
def test_conv_batchnorm_rejects(kw, msg):
    d = _conv_desc(**kw)
    assert N.lib().fo_conv2d(ctypes.byref(d), ctypes.byref(N.tile_cfg(128, 4, 0)), None) == N.FO_EINVAL
    assert msg in N.last_error()


def test_block_k_values():
    assert N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(128, 3, 8, block_k=128))[0]
    ok, why = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(128, 3, 8, block_k=96))
    assert not ok and "block_k" in why
    ok, why = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(256, 3, 8, block_k=128))  # 3 x 96 KB stages
    assert not ok and "shared memory" in why
    # two 64-wide K slices per stage double each stage's bytes
    one = N.config_smem_bytes(0, N.FO_DT_BF16, N.tile_cfg(128, 3, 8))
    two = N.config_smem_bytes(0, N.FO_DT_BF16, N.tile_cfg(128, 3, 8, block_k=128))
    assert two - one == 3 * (128 * 64 * 2 + 128 * 64 * 2)


def test_split_k_field():
    ok, why = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(256, 4, 8, split_k=17))
    assert not ok and "split_k" in why
    assert N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(256, 6, 8, block_m=256, split_k=4))[0]
    d = _desc(M=1000, N=1024, K=4096)
    auto = N.lib().fo_gemm_workspace_size(ctypes.byref(d), ctypes.byref(N.tile_cfg(256, 4, 8)))
    never = N.lib().fo_gemm_workspace_size(ctypes.byref(d), ctypes.byref(N.tile_cfg(256, 4, 8, split_k=1)))
    four = N.lib().fo_gemm_workspace_size(ctypes.byref(d), ctypes.byref(N.tile_cfg(256, 4, 8, split_k=4)))
    # 32 tiles < 148 SMs, 64 k-blocks: at most 4 parts fit the idle SMs; the cost model
    # (k-blocks per part vs reading 128 KB partials at ~30 GB/s) picks 3; 8 counters per
    # tile (one per epilogue warp: 1 KB), then one fp32 partial tile per part
    assert never == 0
    assert auto == 1024 + 32 * 3 * 128 * 256 * 4 and four == 1024 + 32 * 4 * 128 * 256 * 4
    pair = N.lib().fo_gemm_workspace_size(ctypes.byref(d), ctypes.byref(N.tile_cfg(256, 6, 8, block_m=256)))
    assert pair == 1024 + 16 * 2 * 3 * 128 * 256 * 4  # 16 pair tiles, 2 slots each, 3 parts


def test_split_mode_field():
    """split_mode: 0 automatic, 1 workspace, 2 cluster; anything else is rejected."""
    for mode in (0, 1, 2):
        assert N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(128, 6, 8, split_k=2, split_mode=mode))[0]
    for bad in (-1, 3):
        ok, why = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(128, 6, 8, split_mode=bad))
        assert not ok and "split_mode" in why
    assert ctypes.sizeof(N.FoTileCfg) == 10 * 4  # the header's FoTileCfg: ten int32 fields


def test_ln_mode_field_and_workspace():
    """ln_mode: 0 automatic, 1 two kernels, 2 one kernel, 3 one kernel with the slices
    held in TMEM.  The LayerNorm workspace holds
    the 32-row groups' arrival counters (two int32 each, 256-byte padded) and then one
    16-byte statistic per row per half-tile slice."""
    for mode in (0, 1, 2, 3):
        assert N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(128, 6, 8, ln_mode=mode))[0]
    for bad in (-1, 4):
        ok, why = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(128, 6, 8, ln_mode=bad))
        assert not ok and "ln_mode" in why
    d = N.FoGemmDesc()
    d.M, d.N, d.K, d.epilogue = 16384, 4096, 4096, N.FO_EPI_BIAS_LN
    size = N.lib().fo_gemm_workspace_size(ctypes.byref(d), ctypes.byref(N.tile_cfg(256, 3, 8, block_m=256)))
    assert size == 512 * 8 + 32 * 16384 * 16


def test_timeout_setting():
    with pytest.raises(N.FoError):
        N.set_wait_timeout_ns(0)
    N.set_wait_timeout_ns(2_000_000_000)


def test_operators_refuse_cpu_tensors():
    import torch

    from icpp_tuning_b200 import fused

    a = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        fused.gemm(a, a.t().contiguous())
