"""The sm_100a descriptors: every raw config is legal for the C ABI, the Python shared
memory / TMEM model equals the library's, and the BASELINE shapes get a config."""
import pytest

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused
from icpp_tuning_b200.autotuner.cost_model import TuneConfig
from icpp_tuning_b200.autotuner.gpu_spec import known_gpu
from icpp_tuning_b200.autotuner.interface import rank_all, select_best
from icpp_tuning_b200.autotuner import search_space as ss
from icpp_tuning_b200.autotuner.tcgen05_space import smem_bytes, tcgen05_configs
from icpp_tuning_b200.conv import conv2d, conv2d_relu
from icpp_tuning_b200.gemm import gemm, gemm_bias_act, gemm_bias_layernorm

B200 = known_gpu("B200")
SHAPES = [
    (gemm_bias_act.DESCRIPTOR, dict(M=1024, N=1024, K=1024)),
    (gemm.DESCRIPTOR, dict(M=4096, N=4096, K=4096)),
    (gemm_bias_act.DESCRIPTORS["gelu_tanh"], dict(M=8192, N=16384, K=4096)),
    (gemm_bias_layernorm.DESCRIPTOR, dict(M=16384, N=4096, K=4096)),
    (conv2d_relu.DESCRIPTOR, dict(N=256, C=128, H=28, W=28, OC=128, KH=3, KW=3, stride=1, padding=1)),
]


@pytest.mark.parametrize("conv", [False, True])
def test_every_config_legal_for_the_library(conv):
    for raw in tcgen05_configs(conv=conv, stages=range(2, 9)):
        cfg = N.tile_cfg(block_n=raw["block_N"], stages=raw["num_stages"], group_m=raw["group_m"],
                         block_m=raw["block_M"], block_k=raw["block_K"], swap_ab=raw.get("swap_ab", 0))
        ok, why = N.config_legal(1 if conv else 0, N.FO_DT_BF16, cfg)
        assert ok, why
        if raw.get("swap_ab") == 2 or raw["block_K"] != 64:
            continue  # the direct conv's shared memory depends on the image width
        want = smem_bytes(raw["block_N"], raw["num_stages"], raw["block_M"])
        assert N.config_smem_bytes(1 if conv else 0, N.FO_DT_BF16, cfg) == want
        tc = TuneConfig(raw["block_M"], raw["block_N"], 64, raw["num_stages"], raw["thread_num"] // 32, kind="tcgen05")
        assert tc.shared_mem_bytes == want
        assert tc.is_valid_for_backend("tcgen05")


def test_library_rejects_illegal_configs():
    for bn, st, why in [(256, 5, "shared memory"), (96, 4, "block_n"), (128, 1, "stages"), (128, 9, "stages")]:
        ok, msg = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(block_n=bn, stages=st))
        assert not ok and why in msg
    ok, msg = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(block_n=128, stages=4, block_m=64))
    assert not ok and "block_m" in msg
    ok, msg = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(block_n=64, stages=4, block_m=256))
    assert not ok and "block_n >= 128" in msg
    ok, msg = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(block_n=256, stages=6, block_m=256))
    assert ok, msg
    ok, msg = N.config_legal(1, N.FO_DT_BF16, N.tile_cfg(block_n=128, stages=2))
    assert not ok  # conv producer needs >= 3 stages


@pytest.mark.parametrize("desc,shape", SHAPES, ids=lambda v: getattr(v, "name", ""))
def test_baseline_shapes_select_legal(desc, shape):
    raw, score = select_best(desc, hw=B200, **shape)
    assert 0.0 < score <= 1.0
    op = 1 if "conv" in desc.name else 0
    ok, why = N.config_legal(op, N.FO_DT_BF16, fused.as_tile_cfg(raw))
    assert ok, why
    rk = rank_all(desc, hw=B200, detailed=True, **shape)
    assert rk[0]["score"] == score
    assert rk[0]["detail"]["projection"]["predicted_tflops"] > 0


def test_layernorm_configs_are_row_major():
    """The one-kernel LayerNorm is offered the row-major raster only (its slices wait for
    their row block's tiles, which that raster finishes soonest)."""
    cfgs = gemm_bias_layernorm.get_gemm_configs(4096)
    assert {c["group_m"] for c in cfgs} == {0} and {c["block_N"] for c in cfgs} == {64, 128, 256}


def test_search_space_tcgen05_prunes_to_library_legal():
    space = ss.generate_search_space("matmul", B200, backend="tcgen05", mode="exhaustive")
    assert space
    for c in space:
        ok, why = N.config_legal(0, N.FO_DT_BF16, N.tile_cfg(block_n=c.block_N, stages=c.num_stages,
                                                              group_m=c.group_size_m, block_m=c.block_M))
        assert ok, why
    full = ss.generate_exhaustive_configs("matmul", "tcgen05")
    assert len(full) > len(space)  # some stage counts exceed 227 KB


def test_search_space_legacy_backends_run():
    # The reference's generate_search_space raises AttributeError (search_space.py:194).
    a100 = known_gpu("A100")
    for backend in ("tilelang", "triton"):
        for op in ("matmul", "conv2d"):
            space = ss.generate_search_space(op, a100, backend=backend, mode="exhaustive")
            assert space and all(c.is_valid_for_backend(backend) for c in space)
    cold = ss.generate_search_space("matmul", a100, backend="tilelang", mode="cold", seed=0)
    assert cold


def test_lcm_marginal_uniformity():
    pools = {"a": [1, 2, 3], "b": [10, 20], "c": [7, 8, 9, 10]}
    cfgs = ss.lcm_marginal_sample(pools, seed=1)
    assert len(cfgs) == 12
    for k, vals in pools.items():
        counts = {v: sum(1 for c in cfgs if c[k] == v) for v in vals}
        assert len(set(counts.values())) == 1


def test_cluster_split_plan_mirror():
    """The model's mirror of the library's automatic cluster split (plan_cluster_split plus
    the fallback over sizes that do not all fit the GPU at once)."""
    from icpp_tuning_b200.autotuner.tcgen05_model import _smem_bytes, cluster_split_plan, cluster_stages
    from icpp_tuning_b200.autotuner.tcgen05_space import smem_bytes

    assert _smem_bytes(128, 6, 1, 0) == smem_bytes(128, 6)
    assert cluster_split_plan(12, 48, 1, 148, 64, 6) in (6, 8)  # 128 x 768 x 3072: a long K loop
    assert cluster_split_plan(48, 12, 2, 148, 64, 4) == 0      # 128 x 3072 x 768: too little K
    assert cluster_split_plan(100, 64, 1, 148, 64, 6) == 0     # more than half a wave of tiles
    assert cluster_split_plan(6, 48, 1, 148, 128, 6) >= 2      # stages drop to fit the receive area
    assert cluster_stages(128, 6, 1, 8) < 6


def test_residual_layernorm_descriptor_ranks_split_configs():
    """The residual LayerNorm runs a plain GEMM + bias kernel, which may split along K;
    its descriptor ranks configs as that kernel (128-column tiles with a cluster split
    for 1024 x 768 x 3072), unlike the in-kernel LayerNorm descriptor."""
    from icpp_tuning_b200.autotuner.interface import select_best
    from icpp_tuning_b200.gemm import gemm_bias_layernorm as G

    assert G.RESIDUAL_DESCRIPTOR.name == "gemm_bias_residual_layernorm"
    cfg, _ = select_best(G.RESIDUAL_DESCRIPTOR, M=1024, N=768, K=3072)
    assert cfg["block_N"] == 128 and cfg["block_M"] == 128
