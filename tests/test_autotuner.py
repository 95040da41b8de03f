"""Cost model and descriptor API: the reference's published A100 decisions replay
exactly; the B200 descriptors return configs the C ABI accepts."""
import json
from pathlib import Path

import pytest

from icpp_tuning_b200.autotuner import cost_model as cm
from icpp_tuning_b200.autotuner.gpu_spec import known_gpu
from icpp_tuning_b200.autotuner.interface import TileLangKernelBase, rank_all, select_best
from icpp_tuning_b200.autotuner.legacy import LEGACY_DESCRIPTORS

ROWS = json.loads((Path(__file__).parent / "golden" / "autotuner_decisions.json").read_text())


@pytest.mark.parametrize("row", ROWS, ids=lambda r: f"{r['op']}-{'-'.join(map(str, r['shape'].values()))}")
def test_reference_decisions_replay(row):
    d = LEGACY_DESCRIPTORS[row["op"]]
    raw, score = select_best(d, hw=known_gpu("A100"), **row["shape"])
    assert d.format_config(raw) == row["config"]
    assert round(score, 6) == pytest.approx(row["score"], abs=1e-12)


def test_golden_covers_all_ops():
    assert len(ROWS) == 87
    assert {r["op"] for r in ROWS} == {"gemm", "gemm_bias_act", "gemm_bias_layernorm", "conv2d"}


def test_rank_all_sorted_and_detailed():
    d = LEGACY_DESCRIPTORS["gemm_bias_act"]
    rk = rank_all(d, hw=known_gpu("A100"), detailed=True, M=64, N=2304, K=768)
    assert len(rk) == 72
    scores = [e["score"] for e in rk]
    assert scores == sorted(scores, reverse=True)
    best, s = select_best(d, hw=known_gpu("A100"), M=64, N=2304, K=768)
    assert rk[0]["raw_config"] == best and rk[0]["score"] == s
    det = rk[0]["detail"]
    prod = 1.0
    for k in ("eff_mainloop", "eff_memory", "eff_parallel", "eff_pipeline", "eff_implicit_conv",
              "eff_epilogue", "eff_reduction"):
        assert 0.0 < det[k] <= 1.0
        prod *= det[k]
    assert prod == pytest.approx(det["score"], rel=1e-12)


def test_select_best_no_configs_raises():
    class Empty(TileLangKernelBase):
        name = "empty"

        def make_op_spec(self, raw_config=None, **kw):
            return cm.make_matmul_spec(1, 1, 1)

        def get_raw_configs(self, **kw):
            return []

    with pytest.raises(RuntimeError, match="No configs generated"):
        select_best(Empty(), hw=known_gpu("A100"), M=1, N=1, K=1)


def test_unknown_primitive():
    with pytest.raises(KeyError):
        cm.make_matmul_spec(1, 1, 1, primitives=["softmax"])


def test_format_config():
    d = LEGACY_DESCRIPTORS["gemm"]
    assert d.format_config({"block_M": 16, "block_N": 128, "block_K": 64, "split_k": 2, "num_stages": 4,
                            "thread_num": 256}) == "BM16_BN128_BK64_SK2_S4_T256"


def test_conv_spec_geometry():
    op = cm.make_conv2d_spec(256, 128, 28, 28, 128, 3, 3, stride=1, padding=1)
    assert (op.M, op.N, op.K) == (256 * 28 * 28, 128, 1152)
    assert op.mainloop.mainloop_flops == 2 * 256 * 28 * 28 * 128 * 128 * 9
