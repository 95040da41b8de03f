"""The formula-benchmark driver: CSV columns of the reference's evaluation outputs and the
markdown summary (host logic only; the sweeps themselves run on a GPU)."""
import csv

import pytest

from icpp_tuning_b200 import formula_bench as fb


def test_csv_columns_match_reference_schemas(tmp_path):
    # header lines of evaluation/gemm_formula_full.csv:1 and conv2d_formula_changed_after_costmodel.csv:1
    assert ",".join(fb.GEMM_FIELDS) == "op,M,N,K,config,runtime_config,score,formula_ms,torch_ms,speedup"
    assert ",".join(fb.CONV_FIELDS) == ("Index,N,C,H,W,F_out,Kernel_H,Kernel_W,Stride,Pad,Formula_Config,"
                                        "Formula_Score,Formula_Latency_ms,Torch_Latency_ms,Speedup_vs_Torch,Is_Correct")
    rows = [{"op": "gemm", "M": 1, "N": 2304, "K": 768, "config": "c", "runtime_config": "c", "score": "0.1",
             "formula_ms": "0.01", "torch_ms": "0.02", "speedup": "2.0"}]
    fb.write_csv(tmp_path / "x.csv", fb.GEMM_FIELDS, rows)
    with open(tmp_path / "x.csv") as f:
        got = list(csv.DictReader(f))
    assert got[0]["speedup"] == "2.0" and list(got[0]) == fb.GEMM_FIELDS


def test_summary_statistics():
    rows = [{"op": op, "M": m, "config": "c", "formula_ms": "1", "torch_ms": str(s), "speedup": str(s)}
            for op in ("gemm", "gemm_bias_layernorm") for m, s in ((1, 0.9), (6, 1.05), (11, 3.0))]
    md = fb.summarize(rows)
    line = next(l for l in md.splitlines() if l.startswith("| `gemm` "))
    assert line.split("|")[2:9] == [" 3 ", " 0.9000 ", " 1.0500 ", " 1.6500 ", " 3.0000 ", " 1 ", " 1 "]
    assert "### gemm_bias_layernorm" in md


def test_sweep_shapes():
    assert list(range(1, 128, 5))[-1] == 126 and len(range(1, 128, 5)) == 26
    assert len(fb.CONV_SHAPES) == 9


def test_captured_step_rejects_host_inputs():
    import torch

    from icpp_tuning_b200.graphs import CapturedStep

    with pytest.raises(ValueError):
        CapturedStep(lambda t: t, [torch.zeros(4)])
