"""Decision table and adaptive selector (the measured level the reference's autotuner
design describes): table construction, interval merging, lookup, JSON round trip and
the formula fallback, with a deterministic fake timer (no GPU)."""
from icpp_tuning_b200.autotuner import decision_table as dt
from icpp_tuning_b200.gemm import gemm
from icpp_tuning_b200.conv import conv2d_relu

A = {"block_M": 128, "block_N": 64, "block_K": 64, "num_stages": 8, "thread_num": 192, "group_m": 0}
B = {"block_M": 256, "block_N": 256, "block_K": 64, "num_stages": 6, "thread_num": 192, "group_m": 8}


def fake_timer(shape, cfg):
    # narrow tiles win below M = 300, pairs above; config B is illegal for K = 1
    if shape["K"] == 1 and cfg is B:
        return None
    m = shape["M"]
    return (1.0 + m / 100.0) if cfg is A else (3.5 + m / 1000.0)


def test_table_picks_measured_best_and_merges_intervals():
    shapes = [{"M": m, "N": 2304, "K": 768} for m in (1, 64, 128, 256, 512, 1024)]
    table = dt.build_decision_table("gemm", dt.profile(shapes, [A, B], fake_timer))
    assert table.intervals((2304, 768)) == [(1, 256, A), (512, 1024, B)]
    assert table.lookup(M=64, N=2304, K=768) == A
    assert table.lookup(M=700, N=2304, K=768) == B   # nearest profiled point: 512
    assert table.lookup(M=300, N=2304, K=768) == A   # nearer to 256
    assert table.lookup(M=2048, N=2304, K=768) is None  # outside the profiled range
    assert table.lookup(M=64, N=4096, K=768) is None    # unprofiled (N, K)


def test_failed_timings_are_skipped():
    shapes = [{"M": 512, "N": 64, "K": 1}]
    table = dt.build_decision_table("gemm", dt.profile(shapes, [A, B], fake_timer))
    assert table.lookup(M=512, N=64, K=1) == A


def test_json_round_trip(tmp_path):
    shapes = [{"M": m, "N": 2304, "K": 768} for m in (1, 512)]
    table = dt.build_decision_table("gemm", dt.profile(shapes, [A, B], fake_timer))
    table.save(tmp_path / "t.json")
    back = dt.DecisionTable.load(tmp_path / "t.json")
    assert back.groups == table.groups and back.op == "gemm"


def test_adaptive_tuner_levels():
    shapes = [{"M": m, "N": 2304, "K": 768} for m in (1, 512)]
    table = dt.build_decision_table("gemm", dt.profile(shapes, [A, B], fake_timer))
    tuner = dt.AdaptiveTuner(gemm.DESCRIPTOR, table)
    hit = tuner.select(M=1, N=2304, K=768)
    assert hit.level == "table" and hit.config == A and hit.score is None
    miss = tuner.select(M=4096, N=4096, K=4096)
    assert miss.level == "formula" and 0 < miss.score <= 1
    assert miss.config["block_M"] in (128, 256)


def test_conv_groups_by_layer_and_profiles_batch():
    plan = dt.build_sampling_plan("conv2d_relu", m_points=(1, 8))
    assert len(plan) == 8 and {s["N"] for s in plan} == {1, 8}
    cfgs = dt.candidate_configs(conv2d_relu.DESCRIPTOR, plan[:2], top_k=2)
    assert 1 <= len(cfgs) <= 4
    t = lambda sh, cfg: float(sh["N"]) * (1.0 if cfg is cfgs[0] else 2.0)
    table = dt.build_decision_table("conv2d_relu", dt.profile(plan, cfgs, t))
    assert table.lookup(**plan[0]) == cfgs[0]


def test_evaluate_reports_formula_accuracy():
    shapes = [{"M": m, "N": 2304, "K": 768} for m in (1, 1024)]
    cfgs = dt.candidate_configs(gemm.DESCRIPTOR, shapes, top_k=2)
    timer = lambda sh, cfg: 1.0 if cfg is cfgs[-1] else 2.0  # the last candidate is always fastest
    ev = dt.evaluate(gemm.DESCRIPTOR, shapes, dt.profile(shapes, cfgs, timer))
    assert ev["shapes"] == 2 and 0 <= ev["top1"] <= 1 and 0.5 <= ev["mean_ratio"] <= 1.0


def test_shipped_b200_tables_load_and_answer():
    from icpp_tuning_b200.gemm import gemm_bias_layernorm

    for op in ("gemm", "gemm_bias_layernorm", "conv2d_relu"):
        t = dt.shipped_table(op)
        assert t is not None and t.op == op and t.groups
    tuner = dt.AdaptiveTuner(gemm_bias_layernorm.DESCRIPTOR, table="shipped")
    r = tuner.select(M=1024, N=2304, K=768)
    assert r.level == "table" and r.config["block_K"] == 64
    assert dt.AdaptiveTuner(gemm.DESCRIPTOR, table="shipped").select(M=100000, N=2304, K=768).level == "formula"
