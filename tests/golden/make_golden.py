"""Generates the golden fixtures of the test suite from the reference itself.

Run in the build container, where the reference is importable (it is absent on GPU
boxes, so the fixtures are committed):

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden.py /path/to/icpp-tuning

1. autotuner_decisions.json -- every row of the reference's published formula runs
   (evaluation/gemm_formula_full.csv, gemm_bias_act_formula_full.csv,
   gemm_bias_layernorm_formula_full.csv, conv2d_formula_changed_after_costmodel.csv):
   op, shape, chosen config string, score.  These pin the cost model.
2. ref_ops.pt -- small seeded inputs and the outputs of the reference's own PyTorch
   programs (kernel/tilelang/gemm/gemm.py:20-21 ref_program, gemm_bias_act.py:44-47
   ref_program, gemm_bias_layernorm.py:44-50 torch_baseline, conv/conv2d.py:35-62
   get_ref_program, conv/conv2d_relu.py:29-60 get_ref_program), run on CPU with
   torch.compile disabled.  These pin the oracle under oracle/.
"""
from __future__ import annotations

import csv
import json
import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def _decisions(ref: Path) -> list:
    rows = []
    ev = ref / "evaluation"
    for name in ("gemm_formula_full.csv", "gemm_bias_act_formula_full.csv",
                 "gemm_bias_layernorm_formula_full.csv"):
        with open(ev / name) as f:
            for r in csv.DictReader(f):
                rows.append({"op": r["op"], "shape": {"M": int(r["M"]), "N": int(r["N"]), "K": int(r["K"])},
                             "config": r["config"], "score": float(r["score"])})
    with open(ev / "conv2d_formula_changed_after_costmodel.csv") as f:
        for r in csv.DictReader(f):
            rows.append({"op": "conv2d",
                         "shape": {"N": int(r["N"]), "C": int(r["C"]), "H": int(r["H"]), "W": int(r["W"]),
                                   "OC": int(r["F_out"]), "KH": int(r["Kernel_H"]), "KW": int(r["Kernel_W"]),
                                   "stride": int(r["Stride"]), "padding": int(r["Pad"])},
                         "config": r["Formula_Config"], "score": float(r["Formula_Score"])})
    return rows


def _load_module(path: Path, name: str, prelude: str = ""):
    src = prelude + path.read_text()
    mod = types.ModuleType(name)
    mod.__file__ = str(path)
    sys.modules[name] = mod
    exec(compile(src, str(path), "exec"), mod.__dict__)
    return mod


def _ref_outputs(ref: Path) -> dict:
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "kernel" / "tilelang" / "conv"))
    from kernel.tilelang.gemm import gemm as g  # noqa: E402
    from kernel.tilelang.gemm import gemm_bias_act as gba  # noqa: E402
    from kernel.tilelang.conv import conv2d as cv  # noqa: E402
    import conv2d_relu as cvr  # noqa: E402
    gbln = _load_module(ref / "kernel/tilelang/gemm/gemm_bias_layernorm.py", "ref_gbln",
                        "from pathlib import Path\nimport sys\n")

    out = {}
    gen = torch.Generator().manual_seed(1234)

    def rn(*s, dt=torch.float16, scale=1.0):
        return (torch.randn(*s, generator=gen) * scale).to(dt)

    # gemm: C = (A @ B) in fp32 (gemm.py:20-21), ragged shape
    for dt in (torch.float16, torch.bfloat16):
        A, B = rn(72, 136, dt=dt, scale=0.5), rn(136, 200, dt=dt, scale=0.5)
        C = torch.empty(72, 200, dtype=torch.float32)
        g.ref_program(A, B, C)
        out[f"gemm_{str(dt)[6:]}"] = {"A": A, "B": B, "C": C}
    # gemm_bias_act (ReLU), fp32 result (gemm_bias_act.py:44-47)
    A, B, bias = rn(96, 128, scale=0.5), rn(128, 192, scale=0.5), rn(192, scale=0.1)
    out["gemm_bias_relu"] = {"A": A, "B": B, "bias": bias, "C": gba.ref_program(A, B, bias)}
    # gemm_bias_layernorm, fp16 result (gemm_bias_layernorm.py:44-50)
    A, B = rn(64, 128), rn(128, 256, scale=128 ** -0.5)
    bias, gamma, beta = rn(256, scale=0.02), (1 + torch.randn(256, generator=gen) * 0.02).half(), rn(256, scale=0.02)
    out["gemm_bias_layernorm"] = {"A": A, "B": B, "bias": bias, "gamma": gamma, "beta": beta,
                                  "C": gbln.torch_baseline(A, B, bias, gamma, beta)}
    # conv2d NHWC (conv2d.py:35-62) and conv2d+relu (conv2d_relu.py:29-60), 3x3 s1 p1
    X, W = rn(2, 6, 5, 16), rn(3, 3, 16, 24, scale=(9 * 16) ** -0.5)
    Y = torch.empty(2, 6, 5, 24, dtype=torch.float16)
    cv.get_ref_program(stride=1, padding=1, use_compile=False)(X, W, Y)
    out["conv2d"] = {"X": X, "W": W, "Y": Y.clone()}
    Y2 = torch.empty(2, 6, 5, 24, dtype=torch.float16)
    cvr.get_ref_program(stride=1, padding=1)(X, W, Y2)
    out["conv2d_relu"] = {"X": X, "W": W, "Y": Y2}
    # a strided conv without padding
    X, W = rn(1, 9, 7, 8), rn(3, 3, 8, 16, scale=72 ** -0.5)
    Y = torch.empty(1, 4, 3, 16, dtype=torch.float16)
    cv.get_ref_program(stride=2, padding=0, use_compile=False)(X, W, Y)
    out["conv2d_s2p0"] = {"X": X, "W": W, "Y": Y}
    return out


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ICPP_REFERENCE", ""))
    if not (ref / "kernel").is_dir():
        raise SystemExit("usage: make_golden.py <path to the icpp-tuning checkout>")
    rows = _decisions(ref)
    (HERE / "autotuner_decisions.json").write_text(json.dumps(rows, indent=1) + "\n")
    torch.save(_ref_outputs(ref), HERE / "ref_ops.pt")
    print(f"wrote {len(rows)} autotuner decisions and ref_ops.pt")


if __name__ == "__main__":
    main()
