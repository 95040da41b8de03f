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
   torch.compile disabled; the BatchNorm conv programs (conv2d_bn.py:29-65,
   conv2d_bn_relu.py:123-160, conv_bn_add_relu.py:29-70); the BERT forward
   bert_fwd_std and new_gelu of evaluation/end2end.py (:43-89, :37-38).  These pin the
   oracle under oracle/.
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
    out.update(_bn_conv_outputs(ref, gen))
    out.update(_end2end_outputs(ref, gen))
    return out


def _bn_conv_outputs(ref: Path, gen: torch.Generator) -> dict:
    """The BatchNorm conv operators' expected results (conv2d_bn.py:29-65, eps 1e-3;
    conv2d_bn_relu.py:123-160; conv_bn_add_relu.py:29-70, whose variance is clamped at 0:
    one channel gets a negative variance to exercise the clamp).  fp16 NHWC in and out."""
    conv_dir = ref / "kernel" / "tilelang" / "conv"
    bn = _load_module(conv_dir / "conv2d_bn.py", "ref_conv2d_bn")
    bnr = _load_module(conv_dir / "conv2d_bn_relu.py", "ref_conv2d_bn_relu")
    bnar = _load_module(conv_dir / "conv_bn_add_relu.py", "ref_conv_bn_add_relu")
    torch.compile = lambda fn, *a, **k: fn  # eager: the CPU inductor does not build here

    def rn(*s, scale=1.0, shift=0.0):
        return (torch.randn(*s, generator=gen) * scale + shift).half()

    out = {}
    X, W = rn(2, 7, 6, 16), rn(3, 3, 16, 24, scale=(9 * 16) ** -0.5)
    gamma, beta, mean = rn(24, scale=0.1, shift=1.0), rn(24, scale=0.1), rn(24, scale=0.1)
    var = (torch.rand(24, generator=gen) * 0.5 + 0.5).half()
    Y = torch.empty(2, 7, 6, 24, dtype=torch.float16)
    bn.get_ref_program(stride=1, padding=1)(X, W, gamma, beta, mean, var, Y)
    out["conv2d_bn"] = {"X": X, "W": W, "gamma": gamma, "beta": beta, "mean": mean, "var": var, "Y": Y.clone()}
    bnr.get_ref_program(stride=1, padding=1)(X, W, gamma, beta, mean, var, Y)
    out["conv2d_bn_relu"] = {"X": X, "W": W, "gamma": gamma, "beta": beta, "mean": mean, "var": var, "Y": Y.clone()}
    var_neg = var.clone()
    var_neg[3] = -0.25
    R = rn(2, 7, 6, 24, scale=0.5)
    bnar.get_ref_program(stride=1, padding=1)(X, W, R, gamma, beta, mean, var_neg, Y)
    out["conv_bn_add_relu"] = {"X": X, "W": W, "residual": R, "gamma": gamma, "beta": beta, "mean": mean,
                               "var": var_neg, "Y": Y.clone()}
    # strided, unpadded BatchNorm + ReLU
    X2 = rn(1, 9, 8, 8)
    W2 = rn(3, 3, 8, 24, scale=72 ** -0.5)
    Y2 = torch.empty(1, 4, 3, 24, dtype=torch.float16)
    bnr.get_ref_program(stride=2, padding=0)(X2, W2, gamma, beta, mean, var, Y2)
    out["conv2d_bn_relu_s2p0"] = {"X": X2, "W": W2, "gamma": gamma, "beta": beta, "mean": mean, "var": var, "Y": Y2}
    return out


def _end2end_outputs(ref: Path, gen: torch.Generator) -> dict:
    """bert_fwd_std (evaluation/end2end.py:43-89) and new_gelu (:37-38), executed from the
    reference source on CPU.  The module imports helpers from a util/ package that the
    reference does not ship (:11-12); stub modules stand in for the two it calls:
    transpose_for_scores ([b, s, h*d] -> [b, h, s, d], the layout the rearrange patterns
    at :55-58 expect after its permute back) and set_dtype.  bert_fwd_std
    reads its weights and sizes from module globals, set here (the reference's main sets
    them at :215-290), on small sizes, 2 layers, fp16, dropout 0 (its default).  Its
    attention calls baddbmm(torch.empty(...), ..., beta=1.0), which adds an
    uninitialised buffer; torch.empty is made to return zeros during the call, so the
    scores are the scaled products (what beta=0 computes)."""
    util = types.ModuleType("util")
    uu = types.ModuleType("util.utils")
    um = types.ModuleType("util.masks")
    uu.transpose_for_scores = lambda x, h, d: x.view(x.size()[:-1] + (h, d)).permute(0, 2, 1, 3)
    uu.set_dtype = lambda t, dt: t.half() if dt == "fp16" else t
    uu.seqlen_to_mask = uu.torch_cuda_identify = uu.time_stamp_cudasync = None
    um.generate_causal_mask = None
    util.utils, util.masks = uu, um
    sys.modules.update({"util": util, "util.utils": uu, "util.masks": um})
    e2e = _load_module(ref / "evaluation" / "end2end.py", "ref_end2end")

    b, s, heads, hd, layers = 2, 16, 2, 64, 2
    hidden = heads * hd

    def u(*shape):
        return (torch.rand(*shape, generator=gen) * 0.8 - 0.4).half()

    w = {"qkv": [u(b, s, 3 * hidden) for _ in range(layers)], "qkv_bias": [u(3 * hidden) for _ in range(layers)],
         "attr_output_kernel": [u(hidden, hidden) for _ in range(layers)],
         "attr_output_bias": [u(hidden) for _ in range(layers)],
         "attr_ln_gamma": [u(hidden) for _ in range(layers)], "attr_ln_beta": [u(hidden) for _ in range(layers)],
         "inter_kernel": [u(hidden, 4 * hidden) for _ in range(layers)],
         "inter_bias": [u(4 * hidden) for _ in range(layers)],
         "output_kernel": [u(4 * hidden, hidden) for _ in range(layers)],
         "output_bias": [u(hidden) for _ in range(layers)],
         "out_ln_gamma": [u(hidden) for _ in range(layers)], "out_ln_beta": [u(hidden) for _ in range(layers)]}
    x = u(b, s, hidden)
    g = e2e.__dict__
    g.update(input_from_tensor=x, layer_num=layers, head_num=heads, head_size=hd, hidden_dim=hidden,
             batch_size=b, seq_len=s, dropout_p=0.0, transformer_output=[None] * layers,
             qkv_kernel=w["qkv"], qkv_bias=w["qkv_bias"], attr_output_kernel=w["attr_output_kernel"],
             attr_output_bias=w["attr_output_bias"], attr_output_layernorm_gamma=w["attr_ln_gamma"],
             attr_output_layernorm_beta=w["attr_ln_beta"], inter_kernel=w["inter_kernel"],
             inter_bias=w["inter_bias"], output_kernel=w["output_kernel"], output_bias=w["output_bias"],
             output_layernorm_gamma=w["out_ln_gamma"], output_layernorm_beta=w["out_ln_beta"])
    empty = torch.empty
    torch.empty = lambda *a, **k: torch.zeros(*a, **k)
    try:
        e2e.bert_fwd_std(None)
    finally:
        torch.empty = empty
    xs = torch.linspace(-8, 8, 2001)
    return {"bert_fwd_std": {"w": w, "x": x, "head_num": heads, "head_size": hd,
                             "out": g["transformer_output"][-1].clone()},
            "new_gelu": {"x": xs, "y": e2e.new_gelu(xs), "x16": xs.half(), "y16": e2e.new_gelu(xs.half())}}


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
