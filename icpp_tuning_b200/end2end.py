"""BERT encoder forward with the fused B200 operators (reference evaluation/end2end.py).

The reference times a pure-PyTorch BERT / LLaMA forward and calls none of its own
kernels; its fusion sites are the attention output projection + bias + residual +
LayerNorm (end2end.py:76-79), the MLP up-projection + bias + GELU (:82-83) and the
down-projection + bias + residual + LayerNorm (:84-87).  Here those three sites call
`fused.gemm` (epilogues "bias_residual_layernorm" and "bias_gelu_erf"); attention stays
PyTorch (scaled_dot_product_attention, causal), outside this package's operator family.
The reference's util/ helpers are not in its repository; the two it needs
(seqlen masks, transpose_for_scores) are small and restated inline.

    python -m icpp_tuning_b200.end2end --model bert_base --batch_size 8 --seq_len 512
"""
from __future__ import annotations

import argparse
import time
from typing import Dict, List

import torch
import torch.nn.functional as F

from . import fused
from .autotuner.interface import select_best
from .gemm import gemm_bias_act, gemm_bias_layernorm

MODELS = {"bert_small": (8, 6), "bert_base": (12, 12), "bert_large": (16, 24)}  # heads, layers (:222-236)
HEAD_SIZE = 64


def make_weights(layers: int, hidden: int, batch: int, seq: int, device="cuda", dtype=torch.float16,
                 seed: int = 0) -> Dict[str, List[torch.Tensor]]:
    """The reference's weights: U(-0.4, 0.4) for every tensor (end2end.py:271-285)."""
    g = torch.Generator().manual_seed(seed)

    def u(*shape):
        return (torch.rand(*shape, generator=g) * 0.8 - 0.4).to(dtype).to(device)

    w = {k: [] for k in ("qkv", "qkv_bias", "attr_output_kernel", "attr_output_bias", "attr_ln_gamma", "attr_ln_beta",
                         "inter_kernel", "inter_bias", "output_kernel", "output_bias", "out_ln_gamma", "out_ln_beta")}
    for _ in range(layers):
        w["qkv"].append(u(batch, seq, 3 * hidden))
        w["qkv_bias"].append(u(3 * hidden))
        w["attr_output_kernel"].append(u(hidden, hidden))
        w["attr_output_bias"].append(u(hidden))
        w["attr_ln_gamma"].append(u(hidden))
        w["attr_ln_beta"].append(u(hidden))
        w["inter_kernel"].append(u(hidden, 4 * hidden))
        w["inter_bias"].append(u(4 * hidden))
        w["output_kernel"].append(u(4 * hidden, hidden))
        w["output_bias"].append(u(hidden))
        w["out_ln_gamma"].append(u(hidden))
        w["out_ln_beta"].append(u(hidden))
    return w


class FusedBert:
    """One BERT encoder stack; tile configs are chosen once per shape by the autotuner."""

    def __init__(self, w: Dict[str, List[torch.Tensor]], head_num: int, tokens: int):
        self.w, self.head_num = w, head_num
        hidden = w["attr_output_kernel"][0].shape[0]
        self.hidden = hidden
        rln = gemm_bias_layernorm.RESIDUAL_DESCRIPTOR
        self.cfg_out, _ = select_best(rln, M=tokens, N=hidden, K=hidden)
        self.cfg_up, _ = select_best(gemm_bias_act.DESCRIPTORS["gelu_erf"], M=tokens, N=4 * hidden, K=hidden)
        self.cfg_down, _ = select_best(rln, M=tokens, N=hidden, K=4 * hidden)
        # One zero-filled split-K workspace for the three sites (they run in order on one
        # stream, and the library leaves it zeroed): lets tiles of a partial wave split
        # along K when a cluster split does not apply.
        dev = w["attr_output_kernel"][0].device
        need = max(fused.workspace_bytes(tokens, hidden, hidden, "bias", self.cfg_out),
                   fused.workspace_bytes(tokens, 4 * hidden, hidden, "bias_gelu_erf", self.cfg_up),
                   fused.workspace_bytes(tokens, hidden, 4 * hidden, "bias", self.cfg_down))
        self.ws = torch.zeros(max(16, need), dtype=torch.uint8, device=dev)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        w, hn, hidden = self.w, self.head_num, self.hidden
        b, s, _ = x.shape
        h = x.reshape(b * s, hidden)
        for layer in range(len(w["qkv"])):
            inp = h
            qkv = w["qkv"][layer] + w["qkv_bias"][layer]
            q, k, v = (t.reshape(b, s, hn, HEAD_SIZE).transpose(1, 2) for t in qkv.chunk(3, dim=-1))
            ctx = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(b * s, hidden)
            h = fused.gemm(ctx, w["attr_output_kernel"][layer], epilogue="bias_residual_layernorm",
                           bias=w["attr_output_bias"][layer], gamma=w["attr_ln_gamma"][layer],
                           beta=w["attr_ln_beta"][layer], residual=inp, config=self.cfg_out, workspace=self.ws)
            res = h
            u = fused.gemm(h, w["inter_kernel"][layer], epilogue="bias_gelu_erf", bias=w["inter_bias"][layer],
                           config=self.cfg_up, workspace=self.ws)
            h = fused.gemm(u, w["output_kernel"][layer], epilogue="bias_residual_layernorm",
                           bias=w["output_bias"][layer], gamma=w["out_ln_gamma"][layer], beta=w["out_ln_beta"][layer],
                           residual=res, config=self.cfg_down, workspace=self.ws)
        return h.reshape(b, s, hidden)


def torch_sdpa_bert(w: Dict[str, List[torch.Tensor]], head_num: int):
    """FusedBert's graph with PyTorch at the three fusion sites (matmul + bias + residual
    + layer_norm, addmm + gelu): isolates what the fused operators gain from what the
    attention (SDPA in both) gains over the reference's unfused softmax(QK^T)V."""
    hidden = w["attr_output_kernel"][0].shape[0]

    def run(x):
        b, s, _ = x.shape
        h = x.reshape(b * s, hidden)
        for layer in range(len(w["qkv"])):
            inp = h
            qkv = w["qkv"][layer] + w["qkv_bias"][layer]
            q, k, v = (t.reshape(b, s, head_num, HEAD_SIZE).transpose(1, 2) for t in qkv.chunk(3, dim=-1))
            ctx = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(b * s, hidden)
            h = torch.addmm(w["attr_output_bias"][layer], ctx, w["attr_output_kernel"][layer])
            h = F.layer_norm(h + inp, (hidden,), w["attr_ln_gamma"][layer], w["attr_ln_beta"][layer])
            res = h
            u = F.gelu(torch.addmm(w["inter_bias"][layer], h, w["inter_kernel"][layer]))
            h = torch.addmm(w["output_bias"][layer], u, w["output_kernel"][layer])
            h = F.layer_norm(h + res, (hidden,), w["out_ln_gamma"][layer], w["out_ln_beta"][layer])
        return h.reshape(b, s, hidden)

    return run


def torch_native_bert(w: Dict[str, List[torch.Tensor]], head_num: int):
    """The reference's unfused PyTorch formulation (evaluation/end2end.py:43-89): attention
    as explicit scaled scores, a -10000 upper-triangular mask and softmax, then separate
    matmul / bias / residual / layer_norm and matmul / bias / gelu ops."""
    hidden = w["attr_output_kernel"][0].shape[0]

    def run(x):
        b, s, _ = x.shape
        mask = torch.triu(torch.full((s, s), -10000.0, device=x.device), 1).to(x.dtype)
        h = x
        for layer in range(len(w["qkv"])):
            inp = h
            qkv = w["qkv"][layer] + w["qkv_bias"][layer]
            q, k, v = (t.reshape(b, s, head_num, HEAD_SIZE).transpose(1, 2) for t in qkv.chunk(3, dim=-1))
            att = torch.softmax(torch.matmul(q, k.transpose(-1, -2)) * (HEAD_SIZE ** -0.5) + mask, dim=-1)
            ctx = torch.matmul(att, v).transpose(1, 2).reshape(b, s, hidden)
            h = torch.matmul(ctx, w["attr_output_kernel"][layer]) + w["attr_output_bias"][layer]
            h = F.layer_norm(h + inp, (hidden,), w["attr_ln_gamma"][layer], w["attr_ln_beta"][layer])
            res = h
            h = F.gelu(torch.matmul(h, w["inter_kernel"][layer]) + w["inter_bias"][layer])
            h = torch.matmul(h, w["output_kernel"][layer]) + w["output_bias"][layer]
            h = F.layer_norm(h + res, (hidden,), w["out_ln_gamma"][layer], w["out_ln_beta"][layer])
        return h

    return run


def main() -> None:
    ap = argparse.ArgumentParser(description="BERT forward with B200 fused operators")
    ap.add_argument("--model", default="bert_base", choices=sorted(MODELS))
    ap.add_argument("--batch_size", type=int, default=1)
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--method", default="B200Fused", choices=["B200Fused", "TorchNative", "TorchSDPA"],
                    help="TorchNative: the reference's PyTorch formulation; TorchSDPA: this module's graph "
                         "with PyTorch ops at the fusion sites")
    ap.add_argument("--cuda_graph", action="store_true",
                    help="capture one forward into a CUDA graph and time its replays")
    args = ap.parse_args()
    heads, layers = MODELS[args.model]
    hidden = heads * HEAD_SIZE
    torch.manual_seed(0)
    w = make_weights(layers, hidden, args.batch_size, args.seq_len)
    x = (torch.rand(args.batch_size, args.seq_len, hidden) * 0.8 - 0.4).half().cuda()
    if args.method == "B200Fused":
        runner, label = FusedBert(w, heads, args.batch_size * args.seq_len), "B200 Fused"
    elif args.method == "TorchSDPA":
        runner, label = torch_sdpa_bert(w, heads), "Torch SDPA"
    else:
        runner, label = torch_native_bert(w, heads), "Torch Native"
    if args.cuda_graph:
        from .graphs import CapturedStep

        with torch.no_grad():
            runner = CapturedStep(runner, [x])
        label += " (CUDA graph)"
    with torch.no_grad():
        for i in range(20):
            if i == 10:
                torch.cuda.synchronize()
                t0 = time.perf_counter()
            runner(x)
        torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1000 / 10
    print("e2e {} | bs:{} | seq:{}  |  {} : {:.3f} ms / iter".format(args.model, args.batch_size, args.seq_len, label, ms))


if __name__ == "__main__":
    main()
