"""Restatement of the reference's BERT encoder forward (test infrastructure only).

Follows evaluation/end2end.py:43-89 (`bert_fwd_std`) operation by operation in plain
PyTorch on whatever device the tensors live: qkv = precomputed qkv + bias (:48, the
reference feeds a random [b, s, 3h] tensor instead of a projection), causal attention
with scores scaled by 1/sqrt(head_size) and a -10000 upper-triangular mask (:56-68),
output projection + bias + residual + LayerNorm (:76-79), GELU(erf) MLP (:82-83), second
projection + bias + residual + LayerNorm (:84-87).  fp16 throughout, as the reference.
Pinned: tests/golden/ref_ops.pt holds the output of the reference's own bert_fwd_std,
executed from its source on CPU (2 layers, small sizes; tests/golden/make_golden.py
supplies the util/ helpers the reference does not ship), and tests/test_oracle_golden.py
checks this restatement against it.
"""
import math

import torch
import torch.nn.functional as F


def transpose_for_scores(x, head_num, head_size):
    """[b, s, h*d] -> [b, s, h, d].  The reference's helper of this name (imported from
    its missing util/) also permutes to [b, h, s, d], which its code permutes back before
    use; this restatement skips both permutes."""
    return x.view(x.size()[:-1] + (head_num, head_size))


def bert_forward(w, x, head_num, head_size):
    """w: dict of per-layer lists (qkv, qkv_bias, attr_output_kernel, attr_output_bias,
    attr_ln_gamma, attr_ln_beta, inter_kernel, inter_bias, output_kernel, output_bias,
    out_ln_gamma, out_ln_beta); x: [b, s, hidden].  Returns the last layer's output."""
    b, s, hidden = x.shape
    h = x
    for layer in range(len(w["qkv"])):
        inp = h
        qkv = w["qkv"][layer] + w["qkv_bias"][layer]
        q, k, v = (transpose_for_scores(t, head_num, head_size) for t in qkv.chunk(3, dim=-1))
        q = q.permute(0, 2, 1, 3).reshape(b * head_num, s, head_size)
        kt = k.permute(0, 2, 3, 1).reshape(b * head_num, head_size, s)
        scores = torch.baddbmm(torch.empty(b * head_num, s, s, dtype=q.dtype, device=q.device), q, kt, beta=0.0,
                               alpha=1.0 / math.sqrt(head_size)).view(b, head_num, s, s)
        mask = torch.triu(torch.full((s, s), -10000.0, device=x.device), 1)
        att = torch.softmax(scores + mask.to(scores.dtype), dim=-1)
        ctx = torch.einsum("bhts,bshd->bthd", att, v).to(q.dtype).reshape(b, s, hidden)
        h = torch.matmul(ctx, w["attr_output_kernel"][layer]) + w["attr_output_bias"][layer]
        h = F.layer_norm(h + inp, (hidden,), weight=w["attr_ln_gamma"][layer], bias=w["attr_ln_beta"][layer])
        res = h
        h = F.gelu(torch.matmul(h, w["inter_kernel"][layer]) + w["inter_bias"][layer])
        h = torch.matmul(h, w["output_kernel"][layer]) + w["output_bias"][layer]
        h = F.layer_norm(h + res, (hidden,), weight=w["out_ln_gamma"][layer], bias=w["out_ln_beta"][layer])
    return h
