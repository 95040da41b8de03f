"""NHWC conv2d as implicit GEMM (reference kernel/tilelang/conv/conv2d.py).

GEMM view (conv2d.py:208-279): M = N*OH*OW output pixels, N_gemm = F output channels,
K = KH*KW*C with channels fastest, matching the weight layout [KH, KW, C, F] the
reference uses (:224).  The reference gathers im2col element by element through
registers (:238-251); here a 128-thread producer warpgroup gathers each 128 x 64 A tile
with 16-byte cp.async (zero-fill supplies the padding), the weights stream in by TMA as an
MN-major operand, and tcgen05 accumulates in TMEM.

Reference surface kept: get_conv_op_shape_list(), get_ref_program(...), calc_oh_ow,
calc_conv_flops, reduce_shapes_preserve_scale_distribution, get_configs(),
build_conv2d_kernel(N, C, H, W, F_out, KH, KW, S=1, P=1, D=1, config=None) ->
kernel(X, W, Y) writing Y in place, verify_correctness, Conv2dDescriptor / DESCRIPTOR.
"""
from __future__ import annotations

import math
from typing import Any, Dict, List, Optional

import torch
import torch.nn.functional as F

from .. import fused
from ..autotuner.cost_model import make_conv2d_spec
from ..autotuner.interface import select_best
from ..autotuner.tcgen05_space import Tcgen05Descriptor, tcgen05_configs


def calc_oh_ow(H, W, KH, KW, S, P, D):
    OH = (H + 2 * P - D * (KH - 1) - 1) // S + 1
    OW = (W + 2 * P - D * (KW - 1) - 1) // S + 1
    return OH, OW


def calc_conv_flops(N, C, OH, OW, F_out, KH, KW):
    return 2 * N * OH * OW * F_out * C * KH * KW


def get_ref_program(stride=1, padding=1, dilation=1, use_compile=False):
    """The reference's expected result (conv2d.py:35-62): ref(X, W, Y) writes
    conv(X, W) into Y (NHWC in, [KH,KW,C,F] weights).  Eager PyTorch; use_compile is
    accepted for signature compatibility."""

    def ref_program(X, W, Y):
        y = F.conv2d(X.permute(0, 3, 1, 2), W.permute(3, 2, 0, 1), stride=stride, padding=padding,
                     dilation=dilation)
        Y[...] = y.permute(0, 2, 3, 1).to(Y.dtype)

    return ref_program


def get_configs() -> List[Dict[str, Any]]:
    return tcgen05_configs(conv=True, group_ms=(0,), stages=(3, 4, 6, 8))


class Conv2dDescriptor(Tcgen05Descriptor):
    primitives: tuple = ()

    @property
    def name(self) -> str:
        return "conv2d"

    def make_op_spec(self, raw_config=None, N=1, C=1, H=1, W=1, OC=1, KH=1, KW=1, stride=1, padding=0,
                     **kw):
        return make_conv2d_spec(N, C, H, W, OC, KH, KW, stride=stride, padding=padding,
                                primitives=list(self.primitives))

    def get_raw_configs(self, **kw):
        return get_configs()


DESCRIPTOR = Conv2dDescriptor()


def _select(desc, N, C, H, W, F_out, KH, KW, S, P, config):
    if config is None:
        config, _ = select_best(desc, N=N, C=C, H=H, W=W, OC=F_out, KH=KH, KW=KW, stride=S, padding=P)
    return config


def build_conv2d_kernel(N, C, H, W, F_out, KH, KW, S=1, P=1, D=1, config=None):
    """Returns kernel(X, W, Y, bias=None): Y[N,OH,OW,F] = conv(X[N,H,W,C], W[KH,KW,C,F])
    (+ bias), written in place like the reference's callable (conv2d.py:282-290)."""
    config = _select(DESCRIPTOR, N, C, H, W, F_out, KH, KW, S, P, config)
    cfg = fused.as_tile_cfg(config)
    OH, OW = calc_oh_ow(H, W, KH, KW, S, P, D)
    ws_bytes = fused.conv_workspace_bytes(N, H, W, C, F_out, KH, KW, S, P, D, config=cfg)
    # zero-filled once per stream; the kernel leaves its split-K counters zeroed after every call
    wss = fused.StreamWorkspaces(ws_bytes)

    def kernel(X, Wt, Y, bias=None):
        if tuple(X.shape) != (N, H, W, C) or tuple(Wt.shape) != (KH, KW, C, F_out):
            raise ValueError("input shapes differ from the built shape")
        fused.conv2d_nhwc(X, Wt, bias=bias, relu=False, stride=S, padding=P, dilation=D, out=Y, workspace=wss.get(), config=cfg)
        return Y

    kernel.config = config
    kernel.out_shape = (N, OH, OW, F_out)
    kernel.workspace = wss.default
    return kernel


def verify_correctness(kernel, ref_prog, N, C, H, W, F_out, KH, KW, S, P, D, seed: Optional[int] = None):
    """True when kernel matches ref_prog within the reference's tolerance
    (assert_close rtol = atol = 1e-2, conv2d.py:293-314) on fresh randn fp16 inputs."""
    OH, OW = calc_oh_ow(H, W, KH, KW, S, P, D)
    g = torch.Generator(device="cuda")
    if seed is not None:
        g.manual_seed(seed)
    X = torch.randn(N, H, W, C, dtype=torch.float16, device="cuda", generator=g)
    Wt = torch.randn(KH, KW, C, F_out, dtype=torch.float16, device="cuda", generator=g)
    Y_ref = torch.zeros(N, OH, OW, F_out, dtype=torch.float16, device="cuda")
    Y = torch.zeros_like(Y_ref)
    ref_prog(X, Wt, Y_ref)
    kernel(X, Wt, Y)
    try:
        torch.testing.assert_close(Y, Y_ref, rtol=1e-2, atol=1e-2)
        return True
    except AssertionError:
        return False


def reduce_shapes_preserve_scale_distribution(shapes, target_count=200, num_bins=10):
    """Subsample conv shapes keeping their log10-FLOPs distribution (conv2d.py:75-168):
    bin by log10 FLOPs, allocate target_count across bins by size, sample evenly inside
    each bin."""
    if target_count <= 0 or len(shapes) <= target_count:
        return list(shapes)
    logs = []
    for (n, c, h, w, f, kh, kw, s, p) in shapes:
        oh, ow = calc_oh_ow(h, w, kh, kw, s, p, 1)
        logs.append(math.log10(max(calc_conv_flops(n, c, oh, ow, f, kh, kw), 1)))
    lo, hi = min(logs), max(logs)
    step = 1.0 if hi == lo else (hi - lo) / max(num_bins, 1)
    bins = [[] for _ in range(num_bins)]
    for i, v in enumerate(logs):
        b = 0 if hi == lo else min(int((v - lo) / step), num_bins - 1)
        bins[b].append(i)
    if not any(bins):
        return list(shapes)[:target_count]
    want = [len(b) * target_count / len(shapes) for b in bins]
    alloc = [int(x) for x in want]
    if target_count >= sum(1 for b in bins if b):
        alloc = [max(a, 1) if b else a for a, b in zip(alloc, bins)]
    total = sum(alloc)
    if total > target_count:
        for i in sorted(range(num_bins), key=lambda i: (want[i] - alloc[i], -alloc[i])):
            if total == target_count:
                break
            if alloc[i] > 0:
                alloc[i] -= 1
                total -= 1
    elif total < target_count:
        order = sorted(range(num_bins), key=lambda i: (want[i] - alloc[i], len(bins[i])), reverse=True)
        ptr = 0
        while total < target_count and order and ptr <= target_count * max(1, num_bins):
            i = order[ptr % len(order)]
            if alloc[i] < len(bins[i]):
                alloc[i] += 1
                total += 1
            ptr += 1
    picked = []
    for i, b in enumerate(bins):
        k = min(alloc[i], len(b))
        if k == len(b):
            picked.extend(b)
        else:
            picked.extend(b[int(j * len(b) / k)] for j in range(k))
    picked = sorted(set(picked))[:target_count]
    if len(picked) < target_count:
        have = set(picked)
        picked += [i for i in range(len(shapes)) if i not in have][:target_count - len(picked)]
    return [shapes[i] for i in picked]
