"""Cost model of the sm_100a kernels in this package (TuneConfig.kind == "tcgen05").

The reference's factors (kernel/autotuner/cost_model.py:544-757) describe a
register-tiled kernel: outputs per thread, occupancy from registers, warps per block.
None of those exist in a persistent, warp-specialised tcgen05 kernel: the accumulator
lives in TMEM, one CTA owns an SM, and the warp split is fixed.  This module keeps the
reference's shape -- a product of seven factors in (0, 1], the same factor names, the
same `score_formula` entry point -- but derives each factor from a time model of one SM
running this design (docs/cost_model.md of the reference describes the factor idea):

  eff_mainloop      tile padding of M / N / K x tensor-pipe rate of a 128 x BN x 16 MMA
                    (narrow N re-reads A from shared memory more often per FLOP)
  eff_memory        compute time / HBM time, with operand re-reads across waves set by
                    the tile raster (group_m) and the 126 MB L2
  eff_parallel      SM-time actually used: wave quantisation of the persistent grid over
                    148 SMs, plus the fixed launch / prologue / drain time
  eff_pipeline      whether `stages` k-blocks in flight cover the TMA latency
  eff_implicit_conv conv only: rate of the TMA im2col loads relative to tiled loads
  eff_epilogue      overlap of the epilogue (TMEM -> registers -> TMA store) with the
                    next tile's mainloop (two TMEM accumulators)
  eff_reduction     LayerNorm only: the normalisation (in the GEMM kernel for block_n >=
                    128, else a stream-ordered in-place pass)

score = product = (ideal tensor time) / (predicted time).  The constants in CONSTANTS
are fitted to B200 measurements of these kernels.
"""
from __future__ import annotations

import math

from .cost_model import OpSpec, TuneConfig
from .gpu_spec import GPUSpec

CONSTANTS = {
    # relative tensor-pipe rate of one 128 x BN x 16 MMA (shared-memory operand traffic)
    # measured on B200 (4096^3 bf16, same stages / raster): BN=256 1267, BN=128 836,
    # BN=64 462 TFLOP/s -- narrow tiles are bound by shared-memory operand traffic
    "mma_rate_bn": {256: 1.0, 128: 0.66, 64: 0.37},
    # CTA pairs (block_M 256): each SM loads half of B (4096^3: BN=128 pairs 837, BN=256 pairs 1274)
    "mma_rate_bn_pair": {256: 1.03, 128: 0.66},  # measured: pairs do not lift narrow tiles
    "mma_rate_bn_bk128": {256: 0.85, 128: 0.71, 64: 0.39},  # two K slices per stage (4096^3 sweeps)
    # pairs, two K slices per stage: 4096^3 107 vs 127 us and 8192^3 692 vs 860 us against
    # block_K 64 on one box (box-to-box: 0-20% faster, never slower beyond noise)
    "mma_rate_bn_pair_bk128": {256: 1.08, 128: 0.7},
    "hbm_efficiency": 0.8,  # achievable fraction of the HBM figure in the GPU spec
    "mem_overlap": 0.35,  # share of the shorter of (compute, HBM) time that does not overlap
    # stages - 1 loads in flight must cover this latency (4096^3: 3 stages run at 0.9 of 4)
    "tma_latency_s": 0.8e-6,
    # achievable share of the nominal dense peak under the 1 kW power cap (cuBLAS bf16
    # 8192^3 measured 1680 of 2250 TFLOP/s on this pool)
    "tensor_rate_fraction": 0.75,
    "epi_bytes_per_s_sm": 120e9,  # epilogue store throughput of one SM (TMEM ld + TMA store)
    # LayerNorm normalisation pass (separate stream-ordered kernel), read + write bytes/s:
    # 16384 x 4096 bf16 measured ~100 us on top of the GEMM
    "ln_pass_bytes_per_s": 2.6e12,
    # one-kernel LayerNorm (block_n >= 128): the epilogue's statistics and in-place
    # normalisation, per read + write byte of the output (config4: 58 us over the plain
    # GEMM + bias kernel for 2 x 128 MiB)
    "ln_fused_bytes_per_s": 4.6e12,
    "ln_fused_tail_s": 7.4e-6,  # its normalisation after the last unit (2048 x 4096: +2.7 us)
    # slices held in TMEM (<= 4 waves): the extra epilogue time as a share of a separate
    # row pass's (measured 2-5% faster than the two-kernel path on 8192 x 768..1024 and
    # 2048..4096 x 4096 shapes, whose row pass is 8-15% of the call)
    "ln_held_factor": 0.6,
    # TMA im2col loads (one 128-pixel x 64-channel box per filter tap) run at this share
    # of a tiled load's rate: measured 589 vs 836 TFLOP/s for BN=128 conv vs GEMM tiles
    "im2col_rate": 0.7,
    # direct conv: mainloop rate of a 128 x (rows x pitch) tile per taps-per-weight-stage
    # (one MMA issue wait per stage, issued by a warp-uniform loop; config5 224-position
    # tiles measured 56.3 / 56.5 / 59.7 us for 1 tap x 6 stages, 2 x 3 and 3 x 2), and the
    # factor when only one pixel slot fits (its reload is then not overlapped)
    "direct_rate_kps": {1: 0.875, 2: 0.87, 3: 0.82},
    "direct_one_slot": 0.7,
    # residual read of the conv + BN + add + ReLU epilogue, per SM, added to each tile's
    # time (measured against the same kernels without it: the im2col kernel's lane-per-row
    # loads ~17 GB/s, the direct conv's pixel-per-lane loads and transpose ~11 GB/s)
    "residual_bytes_per_s_sm": 17e9,
    "direct_residual_bytes_per_s_sm": 11e9,
    "mma_issue_cycles": 130,  # one thread issuing back-to-back MMAs with a wait per stage
    "fixed_s": 6.0e-6,  # launch + TMEM alloc + pipeline fill + last epilogue
    "pair_fixed_s": 1.0e-6,  # extra fixed cost of a CTA-pair launch (cluster start and exit)
    "split_overhead_s": 2.0e-6,  # partial write -> fence -> atomic -> reduce chain
    # the last-arriving CTA reads each other part's fp32 partial (128 x bn x 4 B) at this rate
    "split_read_bytes_per_s": 30e9,
    # one k-block of a 128 x 256 tile on one SM under the power cap (4096^3: 101 us / 3.46 waves / 64)
    "split_t_kb256_s": 0.45e-6,
    # cluster split-K (fo_api.cu plan_cluster_split): one 64-wide k-block of a single-wave
    # 128-row tile (any block_N), the cluster's start / exchange / exit cost as
    # c0 + c1 x parts per block_N, and how many clusters of each size the GPU holds at
    # once (measured on B200 with one CTA per SM)
    "cluster_t_kb64_s": 0.30e-6,
    "cluster_cost_s": {64: (0.9e-6, 0.32e-6), 128: (1.9e-6, 0.5e-6), 256: (2.3e-6, 1.1e-6)},
    "cluster_capacity": {2: 74, 3: 45, 4: 33, 5: 26, 6: 22, 7: 15, 8: 15},
    "l2_resident_fraction": 0.4,  # share of L2 an operand can hold across waves (two dies)
    "l2_fraction": 0.6,  # share of L2 that holds one wave's operand working set
}


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def _sm_rate(hw: GPUSpec) -> float:
    return CONSTANTS["tensor_rate_fraction"] * hw.peak_fp16_tflops * 1e12 / max(1, hw.num_sm)


def best_split(k_blocks: int, max_split: int, bn: int, conv: bool = False) -> int:
    """Mirror of fo_api.cu best_split: the part count minimising k-blocks-per-part x t_kb
    + (parts - 1) x partial read + chain."""
    K = CONSTANTS
    rate = 1.0 if bn >= 256 else 0.66 if bn >= 128 else 0.37
    t_kb = K["split_t_kb256_s"] * (bn / 256.0) / rate / (K["im2col_rate"] if conv else 1.0)
    part_s = bn * 512.0 / K["split_read_bytes_per_s"]
    best, best_t = 1, k_blocks * t_kb
    for s in range(2, max_split + 1):
        kbp = -(-k_blocks // s)
        parts = -(-k_blocks // kbp)
        t = kbp * t_kb + (parts - 1) * part_s + K["split_overhead_s"]
        if t < best_t:
            best, best_t = s, t
    return best


def split_plan(tiles: int, k_blocks: int, cap: int, bn: int = 256, conv: bool = False):
    """Mirror of the C ABI's split-K tail planner (fo_api.cu plan_split): returns
    (full_units, left_tiles, split).  Only a last wave less than half full (or a problem
    with fewer tiles than CTAs) is split, into the cost-minimising part count (<= 8, and
    <= the idle CTAs per tile)."""
    full = tiles // cap if tiles >= cap else 0
    left = tiles - full * cap
    if left == 0 or 2 * left > cap or k_blocks < 2:
        return full * cap, left, 1
    split = best_split(k_blocks, min(cap // left, 8, k_blocks), bn, conv)
    if split < 2:
        return full * cap, left, 1
    kbp = -(-k_blocks // split)
    split = -(-k_blocks // kbp)
    return full * cap, left, max(1, split)


def _smem_bytes(bn: int, stages: int, kps: int, csplit: int) -> int:
    """fo_kernel.cuh smem_bytes_for of a single-CTA tile with a cluster split's receive area."""
    recv = (csplit - 1) * -(-(4 * (bn // 32)) // csplit) * 32 * 144 if csplit > 1 else 0
    return 1024 + stages * kps * (128 + bn) * 64 * 2 + max(32768, recv) + 1536


def cluster_stages(bn: int, stages: int, kps: int, s: int) -> int:
    while stages > 2 and _smem_bytes(bn, stages, kps, s) > 232448:
        stages -= 1
    return stages if _smem_bytes(bn, stages, kps, s) <= 232448 else 0


def cluster_split_plan(tiles: int, k_blocks: int, kps: int, cap: int, bn: int, stages: int) -> int:
    """Mirror of fo_api.cu plan_cluster_split (automatic mode) and the launch's fallback
    over cluster sizes that do not all fit the GPU: the part count used, or 0."""
    K = CONSTANTS
    nst = -(-k_blocks // kps)
    if 2 * tiles > cap or nst < 2:
        return 0
    t_kb = K["cluster_t_kb64_s"]
    c0, c1 = K["cluster_cost_s"][bn]
    t1 = k_blocks * t_kb
    cands = []
    for s in range(2, 9):
        if tiles * s > cap or s > nst or cluster_stages(bn, stages, kps, s) == 0:
            continue
        t = -(-nst // s) * kps * t_kb + c0 + c1 * s
        if t < 0.8 * t1:
            cands.append((t, s))
    for _, s in sorted(cands):
        if tiles <= K["cluster_capacity"].get(s, 0):
            return s
    return 0


def _traffic_bytes(op: OpSpec, c: TuneConfig, hw: GPUSpec, ctas: int) -> float:
    """HBM bytes: operands re-read once per wave in which they are not L2-resident."""
    ml = op.mainloop
    tiles_m, tiles_n = _cdiv(op.M, c.block_M), _cdiv(op.N, c.block_N)
    a_row = c.block_M * op.K * ml.input_element_bytes   # one 128-row block of A
    b_col = c.block_N * op.K * ml.weight_element_bytes  # one BN-column block of B
    if ml.kind == "implicit_gemm_conv":
        a_total = ml.input_elements * ml.input_element_bytes  # input read once (halo in L2)
    else:
        a_total = tiles_m * a_row
    b_total = tiles_n * b_col
    out = ml.output_elements * ml.output_element_bytes
    l2 = hw.l2_cache_size * CONSTANTS["l2_fraction"]
    if a_total + b_total <= l2:
        return a_total + b_total + out
    # Operands larger than L2.  One operand that fits the resident share of L2 is read
    # once.  Otherwise a grouped raster keeps the group's A row blocks resident while B
    # streams past once per group (measured on 8192 x 16384 x 4096: group 16 > 8 > 32,
    # whose 64 MB of A rows no longer stay resident); without that, each wave re-reads
    # the blocks it touches.
    resident = hw.l2_cache_size * CONSTANTS["l2_resident_fraction"]
    if b_total <= resident or a_total <= resident:
        return a_total + b_total + out
    if c.group_size_m > 0 and ml.kind != "implicit_gemm_conv":
        rows_g = min(tiles_m, c.group_size_m)
        if rows_g * a_row <= resident:
            return a_total + _cdiv(tiles_m, rows_g) * b_total + out
    g = c.group_size_m if c.group_size_m > 0 else 1
    if c.group_size_m > 0:
        rows_per_wave = min(tiles_m, g)
        cols_per_wave = min(tiles_n, _cdiv(ctas, rows_per_wave))
    else:
        cols_per_wave = min(tiles_n, ctas)
        rows_per_wave = max(1, _cdiv(ctas, tiles_n))
    waves = _cdiv(tiles_m * tiles_n, ctas)
    per_wave = rows_per_wave * a_row + cols_per_wave * b_col
    return max(a_total + b_total, waves * per_wave) + out


def direct_plan(geo, block_n: int, sms: int, kps: int, stages: int):
    """The direct conv's geometry as fo_api.cu plan_direct computes it: (P, rows per tile,
    tiles per image, positions per tile, pixel slots, shared bytes), or None when the
    shape does not qualify or nothing fits in shared memory."""
    n, c, h, w, oc, kh, kw, stride, pad = geo
    if stride != 1 or c % 64 != 0:
        return None
    P = _cdiv(w + 2 * pad, 32) * 32
    oh = h + 2 * pad - kh + 1
    if P > block_n or kw - 1 >= P or oh <= 0:
        return None
    tiles_m = _cdiv(oc, 128)
    best, rpt = -1, 1
    for r in range(1, block_n // P + 1):
        cost = _cdiv(n * _cdiv(oh, r) * tiles_m, sms) * (max(r * P, 240) + 32)
        if best < 0 or cost <= best:
            best, rpt = cost, r
    bn = rpt * P
    nr = (bn - 1 + (kh - 1) * P + kw - 1) // P + 1
    slot = nr * P * 128
    for slots in (2, 1):
        smem = 1024 + slots * slot + stages * kps * 128 * 64 * 2 + 32768 + 1536
        if smem <= 232448:
            return P, rpt, _cdiv(oh, rpt), bn, slots, smem
    return None


def _residual_s(op: OpSpec, outputs: int, rate: float) -> float:
    """Time one tile spends reading its residual (a `residual_add` epilogue primitive)."""
    if not any(p.name == "residual_add" for p in op.epilogue):
        return 0.0
    return outputs * op.mainloop.output_element_bytes / rate


def _model_direct(op: OpSpec, c: TuneConfig, hw: GPUSpec) -> dict:
    """Direct conv (swap_ab 2): tiles of rpt padded rows x 128 channels, each input row
    loaded once per channel block and every filter tap a shifted view of it, so the
    mainloop runs near the tensor rate; the padding positions of each row (P - OW) and of
    the last tile of an image are computed and discarded."""
    K = CONSTANTS
    ml = op.mainloop
    geo = ml.conv_geometry
    kps = c.block_K // 64
    pl = direct_plan(geo, c.block_N, hw.num_sm, kps, c.num_stages) if geo else None
    if pl is None or c.block_M != 128:
        return {"score": 0.0, **{f: 0.0 for f in ("eff_mainloop", "eff_memory", "eff_parallel", "eff_pipeline",
                                                   "eff_implicit_conv", "eff_epilogue", "eff_reduction")},
                "projection": {"predicted_s": float("inf"), "predicted_tflops": 0.0}}
    P, rpt, tpi, bn, slots, _ = pl
    n, cin, h, w, oc, kh, kw, _, pad = geo
    tiles = n * tpi * _cdiv(oc, 128)
    ctas = min(tiles, hw.num_sm)
    waves = _cdiv(tiles, ctas)
    rate = _sm_rate(hw)
    e_kps = K["direct_rate_kps"][kps] * (1.0 if slots == 2 else K["direct_one_slot"])
    # one 128 x bn x 16 MMA: bn / 2 tensor cycles at the kps-dependent rate, but no fewer
    # than the issuing thread's cycles per MMA (narrow tiles are issue-bound)
    clk = rate / 8192.0  # the tensor clock implied by the achievable rate (8192 FLOP / cycle)
    n_mma = cin // 16 * kh * kw
    t_tile_mma = n_mma * max(bn / 2.0 / e_kps, K["mma_issue_cycles"]) / clk
    t_epi = 128 * bn * ml.output_element_bytes / K["epi_bytes_per_s_sm"]
    t_tile = max(t_tile_mma, t_epi) + _residual_s(op, min(128, oc) * bn, K["direct_residual_bytes_per_s_sm"])
    t_comp = waves * t_tile + t_epi + K["fixed_s"]
    traffic = (ml.input_elements * ml.input_element_bytes + ml.weight_elements * ml.weight_element_bytes
               + ml.output_elements * ml.output_element_bytes)
    t_mem = traffic / (hw.mem_bandwidth_gbps * 1e9 * K["hbm_efficiency"])
    t_pred = max(t_comp, t_mem) + K["mem_overlap"] * min(t_comp, t_mem)
    t_ideal = ml.mainloop_flops / (_sm_rate(hw) * hw.num_sm)
    score = min(1.0, t_ideal / t_pred)
    oh = h + 2 * pad - kh + 1
    e_main = min(1.0, (oh * (w + 2 * pad - kw + 1)) / float(tpi * rpt * P) * e_kps)
    e_mem = t_comp / t_pred
    e_epi = t_tile_mma / t_tile
    e_par = score / max(1e-12, e_main * e_mem * e_epi)
    return {
        "score": score, "eff_mainloop": e_main, "eff_memory": e_mem, "eff_parallel": e_par,
        "eff_pipeline": 1.0, "eff_implicit_conv": 1.0, "eff_epilogue": e_epi, "eff_reduction": 1.0,
        "projection": {
            "tiles_M": _cdiv(oc, 128), "tiles_N": n * tpi, "tiles_K": cin // 64 * kh * kw, "grid_size": ctas,
            "num_tiles": tiles, "waves": waves, "wave_fill": tiles / float(waves * ctas),
            "predicted_s": t_pred, "predicted_tflops": ml.mainloop_flops / t_pred / 1e12,
            "hbm_bytes": traffic, "t_tile_s": t_tile, "t_epilogue_s": t_epi, "pitch": P, "rows_per_tile": rpt,
            "positions_per_tile": bn, "pixel_slots": slots,
        },
    }


def _model(op: OpSpec, c: TuneConfig, hw: GPUSpec) -> dict:
    K = CONSTANTS
    if c.swap_ab == 2:
        return _model_direct(op, c, hw)
    ml = op.mainloop
    bm, bn, bk = c.block_M, c.block_N, c.block_K
    pair = bm == 256
    # swap_ab (conv): the tile grid runs over (output channels, pixels)
    rows, cols = (op.N, op.M) if c.swap_ab else (op.M, op.N)
    tiles_m, tiles_n = _cdiv(rows, bm), _cdiv(cols, bn)
    k_blocks = max(1, _cdiv(op.K, bk))
    tiles = tiles_m * tiles_n
    sms = hw.num_sm // 2 if pair else hw.num_sm  # persistent units: SMs or SM pairs
    cap = (c.max_ctas // 2 if pair else c.max_ctas) if c.max_ctas > 0 else sms
    ctas = max(1, min(tiles, cap))
    waves = _cdiv(tiles, ctas)
    rate = _sm_rate(hw) * (2 if pair else 1)

    # -- mainloop: padded MMA work of one tile at the BN-dependent tensor rate
    if pair:
        e_bn = (K["mma_rate_bn_pair_bk128"] if bk == 128 else K["mma_rate_bn_pair"]).get(bn, 0.6)
    else:
        e_bn = (K["mma_rate_bn_bk128"] if bk == 128 else K["mma_rate_bn"]).get(bn, 0.6)
    if bk == 128 and waves < 2:
        # a single wave is latency-bound, and two K slices per stage halve the stages in
        # flight: measured 15.4 vs 13.3-14.4 us on 1024^3 with 64-column tiles
        e_bn = K["mma_rate_bn"].get(bn, 0.6) * 0.86
    padding = (rows * cols * op.K) / float(tiles_m * bm * tiles_n * bn * k_blocks * bk)
    t_kb = 2.0 * bm * bn * bk / (rate * e_bn)
    # -- pipeline: stages - 1 loads in flight while one stage is consumed
    e_pipe = min(1.0, (c.num_stages - 1) * t_kb / K["tma_latency_s"])
    # -- conv: the cp.async producer gathers bm x bk 16-bit elements per k-block
    e_conv = 1.0
    if ml.kind == "implicit_gemm_conv":
        e_conv = K["im2col_rate"]
    t_kb_eff = t_kb / (e_pipe * e_conv)
    t_tile_mma = k_blocks * t_kb_eff
    # -- epilogue: overlapped with the next tile's mainloop through two accumulators
    t_epi = bm * bn * ml.output_element_bytes / K["epi_bytes_per_s_sm"]
    e_epi = t_tile_mma / max(t_tile_mma, t_epi)
    t_tile = max(t_tile_mma, t_epi) + _residual_s(op, min(bm, rows) * min(bn, cols), K["residual_bytes_per_s_sm"])
    # -- LayerNorm: one normalisation pass (read + write) per 128-row block
    t_ln = 0.0
    if op.has_reduction_epilogue:
        ln_bytes = 2.0 * op.M * op.N * ml.output_element_bytes
        held = (bn >= 128 and c.group_size_m == 0 and tiles_n - 1 < ctas and waves <= 4 and op.K >= 2048
                and op.M * op.N >= (1 << 22))
        if held:  # the C ABI holds the slices in TMEM (fo_api.cu, automatic ln_mode)
            t_ln = K["ln_held_factor"] * ln_bytes / K["ln_pass_bytes_per_s"]
        elif bn >= 128 and op.M * op.N >= (1 << 24):  # the C ABI runs these as one kernel
            t_ln = ln_bytes / K["ln_fused_bytes_per_s"] + K["ln_fused_tail_s"]
        else:
            t_ln = ln_bytes / K["ln_pass_bytes_per_s"]
    # split-K tail (GEMM, CTA pairs included, and single-CTA conv, with a workspace): the
    # last, less than half-full wave is split along K, so it costs 1/split of a wave plus
    # the partials' reduction
    t_work = waves * t_tile
    csplit = 0
    if not op.has_reduction_epilogue and not pair and ml.kind != "implicit_gemm_conv":
        # cluster split (no workspace needed): each part runs 1/s of the stages
        csplit = cluster_split_plan(tiles, k_blocks * bk // 64, bk // 64, cap, bn, c.num_stages)
        if csplit > 1:
            c0, c1 = K["cluster_cost_s"][bn]
            t_work = t_tile * (-(-k_blocks // csplit)) / k_blocks + c0 + c1 * csplit
    if csplit < 2 and not op.has_reduction_epilogue and not (pair and ml.kind == "implicit_gemm_conv"):
        # the planner sees the whole persistent grid (cap), not just the busy CTAs
        conv = ml.kind == "implicit_gemm_conv"
        dp_units, left, split = split_plan(tiles, k_blocks, cap, bn, conv)
        if split > 1:
            t_work = (dp_units // cap) * t_tile + -(-left * split // cap) * t_tile / split \
                + K["split_overhead_s"] + (split - 1) * bn * 512.0 / K["split_read_bytes_per_s"]
    e_red = t_work / (t_work + t_ln)
    # -- parallel: SM-time used by the persistent grid, plus fixed cost
    quant = tiles / float(waves * sms)
    t_comp = t_work + t_ln + K["fixed_s"] + (K["pair_fixed_s"] if pair else 0.0)
    e_par = quant * (t_work + t_ln) / t_comp
    # -- memory: HBM time of the operand traffic against the compute time
    traffic = _traffic_bytes(op, c, hw, ctas)
    t_mem = traffic / (hw.mem_bandwidth_gbps * 1e9 * K["hbm_efficiency"])
    t_tot = max(t_comp, t_mem) + K["mem_overlap"] * min(t_comp, t_mem)
    e_mem = t_comp / t_tot
    e_main = min(1.0, padding * e_bn)
    t_pred = t_tot
    # score = ideal time (all SMs at the achievable tensor rate) / predicted time; the
    # wave / launch / split share is the residual factor, so the seven multiply to it.
    t_ideal = ml.mainloop_flops / (_sm_rate(hw) * hw.num_sm)
    score = min(1.0, t_ideal / t_pred)
    others = e_main * e_mem * e_pipe * e_conv * e_epi * e_red
    e_par = score / others if others > 0 else 0.0
    factors = {
        "eff_mainloop": e_main, "eff_memory": e_mem, "eff_parallel": e_par,
        "eff_pipeline": e_pipe, "eff_implicit_conv": e_conv, "eff_epilogue": e_epi,
        "eff_reduction": e_red,
    }
    return {
        "score": score, **factors,
        "projection": {
            "tiles_M": tiles_m, "tiles_N": tiles_n, "tiles_K": k_blocks, "grid_size": ctas,
            "num_tiles": tiles, "waves": waves, "wave_fill": tiles / float(waves * ctas),
            "predicted_s": t_pred, "predicted_tflops": ml.mainloop_flops / t_pred / 1e12,
            "hbm_bytes": traffic, "t_tile_s": t_tile, "t_epilogue_s": t_epi,
            "shared_mem_bytes_per_tile": c.shared_mem_bytes, "tmem_columns": c.tmem_columns,
        },
    }


def score_tcgen05(op: OpSpec, config: TuneConfig, hw: GPUSpec) -> float:
    return _model(op, config, hw)["score"]


def score_tcgen05_detailed(op: OpSpec, config: TuneConfig, hw: GPUSpec) -> dict:
    return _model(op, config, hw)


def predicted_seconds(op: OpSpec, config: TuneConfig, hw: GPUSpec) -> float:
    return _model(op, config, hw)["projection"]["predicted_s"]


__all__ = ["CONSTANTS", "predicted_seconds", "score_tcgen05", "score_tcgen05_detailed"]
