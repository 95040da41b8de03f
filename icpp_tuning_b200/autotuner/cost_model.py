"""Trait-driven analytical cost model.

Restates kernel/autotuner/cost_model.py of the reference: an operator is an `OpSpec`
(a `MainloopSpec` plus epilogue `FusionPrimitive`s, :52-151); a candidate tile is a
`TuneConfig` (:154-178); `project_config` (:475-536) turns (op, config, GPU) into
execution features and `score_formula` (:765-775) multiplies seven efficiency factors
in (0, 1]:

    eff_mainloop * eff_memory * eff_parallel * eff_pipeline * eff_implicit_conv
    * eff_epilogue * eff_reduction

The formulas and constants are the reference's, kept identical because the reference's
published decisions (evaluation/*.csv) are the golden tests of this module.  What is
new: `TuneConfig.kind`.  A config of kind "tcgen05" describes the sm_100a kernels of
this package (persistent, warp-specialised, TMEM accumulators) and `score_formula`
routes it to `tcgen05_model.score_tcgen05`, whose factors model that design instead of
a register-tiled SIMT/mma.sync kernel.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Literal, Optional, Sequence, Tuple

from .gpu_spec import GPUSpec

ReductionAxis = Literal["none", "m", "n", "k", "spatial", "channel"]
MainloopKind = Literal["gemm", "implicit_gemm_conv"]


# --------------------------------------------------------------------------- operator
@dataclass(frozen=True)
class FusionPrimitive:
    """One epilogue primitive described by execution traits (reference :52-73)."""

    name: str
    flops_per_output: float
    bytes_per_output: float = 0.0
    reduction_axis: ReductionAxis = "none"
    extra_passes: int = 0
    sync_penalty: float = 0.0
    preferred_outputs_per_thread: float = 16.0
    preferred_tile_m: Optional[float] = None
    preferred_tile_n: Optional[float] = None
    smem_bytes_per_output: float = 0.0

    @property
    def has_reduction(self) -> bool:
        return self.reduction_axis != "none"

    @property
    def work_units(self) -> float:
        return max(1.0, self.flops_per_output + self.bytes_per_output)


@dataclass(frozen=True)
class MainloopSpec:
    """The tiled contraction an operator reduces to (reference :76-110)."""

    kind: MainloopKind
    M: int
    N: int
    K: int
    input_elements: int
    weight_elements: int
    output_elements: int
    input_element_bytes: int = 2
    weight_element_bytes: int = 2
    output_element_bytes: int = 2
    accum_element_bytes: int = 4
    flops_per_fma: int = 2
    input_reuse_hint: float = 1.0
    weight_reuse_hint: float = 1.0
    spatial_reuse_hint: float = 1.0
    preferred_group_m: int = 8
    # conv only: (N, C, H, W, OC, KH, KW, stride, padding), for models that need the image
    # geometry (the tcgen05 model's direct conv); the reference's factors do not read it
    conv_geometry: Optional[Tuple[int, ...]] = None

    @property
    def mainloop_flops(self) -> int:
        return self.flops_per_fma * self.M * self.N * self.K

    @property
    def min_global_bytes(self) -> int:
        return (self.input_elements * self.input_element_bytes
                + self.weight_elements * self.weight_element_bytes
                + self.output_elements * self.output_element_bytes)


@dataclass(frozen=True)
class OpSpec:
    """Operator = mainloop + epilogue primitives (reference :113-151)."""

    name: str
    mainloop: MainloopSpec
    epilogue: Tuple[FusionPrimitive, ...] = field(default_factory=tuple)

    @property
    def M(self) -> int:
        return self.mainloop.M

    @property
    def N(self) -> int:
        return self.mainloop.N

    @property
    def K(self) -> int:
        return self.mainloop.K

    @property
    def flops(self) -> float:
        return float(self.mainloop.mainloop_flops
                     + self.M * self.N * sum(p.flops_per_output for p in self.epilogue))

    @property
    def bytes_accessed(self) -> float:
        return float(self.mainloop.min_global_bytes
                     + self.M * self.N * sum(p.bytes_per_output for p in self.epilogue))

    @property
    def arithmetic_intensity(self) -> float:
        b = self.bytes_accessed
        return self.flops / b if b > 0 else 0.0

    @property
    def has_reduction_epilogue(self) -> bool:
        return any(p.has_reduction for p in self.epilogue)


# --------------------------------------------------------------------------- config
@dataclass(frozen=True)
class TuneConfig:
    """A candidate tile (reference :154-178).

    kind "simt" is the reference's register-tiled kernel; kind "tcgen05" is this
    package's sm_100a kernel, where block_M is the tcgen05 M (128), block_K one
    128-byte swizzle row (64), num_warps the fixed role split (10 gemm, 13 conv),
    group_size_m the tile raster (0 = row-major) and max_ctas the persistent grid cap
    (0 = one CTA per SM).
    """

    block_M: int
    block_N: int
    block_K: int
    num_stages: int
    num_warps: int
    group_size_m: int = 8
    kind: str = "simt"
    max_ctas: int = 0
    swap_ab: int = 0  # tcgen05 conv: tiles over (output channels, pixels) instead

    @property
    def threads(self) -> int:
        return self.num_warps * 32

    @property
    def shared_mem_bytes(self) -> int:
        if self.kind == "tcgen05":
            # A and B stage rings + 4 warps x 2 x 4 KB epilogue staging + barriers / stats
            # + 1 KB alignment slack; equals fo_config_smem_bytes() of the C ABI.
            b_cols = self.block_N // 2 if self.block_M == 256 else self.block_N
            return 1024 + self.num_stages * (128 + b_cols) * self.block_K * 2 + 32768 + 1536
        return (self.block_M * self.block_K * 2 + self.block_K * self.block_N * 2) * self.num_stages

    @property
    def tmem_columns(self) -> int:
        """TMEM columns the kernel allocates: two fp32 accumulators of block_N columns."""
        return 2 * self.block_N if self.kind == "tcgen05" else 0  # per CTA (pairs too)

    @property
    def regs_per_thread_estimate(self) -> int:
        if self.kind == "tcgen05":
            return 200  # accumulators live in TMEM; ptxas reports <= 195 for every variant
        return (self.block_M * self.block_N) // max(1, self.threads) * 2 + 40

    def is_valid_for_backend(self, backend: str) -> bool:
        """Static legality of the tile for a backend (the reference calls this method
        from search_space.py:194 but never defines it)."""
        if backend == "tcgen05":
            return (self.kind == "tcgen05" and self.block_M in (128, 256) and self.block_K == 64
                    and self.block_N in (64, 128, 256) and not (self.block_M == 256 and self.block_N < 128)
                    and 2 <= self.num_stages <= 8
                    and self.tmem_columns <= 512 and self.shared_mem_bytes <= 232448)
        if backend == "triton":
            pow2 = lambda v: v >= 16 and (v & (v - 1)) == 0  # noqa: E731
            return pow2(self.block_M) and pow2(self.block_N) and pow2(self.block_K)
        if backend == "tilelang":
            return self.block_M % 16 == 0 and self.block_N % 16 == 0 and self.block_K % 16 == 0
        raise ValueError(f"unknown backend {backend!r}")


@dataclass(frozen=True)
class ConfigProjection:
    """Execution features of (op, config, GPU) shared by all factors (reference :181-212)."""

    tiles_M: int
    tiles_N: int
    tiles_K: int
    grid_size: int
    tile_outputs: int
    outputs_per_thread: float
    mainloop_iterations: int
    mainloop_flops_per_tile: float
    epilogue_flops_per_tile: float
    total_flops_per_tile: float
    input_bytes_per_tile: float
    weight_bytes_per_tile: float
    output_bytes_per_tile: float
    epilogue_bytes_per_tile: float
    total_global_bytes_per_tile: float
    shared_mem_bytes_per_tile: float
    tile_arithmetic_intensity: float
    occupancy: float
    resident_blocks_per_sm: int
    wave_fill: float
    preferred_num_stages: int
    reduction_work: float
    reduction_passes: int
    epilogue_preferred_outputs: float


# --------------------------------------------------------------------------- primitives
BIAS_ADD = FusionPrimitive("bias_add", 1.0, preferred_outputs_per_thread=16.0)
RELU = FusionPrimitive("relu", 1.0, preferred_outputs_per_thread=16.0)
SILU = FusionPrimitive("silu", 4.0, preferred_outputs_per_thread=12.0)
GELU = FusionPrimitive("gelu", 8.0, preferred_outputs_per_thread=8.0)
ROW_LAYERNORM = FusionPrimitive("row_layernorm", 10.0, 4.0, reduction_axis="n", extra_passes=1,
                                sync_penalty=0.35, preferred_outputs_per_thread=8.0,
                                preferred_tile_n=128.0)
BATCHNORM = FusionPrimitive("batchnorm", 6.0, 2.0, reduction_axis="channel", extra_passes=1,
                            sync_penalty=0.25, preferred_outputs_per_thread=12.0,
                            preferred_tile_n=128.0)

PRIMITIVE_LIBRARY: Dict[str, FusionPrimitive] = {
    p.name: p for p in (BIAS_ADD, RELU, SILU, GELU, ROW_LAYERNORM, BATCHNORM)}


def resolve_primitives(primitives: Iterable) -> Tuple[FusionPrimitive, ...]:
    out: List[FusionPrimitive] = []
    for p in primitives:
        if isinstance(p, FusionPrimitive):
            out.append(p)
        elif p in PRIMITIVE_LIBRARY:
            out.append(PRIMITIVE_LIBRARY[p])
        else:
            raise KeyError(f"Unknown fusion primitive: {p}")
    return tuple(out)


# --------------------------------------------------------------------------- builders
def make_matmul_spec(M: int, N: int, K: int, primitives: Sequence = (), *,
                     input_element_bytes: int = 2, weight_element_bytes: int = 2,
                     output_element_bytes: int = 2, name: Optional[str] = None) -> OpSpec:
    """GEMM OpSpec (reference :293-320)."""
    ml = MainloopSpec(kind="gemm", M=M, N=N, K=K, input_elements=M * K, weight_elements=K * N,
                      output_elements=M * N, input_element_bytes=input_element_bytes,
                      weight_element_bytes=weight_element_bytes,
                      output_element_bytes=output_element_bytes)
    return OpSpec(name=name or "matmul", mainloop=ml, epilogue=resolve_primitives(primitives))


def make_conv2d_spec(N: int, C: int, H: int, W: int, OC: int, KH: int, KW: int, *, stride: int = 1,
                     padding: int = 0, primitives: Sequence = (), input_element_bytes: int = 2,
                     weight_element_bytes: int = 2, output_element_bytes: int = 2,
                     name: Optional[str] = None) -> OpSpec:
    """Implicit-GEMM conv OpSpec: M = N*OH*OW, N = OC, K = C*KH*KW (reference :323-364)."""
    OH = (H + 2 * padding - KH) // stride + 1
    OW = (W + 2 * padding - KW) // stride + 1
    overlap = max(1.0, (KH * KW) / max(1.0, float(stride * stride)))
    ml = MainloopSpec(kind="implicit_gemm_conv", M=N * OH * OW, N=OC, K=C * KH * KW,
                      input_elements=N * C * H * W, weight_elements=OC * C * KH * KW,
                      output_elements=N * OC * OH * OW, input_element_bytes=input_element_bytes,
                      weight_element_bytes=weight_element_bytes,
                      output_element_bytes=output_element_bytes,
                      input_reuse_hint=math.sqrt(overlap),
                      weight_reuse_hint=math.sqrt(max(1.0, overlap)),
                      spatial_reuse_hint=overlap,
                      conv_geometry=(N, C, H, W, OC, KH, KW, stride, padding))
    return OpSpec(name=name or "conv2d", mainloop=ml, epilogue=resolve_primitives(primitives))


# --------------------------------------------------------------------------- constants
_PREFERRED_OCCUPANCY = 0.5
_OCCUPANCY_SATURATION_EXPONENT = 0.15
_WAVE_FILL_EXPONENT = 0.35
_HIGH_WARP_COUNT_PENALTY = 0.9
_MEMORY_EFFICIENCY_EXPONENT = 0.75
_PIPELINE_FILL_EXPONENT = 0.5
_STAGE_MISMATCH_PENALTY = 0.5
_MAINLOOP_TARGET_OUTPUTS_PER_THREAD = 32.0
_MAINLOOP_MIN_OUTPUTS_PER_THREAD = 2.0
_MAINLOOP_OUTPUT_DISTANCE_PENALTY = 0.4
_EPILOGUE_DISTANCE_PENALTY = 0.5
_REDUCTION_DISTANCE_PENALTY = 0.3
_CONV_BLOCK_M_DISTANCE_PENALTY = 0.45
_CONV_BLOCK_N_DISTANCE_PENALTY = 0.6
_CONV_HIGH_WARP_PENALTY = 0.94
_CONV_PLAIN_SPATIAL_WORK_PENALTY = 0.18
_CONV_PLAIN_BLOCK_K_OVERSIZE_PENALTY = 0.45
_CONV_PLAIN_HIGH_WARP_PENALTY = 0.55


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def _resident_blocks_per_sm(cfg: TuneConfig, hw: GPUSpec) -> int:
    by_threads = hw.max_warps_per_sm // max(1, cfg.num_warps)
    smem = cfg.shared_mem_bytes
    by_smem = hw.shared_mem_per_sm // smem if smem > 0 else hw.max_blocks_per_sm
    regs = cfg.regs_per_thread_estimate * cfg.threads
    by_regs = hw.max_regs_per_sm // regs if regs > 0 else hw.max_blocks_per_sm
    return max(0, min(by_threads, by_smem, by_regs, hw.max_blocks_per_sm))


def _estimate_occupancy(cfg: TuneConfig, hw: GPUSpec) -> float:
    if hw.max_warps_per_sm <= 0:
        return 0.0
    return min(1.0, _resident_blocks_per_sm(cfg, hw) * cfg.num_warps / hw.max_warps_per_sm)


def _preferred_block_k(op: OpSpec) -> int:
    return 64 if op.K >= 64 else (32 if op.K >= 32 else 16)


def _warp_count_efficiency(cfg: TuneConfig) -> float:
    if cfg.num_warps <= 4:
        return 1.0
    return _HIGH_WARP_COUNT_PENALTY ** math.log2(cfg.num_warps / 4.0)


def _weighted_preferred_outputs(op: OpSpec) -> float:
    if not op.epilogue:
        return 16.0
    w = sum(p.work_units for p in op.epilogue)
    return sum(p.preferred_outputs_per_thread * p.work_units for p in op.epilogue) / w


def _operand_reuse(op: OpSpec, cfg: TuneConfig, tiles_M: int) -> Tuple[float, float]:
    g = max(1, min(cfg.group_size_m, max(1, tiles_M)))
    if op.mainloop.kind == "gemm":
        return 1.0, max(1.0, g ** 0.5)
    return (max(1.0, op.mainloop.input_reuse_hint),
            max(1.0, (g * op.mainloop.weight_reuse_hint) ** 0.5))


def _preferred_num_stages(op: OpSpec, cfg: TuneConfig, tile_ai: float, hw: GPUSpec) -> int:
    ridge = hw.ridge_point_fp16
    mem_eff = 1.0 if ridge <= 0 else min(1.0, tile_ai / ridge)
    k_iters = max(1, _cdiv(op.K, cfg.block_K))
    pref = 2 + (op.mainloop.kind == "implicit_gemm_conv") + (mem_eff < 0.9) + (mem_eff < 0.5) \
        + op.has_reduction_epilogue
    return min(max(2, pref), max(2, min(6, k_iters)))


def project_config(op: OpSpec, config: TuneConfig, hw: GPUSpec) -> ConfigProjection:
    """Per-tile execution features (reference :475-536)."""
    c = config
    tiles_M, tiles_N, tiles_K = _cdiv(op.M, c.block_M), _cdiv(op.N, c.block_N), _cdiv(op.K, c.block_K)
    grid = tiles_M * tiles_N
    tile_out = c.block_M * c.block_N
    in_reuse, w_reuse = _operand_reuse(op, c, tiles_M)
    ml_flops = op.mainloop.flops_per_fma * c.block_M * c.block_N * op.K
    epi_flops = tile_out * sum(p.flops_per_output for p in op.epilogue)
    in_bytes = op.K * c.block_M * op.mainloop.input_element_bytes / in_reuse
    w_bytes = op.K * c.block_N * op.mainloop.weight_element_bytes / w_reuse
    out_bytes = tile_out * op.mainloop.output_element_bytes
    epi_bytes = tile_out * sum(p.bytes_per_output for p in op.epilogue)
    total_bytes = in_bytes + w_bytes + out_bytes + epi_bytes
    smem = c.shared_mem_bytes + tile_out * sum(p.smem_bytes_per_output for p in op.epilogue)
    ai = 0.0 if total_bytes <= 0 else (ml_flops + epi_flops) / total_bytes
    resident = max(1, _resident_blocks_per_sm(c, hw))
    slots = max(1, hw.num_sm * resident)
    waves = max(1, _cdiv(grid, slots))
    return ConfigProjection(
        tiles_M=tiles_M, tiles_N=tiles_N, tiles_K=tiles_K, grid_size=grid, tile_outputs=tile_out,
        outputs_per_thread=tile_out / max(1, c.threads), mainloop_iterations=max(1, tiles_K),
        mainloop_flops_per_tile=ml_flops, epilogue_flops_per_tile=epi_flops,
        total_flops_per_tile=ml_flops + epi_flops, input_bytes_per_tile=in_bytes,
        weight_bytes_per_tile=w_bytes, output_bytes_per_tile=out_bytes,
        epilogue_bytes_per_tile=epi_bytes, total_global_bytes_per_tile=total_bytes,
        shared_mem_bytes_per_tile=smem, tile_arithmetic_intensity=ai,
        occupancy=_estimate_occupancy(c, hw), resident_blocks_per_sm=resident,
        wave_fill=grid / (waves * slots),
        preferred_num_stages=_preferred_num_stages(op, c, ai, hw),
        reduction_work=sum(p.work_units for p in op.epilogue if p.has_reduction),
        reduction_passes=sum(p.extra_passes for p in op.epilogue if p.has_reduction),
        epilogue_preferred_outputs=_weighted_preferred_outputs(op))


# --------------------------------------------------------------------------- factors
def eff_mainloop(op: OpSpec, config: TuneConfig, proj: ConfigProjection) -> float:
    """Tile padding x outputs-per-thread fit x block_K fit (reference :544-572)."""
    c = config
    padded = proj.tiles_M * c.block_M * proj.tiles_N * c.block_N * proj.tiles_K * c.block_K
    padding = 1.0 if padded == 0 else op.M * op.N * op.K / padded
    launch_fill = min(1.0, proj.wave_fill * max(1, proj.resident_blocks_per_sm))
    occ_fill = min(1.0, proj.occupancy / max(_PREFERRED_OCCUPANCY, 1e-6))
    signal = math.sqrt(max(1e-6, launch_fill * occ_fill))
    target = _MAINLOOP_MIN_OUTPUTS_PER_THREAD + (
        _MAINLOOP_TARGET_OUTPUTS_PER_THREAD - _MAINLOOP_MIN_OUTPUTS_PER_THREAD) * signal
    dist = abs(math.log2(max(1e-6, proj.outputs_per_thread / target)))
    thread_eff = 1.0 / (1.0 + _MAINLOOP_OUTPUT_DISTANCE_PENALTY * dist)
    k_eff = math.sqrt(min(1.0, c.block_K / _preferred_block_k(op)))
    return padding * thread_eff * k_eff


def eff_memory(op: OpSpec, config: TuneConfig, proj: ConfigProjection, hw: GPUSpec) -> float:
    """Tile roofline x shared-memory pressure (reference :575-585)."""
    ridge = hw.ridge_point_fp16
    if ridge <= 0:
        return 1.0
    roof = min(1.0, proj.tile_arithmetic_intensity / ridge)
    pressure = min(1.0, proj.shared_mem_bytes_per_tile / max(1.0, float(hw.shared_mem_per_sm)))
    return (roof ** _MEMORY_EFFICIENCY_EXPONENT) * (1.0 / (1.0 + 0.25 * pressure))


def eff_parallel(op: OpSpec, config: TuneConfig, proj: ConfigProjection, hw: GPUSpec) -> float:
    """Occupancy x wave quantisation x warp count (reference :588-595)."""
    if proj.grid_size == 0 or hw.num_sm == 0:
        return 1.0
    occ = min(1.0, proj.occupancy / _PREFERRED_OCCUPANCY) ** _OCCUPANCY_SATURATION_EXPONENT
    return occ * proj.wave_fill ** _WAVE_FILL_EXPONENT * _warp_count_efficiency(config)


def eff_pipeline(op: OpSpec, config: TuneConfig, proj: ConfigProjection, hw: GPUSpec) -> float:
    """Pipeline fill x stage-count match (reference :598-608)."""
    it, st = proj.mainloop_iterations, config.num_stages
    if st <= 0 or it <= 0:
        return 1.0
    fill = (it / (it + st - 1)) ** _PIPELINE_FILL_EXPONENT
    return fill * (1.0 / (1.0 + _STAGE_MISMATCH_PENALTY * abs(st - proj.preferred_num_stages)))


def eff_implicit_conv(op: OpSpec, config: TuneConfig, proj: ConfigProjection, hw: GPUSpec) -> float:
    """Address-generation / gather cost of implicit-GEMM conv (reference :611-700)."""
    if op.mainloop.kind != "implicit_gemm_conv":
        return 1.0
    overlap = max(1.0, op.mainloop.spatial_reuse_hint)
    if overlap <= 1.0:
        return 1.0
    c = config
    ov_sig = min(1.5, math.log2(overlap) / math.log2(9.0))
    slots = max(1, hw.num_sm * max(1, proj.resident_blocks_per_sm))
    launch_util = min(1.0, proj.grid_size / slots)
    underfill = 1.0 - launch_util

    spatial_eff = bk_eff = plain_warp_eff = 1.0
    in_ch = op.K / overlap
    if not op.epilogue and overlap >= 8.5 and (op.N >= 512 or in_ch <= 96.0):
        work = min(1.0, op.mainloop.mainloop_flops / 1.0e10)
        spatial_eff = 1.0 / (1.0 + _CONV_PLAIN_SPATIAL_WORK_PENALTY * ov_sig * work
                             * max(0.35, launch_util))
        if c.block_K > 32:
            bk_eff = 1.0 / (1.0 + _CONV_PLAIN_BLOCK_K_OVERSIZE_PENALTY * ov_sig * work
                            * math.log2(c.block_K / 32.0))
        if c.num_warps > 4:
            plain_warp_eff = _CONV_PLAIN_HIGH_WARP_PENALTY ** (work * math.log2(c.num_warps / 4.0))
    if underfill <= 0.0:
        return spatial_eff * bk_eff * plain_warp_eff

    pref_n = 64.0 if overlap >= 4.0 and underfill >= 0.2 else 128.0
    pref_m = 32.0 if overlap >= 4.0 and underfill >= 0.5 else 64.0
    m_eff = 1.0 / (1.0 + _CONV_BLOCK_M_DISTANCE_PENALTY * ov_sig * underfill
                   * abs(math.log2(c.block_M / pref_m)))
    n_eff = 1.0 / (1.0 + _CONV_BLOCK_N_DISTANCE_PENALTY * ov_sig * underfill
                   * abs(math.log2(c.block_N / pref_n)))
    warp_eff = (_CONV_HIGH_WARP_PENALTY ** math.log2(c.num_warps / 4.0)
                if overlap >= 4.0 and underfill >= 0.2 and c.num_warps > 4 else 1.0)
    stage_eff = 1.0
    if c.num_stages > 1:
        ridge = hw.ridge_point_fp16
        pressure = 1.0 - min(1.0, proj.tile_arithmetic_intensity / ridge) if ridge > 0 else 0.0
        stage_eff = 1.0 / (1.0 + 0.25 * (c.num_stages - 1) * ov_sig * pressure)
    return m_eff * n_eff * warp_eff * stage_eff * spatial_eff * bk_eff * plain_warp_eff


def _primitive_efficiency(p: FusionPrimitive, config: TuneConfig, proj: ConfigProjection) -> float:
    dist = abs(math.log2(max(1e-6, proj.outputs_per_thread / p.preferred_outputs_per_thread)))
    eff = 1.0 / (1.0 + _EPILOGUE_DISTANCE_PENALTY * dist)
    if p.preferred_tile_m:
        eff *= 1.0 / (1.0 + 0.2 * abs(math.log2(config.block_M / p.preferred_tile_m)))
    if p.preferred_tile_n:
        eff *= 1.0 / (1.0 + 0.2 * abs(math.log2(config.block_N / p.preferred_tile_n)))
    return eff


def eff_epilogue(op: OpSpec, config: TuneConfig, proj: ConfigProjection) -> float:
    """Work-weighted geometric mean of primitive fits (reference :717-733)."""
    if not op.epilogue:
        return 1.0
    total = sum(p.work_units for p in op.epilogue)
    logsum = sum(p.work_units / total * math.log(max(1e-9, _primitive_efficiency(p, config, proj)))
                 for p in op.epilogue)
    share = proj.epilogue_flops_per_tile / max(1.0, proj.total_flops_per_tile)
    strength = min(1.0, 0.25 + 4.0 * share)
    if any(p.has_reduction or p.bytes_per_output > 0.0 or p.sync_penalty > 0.0 for p in op.epilogue):
        strength = max(strength, 0.65)
    return math.exp(logsum * strength)


def eff_reduction(op: OpSpec, config: TuneConfig, proj: ConfigProjection) -> float:
    """Geometric mean of reduction-primitive penalties (reference :736-757)."""
    reds = [p for p in op.epilogue if p.has_reduction]
    if not reds:
        return 1.0
    prod = 1.0
    for p in reds:
        along_n = p.reduction_axis in ("n", "channel")
        extent = config.block_N if along_n else config.block_M
        pref = p.preferred_tile_n if along_n else p.preferred_tile_m
        if pref is None:
            pref = 128.0 if along_n else 64.0
        passes = 1.0 / (1.0 + 0.2 * p.extra_passes)
        sync = 1.0 / (1.0 + p.sync_penalty)
        axis = 1.0 / (1.0 + _REDUCTION_DISTANCE_PENALTY * abs(math.log2(extent / pref)))
        prod *= passes * sync * axis
    return prod ** (1.0 / len(reds))


# --------------------------------------------------------------------------- score
def _factors(op: OpSpec, config: TuneConfig, hw: GPUSpec):
    proj = project_config(op, config, hw)
    return proj, {
        "eff_mainloop": eff_mainloop(op, config, proj),
        "eff_memory": eff_memory(op, config, proj, hw),
        "eff_parallel": eff_parallel(op, config, proj, hw),
        "eff_pipeline": eff_pipeline(op, config, proj, hw),
        "eff_implicit_conv": eff_implicit_conv(op, config, proj, hw),
        "eff_epilogue": eff_epilogue(op, config, proj),
        "eff_reduction": eff_reduction(op, config, proj),
    }


_ORDER = ("eff_mainloop", "eff_memory", "eff_parallel", "eff_pipeline", "eff_implicit_conv",
          "eff_epilogue", "eff_reduction")


def score_formula(op: OpSpec, config: TuneConfig, hw: GPUSpec) -> float:
    """Product of the seven factors; tcgen05 configs use the sm_100a model."""
    if config.kind == "tcgen05":
        from .tcgen05_model import score_tcgen05
        return score_tcgen05(op, config, hw)
    _, f = _factors(op, config, hw)
    s = 1.0
    for k in _ORDER:
        s *= f[k]
    return s


def score_formula_detailed(op: OpSpec, config: TuneConfig, hw: GPUSpec) -> dict:
    """score_formula plus every factor and projected feature (reference :778-819)."""
    if config.kind == "tcgen05":
        from .tcgen05_model import score_tcgen05_detailed
        return score_tcgen05_detailed(op, config, hw)
    proj, f = _factors(op, config, hw)
    s = 1.0
    for k in _ORDER:
        s *= f[k]
    keys = ("tiles_M", "tiles_N", "tiles_K", "grid_size", "tile_outputs", "outputs_per_thread",
            "mainloop_iterations", "tile_arithmetic_intensity", "occupancy",
            "resident_blocks_per_sm", "wave_fill", "preferred_num_stages", "input_bytes_per_tile",
            "weight_bytes_per_tile", "output_bytes_per_tile", "epilogue_bytes_per_tile",
            "shared_mem_bytes_per_tile", "reduction_passes", "epilogue_preferred_outputs")
    return {"score": s, **f, "projection": {k: getattr(proj, k) for k in keys}}


def score_configs(op: OpSpec, configs: Sequence[TuneConfig], hw: GPUSpec) -> List[float]:
    return [score_formula(op, c, hw) for c in configs]


def select_best_config(op: OpSpec, configs: Sequence[TuneConfig], hw: GPUSpec
                       ) -> Tuple[int, TuneConfig, float]:
    scores = score_configs(op, configs, hw)
    i = max(range(len(scores)), key=scores.__getitem__)
    return i, configs[i], scores[i]


__all__ = [
    "BATCHNORM", "BIAS_ADD", "ConfigProjection", "FusionPrimitive", "GELU", "MainloopSpec", "OpSpec",
    "PRIMITIVE_LIBRARY", "RELU", "ROW_LAYERNORM", "SILU", "TuneConfig", "eff_epilogue",
    "eff_mainloop", "eff_memory", "eff_parallel", "eff_pipeline", "eff_implicit_conv",
    "eff_reduction", "make_conv2d_spec", "make_matmul_spec", "project_config",
    "resolve_primitives", "score_configs", "score_formula", "score_formula_detailed",
    "select_best_config",
]
