"""Hardware description consumed by the cost models.

Mirrors kernel/autotuner/gpu_spec.py of the reference (GPUSpec :15-69, table :72-162,
detect_gpu :175-251, get_gpu_spec :280-285) and adds what the sm_100a kernels need:
a B200 entry (the reference has none and falls back to a clock-rate heuristic,
gpu_spec.py:222-232) and the Blackwell-only resources -- tensor memory per SM, the
opt-in shared memory per block and the dense BF16 tensor peak.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional


@dataclass(frozen=True)
class GPUSpec:
    name: str
    compute_capability: tuple
    num_sm: int
    max_threads_per_sm: int
    max_warps_per_sm: int
    warp_size: int
    max_threads_per_block: int
    max_regs_per_block: int
    max_regs_per_sm: int
    shared_mem_per_block: int
    shared_mem_per_sm: int
    l2_cache_size: int
    global_mem_size: int
    mem_bandwidth_gbps: float
    peak_fp16_tflops: float
    peak_fp32_tflops: float
    # Blackwell additions (0 on older parts)
    tmem_cols_per_sm: int = 0
    sm_clock_mhz: float = 0.0

    @property
    def ridge_point_fp16(self) -> float:
        """FLOP per byte at which the fp16/bf16 tensor peak meets the HBM roofline."""
        if self.mem_bandwidth_gbps <= 0:
            return float("inf")
        return self.peak_fp16_tflops * 1e3 / self.mem_bandwidth_gbps

    @property
    def ridge_point_fp32(self) -> float:
        if self.mem_bandwidth_gbps <= 0:
            return float("inf")
        return self.peak_fp32_tflops * 1e3 / self.mem_bandwidth_gbps

    @property
    def max_blocks_per_sm(self) -> int:
        return 32 if self.compute_capability[0] >= 7 else 16

    @property
    def has_tcgen05(self) -> bool:
        return self.compute_capability[0] == 10


def _spec(name, cc, sms, threads_sm, smem_block, smem_sm, l2, mem, bw, fp16, fp32, **kw):
    return GPUSpec(name=name, compute_capability=cc, num_sm=sms, max_threads_per_sm=threads_sm,
                   max_warps_per_sm=threads_sm // 32, warp_size=32, max_threads_per_block=1024,
                   max_regs_per_block=65536, max_regs_per_sm=65536,
                   shared_mem_per_block=smem_block, shared_mem_per_sm=smem_sm,
                   l2_cache_size=l2, global_mem_size=mem, mem_bandwidth_gbps=bw,
                   peak_fp16_tflops=fp16, peak_fp32_tflops=fp32, **kw)


_MB, _GB = 1024 ** 2, 1024 ** 3

# Public datasheet figures.  The first five rows carry the same values as the reference's
# table so its published autotuner decisions reproduce (gpu_spec.py:72-162).
_KNOWN_GPUS = {
    "A100": _spec("NVIDIA A100", (8, 0), 108, 2048, 163840, 167936, 40 * _MB, 80 * _GB, 2039.0, 312.0, 19.5),
    "A800": _spec("NVIDIA A800", (8, 0), 108, 2048, 163840, 167936, 40 * _MB, 80 * _GB, 2039.0, 312.0, 19.5),
    "H100": _spec("NVIDIA H100", (9, 0), 132, 2048, 228 * 1024, 228 * 1024, 50 * _MB, 80 * _GB, 3352.0, 989.0, 67.0),
    "V100": _spec("NVIDIA V100", (7, 0), 80, 2048, 98304, 98304, 6 * _MB, 32 * _GB, 900.0, 125.0, 15.7),
    "4090": _spec("NVIDIA RTX 4090", (8, 9), 128, 1536, 100 * 1024, 100 * 1024, 72 * _MB, 24 * _GB, 1008.0, 330.0, 82.6),
    # B200 (HGX, 1000 W): 148 SMs on two dies, 227 KB opt-in shared memory per block
    # (228 KB per SM), 126 MB L2, 180 GB HBM3e at 8 TB/s, 2.25 PFLOP/s dense BF16,
    # 512 TMEM columns (x 128 lanes x 32 bit) per SM.
    "B200": _spec("NVIDIA B200", (10, 0), 148, 2048, 232448, 233472, 126 * _MB, 180 * _GB, 8000.0, 2250.0, 80.0,
                  tmem_cols_per_sm=512, sm_clock_mhz=1965.0),
}


def known_gpu(key: str) -> GPUSpec:
    return _KNOWN_GPUS[key]


def _match_known_gpu(device_name: str) -> Optional[GPUSpec]:
    up = device_name.upper()
    for key, spec in _KNOWN_GPUS.items():
        if key.upper() in up:
            return spec
    return None


def _cores_per_sm(cc: tuple) -> int:
    major = cc[0]
    if major >= 8:
        return 128
    if major >= 7:
        return 64
    if major >= 6:
        return 128 if cc[1] == 1 else 64
    return 128


def _bandwidth_from_props(props) -> float:
    if hasattr(props, "memory_clock_rate") and hasattr(props, "memory_bus_width"):
        return 2 * (props.memory_clock_rate / 1e6) * (props.memory_bus_width / 8)
    return 1000.0


def detect_gpu(device_id: int = 0) -> GPUSpec:
    """Spec of a CUDA device: queried properties, throughput figures from the table."""
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available")
    props = torch.cuda.get_device_properties(device_id)
    cc = (props.major, props.minor)
    known = _match_known_gpu(props.name)
    smem_block = getattr(props, "shared_memory_per_block_optin",
                         getattr(props, "max_shared_memory_per_block_optin", 49152))
    smem_sm = getattr(props, "shared_memory_per_multiprocessor", smem_block)
    regs = props.regs_per_multiprocessor
    l2 = getattr(props, "l2_cache_size", known.l2_cache_size if known else 40 * _MB)
    if known is not None:
        bw, fp16, fp32 = known.mem_bandwidth_gbps, known.peak_fp16_tflops, known.peak_fp32_tflops
        smem_sm = known.shared_mem_per_sm
        regs_sm = known.max_regs_per_sm
        if smem_block == 0:
            smem_block = known.shared_mem_per_block
        tmem, clk = known.tmem_cols_per_sm, known.sm_clock_mhz
    else:
        clock_ghz = getattr(props, "clock_rate", 0) / 1e6
        fp32 = 2 * _cores_per_sm(cc) * props.multi_processor_count * clock_ghz / 1e3
        fp16 = fp32 * (16 if cc[0] >= 8 else 8)
        bw = _bandwidth_from_props(props)
        regs_sm = regs
        smem_sm = smem_block
        tmem, clk = (512 if cc[0] == 10 else 0), clock_ghz * 1e3
    return GPUSpec(name=props.name, compute_capability=cc, num_sm=props.multi_processor_count,
                   max_threads_per_sm=props.max_threads_per_multi_processor,
                   max_warps_per_sm=props.max_threads_per_multi_processor // 32, warp_size=32,
                   max_threads_per_block=getattr(props, "max_threads_per_block", 1024),
                   max_regs_per_block=regs, max_regs_per_sm=regs_sm,
                   shared_mem_per_block=smem_block, shared_mem_per_sm=smem_sm,
                   l2_cache_size=l2, global_mem_size=props.total_memory,
                   mem_bandwidth_gbps=bw, peak_fp16_tflops=fp16, peak_fp32_tflops=fp32,
                   tmem_cols_per_sm=tmem, sm_clock_mhz=clk)


_cached: Optional[GPUSpec] = None


def get_gpu_spec(device_id: int = 0, force_refresh: bool = False) -> GPUSpec:
    """Process-wide cached spec of `device_id`; without a GPU the B200 table entry."""
    global _cached
    if _cached is None or force_refresh:
        import torch

        _cached = detect_gpu(device_id) if torch.cuda.is_available() else _KNOWN_GPUS["B200"]
    return _cached


__all__ = ["GPUSpec", "detect_gpu", "get_gpu_spec", "known_gpu"]
