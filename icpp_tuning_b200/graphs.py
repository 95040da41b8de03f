"""CUDA-graph capture of a step built from this package's operators.

Every fused operator is stream-ordered and allocation-free inside the library: tensor
maps travel as kernel parameters, the split-K counters reset themselves, and the device
status word is module memory.  A whole forward (dozens of launches) can therefore be
captured once and replayed with one `cudaGraphLaunch`, removing the per-call host cost
(Python descriptor packing plus tensor-map encoding, ~10-20 us a call) that dominates
small, latency-bound shapes.  Output tensors and any workspace a captured call
allocates come from the graph's private memory pool and stay valid across replays.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch


class CapturedStep:
    """Captures `fn(*inputs)` into a CUDA graph and replays it on new inputs.

    The inputs given at construction become the graph's static buffers; `__call__`
    copies new inputs (same shapes and dtypes) into them, replays the graph and returns
    the captured output tensor(s), which the next call overwrites.
    """

    def __init__(self, fn: Callable, inputs: Sequence[torch.Tensor], warmup: int = 2,
                 stream: torch.cuda.Stream | None = None):
        if not inputs or not all(isinstance(t, torch.Tensor) and t.is_cuda for t in inputs):
            raise ValueError("CapturedStep needs CUDA tensor inputs")
        self.fn = fn
        self.static_inputs = [t.clone() for t in inputs]
        self.stream = stream or torch.cuda.Stream(device=inputs[0].device)
        self.graph = torch.cuda.CUDAGraph()
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            # Warm-up on the capture stream: autotuner lookups, first-use kernel setup
            # and allocator growth happen here, outside the graph.
            for _ in range(warmup):
                fn(*self.static_inputs)
        torch.cuda.current_stream().wait_stream(self.stream)
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.static_output = fn(*self.static_inputs)

    def __call__(self, *inputs: torch.Tensor):
        if len(inputs) != len(self.static_inputs):
            raise ValueError(f"expected {len(self.static_inputs)} inputs, got {len(inputs)}")
        for dst, src in zip(self.static_inputs, inputs):
            if src.shape != dst.shape or src.dtype != dst.dtype:
                raise ValueError(f"input {tuple(src.shape)}/{src.dtype} does not match the captured "
                                 f"{tuple(dst.shape)}/{dst.dtype}")
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.static_output

    def replay(self):
        """Replays on whatever the static input buffers hold now."""
        self.graph.replay()
        return self.static_output
