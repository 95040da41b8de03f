"""Shared helpers of the GPU parity tests: seeded inputs drawn on CPU (one generator per
case, tensors drawn in a fixed order) and copied to the device, so the oracle sees the
identical values."""
import torch

from icpp_tuning_b200 import _native as N

# The reference's own tolerance (gemm_bias_act.py:160, conv2d.py:310): |a-b| <= atol + rtol*|b|
TOL = dict(atol=1e-2, rtol=1e-2)
TOL_LN = dict(atol=2e-2, rtol=2e-2)  # after LayerNorm


def gen(seed):
    return torch.Generator().manual_seed(seed)


def randn(g, *shape, dtype=torch.bfloat16, scale=1.0, shift=0.0):
    return (torch.randn(*shape, generator=g) * scale + shift).to(dtype)


def uniform(g, *shape, dtype=torch.float16, lo=-1.0, hi=1.0):
    return (torch.rand(*shape, generator=g) * (hi - lo) + lo).to(dtype)


def cuda(*ts):
    return [t.cuda() if t is not None else None for t in ts]


def assert_close(out, ref, tol=TOL):
    torch.testing.assert_close(out.float().cpu(), ref.float().cpu(), **tol)


def status_clean():
    rc, where = N.device_status(torch.cuda.current_device())
    assert rc == 0, f"device status {rc} at {where:#x}"
