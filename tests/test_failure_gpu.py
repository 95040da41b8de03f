"""Failure detection on the GPU without a fault: a bounded device-side wait that nothing
satisfies runs out, records FO_ETIMEOUT, and the context stays usable."""
import pytest
import torch

from icpp_tuning_b200 import _native as N
from icpp_tuning_b200 import fused

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_context_survives():
    rc = N.lib().fo_selftest_wait_timeout(5_000_000, None)  # 5 ms
    assert rc == N.FO_ETIMEOUT, N.last_error()
    a = torch.randn(256, 128, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(64, 128, device="cuda", dtype=torch.bfloat16)
    out = fused.gemm(a, b, b_layout="nk", out_dtype=torch.float32)
    torch.cuda.synchronize()
    torch.testing.assert_close(out, a.float() @ b.float().t(), rtol=1e-4, atol=1e-4)
    rc, where = N.device_status(torch.cuda.current_device())
    assert rc == 0


def test_launch_counter_counts_native_launches():
    before = N.launch_count()
    a = torch.randn(128, 64, device="cuda", dtype=torch.bfloat16)
    fused.gemm(a, a, b_layout="nk")
    assert N.launch_count() == before + 1
