"""Failure detection without a GPU fault: a bounded wait that nothing satisfies gives
up, reports through a device status word, and leaves the context usable."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_lost_arrival_is_reported_and_context_survives(cuda_device):
    from ictc_o3.backends.cuda import _native, radial
    from ictc_o3.backends.cuda._native import ptr, stream_of
    status = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    t0 = time.perf_counter()
    _native.call("ictc_wait_selftest", ptr(status), 20_000_000, 0, stream_of(status))   # 20 ms, no arrival
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == 1
    assert elapsed < 2.0
    _native.call("ictc_wait_selftest", ptr(status), 20_000_000, 1, stream_of(status))   # arrival: success
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # The context is still healthy: a tensor-core kernel runs and reports no error.
    layers = [torch.nn.Linear(8, 64, bias=False), torch.nn.Linear(64, 64, bias=False),
              torch.nn.Linear(64, 64, bias=False), torch.nn.Linear(64, 192, bias=False)]
    layers = [m.to(cuda_device) for m in layers]
    plan = radial.RadialPlan()
    out = radial.radial_gates(layers, torch.rand(300, 8, device=cuda_device), plan)
    torch.cuda.synchronize()
    radial.check_status(plan)
    assert torch.isfinite(out).all()
