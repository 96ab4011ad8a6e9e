"""Bounded device waits: a wait on a flag that nothing sets gives up after its
limit and reports a status the host reads; the context stays usable."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_on_unset_flag_times_out_and_context_survives():
    from kore_b200 import ops
    C = ops.native()
    flag = torch.zeros(1, dtype=torch.long, device="cuda")
    t0 = time.time()
    assert C.device_wait_flag(flag, 1, 0.5) == 2          # nothing sets it: timed out
    assert 0.4 < time.time() - t0 < 5.0
    flag.fill_(3)
    assert C.device_wait_flag(flag, 1, 0.5) == 0          # already set: seen at once
    x = torch.randn(256, 256, device="cuda", dtype=torch.bfloat16)
    y = ops.mm(x, x)                                       # the context still works
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
