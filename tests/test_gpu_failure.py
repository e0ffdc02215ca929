"""Failure detection on the GPU without a fault: a pipeline wait that runs out ends by itself
after its limit (4 s), reports LITHE_DEVERR_TIMEOUT through the device error word and leaves
the context usable -- the path every LITHE kernel takes when a pipeline stalls."""
import time

import pytest
import torch

from lithe_b200 import _lib, device_errors
from lithe_b200.kernels import PackedBank, _launch
from tests.helpers import random_adapter

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_survives():
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ok = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.monotonic()
    rc = _lib.lib().lithe_selftest_wait_timeout(err.data_ptr(), ok.data_ptr(),
                                                torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "lithe_selftest_wait_timeout")
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert int(err.item()) & _lib.DEVERR_TIMEOUT
    assert int(ok.item()) == 0
    assert 3.5 < elapsed < 30.0, elapsed
    # the context still works: a normal fused call afterwards is correct and error-free
    ads = [random_adapter([("l", 256, 384)], rank=16, seed=s) for s in range(2)]
    bank = PackedBank.from_adapters(ads, "cuda")
    va, vb = bank.views("l")
    x = torch.randn(2, 64, 256, generator=torch.Generator().manual_seed(0)).bfloat16().cuda()
    out1 = torch.zeros(2, 64, 384, dtype=torch.bfloat16, device="cuda")
    out2 = torch.zeros_like(out1)
    ids = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    for out in (out1, out2):
        _launch.sgmv_index_(x, out, accumulate=False, view_a=va, view_b=vb, n_slots=2, ids=ids, weights=None,
                            rank=16, lut=bank.lut, scaling=1.0)
    torch.cuda.synchronize()
    assert torch.equal(out1, out2) and out1.abs().sum() > 0
    assert device_errors() == 0
