"""lithe_sgmv_index_noalloc (built-in static workspace, allocates nothing) against the existing
entry point lithe_sgmv_index, both called through the C ABI on the same inputs.

Tolerance as the other SGMV tests: max-abs-rel <= 2e-2 and relative Frobenius error < 1e-2;
the two forms decode the same factors and accumulate in the same order, so the outputs are
also expected to be bit-identical.  Two calls run back to back with different routes, inputs
and accumulate modes, so the second call finds the first call's factors in the workspace.
This file sorts last so that the entry point also runs after every other test's launches."""
import ctypes

import numpy as np
import pytest
import torch

from lithe_b200 import _lib
from lithe_b200 import codebook as cb
from lithe_b200.kernels import PackedBank, _launch
from tests.helpers import max_abs_rel, random_adapter, rel_fro

MAX_ABS_REL = 2e-2
REL_FRO = 1e-2


def _call(entry, x, out, accumulate, va, vb, n_slots, ids, rank, lut, scaling, err):
    fn = getattr(_lib.lib(), entry)
    with torch.cuda.device(x.device):
        rc = fn(x.data_ptr(), out.data_ptr(), 1 if accumulate else 0, ctypes.byref(va), ctypes.byref(vb), n_slots,
                ids.data_ptr(), None, x.shape[0], x.shape[1], x.shape[2], out.shape[2], rank,
                _launch.lut_array(lut), float(scaling), err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, entry)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("d_in,d_out,r", [(3072, 12288, 16), (12288, 3072, 16), (512, 640, 8)])
def test_noalloc_matches_existing_entry_on_two_calls(d_in, d_out, r):
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=s) for s in range(4)]
    bank = PackedBank.from_adapters(ads, "cuda")
    va, vb = bank.views("l")
    lut = cb.kernel_lut(*cb.twin_pools())
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    g = torch.Generator().manual_seed(d_in + d_out + r)
    calls = [([3, 0, 2, 1, 0, 3], 200, False, 1.0), ([1, 2, 2, 0, 3, -1], 77, True, 0.5)]
    for assign, seq, accumulate, scaling in calls:
        x = (torch.randn(len(assign), seq, d_in, generator=g) * 0.5).bfloat16().cuda()
        base = (torch.randn(len(assign), seq, d_out, generator=g)).bfloat16().cuda()
        ids = torch.tensor(assign, dtype=torch.int32, device="cuda")
        assert _launch.workspace_bytes(len(assign), d_in, d_out) <= _lib.NOALLOC_WS_BYTES
        want = _call("lithe_sgmv_index", x, base.clone(), accumulate, va, vb, len(ads), ids, r, lut, scaling, err)
        got = _call("lithe_sgmv_index_noalloc", x, base.clone(), accumulate, va, vb, len(ads), ids, r, lut,
                    scaling, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        g_d, w_d = got.float().cpu(), want.float().cpu()
        if accumulate:
            g_d, w_d = g_d - base.float().cpu(), w_d - base.float().cpu()
        assert max_abs_rel(g_d, w_d) <= MAX_ABS_REL and rel_fro(g_d, w_d) < REL_FRO
        assert torch.equal(got, want)


@pytest.mark.gpu
def test_noalloc_at_full_capacity_and_small_m():
    """A call whose factors fill the built-in workspace to its limit (batch 34 at 3072 -> 12288:
    4,177,920 of 4,194,304 bytes, the last chunk near the array's end), then a call with m <= 8
    (the small-m form, which uses no workspace), then the full call again: each equal to
    lithe_sgmv_index bit for bit."""
    d_in, d_out, r = 3072, 12288, 16
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=10 + s) for s in range(5)]
    bank = PackedBank.from_adapters(ads, "cuda")
    va, vb = bank.views("l")
    lut = cb.kernel_lut(*cb.twin_pools())
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    g = torch.Generator().manual_seed(5)
    full = 34
    assert _launch.workspace_bytes(full, d_in, d_out) == 4177920
    assert _launch.workspace_bytes(full + 1, d_in, d_out) > _lib.NOALLOC_WS_BYTES
    for batch, seq in ((full, 72), (9, 5), (full, 16)):
        assign = [(7 * b + batch) % 5 for b in range(batch)]
        x = (torch.randn(batch, seq, d_in, generator=g) * 0.5).bfloat16().cuda()
        base = torch.randn(batch, seq, d_out, generator=g).bfloat16().cuda()
        ids = torch.tensor(assign, dtype=torch.int32, device="cuda")
        want = _call("lithe_sgmv_index", x, base.clone(), True, va, vb, len(ads), ids, r, lut, 1.0, err)
        got = _call("lithe_sgmv_index_noalloc", x, base.clone(), True, va, vb, len(ads), ids, r, lut, 1.0, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        g_d, w_d = got.float().cpu() - base.float().cpu(), want.float().cpu() - base.float().cpu()
        assert max_abs_rel(g_d, w_d) <= MAX_ABS_REL and rel_fro(g_d, w_d) < REL_FRO
        assert torch.equal(got, want)


def test_noalloc_rejects_calls_beyond_the_builtin_workspace():
    # Rejected on the host before any CUDA call, so no device memory is touched.
    lib = _lib.lib()
    view = _lib.IndexView(0x1000, _lib.IDX_PACKED9, 3, 100000, 0, 0)
    lut = _lib.float_array([0.0] * 60)
    d_in, d_out = 3072, 12288
    per_sample = _lib.lib().lithe_sgmv_workspace_bytes(1, d_in, d_out)
    batch = _lib.NOALLOC_WS_BYTES // per_sample + 1
    rc = lib.lithe_sgmv_index_noalloc(0x10000, 0x20000, 1, ctypes.byref(view), ctypes.byref(view), 1, 0x30000, None,
                                      batch, 64, d_in, d_out, 16, lut, 1.0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED
    msg = lib.lithe_last_error().decode()
    assert "lithe_sgmv_index_noalloc" in msg and str(_lib.NOALLOC_WS_BYTES) in msg
    assert lib.lithe_sgmv_index_noalloc(0x10000, 0x20000, 1, ctypes.byref(view), ctypes.byref(view), 1, 0x30000,
                                        None, 0, 64, d_in, d_out, 16, lut, 1.0, None, None) == _lib.OK
    assert np.int64(per_sample) == 240 * 512
