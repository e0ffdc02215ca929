"""The C-ABI library loads and exports every entry point include/lithe_b200.h declares;
argument validation runs before any CUDA call, so it is checked here without a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from lithe_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "lithe_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"LITHE_API\s+[\w\s\*]+?\b(lithe_\w+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    syms = declared_symbols()
    assert syms, "no LITHE_API declarations found"
    assert set(syms) == set(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.lithe_abi_version() == _lib.ABI_VERSION


def _call_sgmv(**over):
    lib = _lib.lib()
    view = _lib.IndexView(0x1000, _lib.IDX_PACKED9, 3, 100, 0, 0)
    args = dict(x=0x10000, out=0x20000, accumulate=1, va=view, vb=view, n_slots=1, ids=0x30000, weights=None,
                batch=1, m=64, d_in=256, d_out=384, rank=16, scaling=1.0)
    args.update(over)
    lut = _lib.float_array([0.0] * 60)
    return lib.lithe_sgmv_index(args["x"], args["out"], args["accumulate"], ctypes.byref(args["va"]),
                                ctypes.byref(args["vb"]), args["n_slots"], args["ids"], args["weights"],
                                args["batch"], args["m"], args["d_in"], args["d_out"], args["rank"], lut,
                                args["scaling"], None, None)


@pytest.mark.parametrize("over,code", [
    ({"rank": 3}, _lib.ERR_UNSUPPORTED),
    ({"rank": 32}, _lib.ERR_UNSUPPORTED),
    ({"d_in": 100}, _lib.ERR_ARG),
    ({"d_out": 20}, _lib.ERR_ARG),
    ({"d_out": 8, "rank": 4}, _lib.ERR_ARG),          # d_out * rank not a multiple of 64
    ({"batch": -1}, _lib.ERR_ARG),
    ({"va": _lib.IndexView(0x1000, 7, 3, 0, 0, 0)}, _lib.ERR_ARG),
    ({"vb": _lib.IndexView(0x1000, _lib.IDX_PACKED9, 5, 0, 0, 0)}, _lib.ERR_UNSUPPORTED),
    ({"vb": _lib.IndexView(0x1001, _lib.IDX_PACKED9, 3, 0, 0, 0)}, _lib.ERR_ARG),
    ({"x": 0x10008}, _lib.ERR_ARG),                   # not 16-byte aligned
])
def test_sgmv_argument_errors(over, code):
    assert _call_sgmv(**over) == code
    msg = _lib.lib().lithe_last_error().decode()
    assert msg
    with pytest.raises(ValueError if code == _lib.ERR_ARG else NotImplementedError):
        _lib.check(code, "lithe_sgmv_index")


def test_sgmv_empty_batch_is_a_no_op():
    assert _call_sgmv(batch=0) == _lib.OK
    assert _call_sgmv(m=0) == _lib.OK


def test_decode_argument_errors():
    lib = _lib.lib()
    lut = _lib.float_array([0.0] * 60)
    assert lib.lithe_decode_packed(0x1000, 10, 0, None, lut, 0x2000, 0, None) == _lib.ERR_UNSUPPORTED
    assert lib.lithe_decode_packed(0x1000, 10, 3, None, lut, 0x2008, 0, None) == _lib.ERR_ARG
    assert lib.lithe_decode_packed(0x1000, 10, 3, None, lut, 0x2000, 5, None) == _lib.ERR_ARG
    assert lib.lithe_decode_packed(0x1000, 0, 3, None, lut, 0x2000, 0, None) == _lib.OK
    assert lib.lithe_decode_packed_batch(0x1000, 2, 4, 0x3000, 1, 100, 3, None, lut, 0x2000, 0, None, None) \
        == _lib.ERR_ARG                                    # slot_stride shorter than the stream


def test_custom_ops_registered_with_fake_kernels():
    """The kernels are torch.library ops with fake (meta) kernels: shapes and dtypes of their
    outputs are known without a GPU, which is what torch.compile traces with."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    import lithe_b200.kernels.ops  # noqa: F401  (registers the ops)

    for name in ("sgmv_index_", "lora_prep", "lora_gemm", "decode_packed"):
        assert hasattr(torch.ops.lithe_b200, name)
    view = [0, 3, 64, 0, 0]
    with FakeTensorMode():
        x = torch.empty(2, 256, 512, dtype=torch.bfloat16, device="cuda")
        words = torch.empty(10, 64, dtype=torch.int64, device="cuda")
        ids = torch.empty(2, dtype=torch.int32, device="cuda")
        h, b_dec = torch.ops.lithe_b200.lora_prep(x, words, words, view, view, 10, ids, None, 768, [0.0] * 60, 1.0,
                                                  True)
        assert tuple(h.shape) == (512, 16) and tuple(b_dec.shape) == (2, 768, 16) and h.dtype == torch.bfloat16
        h0, _ = torch.ops.lithe_b200.lora_prep(x, words, words, view, view, 10, ids, None, 768, [0.0] * 60, 1.0, False)
        assert tuple(h0.shape) == (0, 16)
        w = torch.empty(768, 512, dtype=torch.bfloat16, device="cuda")
        out = torch.ops.lithe_b200.lora_gemm(x.view(512, 512), w, None, h, b_dec, 256)
        assert tuple(out.shape) == (512, 768) and out.dtype == torch.bfloat16
        dec = torch.ops.lithe_b200.decode_packed(words.view(-1), 100, 3, None, [0.0] * 60, True)
        assert tuple(dec.shape) == (100, 64) and dec.dtype == torch.float32
        y = torch.empty(2, 256, 768, dtype=torch.bfloat16, device="cuda")
        assert torch.ops.lithe_b200.sgmv_index_(y, x, words, words, view, view, 10, ids, None, 16, [0.0] * 60, 1.0,
                                                True) is None
