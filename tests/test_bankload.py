""".lithe -> resident slot, host side: the oracle's raw-payload pack pinned to the reference's
packed words, the segment table the device pack kernel reads (emulated here in numpy), the
payload reader, and lithe_pack_raw's argument checks (no kernel runs on CPU)."""
import json
from pathlib import Path

import numpy as np
import pytest

from lithe_b200 import _lib, kohya
from lithe_b200.fileio import read_payload
from lithe_b200.kernels import PackedLayout
from oracle import decode_ref
from tests.helpers import load_golden

GOLDEN = Path(__file__).resolve().parent / "golden"


def emulate_pack_raw(raw: np.ndarray, segments: np.ndarray, levels: int) -> np.ndarray:
    """What lithe_pack_raw computes, position by position, from the segment table."""
    raw = np.asarray(raw, dtype=np.int64)
    pos = np.arange(raw.size)
    g, lvl = pos // levels, pos % levels
    s = np.searchsorted(segments[:, 1], g, side="right") - 1
    assert (s >= 0).all() and (g < segments[s, 1] + segments[s, 2]).all()
    src = segments[s, 0] + lvl * segments[s, 2] + (g - segments[s, 1])
    return decode_ref.pack9(raw[src])


def test_oracle_pack_raw_reproduces_reference_words():
    z = load_golden("decode_small.npz")
    mods = json.loads(str(z["modules"]))
    idx = {m["name"]: {s: z[f"idx/{m['name']}/{s}"] for s in ("A", "B")} for m in mods}
    raw = decode_ref.raw_payload(idx, mods)
    assert np.array_equal(decode_ref.pack_raw(raw, mods), z["words"].view(np.uint64))
    back = decode_ref.split_raw(raw, mods)
    assert all(np.array_equal(back[n][s], idx[n][s]) for n in idx for s in ("A", "B"))


def test_read_payload_is_the_reference_stream():
    z = load_golden("small_lithe.npz")
    mods = json.loads(str(z["modules"]))
    header, raw = read_payload(GOLDEN / "small.lithe")
    assert header["modules"] == mods
    idx = {m["name"]: {s: z[f"idx/{m['name']}/{s}"] for s in ("A", "B")} for m in mods}
    assert raw == decode_ref.raw_payload(idx, mods).tobytes()


@pytest.mark.parametrize("which", ["golden", "kohya304", "kohya_small"])
def test_segment_table_matches_oracle(which):
    if which == "golden":
        mods = json.loads(str(load_golden("decode_small.npz")["modules"]))
    elif which == "kohya304":
        mods = kohya.kohya_flux_modules(rank=16)
    else:
        mods = kohya.kohya_flux_modules(rank=4, double_blocks=2, single_blocks=1, hidden=128)
    lay = PackedLayout.from_modules(mods)
    seg = lay.raw_segments()
    assert seg.shape == (2 * len(mods), 3) and (np.diff(seg[:, 1]) > 0).all()
    assert seg[:, 2].sum() == lay.total_blocks and seg[:, 2].sum() * 3 == lay.num_indices
    raw = np.random.default_rng(7).integers(0, 512, lay.num_indices).astype("<u2")
    want = decode_ref.pack_raw(raw, mods)
    assert want.size == lay.num_words
    assert np.array_equal(emulate_pack_raw(raw, seg, 3), want)


def test_pack_raw_argument_errors():
    lib = _lib.lib()
    assert lib.lithe_pack_raw(0x1000, 21, 0x2000, 2, 3, 0x3000, 4, None, None) == _lib.ERR_ARG     # n_words != 3
    assert b"n_words" in lib.lithe_last_error()
    assert lib.lithe_pack_raw(0x1000, 20, 0x2000, 2, 3, 0x3000, 3, None, None) == _lib.ERR_ARG     # 20 % 3 != 0
    assert lib.lithe_pack_raw(0x1000, 20, 0x2000, 2, 5, 0x3000, 3, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.lithe_pack_raw(0x1001, 21, 0x2000, 2, 3, 0x3000, 3, None, None) == _lib.ERR_ARG     # misaligned raw
    assert lib.lithe_pack_raw(0x1000, 21, None, 2, 3, 0x3000, 3, None, None) == _lib.ERR_ARG
    assert lib.lithe_pack_raw(0x1000, 21, 0x2000, 0, 3, 0x3000, 3, None, None) == _lib.ERR_ARG
    assert lib.lithe_pack_raw(None, 0, None, 0, 3, None, 0, None, None) == _lib.OK                # empty


def test_pack_raw_batch_argument_errors():
    lib = _lib.lib()
    seg = 0x2000
    # raw_stride shorter than a payload, and not a multiple of 8
    assert lib.lithe_pack_raw_batch(0x1000, 20, 2, 21, seg, 2, 3, 0x3000, 4, 2, None, 3, None, None) == _lib.ERR_ARG
    assert lib.lithe_pack_raw_batch(0x1000, 25, 2, 21, seg, 2, 3, 0x3000, 4, 2, None, 3, None, None) == _lib.ERR_ARG
    # slot stride shorter than a slot's words; more payloads than slots without slot_ids
    assert lib.lithe_pack_raw_batch(0x1000, 24, 2, 21, seg, 2, 3, 0x3000, 2, 2, None, 3, None, None) == _lib.ERR_ARG
    assert lib.lithe_pack_raw_batch(0x1000, 24, 3, 21, seg, 2, 3, 0x3000, 4, 2, None, 3, None, None) == _lib.ERR_ARG
    assert lib.lithe_pack_raw_batch(0x1000, 24, 70000, 21, seg, 2, 3, 0x3000, 4, 2, 0x4000, 3, None, None) \
        == _lib.ERR_UNSUPPORTED
    assert lib.lithe_pack_raw_batch(0x1000, 24, 0, 21, seg, 2, 3, 0x3000, 4, 2, None, 3, None, None) == _lib.OK
