""".lithe -> resident slot on the device (lithe_pack_raw, PackedBank.load_raw, SlotLoader):
every packed word bit-identical to the oracle's restatement of the reference's
load_lithe -> flat_indices -> pack_indices chain, at golden, small and full FLUX sizes."""
from pathlib import Path

import numpy as np
import pytest
import torch

from lithe_b200 import device_errors, kohya
from lithe_b200.fileio import LitheAdapter, load_lithe, read_payload, save_lithe
from lithe_b200.kernels import PackedBank, PackedLayout, SlotLoader, pack_adapter, packed_codebook_lora_delta_
from lithe_b200.module import FLUX_TARGET_MODULES
from oracle import decode_ref

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def slot_words(bank, slot):
    return bank.words[slot, : bank.layout.num_words].cpu().numpy().view(np.uint64)


def dev_raw(raw):
    arr = np.frombuffer(raw, dtype="<i2") if isinstance(raw, (bytes, bytearray)) else raw.view(np.int16)
    return torch.from_numpy(arr.copy()).cuda()


def test_golden_file_packs_like_the_reference_chain():
    header, raw = read_payload(GOLDEN / "small.lithe")
    mods = header["modules"]
    bank = PackedBank(PackedLayout.from_modules(mods), 3, "cuda")
    bank.load_raw(1, dev_raw(raw))
    torch.cuda.synchronize()
    want = decode_ref.pack_raw(raw, mods)
    assert np.array_equal(slot_words(bank, 1), want)
    assert np.array_equal(slot_words(bank, 1), pack_adapter(load_lithe(GOLDEN / "small.lithe"))[0].numpy().view(np.uint64))
    assert not bank.words[0].any() and not bank.words[2].any()      # other slots untouched
    assert device_errors() == 0


def flux342_modules(rank=16):
    from lithe_b200.flux_model import FluxShapedTransformer, lora_targets
    with torch.device("meta"):
        model = FluxShapedTransformer()
    return [{"name": n, "shape_a": [rank, m.in_features], "shape_b": [m.out_features, rank]}
            for n, m in lora_targets(model)]


@pytest.mark.parametrize("which", ["kohya304", "flux342"])
def test_full_size_payload(which):
    mods = kohya.kohya_flux_modules(rank=16) if which == "kohya304" else flux342_modules()
    if which == "flux342":
        assert len(mods) == 342 and all(any(m["name"].endswith(t) for t in FLUX_TARGET_MODULES) for m in mods)
    lay = PackedLayout.from_modules(mods)
    bank = PackedBank(lay, 2, "cuda")
    raw = np.random.default_rng(3).integers(0, 512, lay.num_indices).astype("<u2")
    bank.load_raw(1, dev_raw(raw))
    torch.cuda.synchronize()
    assert np.array_equal(slot_words(bank, 1), decode_ref.pack_raw(raw, mods))
    if bank.slot_stride > lay.num_words:
        assert int(bank.words[1, -1]) == 0                           # alignment padding untouched
    assert not bank.words[0].any()
    assert device_errors() == 0


def test_out_of_range_values_are_flagged_and_masked():
    mods = [{"name": "l", "shape_a": [16, 128], "shape_b": [64, 16]}]
    lay = PackedLayout.from_modules(mods)
    bank = PackedBank(lay, 1, "cuda")
    raw = np.random.default_rng(4).integers(0, 512, lay.num_indices).astype("<u2")
    raw[5] = 600
    bank.load_raw(0, dev_raw(raw))
    torch.cuda.synchronize()
    assert device_errors() & 2                                        # LITHE_DEVERR_INDEX
    masked = raw.copy()
    masked[5] &= 511
    assert np.array_equal(slot_words(bank, 0), decode_ref.pack_raw(masked, mods))


def random_adapter(mods, seed, rank=8):
    rng = np.random.default_rng(seed)
    idx = {m["name"]: {"A": rng.integers(0, 512, (3, m["shape_a"][0] * m["shape_a"][1] // 64)).astype(np.uint16),
                       "B": rng.integers(0, 512, (3, m["shape_b"][0] * m["shape_b"][1] // 64)).astype(np.uint16)}
           for m in mods}
    return LitheAdapter(modules=mods, indices=idx, rank=rank, alpha=float(rank))


def test_slot_loader_hot_swaps_files_and_serves_them(tmp_path):
    mods = [{"name": "transformer_blocks.0.attn.to_q", "shape_a": [8, 256], "shape_b": [192, 8]},
            {"name": "transformer_blocks.0.ff.net.2", "shape_a": [8, 512], "shape_b": [256, 8]}]
    ads = [random_adapter(mods, s) for s in range(5)]
    paths = []
    for i, ad in enumerate(ads):
        p = tmp_path / f"a{i}.lithe"
        save_lithe(p, ad)
        paths.append(p)
    bank = PackedBank(PackedLayout.from_adapter(ads[0]), 6, "cuda")
    loader = SlotLoader(bank, threads=3, depth=2)
    slots = [4, 0, 2, 5, 1]
    loader.load_many(slots, paths)
    ref = PackedBank.from_adapters(ads, "cuda")
    for s, ad in zip(slots, ads):
        assert np.array_equal(slot_words(bank, s), pack_adapter(ad)[0].numpy().view(np.uint64))
    assert loader.stats["files"] == 5
    # serve right after the swap: the new slots must be visible to work queued on the stream
    x = torch.randn(5, 40, 256, generator=torch.Generator().manual_seed(0)).bfloat16().cuda()
    got = torch.zeros(5, 40, 192, dtype=torch.bfloat16, device="cuda")
    want = torch.zeros_like(got)
    packed_codebook_lora_delta_(got, x, bank, mods[0]["name"], torch.tensor(slots, dtype=torch.int32), accumulate=False)
    packed_codebook_lora_delta_(want, x, ref, mods[0]["name"], torch.arange(5, dtype=torch.int32), accumulate=False)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # a second swap into an occupied slot replaces it
    loader.load(4, paths[3])
    torch.cuda.synchronize()
    assert np.array_equal(slot_words(bank, 4), pack_adapter(ads[3])[0].numpy().view(np.uint64))
    assert device_errors() == 0


def test_slot_loader_rejects_a_foreign_layout(tmp_path):
    mods = [{"name": "a", "shape_a": [8, 128], "shape_b": [64, 8]}]
    other = [{"name": "b", "shape_a": [8, 128], "shape_b": [64, 8]}]
    save_lithe(tmp_path / "o.lithe", random_adapter(other, 1))
    bank = PackedBank(PackedLayout.from_modules(mods), 2, "cuda")
    loader = SlotLoader(bank, threads=1)
    with pytest.raises(ValueError, match="modules do not match"):
        loader.load(0, tmp_path / "o.lithe")
    with pytest.raises(IndexError):
        loader.load(7, tmp_path / "o.lithe")
    assert not bank.words.any()


@pytest.mark.parametrize("levels", [1, 2, 4])
def test_pack_raw_other_level_counts(levels):
    from lithe_b200.kernels import _launch
    # module sides of 5, 12, 7 ... blocks: most 7-block groups straddle a segment boundary
    mods = [{"name": f"m{i}", "shape_a": [4, 64 * (i + 1) + 16], "shape_b": [16 * (i + 2), 4]} for i in range(9)]
    lay = PackedLayout.from_modules(mods, num_levels=levels)
    raw = np.random.default_rng(levels).integers(0, 512, lay.num_indices).astype("<u2")
    words = torch.full((lay.num_words,), -1, dtype=torch.int64, device="cuda")
    _launch.pack_raw_(dev_raw(raw), lay.segments_on("cuda"), levels, words)
    torch.cuda.synchronize()
    assert np.array_equal(words.cpu().numpy().view(np.uint64), decode_ref.pack_raw(raw, mods, levels=levels))
    assert device_errors() == 0


def test_batched_pack_matches_single_launches():
    mods = kohya.kohya_flux_modules(rank=16, double_blocks=2, single_blocks=2, hidden=256)
    lay = PackedLayout.from_modules(mods)
    n = 5
    raws = [np.random.default_rng(40 + i).integers(0, 512, lay.num_indices).astype("<u2") for i in range(n)]
    stride = (lay.num_indices + 7) // 8 * 8 + 8                       # padded rows: a strided batch
    raw2 = torch.zeros(n, stride, dtype=torch.int16)
    for i, r in enumerate(raws):
        raw2[i, : lay.num_indices] = torch.from_numpy(r.view(np.int16))
    raw2 = raw2.cuda()[:, : lay.num_indices]
    bank = PackedBank(lay, 9, "cuda")
    slots = [7, 0, 3, 8, 2]
    bank.load_raw_batch(slots, raw2)
    ref = PackedBank(lay, 9, "cuda")
    for s, r in zip(slots, raws):
        ref.load_raw(s, dev_raw(r))
    torch.cuda.synchronize()
    assert torch.equal(bank.words, ref.words)
    for s, r in zip(slots, raws):
        assert np.array_equal(slot_words(bank, s), decode_ref.pack_raw(r, mods))
    assert device_errors() == 0
    # an out-of-range slot is flagged and skipped
    bank.load_raw_batch([1, 99], raw2[:2])
    torch.cuda.synchronize()
    assert device_errors() & 1                                         # LITHE_DEVERR_SLOT
    assert np.array_equal(slot_words(bank, 1), decode_ref.pack_raw(raws[0], mods))
