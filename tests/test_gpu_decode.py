"""Decode kernel (lithe_decode_packed / _batch) against the oracle and the reference's goldens.

Bar: fp32 output bit-identical to the reference's fp32 decode; bf16 output bit-identical to
that value rounded to nearest even (ref tests/test_kernels.py:67-75,166-179)."""
import numpy as np
import pytest
import torch

from lithe_b200 import codebook as cb
from lithe_b200 import device_errors, quant
from lithe_b200.kernels import packed
from oracle import decode_ref
from tests.helpers import (SMALL, bits_of_bf16, golden_modules, load_golden, oracle_pools, random_adapter)

pytestmark = pytest.mark.gpu


def flux_342_modules():
    mods = []
    for i in range(19):
        for t in ("attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0", "attn.add_q_proj", "attn.add_k_proj",
                  "attn.add_v_proj", "attn.to_add_out"):
            mods.append((f"transformer_blocks.{i}.{t}", 3072, 3072))
        for ff in ("ff", "ff_context"):
            mods.append((f"transformer_blocks.{i}.{ff}.net.0.proj", 3072, 12288))
            mods.append((f"transformer_blocks.{i}.{ff}.net.2", 12288, 3072))
    for i in range(38):
        for t in ("to_q", "to_k", "to_v"):
            mods.append((f"single_transformer_blocks.{i}.attn.{t}", 3072, 3072))
    return mods


def oracle_blocks(ad):
    lay = decode_ref.layout(ad.modules)
    return decode_ref.decode_stream(decode_ref.stream(ad.indices, lay), lay, *oracle_pools())


@pytest.mark.parametrize("modules", [SMALL, SMALL + [("wide", 3072, 9216)]])
def test_decode_packed_bit_exact(modules):
    ad = random_adapter(modules, rank=16, seed=4)
    words, lay = packed.pack_adapter(ad)
    pa, pb = cb.twin_pools()
    w = words.view(torch.int64).cuda()
    ref = oracle_blocks(ad)
    f32 = packed.decode_packed(w, lay, pa.cuda(), pb.cuda(), dtype=torch.float32)
    assert np.array_equal(f32.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    bf = packed.decode_packed(w, lay, pa, pb)
    assert bf.dtype == torch.bfloat16 and bf.shape == (lay.total_blocks, 64)
    assert np.array_equal(bits_of_bf16(bf), decode_ref.f32_to_bf16_bits(ref))
    got = packed.split_decoded(f32, lay)
    for name, (a, b) in decode_ref.split(ref, decode_ref.layout(ad.modules)).items():
        assert torch.equal(got[name][0].cpu(), torch.from_numpy(a))
        assert torch.equal(got[name][1].cpu(), torch.from_numpy(b))


def test_decode_matches_reference_golden():
    z = load_golden("decode_small.npz")
    mods = golden_modules(z)
    lay = packed.PackedLayout.from_modules(mods)
    pa, pb = cb.twin_pools()
    w = torch.from_numpy(z["words"].view(np.int64)).cuda()
    assert np.array_equal(bits_of_bf16(packed.decode_packed(w, lay, pa, pb)), z["blocks_bf16"])
    got = packed.split_decoded(packed.decode_packed(w, lay, pa, pb, dtype=torch.float32), lay)
    for m in mods:
        assert np.array_equal(got[m["name"]][0].cpu().numpy().view(np.uint32), z[f"fac/{m['name']}/A"].view(np.uint32))
        assert np.array_equal(got[m["name"]][1].cpu().numpy().view(np.uint32), z[f"fac/{m['name']}/B"].view(np.uint32))


def test_decode_bank_batch_and_invalid_slot():
    ads = [random_adapter(SMALL, rank=16, seed=s) for s in range(5)]
    bank = packed.PackedBank.from_adapters(ads, "cuda", n_slots=6)
    assert bank.slot_stride % 2 == 0 and bank.slot_stride >= bank.layout.num_words
    device_errors()
    out = bank.decode([4, 0, 2], dtype=torch.float32).cpu().numpy()
    for row, s in enumerate([4, 0, 2]):
        assert np.array_equal(out[row].view(np.uint32), oracle_blocks(ads[s]).view(np.uint32))
    assert device_errors() == 0
    sentinel = torch.full((2, bank.layout.total_blocks, 64), 7.0, device="cuda")
    ids = torch.tensor([1, 9], dtype=torch.int32, device="cuda")
    from lithe_b200.kernels import _launch
    _launch.decode_packed_batch_(bank.words, ids, bank.layout.total_blocks, 3, bank.layout.sides_on("cuda"),
                                 bank.lut, sentinel)
    assert device_errors() & 1
    assert np.array_equal(sentinel[0].cpu().numpy().view(np.uint32), oracle_blocks(ads[1]).view(np.uint32))
    assert bool((sentinel[1] == 7.0).all())             # the invalid slot's rows stay untouched


@pytest.mark.parametrize("shape,side", [((8, 96), "A"), ((160, 8), "B"), ((16, 3072), "A"), ((5, 13), "B")])
def test_level_major_decode(shape, side):
    rng = np.random.default_rng(11)
    n = decode_ref.num_blocks(shape)
    idx = rng.integers(0, 512, (3, n))
    pa, pb = cb.twin_pools()
    opa, opb = oracle_pools()
    pool, opool = (pa, opa) if side == "A" else (pb, opb)
    got = quant.decode(torch.from_numpy(idx), shape, pool).cpu().numpy()
    want = decode_ref.decode_factor(idx, shape, opool)
    assert got.shape == tuple(shape) and np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_decode_full_flux_342_adapter():
    ad = random_adapter(flux_342_modules(), rank=16, seed=123)
    words, lay = packed.pack_adapter(ad)
    assert lay.total_blocks == 700_416 and lay.num_words == 300_179
    pa, pb = cb.twin_pools()
    out = packed.decode_packed(words.view(torch.int64).cuda(), lay, pa, pb, dtype=torch.float32)
    ref = oracle_blocks(ad)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_bf16_pools_decode_through_the_given_pools():
    """Pools cast to bf16 (as the reference's serving kernel does) decode exactly through them."""
    ad = random_adapter(SMALL, rank=16, seed=8)
    words, lay = packed.pack_adapter(ad)
    pa, pb = cb.twin_pools()
    pa16, pb16 = pa.bfloat16(), pb.bfloat16()
    got = packed.decode_packed(words.view(torch.int64).cuda(), lay, pa16, pb16, dtype=torch.float32).cpu().numpy()
    want = decode_ref.decode_stream(decode_ref.stream(ad.indices, decode_ref.layout(ad.modules)),
                                    decode_ref.layout(ad.modules), pa16.float().numpy(), pb16.float().numpy())
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
