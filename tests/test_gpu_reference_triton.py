"""The reference's own GPU kernels as a second checker, on the same device and inputs.

The unmodified reference package (its offline pip install in baseline/_ref; the tests skip
when it is absent) runs its Triton ``shared_codebook_lora_delta`` (lithe/kernels/shared.py:
197-263) and ``decode_packed`` (lithe/kernels/packed.py:205-222) beside ours:

- SGMV: both deltas within max-abs-rel 2e-2 and relative Frobenius error 1e-2 of the fp32
  truth (the tolerance of the other SGMV tests) and of each other, ragged token counts, int32
  index banks, pools in the activation dtype as the reference's IndexLoRALinear holds them;
- decode: our bf16 output equal bit for bit to the reference kernel's on the same packed words;
- the reference's kernel on int32 banks unpacked from our packed bank (the form the denoise
  bench's ``reference_triton`` variant serves) against our kernel on the packed bank itself.
"""
import pytest
import torch

import bench
from lithe_b200.kernels import PackedBank, PackedLayout, packed_codebook_lora_delta_, shared_codebook_lora_delta
from lithe_b200.kernels.packed import decode_packed
from tests.helpers import max_abs_rel, rel_fro

MAX_ABS_REL = 2e-2
REL_FRO = 1e-2


def _reference():
    try:
        return bench.reference_package()
    except ImportError as e:
        pytest.skip(f"reference package unavailable: {e}")


@pytest.mark.gpu
@pytest.mark.parametrize("d_in,d_out,seq", [(3072, 3072, 300), (12288, 3072, 129), (3072, 12288, 64)])
def test_sgmv_against_reference_triton(d_in, d_out, seq):
    ref = _reference()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(d_in + d_out + seq)
    n_slots, rank = 16, 16
    idx_a = torch.randint(0, 512, (n_slots, 3, rank * d_in // 64), generator=g, device=dev, dtype=torch.int32)
    idx_b = torch.randint(0, 512, (n_slots, 3, d_out * rank // 64), generator=g, device=dev, dtype=torch.int32)
    x = torch.randn(5, seq, d_in, generator=g, device=dev, dtype=torch.bfloat16)
    assign = torch.tensor([7, 0, 15, 7, 3], dtype=torch.int32, device=dev)
    pa32, pb32 = (p.to(dev) for p in ref.codebook.twin_pools())
    pa16, pb16 = pa32.to(torch.bfloat16), pb32.to(torch.bfloat16)
    d_ref = ref.kernels.shared.shared_codebook_lora_delta(x, idx_a, pa16, idx_b, pb16, assign, rank, d_out, 1.0,
                                                          out_dtype=torch.bfloat16)
    d_ours = shared_codebook_lora_delta(x, idx_a, pa16, idx_b, pb16, assign, rank, d_out, 1.0)
    truth = bench._fp32_delta(x, idx_a, idx_b, pa32, pb32, assign.cpu(), d_out)
    torch.cuda.synchronize()
    for got in (d_ours, d_ref):
        assert max_abs_rel(got.float(), truth) <= MAX_ABS_REL
        assert rel_fro(got.float(), truth) < REL_FRO
    assert max_abs_rel(d_ours.float(), d_ref.float()) <= MAX_ABS_REL
    assert rel_fro(d_ours.float(), d_ref.float()) < REL_FRO


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["flux342", "kohya304"])
def test_decode_bit_exact_against_reference_triton(kind):
    ref = _reference()
    dev = torch.device("cuda")
    lay = PackedLayout.from_modules(bench.decode_modules(kind))
    bank = PackedBank(lay, 2, dev)
    bank.fill_random(seed=77)
    ref_lay = ref.kernels.packed.PackedLayout(
        names=list(lay.names), shapes_a=list(lay.shapes_a), shapes_b=list(lay.shapes_b), a_off=list(lay.a_off),
        b_off=list(lay.b_off), sides=lay.sides.clone(), num_levels=lay.num_levels, block_size=lay.block_size,
        scaling=lay.scaling)
    pa32, pb32 = ref.codebook.twin_pools()
    for slot in range(2):
        words = bank.words[slot, : lay.num_words]
        want = ref.kernels.packed.decode_packed(words.view(torch.uint64), ref_lay, pa32.to(dev), pb32.to(dev))
        got = decode_packed(words, lay, pa32, pb32)
        assert torch.equal(got, want)


@pytest.mark.gpu
def test_reference_on_unpacked_banks_matches_packed_bank():
    ref = _reference()
    dev = torch.device("cuda")
    shapes = {"q": (3072, 3072), "ff": (3072, 12288), "down": (12288, 3072)}
    lay = PackedLayout.from_modules([{"name": n, "shape_a": [16, a], "shape_b": [b, 16]} for n, (a, b) in shapes.items()])
    bank = PackedBank(lay, 40, dev)
    bank.fill_random(seed=5)
    slots = [31, 2, 17]
    ids = torch.tensor(slots, dtype=torch.int32, device=dev)
    local = torch.arange(len(slots), dtype=torch.int32, device=dev)
    pa16, pb16 = (p.to(device=dev, dtype=torch.bfloat16) for p in ref.codebook.twin_pools())
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    for name, (d_in, d_out) in shapes.items():
        ia, ib = bench.int32_index_banks(bank, name, slots)
        assert ia.shape == (3, 3, 16 * d_in // 64) and ib.shape == (3, 3, d_out * 16 // 64)
        x = torch.randn(3, 200, d_in, generator=g, device=dev, dtype=torch.bfloat16)
        d_ref = ref.kernels.shared.shared_codebook_lora_delta(x, ia, pa16, ib, pb16, local, 16, d_out, 1.0,
                                                              out_dtype=torch.bfloat16)
        d_ours = torch.zeros(3, 200, d_out, device=dev, dtype=torch.bfloat16)
        packed_codebook_lora_delta_(d_ours, x, bank, name, ids, scaling=1.0)
        torch.cuda.synchronize()
        assert max_abs_rel(d_ours.float(), d_ref.float()) <= MAX_ABS_REL
        assert rel_fro(d_ours.float(), d_ref.float()) < REL_FRO
