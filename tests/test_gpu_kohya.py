"""Kohya-format banks served in place: every diffusers target of a fused module (q/k/v of
``attn_qkv``, q/k/v/proj_mlp of ``linear1``) reads its B rows straight from the resident
Kohya slot.  Checked bit for bit against a bank packed from ``kohya.split_indices`` (the
reference's index-level split), and against the fp32 truth of the split factors with the
SGMV tolerance (max-abs-rel <= 2e-2, relative Frobenius < 1e-2)."""
import json

import numpy as np
import pytest
import torch

from lithe_b200 import device_errors, kohya
from lithe_b200.fileio import LitheAdapter
from lithe_b200.flux_model import FluxConfig, FluxShapedTransformer
from lithe_b200.kernels import PackedBank, packed_codebook_lora_delta_, wrap_packed
from oracle import decode_ref
from tests.helpers import load_golden, max_abs_rel, oracle_pools, rel_fro

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
REL_FRO = 1e-2


def random_adapter(mods, seed):
    rng = np.random.default_rng(seed)
    idx = {}
    for m in mods:
        n_a = m["shape_a"][0] * m["shape_a"][1] // 64
        n_b = m["shape_b"][0] * m["shape_b"][1] // 64
        idx[m["name"]] = {"A": rng.integers(0, 512, (3, n_a)).astype(np.uint16),
                          "B": rng.integers(0, 512, (3, n_b)).astype(np.uint16)}
    rank = mods[0]["shape_a"][0]
    return LitheAdapter(modules=[dict(m) for m in mods], indices=idx, rank=rank, alpha=float(rank),
                        key_format="kohya")


def split_adapter(ad, keep=None):
    """The reference's index-level split as a diffusers-format adapter (one module per path)."""
    mods, idx = [], {}
    for path, (ia, ib, sa, sb) in kohya.split_indices(ad).items():
        if keep is not None and path not in keep:
            continue
        mods.append({"name": path, "shape_a": list(sa), "shape_b": list(sb)})
        idx[path] = {"A": np.ascontiguousarray(ia), "B": np.ascontiguousarray(ib)}
    return LitheAdapter(modules=mods, indices=idx, rank=ad.rank, alpha=ad.alpha)


def small_kohya_adapters():
    z = load_golden("kohya_split.npz")
    mods = json.loads(str(z["r16/modules"]))
    first = LitheAdapter(modules=mods, indices={m["name"]: {s: z[f"r16/idx/{m['name']}/{s}"] for s in ("A", "B")}
                                                for m in mods}, rank=16, alpha=16.0, key_format="kohya")
    return [first] + [random_adapter(mods, s) for s in (1, 2)]


def truth(x, ia, ib, sa, sb):
    pa, pb = oracle_pools()
    a = torch.from_numpy(decode_ref.decode_factor(ia, sa, pa))
    b = torch.from_numpy(decode_ref.decode_factor(ib, sb, pb))
    return x.float().cpu() @ a.T @ b.T


def test_every_split_target_matches_split_bank_and_truth():
    ads = small_kohya_adapters()
    bank_k = PackedBank.from_adapters(ads, "cuda")
    split = [split_adapter(a) for a in ads]
    bank_d = PackedBank.from_adapters(split, "cuda")
    lay = bank_k.layout
    targets = kohya.split_targets(lay.names, lay.shapes_a, lay.shapes_b, "kohya")
    assign = [2, 0, 1]
    ids = torch.tensor(assign, dtype=torch.int32, device="cuda")
    g = torch.Generator().manual_seed(0)
    for path, (name, r0, r1) in targets.items():
        rows = None if (r0, r1) == (0, lay.shapes_b[lay.index(name)][0]) else (r0, r1)
        d_in = lay.shapes_a[lay.index(name)][1]
        x = (torch.randn(3, 70, d_in, generator=g) * 0.5).bfloat16().cuda()
        got = torch.zeros(3, 70, r1 - r0, dtype=torch.bfloat16, device="cuda")
        ref = torch.zeros_like(got)
        packed_codebook_lora_delta_(got, x, bank_k, name, ids, rows=rows, accumulate=False)
        packed_codebook_lora_delta_(ref, x, bank_d, path, ids, accumulate=False)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), path
        sp = [kohya.split_indices(a)[path] for a in ads]
        want = torch.stack([truth(x[b], *sp[j]) for b, j in enumerate(assign)])
        assert max_abs_rel(got.float().cpu(), want) <= MAX_ABS_REL and rel_fro(got.float().cpu(), want) < REL_FRO, path
    assert device_errors() == 0


def test_kohya_304_full_size_targets_in_place():
    mods = kohya.kohya_flux_modules(rank=16)
    ads = [random_adapter(mods, s) for s in (10, 11)]
    bank_k = PackedBank.from_adapters(ads, "cuda")
    keep = {"single_transformer_blocks.5.proj_mlp": ("lora_unet_single_blocks_5_linear1", 9216, 21504),
            "single_transformer_blocks.37.attn.to_v": ("lora_unet_single_blocks_37_linear1", 6144, 9216),
            "transformer_blocks.3.attn.add_k_proj": ("lora_unet_double_blocks_3_txt_attn_qkv", 3072, 6144),
            "transformer_blocks.18.norm1_context.linear": ("lora_unet_double_blocks_18_txt_mod_lin", 0, 18432)}
    bank_d = PackedBank.from_adapters([split_adapter(a, keep) for a in ads], "cuda")
    ids = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    g = torch.Generator().manual_seed(1)
    for path, (name, r0, r1) in keep.items():
        m = 1 if path.endswith("norm1_context.linear") else 300
        x = torch.randn(2, m, 3072, generator=g).bfloat16().cuda()
        base = torch.randn(2, m, r1 - r0, generator=g).bfloat16().cuda()
        got, ref = base.clone(), base.clone()
        rows = None if r0 == 0 and r1 == 18432 else (r0, r1)
        packed_codebook_lora_delta_(got, x, bank_k, name, ids, rows=rows)
        packed_codebook_lora_delta_(ref, x, bank_d, path, ids)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), path
    assert device_errors() == 0


def test_flux_shaped_model_served_from_kohya_bank_equals_split_bank():
    cfg = FluxConfig.tiny()
    torch.manual_seed(0)
    model = FluxShapedTransformer(cfg).cuda().bfloat16().eval()
    mods = kohya.kohya_flux_modules(rank=16, double_blocks=cfg.double_blocks, single_blocks=cfg.single_blocks,
                                    hidden=cfg.hidden, mlp_ratio=cfg.mlp_ratio)
    ads = [random_adapter(mods, s) for s in (20, 21, 22)]
    bank_k = PackedBank.from_adapters(ads, "cuda")
    bank_d = PackedBank.from_adapters([split_adapter(a) for a in ads], "cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    lat = torch.randn(3, 64, cfg.in_channels, generator=g, device="cuda").bfloat16()
    txt = torch.randn(3, 16, cfg.text_dim, generator=g, device="cuda").bfloat16()
    pooled = torch.randn(3, cfg.pooled_dim, generator=g, device="cuda").bfloat16()
    t = torch.full((3,), 0.5, device="cuda")
    ids = torch.tensor([2, -1, 0], dtype=torch.int32, device="cuda")
    outs = []
    with torch.no_grad():
        base = model(lat, txt, pooled, t)
        for bank, fmt in ((bank_k, "kohya"), (bank_d, "diffusers")):
            m = FluxShapedTransformer(cfg).cuda().bfloat16().eval()
            m.load_state_dict(model.state_dict())
            wrapped = wrap_packed(m, bank, key_format=fmt)
            assert len(wrapped) == 14 * cfg.double_blocks + 6 * cfg.single_blocks
            for w in wrapped.values():
                w.assign = ids
            outs.append(m(lat, txt, pooled, t))
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(outs[0][1], base[1])          # the unrouted sample sees the base model only
    assert not torch.equal(outs[0][0], base[0])
    assert device_errors() == 0
