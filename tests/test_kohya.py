"""Kohya-304 -> diffusers split (lithe_b200.kohya) against the reference's own outputs
(tests/golden/kohya_split.npz, written by lithe.kohya), plus the in-place row-range views of
the packed bank.  CPU only: the views are pointer arithmetic, no kernel runs."""
import json

import numpy as np
import pytest
import torch

from lithe_b200 import kohya
from lithe_b200.fileio import LitheAdapter
from lithe_b200.flux_model import FluxConfig, FluxShapedTransformer
from lithe_b200.kernels import PackedBank, PackedLayout, PackedLoRALinear, wrap_packed
from oracle import decode_ref
from tests.helpers import load_golden, oracle_pools

G = load_golden("kohya_split.npz")


def golden_adapter(tag):
    mods = json.loads(str(G[f"{tag}/modules"]))
    idx = {m["name"]: {s: G[f"{tag}/idx/{m['name']}/{s}"] for s in ("A", "B")} for m in mods}
    rank = mods[0]["shape_a"][0]
    return LitheAdapter(modules=mods, indices=idx, rank=rank, alpha=float(rank), key_format="kohya")


@pytest.mark.parametrize("tag", ["r4", "r16"])
def test_paths_and_index_split_match_reference(tag):
    ad = golden_adapter(tag)
    assert kohya.diffusers_paths(ad) == json.loads(str(G[f"{tag}/paths"]))
    got = kohya.split_indices(ad)
    want_paths = sorted({k.split("/")[2] for k in G.files if k.startswith(f"{tag}/split/")})
    assert sorted(got) == want_paths
    for path, (ia, ib, sa, sb) in got.items():
        assert np.array_equal(ia, G[f"{tag}/split/{path}/A"]), path
        assert np.array_equal(ib, G[f"{tag}/split/{path}/B"]), path
        assert [*sa, *sb] == G[f"{tag}/split/{path}/shapes"].tolist(), path


def test_split_spec_matches_reference_on_kohya_304():
    want = json.loads(str(G["k304/spec"]))
    mods = kohya.kohya_flux_modules(rank=16)
    assert len(mods) == 304 and sorted(m["name"] for m in mods) == sorted(want)
    n_paths = 0
    for m in mods:
        spec = kohya.split_spec(m["name"], m["shape_a"], m["shape_b"])
        assert [list(s) for s in spec] == want[m["name"]], m["name"]
        n_paths += len(spec)
    assert n_paths == 494
    layout = PackedLayout.from_modules(mods)
    assert layout.num_indices == 3_589_632 and layout.num_words * 8 == 4_102_440


def test_index_split_equals_factor_split():
    ad = golden_adapter("r4")
    pa, pb = oracle_pools()
    factors = {m["name"]: (torch.from_numpy(decode_ref.decode_factor(ad.indices[m["name"]]["A"], m["shape_a"], pa)),
                           torch.from_numpy(decode_ref.decode_factor(ad.indices[m["name"]]["B"], m["shape_b"], pb)))
               for m in ad.modules}
    by_factor = kohya.split_factors(factors)
    for path, (ia, ib, sa, sb) in kohya.split_indices(ad).items():
        a = torch.from_numpy(decode_ref.decode_factor(ia, sa, pa))
        b = torch.from_numpy(decode_ref.decode_factor(ib, sb, pb))
        assert torch.equal(a, by_factor[path][0]) and torch.equal(b, by_factor[path][1]), path


def test_split_errors():
    with pytest.raises(KeyError):
        kohya.split_spec("lora_unet_final_layer_linear", [4, 64], [64, 4])
    with pytest.raises(KeyError):
        kohya.split_spec("lora_unet_double_blocks_0_img_attn_norm", [4, 64], [64, 4])
    rng = np.random.default_rng(0)
    bad = LitheAdapter(modules=[{"name": "lora_unet_double_blocks_0_img_attn_qkv", "shape_a": [4, 8],
                                 "shape_b": [24, 4]}],
                       indices={"lora_unet_double_blocks_0_img_attn_qkv": {
                           "A": rng.integers(0, 512, (3, 1)).astype(np.uint16),
                           "B": rng.integers(0, 512, (3, 2)).astype(np.uint16)}},
                       rank=4, alpha=4.0, key_format="kohya")
    with pytest.raises(ValueError, match="not block aligned"):
        kohya.split_indices(bad)


def test_diffusers_adapters_pass_through():
    rng = np.random.default_rng(1)
    mods = [{"name": "transformer.transformer_blocks.0.attn.to_q", "shape_a": [4, 64], "shape_b": [64, 4]}]
    idx = {mods[0]["name"]: {"A": rng.integers(0, 512, (3, 4)).astype(np.uint16),
                             "B": rng.integers(0, 512, (3, 4)).astype(np.uint16)}}
    ad = LitheAdapter(modules=mods, indices=idx, rank=4, alpha=4.0)
    assert kohya.diffusers_paths(ad) == ["transformer_blocks.0.attn.to_q"]
    (path, (ia, ib, _, _)), = kohya.split_indices(ad).items()
    assert path == "transformer_blocks.0.attn.to_q" and ia is idx[mods[0]["name"]]["A"]


def test_bank_row_views_point_inside_the_fused_module():
    ad = golden_adapter("r16")
    bank = PackedBank.from_adapters([ad], "cpu")
    lay = bank.layout
    targets = kohya.split_targets(lay.names, lay.shapes_a, lay.shapes_b, "kohya")
    assert len(targets) == len(kohya.diffusers_paths(ad))
    for path, (name, r0, r1) in targets.items():
        i = lay.index(name)
        va, vb = bank.views(name, (r0, r1))
        assert va.offset == 3 * lay.a_off[i]
        assert vb.offset == 3 * (lay.b_off[i] + r0 * 16 // 64)
        # the split bank's B stream for this path is exactly these blocks of the fused one
        want_b = G[f"r16/split/{path}/B"]
        full_b = ad.indices[name]["B"]
        assert np.array_equal(full_b[:, r0 * 16 // 64: r1 * 16 // 64], want_b)
    with pytest.raises(ValueError, match="not block aligned"):
        bank.views("lora_unet_double_blocks_0_img_attn_qkv", (1, 129))
    with pytest.raises(ValueError, match="outside"):
        bank.views("lora_unet_double_blocks_0_img_attn_qkv", (0, 10**6))


def test_wrap_packed_covers_every_split_target_of_a_flux_shaped_model():
    cfg = FluxConfig.tiny()
    model = FluxShapedTransformer(cfg)
    mods = kohya.kohya_flux_modules(rank=16, double_blocks=cfg.double_blocks, single_blocks=cfg.single_blocks,
                                    hidden=cfg.hidden, mlp_ratio=cfg.mlp_ratio)
    bank = PackedBank(PackedLayout.from_modules(mods), 2, "cpu")
    wrapped = wrap_packed(model, bank, key_format="kohya")
    assert len(wrapped) == 14 * cfg.double_blocks + 6 * cfg.single_blocks
    k = wrapped["single_transformer_blocks.0.proj_mlp"]
    assert isinstance(k, PackedLoRALinear) and k.rows == (3 * cfg.hidden, 3 * cfg.hidden + 4 * cfg.hidden)
    assert wrapped["transformer_blocks.1.attn.add_v_proj"].rows == (2 * cfg.hidden, 3 * cfg.hidden)
    assert wrapped["transformer_blocks.0.norm1.linear"].rows is None
    assert model.get_submodule("transformer_blocks.0.attn.to_k") is wrapped["transformer_blocks.0.attn.to_k"]
    with pytest.raises(KeyError):
        wrap_packed(FluxShapedTransformer(cfg), bank, key_format="kohya", paths=["transformer_blocks.9.attn.to_q"])
