"""Index-resident LoRA in a (tiny) FLUX-shaped transformer: the 342-target wiring by module
path, packed-bank routing per sample, and agreement with the dense decoded-factor comparator
(the counterpart of the reference's multi-adapter FLUX test, which needs diffusers)."""
import pytest
import torch

from lithe_b200.flux_model import FluxConfig, FluxShapedTransformer, denoise, lora_targets
from lithe_b200.kernels import PackedBank, PackedLayout, PackedLoRALinear, PerSampleLoRALinear, split_decoded, wrap_linears
from tests.helpers import rel_fro

pytestmark = pytest.mark.gpu


def _wire(model, mode, bank, slots):
    targets = [n for n, _ in lora_targets(model)]
    if mode == "lithe":
        wrapped = wrap_linears(model, targets, lambda n, lin: PackedLoRALinear(lin, bank, n, 16, 1.0))
        for m in wrapped.values():
            m.assign = torch.tensor(slots, dtype=torch.int32, device="cuda")
    else:
        dec = bank.decode(slots, dtype=torch.bfloat16)
        per = [split_decoded(dec[i], bank.layout) for i in range(len(slots))]
        wrapped = wrap_linears(model, targets, lambda n, lin: PerSampleLoRALinear(lin, "sgmv"))
        for n, m in wrapped.items():
            m.set_factors([(p[n][0], p[n][1], 1.0) for p in per])
    return wrapped


def test_tiny_flux_lithe_matches_dense_comparator():
    torch.manual_seed(0)
    cfg = FluxConfig.tiny()
    ref = FluxShapedTransformer(cfg).cuda().bfloat16()
    base_state = {k: v.clone() for k, v in ref.state_dict().items()}
    targets = lora_targets(ref)
    assert len(targets) == cfg.double_blocks * 12 + cfg.single_blocks * 3
    layout = PackedLayout.from_modules([{"name": n, "shape_a": [16, m.in_features], "shape_b": [m.out_features, 16]}
                                        for n, m in targets])
    bank = PackedBank(layout, 8, "cuda")
    bank.fill_random(seed=3)
    slots = [5, 1, 6]
    lat = torch.randn(3, 64, cfg.in_channels, device="cuda").bfloat16()
    txt = torch.randn(3, 16, cfg.text_dim, device="cuda").bfloat16()
    pooled = torch.randn(3, cfg.pooled_dim, device="cuda").bfloat16()
    outs = {}
    for mode in ("base", "lithe", "dense"):
        model = FluxShapedTransformer(cfg).cuda().bfloat16()
        model.load_state_dict(base_state)
        if mode != "base":
            _wire(model, mode, bank, slots)
        with torch.no_grad():
            outs[mode] = model(lat, txt, pooled, torch.full((3,), 0.5, device="cuda")).float()
            if mode == "lithe":
                outs["lithe_loop"] = denoise(model, lat, txt, pooled, 2).float()
            if mode == "dense":
                outs["dense_loop"] = denoise(model, lat, txt, pooled, 2).float()
    assert torch.isfinite(outs["lithe"]).all()
    # the adapters change the output, and both LoRA paths agree to bf16 precision
    assert rel_fro(outs["lithe"], outs["base"]) > 1e-3
    assert rel_fro(outs["lithe"], outs["dense"]) < 2e-2
    assert rel_fro(outs["lithe_loop"], outs["dense_loop"]) < 3e-2


def test_tiny_flux_fused_gemm_path_matches_default_path():
    """With 256-token streams every LoRA linear of the tiny model is eligible for the expand-in-
    GEMM path (n % 256, k % 64, tokens % 128): the whole model's output must agree with the
    cuBLAS + SGMV path to bf16 precision, and with the dense comparator."""
    torch.manual_seed(1)
    cfg = FluxConfig.tiny()
    base_model = FluxShapedTransformer(cfg).cuda().bfloat16()
    base_state = {k: v.clone() for k, v in base_model.state_dict().items()}
    targets = lora_targets(base_model)
    layout = PackedLayout.from_modules([{"name": n, "shape_a": [16, m.in_features], "shape_b": [m.out_features, 16]}
                                        for n, m in targets])
    bank = PackedBank(layout, 8, "cuda")
    bank.fill_random(seed=4)
    slots = [2, 7]
    lat = torch.randn(2, 256, cfg.in_channels, device="cuda").bfloat16()
    txt = torch.randn(2, 256, cfg.text_dim, device="cuda").bfloat16()
    pooled = torch.randn(2, cfg.pooled_dim, device="cuda").bfloat16()
    t = torch.full((2,), 0.5, device="cuda")
    outs = {}
    for mode in ("lithe", "fused", "dense"):
        model = FluxShapedTransformer(cfg).cuda().bfloat16()
        model.load_state_dict(base_state)
        wrapped = _wire(model, "dense" if mode == "dense" else "lithe", bank, slots)
        if mode == "fused":
            for m in wrapped.values():
                assert m._gemm_ok(torch.empty(2, 256, m.base.in_features, dtype=torch.bfloat16, device="cuda"))
                m.fused_gemm = True
        with torch.no_grad():
            outs[mode] = model(lat, txt, pooled, t).float()
    assert torch.isfinite(outs["fused"]).all()
    assert rel_fro(outs["fused"], outs["lithe"]) < 2e-2
    assert rel_fro(outs["fused"], outs["dense"]) < 2e-2
