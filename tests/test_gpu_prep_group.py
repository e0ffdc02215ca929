"""Shared-input prep groups (SharedInputPrep) on the fused-GEMM path.

The q / k / v linears of an attention block read one input; grouped, the first of them to run
computes all three h and b_dec with one lithe_lora_prep_multi.  The model's output must be
bit-identical to the same model with every linear preparing its own (lithe_lora_prep), every
group must hand all its results over (none left pending after the forward), and a member called
on another input computes its own."""
import pytest
import torch

from lithe_b200.flux_model import FluxConfig, FluxShapedTransformer, lora_targets
from lithe_b200.kernels import PackedBank, PackedLayout, wrap_packed

pytestmark = pytest.mark.gpu


def _model(seed):
    torch.manual_seed(seed)
    cfg = FluxConfig.tiny()
    model = FluxShapedTransformer(cfg).cuda().bfloat16().eval()
    targets = lora_targets(model)
    lay = PackedLayout.from_modules([{"name": n, "shape_a": [16, m.in_features], "shape_b": [m.out_features, 16]}
                                     for n, m in targets])
    bank = PackedBank(lay, 8, "cuda")
    bank.fill_random(seed=seed + 1)
    wrapped = wrap_packed(model, bank, scaling=20.0, fused_gemm=True)
    ids = torch.tensor([2, 7], dtype=torch.int32, device="cuda")
    for m in wrapped.values():
        m.assign = ids
    lat = torch.randn(2, 256, cfg.in_channels, device="cuda").bfloat16()
    txt = torch.randn(2, 256, cfg.text_dim, device="cuda").bfloat16()
    pooled = torch.randn(2, cfg.pooled_dim, device="cuda").bfloat16()
    return model, wrapped, (lat, txt, pooled, torch.full((2,), 0.5, device="cuda"))


def test_grouped_forward_equals_per_linear_prep():
    model, wrapped, args = _model(5)
    groups = {id(m.prep_group): m.prep_group for m in wrapped.values() if m.prep_group is not None}
    assert len(groups) == 6
    with torch.no_grad():
        grouped = model(*args)
        assert all(g._key is None and not g._ready for g in groups.values())      # every result handed over
        for m in wrapped.values():
            m.prep_group = None
        alone = model(*args)
    assert torch.equal(grouped, alone)


def test_member_on_another_input_computes_its_own():
    model, wrapped, args = _model(6)
    q = wrapped["transformer_blocks.0.attn.to_q"]
    k = wrapped["transformer_blocks.0.attn.to_k"]
    g = q.prep_group
    x = torch.randn(2, 256, q.base.in_features, device="cuda").bfloat16()
    x2 = x.clone()
    with torch.no_grad():
        for m in g.members:
            m.prep_group = None
        want_q, want_k = q(x), k(x)            # each linear preparing its own
        for m in g.members:
            m.prep_group = g
        yq = q(x)                   # prepares q, k and v for x
        assert len(g._ready) == 2
        got_k2 = k(x2)              # another input while x's results are pending: k prepares its own
        assert len(g._ready) == 2
        got_k = k(x)                # taken from the group
        assert len(g._ready) == 1
        again_k = k(x)              # called again on the same input: k prepares its own
    assert torch.equal(yq, want_q)
    assert torch.equal(got_k, want_k) and torch.equal(got_k2, want_k) and torch.equal(again_k, want_k)


def test_attach_adapters_groups_qkv_on_the_fused_path():
    """serve.attach_adapters(fused_gemm=True) groups the q / k / v MultiAdapterLinear layers of
    each attention block; the routed forward is bit-identical to every layer preparing its own."""
    from lithe_b200 import serve
    from tests.helpers import random_adapter

    torch.manual_seed(9)
    cfg = FluxConfig.tiny()
    model = FluxShapedTransformer(cfg).cuda().bfloat16().eval()
    targets = lora_targets(model)
    ads = [random_adapter([(n, m.in_features, m.out_features) for n, m in targets], rank=16, seed=30 + s)
           for s in range(3)]
    router, layers = serve.attach_adapters(model, ads, fused_gemm=True)
    groups = {id(m.prep_group): m.prep_group for m in layers.values() if m.prep_group is not None}
    assert len(groups) == 6 and all(len(g.members) == 3 for g in groups.values())
    router.set([[(2, 1.0)], [(0, 0.5)]])
    lat = torch.randn(2, 256, cfg.in_channels, device="cuda").bfloat16()
    txt = torch.randn(2, 256, cfg.text_dim, device="cuda").bfloat16()
    pooled = torch.randn(2, cfg.pooled_dim, device="cuda").bfloat16()
    args = (lat, txt, pooled, torch.full((2,), 0.5, device="cuda"))
    with torch.no_grad():
        grouped = model(*args)
        assert all(g._key is None and not g._ready for g in groups.values())
        for m in layers.values():
            m.prep_group = None
        alone = model(*args)
        again = model(*args)                         # the B factors from each layer's cache
        router.set([[(1, 1.0)], [(0, 0.5)]])
        rerouted = model(*args)
        for m in layers.values():
            m._bdec_cache = None
        rerouted_fresh = model(*args)
    assert torch.equal(grouped, alone) and torch.equal(again, alone)
    assert not torch.equal(rerouted, alone) and torch.equal(rerouted, rerouted_fresh)


def test_decoded_b_factors_are_reused_while_routing_and_bank_are_unchanged():
    """The fused-GEMM path decodes a layer's (or a group's) B factors once per routing: later
    calls with the same slot-id tensor and unchanged bank take the cached b_dec and give the
    same output bit for bit; a new routing, an in-place change of the slot ids, or a write to
    the bank (torch op or pack kernel) decodes again."""
    model, wrapped, args = _model(11)
    q = wrapped["transformer_blocks.0.attn.to_q"]
    o = wrapped["transformer_blocks.0.attn.to_out.0"]          # not in a group
    g = q.prep_group
    bank = q.bank
    with torch.no_grad():
        first = model(*args)
        bd_solo, bd_group = o._bdec_cache[1], list(g._bdecs)
        second = model(*args)
        assert o._bdec_cache[1] is bd_solo and all(a is b for a, b in zip(g._bdecs, bd_group))
        assert torch.equal(first, second)
        # a new routing (another tensor) decodes again
        ids2 = torch.tensor([7, 2], dtype=torch.int32, device="cuda")
        for m in wrapped.values():
            m.assign = ids2
        routed2 = model(*args)
        assert o._bdec_cache[1] is not bd_solo and not torch.equal(routed2, first)
        # an in-place change of the slot ids decodes again
        ids2.copy_(torch.tensor([2, 7], dtype=torch.int32))
        back = model(*args)
        assert torch.equal(back, first)
        # a write to the bank through the pack kernel decodes again: slot 7 gets slot 2's payload
        keep = o._bdec_cache[1]
        raw = torch.randint(0, 512, (bank.layout.num_indices,), dtype=torch.int16, device="cuda")
        bank.load_raw(7, raw)
        after = model(*args)
        assert o._bdec_cache[1] is not keep and not torch.equal(after, first)
        # against a forward with nothing cached
        for m in wrapped.values():
            m._bdec_cache = None
            if m.prep_group is not None:
                m.prep_group._bdec_key = None
        fresh = model(*args)
    assert torch.equal(after, fresh)
