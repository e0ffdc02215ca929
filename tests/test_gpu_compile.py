"""torch.compile through the index-resident LoRA layers.

The kernels are registered as torch.library custom ops (``lithe_b200::sgmv_index_``,
``lora_prep``, ``lora_gemm``, ``decode_packed``) with fake kernels, so dynamo traces a model
whose linears are ``PackedLoRALinear`` into one graph: ``fullgraph=True`` turns any graph
break into an error.  (The reference's timed renders run the wrapped transformer under
torch.compile, serving/bench_same_batch.py:95-96 there.)

* one wrapped linear on both LoRA paths: aot_eager (functionalised graph, eager kernels)
  bit-identical to eager; inductor bit-identical on the fused-GEMM path, whose graph holds only
  this package's ops, and within bf16 precision on the cuBLAS + SGMV path;
* the tiny FLUX-shaped model with every target linear wrapped, compiled with aot_eager
  (functionalised graph, eager kernels): bit-identical to eager, on both paths;
* the same model compiled with inductor, which fuses the model's own norms and activations
  differently: within bf16 precision of eager (rel-Fro < 1e-2), and far closer to the eager
  output with adapters than to the base model's.
"""
import pytest
import torch

from lithe_b200.flux_model import FluxConfig, FluxShapedTransformer, lora_targets
from lithe_b200.kernels import PackedBank, PackedLayout, PackedLoRALinear, wrap_linears
from tests.helpers import rel_fro

pytestmark = pytest.mark.gpu


def _bank_for(targets, seed):
    layout = PackedLayout.from_modules([{"name": n, "shape_a": [16, m.in_features], "shape_b": [m.out_features, 16]}
                                        for n, m in targets])
    bank = PackedBank(layout, 8, "cuda")
    bank.fill_random(seed=seed)
    return bank


@pytest.mark.parametrize("fused", [False, True])
def test_compiled_linear(fused):
    """One wrapped linear: aot_eager bit-identical to eager; inductor bit-identical on the
    fused path (the graph is only the package's ops) and within bf16 precision on the SGMV
    path (inductor may lower the cuBLAS base linear differently)."""
    torch._dynamo.reset()
    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 768).cuda().bfloat16()
    bank = _bank_for([("l", lin)], seed=5)
    layer = PackedLoRALinear(lin, bank, "l", 16, 1.0, fused_gemm=fused)
    layer.assign = torch.tensor([3, 0, 6], dtype=torch.int32, device="cuda")
    x = torch.randn(3, 256, 512, device="cuda").bfloat16()
    if fused:
        assert layer._gemm_ok(x)
    with torch.no_grad():
        want = layer(x)
        got_ae = torch.compile(layer, fullgraph=True, backend="aot_eager")(x)
        torch._dynamo.reset()
        got_ind = torch.compile(layer, fullgraph=True)(x)
    assert torch.equal(got_ae, want)
    if fused:
        assert torch.equal(got_ind, want)
    else:
        assert rel_fro(got_ind, want) < 1e-2


def _tiny(fused, seed):
    torch.manual_seed(seed)
    cfg = FluxConfig.tiny()
    model = FluxShapedTransformer(cfg).cuda().bfloat16().eval()
    targets = lora_targets(model)
    bank = _bank_for(targets, seed=seed + 1)
    # scaling 20: at the tiny width the adapters' effect on the output must stand well above the
    # bf16-level differences inductor's own fusions make
    wrapped = wrap_linears(model, [n for n, _ in targets], lambda n, lin: PackedLoRALinear(lin, bank, n, 16, 20.0))
    for m in wrapped.values():
        m.assign = torch.tensor([2, 7], dtype=torch.int32, device="cuda")
        m.fused_gemm = fused
    tokens = 256 if fused else 96        # 256-token streams make every target eligible for the GEMM path
    lat = torch.randn(2, tokens, cfg.in_channels, device="cuda").bfloat16()
    txt = torch.randn(2, tokens, cfg.text_dim, device="cuda").bfloat16()
    pooled = torch.randn(2, cfg.pooled_dim, device="cuda").bfloat16()
    return model, wrapped, (lat, txt, pooled, torch.full((2,), 0.5, device="cuda"))


@pytest.mark.parametrize("fused", [False, True])
def test_compiled_tiny_flux_fullgraph(fused):
    torch._dynamo.reset()
    model, wrapped, args = _tiny(fused, seed=3)
    if fused:
        assert all(m._gemm_ok(torch.empty(2, 256, m.base.in_features, dtype=torch.bfloat16, device="cuda"))
                   for m in wrapped.values())
    with torch.no_grad():
        eager = model(*args)
        same = torch.compile(model, fullgraph=True, backend="aot_eager")(*args)
        assert torch.equal(same, eager)
        torch._dynamo.reset()
        inductor = torch.compile(model, fullgraph=True)(*args)
        # the LoRA effect survives compilation: compare with the compiled base model
        for m in wrapped.values():
            m.assign = torch.full((2,), -1, dtype=torch.int32, device="cuda")   # unrouted: no delta
        base_eager = model(*args)
    assert torch.isfinite(inductor).all()
    assert rel_fro(inductor, eager) < 1e-2
    # the compiled output carries the LoRA: it is far closer to eager-with-adapters than to the base
    assert rel_fro(inductor, eager) < 0.5 * rel_fro(inductor, base_eager)
