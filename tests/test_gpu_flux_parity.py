"""Model-level parity of the index-resident LoRA path against the oracle, at FLUX.1-dev's real
widths: a FLUX-shaped transformer with hidden 3072, 24 heads and FFN 12288, cut to 2 double +
2 single blocks, at the 512^2 workload shape (1024 image + 512 text tokens), B = 14 samples
routed to 14 distinct slots of a 10,000-slot packed bank.  It is the counterpart of the
reference's multi-adapter model test (tests/test_diffusers_integration.py:98-130 there, which
checks the routed model against per-sample truth and needs diffusers).

Both adapter layouts are covered -- the diffusers module set (one adapter module per linear)
and the Kohya fused modules (q/k/v and linear1 served on their diffusers linears from row
ranges of one resident slot, modulation linears on one token row per sample) -- and both LoRA
paths: cuBLAS + the fused decode/SGMV kernel, and lithe_lora_prep + the expand inside
lithe_lora_gemm (``fused_gemm=True``, default in_features policy).

(a) Every wrapped linear, on the activations that reach it in the model forward (captured by
    forward hooks): the LoRA delta its kernels compute (run on the captured input with a zero
    base) against oracle/sgmv_ref.serve_delta in fp32 (the reference's serve.py routed forward
    restated) on sampled token rows.  Tolerance: max-abs-rel <= 2e-2 and relative Frobenius
    error < 1e-2, the per-linear bar of the SGMV tests.
(b) The final latent of a 2-step denoise against the same model whose target linears carry the
    oracle-decoded factors (oracle/decode_ref, rounded to bf16 as serve.py does) in a dense
    per-sample bmm: relative Frobenius error < LATENT_REL_FRO, while the adapters move the
    latent by more than 10 x that.
Indices of the 14 routed slots are host-generated (seeded) and loaded into the bank; the other
9,986 slots hold seeded random words.
"""
import numpy as np
import pytest
import torch

from lithe_b200 import kohya
from lithe_b200.fileio import LitheAdapter
from lithe_b200.flux_model import FluxConfig, FluxShapedTransformer, denoise, lora_targets
from lithe_b200.kernels import PackedBank, PackedLayout, PerSampleLoRALinear, _launch
from lithe_b200.kernels.layers import PackedLoRALinear
from lithe_b200.kernels.shared import packed_codebook_lora_delta_
from oracle import codebook_ref, decode_ref, sgmv_ref
from tests.helpers import max_abs_rel, rel_fro

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2          # per-linear LoRA delta vs the fp32 oracle
REL_FRO = 1e-2
LATENT_REL_FRO = 2e-2       # final latent vs the oracle-factor model (bf16 model, 4 blocks, 2 steps)
B, IMG, TXT, RANK = 14, 1024, 512, 16
BANK_SLOTS = 10_000
ROWS = 12                   # sampled token rows per sample for the CPU oracle


def _model(seed):
    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = FluxShapedTransformer(FluxConfig(double_blocks=2, single_blocks=2))
    return model.bfloat16().eval()


def _setup(layout_kind):
    """Model, bank (10,000 slots, the 14 routed ones loaded from host adapters), the adapters,
    the target table {diffusers path: (module name, r0, r1)} and the routed slot ids."""
    model = _model(11)
    if layout_kind == "kohya":
        mods = kohya.kohya_flux_modules(rank=RANK, double_blocks=2, single_blocks=2)
        key_format = "kohya"
    else:
        mods = [{"name": n, "shape_a": [RANK, m.in_features], "shape_b": [m.out_features, RANK]}
                for n, m in lora_targets(model)]
        key_format = "diffusers"
    layout = PackedLayout.from_modules(mods)
    targets = kohya.split_targets(layout.names, layout.shapes_a, layout.shapes_b, key_format)
    bank = PackedBank(layout, BANK_SLOTS, "cuda")
    bank.fill_random(seed=1234)
    slots = torch.randperm(BANK_SLOTS, generator=torch.Generator().manual_seed(300))[:B].tolist()
    ads = []
    for i, slot in enumerate(slots):
        rng = np.random.default_rng(500 + i)
        idx = {m["name"]: {"A": rng.integers(0, 512, (3, decode_ref.num_blocks(m["shape_a"]))).astype(np.uint16),
                           "B": rng.integers(0, 512, (3, decode_ref.num_blocks(m["shape_b"]))).astype(np.uint16)}
               for m in mods}
        ad = LitheAdapter(modules=mods, indices=idx, rank=RANK, alpha=float(RANK), key_format=key_format)
        bank.load_adapter(slot, ad)
        ads.append(ad)
    return model, bank, ads, targets, torch.tensor(slots, dtype=torch.int32, device="cuda")


def _oracle_indices(ads, name, r0, r1, d_out):
    """Index banks (14, L, nA) / (14, L, nB) of target rows [r0, r1) of module ``name``: B row
    range [r0, r1) of a rank-16 factor is its B block range [r0 / 4, r1 / 4)."""
    per_block = 64 // RANK
    ia = np.stack([ad.indices[name]["A"] for ad in ads]).astype(np.int64)
    ib = np.stack([ad.indices[name]["B"][:, r0 // per_block: r1 // per_block] for ad in ads]).astype(np.int64)
    assert ib.shape[2] * per_block == r1 - r0 == d_out
    return ia, ib


def _install(model, table):
    for path, module in table.items():
        parent, _, child = path.rpartition(".")
        setattr(model.get_submodule(parent), child, module)


def _inputs():
    g = torch.Generator(device="cuda").manual_seed(7)
    lat = torch.randn(B, IMG, 64, generator=g, device="cuda").bfloat16()
    txt = torch.randn(B, TXT, 4096, generator=g, device="cuda").bfloat16()
    pooled = torch.randn(B, 768, generator=g, device="cuda").bfloat16()
    return lat, txt, pooled


def _kernel_delta(layer, x3):
    """The LoRA delta the wrapped layer's kernels produce for input x3, on a zero base: the
    decode/SGMV kernel, or (fused path) lithe_lora_prep + the expand inside lithe_lora_gemm."""
    bsz, m, d_in = x3.shape
    d_out = layer.base.out_features
    ids = layer.assign
    if layer.fused_gemm and layer._gemm_ok(x3):
        va, vb = layer.bank.views(layer.name, layer.rows)
        h = torch.empty(bsz * m, RANK, dtype=torch.bfloat16, device="cuda")
        b_dec = torch.empty(bsz, d_out, RANK, dtype=torch.bfloat16, device="cuda")
        _launch.lora_prep_(x3, view_a=va, view_b=vb, n_slots=layer.bank.n_slots, ids=ids, weights=None, d_out=d_out,
                           lut=layer.bank.lut, scaling=layer.scaling, h=h, b_dec=b_dec)
        out = torch.empty(bsz * m, d_out, dtype=torch.bfloat16, device="cuda")
        zero_w = torch.zeros(d_out, d_in, dtype=torch.bfloat16, device="cuda")
        _launch.lora_gemm_(x3.reshape(bsz * m, d_in), zero_w, None, out, h=h, b_dec=b_dec, rows_per_sample=m)
        return out.view(bsz, m, d_out), "gemm"
    out = torch.zeros(bsz, m, d_out, dtype=torch.bfloat16, device="cuda")
    packed_codebook_lora_delta_(out, x3, layer.bank, layer.name, ids, scaling=layer.scaling, rows=layer.rows)
    return out, "sgmv" if m > 8 else "small-m"


@pytest.mark.parametrize("layout_kind", ["diffusers", "kohya"])
def test_flux_3072_per_linear_deltas_and_final_latent_match_oracle(layout_kind):
    model, bank, ads, targets, ids = _setup(layout_kind)
    pa, pb = codebook_ref.twin_pools()
    bases = {path: model.get_submodule(path) for path in targets}
    packed = {}
    for path, (name, r0, r1) in targets.items():
        full = r0 == 0 and r1 == bank.layout.shapes_b[bank.layout.index(name)][0]
        layer = PackedLoRALinear(bases[path], bank, name, RANK, 1.0, rows=None if full else (r0, r1))
        layer.assign = ids
        packed[path] = layer
    # the dense comparator: oracle-decoded fp32 factors, rounded to bf16 by PerSampleLoRALinear
    dense = {}
    for path, (name, r0, r1) in targets.items():
        lin = bases[path]
        ia, ib = _oracle_indices(ads, name, r0, r1, lin.out_features)
        facs = [(torch.from_numpy(decode_ref.decode_factor(ia[i], (RANK, lin.in_features), pa)).cuda(),
                 torch.from_numpy(decode_ref.decode_factor(ib[i], (lin.out_features, RANK), pb)).cuda(), 1.0)
                for i in range(B)]
        d = PerSampleLoRALinear(lin, "sgmv")
        d.set_factors(facs)
        dense[path] = d
    lat, txt, pooled = _inputs()
    t = torch.full((B,), 0.5, device="cuda")
    latents, forms = {}, set()
    for variant in ("base", "dense", "lithe", "fused"):
        _install(model, bases if variant == "base" else dense if variant == "dense" else packed)
        for layer in packed.values():
            layer.fused_gemm = variant == "fused"
        with torch.no_grad():
            latents[variant] = denoise(model, lat, txt, pooled, 2).float()
        if variant not in ("lithe", "fused"):
            continue
        # (a) per-linear deltas on the activations of one forward, captured by hooks
        captured = {}
        hooks = [layer.register_forward_hook(
            lambda mod, inp, out, path=path: captured.__setitem__(path, inp[0].detach().clone()))
            for path, layer in packed.items()]
        with torch.no_grad():
            model(lat, txt, pooled, t)
        for hk in hooks:
            hk.remove()
        assert set(captured) == set(packed)
        sel = torch.Generator().manual_seed(3)
        for path, x in captured.items():
            layer = packed[path]
            x3 = x.unsqueeze(1) if x.dim() == 2 else x
            with torch.no_grad():
                got, form = _kernel_delta(layer, x3.contiguous())
            forms.add(form)
            m = x3.shape[1]
            rows = torch.randperm(m, generator=sel)[: min(ROWS, m)]
            xs = x3[:, rows.cuda()].float().cpu()
            name, r0, r1 = targets[path]
            ia, ib = _oracle_indices(ads, name, r0, r1, layer.base.out_features)
            ids_o, w_o = sgmv_ref.routes_to_tables([[(i, 1.0)] for i in range(B)])
            want = sgmv_ref.serve_delta(xs, ia, ib, [1.0] * B, ids_o, w_o, RANK, layer.base.out_features, pa, pb)
            g = got[:, rows.cuda()].float().cpu()
            err_max, err_fro = max_abs_rel(g, want), rel_fro(g, want)
            assert err_max <= MAX_ABS_REL and err_fro < REL_FRO, \
                f"{layout_kind}/{variant} {path} ({form}): max-abs-rel {err_max:.2e}, rel-Fro {err_fro:.2e}"
        del captured
    # every kernel form the forward uses was exercised: SGMV, small-m (Kohya modulation), fused GEMM
    assert {"sgmv", "gemm"} <= forms
    if layout_kind == "kohya":
        assert "small-m" in forms
    # (b) final latent of the 2-step denoise
    effect = rel_fro(latents["dense"], latents["base"])
    for variant in ("lithe", "fused"):
        assert torch.isfinite(latents[variant]).all()
        err = rel_fro(latents[variant], latents["dense"])
        assert err < LATENT_REL_FRO, f"{layout_kind}/{variant}: latent rel-Fro {err:.2e} vs the oracle-factor model"
        assert effect > 10 * err, f"{layout_kind}: the adapters move the latent by {effect:.2e}, the error is {err:.2e}"
