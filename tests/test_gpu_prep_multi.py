"""lithe_lora_prep_multi: h and b_dec of up to 4 linears that read the same x, x streamed once.

Each target's outputs must equal lithe_lora_prep's for that target alone bit for bit: the
factor chunks are the same bytes (decoded once into the workspace instead of per tile), and
the shrink adds the same products in the same order (the same grid and 64-token tiles).  The
values are also checked against the fp32 truth of the reference's shrink
(h = w_b * scaling * x_b . A_j^T, lithe/kernels/shared.py:36-85 there) with the SGMV tests'
tolerance (max-abs-rel <= 2e-2, relative Frobenius < 1e-2)."""
import pytest
import torch

from lithe_b200 import device_errors
from lithe_b200.kernels import PackedBank, PackedLayout, _launch
from tests.helpers import max_abs_rel, oracle_factors, random_adapter, rel_fro

pytestmark = pytest.mark.gpu

# (batch, m, d_in, d_outs): FLUX q/k/v at B=14 x 4096 and x 512 tokens, ragged m with unrouted
# samples and 1..4 targets of different widths, a few rows per sample
CASES = [(14, 4096, 3072, [3072, 3072, 3072]), (14, 512, 3072, [3072, 3072, 3072]),
         (3, 200, 512, [768, 256, 512, 1024]), (4, 70, 192, [128, 64]), (2, 5, 1024, [256]),
         (5, 1000, 1280, [640, 1280, 384])]


def _bank(d_in, d_outs, n_ad, seed):
    mods = [(f"t{i}", d_in, d) for i, d in enumerate(d_outs)]
    ads = [random_adapter(mods, rank=16, seed=seed + s) for s in range(n_ad)]
    return ads, PackedBank.from_adapters(ads, "cuda")


@pytest.mark.parametrize("bsz,m,d_in,d_outs", CASES)
def test_multi_prep_equals_single_target_preps(bsz, m, d_in, d_outs):
    n_ad = min(bsz, 4)
    ads, bank = _bank(d_in, d_outs, n_ad, seed=bsz * 7 + len(d_outs))
    g = torch.Generator(device="cuda").manual_seed(m + d_in)
    x = torch.randn(bsz, m, d_in, generator=g, device="cuda").bfloat16()
    assign = [(b % (n_ad + 1)) - 1 if bsz > 2 else b % n_ad for b in range(bsz)]        # some unrouted
    ids = torch.tensor(assign, dtype=torch.int32, device="cuda")
    wts = torch.tensor([0.5 + 0.25 * (b % 3) for b in range(bsz)], device="cuda")
    scalings = [0.75 + 0.5 * t for t in range(len(d_outs))]
    names = [f"t{i}" for i in range(len(d_outs))]
    views = [bank.views(nm) for nm in names]
    hs = [torch.full((bsz * m, 16), 7.0, dtype=torch.bfloat16, device="cuda") for _ in names]
    bds = [torch.full((bsz, d, 16), 7.0, dtype=torch.bfloat16, device="cuda") for d in d_outs]
    bds[-1] = None if len(d_outs) > 1 else bds[-1]          # a target without b_dec
    _launch.lora_prep_multi_(x, views_a=[v[0] for v in views], views_b=[v[1] for v in views], d_outs=d_outs,
                             n_slots=bank.n_slots, ids=ids, weights=wts, lut=bank.lut, scalings=scalings, hs=hs,
                             b_decs=bds)
    torch.cuda.synchronize()
    assert device_errors() == 0
    for t, nm in enumerate(names):
        h1 = torch.empty(bsz * m, 16, dtype=torch.bfloat16, device="cuda")
        bd1 = torch.empty(bsz, d_outs[t], 16, dtype=torch.bfloat16, device="cuda")
        _launch.lora_prep_(x, view_a=views[t][0], view_b=views[t][1], n_slots=bank.n_slots, ids=ids, weights=wts,
                           d_out=d_outs[t], lut=bank.lut, scaling=scalings[t], h=h1, b_dec=bd1, split=False)
        torch.cuda.synchronize()
        assert torch.equal(hs[t], h1), nm
        if bds[t] is not None:
            assert torch.equal(bds[t], bd1), nm
        facs = [oracle_factors(a)[nm] for a in ads]
        hv = hs[t].view(bsz, m, 16)
        rows = torch.randperm(m, generator=torch.Generator().manual_seed(t))[:128].cuda()
        for b, j in enumerate(assign):
            if j < 0:
                assert not hv[b].any()
                continue
            want = float(wts[b]) * scalings[t] * (x[b, rows].float().cpu() @ torch.from_numpy(facs[j][0]).T)
            got = hv[b, rows].float().cpu()
            assert max_abs_rel(got, want) <= 2e-2 and rel_fro(got, want) < 1e-2, (nm, b)


def test_multi_prep_rejects_bad_arguments():
    ads, bank = _bank(256, [256, 256], 2, seed=1)
    x = torch.zeros(2, 64, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(2, dtype=torch.int32, device="cuda")
    va, vb = bank.views("t0")
    hs = [torch.empty(128, 16, dtype=torch.bfloat16, device="cuda") for _ in range(5)]
    with pytest.raises(ValueError):          # five targets
        _launch.lora_prep_multi_(x, views_a=[va] * 5, views_b=[vb] * 5, d_outs=[256] * 5, n_slots=2, ids=ids,
                                 weights=None, lut=bank.lut, scalings=[1.0] * 5, hs=hs, b_decs=[None] * 5)
    with pytest.raises(ValueError):          # workspace too small (checked by the library)
        _launch.lora_prep_multi_(x, views_a=[va, va], views_b=[vb, vb], d_outs=[256, 256], n_slots=2, ids=ids,
                                 weights=None, lut=bank.lut, scalings=[1.0, 1.0], hs=hs[:2], b_decs=[None, None],
                                 workspace=torch.empty(1024, dtype=torch.uint8, device="cuda"))
