"""lithe_lora_prep_ws: the shrink of lithe_lora_prep with its x stages split evenly over the SMs.

A 64-token tile may be shared by several CTAs; each stores its fp32 partial h in the workspace
and the B-decode launch that follows adds them in CTA order.  Checked against the fp32 truth of the reference's shrink
(h = w_b * scaling * x_b . A_j^T, lithe/kernels/shared.py:36-85 there) with the SGMV tests'
tolerance (max-abs-rel <= 2e-2, relative Frobenius < 1e-2), against the unsplit prep (the same
partial products summed in another fp32 order, so equal to within one bf16 rounding step),
bit for bit against itself (run twice, and with a reused workspace after a call of another
shape), and with b_dec omitted (the B-decode launch then only combines)."""
import pytest
import torch

from lithe_b200 import device_errors
from lithe_b200.kernels import PackedBank, _launch
from tests.helpers import max_abs_rel, oracle_factors, random_adapter, rel_fro

pytestmark = pytest.mark.gpu

# (batch, m, d_in, d_out): FLUX img and txt streams at B=14 (896 and 112 tiles over 148 SMs),
# tiles spread over many CTAs (2 tiles of 8 stages -> 16 one-stage CTAs), an odd chunk count
# (3 chunks: a one-chunk last stage), a single stage, ragged m
SHAPES = [(14, 4096, 3072, 3072), (14, 512, 3072, 12288), (2, 5, 1024, 256), (3, 70, 192, 128), (1, 64, 64, 64),
          (4, 200, 512, 768), (5, 1000, 1280, 640)]


def _setup(bsz, m, d_in, d_out, seed):
    n_ad = min(bsz, 4)
    ads = [random_adapter([("l", d_in, d_out)], rank=16, seed=seed + s) for s in range(n_ad)]
    bank = PackedBank.from_adapters(ads, "cuda")
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(bsz, m, d_in, generator=g, device="cuda").bfloat16()
    assign = [(b % (n_ad + 1)) - 1 if bsz > 2 else b % n_ad for b in range(bsz)]     # some unrouted (-1)
    wts = [0.5 + 0.25 * (b % 3) for b in range(bsz)]
    return ads, bank, x, assign, wts


def _run(bank, x, assign, wts, scaling, split, workspace=None, with_bdec=True, d_out=None):
    bsz, m, _ = x.shape
    va, vb = bank.views("l")
    h = torch.full((bsz * m, 16), 7.0, dtype=torch.bfloat16, device="cuda")
    bd = torch.full((bsz, d_out, 16), 7.0, dtype=torch.bfloat16, device="cuda") if with_bdec else None
    _launch.lora_prep_(x, view_a=va, view_b=vb, n_slots=bank.n_slots,
                       ids=torch.tensor(assign, dtype=torch.int32, device="cuda"),
                       weights=torch.tensor(wts, device="cuda"), d_out=d_out, lut=bank.lut, scaling=scaling, h=h,
                       b_dec=bd, split=split, workspace=workspace)
    torch.cuda.synchronize()
    return h, bd


@pytest.mark.parametrize("bsz,m,d_in,d_out", SHAPES)
def test_split_prep_matches_truth_and_unsplit(bsz, m, d_in, d_out):
    ads, bank, x, assign, wts = _setup(bsz, m, d_in, d_out, seed=bsz + m + d_in)
    sc = 0.75
    h, bd = _run(bank, x, assign, wts, sc, split=True, d_out=d_out)
    h0, bd0 = _run(bank, x, assign, wts, sc, split=False, d_out=d_out)
    assert device_errors() == 0
    assert torch.equal(bd, bd0)
    # the same products in another fp32 order: equal but for rare one-step bf16 rounding differences
    same = (h == h0).float().mean().item()
    assert same > 0.97, same
    assert max_abs_rel(h.float(), h0.float()) < 1e-2
    # bit for bit against itself
    h2, _ = _run(bank, x, assign, wts, sc, split=True, d_out=d_out)
    assert torch.equal(h, h2)
    facs = [oracle_factors(a)["l"] for a in ads]
    hv = h.view(bsz, m, 16)
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(1))[:256]
    for b, j in enumerate(assign):
        if j < 0:
            assert not hv[b].any()
            continue
        a_f = torch.from_numpy(facs[j][0])
        want = wts[b] * sc * (x[b, rows.cuda()].float().cpu() @ a_f.T)
        got = hv[b, rows.cuda()].float().cpu()
        assert max_abs_rel(got, want) <= 2e-2 and rel_fro(got, want) < 1e-2, (b, j)


def test_split_prep_reused_workspace_and_h_only():
    """One workspace across calls of different shapes, and h without b_dec (the B-decode launch
    then only combines the shared tiles)."""
    big = _setup(14, 512, 3072, 3072, seed=11)
    small = _setup(2, 5, 1024, 256, seed=12)
    need = max(_launch.prep_workspace_bytes(14, 512, 3072), _launch.prep_workspace_bytes(2, 5, 1024))
    assert need > 0
    ws = torch.full((need,), 0xAB, dtype=torch.uint8, device="cuda")      # contents on entry do not matter
    want_big, _ = _run(big[1], big[2], big[3], big[4], 1.0, split=True, d_out=3072)
    want_small, _ = _run(small[1], small[2], small[3], small[4], 1.0, split=True, d_out=256)
    for _ in range(2):
        got_big, _ = _run(big[1], big[2], big[3], big[4], 1.0, split=True, workspace=ws, d_out=3072)
        got_small, _ = _run(small[1], small[2], small[3], small[4], 1.0, split=True, workspace=ws, d_out=256)
        assert torch.equal(got_big, want_big) and torch.equal(got_small, want_small)
    got_h_only, bd = _run(big[1], big[2], big[3], big[4], 1.0, split=True, workspace=ws, with_bdec=False, d_out=3072)
    assert bd is None and torch.equal(got_h_only, want_big)
    assert device_errors() == 0


def test_split_prep_workspace_size_checked():
    _, bank, x, assign, wts = _setup(4, 200, 512, 768, seed=3)
    need = _launch.prep_workspace_bytes(4, 200, 512)
    # 4 samples x 4 tiles x 4 stages (8 chunks of 64 columns, two per stage)
    assert need == min(torch.cuda.get_device_properties(0).multi_processor_count, 64) * 8192
    with pytest.raises(ValueError):
        _run(bank, x, assign, wts, 1.0, split=True, workspace=torch.empty(need - 16, dtype=torch.uint8,
                                                                          device="cuda"), d_out=768)
