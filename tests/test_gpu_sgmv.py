"""Fused decode + SGMV kernel (lithe_sgmv_index) against the oracle and the reference's goldens.

Tolerance (bf16 activations, fp32 accumulation): on the LoRA delta, max-abs-rel
max|got - truth| / max|truth| <= 2e-2 and relative Frobenius error < 1e-2 against the fp32
truth (x_b A_j^T B_j^T with exactly decoded factors), as in the reference's GPU tests
(tests/test_kernels.py:202-216 there).  Exact properties (doubling, sample independence)
are checked bit for bit."""
import numpy as np
import pytest
import torch

from lithe_b200 import codebook as cb
from lithe_b200 import device_errors, serve
from lithe_b200.kernels import IndexLoRALinear, PackedBank, PackedLoRALinear, _launch, shared_codebook_lora_delta
from oracle import decode_ref, sgmv_ref
from tests.helpers import (FLUX_SHAPES, bf16_from_bits, config1_inputs, load_golden, max_abs_rel, oracle_factors,
                           oracle_pools, random_adapter, rel_fro)

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
REL_FRO = 1e-2


def _banks(ads, fmt):
    if fmt == "packed":
        bank = PackedBank.from_adapters(ads, "cuda")
        va, vb = bank.views("l")
        return va, vb, bank
    dt = torch.int16 if fmt == "i16" else torch.int32
    ia = torch.stack([torch.from_numpy(a.indices["l"]["A"].astype(np.int64)) for a in ads]).to(dt).cuda().contiguous()
    ib = torch.stack([torch.from_numpy(a.indices["l"]["B"].astype(np.int64)) for a in ads]).to(dt).cuda().contiguous()
    return _launch.level_major_view(ia), _launch.level_major_view(ib), (ia, ib)


def run_fused(x, ads, assign, fmt="packed", accumulate=False, out=None, weights=None, scaling=1.0, mode=None):
    va, vb, keep = _banks(ads, fmt)
    d_out = ads[0].modules[0]["shape_b"][0]
    r = ads[0].rank
    if out is None:
        out = torch.empty(x.shape[0], x.shape[1], d_out, dtype=torch.bfloat16, device="cuda")
    ids = torch.tensor(assign, dtype=torch.int32, device="cuda")
    w = None if weights is None else torch.tensor(weights, dtype=torch.float32, device="cuda")
    lut = cb.kernel_lut(*cb.twin_pools())
    _launch.sgmv_index_(x, out, accumulate=accumulate, view_a=va, view_b=vb, n_slots=len(ads), ids=ids, weights=w,
                        rank=r, lut=lut, scaling=scaling, mode=mode)
    torch.cuda.synchronize()
    del keep
    return out


def truth_delta(x, ads, assign, weights=None, scaling=1.0):
    facs = [oracle_factors(a)["l"] for a in ads]
    xs = x.float().cpu()
    outs = []
    for b, j in enumerate(assign):
        if j < 0 or j >= len(ads):
            outs.append(torch.zeros(x.shape[1], facs[0][1].shape[0]))
            continue
        a, bm = (torch.from_numpy(f) for f in facs[j])
        w = 1.0 if weights is None else weights[b]
        outs.append((xs[b] @ a.T @ bm.T) * (w * scaling))
    return torch.stack(outs)


CASES = [(256, 3072, 3072, 16), (50, 128, 192, 16), (1, 256, 384, 4), (77, 512, 640, 8), (64, 192, 256, 2),
         (33, 256, 128, 1), (130, 1024, 4096, 16), (200, 4096, 1024, 16)]


@pytest.mark.parametrize("seq,d_in,d_out,r", CASES)
@pytest.mark.parametrize("fmt", ["packed", "i16", "i32"])
def test_fused_delta_matches_truth(seq, d_in, d_out, r, fmt):
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=s) for s in range(3)]
    g = torch.Generator().manual_seed(seq + d_in)
    x = (torch.randn(4, seq, d_in, generator=g) * 0.5).bfloat16().cuda()
    assign = [2, 0, 1, 2]
    got = run_fused(x, ads, assign, fmt).float().cpu()
    want = truth_delta(x, ads, assign)
    assert max_abs_rel(got, want) <= MAX_ABS_REL and rel_fro(got, want) < REL_FRO
    assert device_errors() == 0


@pytest.mark.parametrize("seq,d_in,d_out,r", [(256, 3072, 3072, 16), (50, 128, 192, 16), (1, 256, 384, 4)])
def test_fused_matches_reference_bf16_steps(seq, d_in, d_out, r):
    """Against shared_codebook_lora_delta_reference restated (bf16 pools / factors / y)."""
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=s) for s in range(3)]
    x = (torch.randn(4, seq, d_in, generator=torch.Generator().manual_seed(1)) * 0.5).bfloat16()
    assign = [2, 0, 1, 2]
    ia = np.stack([a.indices["l"]["A"] for a in ads])
    ib = np.stack([a.indices["l"]["B"] for a in ads])
    pa, pb = oracle_pools()
    ref = sgmv_ref.shared_delta(x, ia, pa, ib, pb, assign, r, d_out, 1.0).float()
    got = run_fused(x.cuda(), ads, assign).float().cpu()
    assert rel_fro(got, ref) < REL_FRO and max_abs_rel(got, ref) <= MAX_ABS_REL


def test_accumulate_into_base_output():
    ads = [random_adapter([("l", 512, 768)], rank=16, seed=s) for s in range(2)]
    x = torch.randn(3, 100, 512, generator=torch.Generator().manual_seed(2)).bfloat16().cuda()
    base = (torch.randn(3, 100, 768, generator=torch.Generator().manual_seed(3)) * 0.05).bfloat16().cuda()
    assign = [1, 0, 1]
    got = run_fused(x, ads, assign, accumulate=True, out=base.clone()).float().cpu()
    delta = run_fused(x, ads, assign).float().cpu()
    want = base.float().cpu() + truth_delta(x, ads, assign)
    # one rounding of (base + delta) to bf16 plus the delta's own tolerance
    tol = 2 ** -8 * want.abs() + MAX_ABS_REL * truth_delta(x, ads, assign).abs().max()
    assert bool(((got - want).abs() <= tol).all())
    assert rel_fro(got - base.float().cpu(), delta) < REL_FRO


def test_unrouted_and_invalid_samples():
    ads = [random_adapter([("l", 256, 384)], rank=16, seed=s) for s in range(2)]
    x = torch.randn(4, 70, 256, generator=torch.Generator().manual_seed(4)).bfloat16().cuda()
    base = torch.randn(4, 70, 384, generator=torch.Generator().manual_seed(5)).bfloat16().cuda()
    device_errors()
    acc = run_fused(x, ads, [0, -1, 5, 1], accumulate=True, out=base.clone())
    assert device_errors() == 1                                   # slot 5 >= n_slots reported
    assert torch.equal(acc[1], base[1]) and torch.equal(acc[2], base[2])   # untouched
    delta = run_fused(x, ads, [0, -1, 5, 1])
    device_errors()
    assert bool((delta[1] == 0).all()) and bool((delta[2] == 0).all())
    want = truth_delta(x, ads, [0, -1, -1, 1])
    assert max_abs_rel(delta.float().cpu(), want) <= MAX_ABS_REL


def test_weights_and_scaling():
    ads = [random_adapter([("l", 256, 256)], rank=16, seed=s) for s in range(2)]
    x = torch.randn(3, 40, 256, generator=torch.Generator().manual_seed(6)).bfloat16().cuda()
    got = run_fused(x, ads, [0, 1, 0], weights=[0.25, 1.5, 0.0], scaling=2.0).float().cpu()
    want = truth_delta(x, ads, [0, 1, 0], weights=[0.25, 1.5, 0.0], scaling=2.0)
    assert max_abs_rel(got, want) <= MAX_ABS_REL and bool((got[2] == 0).all())


def test_exact_properties():
    """Doubling x doubles the delta bit for bit; each sample's result is independent of the batch."""
    ads = [random_adapter([("l", 1024, 2048)], rank=16, seed=s) for s in range(4)]
    x = torch.randn(5, 150, 1024, generator=torch.Generator().manual_seed(7)).bfloat16().cuda()
    assign = [3, 1, 0, 2, 1]
    d1 = run_fused(x, ads, assign)
    d2 = run_fused(x * 2, ads, assign)
    assert torch.equal(d2, d1 * 2)
    perm = [4, 2, 0, 3, 1]
    dp = run_fused(x[perm].contiguous(), ads, [assign[p] for p in perm])
    assert torch.equal(dp, d1[perm])
    single = run_fused(x[3:4].contiguous(), ads, [assign[3]])
    assert torch.equal(single[0], d1[3])
    assert torch.equal(run_fused(x, ads, assign, fmt="i16"), d1)
    assert torch.equal(run_fused(x, ads, assign, fmt="i32"), d1)


def test_empty_and_tiny_inputs():
    ads = [random_adapter([("l", 128, 128)], rank=16, seed=0)]
    x0 = torch.zeros(0, 10, 128, dtype=torch.bfloat16, device="cuda")
    assert run_fused(x0, ads, []).shape == (0, 10, 128)
    x1 = torch.randn(2, 1, 128, generator=torch.Generator().manual_seed(8)).bfloat16().cuda()
    got = run_fused(x1, ads, [0, 0]).float().cpu()
    assert max_abs_rel(got, truth_delta(x1, ads, [0, 0])) <= MAX_ABS_REL


def test_shared_api_against_reference_golden():
    z = load_golden("shared_small.npz")
    pa, pb = cb.twin_pools()
    for c in range(int(z["n_cases"])):
        seq, d_in, d_out, r = (int(v) for v in z[f"c{c}/shape"])
        x = bf16_from_bits(z[f"c{c}/x"]).cuda()
        ia, ib = torch.from_numpy(z[f"c{c}/ia"]).cuda(), torch.from_numpy(z[f"c{c}/ib"]).cuda()
        assign = torch.from_numpy(z[f"c{c}/assign"]).cuda()
        want = bf16_from_bits(z[f"c{c}/delta"]).float()
        # bf16 pools: the reference's own dtype steps; fp32 pools: exact decode
        for pools in ((pa.bfloat16().cuda(), pb.bfloat16().cuda()), (pa.cuda(), pb.cuda())):
            got = shared_codebook_lora_delta(x, ia, pools[0], ib, pools[1], assign, r, d_out, float(z["scaling"]))
            assert got.dtype == torch.bfloat16 and got.shape == (4, seq, d_out)
            assert rel_fro(got.float().cpu(), want) < REL_FRO and max_abs_rel(got.float().cpu(), want) <= MAX_ABS_REL


class _Toy(torch.nn.Module):
    def __init__(self, d_in, d_out):
        super().__init__()
        self.fc = torch.nn.Linear(d_in, d_out)
        torch.nn.init.zeros_(self.fc.weight)
        torch.nn.init.zeros_(self.fc.bias)

    def forward(self, x):
        return self.fc(x)


def test_serve_api_against_reference_golden():
    z = load_golden("serve_small.npz")
    rank, d_out = int(z["rank"]), int(z["d_out"])
    x = torch.from_numpy(z["x"])
    from lithe_b200.fileio import LitheAdapter
    ads = [LitheAdapter(modules=[{"name": "fc", "shape_a": [rank, x.shape[-1]], "shape_b": [d_out, rank]}],
                        indices={"fc": {"A": z[f"idx/{a}/A"], "B": z[f"idx/{a}/B"]}}, rank=rank,
                        alpha=float(z["alphas"][a])) for a in range(4)]
    model = _Toy(x.shape[-1], d_out).cuda().bfloat16()
    router, layers = serve.attach_adapters(model, ads)
    ids, w = z["ids"], z["weights"]
    routes = [[(int(i), float(wt)) for i, wt in zip(ids[b], w[b]) if i >= 0] for b in range(ids.shape[0])]
    router.set(routes)
    with torch.no_grad():
        y = model(x.bfloat16().cuda()).float().cpu()
    want = torch.from_numpy(z["y_f32"])
    for b, route in enumerate(routes):
        if not route:
            assert bool((y[b] == 0).all())
            continue
        assert max_abs_rel(y[b], want[b]) <= MAX_ABS_REL and rel_fro(y[b], want[b]) < REL_FRO, b
    router.set([[] for _ in routes])
    with torch.no_grad():
        assert bool((model(x.bfloat16().cuda()) == 0).all())


def test_config1_against_reference_golden():
    """Config 1 (3072->3072, r=16, B=4 x 256, adapters 0..3) through serve.attach_adapters in bf16."""
    z = load_golden("config1_rows.npz")
    ads, x = config1_inputs()
    model = _Toy(3072, 3072).cuda().bfloat16()
    router, _ = serve.attach_adapters(model, ads)
    router.set([[(i, 1.0)] for i in range(4)])
    with torch.no_grad():
        y = model(x.bfloat16().cuda()).float().cpu()
    rows = list(z["rows"])
    want = torch.from_numpy(z["y_rows"])
    assert max_abs_rel(y[:, rows], want) <= MAX_ABS_REL and rel_fro(y[:, rows], want) < REL_FRO
    assert np.allclose(y.double().sum(dim=(1, 2)).numpy(), z["sums"], rtol=5e-2, atol=5.0)
    assert np.allclose(y.double().pow(2).sum(dim=(1, 2)).numpy(), z["sq"], rtol=2e-2)


def test_index_layer_matches_truth():
    ads = [random_adapter([("l", 256, 384)], rank=16, seed=s) for s in range(2)]
    base = torch.nn.Linear(256, 384).cuda().bfloat16()
    pa, pb = (p.cuda() for p in cb.twin_pools())
    ia = torch.stack([torch.from_numpy(a.indices["l"]["A"].astype(np.int32)) for a in ads]).cuda()
    ib = torch.stack([torch.from_numpy(a.indices["l"]["B"].astype(np.int32)) for a in ads]).cuda()
    layer = IndexLoRALinear(base, ia, ib, pa.bfloat16(), pb.bfloat16(), 16, 1.0)
    bank = PackedBank.from_adapters(ads, "cuda")
    player = PackedLoRALinear(base, bank, "l", 16, 1.0)
    assign = torch.tensor([1, 0, 1], device="cuda", dtype=torch.int32)
    layer.assign = player.assign = assign
    facs = [oracle_factors(a)["l"] for a in ads]
    for x in (torch.randn(3, 64, 256, device="cuda").bfloat16(), torch.randn(3, 256, device="cuda").bfloat16()):
        truth = torch.stack([torch.nn.functional.linear(x[i].float(), base.weight.float(), base.bias.float())
                             + x[i].float() @ torch.from_numpy(facs[j][0]).cuda().T @ torch.from_numpy(facs[j][1]).cuda().T
                             for i, j in enumerate(assign.tolist())])
        with torch.no_grad():
            assert rel_fro(layer(x).float(), truth) < REL_FRO
            assert rel_fro(player(x).float(), truth) < REL_FRO


def test_lithe_linear_kernel_path_and_unsupported_shapes():
    """LitheLinear runs the fused kernel; a shape the kernel does not take raises (there is no
    eager second path), while decoded_factors() still decodes it bit-exactly."""
    import lithe_b200 as lb
    torch.manual_seed(0)
    for d_in, d_out, rank in ((256, 384, 16), (192, 160, 8), (96, 160, 8)):
        base = torch.nn.Linear(d_in, d_out).cuda().bfloat16()
        net = torch.nn.Sequential(base)
        layers = lb.inject_lithe(net, ["0"], rank=rank, alpha=2 * rank)
        layer = layers["0"]
        ad = random_adapter([("0", d_in, d_out)], rank=rank, seed=d_in)
        layer.load_indices(torch.from_numpy(ad.indices["0"]["A"].astype(np.int64)),
                           torch.from_numpy(ad.indices["0"]["B"].astype(np.int64)))
        assert layer.fused == (d_in % 64 == 0)
        a, bm = (torch.from_numpy(f) for f in oracle_factors(ad)["0"])
        fa, fb = layer.decoded_factors()
        assert torch.equal(fa.cpu(), a) and torch.equal(fb.cpu(), bm)
        x = torch.randn(2, 40, d_in, device="cuda").bfloat16()
        if not layer.fused:
            with torch.no_grad(), pytest.raises(ValueError):
                net(x)
            continue
        with torch.no_grad():
            y = net(x).float()
        truth = torch.nn.functional.linear(x.float(), base.weight.float(), base.bias.float()) + \
            (x.float() @ a.cuda().T @ bm.cuda().T) * 2.0
        assert rel_fro(y, truth) < REL_FRO
        with torch.no_grad(), pytest.raises(TypeError):
            net(x.float())            # fp32 activations: not a kernel dtype


@pytest.mark.parametrize("d_in,d_out", FLUX_SHAPES)
def test_flux_shapes_full_batch(d_in, d_out):
    """Config-2 shapes at full size (B=14, M=4608, 14 adapters of a resident bank): sampled
    rows against the fp32 truth, and the exact doubling property over the whole output."""
    torch.manual_seed(0)
    B, M, r = 14, 4608, 16
    layout_mods = [{"name": "l", "shape_a": [r, d_in], "shape_b": [d_out, r]}]
    from lithe_b200.kernels.packed import PackedLayout
    bank = PackedBank(PackedLayout.from_modules(layout_mods), 40, "cuda")
    bank.fill_random(seed=d_in * 7 + d_out)
    slots = torch.randperm(40, generator=torch.Generator().manual_seed(1))[:B].tolist()
    ids = torch.tensor(slots, dtype=torch.int32, device="cuda")
    x = torch.randn(B, M, d_in, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(B, M, d_out, device="cuda", dtype=torch.bfloat16)
    va, vb = bank.views("l")
    _launch.sgmv_index_(x, out, accumulate=True, view_a=va, view_b=vb, n_slots=40, ids=ids, weights=None, rank=r,
                        lut=bank.lut, scaling=1.0)
    # exact: doubling the input doubles the (accumulated-into-zero) output
    out2 = torch.zeros_like(out)
    _launch.sgmv_index_(x * 2, out2, accumulate=True, view_a=va, view_b=vb, n_slots=40, ids=ids, weights=None,
                        rank=r, lut=bank.lut, scaling=1.0)
    assert torch.equal(out2, out * 2)
    words = bank.words.cpu().numpy().view(np.uint64)
    pa, pb = oracle_pools()
    lay = decode_ref.layout(layout_mods)
    rows = [0, 63, 64, 2047, M - 1]
    for b in (0, 7, 13):
        flat = decode_ref.unpack9(words[slots[b]], lay.num_indices)
        blocks = decode_ref.decode_stream(flat, lay, pa, pb)
        a, bm = decode_ref.split(blocks, lay)["l"]
        xr = x[b, rows].float().cpu()
        want = xr @ torch.from_numpy(a).T @ torch.from_numpy(bm).T
        got = out[b, rows].float().cpu()
        assert max_abs_rel(got, want) <= MAX_ABS_REL and rel_fro(got, want) < REL_FRO, b
    assert device_errors() == 0


@pytest.mark.parametrize("seq,d_in,d_out,r", [(130, 1024, 4096, 16), (77, 512, 640, 8), (1, 256, 384, 4),
                                              (33, 256, 128, 1), (64, 4096, 1024, 16)])
@pytest.mark.parametrize("fmt", ["packed", "i16"])
def test_staged_and_fused_modes_are_bit_identical(seq, d_in, d_out, r, fmt):
    """lithe_sgmv_index_ws (decode once into a workspace) == lithe_sgmv_index (decode per tile)."""
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=s + 20) for s in range(3)]
    x = torch.randn(5, seq, d_in, generator=torch.Generator().manual_seed(seq)).bfloat16().cuda()
    base = (torch.randn(5, seq, d_out, generator=torch.Generator().manual_seed(d_out)) * 0.1).bfloat16().cuda()
    assign = [2, -1, 0, 1, 2]
    for acc in (False, True):
        a = run_fused(x, ads, assign, fmt, accumulate=acc, out=base.clone() if acc else None, weights=[1.0, 1.0, 0.5, 2.0, 1.0],
                      scaling=0.75, mode="staged")
        b = run_fused(x, ads, assign, fmt, accumulate=acc, out=base.clone() if acc else None, weights=[1.0, 1.0, 0.5, 2.0, 1.0],
                      scaling=0.75, mode="fused")
        assert torch.equal(a, b)
    assert device_errors() == 0


def test_staged_mode_workspace_checks():
    ads = [random_adapter([("l", 256, 256)], rank=16, seed=1)]
    x = torch.randn(2, 8, 256, dtype=torch.bfloat16, device="cuda")
    need = _launch.workspace_bytes(2, 256, 256)
    assert need == 2 * (4 + 4) * 512
    small = torch.empty(need - 512, dtype=torch.uint8, device="cuda")
    va, vb, keep = _banks(ads, "packed")
    out = torch.empty(2, 8, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(2, dtype=torch.int32, device="cuda")
    from lithe_b200 import _lib
    import ctypes
    rc = _lib.lib().lithe_sgmv_index_ws(x.data_ptr(), out.data_ptr(), 0, ctypes.byref(va), ctypes.byref(vb), 1,
                                        ids.data_ptr(), None, 2, 8, 256, 256, 16, _launch.lut_array(cb.kernel_lut(*cb.twin_pools())),
                                        1.0, None, small.data_ptr(), small.numel(), None)
    assert rc == _lib.ERR_ARG and b"workspace" in _lib.lib().lithe_last_error()


# m <= 8 token rows per sample run the small-m form (output columns split over CTAs, h formed
# per CTA); the same tolerance and exact properties as the tensor-core form.
SMALL_CASES = [(1, 3072, 18432, 16), (1, 3072, 9216, 16), (1, 256, 384, 4), (2, 512, 640, 8), (3, 192, 256, 2),
               (5, 256, 128, 1), (8, 1024, 4096, 16), (7, 15360, 3072, 16)]


@pytest.mark.parametrize("seq,d_in,d_out,r", SMALL_CASES)
@pytest.mark.parametrize("fmt", ["packed", "i16", "i32"])
def test_small_m_form_matches_truth(seq, d_in, d_out, r, fmt):
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=s + 40) for s in range(3)]
    x = (torch.randn(14, seq, d_in, generator=torch.Generator().manual_seed(seq * 7 + d_in)) * 0.5).bfloat16().cuda()
    assign = [i % 3 for i in range(14)]
    got = run_fused(x, ads, assign, fmt).float().cpu()
    want = truth_delta(x, ads, assign)
    assert max_abs_rel(got, want) <= MAX_ABS_REL and rel_fro(got, want) < REL_FRO
    assert device_errors() == 0


def test_small_m_routing_accumulate_and_exact_properties():
    ads = [random_adapter([("l", 512, 768)], rank=16, seed=s + 50) for s in range(2)]
    x = torch.randn(6, 3, 512, generator=torch.Generator().manual_seed(51)).bfloat16().cuda()
    base = (torch.randn(6, 3, 768, generator=torch.Generator().manual_seed(52)) * 0.05).bfloat16().cuda()
    assign = [0, -1, 5, 1, 1, 0]
    weights = [1.0, 1.0, 1.0, 0.5, 0.0, 2.0]
    device_errors()
    acc = run_fused(x, ads, assign, accumulate=True, out=base.clone(), weights=weights, scaling=0.75)
    assert device_errors() == 1                                    # slot 5 >= n_slots reported
    for b in (1, 2, 4):                                            # unrouted, invalid, weight 0: untouched
        assert torch.equal(acc[b], base[b])
    routed = [0, -1, -1, 1, 1, 0]
    truth = truth_delta(x, ads, routed, weights=weights, scaling=0.75)
    want = base.float().cpu() + truth
    tol = 2 ** -8 * want.abs() + MAX_ABS_REL * truth.abs().max()
    assert bool(((acc.float().cpu() - want).abs() <= tol).all())
    delta = run_fused(x, ads, assign, weights=weights, scaling=0.75)
    device_errors()
    assert bool((delta[1] == 0).all()) and bool((delta[2] == 0).all()) and bool((delta[4] == 0).all())
    assert max_abs_rel(delta.float().cpu(), truth) <= MAX_ABS_REL
    # exact: doubling, batch independence, index formats, staged == fused
    d1 = run_fused(x, ads, routed)
    assert torch.equal(run_fused(x * 2, ads, routed), d1 * 2)
    assert torch.equal(run_fused(x[3:4].contiguous(), ads, [routed[3]])[0], d1[3])
    assert torch.equal(run_fused(x, ads, routed, fmt="i16"), d1)
    assert torch.equal(run_fused(x, ads, routed, mode="staged"), d1)
    assert device_errors() == 0


def test_small_m_layers_and_serve():
    """One decode token per request through IndexLoRALinear-style packed layers and the router."""
    ads = [random_adapter([("l", 1024, 3072)], rank=16, seed=s + 60) for s in range(4)]
    bank = PackedBank.from_adapters(ads, "cuda")
    base = torch.nn.Linear(1024, 3072).cuda().bfloat16()
    layer = PackedLoRALinear(base, bank, "l", 16, 1.0)
    layer.assign = torch.tensor([3, 1, 0, 2, 1], dtype=torch.int32, device="cuda")
    x = torch.randn(5, 1024, generator=torch.Generator().manual_seed(61)).bfloat16().cuda()   # (batch, d_in)
    with torch.no_grad():
        y = layer(x).float().cpu()
    truth = truth_delta(x.unsqueeze(1), ads, [3, 1, 0, 2, 1])[:, 0]
    want = x.float().cpu() @ base.weight.float().cpu().T + base.bias.float().cpu() + truth
    assert max_abs_rel(y, want) <= MAX_ABS_REL
    assert device_errors() == 0
