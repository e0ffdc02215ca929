"""lithe_lora_gemm (tcgen05 GEMM with the LoRA expand fused into the accumulator) against a
torch fp32 reference of the same op: out = x W^T + bias + h Bdec_sample^T, rounded to bf16.
Tolerance (bf16 inputs, fp32 accumulation in a different order, one bf16 rounding of the
output): max |got - ref| <= 1e-2 * max |ref| and relative Frobenius error < 5e-3."""
import numpy as np
import pytest
import torch

from lithe_b200 import device_errors, kohya, serve
from lithe_b200.fileio import LitheAdapter
from lithe_b200.kernels import PackedBank, PackedLoRALinear, _launch
from oracle import decode_ref
from tests.helpers import max_abs_rel, oracle_factors, oracle_pools, random_adapter, rel_fro

pytestmark = pytest.mark.gpu


def reference(x, w, bias, h=None, bd=None, rps=None):
    ref = x.float() @ w.float().T
    if bias is not None:
        ref += bias.float()
    if h is not None:
        samples = x.shape[0] // rps
        hs = h.float().view(samples, rps, -1)
        ref += torch.bmm(hs, bd.float().transpose(1, 2)).reshape(x.shape[0], -1)
    return ref


def check(got, ref):
    err = (got.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err
    assert rel_fro(got.float().cpu(), ref.cpu()) < 5e-3


@pytest.mark.parametrize("rows,n,k,bias", [(128, 256, 64, True), (300, 512, 192, False), (1000, 768, 1024, True),
                                           (4096, 3072, 3072, True), (2048, 12288, 3072, True),
                                           (2048, 3072, 12288, False)])
def test_plain_gemm(rows, n, k, bias):
    g = torch.Generator(device="cuda").manual_seed(rows + n + k)
    x = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    b = torch.randn(n, generator=g, device="cuda").bfloat16() if bias else None
    out = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    _launch.lora_gemm_(x, w, b, out)
    torch.cuda.synchronize()
    check(out, reference(x, w, b))
    assert device_errors() == 0


@pytest.mark.parametrize("samples,rps,n,k", [(1, 128, 256, 64), (3, 256, 512, 320), (14, 512, 3072, 3072),
                                             (4, 1024, 12288, 3072)])
def test_fused_expand(samples, rps, n, k):
    g = torch.Generator(device="cuda").manual_seed(samples * rps + n)
    rows = samples * rps
    x = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    b = torch.randn(n, generator=g, device="cuda").bfloat16()
    h = torch.randn(rows, 16, generator=g, device="cuda").bfloat16()
    bd = (torch.randn(samples, n, 16, generator=g, device="cuda") * 0.1).bfloat16()
    out = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
    _launch.lora_gemm_(x, w, b, out, h=h, b_dec=bd, rows_per_sample=rps)
    torch.cuda.synchronize()
    ref = reference(x, w, b, h, bd, rps)
    check(out, ref)
    # the expand really is per sample: zero one sample's factor and only its rows change
    bd2 = bd.clone()
    bd2[samples - 1] = 0
    out2 = torch.empty_like(out)
    _launch.lora_gemm_(x, w, b, out2, h=h, b_dec=bd2, rows_per_sample=rps)
    torch.cuda.synchronize()
    assert torch.equal(out2[: (samples - 1) * rps], out[: (samples - 1) * rps])
    check(out2, reference(x, w, b, h, bd2, rps))
    assert device_errors() == 0


def test_unsupported_shapes_are_rejected():
    x = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(200, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NotImplementedError):
        _launch.lora_gemm_(x, w, None, torch.empty(128, 200, dtype=torch.bfloat16, device="cuda"))
    w = torch.zeros(256, 64, dtype=torch.bfloat16, device="cuda")
    h = torch.zeros(128, 16, dtype=torch.bfloat16, device="cuda")
    bd = torch.zeros(2, 256, 16, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(NotImplementedError):        # 64 rows per sample: not a multiple of 128
        _launch.lora_gemm_(x, w, None, torch.empty(128, 256, dtype=torch.bfloat16, device="cuda"), h=h, b_dec=bd,
                           rows_per_sample=64)


# ------------------------------------------------------------------ prep + the fused layer path


def _prep(bank, name, x, ids, weights, scaling, rows=None):
    va, vb = bank.views(name, rows)
    i = bank.layout.index(name)
    d_out = bank.layout.shapes_b[i][0] if rows is None else rows[1] - rows[0]
    h = torch.full((x.shape[0] * x.shape[1], 16), 7.0, dtype=torch.bfloat16, device="cuda")
    bd = torch.full((x.shape[0], d_out, 16), 7.0, dtype=torch.bfloat16, device="cuda")
    _launch.lora_prep_(x, view_a=va, view_b=vb, n_slots=bank.n_slots, ids=ids, weights=weights, d_out=d_out,
                       lut=bank.lut, scaling=scaling, h=h, b_dec=bd)
    torch.cuda.synchronize()
    return h, bd


def test_prep_matches_oracle():
    d_in, d_out = 512, 768
    ads = [random_adapter([("l", d_in, d_out)], rank=16, seed=s) for s in range(3)]
    bank = PackedBank.from_adapters(ads, "cuda")
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, 200, d_in, generator=g).bfloat16().cuda()
    assign, wts, sc = [2, -1, 0, 1], [1.0, 1.0, 0.5, 2.0], 0.75
    ids = torch.tensor(assign, dtype=torch.int32, device="cuda")
    h, bd = _prep(bank, "l", x, ids, torch.tensor(wts, device="cuda"), sc)
    facs = [oracle_factors(a)["l"] for a in ads]
    hv = h.view(4, 200, 16)
    for b, j in enumerate(assign):
        if j < 0:
            assert not hv[b].any() and not bd[b].any()
            continue
        a_f, b_f = (torch.from_numpy(f) for f in facs[j])
        assert torch.equal(bd[b].cpu(), b_f.bfloat16())                 # bit-exact decode
        want = wts[b] * sc * (x[b].float().cpu() @ a_f.T)
        assert max_abs_rel(hv[b].float().cpu(), want) <= 2e-2 and rel_fro(hv[b].float().cpu(), want) < 1e-2
    assert device_errors() == 0


@pytest.mark.parametrize("m", [256, 128, 512])
def test_fused_gemm_layer_matches_truth_and_default_path(m):
    d_in, d_out = 1024, 768
    ads = [random_adapter([("l", d_in, d_out)], rank=16, seed=s) for s in range(4)]
    bank = PackedBank.from_adapters(ads, "cuda")
    torch.manual_seed(0)
    base = torch.nn.Linear(d_in, d_out).cuda().bfloat16()
    layer = PackedLoRALinear(base, bank, "l", 16, 0.5)
    assign = [3, 0, -1, 2]
    layer.assign = torch.tensor(assign, dtype=torch.int32, device="cuda")
    x = torch.randn(4, m, d_in, generator=torch.Generator().manual_seed(m)).bfloat16().cuda()
    with torch.no_grad():
        y0 = layer(x)
        layer.fused_gemm = True
        y1 = layer(x)
    facs = [oracle_factors(a)["l"] for a in ads]
    ref = x.float() @ base.weight.float().T + base.bias.float()
    for b, j in enumerate(assign):
        if j >= 0:
            a_f, b_f = (torch.from_numpy(f).cuda() for f in facs[j])
            ref[b] += 0.5 * (x[b].float() @ a_f.T) @ b_f.T
    for y in (y0, y1):
        check(y.view(-1, d_out), ref.view(-1, d_out))
    with torch.no_grad():                                   # the unrouted sample sees the base linear only
        check(y1[2], x[2].float() @ base.weight.float().T + base.bias.float())
    assert device_errors() == 0


def test_fused_gemm_layer_serves_a_kohya_row_range():
    mods = kohya.kohya_flux_modules(rank=16, double_blocks=1, single_blocks=1, hidden=256, mlp_ratio=4)
    ads = []
    for s in range(2):
        rng = np.random.default_rng(s)
        idx = {mm["name"]: {"A": rng.integers(0, 512, (3, mm["shape_a"][0] * mm["shape_a"][1] // 64)).astype(np.uint16),
                            "B": rng.integers(0, 512, (3, mm["shape_b"][0] * mm["shape_b"][1] // 64)).astype(np.uint16)}
               for mm in mods}
        ads.append(LitheAdapter(modules=mods, indices=idx, rank=16, alpha=16.0, key_format="kohya"))
    bank = PackedBank.from_adapters(ads, "cuda")
    name, rows = "lora_unet_double_blocks_0_img_attn_qkv", (256, 512)        # to_k
    base = torch.nn.Linear(256, 256).cuda().bfloat16()
    layer = PackedLoRALinear(base, bank, name, 16, 1.0, rows=rows)
    layer.assign = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    x = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(9)).bfloat16().cuda()
    with torch.no_grad():
        y0 = layer(x)
        layer.fused_gemm = True
        y1 = layer(x)
    ref = x.float() @ base.weight.float().T + base.bias.float()
    for b, j in enumerate([1, 0]):
        ia, ib, sa, sb = kohya.split_indices(ads[j])["transformer_blocks.0.attn.to_k"]
        pa, pb = oracle_pools()
        a_f = torch.from_numpy(decode_ref.decode_factor(ia, sa, pa)).cuda()
        b_f = torch.from_numpy(decode_ref.decode_factor(ib, sb, pb)).cuda()
        ref[b] += (x[b].float() @ a_f.T) @ b_f.T
    check(y0.view(-1, 256), ref.view(-1, 256))
    check(y1.view(-1, 256), ref.view(-1, 256))
    assert device_errors() == 0


def test_serve_attach_adapters_fused_gemm_path():
    """serve.attach_adapters(fused_gemm=True): single-adapter routes (with gains and an empty
    route) take the expand-in-GEMM path and agree with the default path and the fp32 truth;
    a mixture route falls back to the default path bit for bit."""

    class Toy(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.up = torch.nn.Linear(512, 768)
            self.down = torch.nn.Linear(768, 512)

        def forward(self, x):
            return self.down(torch.nn.functional.gelu(self.up(x)))

    ads = [random_adapter([("up", 512, 768), ("down", 768, 512)], rank=16, seed=s) for s in range(3)]
    torch.manual_seed(3)
    base = Toy().cuda().bfloat16()
    state = {k: v.clone() for k, v in base.state_dict().items()}
    x = torch.randn(3, 256, 512, generator=torch.Generator().manual_seed(4)).bfloat16().cuda()
    routes = [[(0, 1.0)], [(2, 0.5)], []]
    outs = {}
    for fused in (False, True):
        model = Toy().cuda().bfloat16()
        model.load_state_dict(state)
        router, layers = serve.attach_adapters(model, ads, fused_gemm=fused)
        router.set(routes)
        with torch.no_grad():
            outs[fused] = model(x).float()
            if fused:
                router.set([[(0, 0.6), (1, 0.4)], [(2, 1.0)], []])          # mixture: two columns
                mix_fused = model(x)
                for layer in layers.values():
                    layer.fused_gemm = False
                mix_default = model(x)
                assert torch.equal(mix_fused, mix_default)
    # fp32 truth of the two-layer model with the routed deltas on both layers
    facs = [oracle_factors(a) for a in ads]

    def layer_truth(inp, lin, name, route):
        y = inp @ lin.weight.float().T + lin.bias.float()
        for j, wj in route:
            a_f, b_f = (torch.from_numpy(f).cuda() for f in facs[j][name])
            y = y + wj * (inp @ a_f.T) @ b_f.T
        return y

    truth = []
    with torch.no_grad():
        for b, route in enumerate(routes):
            z = torch.nn.functional.gelu(layer_truth(x[b].float(), base.up, "up", route).bfloat16().float())
            truth.append(layer_truth(z.bfloat16().float(), base.down, "down", route))
    truth = torch.stack(truth)
    for fused in (False, True):
        assert rel_fro(outs[fused].cpu(), truth.cpu()) < 2e-2, fused
    assert rel_fro(outs[True].cpu(), outs[False].cpu()) < 2e-2
    assert device_errors() == 0


def test_kohya_split_targets_share_h():
    """q, k, v of one fused Kohya module share A: called with the same input, the fused-GEMM path
    computes h once (the first call) and the others reuse it, with bit-identical outputs; an
    in-place change of the input invalidates the shared h."""
    mods = kohya.kohya_flux_modules(rank=16, double_blocks=1, single_blocks=1, hidden=256, mlp_ratio=4)
    ads = [random_adapter([(m["name"], m["shape_a"][1], m["shape_b"][0]) for m in mods], rank=16, seed=s)
           for s in range(2)]
    for ad in ads:
        ad.key_format = "kohya"
    name = "lora_unet_double_blocks_0_img_attn_qkv"
    torch.manual_seed(5)
    bases = [torch.nn.Linear(256, 256).cuda().bfloat16() for _ in range(3)]
    ids = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    x = torch.randn(2, 256, 256, generator=torch.Generator().manual_seed(6)).bfloat16().cuda()

    def run(bank):
        layers = [PackedLoRALinear(bases[i], bank, name, 16, 1.0, rows=(256 * i, 256 * (i + 1)), fused_gemm=True)
                  for i in range(3)]
        for layer in layers:
            layer.assign = ids
        with torch.no_grad():
            return [layer(x) for layer in layers], layers

    shared_bank = PackedBank.from_adapters(ads, "cuda")
    outs_shared, layers = run(shared_bank)
    assert set(shared_bank._shared_h) == {name}
    h0 = shared_bank._shared_h[name][1]
    assert layers[1]._shared_h(x, ids, None) is h0 and layers[2]._shared_h(x, ids, None) is h0
    # the same three calls, each computing its own h (no sibling to share with)
    separate = []
    for i in range(3):
        bank = PackedBank.from_adapters(ads, "cuda")
        layer = PackedLoRALinear(bases[i], bank, name, 16, 1.0, rows=(256 * i, 256 * (i + 1)), fused_gemm=True)
        layer.assign = ids
        with torch.no_grad():
            separate.append(layer(x))
    for a, b in zip(outs_shared, separate):
        assert torch.equal(a, b)
    # an in-place change of x must not reuse the stale h
    with torch.no_grad():
        x.mul_(0.5)
        y = layers[1](x)
    assert shared_bank._shared_h[name][1] is not h0
    # everything but the bias is linear in x: y(x / 2) = (y(x) - b) / 2 + b
    check(y.view(-1, 256), (0.5 * outs_shared[1].float()).view(-1, 256) + 0.5 * bases[1].bias.float())
    assert device_errors() == 0
