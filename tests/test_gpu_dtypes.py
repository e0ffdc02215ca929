"""fp16 activations and ``out_dtype`` (lithe_sgmv_index_typed), against the oracle.

The reference's shared_codebook_lora_delta takes any activation dtype: pools cast to x.dtype,
the factors and x.A^T rounded to it, the delta in out_dtype (default x.dtype)
(lithe/kernels/shared.py:177-194,210-218).  The kernel computes in fp16 with fp16 MMAs when x
is fp16, and writes the delta alone as fp32 when out_dtype is float32.

Tolerance as the bf16 SGMV tests: max-abs-rel <= 2e-2 and relative Frobenius error < 1e-2 on
the LoRA delta, against the fp32 truth and against the oracle's dtype-step restatement of the
reference (oracle/sgmv_ref.shared_delta); the doubling property is checked bit for bit on
all but the rare rows where fp16's narrow exponent range forces an absolute rounding step."""
import numpy as np
import pytest
import torch

from lithe_b200 import codebook as cb
from lithe_b200 import device_errors
from lithe_b200.kernels import PackedBank, PackedLoRALinear, _launch, shared_codebook_lora_delta
from oracle import sgmv_ref
from tests.helpers import FLUX_SHAPES, max_abs_rel, oracle_factors, oracle_pools, random_adapter, rel_fro

pytestmark = pytest.mark.gpu

MAX_ABS_REL = 2e-2
REL_FRO = 1e-2


def _truth(x, ads, assign, name="l"):
    facs = [oracle_factors(a)[name] for a in ads]
    xs = x.float().cpu()
    return torch.stack([xs[b] @ torch.from_numpy(facs[j][0]).T @ torch.from_numpy(facs[j][1]).T
                        for b, j in enumerate(assign)])


def _ok(got, want, what):
    got = got.float().cpu()
    e1, e2 = max_abs_rel(got, want), rel_fro(got, want)
    assert e1 <= MAX_ABS_REL and e2 < REL_FRO, f"{what}: max-abs-rel {e1:.2e}, rel-Fro {e2:.2e}"


@pytest.mark.parametrize("d_in,d_out", FLUX_SHAPES)
def test_fp16_flux_shapes_full_batch(d_in, d_out):
    """Config-2 shapes at full size in fp16 (B=14, M=4608, 14 adapters of a resident packed bank):
    sampled rows against the fp32 truth; doubling x doubles the output exactly except in the rare
    rows where a rounding leaves fp16's normal range."""
    torch.manual_seed(0)
    bsz, m, r = 14, 4608, 16
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=100 + s) for s in range(bsz)]
    bank = PackedBank.from_adapters(ads, "cuda")
    ids = torch.arange(bsz, dtype=torch.int32, device="cuda")
    x = torch.randn(bsz, m, d_in, device="cuda", dtype=torch.float16)
    # no subnormal activations (|x| < 2^-14), so x and 2x are both exact normal fp16 values
    x = torch.where(x.abs() < 2.0 ** -13, torch.full_like(x, 2.0 ** -13), x)
    out = torch.zeros(bsz, m, d_out, device="cuda", dtype=torch.float16)
    va, vb = bank.views("l")
    _launch.sgmv_index_(x, out, accumulate=True, view_a=va, view_b=vb, n_slots=bsz, ids=ids, weights=None, rank=r,
                        lut=bank.lut, scaling=1.0)
    out2 = torch.zeros_like(out)
    _launch.sgmv_index_(x * 2, out2, accumulate=True, view_a=va, view_b=vb, n_slots=bsz, ids=ids, weights=None,
                        rank=r, lut=bank.lut, scaling=1.0)
    torch.cuda.synchronize()
    assert device_errors() == 0
    # Doubling x doubles the output exactly wherever every rounding on the way stays in fp16's
    # normal range.  fp16 (unlike bf16) has a narrow exponent range: a token row whose rank-16 h
    # has a component below 2^-14 is rounded in absolute steps there, and its whole output row
    # may then differ in the last bit; such rows are rare (a few in 64,512 here).
    normal = out.abs() >= 2.0 ** -14
    exact = (out2 == out * 2) | ~normal
    assert exact.float().mean() > 0.999
    assert max_abs_rel(out2.float(), out.float() * 2) < 1e-3
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(1))[:48]
    want = _truth(x[:, rows.cuda()], ads, list(range(bsz)))
    _ok(out[:, rows.cuda()], want, f"fp16 {d_in}->{d_out}")


CASES = [(256, 3072, 3072, 16), (77, 512, 640, 8), (64, 192, 256, 4), (33, 256, 128, 1), (5, 1024, 384, 16),
         (1, 256, 512, 2)]


@pytest.mark.parametrize("seq,d_in,d_out,r", CASES)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_shared_delta_dtypes_and_out_dtype(seq, d_in, d_out, r, dtype):
    """shared_codebook_lora_delta in fp16 and bf16, out_dtype x.dtype and float32, against the
    fp32 truth and the oracle's dtype-step restatement of the reference; the float32 delta is the
    one the 16-bit delta rounds (bit-equal after rounding)."""
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=7 * s + d_in) for s in range(3)]
    assign = [2, 0, 1, 2]
    x = torch.randn(len(assign), seq, d_in, generator=torch.Generator().manual_seed(seq)).to(dtype).cuda()
    ia = torch.stack([torch.from_numpy(a.indices["l"]["A"].astype(np.int64)) for a in ads]).cuda()
    ib = torch.stack([torch.from_numpy(a.indices["l"]["B"].astype(np.int64)) for a in ads]).cuda()
    pa, pb = cb.twin_pools()
    ids = torch.tensor(assign, dtype=torch.int32, device="cuda")
    got = shared_codebook_lora_delta(x, ia, pa, ib, pb, ids, r, d_out, 1.0)
    got32 = shared_codebook_lora_delta(x, ia, pa, ib, pb, ids, r, d_out, 1.0, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert got.dtype == dtype and got32.dtype == torch.float32
    truth = _truth(x, ads, assign)
    _ok(got, truth, f"{dtype} delta")
    _ok(got32, truth, f"{dtype} -> fp32 delta")
    opa, opb = oracle_pools()
    ref = sgmv_ref.shared_delta(x.cpu(), ia.cpu().numpy(), opa, ib.cpu().numpy(), opb, assign, r, d_out, 1.0)
    _ok(got, ref.float(), f"{dtype} delta vs the reference's dtype steps")
    assert torch.equal(got32.to(dtype), got)       # the 16-bit delta is the fp32 one, rounded


def test_fp16_layer_and_unsupported_out_dtype():
    """PackedLoRALinear on an fp16 model (the SGMV path; the fused-GEMM path is bf16-only and is
    not taken), and the combinations the kernel does not take raise."""
    torch.manual_seed(3)
    d_in, d_out, r = 512, 768, 16
    ads = [random_adapter([("l", d_in, d_out)], rank=r, seed=40 + s) for s in range(3)]
    bank = PackedBank.from_adapters(ads, "cuda")
    lin = torch.nn.Linear(d_in, d_out).cuda().half()
    torch.nn.init.zeros_(lin.weight)              # a zero base: the layer's output is its LoRA delta
    torch.nn.init.zeros_(lin.bias)
    layer = PackedLoRALinear(lin, bank, "l", r, 1.0, fused_gemm=True)
    layer.assign = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
    x = torch.randn(2, 256, d_in, device="cuda").half()
    assert not layer._gemm_ok(x)
    with torch.no_grad():
        y = layer(x)
    assert y.dtype == torch.float16
    _ok(y, _truth(x, ads, [1, 2]), "fp16 layer delta")
    ia = torch.zeros(1, 3, 16 * d_in // 64, dtype=torch.int32, device="cuda")
    ib = torch.zeros(1, 3, 16 * d_out // 64, dtype=torch.int32, device="cuda")
    pa, pb = cb.twin_pools()
    with pytest.raises(NotImplementedError):
        shared_codebook_lora_delta(x, ia, pa, ib, pb, torch.zeros(2, dtype=torch.int32, device="cuda"), 16, d_out,
                                   1.0, out_dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        shared_codebook_lora_delta(x.float(), ia, pa, ib, pb, torch.zeros(2, dtype=torch.int32, device="cuda"), 16,
                                   d_out, 1.0)
