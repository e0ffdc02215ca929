"""A random-init transformer with the shapes and module paths of FLUX.1-dev
(diffusers ``FluxTransformer2DModel``), for timing the index-resident LoRA path in a full
denoise loop.  FLUX weights and diffusers are not available here, so this is a plain PyTorch
restatement of the architecture's dimensions, not a port of diffusers' code:

  19 double-stream blocks  image + text streams, AdaLN-zero modulation, joint attention,
                           GELU(tanh) feed-forward per stream
  38 single-stream blocks  one stream over [text; image] tokens, attention and an MLP branch
                           in parallel, one output projection
  hidden 3072, 24 heads of 128, FFN 12288, latent channels 64, text features 4096

The attention + FFN linears carry the diffusers names that FLUX LoRA adapters target
(``module.FLUX_TARGET_MODULES``; 19 x 12 + 38 x 3 = 342 linears).  Attention applies FLUX's
rotary position embedding: three axes (an index axis, image row, image column) over head-dim
slices of 16, 56 and 56 (scaled with the head size), theta 10000, text tokens at position 0 of
every axis and image tokens on a near-square grid.  Weights are N(0, 0.02); outputs are
meaningless, only shapes and costs are real.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn


@dataclass
class FluxConfig:
    hidden: int = 3072
    heads: int = 24
    mlp_ratio: int = 4
    double_blocks: int = 19
    single_blocks: int = 38
    in_channels: int = 64
    text_dim: int = 4096
    pooled_dim: int = 768
    time_dim: int = 256

    @classmethod
    def tiny(cls) -> "FluxConfig":
        return cls(hidden=256, heads=2, double_blocks=2, single_blocks=2, in_channels=16, text_dim=64, pooled_dim=32,
                   time_dim=32)


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


class RMSNorm(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return _rms(x, self.weight)


class GELUProj(nn.Module):
    """``ff.net.0``: a linear followed by tanh-approximate GELU (diffusers GELU(approximate='tanh'))."""

    def __init__(self, dim: int, inner: int):
        super().__init__()
        self.proj = nn.Linear(dim, inner)

    def forward(self, x):
        return F.gelu(self.proj(x), approximate="tanh")


class FeedForward(nn.Module):
    def __init__(self, dim: int, inner: int):
        super().__init__()
        self.net = nn.ModuleList([GELUProj(dim, inner), nn.Identity(), nn.Linear(inner, dim)])

    def forward(self, x):
        for m in self.net:
            x = m(x)
        return x


class AdaNorm(nn.Module):
    """AdaLN modulation: ``linear`` maps the conditioning vector to n_mod shift/scale/gate vectors."""

    def __init__(self, dim: int, n_mod: int):
        super().__init__()
        self.linear = nn.Linear(dim, n_mod * dim)
        self.n_mod = n_mod

    def forward(self, temb):
        return self.linear(F.silu(temb)).chunk(self.n_mod, dim=-1)


def _ln(x):
    return F.layer_norm(x, x.shape[-1:], eps=1e-6)


def _mod(x, shift, scale):
    return x * (1 + scale[:, None]) + shift[:, None]


def rope_tables(n_txt: int, n_img: int, head_dim: int, device, theta: float = 10000.0):
    """(cos, sin), each (n_txt + n_img, head_dim / 2) fp32, for the joint [text; image] sequence.

    Positions are 3-axis ids (index, row, col): text tokens sit at (0, 0, 0), image token i at
    (0, i // w, i % w) on a grid of width w = ceil(sqrt(n_img)).  Each axis owns a slice of the
    head's rotation pairs (16 / 56 / 56 of 128 dims), with frequencies theta^(-2j / axis_dim).
    """
    axes = (head_dim // 8, 7 * head_dim // 16, head_dim - head_dim // 8 - 7 * head_dim // 16)
    w = max(1, math.ceil(math.sqrt(n_img)))
    idx = torch.arange(n_img, device=device)
    ids = torch.zeros(n_txt + n_img, 3, device=device, dtype=torch.float32)
    ids[n_txt:, 1] = (idx // w).float()
    ids[n_txt:, 2] = (idx % w).float()
    angles = []
    for axis, dim in enumerate(axes):
        freqs = theta ** (-torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim)
        angles.append(ids[:, axis:axis + 1] * freqs[None])
    ang = torch.cat(angles, dim=-1)
    return torch.cos(ang), torch.sin(ang)


def rope_full(cos, sin, dtype):
    """The half-dim tables of ``rope_tables`` spread over the whole head dim in the activation
    dtype: each angle's cos for both members of its pair, and its sin signed (-sin for the
    pair's first member, +sin for the second), so that a rotation is one fused multiply-add."""
    cos_f = cos.repeat_interleave(2, dim=-1)
    sin_f = torch.stack([-sin, sin], dim=-1).flatten(-2)
    return cos_f.to(dtype), sin_f.to(dtype)


def _rotate(t, cos_f, sin_f):
    """Rotate consecutive pairs (t[2j], t[2j+1]) of the last dim by the per-token angles:
    (x0, x1) -> (x0 cos - x1 sin, x1 cos + x0 sin).  t is (b, heads, s, hd); cos_f / sin_f are
    the (s, hd) tables of ``rope_full``.  Three elementwise passes: the pair swap, t * cos, and
    the multiply-add."""
    swapped = t.unflatten(-1, (-1, 2)).flip(-1).flatten(-2)
    return torch.addcmul(t * cos_f, swapped, sin_f)


def _attend(q, k, v, heads, rope=None):
    b, s, d = q.shape
    hd = d // heads
    q, k, v = (t.view(b, s, heads, hd).transpose(1, 2) for t in (q, k, v))
    if rope is not None:
        q, k = _rotate(q, *rope), _rotate(k, *rope)
    o = F.scaled_dot_product_attention(q, k, v)
    return o.transpose(1, 2).reshape(b, s, d)


class JointAttention(nn.Module):
    def __init__(self, dim: int, heads: int, context: bool):
        super().__init__()
        self.heads = heads
        hd = dim // heads
        self.to_q, self.to_k, self.to_v = nn.Linear(dim, dim), nn.Linear(dim, dim), nn.Linear(dim, dim)
        self.norm_q, self.norm_k = RMSNorm(hd), RMSNorm(hd)
        if context:
            self.add_q_proj, self.add_k_proj, self.add_v_proj = nn.Linear(dim, dim), nn.Linear(dim, dim), nn.Linear(dim, dim)
            self.norm_added_q, self.norm_added_k = RMSNorm(hd), RMSNorm(hd)
            self.to_out = nn.ModuleList([nn.Linear(dim, dim)])
            self.to_add_out = nn.Linear(dim, dim)

    def _qkv(self, x, q, k, v, nq, nk):
        b, s, d = x.shape
        hd = d // self.heads
        qq = nq(q(x).view(b, s, self.heads, hd)).view(b, s, d)
        kk = nk(k(x).view(b, s, self.heads, hd)).view(b, s, d)
        return qq, kk, v(x)


class DoubleBlock(nn.Module):
    def __init__(self, cfg: FluxConfig):
        super().__init__()
        d = cfg.hidden
        self.norm1, self.norm1_context = AdaNorm(d, 6), AdaNorm(d, 6)
        self.attn = JointAttention(d, cfg.heads, context=True)
        self.ff = FeedForward(d, d * cfg.mlp_ratio)
        self.ff_context = FeedForward(d, d * cfg.mlp_ratio)

    def forward(self, img, txt, temb, rope=None):
        sh, sc, g, sh2, sc2, g2 = self.norm1(temb)
        csh, csc, cg, csh2, csc2, cg2 = self.norm1_context(temb)
        a = self.attn
        xi = _mod(_ln(img), sh, sc)
        xt = _mod(_ln(txt), csh, csc)
        qi, ki, vi = a._qkv(xi, a.to_q, a.to_k, a.to_v, a.norm_q, a.norm_k)
        qt, kt, vt = a._qkv(xt, a.add_q_proj, a.add_k_proj, a.add_v_proj, a.norm_added_q, a.norm_added_k)
        o = _attend(torch.cat([qt, qi], 1), torch.cat([kt, ki], 1), torch.cat([vt, vi], 1), a.heads, rope)
        ot, oi = o[:, : txt.shape[1]], o[:, txt.shape[1]:]
        img = img + g[:, None] * a.to_out[0](oi.contiguous())
        txt = txt + cg[:, None] * a.to_add_out(ot.contiguous())
        img = img + g2[:, None] * self.ff(_mod(_ln(img), sh2, sc2))
        txt = txt + cg2[:, None] * self.ff_context(_mod(_ln(txt), csh2, csc2))
        return img, txt


class SingleBlock(nn.Module):
    def __init__(self, cfg: FluxConfig):
        super().__init__()
        d = cfg.hidden
        self.norm = AdaNorm(d, 3)
        self.attn = JointAttention(d, cfg.heads, context=False)
        self.proj_mlp = nn.Linear(d, d * cfg.mlp_ratio)
        self.proj_out = nn.Linear(d + d * cfg.mlp_ratio, d)

    def forward(self, x, temb, rope=None):
        sh, sc, g = self.norm(temb)
        h = _mod(_ln(x), sh, sc)
        a = self.attn
        q, k, v = a._qkv(h, a.to_q, a.to_k, a.to_v, a.norm_q, a.norm_k)
        o = _attend(q, k, v, a.heads, rope)
        mlp = F.gelu(self.proj_mlp(h), approximate="tanh")
        return x + g[:, None] * self.proj_out(torch.cat([o, mlp], dim=-1))


class FluxShapedTransformer(nn.Module):
    def __init__(self, cfg: FluxConfig = FluxConfig()):
        super().__init__()
        self.cfg = cfg
        d = cfg.hidden
        self.x_embedder = nn.Linear(cfg.in_channels, d)
        self.context_embedder = nn.Linear(cfg.text_dim, d)
        self.time_in = nn.Sequential(nn.Linear(cfg.time_dim, d), nn.SiLU(), nn.Linear(d, d))
        self.pooled_in = nn.Sequential(nn.Linear(cfg.pooled_dim, d), nn.SiLU(), nn.Linear(d, d))
        self.transformer_blocks = nn.ModuleList([DoubleBlock(cfg) for _ in range(cfg.double_blocks)])
        self.single_transformer_blocks = nn.ModuleList([SingleBlock(cfg) for _ in range(cfg.single_blocks)])
        self.norm_out = AdaNorm(d, 2)
        self.proj_out = nn.Linear(d, cfg.in_channels)
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, std=0.02)
                nn.init.zeros_(m.bias)

    def timestep_embedding(self, t: torch.Tensor) -> torch.Tensor:
        half = self.cfg.time_dim // 2
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        args = t.float()[:, None] * 1000.0 * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)

    def forward(self, latents, text, pooled, t):
        dtype = self.x_embedder.weight.dtype
        temb = self.time_in(self.timestep_embedding(t).to(dtype)) + self.pooled_in(pooled)
        img = self.x_embedder(latents)
        txt = self.context_embedder(text)
        rope = rope_full(*rope_tables(txt.shape[1], img.shape[1], self.cfg.hidden // self.cfg.heads, img.device),
                         img.dtype)
        for blk in self.transformer_blocks:
            img, txt = blk(img, txt, temb, rope)
        x = torch.cat([txt, img], dim=1)
        for blk in self.single_transformer_blocks:
            x = blk(x, temb, rope)
        img = x[:, txt.shape[1]:]
        sh, sc = self.norm_out(temb)
        return self.proj_out(_mod(_ln(img), sh, sc))


def denoise(model: FluxShapedTransformer, latents, text, pooled, steps: int) -> torch.Tensor:
    """Flow-matching Euler loop: ``steps`` forwards from t = 1 to 0."""
    x = latents
    for i in range(steps):
        t = torch.full((x.shape[0],), 1.0 - i / steps, device=x.device)
        v = model(x, text, pooled, t)
        x = x - v / steps
    return x


def lora_targets(model: nn.Module):
    """(path, linear) of the 342 attention + FFN linears LoRA adapters target."""
    from . import _modtree
    from .module import FLUX_TARGET_MODULES
    return list(_modtree.linears_matching(model, FLUX_TARGET_MODULES))
