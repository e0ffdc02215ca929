"""Generate the golden fixtures of tests/golden/ by running the REFERENCE implementation.

Run it with the root of a checkout of the reference package (JianJiang1995/LITHE, the
folder that holds ``lithe/``), given either as the first argument or as LITHE_REF:

    python tests/golden/make_golden.py /path/to/LITHE
    LITHE_REF=/path/to/LITHE python tests/golden/make_golden.py

Every fixture holds seeded inputs and the reference's outputs for them; the tests use the
fixtures to pin the CPU oracle (oracle/) and the CUDA path.  Nothing at test time needs the
reference itself.  Fixtures:

  codebook.npz      integer-table and pool digests, the 10 distinct values of every pool level
  decode_small.npz  a multi-module adapter: its indices, the reference's packed words,
                    quant.decode fp32 factors and decode_packed_reference bf16 blocks
  serve_small.npz   serve.attach_adapters + Router.set + forward (zero base linear, so the
                    output is the routed LoRA delta) in fp32 and bf16, with mixtures and an
                    empty route
  config1_rows.npz  the config-1 workload (3072->3072, r=16, B=4 x 256 tokens, adapters
                    0..3 from seed 0, x ~ N(0,1) seed 0): sampled rows of the fp32 delta and
                    per-sample checksums
  shared_small.npz  shared_codebook_lora_delta_reference (bf16 rounding steps) at the
                    shapes of the reference's GPU test
  small.lithe       a .lithe file written by the reference's save_lithe (+ small_lithe.npz
                    with its indices and header fields)
  kohya_split.npz   lithe.kohya on two Kohya-format adapters (rank 4 at d=64 as in the
                    reference's tests, rank 16 at d=128): diffusers_paths and every
                    split_indices entry; and split_spec over the full Kohya-304 FLUX.1-dev
                    module set (19 double x 10 + 38 single x 3 modules)
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _reference_root() -> str:
    """The reference checkout to import: argv[1], else $LITHE_REF; there is no default."""
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LITHE_REF", "")
    if not ref or not (Path(ref) / "lithe" / "__init__.py").exists():
        raise SystemExit("make_golden.py needs the reference checkout: pass its root as the first argument "
                         "or set LITHE_REF (the folder that contains lithe/__init__.py)")
    return ref


REF = _reference_root()
sys.path.insert(0, REF)

from lithe import codebook as cb  # noqa: E402
from lithe import fileio, kohya, quant, serve  # noqa: E402
from lithe.kernels import packed, shared  # noqa: E402

SMALL = [("blk.0.q", 128, 192), ("blk.0.mlp", 128, 320), ("blk.0.out", 320, 128), ("odd", 96, 40),
         ("wide", 1024, 640)]


def adapter(modules, rank, seed, alpha=None, key_format="diffusers"):
    rng = np.random.default_rng(seed)
    mods, idx = [], {}
    for name, d_in, d_out in modules:
        sa, sb = [rank, d_in], [d_out, rank]
        mods.append({"name": name, "shape_a": sa, "shape_b": sb})
        idx[name] = {"A": rng.integers(0, cb.K, (cb.NUM_LEVELS, quant.num_blocks(sa))).astype(np.uint16),
                     "B": rng.integers(0, cb.K, (cb.NUM_LEVELS, quant.num_blocks(sb))).astype(np.uint16)}
    return fileio.LitheAdapter(modules=mods, indices=idx, rank=rank,
                               alpha=float(rank if alpha is None else alpha), key_format=key_format)


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def make_codebook():
    pa, pb = cb.twin_pools()
    ic = cb.integer_codewords()
    luts = {}
    for side, pool in (("a", pa.numpy()), ("b", pb.numpy())):
        lut = np.zeros((cb.NUM_LEVELS, 10), np.float32)
        for level in range(cb.NUM_LEVELS):
            for n in range(10):
                k, t = np.argwhere(ic == 2 * n - 9)[0]
                lut[level, n] = pool[level, k, t]
        luts[side] = lut
    np.savez_compressed(HERE / "codebook.npz",
                        table_sha256=np.array(cb.codebook_sha256()),
                        pool_a_sha256=np.array(hashlib.sha256(pa.numpy().tobytes()).hexdigest()),
                        pool_b_sha256=np.array(hashlib.sha256(pb.numpy().tobytes()).hexdigest()),
                        lut_a=luts["a"], lut_b=luts["b"], table_row5=ic[5].copy(), table_row300=ic[300].copy())


def make_decode():
    ad = adapter(SMALL, rank=16, seed=4)
    words, layout = packed.pack_adapter(ad)
    pa, pb = cb.twin_pools()
    blocks_bf16 = packed.decode_packed_reference(words, layout, pa, pb)
    facs = {}
    for m in ad.modules:
        i = ad.indices[m["name"]]
        facs[m["name"] + "/A"] = quant.decode(torch.from_numpy(i["A"].astype(np.int64)), m["shape_a"], pa).numpy()
        facs[m["name"] + "/B"] = quant.decode(torch.from_numpy(i["B"].astype(np.int64)), m["shape_b"], pb).numpy()
    arrays = {f"idx/{n}/{s}": ad.indices[n][s] for n in ad.indices for s in ("A", "B")}
    arrays.update({f"fac/{k}": v for k, v in facs.items()})
    np.savez_compressed(HERE / "decode_small.npz", modules=np.array(json.dumps(ad.modules)),
                        words=words.view(torch.int64).numpy().view(np.uint64), sides=layout.sides.numpy(),
                        a_off=np.array(layout.a_off), b_off=np.array(layout.b_off),
                        blocks_bf16=bits16(blocks_bf16), **arrays)


class _Toy(torch.nn.Module):
    def __init__(self, d_in, d_out):
        super().__init__()
        self.fc = torch.nn.Linear(d_in, d_out)
        torch.nn.init.zeros_(self.fc.weight)
        torch.nn.init.zeros_(self.fc.bias)

    def forward(self, x):
        return self.fc(x)


def make_serve():
    d_in, d_out, rank = 256, 384, 16
    ads = [adapter([("fc", d_in, d_out)], rank=rank, seed=10 + s, alpha=[16, 32, 8, 16][s]) for s in range(4)]
    routes = [[(0, 1.0)], [(2, 1.0)], [], [(1, 0.6), (3, 0.4)], [(3, 1.0)], [(1, 0.25)]]
    x = torch.randn(len(routes), 24, d_in, generator=torch.Generator().manual_seed(0))
    out = {}
    for tag, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        model = _Toy(d_in, d_out).to(dtype)
        router, _ = serve.attach_adapters(model, ads)
        router.set(routes)
        with torch.no_grad():
            y = model(x.to(dtype))
        out[tag] = y.float().numpy() if dtype == torch.float32 else bits16(y)
    ids, w = router.ids.numpy(), router.weights.numpy()
    arrays = {f"idx/{a}/{s}": ads[a].indices["fc"][s] for a in range(4) for s in ("A", "B")}
    np.savez_compressed(HERE / "serve_small.npz", x=x.numpy(), ids=ids, weights=w,
                        alphas=np.array([a.alpha for a in ads], np.float32), rank=np.array(rank),
                        d_out=np.array(d_out), y_f32=out["f32"], y_bf16=out["bf16"], **arrays)


def make_config1():
    d, rank, bsz, seq = 3072, 16, 4, 256
    rng = np.random.default_rng(0)
    ads = []
    for _ in range(4):
        idx = {"fc": {"A": rng.integers(0, 512, (3, quant.num_blocks((rank, d)))).astype(np.uint16),
                      "B": rng.integers(0, 512, (3, quant.num_blocks((d, rank)))).astype(np.uint16)}}
        mods = [{"name": "fc", "shape_a": [rank, d], "shape_b": [d, rank]}]
        ads.append(fileio.LitheAdapter(modules=mods, indices=idx, rank=rank, alpha=float(rank)))
    x = torch.randn(bsz, seq, d, generator=torch.Generator().manual_seed(0))
    model = _Toy(d, d)
    router, _ = serve.attach_adapters(model, ads)
    router.set([[(i, 1.0)] for i in range(bsz)])
    with torch.no_grad():
        y = model(x)
    rows = [0, 1, 127, 255]
    np.savez_compressed(HERE / "config1_rows.npz", rows=np.array(rows), y_rows=y[:, rows].numpy(),
                        sums=y.double().sum(dim=(1, 2)).numpy(), sq=y.double().pow(2).sum(dim=(1, 2)).numpy(),
                        x_rows=x[:, rows].numpy(),
                        idx_a0_head=ads[0].indices["fc"]["A"][:, :8], idx_b3_tail=ads[3].indices["fc"]["B"][:, -8:])


def make_shared():
    arrays = {}
    pa, pb = cb.twin_pools()
    for case, (seq, d_in, d_out, r) in enumerate([(50, 128, 192, 16), (1, 256, 384, 4), (33, 192, 256, 8)]):
        ads = [adapter([("l", d_in, d_out)], rank=r, seed=s) for s in range(3)]
        ia = torch.stack([torch.from_numpy(a.indices["l"]["A"].astype(np.int32)) for a in ads])
        ib = torch.stack([torch.from_numpy(a.indices["l"]["B"].astype(np.int32)) for a in ads])
        x = (torch.randn(4, seq, d_in, generator=torch.Generator().manual_seed(case)) * 0.5).bfloat16()
        assign = torch.tensor([2, 0, 1, 2], dtype=torch.int32)
        ref = shared.shared_codebook_lora_delta_reference(x, ia, pa, ib, pb, assign, r, d_out, 0.5)
        arrays.update({f"c{case}/shape": np.array([seq, d_in, d_out, r]), f"c{case}/ia": ia.numpy(),
                       f"c{case}/ib": ib.numpy(), f"c{case}/x": bits16(x), f"c{case}/assign": assign.numpy(),
                       f"c{case}/delta": bits16(ref)})
    np.savez_compressed(HERE / "shared_small.npz", n_cases=np.array(3), scaling=np.array(0.5), **arrays)


def make_lithe_file():
    ad = adapter([("transformer_blocks.0.attn.to_q", 128, 192), ("transformer_blocks.0.ff.net.2", 320, 128),
                  ("single_transformer_blocks.0.attn.to_k", 192, 192)], rank=8, seed=21, alpha=4.0)
    ad.metadata = {"module_set": "toy-3", "note": "golden fixture"}
    fileio.save_lithe(HERE / "small.lithe", ad)
    back = fileio.load_lithe(HERE / "small.lithe")
    arrays = {f"idx/{n}/{s}": back.indices[n][s] for n in back.indices for s in ("A", "B")}
    np.savez_compressed(HERE / "small_lithe.npz", modules=np.array(json.dumps(back.modules)),
                        rank=np.array(back.rank), alpha=np.array(back.alpha),
                        header=np.array(json.dumps(fileio.read_header(HERE / "small.lithe"))), **arrays)


def kohya_like(seed, d, mlp, rank):
    mods = [("lora_unet_double_blocks_0_img_attn_qkv", d, 3 * d),
            ("lora_unet_double_blocks_0_txt_attn_qkv", d, 3 * d),
            ("lora_unet_double_blocks_0_txt_mlp_0", d, mlp),
            ("lora_unet_double_blocks_0_img_mod_lin", d, 6 * d),
            ("lora_unet_single_blocks_0_linear1", d, 3 * d + mlp),
            ("lora_unet_single_blocks_0_linear2", d + mlp, d),
            ("lora_unet_single_blocks_0_modulation_lin", d, 3 * d)]
    return adapter(mods, rank=rank, seed=seed, key_format="kohya")


def kohya_304_names(hidden=3072, mlp=12288, rank=16):
    mods = []
    for i in range(19):
        for s in ("img", "txt"):
            mods += [(f"lora_unet_double_blocks_{i}_{s}_attn_qkv", hidden, 3 * hidden),
                     (f"lora_unet_double_blocks_{i}_{s}_attn_proj", hidden, hidden),
                     (f"lora_unet_double_blocks_{i}_{s}_mlp_0", hidden, mlp),
                     (f"lora_unet_double_blocks_{i}_{s}_mlp_2", mlp, hidden),
                     (f"lora_unet_double_blocks_{i}_{s}_mod_lin", hidden, 6 * hidden)]
    for i in range(38):
        mods += [(f"lora_unet_single_blocks_{i}_linear1", hidden, 3 * hidden + mlp),
                 (f"lora_unet_single_blocks_{i}_linear2", hidden + mlp, hidden),
                 (f"lora_unet_single_blocks_{i}_modulation_lin", hidden, 3 * hidden)]
    return mods


def make_kohya():
    arrays = {}
    for tag, (seed, d, mlp, rank) in {"r4": (5, 64, 128, 4), "r16": (11, 128, 256, 16)}.items():
        ad = kohya_like(seed, d, mlp, rank)
        arrays[f"{tag}/modules"] = np.array(json.dumps(ad.modules))
        arrays[f"{tag}/paths"] = np.array(json.dumps(kohya.diffusers_paths(ad)))
        for name in ad.indices:
            arrays[f"{tag}/idx/{name}/A"] = ad.indices[name]["A"]
            arrays[f"{tag}/idx/{name}/B"] = ad.indices[name]["B"]
        for path, (ia, ib, sa, sb) in kohya.split_indices(ad).items():
            arrays[f"{tag}/split/{path}/A"] = np.asarray(ia)
            arrays[f"{tag}/split/{path}/B"] = np.asarray(ib)
            arrays[f"{tag}/split/{path}/shapes"] = np.array([*sa, *sb])
    spec = {name: kohya.split_spec(name, [16, d_in], [d_out, 16]) for name, d_in, d_out in kohya_304_names()}
    arrays["k304/spec"] = np.array(json.dumps(spec))
    np.savez_compressed(HERE / "kohya_split.npz", **arrays)


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    make_codebook()
    make_decode()
    make_serve()
    make_config1()
    make_shared()
    make_lithe_file()
    make_kohya()
    for p in sorted(HERE.iterdir()):
        if p.suffix in (".npz", ".lithe"):
            print(f"{p.name:22s} {p.stat().st_size:>9d} B")
