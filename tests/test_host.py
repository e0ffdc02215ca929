"""Host-side logic of the product package against the oracle (no GPU needed)."""
import numpy as np
import pytest
import torch

from lithe_b200 import codebook as cb
from lithe_b200 import fileio, quant, serve
from lithe_b200.kernels import packed
from lithe_b200 import _modtree
from lithe_b200.module import FLUX_TARGET_MODULES
from oracle import codebook_ref, decode_ref
from tests.helpers import GOLDEN, SMALL, golden_modules, load_golden, random_adapter


def test_product_codebook_equals_oracle():
    assert np.array_equal(cb.integer_codewords(), codebook_ref.integer_table())
    assert cb.codebook_sha256() == codebook_ref.TABLE_SHA256
    pa, pb = cb.twin_pools()
    oa, ob = codebook_ref.twin_pools()
    assert np.array_equal(pa.numpy().view(np.uint32), oa.view(np.uint32))
    assert np.array_equal(pb.numpy().view(np.uint32), ob.view(np.uint32))
    assert np.array_equal(cb.sylvester_hadamard(64), codebook_ref.hadamard(64))
    assert np.array_equal(cb.sign_table(), codebook_ref.signs())
    c = cb.codewords().double()
    ref = torch.from_numpy(codebook_ref.signs().astype(np.float64)) @ \
        torch.from_numpy(codebook_ref.generator().astype(np.float64)).T / 3.0
    assert torch.equal(c, ref.float().double())


def test_level_lut_matches_golden_and_sigmas():
    z = load_golden("codebook.npz")
    pa, pb = cb.twin_pools()
    assert np.array_equal(cb.level_lut(pa), z["lut_a"]) and np.array_equal(cb.level_lut(pb), z["lut_b"])
    assert np.array_equal(cb.lut_from_sigmas(cb.SIGMA_A), z["lut_a"])
    assert np.array_equal(cb.lut_from_sigmas(cb.SIGMA_B), z["lut_b"])
    lut = cb.kernel_lut(pa, pb)
    assert lut.shape == (2, 3, 10) and lut.dtype == np.float32


def test_level_lut_bf16_pools_reproduce_pool_values():
    pa, _ = cb.twin_pools()
    p16 = pa.to(torch.bfloat16)
    lut = cb.level_lut(p16)
    pc = cb.popcount_table()
    for level in range(3):
        assert torch.equal(torch.from_numpy(lut[level][pc]), p16[level].float())


def test_level_lut_rejects_non_hadamard_pools():
    pa, _ = cb.twin_pools()
    bad = pa.clone()
    bad[1, 7, 3] *= 1.5
    with pytest.raises(ValueError):
        cb.level_lut(bad)
    with pytest.raises(ValueError):
        cb.level_lut(torch.zeros(3, 512, 32))


def test_pack_unpack_product_vs_oracle():
    rng = np.random.default_rng(7)
    for n in (1, 6, 7, 8, 700, 1001):
        v = rng.integers(0, 512, n)
        w = packed.pack_indices(v)
        assert w.dtype == torch.uint64 and w.numel() == -(-n // 7)
        assert np.array_equal(w.view(torch.int64).numpy().view(np.uint64), decode_ref.pack9(v))
        assert np.array_equal(packed.unpack_indices(w, n).numpy(), v)
    with pytest.raises(ValueError):
        packed.pack_indices([512])


def test_layout_and_stream_vs_oracle():
    ad = random_adapter(SMALL, rank=16, seed=5)
    words, lay = packed.pack_adapter(ad)
    olay = decode_ref.layout(ad.modules)
    assert lay.a_off == olay.a_off and lay.b_off == olay.b_off
    assert np.array_equal(lay.sides.numpy(), olay.sides) and lay.num_words == olay.num_words
    assert np.array_equal(packed.flat_indices(ad, lay), decode_ref.stream(ad.indices, olay))
    shapes = ([(3072, 9216)] * 76 + [(3072, 18432)] * 38 + [(3072, 3072)] * 38 + [(3072, 12288)] * 38
              + [(12288, 3072)] * 38 + [(3072, 21504)] * 38 + [(15360, 3072)] * 38)
    mods = [{"name": f"m{i}", "shape_a": [16, a], "shape_b": [b, 16]} for i, (a, b) in enumerate(shapes)]
    k304 = packed.PackedLayout.from_modules(mods)
    assert k304.num_indices == 3_589_632 and k304.num_words * 8 == 4_102_440


def test_blockify_roundtrip():
    w = torch.randn(5, 13)
    b = quant.blockify(w)
    assert b.shape == (2, 64) and quant.num_blocks(w.shape) == 2
    assert torch.equal(quant.unblockify(b, w.shape), w)
    with pytest.raises(ValueError):
        quant.as_index_array(np.array([[0, 512]]))


def test_lithe_file_from_reference_loads():
    z = load_golden("small_lithe.npz")
    ad = fileio.load_lithe(GOLDEN / "small.lithe")
    assert ad.modules == golden_modules(z) and ad.rank == int(z["rank"]) and ad.alpha == float(z["alpha"])
    for m in ad.modules:
        for s in ("A", "B"):
            assert np.array_equal(ad.indices[m["name"]][s], z[f"idx/{m['name']}/{s}"])
    assert fileio.read_header(GOLDEN / "small.lithe")["payload_sha256"] == \
        __import__("json").loads(str(z["header"]))["payload_sha256"]


def test_lithe_file_roundtrip_and_corruption(tmp_path):
    ad = random_adapter(SMALL, rank=8, seed=2, alpha=4.0)
    p = tmp_path / "a.lithe"
    size = fileio.save_lithe(p, ad)
    assert size == p.stat().st_size
    back = fileio.load_lithe(p)
    assert back.rank == 8 and back.alpha == 4.0 and back.modules == ad.modules
    for name in ad.indices:
        for s in ("A", "B"):
            assert np.array_equal(back.indices[name][s], ad.indices[name][s])
    data = bytearray(p.read_bytes())
    bad = tmp_path / "bad_magic.lithe"
    bad.write_bytes(b"NOTLITHE" + bytes(data[8:]))
    with pytest.raises(ValueError):
        fileio.load_lithe(bad)
    trunc = tmp_path / "trunc.lithe"
    trunc.write_bytes(bytes(data[:-20]))
    with pytest.raises(ValueError):
        fileio.load_lithe(trunc)
    # same indices under a different payload digest -> checksum error
    hdr = fileio.read_header(p)
    other = random_adapter(SMALL, rank=8, seed=3, alpha=4.0)
    q = tmp_path / "other.lithe"
    fileio.save_lithe(q, other)
    qd = q.read_bytes()
    n_q = int.from_bytes(qd[8:12], "little")
    n_p = int.from_bytes(bytes(data[8:12]), "little")
    spliced = tmp_path / "spliced.lithe"
    spliced.write_bytes(bytes(data[: 12 + n_p]) + qd[12 + n_q:])
    with pytest.raises(ValueError):
        fileio.load_lithe(spliced)
    assert hdr["num_indices"] == ad.num_indices


def test_stream_codec_and_file_body(tmp_path):
    """pack_stream / unpack_stream round trip, and a saved file's body is pack_stream of the
    raw payload (tests/test_fileio.py:25-28,45-50 of the reference)."""
    raw = np.random.default_rng(3).integers(0, 512, 5000).astype("<u2").tobytes()
    assert fileio.unpack_stream(fileio.pack_stream(raw)) == raw
    ad = random_adapter(SMALL, rank=8, seed=4)
    path = tmp_path / "a.lithe"
    fileio.save_lithe(path, ad)
    blob = path.read_bytes()
    n = int.from_bytes(blob[8:12], "little")
    assert blob[12 + n:] == fileio.pack_stream(ad.raw_stream())
    assert fileio.read_payload(path)[1] == ad.raw_stream()


def test_router_and_parse_route():
    r = serve.Router()
    r.set([[(0, 1.0)], [(2, 1.0)], [], [(1, 0.6), (2, 0.4)]])
    assert r.ids.tolist() == [[0, -1], [2, -1], [-1, -1], [1, 2]]
    assert r.weights[3].tolist() == pytest.approx([0.6, 0.4])
    with pytest.raises(ValueError):
        r.set([[(0, -0.5)]])
    assert serve.parse_route("1") == [(1, 1.0)]
    assert serve.parse_route("0:0.6,2:0.4") == [(0, 0.6), (2, 0.4)]
    assert serve.parse_route("none") == []
    for empty in ("", "  ", "-", "NONE", " None "):
        assert serve.parse_route(empty) == []
    assert serve.parse_route("4:") == [(4, 1.0)]
    assert serve.parse_route(" 1 : 0.25, 3") == [(1, 0.25), (3, 1.0)]
    with pytest.raises(ValueError):
        serve.parse_route("a:1")
    r.set([])
    assert tuple(r.ids.shape) == (0, 1) and r.ids.dtype == torch.int64 and r.weights.dtype == torch.float32


def test_router_columns_fold_weights_and_scales():
    r = serve.Router()
    r.set([[(0, 1.0)], [], [(1, 0.6), (2, 0.4)]])
    cols = r.columns(torch.device("cpu"), (2.0, 0.5, 1.0))
    assert len(cols) == 2
    assert cols[0][0].tolist() == [0, -1, 1] and cols[0][1].tolist() == pytest.approx([2.0, 0.0, 0.3])
    assert cols[1][0].tolist() == [-1, -1, 2] and cols[1][1].tolist() == pytest.approx([0.0, 0.0, 0.4])
    r.set([[(3, 1.0)]])
    with pytest.raises(ValueError):
        r.columns(torch.device("cpu"), (1.0, 1.0))


def test_flux_target_count():
    names = []
    for i in range(19):
        names += [f"transformer_blocks.{i}.{t}" for t in FLUX_TARGET_MODULES]
    for i in range(38):
        names += [f"single_transformer_blocks.{i}.attn.{t}" for t in ("to_q", "to_k", "to_v")]
        names += [f"single_transformer_blocks.{i}.{t}" for t in ("proj_mlp", "proj_out", "norm.linear")]
    assert sum(_modtree.suffix_match(n, FLUX_TARGET_MODULES) for n in names) == 342


def test_flux_shaped_model_targets_342_linears():
    from lithe_b200.flux_model import FluxShapedTransformer, lora_targets
    with torch.device("meta"):
        model = FluxShapedTransformer()
    targets = lora_targets(model)
    assert len(targets) == 342
    shapes = sorted({(m.in_features, m.out_features) for _, m in targets})
    assert shapes == [(3072, 3072), (3072, 12288), (12288, 3072)]
    assert 11.5e9 < sum(p.numel() for p in model.parameters()) < 12.5e9


def test_fused_gemm_in_features_limit():
    """The fused-GEMM path is taken only up to FUSED_GEMM_MAX_K input features (host-side gate)."""
    from lithe_b200.kernels import PackedBank, PackedLayout, PackedLoRALinear
    from lithe_b200.kernels.layers import FUSED_GEMM_MAX_K
    assert FUSED_GEMM_MAX_K == 4096
    for d_in, want in ((3072, True), (4096, True), (12288, False)):
        lay = PackedLayout.from_modules([{"name": "l", "shape_a": [16, d_in], "shape_b": [512, 16]}])
        bank = PackedBank(lay, 1, "cpu")
        layer = PackedLoRALinear(torch.nn.Linear(d_in, 512).bfloat16(), bank, "l", 16, 1.0, fused_gemm=True)
        x3 = torch.zeros(2, 128, d_in, dtype=torch.bfloat16)
        assert layer._gemm_ok(x3) is want
        layer.fused_gemm_max_k = None
        assert layer._gemm_ok(x3)
        assert not layer._gemm_ok(torch.zeros(2, 100, d_in, dtype=torch.bfloat16))   # tokens per sample % 128


def test_module_tree_helpers():
    """Suffix matching works on whole path components; swaps keep the tree's order; a bad
    path leaves the model untouched."""
    from torch import nn
    assert _modtree.suffix_match("blocks.0.attn.to_q", ["attn.to_q"])
    assert _modtree.suffix_match("attn.to_q", ["attn.to_q"])
    assert not _modtree.suffix_match("blocks.0.xattn.to_q", ["attn.to_q"])
    assert not _modtree.suffix_match("blocks.0.attn.to_q2", ["attn.to_q"])
    model = nn.Sequential(nn.Linear(4, 4), nn.ReLU(), nn.Sequential(nn.Linear(4, 8), nn.Linear(8, 4)))
    got = _modtree.replace_linears(model, ["2.1", "0"], lambda p, lin: nn.Sequential(lin))
    assert list(got) == ["2.1", "0"]
    assert isinstance(model[0], nn.Sequential) and isinstance(model[2][1], nn.Sequential)
    assert isinstance(model[2][0], nn.Linear)
    with pytest.raises(TypeError):
        _modtree.replace_linears(model, ["2.0", "1"], lambda p, lin: nn.Sequential(lin))
    assert isinstance(model[2][0], nn.Linear)          # nothing swapped
    assert [p for p, _ in _modtree.linears_matching(model, ["0"])] == ["0.0", "2.0", "2.1.0"]


def test_inject_lithe_and_lithe_layers_on_cpu():
    from torch import nn
    from lithe_b200.module import LitheLinear, inject_lithe, lithe_layers

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.attn = nn.Module()
            self.attn.to_q = nn.Linear(64, 64)
            self.attn.to_k = nn.Linear(64, 64)
            self.xattn = nn.Module()
            self.xattn.to_q = nn.Linear(64, 64)
            self.norm = nn.LayerNorm(64)

    model = nn.Module()
    model.blocks = nn.ModuleList([Block(), Block()])
    wrapped = inject_lithe(model, ["attn.to_q", "attn.to_k"], rank=4)
    assert list(wrapped) == ["blocks.0.attn.to_q", "blocks.0.attn.to_k", "blocks.1.attn.to_q", "blocks.1.attn.to_k"]
    assert all(isinstance(m, LitheLinear) for m in wrapped.values())
    assert isinstance(model.blocks[0].xattn.to_q, nn.Linear)
    assert len({id(m.codebook) for m in wrapped.values()}) == 1
    assert list(lithe_layers(model)) == list(wrapped)
    with pytest.raises(ValueError):
        inject_lithe(model, ["no.such"], rank=4)


def test_attach_adapters_checks_on_cpu():
    """attach_adapters' argument checks and wrapping (host side; the forward needs a GPU)."""
    from torch import nn
    ads = [random_adapter(SMALL[:3], 8, seed=s, alpha=4 * s) for s in (1, 2)]
    names = [m["name"] for m in ads[0].modules]
    with pytest.raises(ValueError):
        serve.attach_adapters(nn.Module(), [])

    def model_for(mods):
        root = nn.Module()
        for m in mods:
            holder = root
            parts = m["name"].split(".")
            for part in parts[:-1]:
                if not hasattr(holder, part):
                    holder.add_module(part, nn.Module())
                holder = getattr(holder, part)
            holder.add_module(parts[-1], nn.Linear(m["shape_a"][1], m["shape_b"][0]))
        return root

    model = model_for(ads[0].modules)
    router, layers = serve.attach_adapters(model, ads)
    assert list(layers) == names
    for n, layer in layers.items():
        assert isinstance(layer, serve.MultiAdapterLinear) and layer.idx_a.shape[0] == 2
        assert model.get_submodule(n) is layer
        assert layer.scales == [ads[0].alpha / ads[0].rank, ads[1].alpha / ads[1].rank]
    other = random_adapter(SMALL[:1], 8, seed=3)
    with pytest.raises(ValueError):
        serve.attach_adapters(model_for(ads[0].modules), [ads[0], other])


def test_attach_accepts_different_module_order():
    """Adapters may list the same modules in different orders (tests/test_serve.py:65-76 of the
    reference); every layer then holds each adapter's indices of its own module."""
    from torch import nn
    mods = [{"name": n, "shape_a": [4, 128], "shape_b": [64, 4]} for n in ("fc", "gc")]
    rng = np.random.default_rng(1)

    def idx():
        return {"A": rng.integers(0, 512, (3, 8)).astype(np.uint16), "B": rng.integers(0, 512, (3, 4)).astype(np.uint16)}

    a = fileio.LitheAdapter(modules=mods, indices={"fc": idx(), "gc": idx()}, rank=4, alpha=8.0)
    b = fileio.LitheAdapter(modules=mods[::-1], indices={"fc": idx(), "gc": idx()}, rank=4, alpha=8.0)
    model = nn.Module()
    model.fc, model.gc = nn.Linear(128, 64), nn.Linear(128, 64)
    _, layers = serve.attach_adapters(model, [a, b])
    assert set(layers) == {"fc", "gc"}
    for name, layer in layers.items():
        for row, ad in enumerate((a, b)):
            assert np.array_equal(layer.idx_a[row].numpy(), ad.indices[name]["A"].astype(np.int16))
            assert np.array_equal(layer.idx_b[row].numpy(), ad.indices[name]["B"].astype(np.int16))


def test_flux_rope_tables():
    """The FLUX-shaped model's rotary embedding: text tokens unrotated, rotations keep norms,
    the fused form equals the pairwise rotation, and a query-key product depends only on the
    offset between image positions of one row."""
    from lithe_b200.flux_model import _rotate, rope_full, rope_tables
    cos, sin = rope_tables(4, 16, 128, "cpu")
    assert tuple(cos.shape) == (20, 64)
    assert torch.equal(cos[:4], torch.ones(4, 64)) and torch.equal(sin[:4], torch.zeros(4, 64))
    cf, sf = rope_full(cos, sin, torch.float32)
    t = torch.randn(1, 2, 20, 128)
    r = _rotate(t, cf, sf)
    x0, x1 = t[..., 0::2], t[..., 1::2]
    assert torch.allclose(r[..., 0::2], x0 * cos - x1 * sin, atol=1e-6)
    assert torch.allclose(r[..., 1::2], x1 * cos + x0 * sin, atol=1e-6)
    assert torch.allclose(r.norm(dim=-1), t.norm(dim=-1), atol=1e-4)
    q, k = torch.randn(128), torch.randn(128)
    grid = 4                                                # 16 image tokens on a 4 x 4 grid

    def dot(i, j):                                          # image tokens i, j (row-major)
        qi = _rotate(q.view(1, 1, 1, 128), cf[4 + i:5 + i], sf[4 + i:5 + i]).flatten()
        kj = _rotate(k.view(1, 1, 1, 128), cf[4 + j:5 + j], sf[4 + j:5 + j]).flatten()
        return float(qi @ kj)

    assert abs(dot(1, 0) - dot(2, 1)) < 1e-3 and abs(dot(grid + 1, 1) - dot(2 * grid + 1, grid + 1)) < 1e-3


def test_numa_binding_reads_sysfs(tmp_path, monkeypatch):
    """bind_host_to_gpu: the GPU's PCI function -> its NUMA node -> that node's CPUs (here a
    fake sysfs tree); unknown nodes change nothing."""
    import os
    from types import SimpleNamespace
    from lithe_b200 import shard
    props = SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1b, pci_device_id=0)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: props)
    dev = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    dev.mkdir(parents=True)
    cpus = sorted(os.sched_getaffinity(0))
    node_dir = tmp_path / "devices" / "system" / "node" / "node1"
    node_dir.mkdir(parents=True)
    (node_dir / "cpulist").write_text(f"{cpus[0]}-{cpus[-1]}\n")
    (dev / "numa_node").write_text("1\n")
    seen = {}
    monkeypatch.setattr(os, "sched_setaffinity", lambda pid, s: seen.setdefault("cpus", set(s)))
    assert shard.gpu_numa_node(0, str(tmp_path)) == 1
    assert shard.bind_host_to_gpu(0, str(tmp_path)) == 1 and seen["cpus"] == set(cpus)
    (dev / "numa_node").write_text("-1\n")
    assert shard.bind_host_to_gpu(0, str(tmp_path)) is None
    assert shard._parse_cpulist("0-2,5,7-8") == [0, 1, 2, 5, 7, 8]


def test_prep_split_choice():
    """The split shrink is chosen only where whole 64-token tiles leave the busiest CTA far above
    the average (FLUX 1024^2 B=14: the 12288- and 15360-wide img inputs, not the 3072-wide ones,
    nor the 4608-token single-block inputs whose 1008 tiles already spread evenly)."""
    from lithe_b200.kernels._launch import prep_split_pays
    assert prep_split_pays(14, 4096, 12288, 148) and prep_split_pays(14, 4096, 15360, 148)
    assert not prep_split_pays(14, 4096, 3072, 148)
    assert not prep_split_pays(14, 4608, 15360, 148) and not prep_split_pays(14, 512, 12288, 148)
    assert not prep_split_pays(4, 4096, 3072, 148) and not prep_split_pays(0, 4096, 3072, 148)


def test_shared_input_groups_on_the_flux_names():
    """wrap_packed(fused_gemm=True) groups the linears that read one input: per double block the
    image and the text stream's q / k / v, per single block its q / k / v (its proj_mlp too when
    it is a target).  Kohya split targets, other banks and other widths do not join."""
    import pytest as _pytest

    from lithe_b200.flux_model import FluxConfig, FluxShapedTransformer, lora_targets
    from lithe_b200.kernels import PackedBank, PackedLayout, PackedLoRALinear, SharedInputPrep, wrap_packed
    model = FluxShapedTransformer(FluxConfig.tiny())
    targets = lora_targets(model)
    lay = PackedLayout.from_modules([{"name": n, "shape_a": [16, m.in_features], "shape_b": [m.out_features, 16]}
                                     for n, m in targets])
    wrapped = wrap_packed(model, PackedBank(lay, 2, "cpu"), fused_gemm=True)
    groups = {id(m.prep_group): m.prep_group for m in wrapped.values() if m.prep_group is not None}
    names = {tuple(sorted(n for n, m in wrapped.items() if m.prep_group is g)) for g in groups.values()}
    assert ("transformer_blocks.0.attn.to_k", "transformer_blocks.0.attn.to_q",
            "transformer_blocks.0.attn.to_v") in names
    assert ("transformer_blocks.1.attn.add_k_proj", "transformer_blocks.1.attn.add_q_proj",
            "transformer_blocks.1.attn.add_v_proj") in names
    assert ("single_transformer_blocks.0.attn.to_k", "single_transformer_blocks.0.attn.to_q",
            "single_transformer_blocks.0.attn.to_v") in names
    assert len(groups) == 6 and all(len(g.members) == 3 for g in groups.values())
    assert wrapped["transformer_blocks.0.attn.to_out.0"].prep_group is None
    # without the fused-GEMM path nothing is grouped
    model2 = FluxShapedTransformer(FluxConfig.tiny())
    assert all(m.prep_group is None for m in wrap_packed(model2, PackedBank(lay, 2, "cpu")).values())
    # members must share a bank
    other = PackedBank(lay, 2, "cpu")
    q = wrapped["transformer_blocks.0.attn.to_q"]
    lin = torch.nn.Linear(q.base.in_features, q.base.out_features)
    stray = PackedLoRALinear(lin, other, "transformer_blocks.0.attn.to_q", 16, 1.0, fused_gemm=True)
    with _pytest.raises(ValueError):
        SharedInputPrep([PackedLoRALinear(lin, q.bank, "transformer_blocks.0.attn.to_q", 16, 1.0), stray])
    with _pytest.raises(ValueError):
        SharedInputPrep([stray])


def test_traffic_digest_ignores_comments_only():
    """The recorded DRAM traffic is keyed on the kernel's code: comments and whitespace do not
    change the digest, code does; string and character literals are kept verbatim."""
    import bench
    a = 'int f(int x) {  // note\n  return x + 1; /* block */ }\nconst char* s = "a//b/*c*/";\n'
    b = 'int f(int x) {\n\n    return x + 1;   }\nconst char* s = "a//b/*c*/";  // other\n'
    c = 'int f(int x) { return x + 2; }\nconst char* s = "a//b/*c*/";\n'
    assert bench._code_only(a) == bench._code_only(b) != bench._code_only(c)
    assert '"a//b/*c*/"' in bench._code_only(a)


def test_int32_index_banks_unpack_the_packed_stream():
    """The bench's reference_triton variant feeds the reference's IndexLoRALinear int32 banks
    unpacked from the packed slots: they must be each adapter's own (L, n_blocks) indices."""
    import bench
    mods = [("a", 3072, 3072), ("b", 3072, 12288), ("c", 12288, 3072), ("odd", 96, 40), ("e", 15360, 3072)]
    ads = [random_adapter(mods, rank=16, seed=s) for s in range(3)]
    bank = packed.PackedBank.from_adapters(ads, "cpu")
    order = [2, 0, 1]
    for name, d_in, d_out in mods:
        a, b = bench.int32_index_banks(bank, name, order)
        assert a.dtype == torch.int32 and a.shape == (3, 3, quant.num_blocks((16, d_in)))
        assert b.shape == (3, 3, quant.num_blocks((d_out, 16)))
        for k, s in enumerate(order):
            assert np.array_equal(a[k].numpy(), ads[s].indices[name]["A"].astype(np.int32))
            assert np.array_equal(b[k].numpy(), ads[s].indices[name]["B"].astype(np.int32))


def test_reference_install_missing_is_reported_and_cpu_arm_falls_back(tmp_path, monkeypatch):
    """Without the reference's install the GPU comparators report why (ImportError, printed as
    an unavailable line) and the CPU arm times the oracle port instead (kind "port")."""
    import bench
    monkeypatch.setattr(bench, "REF_INSTALL", tmp_path / "absent")
    monkeypatch.setattr(bench, "SHAPES", [(128, 192)])
    monkeypatch.setattr(bench, "CPU_SAMPLE_TOKENS", 64)
    with pytest.raises(ImportError, match="baseline/_ref"):
        bench.reference_package()
    rec = bench.cpu_reference_passes(2, warmup=1)
    assert rec["kind"] == "port" and rec["passes"] == 2 and rec["value"] > 0
    assert rec["spread"]["min"] <= rec["spread"]["median"] <= rec["spread"]["max"]


def test_cpu_arm_runs_the_reference_when_installed(monkeypatch):
    import bench
    try:
        bench.reference_package(require_triton=False)
    except ImportError as e:
        pytest.skip(f"reference install absent: {e}")
    monkeypatch.setattr(bench, "SHAPES", [(128, 192)])
    monkeypatch.setattr(bench, "CPU_SAMPLE_TOKENS", 64)
    rec = bench.cpu_reference_passes(2, warmup=1)
    assert rec["kind"] == "reference" and "MultiAdapterLinear" in rec["path"]
