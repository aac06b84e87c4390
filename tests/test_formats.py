"""L0 format tests: planar pack/unpack round trips, runtime tile-block layout, files and deltas (CPU)."""
import torch

from arcagi2_flashnext_dots3_b200.formats import deltas, lowbit_file, planar, runtime as rt


def _codes(R, K, bits, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1 << bits, (R, K), generator=g, dtype=torch.int32)


def test_planar_roundtrip_and_reference_bit_layout():
    for bits in (2, 3, 4):
        q = _codes(8, 256, bits)
        pl = planar.pack_planar(q, bits)
        assert torch.equal(planar.unpack_planar(pl, bits, 256), q)
    # explicit bit positions of the reference layout: 4-bit field j of word w = column 32j + w
    q = torch.zeros(1, 128, dtype=torch.int32)
    q[0, 32 * 2 + 5] = 9
    p4 = planar.pack_planar(q, 4)["p4"]
    assert int(p4[0, 5]) & 0xFFFF == 9 << 8
    # 3-bit: 2-bit field j of word w = column 16j + w, bit j of byte w = third bit
    q = torch.zeros(1, 128, dtype=torch.int32)
    q[0, 16 * 3 + 7] = 6
    pl = planar.pack_planar(q, 3)
    assert int(pl["p2"][0, 7]) & 0xFFFF == 2 << 6
    assert int(pl["p1"][0, 7]) == 1 << 3


def test_dequant_matches_formula():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(64, 256, generator=g) * 0.02
    for bits in (2, 3, 4):
        q, s, z = planar.quantize_rtn(w, bits, clip_search=4)
        wd = planar.dequant(planar.pack_planar(q, bits), bits, s, z)
        ref = (q.view(64, 2, 128).float() - z.float()[..., None]) * s.float()[..., None]
        assert torch.allclose(wd, ref.view(64, 256))
        assert (wd - w).abs().mean() < 0.02 * (0.6 if bits > 2 else 1.0)


def test_symmetric_quant_zero_point():
    w = torch.randn(16, 128) * 0.02
    q, s, z = planar.quantize_rtn(w, 4, symmetric=True)
    assert bool((z == 8).all())


def test_runtime_blocks_roundtrip():
    g = torch.Generator().manual_seed(2)
    for bits in (2, 3, 4):
        R, K = 200, 384
        q = torch.randint(0, 1 << bits, (R, K), generator=g, dtype=torch.int32)
        s = (torch.rand(R, K // 128, generator=g) * 0.01 + 1e-3).half()
        z = torch.randint(0, 1 << bits, (R, K // 128), generator=g).to(torch.uint8)
        blob = rt.pack_q(q, s, z, bits)
        assert blob.shape == (2, 3, rt.block_bytes(bits))
        w = rt.unpack_blocks(blob, bits, R, K)
        ref = ((q.view(R, 3, 128).float() - z.float()[..., None]) * s.float()[..., None]).view(R, K)
        assert torch.allclose(w, ref)
    w = torch.randn(130, 256, generator=g) * 0.05
    w8, sc = rt.quantize_fp8_blocks(w)
    assert torch.allclose(rt.unpack_blocks(rt.pack_fp8(w8, sc), 8, 130, 256), rt.dequant_fp8_blocks(w8, sc))
    assert (rt.dequant_fp8_blocks(w8, sc) - w).abs().max() < w.abs().max() * 0.04
    wh = torch.randn(64, 128, generator=g)
    assert torch.allclose(rt.unpack_blocks(rt.pack_f16(wh), 16, 64, 128), wh.half().float())


def test_tensor_core_operands_are_fp16_products():
    """The operand view equals the dequant stage's arithmetic: fp16 value times fp16 scale, rounded once."""
    g = torch.Generator().manual_seed(3)
    for bits in (2, 3, 4):
        R, K = 200, 256
        q = torch.randint(0, 1 << bits, (R, K), generator=g, dtype=torch.int32)
        s = (torch.rand(R, K // 128, generator=g) * 0.01 + 1e-3).half()
        z = torch.randint(0, 1 << bits, (R, K // 128), generator=g).to(torch.uint8)
        op = rt.tensor_core_operands(rt.pack_q(q, s, z, bits), bits, R, K)
        want = ((q.view(R, 2, 128) - z.int()[..., None]).half() * s[..., None]).view(R, K)
        assert op.dtype == torch.float16 and torch.equal(op, want)
    w = torch.randn(130, 256, generator=g) * 0.05
    w8, sc = rt.quantize_fp8_blocks(w)
    op = rt.tensor_core_operands(rt.pack_fp8(w8, sc), 8, 130, 256)
    s16 = sc.half().repeat_interleave(128, 0)[:130].repeat_interleave(128, 1)
    assert torch.equal(op, w8.half() * s16)
    assert (op.float() - rt.dequant_fp8_blocks(w8, sc)).abs().max() <= rt.dequant_fp8_blocks(w8, sc).abs().max() * 2e-3


def test_gate_up_perm():
    p = rt.gate_up_perm(128)
    assert p[:64].tolist() == list(range(64)) and p[64:128].tolist() == list(range(128, 192))
    assert p[128:192].tolist() == list(range(64, 128))


def test_lowbit_files_and_fn_delta_roundtrip(tmp_path):
    g = torch.Generator().manual_seed(3)
    base = tmp_path / "base"
    layers = {}
    for l in range(2):
        lay = lowbit_file.random_layer(4, 128, 128, [4, 3, 4, 2], g, n_orig=8)
        lowbit_file.save_layer(base, l, lay)
        layers[l] = lay
    lowbit_file.save_keep(base, [lay.keep for lay in layers.values()])
    back = lowbit_file.load_layer(base, 1)
    assert back.experts == layers[1].experts and back.blobs[1].bits == 3
    wgu, wd = back.blobs[1].dense()
    assert wgu.shape == (256, 128) and wd.shape == (128, 128)
    # derived build: change one layer's scales and router, make a delta, rebuild, check
    der = tmp_path / "der"
    import shutil
    shutil.copytree(base, der)
    d = torch.load(der / "lowbit-L01.pt", weights_only=False)
    e0 = d["experts"][0]
    d[e0]["gu_s"] = (d[e0]["gu_s"].float() * 1.01).half()
    torch.save(d, der / "lowbit-L01.pt")
    delta = tmp_path / "delta"
    deltas.make(base, der, delta)
    assert (delta / "manifest.json").exists()
    reb = tmp_path / "reb"
    deltas.build(base, [delta], reb)
    diff = deltas.verify_build(reb, der)
    assert diff.ok and diff.identical, diff
    assert deltas.content_digest({"a": torch.ones(2)}) != deltas.content_digest({"a": torch.ones(2).half()})
    assert deltas.content_digest([1, (2, 3)]) != deltas.content_digest([1, [2, 3]])
    # a corrupted delta is refused by its manifest
    with open(delta / "router-L00.pt", "ab") as f:
        f.write(b"x")
    try:
        deltas.build(base, [delta], tmp_path / "reb2")
        raise AssertionError("corrupt delta accepted")
    except ValueError:
        pass


def test_ulp_overlay_roundtrip_and_base_guard(tmp_path):
    g = torch.Generator().manual_seed(4)
    lay = lowbit_file.random_layer(3, 128, 128, 3, g)
    lowbit_file.save_layer(tmp_path, 5, lay)
    base = torch.load(tmp_path / "lowbit-L05.pt", weights_only=False)
    new = torch.load(tmp_path / "lowbit-L05.pt", weights_only=False)
    for e in new["experts"]:
        b = new[e]["gu_s"].view(torch.int16).to(torch.int32) + torch.randint(-3, 4, new[e]["gu_s"].shape, generator=g,
                                                                             dtype=torch.int32)
        new[e]["gu_s"] = b.to(torch.int16).view(torch.float16)
    ov = deltas.make_ulp_overlay({5: base}, {5: new}, dense={"model.norm.weight": torch.ones(4)})
    deltas.save_overlay(tmp_path / "p1s_delta.safetensors", ov)
    ov = deltas.load_overlay(tmp_path / "p1s_delta.safetensors")
    assert ov["lowbit.L05.gu_s"].dtype == torch.int8
    tgt = torch.load(tmp_path / "lowbit-L05.pt", weights_only=False)
    assert deltas.apply_ulp_overlay(ov, 5, tgt)
    for e in tgt["experts"]:
        assert torch.equal(tgt[e]["gu_s"].view(torch.int16), new[e]["gu_s"].view(torch.int16))
    assert not deltas.apply_ulp_overlay(ov, 6, tgt)
    # applying again on the patched scales is refused (checksum of the base differs)
    try:
        deltas.apply_ulp_overlay(ov, 5, tgt)
        raise AssertionError("overlay applied to a different base")
    except ValueError:
        pass
    assert list(deltas.dense_replacements(ov)) == ["model.norm.weight"]
