"""Safetensors checkpoints into resident matrices (urbilateria_b200.checkpoint): header parsing,
the layout and sidecar rules of src/storage/weight.rs:118-310 (CPU), and uploads whose products
match the oracle on the same bytes (GPU)."""
import json
import os

import numpy as np
import pytest

from urbilateria_b200 import synthetic as syn
from urbilateria_b200.checkpoint import (CheckpointError, SafetensorIndex, inspect_weight_matrix,
                                         load_consolidated_mxfp8_expert, load_weight_matrix,
                                         write_safetensors)


def mx4(g, rows, cols):
    packed, scales = syn.mxfp4_matrix(g, rows, cols)
    return packed, scales


def mx8(g, rows, cols, br, bc, lo=117, hi=123):
    values = syn.encode_e4m3fn(g.standard_normal((rows, cols), dtype=np.float32))
    scales = g.integers(lo, hi + 1, size=(-(-rows // br), -(-cols // bc)), dtype=np.uint8)
    return values, scales


@pytest.fixture
def ckpt(tmp_path):
    g = syn.rng(1234)
    t = {}
    p, s = mx4(g, 64, 96)
    t["a.weight"] = ("I8", (64, 48), p.view(np.int8))
    t["a.scale"] = ("F8_E8M0", (64, 3), s)
    p, s = mx4(g, 32, 64)
    t["b.weight_packed"] = ("U8", (32, 32), p)
    t["b.weight_scale"] = ("U8", (32, 2), s)
    v, s = mx8(g, 48, 64, 1, 32)
    t["c.weight"] = ("F8_E4M3", (48, 64), v)
    t["c.weight_scale"] = ("U8", (48, 2), s)
    v, s = mx8(g, 256, 384, 128, 128)
    t["d.weight"] = ("F8_E4M3FN", (256, 384), v)
    t["d.scale"] = ("F8_E8M0FNU", (2, 3), s)
    v, s = mx8(g, 64, 64, 32, 32)
    t["e.weight"] = ("F8_E4M3", (64, 64), v)
    t["e.scale"] = ("F8_E8M0", (2, 2), s)
    bits = syn.bf16_normal(g, (16, 40), 0.02)
    t["f.weight"] = ("BF16", (16, 40), bits)
    t["g.weight"] = ("F32", (8, 8), g.standard_normal((8, 8), dtype=np.float32))
    # A matrix with two candidate sidecars, and an MXFP8 matrix with a wrong scale shape.
    v, s = mx8(g, 32, 64, 1, 32)
    t["h.weight"] = ("F8_E4M3", (32, 64), v)
    t["h.weight_scale"] = ("U8", (32, 2), s)
    t["h.weight_scale_inv"] = ("BF16", (1, 1), np.zeros((1, 1), np.uint16))
    t["i.weight"] = ("F8_E4M3", (32, 64), v)
    t["i.scale"] = ("F8_E8M0", (3, 3), np.full((3, 3), 127, np.uint8))
    # Consolidated experts (Hy4 layout): 3 experts, hidden 64, inter 32.
    E, H, I = 3, 64, 32
    gu = syn.encode_e4m3fn(g.standard_normal((E, 2 * I, H), dtype=np.float32))
    gus = g.integers(117, 124, size=(E, 2 * I, H // 32), dtype=np.uint8)
    dn = syn.encode_e4m3fn(g.standard_normal((E, H, I), dtype=np.float32))
    dns = g.integers(117, 124, size=(E, H, I // 32), dtype=np.uint8)
    t["m.experts.gate_up_proj"] = ("F8_E4M3", (E, 2 * I, H), gu)
    t["m.experts.gate_up_proj_scale"] = ("U8", (E, 2 * I, H // 32), gus)
    t["m.experts.down_proj"] = ("F8_E4M3", (E, H, I), dn)
    t["m.experts.down_proj_scale"] = ("U8", (E, H, I // 32), dns)
    # Split across two shards with an index file.
    names = list(t)
    half = {n: t[n] for n in names[: len(names) // 2]}
    rest = {n: t[n] for n in names[len(names) // 2:]}
    write_safetensors(str(tmp_path / "model-00001.safetensors"), half)
    write_safetensors(str(tmp_path / "model-00002.safetensors"), rest)
    wm = {n: "model-00001.safetensors" for n in half}
    wm.update({n: "model-00002.safetensors" for n in rest})
    json.dump({"weight_map": wm}, open(tmp_path / "model.safetensors.index.json", "w"))
    return str(tmp_path), t


def test_layouts(ckpt):
    d, t = ckpt
    idx = SafetensorIndex(d)
    assert inspect_weight_matrix(idx, "a.weight", 64, 96).format == "mxfp4"
    assert inspect_weight_matrix(idx, "b.weight_packed", 32, 64).format == "mxfp4"
    lc = inspect_weight_matrix(idx, "c.weight", 48, 64)
    assert (lc.format, lc.block_rows, lc.block_cols, lc.scale_name) == ("mxfp8", 1, 32, "c.weight_scale")
    ld = inspect_weight_matrix(idx, "d.weight", 256, 384)
    assert (ld.format, ld.block_rows, ld.block_cols) == ("mxfp8", 128, 128)
    le = inspect_weight_matrix(idx, "e.weight", 64, 64)
    assert (le.block_rows, le.block_cols) == (32, 32)
    assert inspect_weight_matrix(idx, "f.weight", 16, 40).format == "bf16"
    assert inspect_weight_matrix(idx, "g.weight", 8, 8).format == "f32"
    assert np.array_equal(np.asarray(idx.read("a.scale")), t["a.scale"][2].ravel())


@pytest.mark.parametrize("name,rows,cols,kind", [
    ("h.weight", 32, 64, "Unsupported"),   # conflicting sidecars
    ("i.weight", 32, 64, "InvalidShape"),  # no supported E8M0 scale shape
    ("a.weight", 64, 98, "InvalidShape"),  # packed shape disagrees with cols
    ("f.weight", 16, 41, "InvalidShape"),
    ("zz.weight", 4, 4, "Missing"),
])
def test_layout_errors(ckpt, name, rows, cols, kind):
    idx = SafetensorIndex(ckpt[0])
    with pytest.raises(CheckpointError) as e:
        inspect_weight_matrix(idx, name, rows, cols)
    assert e.value.kind == kind


def test_corrupt_header_is_rejected(tmp_path):
    p = tmp_path / "x.safetensors"
    p.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json}      ")
    with pytest.raises(CheckpointError) as e:
        SafetensorIndex(str(tmp_path))
    assert e.value.kind == "InvalidHeader"


@pytest.mark.gpu
def test_uploads_match_oracle(ckpt, oracle, ctx):
    d, t = ckpt
    idx = SafetensorIndex(d)
    g = syn.rng(5)
    cases = [("a.weight", 64, 96, oracle.Matrix(oracle.MXFP4, 64, 96, t["a.weight"][2].view(np.uint8),
                                                  t["a.scale"][2], group_size=32)),
             ("d.weight", 256, 384, oracle.Matrix(oracle.MXFP8, 256, 384, t["d.weight"][2],
                                                   t["d.scale"][2], block_rows=128, block_cols=128)),
             ("f.weight", 16, 40, oracle.Matrix(oracle.BF16, 16, 40, t["f.weight"][2]))]
    for name, rows, cols, om in cases:
        m = load_weight_matrix(ctx, idx, name, rows, cols)
        x = syn.normal_f32(g, cols)
        got = m.matvec(x)
        want = om.matvec(x)
        assert np.allclose(got, want, rtol=1e-5, atol=1e-5 * np.abs(want).max()), name


@pytest.mark.gpu
def test_consolidated_expert_matches_oracle(ckpt, oracle, ctx):
    d, t = ckpt
    idx = SafetensorIndex(d)
    E, H, I = 3, 64, 32
    gu, gus = t["m.experts.gate_up_proj"][2], t["m.experts.gate_up_proj_scale"][2]
    dn, dns = t["m.experts.down_proj"][2], t["m.experts.down_proj_scale"][2]
    x = syn.normal_f32(syn.rng(6), H)
    for e in range(E):
        mlp = load_consolidated_mxfp8_expert(ctx, idx, "m.experts", e, E, H, I)
        og = oracle.Matrix(oracle.MXFP8, I, H, gu[e, :I], gus[e, :I], block_rows=1, block_cols=32)
        ou = oracle.Matrix(oracle.MXFP8, I, H, gu[e, I:], gus[e, I:], block_rows=1, block_cols=32)
        od = oracle.Matrix(oracle.MXFP8, H, I, dn[e], dns[e], block_rows=1, block_cols=32)
        want = oracle.gated_mlp_forward(og, ou, od, x)
        got = mlp.forward(x)
        assert np.allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max()), e
