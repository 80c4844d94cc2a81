"""Parity of the device matrix products (C ABI) with the CPU oracle.

Bar: relative L2 <= 1e-3 and max-abs <= 2e-2 (outputs normalised to unit RMS) against the
reference's f32 outputs; decoded weights bit-exact; error variants as in the reference.
"""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

from helpers import assert_close, bf16_pair, mxfp4_pair, mxfp8_pair

pytestmark = pytest.mark.gpu


def test_mxfp4_decode_is_exact_and_low_nibble_first(oracle, ctx):
    # Identity batch: y[t][r] = W[r][t], a single exact product per output.
    g = syn.rng(11)
    rows, cols = 35, 160
    dev, orc = mxfp4_pair(oracle, ctx, g, rows, cols, lo=112, hi=134)
    eye = np.eye(cols, dtype=np.float32)
    got = dev.matmul_rows(eye, cols)
    want = np.stack([orc.matvec(eye[c]) for c in range(cols)])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_mxfp8_decode_is_exact(oracle, ctx):
    g = syn.rng(12)
    rows, cols = 33, 96
    dev, orc = mxfp8_pair(oracle, ctx, g, rows, cols, lo=110, hi=130)
    eye = np.eye(cols, dtype=np.float32)
    got = dev.matmul_rows(eye, cols)
    want = np.stack([orc.matvec(eye[c]) for c in range(cols)])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_bf16_decode_is_exact(oracle, ctx):
    g = syn.rng(13)
    dev, orc = bf16_pair(oracle, ctx, g, 20, 136)
    eye = np.eye(136, dtype=np.float32)
    got = dev.matmul_rows(eye, 136)
    want = np.stack([orc.matvec(eye[c]) for c in range(136)])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_c0_mxfp4_matvec_4096x7168(oracle, ctx):
    # W 4096x7168, E8M0 119..127, x ~ N(0,1).
    g = syn.rng(2024)
    dev, orc = mxfp4_pair(oracle, ctx, g, 4096, 7168)
    x = syn.normal_f32(g, 7168)
    assert_close(dev.matvec(x), orc.matvec(x))


@pytest.mark.parametrize("rows,cols", [(1, 32), (17, 129), (35, 2049), (300, 1000), (64, 4096)])
def test_mxfp4_odd_shapes(oracle, ctx, rows, cols):
    g = syn.rng(rows * 1000 + cols)
    dev, orc = mxfp4_pair(oracle, ctx, g, rows, cols)
    for batch in (1, 3, 12, 13):
        x = syn.normal_f32(g, (batch, cols))
        assert_close(dev.matmul_rows(x, batch), orc.matmul_rows(x, batch))


@pytest.mark.parametrize("group", [8, 16, 33, 128])
def test_mxfp4_other_group_sizes_use_generic_path(oracle, ctx, group):
    g = syn.rng(group)
    dev, orc = mxfp4_pair(oracle, ctx, g, 40, 300, group=group)
    x = syn.normal_f32(g, (3, 300))
    assert_close(dev.matmul_rows(x, 3), orc.matmul_rows(x, 3))


def test_mxfp4_wide_scale_range_uses_generic_path(oracle, ctx):
    g = syn.rng(5)
    dev, orc = mxfp4_pair(oracle, ctx, g, 16, 256, lo=60, hi=190)
    x = syn.normal_f32(g, 256)
    assert_close(dev.matvec(x), orc.matvec(x))


@pytest.mark.parametrize("block", [(1, 32), (128, 128), (32, 64)])
def test_mxfp8_blocks(oracle, ctx, block):
    g = syn.rng(block[0] * 7 + block[1])
    dev, orc = mxfp8_pair(oracle, ctx, g, 300, 1536, *block)
    for batch in (1, 5, 12):
        x = syn.normal_f32(g, (batch, 1536))
        assert_close(dev.matmul_rows(x, batch), orc.matmul_rows(x, batch))


def test_bf16_and_f32(oracle, ctx):
    g = syn.rng(21)
    dev, orc = bf16_pair(oracle, ctx, g, 768, 2048)
    x = syn.normal_bf16_as_f32(g, (4, 2048))
    assert_close(dev.matmul_rows(x, 4), orc.matmul_rows(x, 4))
    w = syn.normal_f32(g, (50, 70))
    d = urb.DenseMatrix.new(50, 70, w, ctx=ctx)
    o = oracle.Matrix(oracle.F32, 50, 70, w)
    x = syn.normal_f32(g, 70)
    assert_close(d.matvec(x), o.matvec(x))


def test_row_ranges(oracle, ctx):
    g = syn.rng(31)
    dev, orc = mxfp4_pair(oracle, ctx, g, 100, 256)
    x = syn.normal_f32(g, 256)
    for start, count in [(0, 100), (5, 20), (17, 1), (99, 1), (16, 64)]:
        assert_close(dev.matvec_rows(start, count, x), orc.matvec_rows(start, count, x))
    xb = syn.normal_f32(g, (3, 256))
    assert_close(dev.matmul_row_range(7, 50, xb, 3),
                 np.stack([orc.matvec_rows(7, 50, xb[t]) for t in range(3)]))


def test_error_variants(ctx):
    g = syn.rng(41)
    packed, scales = syn.mxfp4_matrix(g, 4, 64)
    bad = scales.copy()
    bad[1, 1] = 0xFF
    with pytest.raises(urb.UrbError) as e:
        urb.MxFp4Matrix.from_packed(4, 64, 32, packed, bad, ctx=ctx)
    assert e.value.kind == "InvalidScale"
    with pytest.raises(urb.UrbError) as e:
        urb.MxFp4Matrix.from_packed(4, 64, 32, packed[:, :10], scales, ctx=ctx)
    assert e.value.kind == "Shape"
    vals = np.full((4, 64), 0x38, np.uint8)
    vals[2, 3] = 0xFF
    with pytest.raises(urb.UrbError) as e:
        urb.MxFp8Matrix.from_packed(4, 64, 1, 32, vals, np.full((4, 2), 127, np.uint8), ctx=ctx)
    assert e.value.kind == "NonFinite"
    m = urb.MxFp4Matrix.from_packed(4, 64, 32, packed, scales, ctx=ctx)
    x = np.ones(64, np.float32)
    x[5] = np.nan
    with pytest.raises(urb.UrbError) as e:
        m.matvec(x)
    assert e.value.kind == "NonFinite"
    with pytest.raises(urb.UrbError) as e:
        m.matvec(np.ones(63, np.float32))
    assert e.value.kind == "Shape"
    with pytest.raises(urb.UrbError) as e:
        m.matvec_rows(2, 3, np.ones(64, np.float32))
    assert e.value.kind == "Shape"


def test_mxfp8_nonfinite_output_is_rejected(ctx):
    # E4M3 448 * 2^127 overflows f32: the reference rejects MXFP8 outputs that are not finite.
    vals = np.full((1, 32), 0x7E, np.uint8)
    m = urb.MxFp8Matrix.from_packed(1, 32, 1, 32, vals, np.array([[254]], np.uint8), ctx=ctx)
    with pytest.raises(urb.UrbError) as e:
        m.matvec(np.ones(32, np.float32))
    assert e.value.kind == "NonFinite"


@pytest.mark.parametrize("fmt,rows,cols", [("mxfp4", 3840, 25600), ("mxfp8", 700, 9000),
                                           ("mxfp4", 38400, 256)])
def test_single_token_wide_and_tall(oracle, ctx, fmt, rows, cols):
    # Single-token products of wide, tall and ragged matrices (many row blocks per SM, long K,
    # partial last blocks).  Deterministic: two calls agree bit for bit.
    g = syn.rng(rows + cols)
    pair = mxfp4_pair if fmt == "mxfp4" else mxfp8_pair
    dev, orc = pair(oracle, ctx, g, rows, cols)
    x = syn.normal_f32(g, cols)
    got = dev.matvec(x)
    assert_close(got, orc.matvec(x))
    assert np.array_equal(dev.matvec(x).view(np.uint32), got.view(np.uint32))


def test_single_token_row_ranges_long_k(oracle, ctx):
    g = syn.rng(77)
    dev, orc = mxfp4_pair(oracle, ctx, g, 300, 7168)
    x = syn.normal_f32(g, 7168)
    for start, count in [(130, 100), (0, 300), (255, 2), (299, 1)]:
        assert_close(dev.matvec_rows(start, count, x), orc.matvec_rows(start, count, x))


@pytest.mark.parametrize("rows,cols", [(37, 1001), (130, 2048), (5, 8), (64, 7168)])
def test_bf16_streaming_products(oracle, ctx, rows, cols):
    # Up to 32 tokens take the streaming CUDA-core pass: ragged columns (not a multiple of 8),
    # partial token tiles (1, 3, 9, 32 tokens) and row ranges.
    g = syn.rng(rows * 7 + cols)
    dev, orc = bf16_pair(oracle, ctx, g, rows, cols, std=0.5)
    for batch in (1, 3, 9, 32):
        x = syn.normal_f32(g, (batch, cols))
        assert_close(dev.matmul_rows(x, batch), orc.matmul_rows(x, batch))
    x = syn.normal_f32(g, cols)
    start, count = rows // 3, rows - rows // 3 - 1 if rows > 2 else 1
    assert_close(dev.matvec_rows(start, count, x), orc.matvec_rows(start, count, x))


@pytest.mark.parametrize("tokens", [1, 5, 17, 32])
def test_bf16_gated_mlp_streaming(oracle, ctx, tokens):
    g = syn.rng(8800 + tokens)
    gd, go = bf16_pair(oracle, ctx, g, 768, 2048)
    ud, uo = bf16_pair(oracle, ctx, g, 768, 2048)
    dd, do = bf16_pair(oracle, ctx, g, 2048, 768)
    x = syn.normal_bf16_as_f32(g, (tokens, 2048))
    got = urb.GatedMlp(gd, ud, dd).forward_batch(x, tokens)
    want = np.stack([oracle.gated_mlp_forward(go, uo, do, x[t]) for t in range(tokens)])
    assert_close(got, want)


def test_host_matvec_rows_allocates_nothing_in_steady_state(ctx):
    """urb_matvec_rows / urb_matmul_rows stage x and y through the context's grow-only device
    and pinned buffers: once they have grown, further calls leave the device's memory alone."""
    from helpers import memory_state
    import torch
    g = syn.rng(9200)
    p, s = syn.mxfp4_matrix(g, 4096, 7168)
    m = urb.MxFp4Matrix.from_packed(4096, 7168, 32, p, s, ctx=ctx)
    x = syn.normal_f32(g, (3, 7168))
    for _ in range(2):
        m.matvec_rows(10, 300, x[0])
        m.matmul_rows(x, 3)
    torch.cuda.synchronize()
    before = memory_state(ctx.device)
    ys = [m.matvec_rows(10, 300, x[0]) for _ in range(3)] + [m.matmul_rows(x, 3) for _ in range(3)]
    after = memory_state(ctx.device)
    assert before == after, (before, after)
    assert all(np.array_equal(ys[0], y) for y in ys[:3])
    m.free()


@pytest.mark.parametrize("fmt", ["mxfp4", "mxfp8"])
def test_mx_matrix_keeps_one_resident_copy(ctx, fmt):
    """An MX upload keeps only its block-scaled tensor-core tiles (payload + scales, the
    reference's resident_bytes) and one exponent byte per row: every product path reads them."""
    from helpers import memory_state
    import torch
    g = syn.rng(9300)
    rows, cols = 4096, 7168
    torch.cuda.synchronize()
    before = memory_state(ctx.device)[0]
    if fmt == "mxfp4":
        m = urb.MxFp4Matrix.from_packed(rows, cols, 32, *syn.mxfp4_matrix(g, rows, cols), ctx=ctx)
    else:
        v = g.integers(0, 0x7e, size=(rows, cols), dtype=np.uint8)
        m = urb.MxFp8Matrix.from_packed(rows, cols, 1, 32, v, g.integers(117, 124, size=(rows, cols // 32),
                                                                          dtype=np.uint8), ctx=ctx)
    torch.cuda.synchronize()
    grew = memory_state(ctx.device)[0] - before
    assert grew <= m.resident_bytes() + rows + 4096, (grew, m.resident_bytes())
    x = syn.normal_f32(g, (3, cols))
    assert np.isfinite(m.matmul_rows(x, 3)).all()
    m.free()


@pytest.mark.parametrize("rows,cols", [(300, 200), (2048, 768), (768, 2048), (5, 8), (130, 7168)])
def test_bf16_split_k_tensor_core_products(oracle, ctx, rows, cols):
    # BF16 with cols % 8 == 0, 1..32 tokens, whole rows: tcgen05 kind::f16 with K split over a
    # cluster (TMA boxes past the matrix's last row / column read as zero; ragged K stages).
    g = syn.rng(rows + 3 * cols)
    dev, orc = bf16_pair(oracle, ctx, g, rows, cols, std=0.5)
    for batch in (1, 2, 7, 16, 31, 32):
        x = syn.normal_f32(g, (batch, cols))
        assert_close(dev.matmul_rows(x, batch), orc.matmul_rows(x, batch))


@pytest.mark.parametrize("batch", [33, 77])
def test_bf16_batched_products_on_the_grouped_pass(oracle, ctx, batch):
    # More than 32 tokens: the grouped tcgen05 pass (all tokens in one group), row ranges too.
    g = syn.rng(batch)
    dev, orc = bf16_pair(oracle, ctx, g, 300, 200, std=0.5)
    x = syn.normal_f32(g, (batch, 200))
    assert_close(dev.matmul_rows(x, batch), orc.matmul_rows(x, batch))
    got = dev.matmul_row_range(37, 150, x, batch)
    want = orc.matmul_rows(x, batch)[:, 37:187]
    assert_close(got, want)


@pytest.mark.parametrize("tokens", [40, 96])
def test_bf16_gated_mlp_grouped_pass(oracle, ctx, tokens):
    g = syn.rng(8900 + tokens)
    gd, go = bf16_pair(oracle, ctx, g, 768, 2048)
    ud, uo = bf16_pair(oracle, ctx, g, 768, 2048)
    dd, do = bf16_pair(oracle, ctx, g, 2048, 768)
    x = syn.normal_f32(g, (tokens, 2048))
    got = urb.GatedMlp(gd, ud, dd).forward_batch(x, tokens)
    want = np.stack([oracle.gated_mlp_forward(go, uo, do, x[t]) for t in range(tokens)])
    assert_close(got, want)
