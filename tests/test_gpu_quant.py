"""Int8Matrix / Int4Matrix (src/math/quant.rs) on the device against the oracle: the reference's
known-answer cases (quant.rs:622-720, weight.rs:416-616), the INT4 grouped quantiser bit for bit,
row products on every kernel shape (16-byte chunks with one scale per chunk, per-element
groups, byte-wise rows), transposes and decoded rows bit for bit, and the constructors' error
order.

Row products sum exactly in integers over x on a 38-bit fixed-point grid (16-byte rows) or sum
exact f64 products in a fixed lane order (other shapes), so they agree with the reference's
ordered f64 sum to within |gpu - oracle| <= 2^-38 * sum_c |w_c x_c| (twice the worst-case f64
summation error at 7168 columns) + 2^-38 * max|x| * sum_c |w_c| (the grid) + one f32 ulp of the
result, per element: at most one-ulp flips where the sum sits on an f32 rounding boundary, or a
row sum that cancels.  At least 99% of elements must be bit-identical.  Dyadic data, whose
products and sums are exact, must match bit for bit."""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import native
from urbilateria_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _rust_i8_rem31(index):
    v = ((index & 0xFF) ^ 0x80) - 0x80
    return v % 31 if v >= 0 else -((-v) % 31)


def int8_pair(oracle, ctx, g, rows, cols):
    data = g.integers(-128, 128, size=(rows, cols)).astype(np.int8)
    scales = (np.abs(g.standard_normal(rows)) * 0.01 + 1e-4).astype(np.float32)
    return (urb.Int8Matrix.from_packed(rows, cols, data, scales, ctx=ctx),
            oracle.Matrix(oracle.INT8, rows, cols, data.view(np.uint8), scales))


def int4_pair(oracle, ctx, g, rows, cols, group):
    packed = g.integers(0, 256, size=rows * ((cols + 1) // 2), dtype=np.uint8)
    scales = (np.abs(g.standard_normal(rows * ((cols + group - 1) // group))) * 0.02 + 1e-4).astype(np.float32)
    return (urb.Int4Matrix.from_packed(rows, cols, group, packed, scales, ctx=ctx),
            oracle.Matrix(oracle.INT4, rows, cols, packed, scales, group_size=group))


def assert_rows_close(got, want, mat, x):
    """The bar in the module docstring; mat [rows, cols] decoded weights, x [batch, cols]."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    mag = np.abs(x.astype(np.float64)) @ np.abs(mat.astype(np.float64)).T  # [batch, rows]
    # x on the fixed-point grid: each element within 2^-38 of its token's largest magnitude.
    grid = np.abs(x).max(axis=1, keepdims=True).astype(np.float64) * \
        np.abs(mat.astype(np.float64)).sum(axis=1)[None, :] * 2.0 ** -38
    ulp = np.spacing(np.abs(want)).astype(np.float64)
    bound = mag * 2.0 ** -38 + grid + ulp
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= bound), float((err - bound).max())
    assert np.mean(bits(got) == bits(want)) >= 0.99


def test_int_golden_mixed_formats(ctx):
    # src/model/weight.rs:416-442
    i8 = urb.Int8Matrix.from_packed(2, 2, np.array([0xff, 2, 3, 0xfc], np.uint8),
                                    np.array([1.0, 1.0], np.float32), ctx=ctx)
    i4 = urb.Int4Matrix.from_packed(2, 2, 2, np.array([0xa7, 0x4b], np.uint8),
                                    np.array([1.0, 1.0], np.float32), ctx=ctx)
    for m in (i8, i4):
        assert list(m.row(0)) == [-1.0, 2.0]
        assert list(m.matvec([0.5, 2.0])) == [3.5, -6.5]
        assert list(m.matmul_rows([0.5, 2.0, 1.0, -1.0], 2).ravel()) == [3.5, -6.5, -3.0, 7.0]
        assert list(m.transpose_matvec([0.5, 2.0])) == [5.5, -7.0]
        assert list(m.transpose_rows_matvec(1, [2.0])) == [6.0, -8.0]
        assert list(m.matvec_rows(1, 1, [0.5, 2.0])) == [-6.5]


def test_int8_golden_twos_complement(ctx):
    # src/math/quant.rs:694-720
    m = urb.Int8Matrix.from_packed(2, 3, np.array([0xff, 0x00, 0x7f, 0x80, 0x02, 0xfe], np.uint8),
                                   np.array([0.5, 0.25], np.float32), ctx=ctx)
    assert list(m.row(0)) == [-0.5, 0.0, 63.5]
    assert list(m.row(1)) == [-32.0, 0.5, -0.5]
    assert list(m.matvec([2.0, -1.0, 0.5])) == [30.75, -64.75]
    assert m.resident_bytes() == 6 + 2 * 4


def test_int4_golden_quantiser(ctx):
    # src/math/quant.rs:622-641
    m = urb.Int4Matrix.quantize_per_row(1, 3, [-8.0, 7.0, 0.0], ctx=ctx)
    p = m.packed()
    assert p.size == 2 and p[0] & 0x0F == 1 and p[0] >> 4 == 14 and p[1] == 0x88
    assert m.scales()[0] == np.float32(8.0) / np.float32(7.0)
    values = [100.0, 0.5, 0.5, 0.5]
    per_row = urb.Int4Matrix.quantize_per_row(1, 4, values, ctx=ctx)
    grouped = urb.Int4Matrix.quantize_grouped(1, 4, 2, values, ctx=ctx)
    assert abs(grouped.row(0)[2] - 0.5) < abs(per_row.row(0)[2] - 0.5)
    assert per_row.resident_bytes() == 2 + 4


def test_int_large_kernels_bit_exact(ctx, oracle):
    # src/model/weight.rs:497-616 (65 x 1025): dyadic data, so every order is exact.
    rows, cols = 65, 1025
    x = np.array([(c % 17 - 8.0) / 16.0 for c in range(cols)], np.float32)
    tx = np.array([(r % 11 - 5.0) / 8.0 for r in range(rows)], np.float32)
    d8 = np.array([_rust_i8_rem31(i) & 0xFF for i in range(rows * cols)], np.uint8)
    p4 = np.array([(i * 37) & 0xFF for i in range(rows * ((cols + 1) // 2))], np.uint8)
    s4 = np.full(rows * ((cols + 63) // 64), 0.0625, np.float32)
    pairs = [(urb.Int8Matrix.from_packed(rows, cols, d8, np.full(rows, 0.03125, np.float32), ctx=ctx),
              oracle.Matrix(oracle.INT8, rows, cols, d8, np.full(rows, 0.03125, np.float32))),
             (urb.Int4Matrix.from_packed(rows, cols, 64, p4, s4, ctx=ctx),
              oracle.Matrix(oracle.INT4, rows, cols, p4, s4, group_size=64))]
    for dev, ref in pairs:
        assert np.array_equal(bits(dev.matvec(x)), bits(ref.matvec(x)))
        assert np.array_equal(bits(dev.transpose_matvec(tx)), bits(ref.transpose_rows_matvec(0, tx)))
        assert np.array_equal(bits(dev.write_rows(0, rows)),
                              bits(np.stack([ref.write_row(r) for r in range(rows)])))


@pytest.mark.parametrize("rows,cols,group", [
    (3, 7, 3),          # the reference's odd-group case (quant.rs:662-691)
    (65, 1025, 64),
    (96, 7168, 64),     # GLM expert hidden width, 64-column groups
    (40, 2048, 2048),   # per-row (quantize_per_row)
    (17, 333, 10),
])
def test_int4_quantize_bit_exact(oracle, ctx, rows, cols, group):
    g = syn.rng(rows * 7 + cols)
    v = (g.standard_normal((rows, cols)) * np.exp(g.standard_normal((rows, 1)))).astype(np.float32)
    v[0, : min(cols, 5)] = [0.0, -0.0, 1e-9, -3e-8, 2.5][: min(cols, 5)]  # tiny rows/groups hit the 1e-8 floor
    want_p, want_s = oracle.int4_quantize_grouped(rows, cols, group, v)
    m = urb.Int4Matrix.quantize_grouped(rows, cols, group, v, ctx=ctx)
    assert np.array_equal(m.packed(), want_p)
    assert np.array_equal(bits(m.scales()), bits(want_s))


@pytest.mark.parametrize("fmt,rows,cols,group", [
    ("int8", 256, 7168, 0),    # 16-byte chunks
    ("int8", 37, 100, 0),      # byte-wise rows (cols % 16 != 0)
    ("int8", 65, 1025, 0),
    ("int4", 256, 7168, 64),   # 16-byte chunks, one scale per 32-column chunk
    ("int4", 64, 2048, 48),    # 16-byte chunks, per-element groups
    ("int4", 65, 1025, 64),    # byte-wise rows (odd columns)
    ("int4", 40, 1536, 1536),  # per-row scale
])
@pytest.mark.parametrize("batch", [1, 3, 8, 13])
def test_int_products_match_oracle(oracle, ctx, fmt, rows, cols, group, batch):
    g = syn.rng(rows * 131 + cols + batch)
    dev, ref = int8_pair(oracle, ctx, g, rows, cols) if fmt == "int8" else \
        int4_pair(oracle, ctx, g, rows, cols, group)
    x = g.standard_normal((batch, cols)).astype(np.float32)
    mat = np.stack([ref.write_row(r) for r in range(rows)])
    assert_rows_close(dev.matmul_rows(x, batch), ref.matmul_rows(x, batch), mat, x)
    s, c = rows // 3, rows // 2
    assert_rows_close(dev.matmul_row_range(s, c, x, batch), ref.matmul_rows(x, batch)[:, s:s + c],
                      mat[s:s + c], x)
    assert_rows_close(dev.matvec_rows(1, rows - 1, x[0])[None], ref.matvec_rows(1, rows - 1, x[0])[None],
                      mat[1:], x[:1])
    assert_rows_close(dev.matmul_rows_fp32_accum(x, batch), ref.matmul_rows(x, batch), mat, x)


@pytest.mark.parametrize("fmt,rows,cols,group,start,n", [
    ("int8", 300, 1536, 0, 17, 255),
    ("int8", 33, 70, 0, 0, 33),
    ("int4", 300, 7168, 64, 130, 100),
    ("int4", 41, 333, 10, 3, 37),
])
def test_int_transpose_and_rows_bit_exact(oracle, ctx, fmt, rows, cols, group, start, n):
    g = syn.rng(rows + cols * 3)
    dev, ref = int8_pair(oracle, ctx, g, rows, cols) if fmt == "int8" else \
        int4_pair(oracle, ctx, g, rows, cols, group)
    x = (g.standard_normal(n) * 3).astype(np.float32)
    assert np.array_equal(bits(dev.transpose_rows_matvec(start, x)),
                          bits(ref.transpose_rows_matvec(start, x)))
    assert np.array_equal(bits(dev.write_rows(start, n)),
                          bits(np.stack([ref.write_row(r) for r in range(start, start + n)])))


def test_write_rows_block_scaled_tiles(oracle, ctx):
    # MXFP4 with 32-column groups keeps only the tensor-core tiles: rows decode from them.
    from helpers import mxfp4_pair
    g = syn.rng(77)
    dev, ref = mxfp4_pair(oracle, ctx, g, 160, 7168)
    assert np.array_equal(bits(dev.write_rows(5, 150)),
                          bits(np.stack([ref.write_row(r) for r in range(5, 155)])))


def test_int_error_order(ctx):
    E = urb.UrbError
    with pytest.raises(E) as e:
        urb.Int4Matrix.from_packed(1, 2, 0, np.zeros(1, np.uint8), np.ones(1, np.float32), ctx=ctx)
    assert e.value.code == native.ERR_INVALID_GROUP
    with pytest.raises(E) as e:
        urb.Int4Matrix.quantize_grouped(1, 2, 0, [1.0, 2.0], ctx=ctx)
    assert e.value.code == native.ERR_INVALID_GROUP
    with pytest.raises(E) as e:
        urb.Int4Matrix.from_packed(2, 3, 2, np.zeros(3, np.uint8), np.ones(4, np.float32), ctx=ctx)
    assert e.value.code == native.ERR_SHAPE
    with pytest.raises(E) as e:
        urb.Int8Matrix.from_packed(2, 3, np.zeros(6, np.uint8), np.ones(3, np.float32), ctx=ctx)
    assert e.value.code == native.ERR_SHAPE
    for bad in (0.0, -1.0, np.inf, np.nan):
        with pytest.raises(E) as e:
            urb.Int8Matrix.from_packed(2, 3, np.zeros(6, np.uint8), np.array([1.0, bad], np.float32), ctx=ctx)
        assert e.value.code == native.ERR_NONFINITE
        with pytest.raises(E) as e:
            urb.Int4Matrix.from_packed(1, 4, 2, np.zeros(2, np.uint8), np.array([bad, 1.0], np.float32), ctx=ctx)
        assert e.value.code == native.ERR_NONFINITE
    with pytest.raises(E) as e:
        urb.Int4Matrix.quantize_grouped(2, 3, 2, [1.0, 2.0, np.inf, 0.0, 0.0, 0.0], ctx=ctx)
    assert e.value.code == native.ERR_NONFINITE
    m = urb.Int8Matrix.from_packed(2, 3, np.ones(6, np.uint8), np.ones(2, np.float32), ctx=ctx)
    with pytest.raises(E) as e:
        m.matvec([1.0, np.nan, 0.0])
    assert e.value.code == native.ERR_NONFINITE
    with pytest.raises(E) as e:
        m.matvec_rows(1, 2, [1.0, 1.0, 0.0])
    assert e.value.code == native.ERR_SHAPE
    with pytest.raises(E) as e:
        m.write_rows(2, 1)
    assert e.value.code == native.ERR_SHAPE


def test_int_device_status_flags_nonfinite_input(ctx):
    import torch
    g = syn.rng(5)
    m = urb.Int4Matrix.quantize_grouped(64, 256, 64, g.standard_normal(64 * 256).astype(np.float32), ctx=ctx)
    x = torch.randn(3, 256, device="cuda")
    x[2, 17] = float("inf")
    y = torch.empty(3, 64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    m.matmul_rows_device(x.data_ptr(), 3, y.data_ptr(), status.data_ptr())
    ctx.synchronize()
    assert int(status.item()) == native.ERR_NONFINITE


@pytest.mark.parametrize("kinds,tokens", [
    (("int4", "int4", "int4"), 1),    # GLM INT4 expert, decode
    (("int4", "int4", "int4"), 5),
    (("int8", "int8", "int8"), 3),
    (("int8", "int4", "f32"), 2),     # GatedMlp::new_mixed (mlp.rs:60-81)
])
def test_int_gated_mlp_matches_oracle(oracle, ctx, kinds, tokens):
    # GatedMlp::forward (src/model/mlp.rs:90-99) over INT projections: three row products and
    # f32 SwiGLU with libm expf.  Bar: the product bar above carried through SwiGLU, written as
    # |gpu - oracle| <= 1e-5 * max|oracle| + 4 ulp per element.
    hidden, inter = 1024, 512
    g = syn.rng(hash(kinds) % 1000 + tokens)

    def make(kind, rows, cols):
        if kind == "int8":
            return int8_pair(oracle, ctx, g, rows, cols)
        if kind == "int4":
            return int4_pair(oracle, ctx, g, rows, cols, 64)
        v = (g.standard_normal((rows, cols)) * 0.03).astype(np.float32)
        return urb.DenseMatrix.new(rows, cols, v, ctx=ctx), oracle.Matrix(oracle.F32, rows, cols, v)

    (dg, og), (du, ou), (dd, od) = make(kinds[0], inter, hidden), make(kinds[1], inter, hidden), \
        make(kinds[2], hidden, inter)
    x = g.standard_normal((tokens, hidden)).astype(np.float32)
    got = urb.GatedMlp(dg, du, dd).forward_batch(x, tokens)
    want = np.stack([oracle.gated_mlp_forward(og, ou, od, x[t]) for t in range(tokens)])
    err = np.abs(got.astype(np.float64) - want)
    bound = 1e-5 * np.abs(want).max() + 4 * np.spacing(np.abs(want)).astype(np.float64)
    assert np.all(err <= bound), float((err - bound).max())


@pytest.mark.parametrize("kind,tokens", [("int4", 1), ("int4", 6), ("int8", 3)])
def test_int_expert_glm_layer_matches_oracle(oracle, ctx, kind, tokens):
    # RuntimeMoeLayer::forward (glm/runtime/moe.rs:138-176) with GLM's converted INT experts
    # (INT4 with 64-column groups, or INT8 per row), an INT shared expert and a BF16 router:
    # routes bit-exact; outputs within the INT product bar carried through SwiGLU and the f64
    # combine, |gpu - oracle| <= 1e-5 * max|oracle| + 4 ulp.
    from helpers import bf16_pair
    hidden, inter, E, K = 512, 256, 16, 4
    g = syn.rng(900 + tokens + (kind == "int8"))

    def mlp():
        mk = (lambda r, c: int4_pair(oracle, ctx, g, r, c, 64)) if kind == "int4" else \
            (lambda r, c: int8_pair(oracle, ctx, g, r, c))
        (dg, og), (du, ou), (dd, od) = mk(inter, hidden), mk(inter, hidden), mk(hidden, inter)
        return urb.GatedMlp(dg, du, dd), (og, ou, od)

    experts = [mlp() for _ in range(E)]
    shared = mlp()
    rdev, rorc = bf16_pair(oracle, ctx, g, E, hidden)
    bias = (g.standard_normal(E) * 0.01).astype(np.float32)
    geo = urb.MoeGeometry(top_k=K, routed_scaling_factor=2.5)
    layer = urb.RuntimeMoeLayer(rdev, bias, [e[0] for e in experts], shared[0], geo)
    ref = oracle.MoeLayer(rorc, bias, [e[1][0] for e in experts], [e[1][1] for e in experts],
                          [e[1][2] for e in experts], shared[1], top_k=K, scaling=2.5)
    x = g.standard_normal((tokens, hidden)).astype(np.float32)
    out, ids, w, extra = layer.forward_batch(x, tokens, details=True)
    r_out, r_ids, r_w, r_s, r_logits = ref.forward(x)
    assert np.array_equal(ids, r_ids)
    assert np.array_equal(bits(w), bits(r_w))
    assert np.array_equal(bits(extra["router_logits"]), bits(r_logits))
    want_counts = np.bincount(r_ids.ravel(), minlength=E)
    assert np.array_equal(extra["counts"], want_counts)
    err = np.abs(out.astype(np.float64) - r_out)
    bound = 1e-5 * np.abs(r_out).max() + 4 * np.spacing(np.abs(r_out)).astype(np.float64)
    assert np.all(err <= bound), float((err - bound).max())
    # The graph-capturable device entry point does not take these layers.
    import torch
    d_x = torch.from_numpy(x).cuda()
    d_out = torch.empty_like(d_x)
    torch.cuda.synchronize()
    with pytest.raises(urb.UrbError) as e:
        layer.forward_device(d_x.data_ptr(), tokens, d_out.data_ptr())
    assert e.value.code == native.ERR_UNSUPPORTED
