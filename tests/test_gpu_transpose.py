"""WeightMatrix::transpose_rows_matvec (src/model/weight.rs:332-343) on the device against the
oracle, bit for bit: every format sums a column over the row range in order in f64 and rounds
once, so the device's ordered f64 chain lands on the same f32.  Covers the reference's golden
case (bf16.rs:960-974, weight.rs:425-440), every weight copy the device keeps (row-major
uploads and the block-scaled tiles), ragged shapes, empty ranges and the error order."""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

from helpers import bf16_pair, mxfp4_pair, mxfp8_pair

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_transpose_golden(ctx):
    b = (np.array([-1.0, 2.0, 3.0, -4.0], np.float32).view(np.uint32) >> 16).astype(np.uint16)
    for m in (urb.Bf16Matrix.from_bits(2, 2, b, ctx=ctx),
              urb.DenseMatrix.new(2, 2, np.array([-1.0, 2.0, 3.0, -4.0], np.float32), ctx=ctx)):
        assert list(m.transpose_matvec([0.5, 2.0])) == [5.5, -7.0]
        assert list(m.transpose_rows_matvec(1, [2.0])) == [6.0, -8.0]
        assert list(m.transpose_rows_matvec(2, [])) == [0.0, 0.0]


@pytest.mark.parametrize("kind,rows,cols,start,n", [
    ("mxfp4", 300, 7168, 130, 100),   # block-scaled tiles, ragged last row tile
    ("mxfp4g16", 40, 300, 3, 37),     # 16-column groups: the row-major upload
    ("mxfp8", 700, 1536, 0, 700),     # 1 x 32 blocks: tiles
    ("mxfp8b", 300, 1536, 17, 255),   # 128 x 128 blocks: tiles
    ("mxfp8r", 64, 200, 5, 50),       # 16-column blocks: the row-major upload
    ("bf16", 257, 1001, 1, 256),
    ("f32", 33, 70, 0, 33),
])
def test_transpose_matches_oracle(oracle, ctx, kind, rows, cols, start, n):
    g = syn.rng(rows * 31 + cols)
    if kind == "mxfp4":
        dev, orc = mxfp4_pair(oracle, ctx, g, rows, cols)
    elif kind == "mxfp4g16":
        dev, orc = mxfp4_pair(oracle, ctx, g, rows, cols, group=16)
    elif kind == "mxfp8":
        dev, orc = mxfp8_pair(oracle, ctx, g, rows, cols)
    elif kind == "mxfp8b":
        dev, orc = mxfp8_pair(oracle, ctx, g, rows, cols, 128, 128)
    elif kind == "mxfp8r":
        dev, orc = mxfp8_pair(oracle, ctx, g, rows, cols, 2, 16)
    elif kind == "bf16":
        dev, orc = bf16_pair(oracle, ctx, g, rows, cols, std=0.5)
    else:
        w = syn.normal_f32(g, (rows, cols))
        dev = urb.DenseMatrix.new(rows, cols, w, ctx=ctx)
        orc = oracle.Matrix(oracle.F32, rows, cols, w)
    x = (g.standard_normal(n) * np.exp2(g.integers(-8, 8, n))).astype(np.float32)
    got = dev.transpose_rows_matvec(start, x)
    want = orc.transpose_rows_matvec(start, x)
    assert np.array_equal(bits(got), bits(want))


def test_transpose_errors(ctx):
    g = syn.rng(5)
    packed, scales = syn.mxfp4_matrix(g, 8, 64)
    m = urb.MxFp4Matrix.from_packed(8, 64, 32, packed, scales, ctx=ctx)
    with pytest.raises(urb.UrbError) as e:
        m.transpose_rows_matvec(7, [np.nan, 1.0])  # non-finite is reported before the range
    assert e.value.kind == "NonFinite"
    with pytest.raises(urb.UrbError) as e:
        m.transpose_rows_matvec(7, [1.0, 1.0])
    assert e.value.kind == "Shape"
    with pytest.raises(urb.UrbError) as e:
        m.transpose_matvec(np.ones(7, np.float32))
    assert e.value.kind == "Shape"
    # MXFP8 rejects outputs that overflow f32 (mxfp.rs:851-856).
    vals = np.full((2, 32), 0x7E, np.uint8)
    big = urb.MxFp8Matrix.from_packed(2, 32, 1, 32, vals, np.full((2, 1), 254, np.uint8), ctx=ctx)
    with pytest.raises(urb.UrbError) as e:
        big.transpose_rows_matvec(0, [3e38, 3e38])
    assert e.value.kind == "NonFinite"
