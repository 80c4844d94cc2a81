"""Pins the CPU oracle to the reference's own known-answer tests.

Each test replays a unit test of Urbilateria v0.2.4 (file:line cited) against the C++ oracle
(oracle/urb_oracle.cpp).  Where the reference test computes its expectation with a scalar
formula (ordered F64 / ordered F32 sums), the formula is re-implemented here independently in
numpy and compared bit for bit.
"""
import math
import os
import struct

import numpy as np
import pytest


def f32(x):
    return np.float32(x)


def bits(v):
    return struct.unpack("<I", struct.pack("<f", float(v)))[0]


# --- codecs ------------------------------------------------------------------------------------

def test_real_checkpoint_fp8_prefix_decodes_exactly(oracle):
    # src/math/mxfp.rs:2210-2214
    lib = oracle.lib()
    assert lib.urbo_decode_e4m3fn(0xE0) == -32.0
    assert lib.urbo_decode_e8m0(115) == 2.0 ** -12
    assert f32(lib.urbo_decode_e4m3fn(0xE0)) * f32(lib.urbo_decode_e8m0(115)) == f32(-0.0078125)


def test_e8m0_decode_matches_power_of_two_exhaustively(oracle):
    # src/math/mxfp.rs:2217-2224
    lib = oracle.lib()
    for code in range(0xFF):
        assert bits(lib.urbo_decode_e8m0(code)) == bits(np.ldexp(np.float32(1.0), code - 127))


def test_e4m3_decode_matches_ocp_definition_exhaustively(oracle):
    # src/math/mxfp.rs:2236-2300 checks the AVX2 decode against the scalar definition for all
    # 256 codes; the oracle's decode is checked against the OCP E4M3FN definition (ml_dtypes).
    ml_dtypes = pytest.importorskip("ml_dtypes")
    lib = oracle.lib()
    ref = np.arange(256, dtype=np.uint8).view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    for code in range(256):
        got = lib.urbo_decode_e4m3fn(code)
        if code & 0x7F == 0x7F:
            assert math.isnan(got)
        else:
            assert bits(got) == bits(ref[code]), hex(code)


def test_e4m3_encoder_roundtrips_every_finite_code(oracle):
    # encode_e4m3fn_finite (src/math/mxfp.rs:247-275) inverts the decoder on finite codes.
    lib = oracle.lib()
    for code in range(256):
        if code & 0x7F == 0x7F:
            continue
        v = lib.urbo_decode_e4m3fn(code)
        enc = lib.urbo_encode_e4m3fn(v)
        if v == 0.0:
            assert enc == 0  # -0.0 encodes to +0 (code 0) in the reference
        else:
            assert enc == code


def test_e2m1_table_low_nibble_first_golden(oracle):
    # src/math/mxfp.rs:2583-2591: packed [0x8c], scale 120 -> row [-0.015625, 0.0]; 0xFF rejected.
    m = oracle.Matrix(oracle.MXFP4, 1, 2, np.array([0x8C], np.uint8), np.array([120], np.uint8),
                      group_size=2)
    row = [m.matvec(np.array([1.0, 0.0], np.float32))[0],
           m.matvec(np.array([0.0, 1.0], np.float32))[0]]
    assert row == [-0.015625, 0.0]
    with pytest.raises(oracle.OracleError) as e:
        oracle.Matrix(oracle.MXFP4, 1, 2, np.array([0x8C], np.uint8), np.array([0xFF], np.uint8),
                      group_size=2)
    assert e.value.code == oracle.ERR_INVALID_SCALE


def test_fp8_block_scales_follow_both_matrix_axes(oracle):
    # src/math/mxfp.rs:2668-2675
    m = oracle.Matrix(oracle.MXFP8, 3, 3, np.full(9, 0x38, np.uint8),
                      np.array([127, 128, 129, 130], np.uint8), block_rows=2, block_cols=2)
    eye = np.eye(3, dtype=np.float32)
    rows = np.stack([m.matvec(eye[c]) for c in range(3)], axis=1)
    assert list(rows[0]) == [1.0, 1.0, 2.0]
    assert list(rows[2]) == [4.0, 4.0, 8.0]


# --- ordered dot products --------------------------------------------------------------------

def _input(cols):
    # ((index * 29 % 127) as f32 - 63.0) / 131.0
    return ((np.arange(cols) * 29 % 127).astype(np.float32) - f32(63.0)) / f32(131.0)


E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6], np.float32)


def _e8m0(code):
    return np.float32(2.0 ** (int(code) - 127)) if code else np.float32(2.0 ** -127)


def test_fp8_scalar_blocks_preserve_ordered_dot_bits_across_partial_blocks(oracle):
    # src/math/mxfp.rs:2678-2716
    import ml_dtypes
    rows = 35
    for block_rows, block_cols in [(32, 32), (128, 128)]:
        for cols in [1, 31, 32, 65, 129, 2049]:
            idx = np.arange(rows * cols)
            values = (((idx * 79 + 17) % 127) | ((idx % 2) * 128)).astype(np.uint8)
            scale_cols = -(-cols // block_cols)
            ns = -(-rows // block_rows) * scale_cols
            scales = (115 + np.arange(ns) % 19).astype(np.uint8)
            x = _input(cols)
            m = oracle.Matrix(oracle.MXFP8, rows, cols, values, scales, block_rows=block_rows,
                              block_cols=block_cols)
            got = m.matvec_rows(1, rows - 2, x)
            dec = values.view(ml_dtypes.float8_e4m3fn).astype(np.float32).reshape(rows, cols)
            for i, r in enumerate(range(1, rows - 1)):
                acc = 0.0
                for c in range(cols):
                    w = dec[r, c] * _e8m0(scales[(r // block_rows) * scale_cols + c // block_cols])
                    acc += float(np.float32(w)) * float(x[c])
                assert bits(got[i]) == bits(np.float32(acc)), (block_rows, cols, r)


def test_fp4_fp32_groups_preserve_ordered_dot_bits_across_odd_nibble_boundaries(oracle):
    # src/math/mxfp.rs:2719-2759
    rows = 35
    for cols in [1, 31, 32, 65, 2049]:
        for group in [1, 3, 7, 32, 33]:
            row_bytes = -(-cols // 2)
            groups = -(-cols // group)
            packed = ((np.arange(rows * row_bytes) * 83 + 11) % 256).astype(np.uint8)
            scales = (115 + np.arange(rows * groups) % 19).astype(np.uint8)
            x = _input(cols)
            m = oracle.Matrix(oracle.MXFP4, rows, cols, packed, scales, group_size=group)
            got = m.matvec_fp32(x, start=1, count=rows - 2)
            for i, r in enumerate(range(1, rows - 1)):
                acc = np.float32(0.0)
                for c in range(cols):
                    byte = packed[r * row_bytes + c // 2]
                    code = byte & 15 if c % 2 == 0 else byte >> 4
                    s = _e8m0(scales[r * groups + c // group])
                    acc = np.float32(acc + np.float32(np.float32(E2M1[code] * s) * x[c]))
                assert bits(got[i]) == bits(acc), (cols, group, r)


ADVERSARIAL = np.array([0.0, -0.0, np.float32(1.4e-45), -np.float32(1.4e-45),
                        np.finfo(np.float32).tiny, -np.finfo(np.float32).tiny, 0.5, -0.5,
                        np.finfo(np.float32).max / np.float32(8), -np.finfo(np.float32).max / np.float32(8),
                        16777216.0, 1.0, -16777216.0], dtype=np.float32)


def _f64_ordered(packed, scales, x, group):
    acc = 0.0
    for c in range(x.size):
        byte = packed[c // 2]
        code = byte & 15 if c % 2 == 0 else byte >> 4
        w = np.float32(E2M1[code] * _e8m0(scales[c // group]))
        acc += float(w) * float(x[c])
    return np.float32(acc)


@pytest.mark.parametrize("group", [8, 10, 16, 32, 34, 128])
def test_fp4_ordered_matches_formula_for_extreme_scales_and_partial_groups(oracle, group):
    # src/math/mxfp.rs:2763-2834 (the scalar formula is the expectation there).
    with np.errstate(all="ignore"):
        for cols in [1, 7, 8, 9, 15, 16, 17, 31, 32, 33, 65, 129]:
            x = ADVERSARIAL[np.arange(cols) % ADVERSARIAL.size]
            for scale in [0, 1, 2, 125, 126, 127, 128, 251, 252, 253, 254]:
                for code in (0, 1, 7, 8, 9, 15):
                    packed = np.full(-(-cols // 2), code | ((15 - code) << 4), np.uint8)
                    scales = np.full(-(-cols // group), scale, np.uint8)
                    m = oracle.Matrix(oracle.MXFP4, 1, cols, packed, scales, group_size=group)
                    got = m.matvec(x)[0]
                    want = _f64_ordered(packed, scales, x, group)
                    if np.isnan(want):
                        assert np.isnan(got)
                    else:
                        assert bits(got) == bits(want), (cols, scale, code)
    m = oracle.Matrix(oracle.MXFP4, 1, 32, np.full(16, 0x22, np.uint8), np.array([127], np.uint8))
    for bad in [np.inf, -np.inf, np.nan]:
        x = np.ones(32, np.float32)
        x[7] = bad
        with pytest.raises(oracle.OracleError) as e:
            m.matvec_fp32(x)
        assert e.value.code == oracle.ERR_NONFINITE


def test_mxfp8_fma_lanes_within_fp32_accumulation_error(oracle):
    # src/math/mxfp.rs:2296-2343: |actual - F64| <= 64 eps sum|p|.
    import ml_dtypes
    rows, cols = 17, 97
    codes = np.array([0x00, 0x07, 0x18, 0x38, 0x48, 0x70, 0x7E, 0xB8, 0xFE], np.uint8)
    values = codes[(np.arange(rows * cols) * 17) % codes.size]
    scale_cols = -(-cols // 32)
    scales = (119 + (np.arange(rows * scale_cols) * 13) % 17).astype(np.uint8)
    x = ((np.arange(cols) * 29 % 127).astype(np.float32) - f32(63)) / f32(128)
    m = oracle.Matrix(oracle.MXFP8, rows, cols, values, scales, block_rows=1, block_cols=32)
    got = m.matvec(x)
    dec = values.view(ml_dtypes.float8_e4m3fn).astype(np.float64).reshape(rows, cols)
    for r in range(rows):
        w = dec[r] * np.array([2.0 ** (int(scales[r * scale_cols + c // 32]) - 127)
                               for c in range(cols)])
        p = w * x.astype(np.float64)
        err = abs(float(got[r]) - p.sum())
        assert err <= 64 * np.finfo(np.float32).eps * max(np.abs(p).sum(), 1.0)


def test_batched_equals_independent_matvec_bits(oracle):
    # src/math/mxfp.rs:2595-2665 (MXFP4) and :2347 (MXFP8): batched == per-token, bitwise.
    g = np.random.default_rng(7)
    rows, cols = 17, 129
    packed = g.integers(0, 256, (rows, 65), dtype=np.uint8)
    scales = g.integers(118, 128, (rows, 5), dtype=np.uint8)
    m4 = oracle.Matrix(oracle.MXFP4, rows, cols, packed, scales, group_size=32)
    v8 = g.integers(0, 0x7E, (rows, 128), dtype=np.uint8)
    s8 = g.integers(118, 128, (rows, 4), dtype=np.uint8)
    m8 = oracle.Matrix(oracle.MXFP8, rows, 128, v8, s8, block_rows=1, block_cols=32)
    for m, c in ((m4, cols), (m8, 128)):
        for batch in [2, 3, 7, 12, 13, 25]:
            x = g.standard_normal((batch, c)).astype(np.float32)
            got = m.matmul_rows(x, batch)
            want = np.stack([m.matvec(x[t]) for t in range(batch)])
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# --- routing -----------------------------------------------------------------------------------

def test_correction_bias_changes_selection_but_not_gate_weight(oracle):
    # src/math/routing.rs:162-174
    e, w, _ = oracle.route_noaux_tc([2.0, 1.0, 0.0, -1.0], [0.0] * 4, 2, 1, 1, False, 1.0)
    assert list(e) == [0, 1]
    e, w, _ = oracle.route_noaux_tc([2.0, 1.0, 0.0, -1.0], [0.0, 0.0, 2.0, 0.0], 2, 1, 1,
                                    False, 1.0)
    assert list(e) == [2, 0]
    assert abs(w[0] - 0.5) < 1e-6


def test_normalized_weights_sum_to_routed_scale(oracle):
    # src/math/routing.rs:176-181
    _, w, _ = oracle.route_noaux_tc([3.0, 2.0, 1.0, 0.0], [0.0] * 4, 3, 1, 1, True, 2.5)
    assert abs(float(np.sum(w, dtype=np.float32)) - 2.5) < 1e-6


def test_grouped_router_masks_losing_groups(oracle):
    # src/math/routing.rs:183-196
    e, _, _ = oracle.route_noaux_tc([3.0, 2.0, -3.0, -4.0, 1.0, 0.5, 0.0, -1.0], [0.0] * 8,
                                    2, 2, 1, True, 1.0)
    assert all(x < 4 for x in e)


def test_normalization_epsilon_matches_underflowed_router(oracle):
    # src/math/routing.rs:198-204
    e, w, _ = oracle.route_noaux_tc([-1000.0] * 4, [0.0] * 4, 2, 1, 1, True, 2.5)
    assert len(e) == 2 and all(x == 0.0 for x in w)


def test_896_expert_tie_order(oracle):
    # src/models/kimi_k3/moe.rs:778-796 (tie order of the same noaux_tc selection rule).
    bias = np.zeros(896, np.float32)
    bias[895] = 1.0
    e, w, s = oracle.route_noaux_tc(np.zeros(896, np.float32), bias, 16, 1, 1, True, 1.0)
    assert e[0] == 895 and list(e[1:]) == list(range(15))
    assert s[0] == 1.5
    assert all(abs(x - 1.0 / 16.0) < 1e-7 for x in w)


def test_softmax_router_tie_break_and_renormalisation(oracle):
    # src/models/qwen3_8/moe.rs:446-466
    e, w = oracle.route_softmax_top_k([2.0, 2.0, 2.0, 1.0], 2)
    assert list(e) == [0, 1] and all(abs(x - 0.5) < 1e-7 for x in w)
    e, w = oracle.route_softmax_top_k(np.log(np.array([4.0, 2.0, 1.0], np.float32)), 2)
    assert list(e) == [0, 1]
    assert abs(w[0] - 2 / 3) < 1e-6 and abs(w[1] - 1 / 3) < 1e-6


def test_route_geometry_errors(oracle):
    # src/math/routing.rs:47-99 validation order.
    with pytest.raises(oracle.OracleError) as e:
        oracle.route_noaux_tc([0.0, np.nan], [0.0, 0.0], 1, 1, 1, True, 1.0)
    assert e.value.code == oracle.ERR_NONFINITE
    with pytest.raises(oracle.OracleError) as e:
        oracle.route_noaux_tc([0.0] * 4, [0.0] * 4, 1, 3, 1, True, 1.0)
    assert e.value.code == oracle.ERR_INVALID_GEOMETRY
    with pytest.raises(oracle.OracleError) as e:
        oracle.route_noaux_tc([0.0] * 4, [0.0] * 4, 1, 1, 1, True, 0.0)
    assert e.value.code == oracle.ERR_INVALID_GEOMETRY


# --- SwiGLU / grouping -----------------------------------------------------------------------

def test_gated_mlp_matches_explicit_formula(oracle):
    # src/model/mlp.rs:107-117
    gate = oracle.Matrix(oracle.F32, 2, 2, np.array([1, 0, 0, 1], np.float32))
    up = oracle.Matrix(oracle.F32, 2, 2, np.array([2, 0, 0, 3], np.float32))
    down = oracle.Matrix(oracle.F32, 2, 2, np.array([1, 1, 1, -1], np.float32))
    out = oracle.gated_mlp_forward(gate, up, down, np.array([1.0, -2.0], np.float32))
    silu = lambda v: v / (1 + math.exp(-v))
    first, second = silu(1.0) * 2.0, silu(-2.0) * -6.0
    assert abs(out[0] - (first + second)) < 1e-6
    assert abs(out[1] - (first - second)) < 1e-6


def test_grouping_is_experts_then_tokens_ascending(oracle):
    # src/models/qwen3_6/runtime.rs:1123-1132: BTreeMap by expert over token-major routes.
    g = np.random.default_rng(3)
    ids = np.stack([g.choice(37, 6, replace=False) for _ in range(50)]).astype(np.int32)
    counts, offsets, pt, ps = oracle.group_routes(ids, 37)
    order = sorted(range(ids.size), key=lambda i: (ids.flat[i], i))
    assert list(pt) == [i // 6 for i in order]
    assert list(ps) == [i % 6 for i in order]
    assert list(counts) == list(np.bincount(ids.ravel(), minlength=37))
    assert offsets[-1] == ids.size


# ---- checkpoint numerics (DeepSeek-V4), pinned by the reference's own tests ----------------

def test_e4m3_activation_simulation_golden(oracle):
    # src/math/mxfp.rs:2885-2889 (activation_simulation_uses_power_of_two_blocks).
    v = oracle.simulate_e4m3_activation([448.0, 0.1, 896.0, -896.0], 2)
    assert v[0] == 448.0 and v[2] == 896.0 and v[3] == -896.0


def test_power_of_two_ceiling_matches_float_formula(oracle):
    # src/math/mxfp.rs:2893-2917: bitwise equal to 2^ceil(log2(v)) (glibc log2f / powf) on the
    # bands around powers of two and on seeded interior mantissas, for every exponent.
    rng = np.random.default_rng(7)
    for exponent in range(0, 255, 3):
        mants = list(range(0, 8193, 97)) + list(range(0x7FFFFF - 8192, 0x800000, 97))
        mants += [int(m) for m in rng.integers(0, 0x800000, size=64)]
        for m in mants:
            v = np.uint32((exponent << 23) | m).view(np.float32)
            if not np.isfinite(v) or v <= 0:
                continue
            got = np.float32(oracle.power_of_two_ceiling(float(v)))
            ref = np.float32(2.0) ** np.ceil(np.log2(v))
            assert got == ref, (exponent, m, got, ref)


def test_round_bf16_and_bounded_swiglu_golden(oracle):
    # deepseek_v4/math.rs:788-798 (bounded_swiglu_clamps_the_two_branches_asymmetrically).
    a = oracle.bounded_swiglu(20.0, 20.0, 10.0)
    assert abs(a - 10.0 / (1.0 + math.exp(-10.0)) * 10.0) < 1e-5
    b = oracle.bounded_swiglu(-20.0, -20.0, 10.0)
    assert 0.0 < b < 1e-6
    # Round to nearest even on the upper half: 1 + 2^-8 is a tie (stays 1), 1 + 3*2^-8 rounds up.
    assert oracle.round_bf16(1.0 + 2.0 ** -8) == 1.0
    assert oracle.round_bf16(1.0 + 3 * 2.0 ** -8) == 1.0 + 2.0 ** -6
    assert oracle.round_bf16(-2.5) == -2.5



def test_route_sqrt_softplus_golden(oracle):
    # deepseek_v4/math.rs:764-775 (hash_router_uses_fixed_ids_but_learned_weights).
    e, w, _ = oracle.route_sqrt_softplus([0.0, 1.0, 2.0, 3.0], None, [3, 0], 2, 1.5)
    assert list(e) == [3, 0]
    assert abs(float(np.sum(w)) - 1.5) < 1e-6
    # :778-786 (correction_bias_selects_but_does_not_weight).
    e, w, _ = oracle.route_sqrt_softplus([3.0, 2.0, 1.0], None, None, 1, 1.0)
    assert e[0] == 0
    e, w, _ = oracle.route_sqrt_softplus([3.0, 2.0, 1.0], [0.0, 0.0, 10.0], None, 1, 1.0)
    assert e[0] == 2 and w[0] == 1.0


# ---- checkpoint numerics (Qwen3.6) ------------------------------------------------------------

def test_finegrained_e4m3_golden(oracle):
    # src/math/mxfp.rs:2949-2955 (finegrained_activation_uses_exact_absmax_scale).
    v = oracle.simulate_finegrained_e4m3([1.0, 0.3, 0.0, 0.0], 2)
    assert v[0] == 1.0
    assert abs(v[1] - oracle.lib().urbo_decode_e4m3fn(0x70) / 448.0) < 1e-7
    assert v[2] == 0.0 and v[3] == 0.0


def test_bf16_fp32_lanes_formula(oracle):
    # The eight-lane FMA tree of src/model/bf16.rs:591-613, restated in numpy (FMA via f64: a
    # bf16 x f32 product is exact in f64 and one rounding of product + lane equals fma), over
    # the shapes of the reference's own tests (:860-887, :903-920: 1..2048 columns, tails).
    def bf16(v):
        b = np.asarray(v, np.float32).view(np.uint32)
        return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    for cols in [1, 7, 8, 9, 31, 65, 512, 2048]:
        w = bf16([((i * 137 % 251) - 125.0) / 37.0 for i in range(cols)])
        x = np.array([((i * 19 % 97) - 48.0) / 31.0 for i in range(cols)], np.float32)
        wf = (w.astype(np.uint32) << 16).view(np.float32)
        lanes = np.zeros(8, np.float32)
        complete = cols // 8 * 8
        for c in range(complete):
            lanes[c % 8] = np.float32(np.float64(wf[c]) * np.float64(x[c]) + np.float64(lanes[c % 8]))
        s = np.float32(-0.0)
        for v in lanes:
            s = np.float32(s + v)
        for c in range(complete, cols):
            s = np.float32(s + np.float32(wf[c] * x[c]))
        assert bits(oracle.dot_bf16_fp32_lanes(w, x)) == bits(s), cols


def test_transpose_rows_matvec_golden(oracle):
    # src/model/bf16.rs:960-974 and src/model/weight.rs:425-440: W = [[-1, 2], [3, -4]].
    def bf16(v):
        return (np.asarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)
    for m in (oracle.Matrix(oracle.BF16, 2, 2, bf16([-1.0, 2.0, 3.0, -4.0])),
              oracle.Matrix(oracle.F32, 2, 2, np.array([-1.0, 2.0, 3.0, -4.0], np.float32))):
        assert list(m.transpose_rows_matvec(0, [0.5, 2.0])) == [5.5, -7.0]
        assert list(m.transpose_rows_matvec(1, [2.0])) == [6.0, -8.0]
        assert list(m.transpose_rows_matvec(2, [])) == [0.0, 0.0]
        with pytest.raises(oracle.OracleError):
            m.transpose_rows_matvec(1, [1.0, 1.0])
        with pytest.raises(oracle.OracleError):
            m.transpose_rows_matvec(0, [np.inf])


def test_transpose_rows_matvec_formula(oracle):
    # Ordered f64 column sums (mxfp.rs:785-858, 1782-1821) restated in numpy over decoded
    # weights, MXFP4 with odd columns and MXFP8 with 2 x 64 scale blocks.
    from urbilateria_b200 import synthetic as syn
    g = syn.rng(4242)
    packed, scales = syn.mxfp4_matrix(g, 9, 37)
    m4 = oracle.Matrix(oracle.MXFP4, 9, 37, packed, scales, group_size=32)
    vals = syn.encode_e4m3fn(g.standard_normal((9, 130)).astype(np.float32))
    sc8 = g.integers(117, 124, size=(5, 3), dtype=np.uint8)
    m8 = oracle.Matrix(oracle.MXFP8, 9, 130, vals, sc8, block_rows=2, block_cols=64)
    x = (g.standard_normal(6) * 3).astype(np.float32)
    for m, dec in ((m4, lambda r, c: oracle.lib().urbo_decode_e2m1(
                        int(packed[r, c // 2]) >> (4 * (c % 2)) & 15) *
                    oracle.lib().urbo_decode_e8m0(int(scales[r, c // 32]))),
                   (m8, lambda r, c: oracle.lib().urbo_decode_e4m3fn(int(vals[r, c])) *
                    oracle.lib().urbo_decode_e8m0(int(sc8[r // 2, c // 64])))):
        got = m.transpose_rows_matvec(2, x)
        for c in range(m.cols):
            s = 0.0
            for i in range(6):
                s += float(np.float32(x[i])) * float(np.float32(dec(2 + i, c)))
            assert np.float32(s) == got[c], c


# --- INT8 per-row / INT4 grouped (GLM converted checkpoints) -----------------------------------

def _seq_f64(pairs, start=0.0):
    """Ordered f64 sum of exact widened products, as the reference's scalar loops."""
    s = start
    for w, v in pairs:
        s = s + float(np.float32(w)) * float(np.float32(v))
    return s


def test_int8_twos_complement_bytes_and_row_scales(oracle):
    # src/math/quant.rs:694-720
    m = oracle.Matrix(oracle.INT8, 2, 3, np.array([0xff, 0x00, 0x7f, 0x80, 0x02, 0xfe], np.uint8),
                      np.array([0.5, 0.25], np.float32))
    assert list(m.write_row(0)) == [-0.5, 0.0, 63.5]
    assert list(m.write_row(1)) == [-32.0, 0.5, -0.5]
    x = np.array([2.0, -1.0, 0.5], np.float32)
    explicit = [np.float32(sum(np.float32(w) * np.float32(v) for w, v in zip(m.write_row(r), x)))
                for r in range(2)]
    assert list(m.matvec(x)) == explicit


def test_int_formats_share_matvec_and_row_contracts(oracle):
    # src/model/weight.rs:416-442 (the INT8 and INT4 matrices of the mixed-format test)
    i8 = oracle.Matrix(oracle.INT8, 2, 2, np.array([0xff, 2, 3, 0xfc], np.uint8),
                       np.array([1.0, 1.0], np.float32))
    i4 = oracle.Matrix(oracle.INT4, 2, 2, np.array([0xa7, 0x4b], np.uint8),
                       np.array([1.0, 1.0], np.float32), group_size=2)
    for m in (i8, i4):
        assert list(m.write_row(0)) == [-1.0, 2.0]
        assert list(m.matvec(np.array([0.5, 2.0], np.float32))) == [3.5, -6.5]
        assert list(m.matmul_rows(np.array([0.5, 2.0, 1.0, -1.0], np.float32), 2).ravel()) == \
            [3.5, -6.5, -3.0, 7.0]
        assert list(m.transpose_rows_matvec(0, [0.5, 2.0])) == [5.5, -7.0]
        assert list(m.transpose_rows_matvec(1, [2.0])) == [6.0, -8.0]
        assert list(m.matvec_rows(1, 1, np.array([0.5, 2.0], np.float32))) == [-6.5]


def test_int4_packs_low_nibble_first_with_zero_tail(oracle):
    # src/math/quant.rs:622-631
    packed, scales = oracle.int4_quantize_grouped(1, 3, 3, [-8.0, 7.0, 0.0])
    assert packed.size == 2
    assert packed[0] & 0x0F == 1 and packed[0] >> 4 == 14
    assert packed[1] & 0x0F == 8 and packed[1] >> 4 == 8
    assert scales[0] == np.float32(8.0) / np.float32(7.0)


def test_int4_grouped_scales_reduce_outlier_damage(oracle):
    # src/math/quant.rs:633-641
    values = [100.0, 0.5, 0.5, 0.5]
    per_row = oracle.Matrix(oracle.INT4, 1, 4, *oracle.int4_quantize_grouped(1, 4, 4, values),
                            group_size=4)
    grouped = oracle.Matrix(oracle.INT4, 1, 4, *oracle.int4_quantize_grouped(1, 4, 2, values),
                            group_size=2)
    assert abs(grouped.write_row(0)[2] - 0.5) < abs(per_row.write_row(0)[2] - 0.5)


def test_int4_matvec_matches_explicit_dequantization(oracle):
    # src/math/quant.rs:643-660
    packed, scales = oracle.int4_quantize_grouped(2, 4, 2, [1.0, -2.0, 3.0, 4.0, -1.0, 0.5, 2.0, -3.0])
    m = oracle.Matrix(oracle.INT4, 2, 4, packed, scales, group_size=2)
    x = np.array([0.25, 2.0, -1.0, 0.5], np.float32)
    for r, actual in enumerate(m.matvec(x)):
        expected = np.float32(sum(np.float32(w) * v for w, v in zip(m.write_row(r), x)))
        assert abs(actual - expected) < 1e-5


def test_int4_row_range_kernels_handle_odd_groups_and_tail_nibbles(oracle):
    # src/math/quant.rs:662-691: 3 x 7 with 3-column groups; bit-exact ordered f64 sums.
    values = [np.float32((np.float32(i) - np.float32(10.0)) * np.float32(0.17)) for i in range(21)]
    packed, scales = oracle.int4_quantize_grouped(3, 7, 3, values)
    m = oracle.Matrix(oracle.INT4, 3, 7, packed, scales, group_size=3)
    x = np.array([0.2, -0.4, 0.6, -0.8, 1.0, -1.2, 1.4], np.float32)
    for off, actual in enumerate(m.matvec_rows(1, 2, x)):
        assert bits(actual) == bits(np.float32(_seq_f64(zip(m.write_row(off + 1), x))))
    t = m.transpose_rows_matvec(1, [0.25, -0.75])
    for c in range(7):
        expected = np.float32(_seq_f64([(m.write_row(r)[c], v) for r, v in zip((1, 2), (0.25, -0.75))]))
        assert bits(t[c]) == bits(expected)


def _rust_i8_rem31(index):
    """`(index as i8 % 31)`: wrapping cast to i8, then Rust's truncating remainder."""
    v = ((index & 0xFF) ^ 0x80) - 0x80
    return v % 31 if v >= 0 else -((-v) % 31)


def test_int_large_kernels_bit_exact_against_ordered_scalar_dots(oracle):
    # src/model/weight.rs:497-616, the INT8 and INT4 matrices (65 x 1025).
    rows, cols = 65, 1025
    x = np.array([(c % 17 - 8.0) / 16.0 for c in range(cols)], np.float32)
    tx = np.array([(r % 11 - 5.0) / 8.0 for r in range(rows)], np.float32)
    i8 = oracle.Matrix(oracle.INT8, rows, cols,
                       np.array([_rust_i8_rem31(i) & 0xFF for i in range(rows * cols)], np.uint8),
                       np.full(rows, 0.03125, np.float32))
    i4 = oracle.Matrix(oracle.INT4, rows, cols,
                       np.array([(i * 37) & 0xFF for i in range(rows * ((cols + 1) // 2))], np.uint8),
                       np.full(rows * ((cols + 63) // 64), 0.0625, np.float32), group_size=64)
    for m in (i8, i4):
        mat = np.stack([m.write_row(r) for r in range(rows)])
        y = m.matvec(x)
        for r in range(rows):
            assert bits(y[r]) == bits(np.float32(_seq_f64(zip(mat[r], x), -0.0)))
        t = m.transpose_rows_matvec(0, tx)
        for c in range(0, cols, 7):
            assert bits(t[c]) == bits(np.float32(_seq_f64(zip(mat[:, c], tx))))


def test_int_constructor_validation(oracle):
    # quant.rs:92-131 (group size, shape, then scales finite and positive), :363-396
    with pytest.raises(oracle.OracleError) as e:
        oracle.Matrix(oracle.INT4, 1, 2, np.zeros(1, np.uint8), np.ones(1, np.float32), group_size=0)
    assert e.value.code == oracle.ERR_INVALID_GROUP
    for bad in (0.0, -1.0, np.inf, np.nan):
        for fmt, vals in ((oracle.INT8, np.zeros(2, np.uint8)), (oracle.INT4, np.zeros(1, np.uint8))):
            with pytest.raises(oracle.OracleError) as e:
                oracle.Matrix(fmt, 1, 2, vals, np.array([bad], np.float32), group_size=2)
            assert e.value.code == oracle.ERR_NONFINITE
    with pytest.raises(oracle.OracleError) as e:
        oracle.int4_quantize_grouped(1, 2, 2, [1.0, np.nan])
    assert e.value.code == oracle.ERR_NONFINITE


def _fixture_close(name, got, want):
    """The reference fixture test's tolerance (deepseek_v4/runtime.rs:4221-4230):
    |got - want| <= max(2e-5, 2e-5 * |want|) elementwise."""
    got = np.asarray(got, np.float32).ravel()
    want = np.asarray(want, np.float32).ravel()
    assert got.shape == want.shape, name
    tol = np.maximum(np.float32(2e-5), np.abs(want) * np.float32(2e-5))
    assert np.all(np.abs(got - want) <= tol), (name, got, want)


def test_deepseek_v4_tiny_fixture_moe_layer(oracle):
    """The reference's layer-level fixture (tests/fixtures/deepseek_v4_tiny_oracle.json, replayed
    at src/models/deepseek_v4/runtime.rs:4603-4646): hash-routed MoE with F32 experts.  Router
    logits, routes, each routed expert's output (route weight before the down projection), the
    shared expert and the BF16 MoE branch."""
    import json
    d = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "deepseek_v4_tiny_moe.json")))
    H, E, K = d["hidden"], d["experts"], d["top_k"]
    limit, scale = np.float32(d["swiglu_limit"]), np.float32(d["routed_scaling_factor"])

    def mat(t):
        r, c = t["shape"]
        return oracle.Matrix(oracle.F32, r, c, np.array(t["values"], np.float32))

    router = mat(d["router"])
    routed = [(mat(e["w1"]), mat(e["w3"]), mat(e["w2"])) for e in d["routed"]]
    shared = (mat(d["shared"]["w1"]), mat(d["shared"]["w3"]), mat(d["shared"]["w2"]))
    x = np.array(d["ffn_input"], np.float32)
    want = d["expected"]
    logits = router.matvec(x)
    _fixture_close("router logits", logits, want["router_logits"])
    ids, w, sel = oracle.route_sqrt_softplus(logits, None, d["hash_experts"], K, scale)
    assert ids.tolist() == [r["expert"] for r in want["routes"]]
    _fixture_close("route weight", w, [r["weight"] for r in want["routes"]])
    _fixture_close("route selection score", sel, [r["selection_score"] for r in want["routes"]])
    for k in range(K):
        g, u, dn = routed[ids[k]]
        y = oracle.deepseek_expert_forward(g, u, dn, x, limit, route_weight=w[k])
        _fixture_close("routed expert %d" % k, y, want["routed_experts"][k])
    _fixture_close("shared expert", oracle.deepseek_expert_forward(*shared, x, limit),
                   want["shared_expert"])
    layer = oracle.MoeLayer(router, np.zeros(E, np.float32), [m[0] for m in routed],
                            [m[1] for m in routed], [m[2] for m in routed], shared, top_k=K,
                            scaling=float(scale))
    out, e, lw = oracle.moe_deepseek_layer_forward(layer, x, float(limit),
                                                   hash_experts=np.array([d["hash_experts"]]))
    assert e.ravel().tolist() == ids.tolist()
    _fixture_close("moe branch", out, want["moe_branch"])
