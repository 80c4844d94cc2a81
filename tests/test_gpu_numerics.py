"""Checkpoint numerics (DeepSeek-V4) on the GPU against the oracle: the E4M3 activation
simulation bit for bit (src/math/mxfp.rs:91-115, including power_of_two_ceiling's band near
powers of two, :300-319), and the DeepSeek-V4 routed-expert composition (E4M3-simulated inputs,
BF16 boundaries, bounded SwiGLU, route weight before the down projection, f32 expert-order
combine; deepseek_v4/runtime.rs:2500-2650, :3081-3104) within the parity bar."""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

from helpers import assert_close, rel_err
from test_gpu_moe import build_layer

pytestmark = pytest.mark.gpu


def test_simulate_e4m3_golden(oracle, ctx):
    # src/math/mxfp.rs:2885-2889.
    got = urb.simulate_e4m3_activation([448.0, 0.1, 896.0, -896.0], 2, ctx=ctx)
    assert got[0] == 448.0 and got[2] == 896.0 and got[3] == -896.0
    want = oracle.simulate_e4m3_activation([448.0, 0.1, 896.0, -896.0], 2)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("block", [1, 2, 3, 7, 32, 128, 1000])
def test_simulate_e4m3_matches_oracle(oracle, ctx, block):
    g = syn.rng(9700 + block)
    mant = g.uniform(1.0, 2.0, 4096)
    expo = g.integers(-30, 20, 4096)
    sign = np.where(g.random(4096) < 0.5, -1.0, 1.0)
    x = (sign * mant * np.exp2(expo)).astype(np.float32)
    x[::11] = 0.0
    got = urb.simulate_e4m3_activation(x, block, ctx=ctx)
    want = oracle.simulate_e4m3_activation(x, block)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_simulate_e4m3_power_of_two_band(oracle, ctx):
    # Block maxima whose max/448 falls within 4,096 mantissa units of a power of two, where the
    # reference keeps 2^ceil(log2f(v)) instead of the exponent step.
    vals = []
    for k in (-40, -12, -3, 0, 5, 30):
        for j in list(range(0, 5000, 37)) + list(range(0x7FFFFF - 5000, 0x800000, 41)):
            v = np.uint32((127 + k) << 23 | j).view(np.float32) * np.float32(448.0)
            vals.append([v, np.float32(0.3) * v, -np.float32(0.7) * v, np.float32(1e-3) * v])
    x = np.array(vals, np.float32).ravel()
    got = urb.simulate_e4m3_activation(x, 4, ctx=ctx)
    want = oracle.simulate_e4m3_activation(x, 4)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("fmt,limit", [("mxfp4", 7.0), ("mxfp4", 1e4), ("mxfp8", 7.0)])
def test_deepseek_v4_routed_composition(oracle, ctx, fmt, limit):
    g = syn.rng(9800 + int(limit))
    hidden, inter, experts, k, tokens = 512, 256, 16, 4, 21
    dev, orc = build_layer(oracle, ctx, g, hidden, inter, experts, fmt, top_k=k, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    ids = np.stack([g.permutation(experts)[:k] for _ in range(tokens)]).astype(np.int32)
    w = g.uniform(0.05, 1.5, (tokens, k)).astype(np.float32)
    got = dev.forward_routed(x, tokens, ids, w, numerics="deepseek_v4", swiglu_limit=limit)
    want = oracle.moe_deepseek_forward(orc, x, ids, w, limit)
    r, m = rel_err(got, want)
    print("%s limit %g relL2=%.3e maxabs=%.3e" % (fmt, limit, r, m))
    assert np.linalg.norm(want) > 0 and np.abs(want).max() > 1e-3
    assert_close(got, want)
    # Outputs are BF16 values.
    assert np.all((got.view(np.uint32) & 0xFFFF) == 0)


def test_deepseek_v4_rejects_bad_weights_and_limits(oracle, ctx):
    g = syn.rng(9900)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 8, "mxfp4", top_k=2, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (2, 256))
    ids = np.array([[0, 1], [2, 3]], np.int32)
    with pytest.raises(urb.UrbError) as e:
        dev.forward_routed(x, 2, ids, np.array([[0.5, -0.1], [1, 1]], np.float32),
                           numerics="deepseek_v4", swiglu_limit=7.0)
    assert e.value.kind == "InvalidArgument"
    with pytest.raises(urb.UrbError) as e:
        dev.forward_routed(x, 2, ids, np.ones((2, 2), np.float32), numerics="deepseek_v4",
                           swiglu_limit=0.0)
    assert e.value.kind == "InvalidArgument"
    # The GLM numerics of the same call are unaffected.
    dev.forward_routed(x, 2, ids, np.ones((2, 2), np.float32))


def test_route_sqrt_softplus_golden_device(oracle, ctx):
    # deepseek_v4/math.rs:764-786.
    e, w, _ = urb.route_sqrt_softplus([0.0, 1.0, 2.0, 3.0], None, [[3, 0]], 2, 1.5, ctx=ctx)
    assert list(e[0]) == [3, 0] and abs(float(w.sum()) - 1.5) < 1e-6
    e, w, _ = urb.route_sqrt_softplus([3.0, 2.0, 1.0], None, None, 1, 1.0, ctx=ctx)
    assert e[0, 0] == 0
    e, w, _ = urb.route_sqrt_softplus([3.0, 2.0, 1.0], [0.0, 0.0, 10.0], None, 1, 1.0, ctx=ctx)
    assert e[0, 0] == 2 and w[0, 0] == 1.0


@pytest.mark.parametrize("with_bias,with_hash", [(True, False), (False, False), (True, True)])
def test_route_sqrt_softplus_matches_oracle(oracle, ctx, with_bias, with_hash):
    g = syn.rng(9950 + 2 * with_bias + with_hash)
    tokens, experts, k = 96, 256, 8
    logits = (g.standard_normal((tokens, experts)) * 4.0).astype(np.float32)
    logits[:, ::17] = np.float32(-120.0)   # softplus underflows toward 0
    logits[:, 5::29] = np.float32(90.0)    # v + log1p(exp(-v)) branch, exp(-v) tiny
    logits[3, :] = 0.25                    # every selection ties: lower ids win
    bias = syn.normal_f32(g, experts, 0.01) if with_bias else None
    hash_ids = np.stack([g.permutation(experts)[:k] for _ in range(tokens)]).astype(np.int32) \
        if with_hash else None
    e, w, s = urb.route_sqrt_softplus(logits, bias, hash_ids, k, 2.5, ctx=ctx)
    for t in range(tokens):
        oe, ow, os_ = oracle.route_sqrt_softplus(logits[t], bias,
                                                 None if hash_ids is None else hash_ids[t], k, 2.5)
        assert np.array_equal(e[t], oe), t
        assert np.array_equal(w[t].view(np.uint32), ow.view(np.uint32)), t
        assert np.array_equal(s[t].view(np.uint32), os_.view(np.uint32)), t


@pytest.mark.parametrize("use_hash", [False, True])
def test_deepseek_v4_layer_forward(oracle, ctx, use_hash):
    g = syn.rng(9960 + use_hash)
    hidden, inter, experts, k, tokens = 512, 256, 32, 6, 19
    dev, orc = build_layer(oracle, ctx, g, hidden, inter, experts, "mxfp4", top_k=k, scale=2.5)
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    h = np.stack([g.permutation(experts)[:k] for _ in range(tokens)]).astype(np.int32) \
        if use_hash else None
    out, ids, w = dev.forward_ex(x, tokens, numerics="deepseek_v4", swiglu_limit=10.0,
                                 hash_experts=h)
    o_out, o_ids, o_w = oracle.moe_deepseek_layer_forward(orc, x, 10.0, hash_experts=h)
    assert np.array_equal(ids, o_ids)
    assert np.array_equal(w.view(np.uint32), o_w.view(np.uint32))
    r, m = rel_err(out, o_out)
    print("deepseek layer hash=%s relL2=%.3e maxabs=%.3e" % (use_hash, r, m))
    assert np.abs(o_out).max() > 1e-3
    assert_close(out, o_out)
