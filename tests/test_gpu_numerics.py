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
