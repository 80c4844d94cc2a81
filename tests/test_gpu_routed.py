"""urb_moe_forward_routed: the grouped experts + combine for routes chosen by the caller.
Routes from the layer's own router reproduce urb_moe_forward bit for bit; softmax top-k routes
(src/models/qwen3_8/moe.rs:91-159) and config-3 style Zipf(1.1) routes over MXFP8 experts of
the config-3 shape (src/math/mxfp.rs 1x32 E8M0) match the oracle's GatedMlp per route with the
f64 combine of src/models/glm/runtime/moe.rs:164-175."""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

from helpers import assert_close, mxfp8_pair
from test_gpu_moe import build_layer

pytestmark = pytest.mark.gpu


def combine_ref(oracle, mats, shared, x, ids, w):
    """f32(f64(shared(x)) + sum_k f64(w_k) * f64(expert_{ids_k}(x))), routes in given order."""
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        acc = oracle.gated_mlp_forward(*shared, x[t]).astype(np.float64)
        for k in range(ids.shape[1]):
            y = oracle.gated_mlp_forward(*mats[ids[t, k]], x[t])
            acc = acc + np.float64(w[t, k]) * y.astype(np.float64)
        out[t] = acc.astype(np.float32)
    return out


@pytest.mark.parametrize("path", ["tc", "mma"])
def test_routed_with_own_routes_is_the_layer_forward(oracle, ctx, path, monkeypatch):
    monkeypatch.setenv("URB_MOE_PATH", path)
    g = syn.rng(8100)
    dev, _ = build_layer(oracle, ctx, g, 512, 256, 32, "mxfp4", top_k=8, scale=2.5)
    x = syn.normal_bf16_as_f32(g, (20, 512))
    out, ids, w, _ = dev.forward_batch(x, 20)
    got = dev.forward_routed(x, 20, ids, w)
    assert np.array_equal(got.view(np.uint32), out.view(np.uint32))


def test_routed_softmax_top_k_routes(oracle, ctx):
    g = syn.rng(8200)
    hidden, inter, experts, k, tokens = 256, 128, 16, 4, 11
    dev, orc = build_layer(oracle, ctx, g, hidden, inter, experts, "mxfp4", top_k=k, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    logits = orc.forward(x)[4]
    ids = np.empty((tokens, k), np.int32)
    w = np.empty((tokens, k), np.float32)
    for t in range(tokens):
        ids[t], w[t] = oracle.route_softmax_top_k(logits[t], k)
    got = dev.forward_routed(x, tokens, ids, w)
    mats = [(a, b, c) for a, b, c in zip(orc._keep[0], orc._keep[1], orc._keep[2])]
    assert_close(got, combine_ref(oracle, mats, orc._keep[3], x, ids, w))


def test_routed_c3_shape_zipf(oracle, ctx):
    # Config 3 shapes (hidden 4096, intermediate 1536, E4M3 + E8M0 1x32, scales 117..123) with
    # Zipf(1.1) top-8 routes over the experts; fewer experts and tokens than the full config so
    # the oracle finishes in seconds.
    g = syn.rng(8300)
    hidden, inter, experts, k, tokens = 4096, 1536, 12, 8, 24
    mats, orc_m, dev_e = [], [], []
    for _ in range(experts + 1):
        gd, go = mxfp8_pair(oracle, ctx, g, inter, hidden)
        ud, uo = mxfp8_pair(oracle, ctx, g, inter, hidden)
        dd, do = mxfp8_pair(oracle, ctx, g, hidden, inter)
        dev_e.append(urb.GatedMlp(gd, ud, dd))
        orc_m.append((go, uo, do))
    bits = syn.bf16_normal(g, (experts, hidden), 0.02)
    router = urb.Bf16Matrix.from_bits(experts, hidden, bits, ctx=ctx)
    layer = urb.RuntimeMoeLayer(router, np.zeros(experts, np.float32), dev_e[:experts],
                                dev_e[experts], urb.MoeGeometry(k, 1, 1, True, 1.0))
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    ids = syn.zipf_routes(g, tokens, experts, k).astype(np.int32)
    w = g.uniform(0.01, 0.3, size=(tokens, k)).astype(np.float32)
    got = layer.forward_routed(x, tokens, ids, w)
    assert_close(got, combine_ref(oracle, orc_m[:experts], orc_m[experts], x, ids, w))


def test_routed_rejects_bad_expert_ids(oracle, ctx):
    g = syn.rng(8400)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 16, "mxfp4", top_k=4, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (2, 256))
    ids = np.array([[0, 1, 2, 16], [3, 4, 5, 6]], np.int32)
    with pytest.raises(urb.UrbError) as e:
        dev.forward_routed(x, 2, ids, np.ones((2, 4), np.float32))
    assert e.value.kind == "Shape"
