"""Bit-exact routing on the device: route_noaux_tc, route_softmax_top_k, libm-exact sigmoid,
the token->expert grouping, and the router logits of the MoE layer."""
import os

import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def oracle_routes(oracle, logits, bias, k, n_group=1, topk_group=1, normalize=True, scale=2.5):
    out = [oracle.route_noaux_tc(l, bias, k, n_group, topk_group, normalize, scale) for l in logits]
    return (np.stack([o[0] for o in out]), np.stack([o[1] for o in out]),
            np.stack([o[2] for o in out]))


@pytest.mark.parametrize("experts,k,n_group,topk_group", [(256, 8, 1, 1), (384, 8, 1, 1),
                                                          (256, 8, 8, 4), (64, 6, 4, 2),
                                                          (896, 16, 1, 1)])
def test_noaux_tc_bit_exact(oracle, ctx, experts, k, n_group, topk_group):
    g = syn.rng(experts + k)
    logits = syn.normal_f32(g, (128, experts), 1.7)
    bias = syn.normal_f32(g, experts, 0.01)
    ids, w, s = urb.route_noaux_tc(logits, bias, k, n_group, topk_group, True, 2.5, ctx=ctx)
    oi, ow, os_ = oracle_routes(oracle, logits, bias, k, n_group, topk_group)
    assert np.array_equal(ids, oi)
    assert np.array_equal(w.view(np.uint32), ow.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))


def test_reference_router_cases(ctx):
    # src/math/routing.rs:162-204 and src/models/kimi_k3/moe.rs:778-796.
    r = urb.route_noaux_tc([2.0, 1.0, 0.0, -1.0], [0.0] * 4, 2, 1, 1, False, 1.0, ctx=ctx)
    assert [c.expert for c in r] == [0, 1]
    r = urb.route_noaux_tc([2.0, 1.0, 0.0, -1.0], [0, 0, 2.0, 0], 2, 1, 1, False, 1.0, ctx=ctx)
    assert [c.expert for c in r] == [2, 0] and abs(r[0].weight - 0.5) < 1e-6
    r = urb.route_noaux_tc([3.0, 2.0, 1.0, 0.0], [0.0] * 4, 3, 1, 1, True, 2.5, ctx=ctx)
    assert abs(sum(np.float32(c.weight) for c in r) - 2.5) < 1e-6
    r = urb.route_noaux_tc([3, 2, -3, -4, 1, 0.5, 0, -1], [0.0] * 8, 2, 2, 1, True, 1.0, ctx=ctx)
    assert all(c.expert < 4 for c in r)
    r = urb.route_noaux_tc([-1000.0] * 4, [0.0] * 4, 2, 1, 1, True, 2.5, ctx=ctx)
    assert all(c.weight == 0.0 for c in r)
    bias = np.zeros(896, np.float32)
    bias[895] = 1.0
    r = urb.route_noaux_tc(np.zeros(896, np.float32), bias, 16, 1, 1, True, 1.0, ctx=ctx)
    assert [c.expert for c in r] == [895] + list(range(15)) and r[0].selection_score == 1.5
    with pytest.raises(urb.UrbError) as e:
        urb.route_noaux_tc([0.0, np.inf], [0.0, 0.0], 1, 1, 1, True, 1.0, ctx=ctx)
    assert e.value.kind == "NonFinite"
    with pytest.raises(urb.UrbError) as e:
        urb.route_noaux_tc([0.0] * 4, [0.0] * 4, 1, 3, 1, True, 1.0, ctx=ctx)
    assert e.value.kind == "InvalidGeometry"


def test_sigmoid_matches_libm_expf_on_exception_inputs(oracle, ctx):
    # The selection score with zero bias is the gate 1/(1+expf(-logit)) itself.  Logits are
    # drawn from the inputs where libm expf is not a single rounding of exp (the embedded
    # table), plus random ones.
    table = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                         "urbilateria_b200", "csrc", "_gen", "expf_table.bin")
    pairs = np.fromfile(table, dtype=np.uint32).reshape(-1, 2)
    g = syn.rng(99)
    keys = pairs[g.choice(len(pairs), 8192, replace=False), 0].view(np.float32)
    logits = -keys[np.abs(keys) < 80]
    logits = np.concatenate([logits, syn.normal_f32(g, 4096, 3.0)])
    n = logits.size // 256 * 256
    logits = logits[:n].reshape(-1, 256).astype(np.float32)
    ids, _, s = urb.route_noaux_tc(logits, np.zeros(256, np.float32), 256, 1, 1, False, 1.0,
                                   ctx=ctx)
    lib = oracle.lib()
    for t in range(logits.shape[0]):
        for j in range(256):
            e = ids[t, j]
            want = np.float32(1.0) / (np.float32(1.0) + np.float32(lib.urbo_expf(-logits[t, e])))
            assert s[t, j].view(np.uint32) == np.float32(want).view(np.uint32)


def test_softmax_top_k_bit_exact(oracle, ctx):
    g = syn.rng(5)
    logits = syn.normal_f32(g, (64, 256), 2.0)
    ids, w = urb.route_softmax_top_k(logits, 8, ctx=ctx)
    for t in range(64):
        oe, ow = oracle.route_softmax_top_k(logits[t], 8)
        assert np.array_equal(ids[t], oe)
        assert np.array_equal(w[t].view(np.uint32), ow.view(np.uint32))
    r = urb.route_softmax_top_k(np.array([2.0, 2.0, 2.0, 1.0], np.float32), 2, ctx=ctx)
    assert [e for e, _ in r] == [0, 1]


@pytest.mark.parametrize("tokens,experts,k", [(128, 256, 8), (512, 128, 8), (1, 384, 8),
                                              (64, 384, 8), (3, 7, 2)])
def test_grouping_bit_exact(oracle, ctx, tokens, experts, k):
    g = syn.rng(tokens * 31 + experts)
    ids = syn.zipf_routes(g, tokens, experts, k) if experts == 128 else \
        np.stack([g.choice(experts, k, replace=False) for _ in range(tokens)]).astype(np.int32)
    got = urb.group_routes(ids, experts, ctx=ctx)
    want = oracle.group_routes(ids, experts)
    for a, b in zip(got, want):
        assert np.array_equal(a, b)
