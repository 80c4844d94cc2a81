"""Parity at the benchmark configs' full shapes (3 and 4), against the oracle.

* C2: the MXFP4 MoE layer of src/models/glm/runtime/moe.rs:138-176 at hidden 7168 with 256
  routed experts + 1 shared expert (intermediate 2048), a 128-token chunk: router logits,
  top-8 ids, weights and selection scores bit-exact for every token; outputs of 16 tokens
  (spread over the chunk) within the parity bar.
* C3: 128 MXFP8 experts (hidden 4096, intermediate 1536, E4M3 + E8M0 1x32) over 512 tokens
  with Zipf(1.1) top-8 routes: the grouping (counts, permutation) bit-exact, and the outputs of
  tokens routed to the head expert (which takes ~460 tokens, i.e. 15 sub-segments of 32 in
  the grouped passes) and to tail experts, against the oracle's GatedMlp (the reference's
  AVX2-FMA lane order) with the f64 route-order combine.
* C4: one 384-routed-expert layer of the stacked decode (config-2 routing) at B = 1, 8 and 64
  tokens: routes bit-exact for every token, outputs of up to 8 tokens within the bar.

Every comparison prints the relative L2 error, the literal max-abs error and the max-abs error
over the reference output's RMS (the normalised form the parity bar applies, see helpers.py).
"""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

from helpers import MAX_ABS, REL_L2, rel_err

pytestmark = pytest.mark.gpu

HIDDEN, INTER, TOP_K, SCALE = 7168, 2048, 8, 2.5


def report(name, got, want):
    """Prints relL2 / literal max-abs / normalised max-abs and applies the parity bar."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    rel, mx_norm = rel_err(got, want)
    mx = float(np.abs(got - want).max())
    rms = float(np.sqrt(np.mean(want * want)))
    print("%s: relL2=%.3e max_abs=%.3e (output rms %.3e, max|ref| %.3e) max_abs/rms=%.3e"
          % (name, rel, mx, rms, float(np.abs(want).max()), mx_norm))
    assert rel <= REL_L2 and mx_norm <= MAX_ABS, name


def mxfp4_layer(oracle, ctx, g, experts, hidden=HIDDEN, inter=INTER):
    """A config-2 style layer: routed MXFP4 experts + 1 shared (E8M0 119..127), bf16 router
    ~N(0, 0.02), bias ~N(0, 0.01), noaux_tc top-8 x2.5; device and oracle views of the same
    bytes."""
    dev_e, orc_e = [], []
    for _ in range(experts + 1):
        mats = [syn.mxfp4_matrix(g, r, c) for r, c in ((inter, hidden), (inter, hidden), (hidden, inter))]
        dev_e.append(urb.GatedMlp(*[urb.MxFp4Matrix.from_packed(r, c, 32, p, s, ctx=ctx)
                                    for (p, s), (r, c) in zip(mats, ((inter, hidden), (inter, hidden),
                                                                     (hidden, inter)))]))
        orc_e.append(tuple(oracle.Matrix(oracle.MXFP4, r, c, p, s, group_size=32, validate=False)
                           for (p, s), (r, c) in zip(mats, ((inter, hidden), (inter, hidden),
                                                            (hidden, inter)))))
    bits = syn.bf16_normal(g, (experts, hidden), 0.02)
    bias = syn.normal_f32(g, experts, 0.01)
    router = urb.Bf16Matrix.from_bits(experts, hidden, bits, ctx=ctx)
    geo = urb.MoeGeometry(TOP_K, 1, 1, True, SCALE)
    dev = urb.RuntimeMoeLayer(router, bias, dev_e[:experts], dev_e[experts], geo)
    orouter = oracle.Matrix(oracle.BF16, experts, hidden, bits)
    orc = oracle.MoeLayer(orouter, bias, [m[0] for m in orc_e[:experts]], [m[1] for m in orc_e[:experts]],
                          [m[2] for m in orc_e[:experts]], orc_e[experts], TOP_K, 1, 1, True, SCALE)

    def free():
        dev.free()
        for e in dev_e:
            for m in (e.gate, e.up, e.down):
                m.free()
        router.free()
    return dev, orc, orouter, bias, free


def check_routes(oracle, orouter, bias, x, ids, w, score, logits):
    """Router logits, ids, weights and selection scores of every token, bit for bit."""
    for t in range(x.shape[0]):
        lg = orouter.matvec(x[t])
        assert np.array_equal(lg.view(np.uint32), logits[t].view(np.uint32)), t
        e, wt, s = oracle.route_noaux_tc(lg, bias, TOP_K, 1, 1, True, SCALE)
        assert np.array_equal(e, ids[t]), t
        assert np.array_equal(np.asarray(wt, np.float32).view(np.uint32), w[t].view(np.uint32)), t
        assert np.array_equal(np.asarray(s, np.float32).view(np.uint32), score[t].view(np.uint32)), t


def test_c2_full_layer(oracle, ctx):
    g = syn.rng(20261201)
    dev, orc, orouter, bias, free = mxfp4_layer(oracle, ctx, g, 256)
    T = 128
    x = syn.normal_bf16_as_f32(g, (T, HIDDEN))
    out, ids, w, extra = dev.forward_batch(x, T, details=True)
    check_routes(oracle, orouter, bias, x, ids, w, extra["selection_score"], extra["router_logits"])
    sample = np.linspace(0, T - 1, 16).astype(int)
    o_out, o_ids = orc.forward(x[sample])[:2]
    assert np.array_equal(o_ids, ids[sample])
    report("C2 16 of 128 tokens", out[sample], o_out)
    print("C2 touched experts: %d" % int((extra["counts"] > 0).sum()))
    free()


def test_c3_full_grouped_mxfp8(oracle, ctx):
    g = syn.rng(20261203)
    H, I, E, T, K = 4096, 1536, 128, 512, 8
    # E4M3 payloads (fp8-cast N(0,1)) are drawn for a pool of 12 matrices (a gate/up and a down
    # payload have the same size), each expert projection takes one of them with its own
    # E8M0 scales (uniform 117..123), so all 384 uploads differ.
    pool = [syn.encode_e4m3fn(g.standard_normal(I * H, dtype=np.float32)) for _ in range(12)]
    dev_e, orc_e = [], []
    for e in range(E):
        dm, om = [], []
        for j, (r, c) in enumerate(((I, H), (I, H), (H, I))):
            v = pool[(3 * e + j) % len(pool)].reshape(r, c)
            s = g.integers(117, 124, size=(r, c // 32), dtype=np.uint8)
            dm.append(urb.MxFp8Matrix.from_packed(r, c, 1, 32, v, s, ctx=ctx))
            om.append(oracle.Matrix(oracle.MXFP8, r, c, v, s, block_rows=1, block_cols=32,
                                    validate=False))
        dev_e.append(urb.GatedMlp(*dm))
        orc_e.append(tuple(om))
    router = urb.Bf16Matrix.from_bits(E, H, syn.bf16_normal(g, (E, H), 0.02), ctx=ctx)
    layer = urb.RuntimeMoeLayer(router, np.zeros(E, np.float32), dev_e, None,
                                urb.MoeGeometry(K, 1, 1, True, 1.0))
    x = syn.normal_bf16_as_f32(g, (T, H))
    ids = syn.zipf_routes(g, T, E, K).astype(np.int32)
    w = g.random((T, K)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    # Grouping of these routes (qwen3_6/runtime.rs:1083-1132) bit-exact.
    counts, offsets, ptok, pslot = urb.group_routes(ids, E, ctx=ctx)
    o_counts, o_offsets, o_tok, o_slot = oracle.group_routes(ids, E)
    assert np.array_equal(counts, o_counts) and np.array_equal(offsets, o_offsets)
    assert np.array_equal(ptok, o_tok) and np.array_equal(pslot, o_slot)
    got = layer.forward_routed(x, T, ids, w)
    head = int(np.argmax(counts))
    head_tokens = np.nonzero((ids == head).any(axis=1))[0]
    print("C3 head expert %d: %d tokens" % (head, head_tokens.size))
    assert head_tokens.size > 15 * 32 - 32  # the head expert spans many 32-token sub-segments
    # Tokens of the head expert spread over its sub-segments, plus tokens of the tail.
    pick = list(head_tokens[np.linspace(0, head_tokens.size - 1, 12).astype(int)])
    tail = [t for t in range(T) if head not in ids[t]][:4]
    pick = np.array(sorted(set(pick + tail)))
    want = np.empty((pick.size, H), np.float32)
    for i, t in enumerate(pick):
        acc = np.zeros(H, np.float64)
        for k in range(K):
            y = oracle.gated_mlp_forward(*orc_e[ids[t, k]], x[t])
            acc = acc + np.float64(w[t, k]) * y.astype(np.float64)
        want[i] = acc.astype(np.float32)
    report("C3 %d tokens (head expert + tail)" % pick.size, got[pick], want)
    layer.free()
    for e in dev_e:
        for m in (e.gate, e.up, e.down):
            m.free()
    router.free()


def test_c4_full_layer_decode_batches(oracle, ctx):
    g = syn.rng(20261204)
    dev, orc, orouter, bias, free = mxfp4_layer(oracle, ctx, g, 384)
    for B in (1, 8, 64):
        x = syn.normal_bf16_as_f32(g, (B, HIDDEN))
        out, ids, w, extra = dev.forward_batch(x, B, details=True)
        check_routes(oracle, orouter, bias, x, ids, w, extra["selection_score"],
                     extra["router_logits"])
        sample = np.linspace(0, B - 1, min(B, 8)).astype(int)
        o_out, o_ids = orc.forward(x[sample])[:2]
        assert np.array_equal(o_ids, ids[sample])
        report("C4 B=%d (%d tokens checked)" % (B, sample.size), out[sample], o_out)
    free()
