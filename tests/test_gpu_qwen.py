"""Qwen3.6 checkpoint numerics on the GPU against the oracle: the fine-grained E4M3 activation
simulation (src/math/mxfp.rs:122-149) and the FP32-lane BF16 linear (qwen3_8/math.rs:10-26 over
dot_bf16_fp32_avx2_fma, src/model/bf16.rs:591-613) bit for bit; the layer forward of
execute_batched_moe (qwen3_6/runtime.rs:1067-1215: BF16 router, softmax top-k with BF16 weights,
BF16 boundaries, expert-order BF16 accumulation, sigmoid-gated shared expert) with routes
bit-exact and outputs within the parity bar."""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

from helpers import assert_close, bf16_pair, mxfp4_pair, mxfp8_pair, rel_err

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def test_finegrained_e4m3_golden(oracle, ctx):
    # src/math/mxfp.rs:2949-2955 (finegrained_activation_uses_exact_absmax_scale).
    got = urb.simulate_finegrained_e4m3_activation([1.0, 0.3, 0.0, 0.0], 2, ctx=ctx)
    assert got[0] == 1.0
    assert abs(got[1] - oracle.lib().urbo_decode_e4m3fn(0x70) / 448.0) < 1e-7
    assert got[2] == 0.0 and got[3] == 0.0


@pytest.mark.parametrize("block", [1, 7, 32, 128, 1000])
def test_finegrained_e4m3_matches_oracle(oracle, ctx, block):
    g = syn.rng(9800 + block)
    v = (g.standard_normal(4099) * np.exp2(g.integers(-30, 30, 4099))).astype(np.float32)
    v[256:384] = 0.0  # an all-zero block stays zero
    v[5] = 448.0 * 3.0
    got = urb.simulate_finegrained_e4m3_activation(v, block, ctx=ctx)
    want = oracle.simulate_finegrained_e4m3(v, block)
    assert np.array_equal(bits(got), bits(want))


def test_finegrained_e4m3_rejects(ctx):
    with pytest.raises(urb.UrbError) as e:
        urb.simulate_finegrained_e4m3_activation([1.0, np.nan], 2, ctx=ctx)
    assert e.value.kind == "NonFinite"
    with pytest.raises(urb.UrbError) as e:
        urb.simulate_finegrained_e4m3_activation([1.0], 0, ctx=ctx)
    assert e.value.kind == "Shape"


@pytest.mark.parametrize("cols", [1, 7, 8, 9, 31, 65, 301, 2048])
def test_linear_bf16_fp32_lanes_bit_exact(oracle, ctx, cols):
    # The lane order, the -0.0 start of the lane sum and the unfused tail: with activations over
    # 2^-20..2^20 the FP32 rounding of every step shows, so only the same tree matches.
    g = syn.rng(9900 + cols)
    rows, tokens = 37, 6
    wbits = syn.bf16_normal(g, (rows, cols), 1.0)
    wd = urb.Bf16Matrix.from_bits(rows, cols, wbits, ctx=ctx)
    x = (g.standard_normal((tokens, cols)) * np.exp2(g.integers(-20, 20, (tokens, cols))))
    x = x.astype(np.float32)
    got = urb.linear_bf16_fp32_lanes(wd, x, tokens)
    for t in range(tokens):
        for r in range(rows):
            want = oracle.round_bf16(oracle.dot_bf16_fp32_lanes(wbits[r], x[t]))
            assert bits(got[t, r]) == bits(want), (t, r)


def build_qwen_layer(oracle, ctx, g, hidden, inter, experts, fmt, top_k):
    pair = {"bf16": bf16_pair, "mxfp4": mxfp4_pair, "mxfp8": mxfp8_pair}[fmt]
    dev_e, og, ou, od = [], [], [], []
    for _ in range(experts + 1):  # routed experts, then the shared expert
        gd, go = pair(oracle, ctx, g, inter, hidden)
        ud, uo = pair(oracle, ctx, g, inter, hidden)
        dd, do = pair(oracle, ctx, g, hidden, inter)
        dev_e.append(urb.GatedMlp(gd, ud, dd))
        og.append(go); ou.append(uo); od.append(do)
    rd, ro = bf16_pair(oracle, ctx, g, experts, hidden, std=0.05)
    gate_d, gate_o = bf16_pair(oracle, ctx, g, 1, hidden, std=0.05)
    bias = np.zeros(experts, np.float32)
    geo = urb.MoeGeometry(top_k, 1, 1, True, 1.0)
    dev = urb.RuntimeMoeLayer(rd, bias, dev_e[:experts], dev_e[experts], geo)
    dev.set_shared_expert_gate(gate_d)
    orc = oracle.MoeLayer(ro, bias, og[:experts], ou[:experts], od[:experts],
                          (og[experts], ou[experts], od[experts]), top_k, 1, 1, True, 1.0)
    return dev, orc, gate_o


@pytest.mark.parametrize("fmt,tokens", [("bf16", 1), ("bf16", 21), ("mxfp4", 19), ("mxfp8", 13)])
def test_qwen36_layer_forward(oracle, ctx, fmt, tokens):
    g = syn.rng(9700 + tokens)
    hidden, inter, experts, k = 512, 256, 32, 8
    dev, orc, gate_o = build_qwen_layer(oracle, ctx, g, hidden, inter, experts, fmt, k)
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    out, ids, w = dev.forward_ex(x, tokens, numerics="qwen36")
    o_out, o_ids, o_w = oracle.moe_qwen_layer_forward(orc, gate_o, x)
    assert np.array_equal(ids, o_ids)
    assert np.array_equal(bits(w), bits(o_w))
    r, m = rel_err(out, o_out)
    print("qwen36 layer %s T=%d relL2=%.3e maxabs=%.3e" % (fmt, tokens, r, m))
    assert np.abs(o_out).max() > 1e-3
    assert_close(out, o_out)
    # Outputs are BF16 values.
    assert np.all((bits(out) & 0xFFFF) == 0)


@pytest.mark.parametrize("fmt", ["bf16", "mxfp4"])
def test_qwen36_routed_composition(oracle, ctx, fmt):
    # The oracle's routes passed in by the caller: the same experts half of the forward.
    g = syn.rng(9650)
    hidden, inter, experts, k, tokens = 256, 128, 16, 4, 9
    dev, orc, gate_o = build_qwen_layer(oracle, ctx, g, hidden, inter, experts, fmt, k)
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    _, o_ids, o_w = oracle.moe_qwen_layer_forward(orc, gate_o, x)
    out = dev.forward_routed(x, tokens, o_ids, o_w, numerics="qwen36")
    o_out, _, _ = oracle.moe_qwen_layer_forward(orc, gate_o, x)
    assert_close(out, o_out)


def test_qwen36_requires_gate_and_bf16_router(oracle, ctx):
    g = syn.rng(9600)
    dev, orc, _ = build_qwen_layer(oracle, ctx, g, 256, 128, 16, "bf16", 4)
    x = syn.normal_bf16_as_f32(g, (3, 256))
    bad, _ = bf16_pair(oracle, ctx, g, 2, 256)
    with pytest.raises(urb.UrbError) as e:
        dev.set_shared_expert_gate(bad)
    assert e.value.kind == "Shape"
    dev.set_shared_expert_gate(None)
    with pytest.raises(urb.UrbError) as e:
        dev.forward_ex(x, 3, numerics="qwen36")
    assert e.value.kind == "Unsupported"
    with pytest.raises(urb.UrbError) as e:
        dev.forward_ex(x, 3, numerics="qwen36", hash_experts=np.zeros((3, 4), np.int32))
    assert e.value.kind == "InvalidArgument"


def test_qwen36_rejects_nonfinite_router(oracle, ctx):
    g = syn.rng(9601)
    dev, _, _ = build_qwen_layer(oracle, ctx, g, 256, 128, 16, "bf16", 4)
    x = syn.normal_bf16_as_f32(g, (2, 256))
    x[1, 7] = np.inf
    with pytest.raises(urb.UrbError) as e:
        dev.forward_ex(x, 2, numerics="qwen36")
    assert e.value.kind == "NonFinite"


def test_qwen36_bf16_layer_records_into_a_cuda_graph(oracle):
    # BF16 experts run the tcgen05 kind::f16 passes, whose device forward makes no host copy or
    # synchronisation: with caller routes it records into a CUDA graph (after one call has
    # sized the context's workspace) and the replay reproduces the eager output bit for bit.
    import ctypes
    import torch
    from urbilateria_b200 import native
    c = urb.Context(0)
    stream = torch.cuda.Stream()
    c.set_stream(stream.cuda_stream)
    g = syn.rng(9800)
    hidden, inter, experts, k, tokens = 256, 128, 16, 4, 11
    dev, orc, gate_o = build_qwen_layer(oracle, c, g, hidden, inter, experts, "bf16", k)
    x = syn.normal_f32(g, (tokens, hidden))
    o_out, o_ids, o_w = oracle.moe_qwen_layer_forward(orc, gate_o, x)
    want = dev.forward_routed(x, tokens, o_ids, o_w, numerics="qwen36")
    assert_close(want, o_out)
    d_x = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    d_ids = torch.from_numpy(np.ascontiguousarray(o_ids, np.int32)).cuda()
    d_w = torch.from_numpy(np.ascontiguousarray(o_w, np.float32)).cuda()
    d_out = torch.zeros_like(d_x)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    num = native.Numerics(2, 0.0)

    def call():
        c.check(c.lib.urb_moe_forward_routed_ex_device(c.h, dev.h, d_x.data_ptr(), tokens,
                                                       d_ids.data_ptr(), d_w.data_ptr(),
                                                       ctypes.byref(num), d_out.data_ptr(),
                                                       st.data_ptr()))
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        call()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        call()
    d_out.zero_()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert np.array_equal(bits(d_out.cpu().numpy()), bits(want))
    del graph
    dev.free()
    c.close()  # objects still holding this context drop their handles (Matrix.free)
