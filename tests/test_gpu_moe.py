"""Parity of the device SwiGLU experts and the MoE layer with the GLM composition oracle
(src/models/glm/runtime/moe.rs:138-176).  Routes, counts and the permutation are bit-exact;
outputs within relative L2 1e-3 / max-abs 2e-2 (normalised)."""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import synthetic as syn

from helpers import assert_close, bf16_pair, mxfp4_pair, mxfp8_pair, profiled_kinds

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens", [1, 32])
def test_c1_bf16_swiglu(oracle, ctx, tokens):
    # hidden 2048, intermediate 768, bf16 N(0, 0.02), x bf16 N(0, 1).
    g = syn.rng(100 + tokens)
    gd, go = bf16_pair(oracle, ctx, g, 768, 2048)
    ud, uo = bf16_pair(oracle, ctx, g, 768, 2048)
    dd, do = bf16_pair(oracle, ctx, g, 2048, 768)
    x = syn.normal_bf16_as_f32(g, (tokens, 2048))
    got = urb.GatedMlp(gd, ud, dd).forward_batch(x, tokens)
    want = np.stack([oracle.gated_mlp_forward(go, uo, do, x[t]) for t in range(tokens)])
    assert_close(got, want)


def test_mxfp8_swiglu(oracle, ctx):
    g = syn.rng(7)
    gd, go = mxfp8_pair(oracle, ctx, g, 1536, 4096)
    ud, uo = mxfp8_pair(oracle, ctx, g, 1536, 4096)
    dd, do = mxfp8_pair(oracle, ctx, g, 4096, 1536)
    x = syn.normal_bf16_as_f32(g, (6, 4096))
    got = urb.GatedMlp(gd, ud, dd).forward_batch(x, 6)
    want = np.stack([oracle.gated_mlp_forward(go, uo, do, x[t]) for t in range(6)])
    assert_close(got, want)


def build_layer(oracle, ctx, g, hidden, inter, experts, fmt="mxfp4", top_k=8, n_group=1,
                topk_group=1, scale=2.5):
    pair = {"mxfp4": mxfp4_pair, "mxfp8": mxfp8_pair, "bf16": bf16_pair}[fmt]
    dev_e, orc_g, orc_u, orc_d = [], [], [], []
    for _ in range(experts):
        gd, go = pair(oracle, ctx, g, inter, hidden)
        ud, uo = pair(oracle, ctx, g, inter, hidden)
        dd, do = pair(oracle, ctx, g, hidden, inter)
        dev_e.append(urb.GatedMlp(gd, ud, dd))
        orc_g.append(go); orc_u.append(uo); orc_d.append(do)
    sg, sgo = pair(oracle, ctx, g, inter, hidden)
    su, suo = pair(oracle, ctx, g, inter, hidden)
    sd, sdo = pair(oracle, ctx, g, hidden, inter)
    rd, ro = bf16_pair(oracle, ctx, g, experts, hidden)
    bias = syn.normal_f32(g, experts, 0.01)
    geo = urb.MoeGeometry(top_k, n_group, topk_group, True, scale)
    dev = urb.RuntimeMoeLayer(rd, bias, dev_e, urb.GatedMlp(sg, su, sd), geo)
    orc = oracle.MoeLayer(ro, bias, orc_g, orc_u, orc_d, (sgo, suo, sdo), top_k, n_group,
                          topk_group, True, scale)
    return dev, orc


@pytest.mark.parametrize("fmt,tokens", [("mxfp4", 1), ("mxfp4", 24), ("mxfp8", 17), ("bf16", 1),
                                        ("bf16", 37)])
def test_moe_layer_reduced(oracle, ctx, fmt, tokens):
    g = syn.rng(300 + tokens)
    dev, orc = build_layer(oracle, ctx, g, 512, 256, 32, fmt)
    x = syn.normal_bf16_as_f32(g, (tokens, 512))
    out, ids, w, extra = dev.forward_batch(x, tokens, details=True)
    o_out, o_ids, o_w, o_s, o_logits = orc.forward(x)
    assert np.array_equal(extra["router_logits"].view(np.uint32), o_logits.view(np.uint32))
    assert np.array_equal(ids, o_ids)
    assert np.array_equal(w.view(np.uint32), o_w.view(np.uint32))
    counts, offsets, pt, ps = oracle.group_routes(o_ids, 32)
    assert np.array_equal(extra["counts"], counts)
    assert np.array_equal(extra["perm_token"], pt) and np.array_equal(extra["perm_slot"], ps)
    assert_close(out, o_out)


def test_moe_layer_grouped_router(oracle, ctx):
    g = syn.rng(77)
    dev, orc = build_layer(oracle, ctx, g, 256, 128, 16, "mxfp4", top_k=4, n_group=4,
                           topk_group=2, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (9, 256))
    out, ids, w, _ = dev.forward_batch(x, 9)
    o_out, o_ids, o_w, _, _ = orc.forward(x)
    assert np.array_equal(ids, o_ids)
    assert_close(out, o_out)


def test_single_token_forward_api(oracle, ctx):
    g = syn.rng(78)
    dev, orc = build_layer(oracle, ctx, g, 256, 128, 16)
    x = syn.normal_bf16_as_f32(g, 256)
    out, routes = dev.forward(x)
    o_out, o_ids, o_w, o_s, _ = orc.forward(x)
    assert [r.expert for r in routes] == list(o_ids[0])
    assert [np.float32(r.selection_score) for r in routes] == list(o_s[0])
    assert_close(out, o_out[0])


def test_moe_rejects_nonfinite_input(oracle, ctx):
    g = syn.rng(79)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 16)
    x = syn.normal_bf16_as_f32(g, (2, 256))
    x[1, 3] = np.inf
    with pytest.raises(urb.UrbError) as e:
        dev.forward_batch(x, 2)
    assert e.value.kind == "NonFinite"


@pytest.mark.parametrize("fmt", ["mxfp4", "bf16"])
@pytest.mark.parametrize("path", ["tc", "mma"])
def test_both_grouped_paths_many_tokens(oracle, ctx, path, fmt, monkeypatch):
    # 160 tokens of f32 (not bf16-exact) activations: hi/lo columns, two shared-expert chunks,
    # experts with >64 routed tokens on the tcgen05 path (BF16: three BF16 terms per value).
    monkeypatch.setenv("URB_MOE_PATH", path)
    g = syn.rng(500)
    dev, orc = build_layer(oracle, ctx, g, 256, 256, 8, fmt, top_k=4, scale=1.0)
    x = syn.normal_f32(g, (160, 256))
    out, ids, w, _ = dev.forward_batch(x, 160)
    o_out, o_ids, o_w, _, _ = orc.forward(x)
    assert np.array_equal(ids, o_ids)
    assert_close(out, o_out)


def test_bf16_layer_runs_the_tensor_core_passes(oracle, ctx):
    # BF16 experts take the tcgen05 kind::f16 passes (tiles through the TMA tensor map): the
    # layer runs the activation-term prep and no mma.sync row shift.
    g = syn.rng(510)
    dev, orc = build_layer(oracle, ctx, g, 256, 128, 16, "bf16", top_k=4, scale=1.0)
    x = syn.normal_f32(g, (12, 256))
    res = {}
    kinds = profiled_kinds(ctx, lambda: res.update(r=dev.forward_batch(x, 12)))
    assert "prep" in kinds and "row_shift" not in kinds, kinds
    out, ids, w, _ = res["r"]
    o_out, o_ids, _, _, _ = orc.forward(x)
    assert np.array_equal(ids, o_ids)
    assert_close(out, o_out)


@pytest.mark.parametrize("experts,tokens", [(64, 32), (768, 32)])
def test_decode_grouping_kernel_and_its_fallback(oracle, ctx, experts, tokens):
    # Up to 32 tokens route, group and build the pass tables in one CTA (k_decode_group);
    # with 768 experts its per-token routing scratch no longer fits one CTA's shared memory
    # and the separate routing / grouping / table kernels run instead.  Routes, counts and
    # the permutation bit-exact, outputs within the bar, either way.
    g = syn.rng(7000 + experts)
    dev, orc = build_layer(oracle, ctx, g, 256, 128, experts, "mxfp4", top_k=8, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (tokens, 256))
    out, ids, w, extra = dev.forward_batch(x, tokens, details=True)
    o_out, o_ids, o_w, _, _ = orc.forward(x)
    assert np.array_equal(ids, o_ids)
    assert np.array_equal(w.view(np.uint32), o_w.view(np.uint32))
    counts, offsets, pt, ps = oracle.group_routes(o_ids, experts)
    assert np.array_equal(extra["counts"], counts)
    assert np.array_equal(extra["perm_token"], pt) and np.array_equal(extra["perm_slot"], ps)
    assert_close(out, o_out)


@pytest.mark.parametrize("fmt", ["mxfp4", "mxfp8", "bf16"])
def test_one_token_decode_matches_caller_routes_and_replays_from_a_graph(oracle, fmt):
    # One token: every gate/up group reads one activation-stage set, whose prep runs on the
    # context's side stream while the router runs.  The same token with its routes given by the
    # caller (per-group stages, no side stream) gives the same bits; the device forward records
    # into a CUDA graph (the fork and join included) whose replay gives them again.
    import torch
    c = urb.Context(0)
    stream = torch.cuda.Stream()
    c.set_stream(stream.cuda_stream)
    g = syn.rng(7100 + len(fmt))
    dev, orc = build_layer(oracle, c, g, 256, 128, 32, fmt, top_k=8, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (1, 256))
    out, ids, w, _ = dev.forward_batch(x, 1)
    o_out, o_ids, _, _, _ = orc.forward(x)
    assert np.array_equal(ids, o_ids)
    assert_close(out, o_out)
    routed = dev.forward_routed(x, 1, ids, w)
    assert np.array_equal(out.view(np.uint32), routed.view(np.uint32))
    d_x = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    d_out = torch.zeros_like(d_x)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        dev.forward_device(d_x.data_ptr(), 1, d_out.data_ptr(), 0, 0, st.data_ptr())
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        dev.forward_device(d_x.data_ptr(), 1, d_out.data_ptr(), 0, 0, st.data_ptr())
    d_out.zero_()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert np.array_equal(d_out.cpu().numpy().view(np.uint32), out.view(np.uint32))
    del graph
    dev.free()
    c.close()  # objects still holding this context drop their handles (Matrix.free)


def test_one_token_nonfinite_input_is_rejected_and_the_context_recovers(oracle, ctx):
    # One token takes the side-stream prep; a non-finite input is still rejected (by the prep
    # and by the router's gates), and the next call on the same context gives the oracle's
    # answer.
    g = syn.rng(80)
    dev, orc = build_layer(oracle, ctx, g, 256, 128, 16)
    x = syn.normal_bf16_as_f32(g, (1, 256))
    bad = x.copy()
    bad[0, 5] = np.nan
    with pytest.raises(urb.UrbError) as e:
        dev.forward_batch(bad, 1)
    assert e.value.kind == "NonFinite"
    out, ids, _, _ = dev.forward_batch(x, 1)
    o_out, o_ids, _, _, _ = orc.forward(x)
    assert np.array_equal(ids, o_ids)
    assert_close(out, o_out)
