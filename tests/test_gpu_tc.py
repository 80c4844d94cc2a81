"""Parity of the block-scaled tensor-core MoE passes (tcgen05.mma kind::mxf4 / kind::mxf8f6f4
with residual-term activations) with the GLM composition oracle
(src/models/glm/runtime/moe.rs:138-176).  Routing stays bit-exact; outputs within the parity
bar.  Shapes cover experts cut into several 32-token sub-segments, partial 128-row tiles and
partial K stages."""
import numpy as np
import pytest

from helpers import assert_close, rel_err
from test_gpu_moe import build_layer
from urbilateria_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


@pytest.fixture
def tc_path(monkeypatch):
    monkeypatch.setenv("URB_MOE_PATH", "tc")


@pytest.mark.parametrize("fmt,hidden,inter,experts,top_k,tokens", [
    ("mxfp4", 512, 256, 32, 8, 24),     # few tokens per expert
    ("mxfp4", 256, 256, 8, 4, 160),     # ~80 tokens per expert: three sub-segments
    ("mxfp4", 320, 192, 8, 2, 37),      # partial row tiles and a partial K stage
    ("mxfp8", 512, 256, 16, 4, 70),
    ("mxfp8", 384, 160, 8, 2, 33),      # MXFP8: 128-column stages, partial tiles
])
def test_tc_layer_parity(oracle, ctx, tc_path, fmt, hidden, inter, experts, top_k, tokens):
    g = syn.rng(900 + tokens + hidden)
    dev, orc = build_layer(oracle, ctx, g, hidden, inter, experts, fmt, top_k=top_k, scale=1.0)
    x = syn.normal_f32(g, (tokens, hidden))
    out, ids, w, extra = dev.forward_batch(x, tokens, details=True)
    o_out, o_ids, o_w, _, _ = orc.forward(x)
    assert np.array_equal(ids, o_ids)
    assert np.array_equal(w.view(np.uint32), o_w.view(np.uint32))
    r, m = rel_err(out, o_out)
    print("%s relL2=%.3e maxabs=%.3e" % (fmt, r, m))
    assert_close(out, o_out)


def test_tc_layer_repeat_is_deterministic(oracle, ctx, tc_path):
    g = syn.rng(31)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 16, "mxfp4", top_k=4, scale=1.0)
    x = syn.normal_bf16_as_f32(g, (40, 256))
    a, _, _, _ = dev.forward_batch(x, 40)
    b, _, _, _ = dev.forward_batch(x, 40)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_tc_rejects_nonfinite_input(oracle, ctx, tc_path):
    import urbilateria_b200 as urb
    g = syn.rng(32)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 16, "mxfp4", top_k=4)
    x = syn.normal_bf16_as_f32(g, (3, 256))
    x[2, 7] = np.nan
    with pytest.raises(urb.UrbError) as e:
        dev.forward_batch(x, 3)
    assert e.value.kind == "NonFinite"
    # The context stays usable after the rejected call.
    x[2, 7] = 0.5
    dev.forward_batch(x, 3)


@pytest.mark.parametrize("hidden", [301, 4098, 4100, 7168])
def test_router_logits_bit_exact_adversarial(oracle, ctx, hidden):
    # The logits run as f64 tensor-core chains; they must equal the reference's sequential
    # F64 sum bit for bit even when the order of roundings matters: activations spread over
    # 2^-60 .. 2^30 with alternating signs (heavy cancellation), expert / token counts that are
    # not multiples of 8, and hidden sizes covering the staged kernel's full stages (7168),
    # its MMA remainder (4100) and scalar tail (4098), and the odd-width direct kernel (301).
    g = syn.rng(4242 + hidden)
    experts, tokens = 20, 13
    dev, orc = build_layer(oracle, ctx, g, hidden, 64, experts, "mxfp4", top_k=4, scale=1.0)
    mant = g.uniform(1.0, 2.0, size=(tokens, hidden))
    expo = g.integers(-60, 31, size=(tokens, hidden))  # experts' outputs stay finite
    sign = np.where(g.random((tokens, hidden)) < 0.5, -1.0, 1.0)
    x = (sign * mant * np.exp2(expo)).astype(np.float32)
    x[:, ::7] = 0.0
    out, ids, w, extra = dev.forward_batch(x, tokens, details=True)
    o_logits = orc.forward(x)[4]
    assert np.array_equal(extra["router_logits"].view(np.uint32), o_logits.view(np.uint32))
