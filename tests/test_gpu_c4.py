"""Config 4 composition: stacked MoE layers applied as a decode step, h <- h + MoE_l(h), for a
few sequences of one token each (no attention, no norm).  Each layer is checked against the
oracle on the oracle's own input (routes bit-exact, outputs within the parity bar), and the
free-running stack end to end within the bar."""
import numpy as np
import pytest

from helpers import assert_close
from test_gpu_moe import build_layer
from urbilateria_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 8])
def test_stacked_decode_layers(oracle, ctx, batch):
    g = syn.rng(9400 + batch)
    layers = [build_layer(oracle, ctx, g, 512, 256, 48, "mxfp4", top_k=8, scale=2.5)
              for _ in range(3)]
    h0 = syn.normal_bf16_as_f32(g, (batch, 512))
    h_dev, h_orc = h0.copy(), h0.copy()
    for dev, orc in layers:
        o_out, o_ids, o_w, _, _ = orc.forward(h_orc)
        out, ids, w, _ = dev.forward_batch(h_orc, batch)  # same input as the oracle layer
        assert np.array_equal(ids, o_ids)
        assert np.array_equal(w.view(np.uint32), o_w.view(np.uint32))
        assert_close(out, o_out)
        free, _, _, _ = dev.forward_batch(h_dev, batch)
        h_dev = (h_dev + free).astype(np.float32)
        h_orc = (h_orc + o_out).astype(np.float32)
    assert_close(h_dev, h_orc)
