"""urb_gated_mlp_forward_device_noalloc: the gated MLP on device pointers with every temporary
in the library's static per-device scratch.  Called through the C ABI twice in a row, it must
equal urb_gated_mlp_forward_device bit for bit (and the oracle within the parity bar); calls
whose temporaries exceed the scratch are rejected.  Collected last, and also run alone in a
fresh process (the first call on a device resolves the scratch)."""
import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import native
from urbilateria_b200 import synthetic as syn

from helpers import assert_close, bf16_pair, mxfp4_pair

pytestmark = pytest.mark.gpu


def run(ctx, fn, mats, d_x, tokens, d_out, d_status):
    import torch
    torch.cuda.synchronize()
    rc = fn(ctx.h, mats[0].h, mats[1].h, mats[2].h, d_x.data_ptr(), tokens, d_out.data_ptr(),
            d_status.data_ptr())
    ctx.check(rc)
    ctx.synchronize()
    return d_out.cpu().numpy().copy()


@pytest.mark.parametrize("fmt,hidden,inter,tokens", [("bf16", 2048, 768, 1), ("bf16", 2048, 768, 32),
                                                     ("mxfp4", 1024, 512, 7)])
def test_noalloc_matches_gated_mlp_device(oracle, ctx, fmt, hidden, inter, tokens):
    import torch
    g = syn.rng(7000 + tokens)
    pair = bf16_pair if fmt == "bf16" else mxfp4_pair
    gd, go = pair(oracle, ctx, g, inter, hidden)
    ud, uo = pair(oracle, ctx, g, inter, hidden)
    dd, do = pair(oracle, ctx, g, hidden, inter)
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    dev = torch.device("cuda", ctx.device)
    d_x = torch.from_numpy(x).to(dev)
    d_out = torch.full((tokens, hidden), float("nan"), device=dev)
    d_status = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = ctx.lib
    want = run(ctx, lib.urb_gated_mlp_forward_device, (gd, ud, dd), d_x, tokens, d_out, d_status)
    for _ in range(2):
        d_out.fill_(float("nan"))
        got = run(ctx, lib.urb_gated_mlp_forward_device_noalloc, (gd, ud, dd), d_x, tokens,
                  d_out, d_status)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert int(d_status.item()) == 0
    ref = np.stack([oracle.gated_mlp_forward(go, uo, do, x[t]) for t in range(tokens)])
    assert_close(got, ref)


def test_noalloc_rejects_oversized_calls(oracle, ctx):
    import torch
    g = syn.rng(7100)
    gd, _ = bf16_pair(oracle, ctx, g, 2048, 256)
    ud, _ = bf16_pair(oracle, ctx, g, 2048, 256)
    dd, _ = bf16_pair(oracle, ctx, g, 256, 2048)
    tokens = 1100  # h alone is 1100 * 2048 * 4 bytes > 8 MiB
    dev = torch.device("cuda", ctx.device)
    d_x = torch.zeros((tokens, 256), device=dev)
    d_out = torch.zeros((tokens, 256), device=dev)
    d_status = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = ctx.lib.urb_gated_mlp_forward_device_noalloc(ctx.h, gd.h, ud.h, dd.h, d_x.data_ptr(),
                                                      tokens, d_out.data_ptr(),
                                                      d_status.data_ptr())
    assert rc == native.ERR_UNSUPPORTED
    with pytest.raises(urb.UrbError) as e:
        ctx.check(rc)
    assert "scratch" in str(e.value)
