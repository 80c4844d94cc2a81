"""urb_gated_mlp_forward_device_noalloc: the gated MLP on device pointers with every temporary
in the library's static per-device scratch, for callers that cannot allocate device memory
while they run (a serving loop that reserved all free HBM up front, a decode loop where a
cudaMalloc would synchronise the device).

Called through the C ABI twice in a row on a fresh context, it must equal
urb_gated_mlp_forward_device bit for bit (and the oracle within the parity bar) while the
device's stream-ordered pool and free memory stay unchanged; calls whose temporaries exceed
the scratch, and formats without a shared tiled layout, are rejected.  The file is collected
last; `test_noalloc_in_fresh_process` also runs the comparison alone in a new process, where
the first call resolves the scratch's address."""
import os
import subprocess
import sys

import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import native
from urbilateria_b200 import synthetic as syn

from helpers import assert_close, bf16_pair, memory_state, mxfp4_pair, mxfp8_pair, rel_err

pytestmark = pytest.mark.gpu

CHILD_ENV = "URB_NOALLOC_CHILD"


def run(ctx, fn, mats, d_x, tokens, d_out, d_status):
    import torch
    torch.cuda.synchronize()
    rc = fn(ctx.h, mats[0].h, mats[1].h, mats[2].h, d_x.data_ptr(), tokens, d_out.data_ptr(),
            d_status.data_ptr())
    ctx.check(rc)
    ctx.synchronize()
    return d_out.cpu().numpy().copy()


def wide_bf16_pair(oracle, ctx, g, rows, cols):
    """BF16 weights whose rows span 2^-20 .. 2^20 (a wide exponent range per matrix)."""
    w = g.standard_normal((rows, cols)) * 0.02 * np.exp2(g.integers(-20, 21, size=(rows, 1)))
    bits = syn.f32_to_bf16_bits(w.astype(np.float32))
    dev = urb.Bf16Matrix.from_bits(rows, cols, bits, ctx=ctx)
    return dev, oracle.Matrix(oracle.BF16, rows, cols, bits)


CASES = [("bf16", 2048, 768, 1), ("bf16", 2048, 768, 32), ("bf16wide", 1024, 384, 3),
         ("mxfp4", 1024, 512, 7), ("mxfp8", 1024, 512, 5)]


@pytest.mark.parametrize("fmt,hidden,inter,tokens", CASES)
def test_noalloc_matches_gated_mlp_device(oracle, fmt, hidden, inter, tokens):
    import torch
    # A fresh context: its workspace is empty, so any allocation inside the no-alloc call would
    # show in the pool's figures below.
    ctx = urb.Context(0)
    g = syn.rng(7000 + tokens)
    pair = {"bf16": bf16_pair, "bf16wide": wide_bf16_pair, "mxfp4": mxfp4_pair,
            "mxfp8": mxfp8_pair}[fmt]
    gd, go = pair(oracle, ctx, g, inter, hidden)
    ud, uo = pair(oracle, ctx, g, inter, hidden)
    dd, do = pair(oracle, ctx, g, hidden, inter)
    x = syn.normal_bf16_as_f32(g, (tokens, hidden))
    dev = torch.device("cuda", ctx.device)
    d_x = torch.from_numpy(x).to(dev)
    d_out = torch.full((tokens, hidden), float("nan"), device=dev)
    d_status = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = ctx.lib
    torch.cuda.synchronize()
    before = memory_state(ctx.device)
    outs = []
    for i in range(2):
        d_out.fill_(float("nan"))
        outs.append(run(ctx, lib.urb_gated_mlp_forward_device_noalloc, (gd, ud, dd), d_x, tokens,
                        d_out, d_status))
        if i == 0:
            steady = memory_state(ctx.device)
    after = memory_state(ctx.device)
    # No stream-ordered allocation at all (the context's workspace never grew), and no device
    # allocation of any kind between the first and the second call.
    assert after[:2] == before[:2], (before, after)
    assert after[2] == steady[2], (steady, after)
    assert int(d_status.item()) == 0
    want = run(ctx, lib.urb_gated_mlp_forward_device, (gd, ud, dd), d_x, tokens, d_out, d_status)
    for got in outs:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    ref = np.stack([oracle.gated_mlp_forward(go, uo, do, x[t]) for t in range(tokens)])
    rel, mx = rel_err(outs[1], ref)
    print("%s T=%d relL2=%.3e max_abs=%.3e max_abs/rms=%.3e" % (
        fmt, tokens, rel, np.abs(outs[1].astype(np.float64) - ref).max(), mx))
    assert_close(outs[1], ref)
    for m in (gd, ud, dd):
        m.free()
    ctx.close()


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


def test_noalloc_rejects_formats_without_tiles(ctx):
    import torch
    g = syn.rng(7200)
    mats = [urb.DenseMatrix.new(r, c, g.standard_normal((r, c)).astype(np.float32), ctx=ctx)
            for r, c in ((64, 128), (64, 128), (128, 64))]
    dev = torch.device("cuda", ctx.device)
    d_x = torch.zeros((2, 128), device=dev)
    d_out = torch.zeros((2, 128), device=dev)
    rc = ctx.lib.urb_gated_mlp_forward_device_noalloc(ctx.h, mats[0].h, mats[1].h, mats[2].h,
                                                      d_x.data_ptr(), 2, d_out.data_ptr(), None)
    assert rc == native.ERR_UNSUPPORTED
    with pytest.raises(urb.UrbError) as e:
        ctx.check(rc)
    assert "tiled format" in str(e.value)


@pytest.mark.skipif(os.environ.get(CHILD_ENV) == "1", reason="already the fresh process")
def test_noalloc_in_fresh_process():
    """The comparison above, alone in a new interpreter (no earlier call on the device)."""
    env = dict(os.environ, **{CHILD_ENV: "1"})
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        "-m", "gpu", os.path.abspath(__file__) + "::test_noalloc_matches_gated_mlp_device"],
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))), env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
