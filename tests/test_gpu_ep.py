"""Expert-parallel layer (urb_ep_*) on the GPU.  One GPU: a one-rank group runs the whole
exchange path (publish, barriers, route gather, peer-window gate/up sources, owner-window
down outputs, owner combine) and must equal the single-GPU layer bit for bit; a group whose
ranks share a GPU is refused before anything waits.  Two GPUs (skipped with fewer): one process
per GPU against the single-GPU layer, error propagation and barrier timeouts
(tests/ep_worker.py, mode "gpu")."""
import ctypes
import os

import numpy as np
import pytest

import urbilateria_b200 as urb
from urbilateria_b200 import native
from urbilateria_b200 import synthetic as syn
from urbilateria_b200.expert_parallel import ExpertParallelMoeLayer, shard_range
from test_gpu_moe import build_layer
from test_ep_host import run_ranks

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("fmt,hidden,inter,experts,top_k,tokens,tmax", [
    ("mxfp4", 512, 256, 32, 8, 24, 24),
    ("mxfp4", 320, 192, 8, 2, 37, 64),   # partial tiles, fewer tokens than the window holds
    ("mxfp8", 384, 160, 8, 2, 33, 40),
    ("bf16", 320, 192, 8, 2, 37, 64),    # BF16 experts (kind::f16 through the tensor maps)
])
def test_ep_one_rank_matches_layer(oracle, ctx, fmt, hidden, inter, experts, top_k, tokens, tmax):
    g = syn.rng(5100 + tokens)
    dev, _ = build_layer(oracle, ctx, g, hidden, inter, experts, fmt, top_k=top_k, scale=1.0)
    x = syn.normal_f32(g, (tokens, hidden))
    ref, ref_ids, ref_w, _ = dev.forward_batch(x, tokens)
    ep = ExpertParallelMoeLayer(dev, 1, 0, tmax)
    for _ in range(3):
        out, ids, w = ep.forward_batch(x, tokens)
        assert np.array_equal(ids, ref_ids)
        assert np.array_equal(bits(w), bits(ref_w))
        assert np.array_equal(bits(out), bits(ref))
    out, _, _ = ep.forward_batch(x[:5], 5)
    assert np.array_equal(bits(out), bits(ref[:5]))
    ep.forward_batch(x[:0], 0)
    with pytest.raises(urb.UrbError) as e:
        ep.forward_batch(np.zeros((tmax + 1, hidden), np.float32), tmax + 1)
    assert e.value.kind == "Shape"
    ep.free()


def test_ep_one_rank_rejects_nonfinite(oracle, ctx):
    g = syn.rng(5200)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 16, "mxfp4", top_k=4, scale=1.0)
    ep = ExpertParallelMoeLayer(dev, 1, 0, 8)
    x = syn.normal_bf16_as_f32(g, (6, 256))
    ref, _, _, _ = dev.forward_batch(x, 6)
    bad = x.copy()
    bad[4, 100] = np.inf
    with pytest.raises(urb.UrbError) as e:
        ep.forward_batch(bad, 6)
    assert e.value.kind == "NonFinite"
    out, _, _ = ep.forward_batch(x, 6)
    assert np.array_equal(bits(out), bits(ref))
    ep.free()


def test_sharded_layer_runs_only_through_the_group(oracle, ctx):
    g = syn.rng(5300)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 16, "mxfp4", top_k=4, scale=1.0)
    half = urb.RuntimeMoeLayer(dev.router, dev.bias, dev.experts[:8], dev.shared, dev.geometry,
                               expert_range=(0, 8))
    with pytest.raises(urb.UrbError) as e:
        half.forward_batch(np.zeros((2, 256), np.float32), 2)
    assert e.value.kind == "Unsupported"


def test_group_on_one_gpu_is_refused(oracle, ctx):
    # Two ranks on one device would wait on one another from separate launches on one GPU; the
    # group is refused at connect time, before any kernel of the group runs.
    g = syn.rng(5400)
    dev, _ = build_layer(oracle, ctx, g, 256, 128, 16, "mxfp4", top_k=4, scale=1.0)
    shards = [urb.RuntimeMoeLayer(dev.router, dev.bias, dev.experts[b:b + c], dev.shared,
                                  dev.geometry, expert_range=(b, c))
              for b, c in (shard_range(16, 2, r) for r in range(2))]
    lib = ctx.lib
    hs, blobs = [], []
    for r in range(2):
        h = ctypes.c_void_p()
        ctx.check(lib.urb_ep_create(ctx.h, shards[r].h, 2, r, 8, 0, ctypes.byref(h)))
        b = (ctypes.c_uint8 * native.EP_HANDLE_BYTES)()
        ctx.check(lib.urb_ep_export(h, ctypes.cast(b, ctypes.c_void_p)))
        hs.append(h)
        blobs.append(bytes(b))
    joined = (ctypes.c_uint8 * (2 * native.EP_HANDLE_BYTES)).from_buffer_copy(b"".join(blobs))
    rc = lib.urb_ep_connect(hs[0], ctypes.cast(joined, ctypes.c_void_p))
    assert rc == native.ERR_UNSUPPORTED
    for h in hs:
        lib.urb_ep_free(h)


def test_ep_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    run_ranks("gpu", 2, 23, timeout=600, env=env)
