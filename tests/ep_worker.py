"""One rank of the expert-parallel tests, run as a child process by test_ep_host.py (CPU, gloo)
and test_gpu_ep.py (one GPU per rank).

    python tests/ep_worker.py MODE RANK WORLD PORT TOKENS

MODE "model": the expert-parallel decomposition restated on the CPU with the oracle and gloo
collectives: each rank routes its own tokens, the ranks exchange (routes, token rows), each rank
runs the experts it holds for every rank's routes, the outputs travel back to the token owners
by route index (q * tmax + t) * top_k + k, and each owner combines in selection order in f64.
The result must equal the oracle's single-process layer bit for bit.

MODE "gpu": the library's expert-parallel layer (urb_ep_*), rank r on cuda:r, against the
single-GPU layer on the same device: outputs, routes and weights bit-identical; then a forward
in which one rank's input is not finite (every rank fails it: NonFinite there, Peer elsewhere,
and the group stays usable), and a forward that one rank skips (the others' barriers time out).

Exits 0 on success; any failed check raises.
"""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

HIDDEN, INTER, EXPERTS, TOP_K, SEED = 256, 128, 16, 4, 4711


def oracle_layer(oracle, g, fmt="mxfp4"):
    """Oracle matrices drawn in the same order as test_gpu_moe.build_layer."""
    from urbilateria_b200 import synthetic as syn

    def mx(rows, cols):
        packed, scales = syn.mxfp4_matrix(g, rows, cols, 119, 127, 32)
        return oracle.Matrix(oracle.MXFP4, rows, cols, packed, scales, group_size=32)

    gates, ups, downs = [], [], []
    for _ in range(EXPERTS):
        gates.append(mx(INTER, HIDDEN))
        ups.append(mx(INTER, HIDDEN))
        downs.append(mx(HIDDEN, INTER))
    shared = (mx(INTER, HIDDEN), mx(INTER, HIDDEN), mx(HIDDEN, INTER))
    bits = syn.bf16_normal(g, (EXPERTS, HIDDEN), 0.02)
    router = oracle.Matrix(oracle.BF16, EXPERTS, HIDDEN, bits)
    bias = syn.normal_f32(g, EXPERTS, 0.01)
    layer = oracle.MoeLayer(router, bias, gates, ups, downs, shared, TOP_K, 1, 1, True, 1.0)
    return layer, gates, ups, downs, shared


def run_model(rank, world, tokens):
    import torch.distributed as dist
    import urb_oracle as oracle
    from urbilateria_b200 import synthetic as syn
    from urbilateria_b200.expert_parallel import shard_range, token_range

    oracle.build()
    g = syn.rng(SEED)
    layer, gates, ups, downs, shared = oracle_layer(oracle, g)
    x_all = syn.normal_bf16_as_f32(g, (tokens, HIDDEN))
    tb, tc = token_range(tokens, world, rank)
    eb, ec = shard_range(EXPERTS, world, rank)
    tmax = -(-tokens // world)
    x = x_all[tb:tb + tc]
    if tc:
        _, ids, w, _, _ = layer.forward(x)
    else:
        ids = np.zeros((0, TOP_K), np.int32)
        w = np.zeros((0, TOP_K), np.float32)
    # Publish (routes, rows) of the own tokens; every rank sees every rank's.
    pub = [None] * world
    dist.all_gather_object(pub, (ids, x))
    # Held experts over every rank's routes, keyed by route index.
    produced = {}
    for q, (q_ids, q_x) in enumerate(pub):
        for t in range(q_ids.shape[0]):
            for k in range(TOP_K):
                e = int(q_ids[t, k])
                if eb <= e < eb + ec:
                    i = (q * tmax + t) * TOP_K + k
                    produced[i] = oracle.gated_mlp_forward(gates[e], ups[e], downs[e], q_x[t])
    back = [None] * world
    dist.all_gather_object(back, produced)
    # Owner combine: route i lands in rank i // (tmax * top_k), row i % (tmax * top_k).
    y = np.full((tmax * TOP_K, HIDDEN), np.nan, np.float32)
    for part in back:
        for i, row in part.items():
            if i // (tmax * TOP_K) == rank:
                y[i % (tmax * TOP_K)] = row
    out = np.empty((tc, HIDDEN), np.float32)
    for t in range(tc):
        acc = oracle.gated_mlp_forward(shared[0], shared[1], shared[2], x[t]).astype(np.float64)
        for k in range(TOP_K):
            acc = acc + np.float64(w[t, k]) * y[t * TOP_K + k].astype(np.float64)
        out[t] = acc.astype(np.float32)
    if tc:
        ref = layer.forward(x_all)[0][tb:tb + tc]
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), "EP model != layer"


def run_gpu(rank, world, tokens):
    import urb_oracle as oracle
    import urbilateria_b200 as urb
    from urbilateria_b200 import synthetic as syn
    from urbilateria_b200.expert_parallel import (ExpertParallelMoeLayer, all_gather_bytes,
                                                  shard_range, token_range)
    from test_gpu_moe import build_layer

    oracle.build()
    ctx = urb.Context(rank)
    g = syn.rng(SEED)
    dev, _ = build_layer(oracle, ctx, g, HIDDEN, INTER, EXPERTS, "mxfp4", top_k=TOP_K, scale=1.0)
    x_all = syn.normal_bf16_as_f32(g, (tokens, HIDDEN))
    tb, tc = token_range(tokens, world, rank)
    eb, ec = shard_range(EXPERTS, world, rank)
    tmax = -(-tokens // world)
    shard = urb.RuntimeMoeLayer(dev.router, dev.bias, dev.experts[eb:eb + ec], dev.shared,
                                dev.geometry, expert_range=(eb, ec))
    ep = ExpertParallelMoeLayer(shard, world, rank, tmax, exchange=all_gather_bytes,
                                timeout_ms=2000)
    ref_out, ref_ids, ref_w, _ = dev.forward_batch(x_all, tokens)
    x = np.ascontiguousarray(x_all[tb:tb + tc])
    for _ in range(2):  # twice: the barrier words alternate by epoch parity
        out, ids, w = ep.forward_batch(x, tc)
        assert np.array_equal(ids, ref_ids[tb:tb + tc])
        assert np.array_equal(w.view(np.uint32), ref_w[tb:tb + tc].view(np.uint32))
        assert np.array_equal(out.view(np.uint32), ref_out[tb:tb + tc].view(np.uint32)), \
            "rank %d: EP output differs from the single-GPU layer" % rank
    # A forward in which the last rank's input is not finite fails on every rank.
    bad = x.copy()
    if rank == world - 1 and tc:
        bad[0, 3] = np.nan
    try:
        ep.forward_batch(bad, tc)
        raise AssertionError("forward with a non-finite input on a peer succeeded")
    except urb.UrbError as e:
        want = "NonFinite" if rank == world - 1 else "Peer"
        assert e.kind == want, (rank, e.kind)
    # The group is still usable.
    out, _, _ = ep.forward_batch(x, tc)
    assert np.array_equal(out.view(np.uint32), ref_out[tb:tb + tc].view(np.uint32))
    # Zero tokens on one rank.
    if rank == 0:
        ep.forward_batch(x[:0], 0)
    else:
        out, _, _ = ep.forward_batch(x, tc)
        assert np.array_equal(out.view(np.uint32), ref_out[tb:tb + tc].view(np.uint32))
    import torch.distributed as dist
    dist.barrier()
    # Rank 0 runs a forward the others skip: its barriers run out and report Timeout, and its
    # context stays usable.  The group is not used again after this.
    if rank == 0:
        try:
            ep.forward_batch(x, tc)
            raise AssertionError("forward without peers succeeded")
        except urb.UrbError as e:
            assert e.kind == "Timeout", e.kind
        again, _, _, _ = dev.forward_batch(x_all, tokens)
        assert np.array_equal(again.view(np.uint32), ref_out.view(np.uint32))
    dist.barrier()
    ep.free()


def main():
    mode, rank, world, port, tokens = sys.argv[1], *map(int, sys.argv[2:6])
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        (run_model if mode == "model" else run_gpu)(rank, world, tokens)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
