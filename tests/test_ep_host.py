"""Host side of the expert-parallel layer on the CPU: shard and token ranges, the handle
all-gather, and the expert-parallel decomposition itself restated with the oracle over a
world-size-2 gloo group (tests/ep_worker.py, mode "model"), which must reproduce the
single-process layer bit for bit."""
import os
import socket
import subprocess
import sys

import pytest

from urbilateria_b200.expert_parallel import shard_range, token_range

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(mode, world, tokens, timeout=300, env=None):
    port = free_port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ep_worker.py"), mode, str(r),
                               str(world), str(port), str(tokens)],
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                              env=env)
             for r in range(world)]
    outs = []
    try:
        for p in procs:
            outs.append(p.communicate(timeout=timeout)[0])
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, "rank %d failed:\n%s" % (r, o[-4000:])


@pytest.mark.parametrize("experts,world", [(256, 1), (256, 2), (256, 8), (16, 3), (384, 8),
                                           (10, 4), (7, 7)])
def test_shard_ranges_tile_the_experts(experts, world):
    seen = []
    for r in range(world):
        b, c = shard_range(experts, world, r)
        assert c >= 1
        seen.extend(range(b, b + c))
    assert seen == list(range(experts))
    sizes = [shard_range(experts, world, r)[1] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("tokens,world", [(128, 8), (9, 2), (1, 2), (0, 4), (5, 8)])
def test_token_ranges_partition_the_batch(tokens, world):
    seen = []
    for r in range(world):
        b, c = token_range(tokens, world, r)
        seen.extend(range(b, b + c))
    assert seen == list(range(tokens))


def test_shard_range_rejects_more_ranks_than_experts():
    with pytest.raises(ValueError):
        shard_range(4, 5, 0)


def test_all_gather_bytes_rank_order():
    # The handle exchange over a gloo group returns every rank's blob in rank order.
    code = r'''
import datetime, sys
import torch.distributed as dist
from urbilateria_b200.expert_parallel import all_gather_bytes
r, port = int(sys.argv[1]), int(sys.argv[2])
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=r, world_size=2,
                        timeout=datetime.timedelta(seconds=60))
got = all_gather_bytes(bytes([r]) * 256)
assert got == [bytes([0]) * 256, bytes([1]) * 256], got
dist.destroy_process_group()
'''
    port = free_port()
    env = dict(os.environ, PYTHONPATH=os.path.dirname(HERE))
    procs = [subprocess.Popen([sys.executable, "-c", code, str(r), str(port)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(2)]
    outs = [p.communicate(timeout=120)[0] for p in procs]
    assert all(p.returncode == 0 for p in procs), outs


@pytest.mark.parametrize("tokens", [9, 1])  # 1 token: rank 1 owns none
def test_expert_parallel_decomposition_matches_layer(tokens):
    run_ranks("model", 2, tokens)
