"""The multi-GPU plumbing of bench.py on CPU: two ranks over gloo (the GPU
runs use NCCL for the same two calls only).  The path shards into
independent replicas, so the only collectives are the start/stop barrier and
the max over ranks of the device time; each rank decodes its own inputs."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import bench
from tir import synth


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    d = bench.Dist("gloo")
    d.barrier()
    ms = d.max(10.0 * rank + 3.0)  # each rank's own step time
    prompt = synth.prompt_ids(16, 32000, seed=bench.decode_seed(0, rank))
    d.barrier()
    d.close()
    out.put((rank, ms, prompt.tolist()))


@pytest.mark.timeout(120)
def test_two_ranks_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=100) for _ in ps)
    for p in ps:
        p.join(timeout=30)
        assert p.exitcode == 0
    # max over ranks, seen by every rank
    assert [r[1] for r in res] == [13.0, 13.0]
    # each rank decodes its own sequence (weak scaling, no shared inputs)
    assert res[0][2] != res[1][2]
    assert res[0][2] == synth.prompt_ids(16, 32000, seed=0).tolist()


def test_single_rank_needs_no_process_group():
    d = bench.Dist("gloo")
    assert d.world == 1 and d.pg is None
    assert d.max(7.5) == 7.5
    d.barrier()
    d.close()


def test_batched_shards_differ():
    a = np.random.default_rng(bench.batched_seed(0, 0)).integers(3, 32000, 64)
    b = np.random.default_rng(bench.batched_seed(0, 1)).integers(3, 32000, 64)
    assert not np.array_equal(a, b)
