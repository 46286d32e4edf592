"""Multi-rank host logic on CPU: env sharding and the episode-statistics
all-reduce over a 2-rank gloo group (the NCCL path on B200 uses the same code)."""
import os
import socket

import numpy as np
import pytest

from neurips2026_smart_building_challenge_b200 import dist as sbdist


def test_shard_partitions_exactly():
    for n in (960, 7680, 15360, 61440, 1001):
        for world in (1, 2, 3, 4, 8):
            parts = [sbdist.shard(n, world, r) for r in range(world)]
            assert parts[0][0] == 0
            for (s0, c0), (s1, _) in zip(parts, parts[1:]):
                assert s0 + c0 == s1
            assert sum(c for _, c in parts) == n
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
    with pytest.raises(ValueError):
        sbdist.shard(4, 8, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        live = np.full((3, 4), rank + 1.0)
        ep = np.full((3, 2), 10.0 * (rank + 1))
        out = sbdist.allreduce_stats(sbdist.scenario_stats(live, ep))
        q.put((rank, out.tolist(), sbdist.summarize(out)))
    finally:
        dist.destroy_process_group()


def test_stats_allreduce_gloo_two_ranks():
    import torch.multiprocessing as tmp

    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out, summ in res:
        out = np.array(out)
        assert np.allclose(out[:, :4], 3.0) and np.allclose(out[:, 4:], 30.0)
        assert summ["steps"] == 9.0 and summ["episodes"] == 90.0
