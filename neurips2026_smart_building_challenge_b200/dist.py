"""Multi-GPU plumbing: one process per GPU, each owning a disjoint slice of envs.

The env step has no cross-env term, so ranks never exchange data while stepping.
The only collective is the reduction of episode statistics at log time (the
reference reads them per device with no collective at all,
complete_port/gpu/smart_buildings.cu:3069-3229): per-scenario sums of reward,
comfort deviation and step counts are summed over ranks with one all-reduce
(NCCL over NVLink on B200, gloo in CPU tests).
"""
from __future__ import annotations

import numpy as np

STAT_KEYS = ("reward", "comfort_dev_K", "steps", "reward_sq", "episode_mean_sum", "episodes")


def shard(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, count) of the envs rank owns: contiguous, sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world or n_total < world:
        raise ValueError("need 0 <= rank < world <= n_total")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def scenario_stats(live_scn: np.ndarray, ep_scn: np.ndarray) -> np.ndarray:
    """Per-scenario statistics matrix [n_scn][6] from the device sums (live_scn [n][4], ep_scn [n][2])."""
    live_scn = np.asarray(live_scn, dtype=np.float64).reshape(-1, 4)
    ep_scn = np.asarray(ep_scn, dtype=np.float64).reshape(-1, 2)
    return np.concatenate([live_scn, ep_scn], axis=1)


def allreduce_stats(stats: np.ndarray, device=None) -> np.ndarray:
    """Sums a per-scenario statistics matrix over all ranks of the default process group."""
    import torch
    import torch.distributed as dist

    t = torch.as_tensor(np.ascontiguousarray(stats, dtype=np.float64), device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.cpu().numpy()


def summarize(stats: np.ndarray) -> dict:
    """Means from summed statistics: per-step reward / deviation and the episode score."""
    s = np.asarray(stats, dtype=np.float64).reshape(-1, len(STAT_KEYS))
    steps = s[:, 2].sum()
    eps = s[:, 5].sum()
    return {"steps": steps, "mean_reward": s[:, 0].sum() / steps if steps else 0.0,
            "mean_comfort_dev_K": s[:, 1].sum() / steps if steps else 0.0,
            "episodes": eps, "episode_score": -s[:, 4].sum() / eps if eps else 0.0}
