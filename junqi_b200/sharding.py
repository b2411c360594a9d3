"""Env sharding over ranks (one process per GPU) and the per-rollout reduction.

Envs are independent games, so the data-parallel layout needs no exchange on
the data path: rank r owns its own slice of envs, seeded
``seed + 10_000 * r`` (the convention of ``scripts/train.py:69-95`` in the
reference, which offsets ``cfg.env.seed`` by ``global_rank * 10_000``), and
steps it on its own GPU.  The only collective is one all-reduce (sum) of the
int64 episode-statistics vector per rollout; timings are reduced with max.

Works with any initialised ``torch.distributed`` backend (NCCL on GPUs,
gloo on CPU for the host-side tests) and degrades to a no-op when no process
group is initialised or the world has one rank.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

RANK_SEED_STRIDE = 10_000
# jq_ply's statistics vector: the reference's per-rollout episode statistics
# (wins per team, draws, episodes, summed episode length) plus plies applied
STAT_NAMES = ("wins_team0", "wins_team1", "draws", "episodes", "sum_len", "plies_applied")


def _world() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def rank_seed(seed: int, rank: int) -> int:
    """Seed of rank ``rank``'s env slice."""
    if rank < 0:
        raise ValueError(f"rank must be non-negative, got {rank}")
    return int(seed) + RANK_SEED_STRIDE * int(rank)


def env_slice(total_envs: int, rank: int, world: int) -> tuple[int, int]:
    """(first env, count) of rank's share when a fixed total is split
    (strong scaling); shares differ by at most one env."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(int(total_envs), world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def reduce_episode_stats(stats: torch.Tensor) -> torch.Tensor:
    """Sum the per-rank episode-statistics vector over all ranks, in place."""
    if stats.dtype != torch.int64 or stats.numel() != len(STAT_NAMES):
        raise ValueError(f"episode stats must be int64 of length {len(STAT_NAMES)}")
    if _world() > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.SUM)
    return stats


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """Maximum of a per-rank scalar (e.g. the timed region's device ms)."""
    if _world() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: int, device: torch.device | str = "cpu") -> int:
    """Sum of a per-rank count (e.g. plies applied)."""
    if _world() == 1:
        return int(value)
    t = torch.tensor([int(value)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())


def core_slice(cores: list[int], local_rank: int, local_world: int) -> list[int]:
    """The host cores of ``local_rank`` when the node's ``cores`` are split
    into ``local_world`` disjoint, contiguous shares (differing by at most
    one core).  With fewer cores than ranks, ranks share cores round-robin."""
    if local_world <= 0 or not 0 <= local_rank < local_world:
        raise ValueError(f"bad local rank {local_rank} for {local_world} ranks per node")
    cores = sorted(int(c) for c in cores)
    if not cores:
        raise ValueError("no host cores given")
    if len(cores) < local_world:
        return [cores[local_rank % len(cores)]]
    base, extra = divmod(len(cores), local_world)
    start = local_rank * base + min(local_rank, extra)
    return cores[start:start + base + (1 if local_rank < extra else 0)]


def pin_rank_cores(local_rank: int, local_world: int) -> list[int]:
    """Restrict this process to its share of the cores it may run on, so
    ranks of one node do not contend for the host threads that feed their
    GPUs; returns the cores kept (all of them where affinity is not
    supported)."""
    import os
    if not hasattr(os, "sched_getaffinity"):
        return []
    mine = core_slice(sorted(os.sched_getaffinity(0)), local_rank, local_world)
    os.sched_setaffinity(0, mine)
    return mine


def gather_over_ranks(obj) -> list:
    """Every rank's ``obj`` (a small picklable record), in rank order, on
    every rank; ``[obj]`` without a process group."""
    if _world() == 1:
        return [obj]
    out = [None] * _world()
    dist.all_gather_object(out, obj)
    return out


def stats_dict(stats: torch.Tensor) -> dict[str, int]:
    vals = stats.detach().cpu().tolist()
    return dict(zip(STAT_NAMES, (int(v) for v in vals)))
