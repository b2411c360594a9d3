"""Host-side logic of the multi-GPU layout, on CPU with gloo ranks.

Each rank owns an independent env slice seeded ``rank_seed(seed, rank)``
and steps it alone (here on the CPU oracle); the only collective is the
per-rollout all-reduce of the episode statistics, plus max/sum reductions of
the bench's timing and ply counts.  A world of 2 ranks must produce exactly
the statistics of the two slices run one after the other in one process.
"""
from __future__ import annotations

import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

from junqi_b200 import sharding
from junqi_b200 import tables

ENVS, PLIES, SEED = 12, 700, 77


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def shard_rollout(rank: int) -> tuple[np.ndarray, int]:
    """Statistics vector (wins0, wins1, draws, episodes, sum_len, plies
    applied) and applied plies of rank's slice: GameState rules, uniform
    policy, auto-reset."""
    from oracle import oracle as O
    seed = sharding.rank_seed(SEED, rank)
    pool = tables.build_setup_pool(32, seed=seed)
    b = O.OracleBatch(ENVS, 2, rules=1)
    rng = np.random.default_rng(seed)
    for e in range(ENVS):
        b.reset_env(e, pool[e % len(pool)])
    stats = np.zeros(6, np.int64)
    applied = 0
    for _ in range(PLIES):
        off, val = b.legal()
        cnt = np.diff(off)
        acts = np.full(ENVS, -1, np.int32)
        for e in np.nonzero(cnt)[0]:
            acts[e] = val[off[e] + rng.integers(cnt[e])]
        r = b.step(acts)
        applied += int(r["valid"].sum())
        for e in np.nonzero(r["terminated"] & (r["valid"] == 1))[0]:
            if r["draw"][e]:
                stats[2] += 1
            elif r["winner"][e] >= 0:
                stats[int(r["winner"][e])] += 1
            stats[3] += 1
            stats[4] += int(b["move_counter"][e])
            b.reset_env(int(e), pool[int(rng.integers(len(pool)))])
    stats[5] = applied
    return stats, applied


def _rank_main(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        stats, applied = shard_rollout(rank)
        t = torch.from_numpy(stats.copy())
        sharding.reduce_episode_stats(t)
        ms = sharding.max_over_ranks(10.0 + rank)
        tot = sharding.sum_over_ranks(applied)
        recs = sharding.gather_over_ranks({"rank": rank, "applied": applied})
        q.put((rank, t.numpy().tolist(), ms, tot, applied, recs))
    finally:
        dist.destroy_process_group()


def test_rank_seed_and_env_slice():
    assert sharding.rank_seed(5, 0) == 5 and sharding.rank_seed(5, 3) == 30_005
    parts = [sharding.env_slice(1003, r, 4) for r in range(4)]
    assert parts[0][0] == 0 and sum(c for _, c in parts) == 1003
    assert all(parts[i][0] + parts[i][1] == parts[i + 1][0] for i in range(3))
    with pytest.raises(ValueError):
        sharding.env_slice(10, 4, 4)
    with pytest.raises(ValueError):
        sharding.reduce_episode_stats(torch.zeros(6, dtype=torch.int32))


def test_single_process_reductions_are_identity():
    t = torch.tensor([1, 2, 3, 4, 5, 6], dtype=torch.int64)
    assert sharding.reduce_episode_stats(t) is t and t.tolist() == [1, 2, 3, 4, 5, 6]
    assert sharding.max_over_ranks(2.5) == 2.5 and sharding.sum_over_ranks(7) == 7
    assert sharding.stats_dict(t)["episodes"] == 4


def test_two_gloo_ranks_reduce_episode_stats_of_independent_slices():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect_stats = np.zeros(6, np.int64)
    expect_tot = 0
    for r in range(2):
        s, a = shard_rollout(r)
        expect_stats += s
        expect_tot += a
    assert expect_stats[3] > 0, "the rollout must finish some episodes"
    for rank, stats, ms, tot, applied, recs in got:
        assert stats == expect_stats.tolist(), f"rank {rank}"
        assert ms == 11.0
        assert tot == expect_tot
        assert [r["rank"] for r in recs] == [0, 1] and sum(r["applied"] for r in recs) == expect_tot


def test_core_slices_are_disjoint_and_cover_the_node():
    cores = [0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16]
    for world in (1, 2, 4, 8):
        parts = [sharding.core_slice(cores, r, world) for r in range(world)]
        assert sorted(c for p in parts for c in p) == cores
        assert max(map(len, parts)) - min(map(len, parts)) <= 1
    assert sharding.core_slice([3, 1], 2, 4) == [1]  # fewer cores than ranks: shared round-robin
    assert sharding.gather_over_ranks({"a": 1}) == [{"a": 1}]
    with pytest.raises(ValueError):
        sharding.core_slice(cores, 2, 2)
