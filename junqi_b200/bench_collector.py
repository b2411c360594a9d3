"""Throughput of RolloutCollector, eager against one CUDA graph per rollout.

    python -m junqi_b200.bench_collector [--envs 256 4096] [--plies 64] [--rollouts 3]

The policy is a stand-in for a network: a masked argmax over fixed random
per-action scores (one pass over the canonical mask), so the numbers show
the collector's own cost.  GameState rules, HALF_DARK, compact history on.
Prints one JSON line per (envs, mode).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _native as N
from . import tables
from .collector import RolloutCollector
from .env import HALF_DARK, JunqiEnvB200


class ArgmaxPolicy:
    def __init__(self, device):
        g = torch.Generator(device="cpu").manual_seed(0)
        self.score = torch.rand(16641, generator=g).to(device)

    def __call__(self, sp, gl, mask):
        v, a = torch.where(mask, self.score, -1.0).max(1)
        return a, v, gl[:, 0]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--envs", type=int, nargs="+", default=[256, 4096])
    ap.add_argument("--plies", type=int, default=64)
    ap.add_argument("--rollouts", type=int, default=3)
    args = ap.parse_args()
    pool = tables.build_setup_pool(1024, seed=2)
    for n in args.envs:
        for graph in (False, True):
            env = JunqiEnvB200(n, show_mode=HALF_DARK, pool=pool, rules=N.RULES_GAMESTATE)
            env.reset(seed=1)
            col = RolloutCollector(env, ArgmaxPolicy(env.device), args.plies, seed=3, graph=graph)
            col.collect()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(args.rollouts):
                col.collect()
            t1.record()
            torch.cuda.synchronize()
            ms = t0.elapsed_time(t1) / args.rollouts
            print(json.dumps({"envs": n, "plies": args.plies, "graph": graph, "ms_per_rollout": round(ms, 3),
                              "plies_per_s": round(args.plies * n / ms * 1e3)}), flush=True)


if __name__ == "__main__":
    main()
