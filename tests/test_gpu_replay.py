"""Replay records of device rollouts, and replay validation on the device.

* The games junqi_core recorded (tests/golden/replay) validate on the
  device; the same games with one planted fault each (swapped plies, a
  wrong seat column, a wrong final hash) do not.
* A device rollout recorded with ReplayRecorder cuts into per-game
  trajectories whose action logs replay on the CPU oracle to the hash the
  device recorded, and which also validate on the device, after a save /
  load round trip through the reference file format.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from junqi_b200 import _native as N
from junqi_b200 import tables
from junqi_b200.env import DARK, HALF_DARK, JunqiEnvB200
from junqi_b200.replay import ReplayRecorder, Trajectory, validate_on_device

pytestmark = pytest.mark.gpu

GOLD = sorted((Path(__file__).parent / "golden" / "replay").glob("ref_game_*.npz"))


def _faulty(tr: Trajectory, kind: str) -> Trajectory:
    a, h = tr.actions.copy(), tr.final_state_hash
    if kind == "swap":
        a[[10, 11]] = a[[11, 10]]
    elif kind == "seat":
        a[20, 0] = (a[20, 0] + 1) % 4
    else:
        h ^= 1
    return Trajectory(setups=tr.setups, actions=a, rng_seed=-1, final_state_hash=h, first_seat=tr.first_seat,
                      show_mode=tr.show_mode)


def test_reference_games_validate_on_the_device():
    games = [Trajectory.load(p) for p in GOLD]
    assert validate_on_device(games).all()
    bad = [_faulty(g, k) for g in games for k in ("swap", "seat", "hash")]
    assert not validate_on_device(bad).any()


@pytest.mark.parametrize("mode", [HALF_DARK, DARK])
def test_recorded_rollout_replays_to_the_device_hashes(mode, tmp_path):
    from tests.test_replay_cpu import oracle_replay
    n, plies = 96, 900
    env = JunqiEnvB200(n, show_mode=mode, pool=tables.build_setup_pool(40, seed=8), with_obs=False,
                       rules=N.RULES_GAMESTATE)
    rec = ReplayRecorder(env, plies)
    rec.reset(seed=21)
    for t in range(plies):
        rec.ply(env.sample_softmax(21, t + 1), seed=21, ply=t + 1)
    games = rec.trajectories(include_unfinished=True)
    finished = [g for g in games if g.meta["finished"]]
    assert len(finished) >= 20 and len(finished) < len(games) <= len(finished) + n
    assert sum(g.num_steps for g in games) == int(rec.valid[:rec.t].sum())
    paths = []
    for i, g in enumerate(games[:: max(1, len(games) // 12)]):
        paths.append(tmp_path / f"g{i}.npz")
        g.save(paths[-1])
        h, ok = oracle_replay(g)
        assert ok and h == g.final_state_hash, g.meta
    back = [Trajectory.load(p) for p in paths]
    assert validate_on_device(games).all()
    assert validate_on_device(back).all()
