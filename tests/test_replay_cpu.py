"""The replay format (junqi_core/replay.py) on the CPU.

Games recorded and saved by junqi_core itself (tests/golden/replay, made by
make_replay_golden.py) load through ``junqi_b200.replay.Trajectory``;
replaying their action logs on the oracle (GameState rule set) reaches the
recorded final Zobrist hash; saving and loading round-trips every field;
malformed logs are refused at the file boundary as the reference refuses
them (replay.py:126-156); a planted corruption of the log breaks the
self-check.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from junqi_b200.replay import Trajectory
from oracle import oracle as O

GOLD = sorted((Path(__file__).parent / "golden" / "replay").glob("ref_game_*.npz"))


def oracle_replay(tr: Trajectory) -> tuple[int, bool]:
    """Final hash, and whether every action was a legal move of its row's
    seat on that seat's turn, replayed on the CPU oracle."""
    orc = O.OracleBatch(1, tr.show_mode, rules=1)
    orc.reset_env(0, tr.setups.reshape(120))
    if tr.first_seat:
        orc.a["turn"][0] = tr.first_seat
        orc.a["zobrist"][:] = O.zobrist_recompute(orc.a, tr.show_mode)
    ok = True
    for row, a in zip(tr.actions, tr.world_actions()):
        _, legal = orc.legal()
        ok &= bool(a in legal) and int(row[0]) == int(orc["turn"][0])  # GameState.step_inplace's checks
        ok &= bool(orc.step(np.array([a], np.int32))["valid"][0])
    return int(orc["zobrist"][0]), ok


def test_reference_games_load_and_replay_to_their_hash():
    assert len(GOLD) == 3
    for path in GOLD:
        tr = Trajectory.load(path)
        assert tr.rules_version == "1.1.0" and tr.state_version == "2.0"
        h, ok = oracle_replay(tr)
        assert ok, path.name
        assert h == tr.final_state_hash, path.name


def test_save_load_round_trip_keeps_the_reference_keys(tmp_path):
    tr = Trajectory.load(GOLD[0])
    tr.meta = {"source": "test", "env": 3}
    p = tmp_path / "g.npz"
    tr.save(p)
    with np.load(p) as a, np.load(GOLD[0]) as b:
        assert set(b.files) <= set(a.files)
        for k in b.files:
            if k != "meta_json":
                assert a[k].dtype == b[k].dtype and np.array_equal(a[k], b[k]), k
    back = Trajectory.load(p)
    assert np.array_equal(back.setups, tr.setups) and np.array_equal(back.actions, tr.actions)
    assert (back.final_state_hash, back.first_seat, back.show_mode, back.meta) == \
        (tr.final_state_hash, tr.first_seat, tr.show_mode, tr.meta)


@pytest.mark.parametrize("row,msg", [((4, 6, 16, 6, 15), "seat"), ((0, 17, 16, 6, 15), "coordinates"),
                                     ((0, 6, 16, 6, 16), "differ"), ((0, 0, 0, 6, 15), "off playable")])
def test_malformed_rows_are_refused(row, msg):
    tr = Trajectory.load(GOLD[0])
    with pytest.raises(ValueError, match=msg):
        Trajectory(setups=tr.setups, actions=np.array([row], np.int16), rng_seed=-1, final_state_hash=0)


def test_planted_corruption_breaks_the_self_check():
    tr = Trajectory.load(GOLD[1])
    bad = tr.actions.copy()
    bad[[10, 11]] = bad[[11, 10]]  # two plies swapped
    h, ok = oracle_replay(Trajectory(setups=tr.setups, actions=bad, rng_seed=-1,
                                     final_state_hash=tr.final_state_hash, show_mode=tr.show_mode))
    assert not ok or h != tr.final_state_hash
