"""Observations from caller-given per-cell beliefs: the oracle against the reference.

``tests/golden/ref_obs_beliefs.npz`` (made by make_belief_golden.py) holds
reference observations built by ``ObservationBuilder`` from a
``BeliefTensor`` whose per-cell ``probs`` were set to arbitrary vectors
(zero, one-hot, random, normalised).  Replaying each game on the oracle and
building the observation from the same per-cell beliefs must reproduce the
reference's belief planes (channels 12-50) bit for bit.  The reference CPU
path has no per-cell-belief form of global[0:24] (it reads integer
inventories); that part follows the reference GPU encoder and is checked
here against its definition: ordered float32 sums over enemy cells.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle import oracle as O

GOLD = Path(__file__).parent / "golden" / "ref_obs_beliefs.npz"


def _state_at(d, game: int, ply: int) -> O.OracleBatch:
    orc = O.OracleBatch(1, int(d["show_mode"][game]), rules=1)
    orc.reset_env(0, d["setups"][game].reshape(120))
    for a in d["actions"][game, :ply]:
        r = orc.step(np.array([a], np.int32))
        assert r["valid"][0]
    return orc


def test_belief_planes_match_the_reference():
    d = np.load(GOLD)
    assert len(d["ply"]) == 24
    for i in range(len(d["ply"])):
        g, t, o = int(d["game"][i]), int(d["ply"][i]), int(d["observer"][i])
        orc = _state_at(d, g, t)
        bel = np.zeros((1, 4, 12, 289), np.float32)
        bel[0, o] = d["beliefs"][i]
        sp, gl = orc.obs_beliefs(bel, np.array([o], np.int8))
        assert np.array_equal(sp[0, 12:51], d["planes"][i]), (g, t, o)
        # every other channel is the ordinary observation
        sp0, gl0 = orc.obs(np.array([o], np.int8))
        assert np.array_equal(sp[0, :12], sp0[0, :12]) and np.array_equal(sp[0, 51:], sp0[0, 51:])
        assert np.array_equal(gl[0, 24:], gl0[0, 24:])
        # global[0:24]: float32 sums, ascending pid, over left / right enemy cells
        a = orc.a
        for side, lo in ((1, 0), (3, 12)):
            seat = (o + side) % 4
            acc = np.zeros(12, np.float32)
            for p in range(120):
                if a["alive"][0, p] and a["piece_seat"][0, p] == seat:
                    acc = (acc + bel[0, o, :, int(a["pos_y"][0, p]) * 17 + int(a["pos_x"][0, p])]).astype(np.float32)
            assert np.array_equal(gl[0, lo:lo + 12], acc), (g, t, o, side)
