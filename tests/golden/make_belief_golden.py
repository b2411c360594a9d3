"""Generate the fixture that pins observations built from caller-given beliefs.

Run in a container where the reference checkout is importable, e.g.::

    PYTHONPATH=<reference checkout> python tests/golden/make_belief_golden.py

Writes ``tests/golden/ref_obs_beliefs.npz``.  A few games are played with
``GameState.step`` from seeded random setups; at chosen plies the
observer's ``BeliefTensor`` gets arbitrary per-cell probability vectors
(its ``probs`` dict is keyed by cell, exactly the per-cell belief input of
the reference GPU encoder), and ``ObservationBuilder`` builds the
observation.  Recorded per case: the game (setups + actions up to the
ply), the observer, the per-cell beliefs and the reference's belief planes
(channels 12-50).  Nothing here runs during the test suite.
"""
from __future__ import annotations

import random
from pathlib import Path

import numpy as np

from junqi_core.info_model import BeliefTensor
from junqi_core.observation import ObservationBuilder
from junqi_core.rules import Seat, ShowMode
from junqi_core.setup import generate_random_setup
from junqi_core.state import Action, GameState

OUT = Path(__file__).resolve().parent / "ref_obs_beliefs.npz"
GAMES = [(11, ShowMode.HALF_DARK, (0, 37, 120)), (12, ShowMode.DARK, (5, 90)), (13, ShowMode.BRIGHT, (64,))]


def main() -> None:
    builder = ObservationBuilder()
    sp = np.zeros((317, 17, 17), np.float32)
    gl = np.zeros(28, np.float32)
    rows = {k: [] for k in ("game", "ply", "observer", "beliefs", "planes")}
    setups, actions, modes = [], [], []
    for gi, (seed, mode, plies) in enumerate(GAMES):
        rng = random.Random(seed)
        vrng = np.random.default_rng(seed)
        lineups = generate_random_setup(random.Random(seed))
        g = GameState.new_game(lineups, show_mode=mode)
        setups.append(np.array([[int(t) for t in lu] for lu in lineups], np.int8))
        modes.append(int(mode.value))
        acts = []
        for t in range(max(plies) + 1):
            if t in plies:
                for o in range(4):
                    bel = BeliefTensor.initial(g, Seat(o))
                    cells = np.zeros((12, 289), np.float32)
                    for pid in np.flatnonzero(g.alive):
                        f = int(g.pos_y[pid]) * 17 + int(g.pos_x[pid])
                        kind = vrng.integers(4)
                        if kind == 0:
                            v = np.zeros(12, np.float32)
                        elif kind == 1:
                            v = np.eye(12, dtype=np.float32)[vrng.integers(12)]
                        else:
                            v = vrng.random(12).astype(np.float32)
                            v[vrng.random(12) < 0.3] = 0.0
                            if kind == 3:
                                v /= max(float(v.sum()), 1e-6)
                                v = v.astype(np.float32)
                        bel.probs[(int(g.pos_x[pid]), int(g.pos_y[pid]))] = v
                        cells[:, f] = v
                    builder.build_into(g, bel, Seat(o), sp, gl)
                    rows["game"].append(gi)
                    rows["ply"].append(t)
                    rows["observer"].append(o)
                    rows["beliefs"].append(cells)
                    rows["planes"].append(sp[12:51].copy())
            ids = g.legal_action_ids()
            if g.terminated or len(ids) == 0:
                break
            a = int(rng.choice(list(ids)))
            acts.append(a)
            sf, df = a // 289, a % 289
            g, _ = g.step(Action(seat=g.turn, src=(sf % 17, sf // 17), dst=(df % 17, df // 17)))
        actions.append(np.array(acts, np.int32))
    T = max(len(a) for a in actions)
    act = np.full((len(GAMES), T), -1, np.int32)
    for i, a in enumerate(actions):
        act[i, :len(a)] = a
    np.savez_compressed(OUT, setups=np.stack(setups), show_mode=np.array(modes, np.int8), actions=act,
                        **{k: np.array(v) for k, v in rows.items()})
    print("cases", len(rows["ply"]), "->", OUT)


if __name__ == "__main__":
    main()
