"""The per-piece 80-slot legal mask (reference GPU format, game_state.cu:
1985-2197) on the CPU oracle.

junqi_core has no version of this format, so its slot order is the
restatement of the reference kernel.  What the slots encode is pinned here
against junqi_core: on every golden state and along oracle rollouts, the
(source, destination) pairs of the set slots are exactly the legal actions
junqi_core generates, and no destination appears twice.  The format's own
tables (straight rays, rail adjacency) equal junqi_core's.
"""
from __future__ import annotations

import numpy as np
import pytest

from junqi_b200 import tables
from oracle import oracle as O
from tests import _golden as G


def _pairs_equal_legal(b: O.OracleBatch) -> int:
    mask, dst = b.slot_mask()
    off, val = b.legal()
    checked = 0
    for e in range(b.n):
        seat = int(b["turn"][e])
        if b["terminated"][e] or b["seat_dead"][e][seat]:
            continue
        pairs = []
        for pid in np.nonzero((b["piece_seat"][e] == seat) & (b["alive"][e] == 1))[0]:
            src = int(b["pos_y"][e, pid]) * 17 + int(b["pos_x"][e, pid])
            ds = dst[e, pid][mask[e, pid]]
            assert np.all(ds >= 0)
            pairs += [src * 289 + int(d) for d in ds]
        assert len(pairs) == len(set(pairs)), f"env {e}: a destination is encoded twice"
        assert sorted(pairs) == val[off[e]:off[e + 1]].tolist(), f"env {e}: slots differ from the legal actions"
        assert not mask[e][b["piece_seat"][e] != seat].any()
        checked += 1
    return checked


def test_slot_tables_equal_reference_rays_and_rail_graph():
    st, ref = O.slot_tables(), G.tables()
    assert np.array_equal(st["srays"], ref["srays"])
    assert np.array_equal(st["rail_adj"][:, :4], ref["rail_adj"]) and np.all(st["rail_adj"][:, 4:] == -1)


@pytest.mark.parametrize("name", G.TRAJECTORIES)
def test_slots_encode_the_reference_legal_actions_on_golden_states(name):
    fx = G.load(name)
    for pre in ("init_", "final_"):
        st = {k[len(pre):]: v for k, v in fx.items() if k.startswith(pre)}
        b = O.OracleBatch(st["turn"].shape[0], int(fx["show_mode"]), rules=int(fx["rules"]) if "rules" in fx else 0)
        O.load_state(b, st)
        _pairs_equal_legal(b)


def test_slots_encode_the_legal_actions_along_a_rollout():
    n = 32
    pool = tables.build_setup_pool(n, seed=8)
    b = O.OracleBatch(n, 2, rules=1)
    for e in range(n):
        b.reset_env(e, pool[e])
    rng = np.random.default_rng(8)
    checked = 0
    for t in range(240):
        if t % 20 == 0:
            checked += _pairs_equal_legal(b)
        off, val = b.legal()
        cnt = np.diff(off)
        acts = np.array([val[off[e] + rng.integers(cnt[e])] if cnt[e] else -1 for e in range(n)], np.int32)
        r = b.step(acts)
        for e in np.nonzero(r["terminated"])[0]:
            b.reset_env(int(e), pool[int(rng.integers(n))])
    assert checked > 200
