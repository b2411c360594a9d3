"""Pin the CPU oracle to the reference (junqi_core) through the golden fixtures.

Every artefact the fixtures record was produced by junqi_core itself
(tests/golden/make_golden.py); the oracle must reproduce all of them
bit-exactly.  No GPU needed.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests import _golden as G


class OracleDriver:
    def load(self, init, show_mode, rules):
        n = init["turn"].shape[0]
        self.b = O.OracleBatch(n, show_mode, rules=rules)
        O.load_state(self.b, init)

    def legal(self):
        return self.b.legal()

    def masks(self):
        off, val = self.b.legal()
        return np.stack([self.b.canonical_mask(val[off[e]:off[e + 1]], int(self.b["turn"][e]))
                         for e in range(self.b.n)])

    def step(self, actions):
        return self.b.step(actions)

    def state(self):
        return self.b.a

    def obs(self, e, s):
        return self.b.obs_one(e, s)


def test_topology_matches_reference():
    ref = G.tables()
    mine = O.topology()
    for k in ("on_board", "rail", "curve", "rail_adj", "srays", "crays", "compact_to_flat"):
        assert np.array_equal(mine[k], ref[k]), k


def test_prior_table_matches_reference():
    assert np.array_equal(O.prior_table(), G.tables()["prior"])


def test_zobrist_tables_match_reference():
    z = O.zobrist_tables()
    man = G.manifest()["zobrist"]
    for mine, ref in (("piece", "ZOB_PIECE"), ("turn", "ZOB_TURN"), ("mc", "ZOB_MOVE_COUNTER"),
                      ("mslc", "ZOB_MOVES_SINCE_COMBAT"), ("winner", "ZOB_WINNER"),
                      ("seat_dead", "ZOB_SEAT_DEAD"), ("seat_flag", "ZOB_SEAT_FLAG_REVEALED"),
                      ("show_mode", "ZOB_SHOW_MODE")):
        assert G.sha(z[mine]) == man[ref], ref
    assert str(int(z["terminated"][0])) == man["ZOB_TERMINATED"]
    assert str(int(z["draw"][0])) == man["ZOB_DRAW"]


def test_recency_lut_is_elementwise_stable():
    """The LUT equals numpy's exp evaluated one element at a time."""
    lut = O.recency_lut()
    for row, tau in enumerate((32.0, 256.0, 64.0, 128.0)):
        for e in (0, 1, 7, 31, 100, 1000, 4000, 4096):
            one = np.exp(-np.maximum(np.array([e], np.float32), 0.0) / tau, dtype=np.float32)[0]
            assert one.view(np.uint32) == lut[row, e].view(np.uint32)


@pytest.mark.parametrize("name", G.TRAJECTORIES)
def test_oracle_replays_reference_trajectory(name):
    fx = G.load(name)
    n = G.replay(fx, OracleDriver())
    assert n == fx["actions"].shape[0]


@pytest.mark.parametrize("name", G.TRAJECTORIES)
def test_zobrist_recompute_matches_reference_hashes(name):
    """The vectorised from-scratch hash (state.py:1761) equals the reference's
    incremental hash on the initial and final states of every trajectory."""
    fx = G.load(name)
    for pre in ("init_", "final_"):
        st = {k[len(pre):]: v for k, v in fx.items() if k.startswith(pre)}
        assert np.array_equal(O.zobrist_recompute(st, int(fx["show_mode"])), st["zobrist"].astype(np.int64)), pre
