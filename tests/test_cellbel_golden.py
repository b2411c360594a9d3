"""The oracle's restatement of the reference's GPU belief kernels, pinned to
the reference itself.

tests/golden/ref_cell_beliefs.npz was recorded by make_cellbel_golden.py from
the reference's own junqi_cuda extension on a B200 (a HALF_DARK GpuRollout
of 5 envs, 600 plies); ref_cell_beliefs_late.npz by the same script with
--late (16 thinned late-game positions, 600 plies, with flag captures and
eats of non-flag pieces on strongholds, the only plies belief.cu's R4 and
R6 act on).  Here the oracle seeds beliefs on the recorded reset
state (belief.cu:172-248), then applies every recorded step to the recorded
post-step state (belief.cu:255-565); at each recorded ply its belief planes
-- encoded by the oracle's caller-belief observation, the reference GPU
encoder's rule (observation.cu:330-370) -- must equal the reference's.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
FIELDS = {"piece_seat_arr": "piece_seat", "piece_type_arr": "piece_type", "alive": "alive", "pos_x": "pos_x",
          "pos_y": "pos_y", "cell_piece_id": "cell_pid", "seat_dead_arr": "seat_dead", "terminated": "terminated"}


def _load(orc, z, prefix, t=None):
    for k, name in FIELDS.items():
        a = z[prefix + k] if t is None else z[prefix + k][t]
        orc.a[name][...] = a.reshape(orc.a[name].shape).astype(orc.a[name].dtype)


def _planes(orc, bel, ch):
    out = np.zeros((orc.n, 4, len(ch), 17, 17), np.float32)
    for o in range(4):
        sp, _ = orc.obs_beliefs(bel, observers=np.full(orc.n, o, np.int8))
        out[:, o] = sp[:, ch]
    return out


@pytest.mark.parametrize("name", ["ref_cell_beliefs", "ref_cell_beliefs_late"])
def test_oracle_cell_beliefs_match_the_reference_gpu_rollout(name):
    z = np.load(GOLDEN / f"{name}.npz")
    n = z["init_alive"].shape[0]
    ch = z["bel_channels"]
    starts = np.concatenate([[0], np.cumsum(z["snap_len"])])
    # sparse planes: flat indices stored as differences within each snapshot
    snaps = {int(t): (np.cumsum(z["snap_index_delta"][starts[k]:starts[k + 1]].astype(np.int64)),
                      z["snap_value"][starts[k]:starts[k + 1]])
             for k, t in enumerate(z["snap_ply"])}
    orc = O.OracleBatch(n, 2, rules=1)
    _load(orc, z, "init_")
    bel = np.zeros((n, 4, 12, 289), np.float32)
    orc.cellbel_init(z["prior"], bel)

    def check(t):
        idx, val = snaps[t]
        ref = np.zeros(n * 4 * len(ch) * 289, np.float32)
        ref[idx] = val
        got = _planes(orc, bel, ch)
        ref = ref.reshape(got.shape)
        if not np.array_equal(got, ref):
            bad = np.argwhere(got != ref)[:5]
            raise AssertionError(f"ply {t}: belief planes differ at {bad.tolist()}")

    check(0)
    plies = z["event"].shape[0]
    for t in range(1, plies + 1):
        _load(orc, z, "post_", t - 1)
        orc.cellbel_update(z["event"][t - 1], z["flag_captured"][t - 1], z["world_action"][t - 1],
                           z["prev_dead"][t - 1], z["strongholds"], bel)
        if t in snaps:
            check(t)
    assert len(snaps) >= 10
    ev = z["event"]
    assert (ev == 2).any() and (ev == 3).any() and (ev == 4).any()
    if name.endswith("_late"):  # the capture rules fired
        dst = z["world_action"] % 289
        sh_eat = (ev == 2) & (z["flag_captured"] == 0) & np.isin(dst, z["strongholds"]) & (z["world_action"] >= 0)
        assert z["flag_captured"].sum() > 0 and sh_eat.sum() > 0
