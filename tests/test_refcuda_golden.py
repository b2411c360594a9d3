"""The two formats junqi_core does not define, pinned to the reference's own
CUDA extension (tests/golden/ref_cuda_slots_beliefs.npz, recorded on a B200
by tests/golden/make_refcuda_golden.py):

* the per-piece 80-slot legal mask of ``legal_action_mask_batch``
  (game_state.cu:1985-2197): every slot of every piece, for the side to move
  and for the next seat, on fresh, mid-game (finished games and dead seats
  included) and late-game positions;
* observations from caller-given per-cell beliefs
  (``build_observation_batch``): the belief planes 12-23 / 27-50 and all 28
  globals, global[0:24] being the reference's float sums of the beliefs over
  the enemy cells (exact here: the inputs are multiples of 1/16).

The CPU oracle restatement is checked without a GPU; the CUDA path
(jq_legal_slots, jq_observe_beliefs) with one.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden.make_refcuda_golden import beliefs_x16

FIXTURE = Path(__file__).resolve().parent / "golden" / "ref_cuda_slots_beliefs.npz"


def _fixture() -> dict:
    with np.load(FIXTURE) as z:
        return {k: z[k] for k in z.files}


def _state(fx) -> dict:
    return {k[len("init_"):]: v for k, v in fx.items() if k.startswith("init_")}


def _ref_masks(fx) -> np.ndarray:
    return np.unpackbits(fx["ref_slot_mask"], axis=-1)[..., :80].astype(bool)


def _ref_planes(fx, n) -> np.ndarray:
    nch = len(fx["bel_channels"])
    planes = np.zeros(len(fx["show_modes"]) * n * 4 * nch * 289, np.float32)
    planes[fx["ref_bel_index"]] = fx["ref_bel_value"]
    return planes.reshape(len(fx["show_modes"]), n, 4, nch, 289)


def _first_diff(got, exp) -> str:
    d = np.argwhere(got != exp)
    return f"{len(d)} entries differ, first at {d[0].tolist()}" if len(d) else ""


def test_oracle_slot_mask_equals_the_reference_extension():
    fx = _fixture()
    st = _state(fx)
    n = st["turn"].shape[0]
    orc = O.OracleBatch(n, 2, rules=1)
    O.load_state(orc, st, init_beliefs=False)
    ref = _ref_masks(fx)
    assert ref.any()
    for j, seats in enumerate(fx["slot_seats"]):
        got, _ = orc.slot_mask(seats)
        assert np.array_equal(got.astype(bool), ref[j]), _first_diff(got.astype(bool), ref[j])


def test_oracle_caller_belief_observation_equals_the_reference_extension():
    fx = _fixture()
    st = _state(fx)
    n = st["turn"].shape[0]
    bel = beliefs_x16(n).astype(np.float32) / 16.0
    planes = _ref_planes(fx, n)
    ch = fx["bel_channels"]
    for m, mode in enumerate(fx["show_modes"]):
        orc = O.OracleBatch(n, int(mode), rules=1)
        O.load_state(orc, st, init_beliefs=False)
        for j in range(4):
            sp, gl = orc.obs_beliefs(bel, np.ascontiguousarray(fx["observers"][:, j]))
            got = sp.reshape(n, 317, 289)[:, ch]
            assert np.array_equal(got, planes[m, :, j]), f"mode {mode} slot {j}: " + _first_diff(got, planes[m, :, j])
            assert np.array_equal(gl.view(np.uint32), fx["ref_global"][m, :, j].view(np.uint32)), \
                f"mode {mode} slot {j}: globals " + _first_diff(gl, fx["ref_global"][m, :, j])


@pytest.mark.gpu
def test_cuda_slot_mask_and_caller_belief_observation_equal_the_reference_extension():
    import torch

    from junqi_b200 import _native as N
    from junqi_b200 import tables
    from junqi_b200.env import JunqiEnvB200
    fx = _fixture()
    st = _state(fx)
    n = st["turn"].shape[0]
    ref = _ref_masks(fx)
    planes = _ref_planes(fx, n)
    bel = torch.from_numpy(beliefs_x16(n).astype(np.float32) / 16.0).cuda()
    observers = torch.from_numpy(np.ascontiguousarray(fx["observers"].reshape(-1))).cuda()
    ch = torch.from_numpy(fx["bel_channels"].astype(np.int64)).cuda()
    for m, mode in enumerate(fx["show_modes"]):
        env = JunqiEnvB200(n, show_mode=int(mode), pool=tables.build_setup_pool(4, seed=1), rules=N.RULES_GAMESTATE)
        env.load_state(st, init_beliefs=False)
        if m == 0:
            for j, seats in enumerate(fx["slot_seats"]):
                got = env.legal_slots(torch.from_numpy(np.ascontiguousarray(seats))).cpu().numpy().astype(bool)
                assert np.array_equal(got, ref[j]), _first_diff(got, ref[j])
        sp, gl = env.observe(observers, seats_per_env=4, beliefs=bel)
        got = sp.reshape(n, 4, 317, 289).index_select(2, ch).cpu().numpy()
        assert np.array_equal(got, planes[m]), f"mode {mode}: " + _first_diff(got, planes[m])
        g = gl.reshape(n, 4, 28).cpu().numpy()
        assert np.array_equal(g.view(np.uint32), fx["ref_global"][m].view(np.uint32)), \
            f"mode {mode}: globals " + _first_diff(g, fx["ref_global"][m])
