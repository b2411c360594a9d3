"""The reference-compatible ``junqi_cuda`` surface (junqi_b200.junqi_cuda).

Drives the module the way the reference's own GPU parity tests drive the
original extension (tests/test_gpu_step_batch.py, test_gpu_csr_mask.py,
test_gpu_obs_parity.py in freezeng123456/JunQi): upload a batch through
``copy_from_host`` with the reference's dictionary keys, step it with
``step_batch``, query legal actions in the dense / CSR / canonical-mask
forms, build observations, reset from an uploaded pool -- and compare with
the CPU oracle at every step.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from junqi_b200 import junqi_cuda as jc
from junqi_b200 import tables
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REF_KEYS = {"piece_seat_arr": "piece_seat", "piece_type_arr": "piece_type", "alive": "alive", "pos_x": "pos_x",
            "pos_y": "pos_y", "zero_x": "zero_x", "zero_y": "zero_y", "move_count_arr": "move_count",
            "active_eat_arr": "active_eat", "passive_surv_arr": "passive_surv", "death_reason_arr": "death_reason",
            "death_step_arr": "death_step", "death_loc_flat_arr": "death_loc", "cell_piece_id": "cell_pid",
            "seat_dead_arr": "seat_dead", "seat_flag_revealed_arr": "seat_flag", "turn": "turn",
            "zobrist": "zobrist", "move_counter": "move_counter", "moves_since_last_combat": "mslc"}


def _setup():
    jc.set_device(0)
    jc.init_tables()
    jc.gpu_scratch_reset()
    z = tables.zobrist_tables()
    jc.upload_zobrist_tables(z["piece"].ravel(), z["turn"], z["move_counter"], z["mslc"], z["winner"],
                             int(z["terminated"][0]), int(z["draw"][0]), z["seat_dead"], z["seat_flag"])


def _pack(orc: O.OracleBatch) -> dict:
    d = {ref: orc.a[m].reshape(-1).copy() for ref, m in REF_KEYS.items()}
    for k in ("alive", "seat_dead_arr", "seat_flag_revealed_arr"):
        d[k] = d[k].astype(bool)
    return d


def test_step_batch_and_legal_forms_match_oracle():
    _setup()
    n = 24
    pool = tables.build_setup_pool(n, seed=31)
    orc = O.OracleBatch(n, 2)
    for e in range(n):
        orc.reset_env(e, pool[e])
    state = jc.DeviceGameStateBatch(n)
    state.copy_from_host(_pack(orc))
    state.copy_termination_from_host(np.zeros(n, bool), np.full(n, -1, np.int8), np.zeros(n, bool))
    rng = np.random.default_rng(4)
    for step in range(120):
        turn = state.copy_turn_to_host()
        assert np.array_equal(turn, orc["turn"])
        ids, counts = jc.legal_action_ids_batch(state, turn)
        off, val = jc.legal_action_ids_batch_csr(state, turn)
        o_off, o_val = orc.legal()
        assert np.array_equal(off, o_off) and np.array_equal(val, o_val), f"CSR differs at step {step}"
        for e in range(n):
            assert np.array_equal(ids[e, :counts[e]], o_val[o_off[e]:o_off[e + 1]])
        ptr = jc.legal_mask_canonical_batch(state, turn)
        mask = state._mask.cpu().numpy().astype(bool)
        assert ptr == state._mask.data_ptr()
        for e in range(0, n, 5):
            assert np.array_equal(mask[e], orc.canonical_mask(o_val[o_off[e]:o_off[e + 1]], int(turn[e])))
        acts = np.array([val[off[e] + rng.integers(counts[e])] if counts[e] else 0 for e in range(n)], np.int32)
        r = state.step_batch(acts)
        ro = orc.step(acts)
        for k, ok in (("valid", "valid"), ("event", "event"), ("terminated", "terminated"),
                      ("winner_team", "winner"), ("draw", "draw"), ("flag_captured", "flag_captured")):
            assert np.array_equal(np.asarray(r[k]).astype(np.int64), ro[ok].astype(np.int64)), (step, k)
        h = state.copy_to_host()
        for ref, m in REF_KEYS.items():
            assert np.array_equal(np.asarray(h[ref]).astype(np.int64).reshape(-1),
                                  orc.a[m].astype(np.int64).reshape(-1)), (step, ref)
    cm = state.cm_copy_to_host()
    assert np.array_equal(cm["chain_lo"], orc["cm_chain_lo"].reshape(-1))
    assert np.array_equal(cm["rank_floor"], orc["cm_rank_floor"].reshape(-1))


def test_reset_pool_and_single_seat_observation_match_oracle():
    _setup()
    n = 16
    pool = tables.build_setup_pool(40, seed=12)
    jc.upload_setup_pool(pool)
    state = jc.DeviceGameStateBatch(n)
    state.copy_termination_from_host(np.ones(n, bool), np.full(n, -1, np.int8), np.zeros(n, bool))
    jc.reset_terminated_envs(state, 99)
    from junqi_b200 import _native as N
    orc = O.OracleBatch(n, 2)
    for e in range(n):
        orc.reset_env(e, pool[N.lib().jq_pool_index(99, 1, e, pool.shape[0])])
    h = state.copy_to_host()
    assert np.array_equal(h["zobrist"], orc["zobrist"])
    obs = jc.DeviceObservationSingleBatch(n)
    seats = torch.from_numpy(orc["turn"].copy()).cuda()
    jc.build_observation_single_seat(state, obs, seats.data_ptr(), 2)
    sp, gl = obs.copy_to_host()
    osp, ogl = orc.obs()
    assert np.array_equal(sp, osp) and np.array_equal(gl, ogl)
    # build_observation_batch with per-cell beliefs (a belief network's output, say)
    bel = np.random.default_rng(3).random((n, 4, 12, 289)).astype(np.float32)
    bel[bel < 0.3] = 0.0
    obs4 = jc.DeviceObservationBatch(n)
    jc.build_observation_batch(state, bel, np.tile(np.arange(4, dtype=np.int8), (n, 1)), obs4, 2)
    sp4, gl4 = obs4.copy_to_host()
    for s in range(4):
        o_sp, o_gl = orc.obs_beliefs(bel, np.full(n, s, np.int8))
        assert np.array_equal(sp4[:, s], o_sp) and np.array_equal(gl4[:, s], o_gl)
    # the uploaded beliefs stay in use (resident / single-seat builds) until init_all_beliefs
    jc.build_observation_single_seat(state, obs, seats.data_ptr(), 2)
    sp1, gl1 = obs.copy_to_host()
    o_sp, o_gl = orc.obs_beliefs(bel)
    assert np.array_equal(sp1, o_sp) and np.array_equal(gl1, o_gl)
    jc.init_all_beliefs(state)
    jc.build_observation_single_seat(state, obs, seats.data_ptr(), 2)
    assert np.array_equal(obs.copy_to_host()[0], osp)


def test_step_device_pointer_dict():
    _setup()
    n = 8
    state = jc.DeviceGameStateBatch(n)
    jc.upload_setup_pool(tables.build_setup_pool(8, seed=2))
    state.copy_termination_from_host(np.ones(n, bool), np.full(n, -1, np.int8), np.zeros(n, bool))
    jc.reset_terminated_envs(state, 5)
    turn = torch.zeros(n, dtype=torch.int8, device="cuda")
    acts = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    d = jc.step_device(state, acts.data_ptr(), turn.data_ptr())
    assert d["N"] == n and all(isinstance(v, int) for v in d.values())
    assert not state._out["valid"].any()


def test_legal_action_mask_batch_is_the_80_slot_mask():
    _setup()
    n = 12
    pool = tables.build_setup_pool(n, seed=41)
    orc = O.OracleBatch(n, 2)
    for e in range(n):
        orc.reset_env(e, pool[e])
    state = jc.DeviceGameStateBatch(n)
    state.copy_from_host(_pack(orc))
    seats = orc["turn"].copy()
    m = jc.legal_action_mask_batch(state, seats)
    assert m.shape == (n, 120, 80) and m.dtype == bool
    exp, _ = orc.slot_mask(seats)
    assert np.array_equal(m, exp)


def test_reference_gpu_belief_calls_follow_the_oracle():
    """use_reference_gpu_beliefs(True): the reference's belief calls
    (init_all_beliefs, snapshot_pre_step_flags, update_beliefs_after_step,
    init_beliefs_for_reset_envs) keep a resident per-cell tensor equal to
    the oracle's restatement of belief.cu, and the resident observation
    reads it."""
    _setup()
    n = 16
    pool = tables.build_setup_pool(n, seed=57)
    orc = O.OracleBatch(n, 2, rules=1)
    for e in range(n):
        orc.reset_env(e, pool[e])
    state = jc.DeviceGameStateBatch(n, rules=1)
    state.copy_from_host(_pack(orc))
    state.copy_termination_from_host(np.zeros(n, bool), np.full(n, -1, np.int8), np.zeros(n, bool))
    prior = tables.prior_table()
    zx, zy = orc["zero_x"][0].astype(int), orc["zero_y"][0].astype(int)
    sh = np.array([zy[s * 30 + k] * 17 + zx[s * 30 + k] for s in range(4) for k in (26, 28)], np.int16)
    jc.upload_belief_prior_table(prior.ravel())
    jc.upload_seat_strongholds(sh)
    jc.use_reference_gpu_beliefs(True)
    try:
        jc.init_all_beliefs(state)
        bel = np.zeros((n, 4, 12, 289), np.float32)
        orc.cellbel_init(prior, bel)
        assert np.array_equal(jc._beliefs.cpu().numpy(), bel)
        rng = np.random.default_rng(5)
        for t in range(60):
            off, val = orc.legal()
            acts = np.array([val[off[e] + rng.integers(off[e + 1] - off[e])] if off[e + 1] > off[e] else -1
                             for e in range(n)], np.int32)
            prev_dead = orc["seat_dead"].copy()
            jc.snapshot_pre_step_flags(state)
            state.step_batch(acts)
            d_acts = torch.from_numpy(acts).cuda()
            jc.update_beliefs_after_step(state, state._out["event"].data_ptr(),
                                         state._out["flag_captured"].data_ptr(), d_acts.data_ptr())
            r = orc.step(acts)
            orc.cellbel_update(r["event"], r["flag_captured"], acts, prev_dead, sh, bel)
            assert np.array_equal(jc._beliefs.cpu().numpy(), bel), t
        # re-seed the envs a snapshot sees terminated, as after a reset
        term = np.zeros(n, bool)
        term[::3] = True
        state.copy_termination_from_host(term, np.full(n, -1, np.int8), np.zeros(n, bool))
        jc.snapshot_pre_step_flags(state)
        jc.init_beliefs_for_reset_envs(state)
        orc.cellbel_init(prior, bel, envs=np.nonzero(term)[0])
        assert np.array_equal(jc._beliefs.cpu().numpy(), bel)
        # the resident observation reads the tensor
        jc.upload_observer_seats(n, np.tile(np.arange(4, dtype=np.int8), (n, 1)))
        obs = jc.DeviceObservationBatch(n)
        jc.build_observation_batch_resident(state, obs, 2)
        sp, _ = obs.copy_to_host()
        o_sp, _ = orc.obs_beliefs(bel, observers=np.zeros(n, np.int8))
        assert np.array_equal(np.asarray(sp).reshape(n, 4, 317, 17, 17)[:, 0, 12:51], o_sp[:, 12:51])
    finally:
        jc.use_reference_gpu_beliefs(False)
        jc.gpu_scratch_reset()


def test_leaving_reference_belief_mode_restores_default_observations():
    """use_reference_gpu_beliefs(False) drops the resident per-cell tensor:
    the next resident observation is the default-mode one again, and
    gpu_scratch_reset also leaves the mode."""
    _setup()
    n = 12
    pool = tables.build_setup_pool(n, seed=61)
    orc = O.OracleBatch(n, 2, rules=1)
    for e in range(n):
        orc.reset_env(e, pool[e])
    state = jc.DeviceGameStateBatch(n, rules=1)
    state.copy_from_host(_pack(orc))
    state.copy_termination_from_host(np.zeros(n, bool), np.full(n, -1, np.int8), np.zeros(n, bool))
    jc.init_all_beliefs(state)
    jc.upload_observer_seats(n, np.tile(np.arange(4, dtype=np.int8), (n, 1)))
    obs = jc.DeviceObservationBatch(n)
    jc.build_observation_batch_resident(state, obs, 2)
    default_sp, default_gl = (np.array(a) for a in obs.copy_to_host())
    prior = tables.prior_table()
    zx, zy = orc["zero_x"][0].astype(int), orc["zero_y"][0].astype(int)
    sh = np.array([zy[s * 30 + k] * 17 + zx[s * 30 + k] for s in range(4) for k in (26, 28)], np.int16)
    jc.upload_belief_prior_table(prior.ravel())
    jc.upload_seat_strongholds(sh)
    jc.use_reference_gpu_beliefs(True)
    try:
        jc.init_all_beliefs(state)
        assert jc._beliefs is not None
        jc.use_reference_gpu_beliefs(False)
        assert jc._beliefs is None
        jc.build_observation_batch_resident(state, obs, 2)
        sp, gl = obs.copy_to_host()
        assert np.array_equal(sp, default_sp) and np.array_equal(gl, default_gl)
        jc.use_reference_gpu_beliefs(True)
        jc.gpu_scratch_reset()
        assert not jc._cell_mode and jc._beliefs is None
    finally:
        jc.use_reference_gpu_beliefs(False)
        jc.gpu_scratch_reset()
