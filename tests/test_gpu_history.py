"""Compact rollout history: records rebuild exactly what the rollout saw.

Mirrors tests/test_compact_rollout_history.py of freezeng123456/JunQi: during
a rollout every env is recorded before each ply; for a sample of (ply, env)
pairs the live observation, global features, legal ids, counts and canonical
mask of the recorded seat are kept.  Rebuilding those records later, in
shuffled order and mixed across plies, must reproduce every kept tensor bit
for bit -- for the acting seat and for another observer seat, in two show
modes.  Out-of-range indices rebuild an empty, terminated env.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N
from junqi_b200 import junqi_cuda as jc
from junqi_b200 import tables
from junqi_b200.env import DARK, HALF_DARK, JunqiEnvB200
from junqi_b200.history import RolloutHistory

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,other_seat", [(HALF_DARK, False), (DARK, True)])
def test_reconstructed_minibatch_equals_the_rollout(mode, other_seat):
    n, plies, keep = 192, 48, 12
    env = JunqiEnvB200(n, show_mode=mode, pool=tables.build_setup_pool(64, seed=3), obs_seats=1,
                       rules=N.RULES_GAMESTATE)
    env.reset(seed=17)
    hist = RolloutHistory(plies, n)
    rng = np.random.default_rng(5)
    kept = []
    for t in range(plies):
        seats = None
        if other_seat:
            seats = ((env.batch["turn"].to(torch.int32) + 2) % 4).to(torch.int8)
            env.legal(seats)
        hist.snapshot(env.batch, t, seats)
        sp, gl = env.observe(seats, seats_per_env=1)
        for e in rng.choice(n, keep, replace=False):
            e = int(e)
            c = int(env.counts[e])
            kept.append((t * n + e, sp[e].clone(), gl[e].clone(), env.mask[e].clone(), c, env.ids[e, :c].clone()))
        if other_seat:
            env.legal()
        env.ply(env.sample_softmax(17, t + 1), seed=17, ply=t + 1)
    order = rng.permutation(len(kept))
    for lo in range(0, len(order), 100):
        sel = [kept[i] for i in order[lo:lo + 100]]
        out = hist.reconstruct([s[0] for s in sel], show_mode=mode)
        for j, (idx, sp, gl, mask, c, ids) in enumerate(sel):
            assert torch.equal(out["spatial"][j].view(torch.int32), sp.view(torch.int32)), f"record {idx}: observation"
            assert torch.equal(out["global"][j].view(torch.int32), gl.view(torch.int32)), f"record {idx}: globals"
            assert torch.equal(out["mask"][j], mask), f"record {idx}: canonical mask"
            assert int(out["counts"][j]) == c, f"record {idx}: legal count"
            assert torch.equal(out["ids"][j, :c], ids), f"record {idx}: legal ids"


def test_out_of_range_index_is_an_empty_env():
    hist = RolloutHistory(2, 8)
    env = JunqiEnvB200(8, pool=tables.build_setup_pool(8, seed=1), with_obs=False)
    env.reset(seed=1)
    hist.snapshot(env.batch, 0)
    out = hist.reconstruct([0, 16, -1, 7])
    counts = out["counts"].cpu().numpy()
    assert counts[0] > 0 and counts[3] > 0 and counts[1] == 0 and counts[2] == 0
    assert not out["mask"][1].any() and not out["mask"][2].any()
    assert hist.record_bytes % 16 == 0 and hist.history_bytes == 16 * hist.record_bytes


def test_reference_surface_device_rollout_history():
    """The junqi_cuda surface: snapshot with device acting seats, reconstruct
    from device indices, read the outputs through the returned pointers."""
    jc.set_device(0)
    jc.init_tables()
    n, steps = 8, 4
    jc.upload_setup_pool(tables.build_setup_pool(16, seed=4))
    state = jc.DeviceGameStateBatch(n)
    state.copy_termination_from_host(np.ones(n, bool), np.full(n, -1, np.int8), np.zeros(n, bool))
    jc.reset_terminated_envs(state, 9)
    h = jc.DeviceRolloutHistory(steps, n)
    obs = jc.DeviceObservationSingleBatch(n)
    rng = np.random.default_rng(2)
    exp_sp, exp_gl, exp_mask, exp_seats = [], [], [], []
    for t in range(steps):
        acting = torch.from_numpy(state.copy_turn_to_host()).cuda()
        jc.build_observation_single_seat(state, obs, acting.data_ptr(), 2)
        ptr = jc.legal_mask_canonical_batch_from_device(state, acting.data_ptr())
        h.snapshot(state, acting.data_ptr(), t)
        exp_sp.append(obs.spatial.clone())
        exp_gl.append(obs.global_.clone())
        exp_mask.append(jc._device_view(ptr, (n, 16641), torch.uint8, "cuda").clone())
        exp_seats.append(acting.clone())
        ids, counts = jc.legal_action_ids_batch(state, acting.cpu().numpy())
        state.step_batch(np.array([ids[e, rng.integers(counts[e])] if counts[e] else 0 for e in range(n)],
                                  np.int32))
        jc.reset_terminated_envs(state, 100 + t)
    idx = torch.tensor([0, n + 1, 2 * n + 2, 3 * n + 3, 5, 3 * n], dtype=torch.int64, device="cuda")
    seats = torch.stack(exp_seats).reshape(-1).index_select(0, idx).contiguous()
    d = h.reconstruct(idx.data_ptr(), seats.data_ptr(), int(idx.numel()), 2)
    b = d["batch_size"]
    assert b == idx.numel() and h.replay_capacity >= b and h.history_bytes == steps * n * h._h.record_bytes
    sp = jc._device_view(d["d_spatial_ptr"], (b, 317, 17, 17), torch.float32, "cuda")
    gl = jc._device_view(d["d_global_ptr"], (b, 28), torch.float32, "cuda")
    mk = jc._device_view(d["d_legal_mask_ptr"], (b, 16641), torch.uint8, "cuda")
    assert torch.equal(sp, torch.stack(exp_sp).reshape(steps * n, 317, 17, 17).index_select(0, idx))
    assert torch.equal(gl, torch.stack(exp_gl).reshape(steps * n, 28).index_select(0, idx))
    assert torch.equal(mk, torch.stack(exp_mask).reshape(steps * n, 16641).index_select(0, idx))
