"""jq_cell_beliefs_* against the oracle restatement of the reference's GPU
belief kernels (belief.cu:172-248 init, 255-565 update), bit for bit over
whole (N, 4, 12, 289) tensors.

Rollouts from late-game starts (few pieces, so combats, stronghold eats and
flag captures come early) step through jq_step without resets; the device
tensor and the oracle's are compared after the initial seeding, after every
ply and after a masked re-seeding of half the envs.  Beliefs uploaded with
values the rules never produce (tiny, one-hot-like, NaN-free noise) go
through the same comparison, which exercises the float tests on them.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N
from junqi_b200 import tables
from junqi_b200.env import JunqiEnvB200
from junqi_b200.workloads import late_game_starts
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def stronghold_cells(lineup: np.ndarray) -> np.ndarray:
    """Each seat's two stronghold flat cells (slots 26 and 28), from a reset."""
    o = O.OracleBatch(1)
    o.reset_env(0, lineup)
    zx, zy = o.a["zero_x"][0].astype(int), o.a["zero_y"][0].astype(int)
    return np.array([zy[s * 30 + k] * 17 + zx[s * 30 + k] for s in range(4) for k in (26, 28)], np.int16)


def _rollout(n, seed, plies, prior, noise=False):
    pool = tables.build_setup_pool(64, seed=seed)
    env = JunqiEnvB200(n, pool=pool, rules=N.RULES_GAMESTATE)
    env.reset(seed=seed)
    late_game_starts(env, seed)
    orc = O.OracleBatch(n, env.show_mode, rules=N.RULES_GAMESTATE)
    O.load_state(orc, env.state(), init_beliefs=False)
    sh = stronghold_cells(pool[0])
    sh_d = torch.from_numpy(sh).cuda()
    prior_d = torch.from_numpy(prior).cuda()
    bel_d = torch.full((n, 4, 12, 289), 7.0, dtype=torch.float32, device="cuda")
    bel_o = np.full((n, 4, 12, 289), 7.0, np.float32)
    env.cell_beliefs_init(bel_d, prior_d)
    orc.cellbel_init(prior, bel_o)
    assert np.array_equal(bel_d.cpu().numpy(), bel_o), "initial seeding"
    if noise:
        rng = np.random.default_rng(seed)
        pick = rng.random(bel_o.shape) < 0.02
        vals = rng.choice(np.array([1e-9, 3e-9, 0.9999995, 0.5, 1.0, 0.0], np.float32), size=bel_o.shape)
        bel_o[pick] = vals[pick]
        bel_d.copy_(torch.from_numpy(bel_o))
    seen = np.zeros(5, np.int64)
    fcaps = 0
    for t in range(1, plies + 1):
        prev_dead, _ = env.cell_beliefs_snapshot()
        pd_o = orc.a["seat_dead"].copy()
        acts = env.sample_uniform(seed, t)
        a = acts.cpu().numpy().copy()
        out = env.step(acts)
        r = orc.step(a)
        assert np.array_equal(out["event"].cpu().numpy().astype(r["event"].dtype), r["event"]), t
        env.cell_beliefs_update(bel_d, acts, prev_dead, sh_d)
        orc.cellbel_update(r["event"], r["flag_captured"], a, pd_o, sh, bel_o)
        got = bel_d.cpu().numpy()
        if not np.array_equal(got, bel_o):
            bad = np.nonzero((got != bel_o).reshape(n, -1).any(1))[0]
            raise AssertionError(f"ply {t}: beliefs differ in envs {bad[:8]}")
        seen += np.bincount(r["event"].astype(np.int64), minlength=5)[:5]
        fcaps += int(r["flag_captured"].sum())
    return env, orc, bel_d, bel_o, prior, prior_d, seen, fcaps


def test_cell_beliefs_follow_the_oracle_through_rollouts():
    prior = tables.prior_table()
    env, orc, bel_d, bel_o, prior, prior_d, seen, fcaps = _rollout(64, 31, 160, prior)
    assert seen[1] > 0 and seen[2] > 0 and seen[3] > 0 and seen[4] > 0, seen
    assert fcaps > 0, "no flag capture: R4 not exercised"
    # masked re-seeding (init_beliefs_for_reset_envs): every other env
    mask = (np.arange(env.n) % 2).astype(np.uint8)
    env.cell_beliefs_init(bel_d, prior_d, torch.from_numpy(mask).cuda())
    orc.cellbel_init(prior, bel_o, envs=np.nonzero(mask)[0])
    assert np.array_equal(bel_d.cpu().numpy(), bel_o)


def test_cell_beliefs_with_uploaded_values_the_rules_never_write():
    _rollout(32, 47, 60, tables.prior_table(), noise=True)


def test_cell_beliefs_reject_bad_buffers():
    env = JunqiEnvB200(4, pool=tables.build_setup_pool(4, seed=1))
    env.reset(seed=1)
    prior = torch.from_numpy(tables.prior_table()).cuda()
    with pytest.raises(ValueError):
        env.cell_beliefs_init(torch.zeros((4, 4, 12, 288), device="cuda"), prior)
    bel = torch.zeros((4, 4, 12, 289), device="cuda")
    st = N.lib().jq_cell_beliefs_init(ctypes.byref(env.batch.struct), None, prior.data_ptr(), bel.data_ptr() + 4,
                                      None)
    assert N.STATUS_NAMES.get(st) == "JQ_ERR_ARG"  # misaligned belief buffer
