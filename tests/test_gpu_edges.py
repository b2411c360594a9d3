"""Edge cases of the device path against the oracle.

* Batches that fill no CTA evenly (1 and 13 envs) roll out bit-exactly,
  through terminations and auto-resets from late-game starts.
* A legal-id capacity below the move count keeps the full count, the first
  `cap` ids and a complete canonical mask; the CSR holds min(count, cap).
* Terminated envs and envs whose acting seat is dead have no legal moves
  and an all-zero mask row (batched_state.py:394-399).
* Invalid actions (none, out of range, from an empty cell, in a finished
  game) leave the env untouched and report valid = 0.
* Explicit observer lists of any order give the oracle's observation of
  each listed seat.
* Belief codes uploaded out of step with the board are repaired by the
  next ply's sweep as the oracle repairs them.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N
from junqi_b200 import tables
from junqi_b200.env import HALF_DARK, JunqiEnvB200
from junqi_b200.workloads import late_game_starts
from oracle import oracle as O
from tests.test_gpu_parity import _compare_legal, _compare_obs, _compare_state

pytestmark = pytest.mark.gpu


def _pair(n, seed, rules=N.RULES_GAMESTATE, late=False, **kw):
    pool = tables.build_setup_pool(64, seed=seed)
    env = JunqiEnvB200(n, pool=pool, rules=rules, **kw)
    env.reset(seed=seed)
    if late:
        late_game_starts(env, seed)
    orc = O.OracleBatch(n, env.show_mode, rules=rules)
    O.load_state(orc, env.state(), init_beliefs=False)
    return env, orc, pool


@pytest.mark.parametrize("n", [1, 13])
def test_ragged_batches_roll_out_bit_exactly(n):
    env, orc, pool = _pair(n, 21, late=True)
    L = N.lib()
    ends = 0
    for t in range(1, 401):
        acts = env.sample_uniform(21, t)
        a = acts.cpu().numpy().copy()
        out = env.ply(acts, seed=21, ply=t)
        r = orc.step(a)
        for k in ("valid", "event", "terminated", "winner", "draw", "reward"):
            assert np.array_equal(out[k].cpu().numpy().astype(r[k].dtype), r[k]), (t, k)
        for e in np.nonzero(r["terminated"])[0]:
            orc.reset_env(int(e), pool[L.jq_pool_index(21, t, int(e), pool.shape[0])])
            ends += 1
        _compare_state(env, orc, t)
        _compare_legal(env, orc, t, masks=(t % 25 == 0))
        if t % 100 == 0:
            _compare_obs(env, orc, t, seats=1)
    assert ends >= 1


def test_small_legal_capacity_truncates_ids_not_counts():
    env, orc, _ = _pair(32, 5, legal_cap=4)
    for t in range(1, 30):
        env.ply(env.sample_uniform(5, t), seed=5, ply=t)
    O.load_state(orc, env.state(), init_beliefs=False)
    o_off, o_val = orc.legal()
    counts = env.counts.cpu().numpy()
    ids = env.ids.cpu().numpy()
    assert np.array_equal(counts, np.diff(o_off)) and (counts > 4).any()
    for e in range(32):
        k = min(int(counts[e]), 4)
        assert np.array_equal(ids[e, :k], o_val[o_off[e]:o_off[e] + k])
        exp = orc.canonical_mask(o_val[o_off[e]:o_off[e + 1]], int(orc["turn"][e]))
        assert np.array_equal(env.mask[e].cpu().numpy().astype(bool), exp)
    off, val = env.csr()
    assert np.array_equal(np.diff(off.cpu().numpy()), np.minimum(counts, 4))


def test_finished_games_and_dead_seats_have_no_moves():
    env, orc, _ = _pair(8, 9)
    st = env.state()
    st["terminated"][:3] = 1
    turn = st["turn"].astype(np.int64)
    st["seat_dead"].reshape(8, 4)[3:6, :] = 0
    for e in range(3, 6):
        st["seat_dead"].reshape(8, 4)[e, turn[e]] = 1
    env.batch.load({"terminated": st["terminated"], "seat_dead": st["seat_dead"]})
    env.mask.fill_(1)
    counts, _ = env.legal()
    c = counts.cpu().numpy()
    assert (c[:6] == 0).all() and (c[6:] > 0).all()
    assert not env.mask[:6].any() and env.mask[6:].any()


def test_invalid_actions_leave_the_env_untouched():
    env, orc, _ = _pair(6, 3)
    st = env.state()
    st["terminated"][5] = 1
    env.batch.load({"terminated": st["terminated"]})
    before = env.state()
    empty_src = int(np.nonzero(before["cell_pid"][2] < 0)[0][0])
    acts = torch.tensor([-1, 289 * 289, empty_src * 289 + 10, 16641 * 5 + 7, -7, 0], dtype=torch.int32)
    out = env.step(acts.cuda())
    assert not out["valid"].any()
    after = env.state()
    for k in ("zobrist", "cell_pid", "turn", "move_counter", "alive", "pos_x", "pos_y"):
        assert np.array_equal(before[k], after[k]), k


def test_explicit_observer_lists():
    env, orc, _ = _pair(10, 4)
    for t in range(1, 25):
        env.ply(env.sample_uniform(4, t), seed=4, ply=t)
    O.load_state(orc, env.state(), init_beliefs=False)
    rng = np.random.default_rng(0)
    obs = np.stack([rng.permutation(4)[:3] for _ in range(10)]).astype(np.int8)  # 3 seats per env, any order
    sp, gl = env.observe(torch.from_numpy(obs).cuda(), seats_per_env=3)
    sp, gl = sp.cpu().numpy().reshape(10, 3, 317, 17, 17), gl.cpu().numpy().reshape(10, 3, 28)
    for j in range(3):
        o_sp, o_gl = orc.obs(obs[:, j].copy())
        assert np.array_equal(sp[:, j], o_sp) and np.array_equal(gl[:, j], o_gl), j


@pytest.mark.parametrize("rules", [N.RULES_BATCHED, N.RULES_GAMESTATE])
def test_episode_cap_draws_like_the_oracle(rules):
    """jq_batch.max_moves: games reaching the cap end as draws (after the
    ply's own victory and Q12 rules), with auto-resets continuing."""
    env, orc, pool = _pair(24, 17, rules=rules, max_moves=23)
    orc._c.max_moves = 23
    L = N.lib()
    draws = 0
    for t in range(1, 120):
        acts = env.sample_uniform(17, t)
        a = acts.cpu().numpy().copy()
        out = env.ply(acts, seed=17, ply=t)
        r = orc.step(a)
        for k in ("valid", "terminated", "winner", "draw", "reward"):
            assert np.array_equal(out[k].cpu().numpy().astype(r[k].dtype), r[k]), (t, k)
        draws += int(r["draw"].sum())
        for e in np.nonzero(r["terminated"])[0]:
            orc.reset_env(int(e), pool[L.jq_pool_index(17, t, int(e), pool.shape[0])])
        _compare_state(env, orc, t)
    assert draws >= 24


def test_belief_sweep_repairs_codes_written_by_the_host():
    """Belief codes that contradict the board -- an alive piece with no code,
    a dead piece holding one, as a caller's state upload can leave them --
    are repaired by the next ply's I5 sweep exactly as the oracle repairs
    them, in every 16-code chunk (the sweep skips only chunks whose codes
    already agree with the alive bits)."""
    n, seed = 32, 29
    env, orc, pool = _pair(n, seed, late=True)
    st = env.state()
    codes = np.asarray(st["bel_code"]).reshape(n, 4, 120).copy()
    alive = np.asarray(st["alive"]).reshape(n, 120).astype(bool)
    rng = np.random.default_rng(seed)
    planted = 0
    for e in range(n):
        live, dead = np.nonzero(alive[e])[0], np.nonzero(~alive[e])[0]
        for o in range(4):
            if len(live):
                codes[e, o, rng.choice(live, size=min(3, len(live)), replace=False)] = 0
                planted += 1
            if len(dead):
                codes[e, o, rng.choice(dead, size=min(2, len(dead)), replace=False)] = 14
                planted += 1
    assert planted > 0
    env.batch.load({"bel_code": codes})
    O.load_state(orc, {"bel_code": codes}, init_beliefs=False)
    L = N.lib()
    stepped = np.zeros(n, dtype=bool)
    for t in range(1, 4):
        acts = env.sample_uniform(seed, t)
        a = acts.cpu().numpy().copy()
        out = env.ply(acts, seed=seed, ply=t)
        r = orc.step(a)
        assert np.array_equal(out["valid"].cpu().numpy().astype(r["valid"].dtype), r["valid"]), t
        stepped |= r["valid"].astype(bool)
        for e in np.nonzero(r["terminated"])[0]:
            orc.reset_env(int(e), pool[L.jq_pool_index(seed, t, int(e), pool.shape[0])])
        _compare_state(env, orc, t)
    assert stepped.sum() >= n // 2
    fixed = np.asarray(env.state()["bel_code"]).reshape(n, 4, 120)[stepped]
    alive = np.asarray(env.state()["alive"]).reshape(n, 120).astype(bool)[stepped]
    assert ((fixed != 0) == alive[:, None, :]).all()
    _compare_obs(env, orc, 3, seats=1)


def test_each_env_resets_from_its_own_pool():
    """The setup pool belongs to the batch (jq_batch.pool): two envs alive in
    one process with different pools each reset from their own, whichever
    was built last, and an env's pool outlives another env's."""
    pa = tables.build_setup_pool(16, seed=101)
    pb = tables.build_setup_pool(9, seed=202)
    a = JunqiEnvB200(32, pool=pa, with_obs=False)
    b = JunqiEnvB200(32, pool=pb, with_obs=False)
    L = N.lib()
    for env, pool, seed in ((a, pa, 7), (b, pb, 8), (a, pa, 9)):
        env.reset(seed=seed)
        got = env.batch["piece_type"].cpu().numpy()
        for e in range(env.n):
            lineup = pool[L.jq_pool_index(seed, 0, e, pool.shape[0])]
            exp = np.where(lineup != 0, lineup, -1)
            assert np.array_equal(got[e], exp), (seed, e)
    del b
    import gc
    gc.collect()
    torch.cuda.empty_cache()
    junk = torch.full((1 << 20,), 3, dtype=torch.int8, device="cuda")  # reuse freed memory
    a.reset(seed=10)
    got = a.batch["piece_type"].cpu().numpy()
    for e in range(a.n):
        lineup = pa[L.jq_pool_index(10, 0, e, pa.shape[0])]
        assert np.array_equal(got[e], np.where(lineup != 0, lineup, -1))
    del junk


def test_io_buffer_prefix_holds_results_and_csr():
    """env.io lays out the step results, the CSR offsets and the CSR values
    in that order: one host copy of io_prefix_bytes(total) reads them all."""
    env = JunqiEnvB200(37, pool=tables.build_setup_pool(8, seed=3), with_obs=False)
    env.reset(seed=2)
    for t in range(1, 6):
        env.ply(env.sample_uniform(2, t), seed=2, ply=t)
    off, val = env.csr()
    tot = int(off[-1].item())
    host = env.io[: env.io_prefix_bytes(tot)].cpu().numpy()
    base = env.io.data_ptr()
    for k, v in env.out.items():
        o = v.data_ptr() - base
        assert o % 16 == 0
        got = host[o:o + v.numel() * v.element_size()].view(v.cpu().numpy().dtype)
        assert np.array_equal(got, v.cpu().numpy()), k
    o = off.data_ptr() - base
    assert np.array_equal(host[o:o + 4 * (env.n + 1)].view(np.int32), off.cpu().numpy())
    assert np.array_equal(host[env.values_byte_offset:].view(np.int32), val[:tot].cpu().numpy())
