"""GPU parity: the CUDA path through the C ABI against the reference.

1. The reference golden trajectories (junqi_core output recorded in
   tests/golden; four stepped by BatchedGameState, three by GameState) replayed through jq_step / jq_legal / jq_csr / jq_observe:
   every legal CSR, canonical mask, MoveResult, Zobrist, combat-memory
   digest, observation digest and the final SoA state must match bit for bit.
2. Long seeded rollouts through the fused ply kernel with auto-reset from a
   setup pool, checked against the CPU oracle after every ply (state,
   MoveResult, CSR, masks, observations), in all three show modes and under
   both rule sets.
All comparisons are exact (integer / byte work, float32 values compared by
bit pattern).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N
from junqi_b200 import tables
from junqi_b200.env import BRIGHT, DARK, HALF_DARK, JunqiEnvB200
from oracle import oracle as O
from tests import _golden as G

pytestmark = pytest.mark.gpu


class CudaDriver:
    def load(self, init, show_mode, rules):
        n = init["turn"].shape[0]
        self.env = JunqiEnvB200(n, show_mode=show_mode, pool_size=4, obs_seats=4, rules=rules)
        self.env.load_state(init)
        self.ver, self.obs_ver, self.obs_cache = 0, -1, None

    def legal(self):
        self.env.legal(with_mask=True)
        off, val = self.env.csr()
        off = off.cpu().numpy()
        return off, val[: int(off[-1])].cpu().numpy()

    def masks(self):
        return self.env.mask.cpu().numpy().astype(bool)

    def step(self, actions):
        out = self.env.step(torch.from_numpy(np.ascontiguousarray(actions, np.int32)).cuda())
        self.ver += 1
        return {k: v.cpu().numpy() for k, v in out.items()}

    def state(self):
        return self.env.state()

    def obs(self, e, s):
        if self.obs_ver != self.ver:
            sp, gl = self.env.observe(seats_per_env=4)
            self.obs_cache = (sp.cpu().numpy(), gl.cpu().numpy())
            self.obs_ver = self.ver
        sp, gl = self.obs_cache
        return sp[e * 4 + s], gl[e * 4 + s]


@pytest.mark.parametrize("name", G.TRAJECTORIES)
def test_cuda_replays_reference_trajectory(name):
    """Every recorded digest, and after every ply every field the
    observation reads against the oracle stepped in lockstep."""
    from tests.test_oracle_golden import OracleDriver
    fx = G.load(name)
    assert G.replay(fx, CudaDriver(), shadow=OracleDriver()) == fx["actions"].shape[0]


# ---------------------------------------------------------------------------
# Rollouts against the oracle
# ---------------------------------------------------------------------------
STATE_CHECK = G.STATE_KEYS + ["hist_src", "hist_dst", "hist_count", "bel_code", "remaining", "rem_tracked"]


def _compare_state(env, orc, t):
    g = env.state()
    for k in STATE_CHECK:
        a, b = np.asarray(g[k]), np.asarray(orc.a[k])
        if not np.array_equal(a.reshape(b.shape).astype(b.dtype), b):
            bad = np.nonzero((a.reshape(b.shape) != b).reshape(b.shape[0], -1).any(1))[0]
            raise AssertionError(f"ply {t}: state field {k} differs in envs {bad[:8]}")


def _compare_legal(env, orc, t, masks):
    off, val = env.csr()
    off = off.cpu().numpy()
    val = val[: int(off[-1])].cpu().numpy()
    o_off, o_val = orc.legal()
    assert np.array_equal(off, o_off), f"ply {t}: CSR offsets differ"
    assert np.array_equal(val, o_val), f"ply {t}: CSR values differ"
    if masks:
        m = env.mask.cpu().numpy().astype(bool)
        for e in range(orc.n):
            exp = orc.canonical_mask(o_val[o_off[e]:o_off[e + 1]], int(orc["turn"][e]))
            assert np.array_equal(m[e], exp), f"ply {t}: canonical mask differs in env {e}"


def _compare_obs(env, orc, t, seats):
    if seats == 1:
        sp, gl = env.observe(seats_per_env=1)
        osp, ogl = orc.obs()
    else:
        sp, gl = env.observe(seats_per_env=4)
        obs = [orc.obs(np.full(orc.n, s, np.int8)) for s in range(4)]
        osp = np.stack([o[0] for o in obs], 1).reshape(-1, 317, 17, 17)
        ogl = np.stack([o[1] for o in obs], 1).reshape(-1, 28)
    sp = sp.cpu().numpy()
    gl = gl.cpu().numpy()
    if not np.array_equal(sp.view(np.uint32), osp.view(np.uint32)):
        u, c = np.nonzero((sp != osp).reshape(sp.shape[0], 317, -1).any(2))
        raise AssertionError(f"ply {t}: observation differs (unit, channel) {list(zip(u[:6], c[:6]))}")
    assert np.array_equal(gl.view(np.uint32), ogl.view(np.uint32)), f"ply {t}: global features differ"


@pytest.mark.parametrize("mode,n,plies,policy,rules", [
    (HALF_DARK, 256, 400, "uniform", N.RULES_BATCHED),
    (DARK, 128, 300, "softmax", N.RULES_BATCHED),
    (BRIGHT, 128, 300, "uniform", N.RULES_BATCHED),
    (HALF_DARK, 256, 600, "softmax", N.RULES_GAMESTATE),
    (DARK, 128, 500, "uniform", N.RULES_GAMESTATE),
])
def test_rollout_with_autoreset_matches_oracle(mode, n, plies, policy, rules):
    pool = tables.build_setup_pool(257, seed=5)
    L = N.lib()
    env = JunqiEnvB200(n, show_mode=mode, pool=pool, obs_seats=1, rules=rules)
    orc = O.OracleBatch(n, mode, rules=rules)
    seed = 1234 + mode + 17 * rules
    env.reset(seed=seed, ply=0, all_envs=True)
    for e in range(n):
        orc.reset_env(e, pool[L.jq_pool_index(seed, 0, e, pool.shape[0])])
    _compare_state(env, orc, 0)
    _compare_legal(env, orc, 0, masks=True)
    _compare_obs(env, orc, 0, seats=1)
    terminations = 0
    for t in range(1, plies + 1):
        acts = env.sample_uniform(seed, t) if policy == "uniform" else env.sample_softmax(seed, t)
        acts_np = acts.cpu().numpy().copy()
        out = env.ply(acts, seed=seed, ply=t, autoreset=True)
        r = orc.step(acts_np)
        for k in ("valid", "event", "terminated", "winner", "draw", "flag_captured", "reward"):
            got = out[k].cpu().numpy()
            assert np.array_equal(got.astype(r[k].dtype), r[k]), f"ply {t}: MoveResult.{k} differs"
        for e in np.nonzero(r["terminated"])[0]:
            orc.reset_env(int(e), pool[L.jq_pool_index(seed, t, int(e), pool.shape[0])])
            terminations += 1
        _compare_state(env, orc, t)
        _compare_legal(env, orc, t, masks=(t % 10 == 0))
        if t % 50 == 0:
            _compare_obs(env, orc, t, seats=1)
    _compare_obs(env, orc, plies, seats=4)
    assert terminations >= 0


def test_episode_stats_count_terminations():
    pool = tables.build_setup_pool(64, seed=9)
    env = JunqiEnvB200(64, pool=pool, with_obs=False)
    env.reset(seed=3)
    ends = applied = 0
    for t in range(1, 1501):
        env.ply(env.sample_uniform(3, t), seed=3, ply=t)
        ends += int(env.out["terminated"].sum().item())
        applied += int(env.out["valid"].sum().item())
    s = env.stats.cpu().numpy()
    assert s[3] == ends
    assert s[0] + s[1] + s[2] == s[3]
    assert s[5] == applied


def test_step_canonical_equals_world_step():
    pool = tables.build_setup_pool(32, seed=1)
    a = JunqiEnvB200(64, pool=pool, with_obs=False)
    b = JunqiEnvB200(64, pool=pool, with_obs=False)
    a.reset(seed=11)
    b.reset(seed=11)
    for t in range(1, 60):
        can = a.compact_actions
        world = a.sample_softmax(11, t).clone()
        a.step(world)
        b.out["world_action"].zero_()
        N.check(N.lib().jq_step_canonical(ctypes.byref(b.batch.struct), can.data_ptr(), None, b.show_mode,
                                          ctypes.byref(b._out), torch.cuda.current_stream().cuda_stream),
                "jq_step_canonical")
        assert torch.equal(b.out["world_action"], world)
        a.legal()
        b.legal()
        assert torch.equal(a.batch["zobrist"], b.batch["zobrist"])


def test_sampled_actions_are_legal():
    env = JunqiEnvB200(128, pool=tables.build_setup_pool(16, seed=2), with_obs=False)
    env.reset(seed=5)
    for t in range(1, 40):
        for sampler in (env.sample_uniform, env.sample_softmax):
            acts = sampler(5, t).cpu().numpy()
            cnt = env.counts.cpu().numpy()
            ids = env.ids.cpu().numpy()
            for e in range(env.n):
                if cnt[e] == 0:
                    assert acts[e] == -1
                else:
                    assert acts[e] in ids[e, : cnt[e]]
        env.ply(env.sample_uniform(5, t), seed=5, ply=t)


def test_status_codes_surface_as_errors():
    env = JunqiEnvB200(8, pool=tables.build_setup_pool(4, seed=2), with_obs=False)
    L = N.lib()
    sp = torch.empty((8, 317, 17, 17), device="cuda")
    gl = torch.empty((8, 28), device="cuda")
    st = L.jq_observe(ctypes.byref(env.batch.struct), None, 1, 7, sp.data_ptr(), gl.data_ptr(), None)
    assert st == 1 and b"show_mode" in L.jq_last_error()
    st = L.jq_observe(ctypes.byref(env.batch.struct), None, 3, 2, sp.data_ptr(), gl.data_ptr(), None)
    assert st == 1
    with pytest.raises(RuntimeError, match="JQ_ERR_ARG"):
        N.check(L.jq_legal(ctypes.byref(env.batch.struct), None, None, None, 0, None, None), "jq_legal")


@pytest.mark.parametrize("late", [False, True])
def test_slot_mask_matches_oracle(late):
    """jq_legal_slots (per-piece 80-slot mask) against the oracle restatement,
    including late-game positions with engineers on the railway."""
    from junqi_b200 import workloads
    n, seed = 96, 21 + int(late)
    pool = tables.build_setup_pool(64, seed=seed)
    env = JunqiEnvB200(n, pool=pool, with_obs=False, rules=N.RULES_GAMESTATE)
    if late:
        workloads.late_game_starts(env, seed)
    else:
        env.reset(seed=seed)
    for t in range(1, 121):
        if t % 10 == 1:
            orc = O.OracleBatch(n, env.show_mode, rules=N.RULES_GAMESTATE)
            O.load_state(orc, env.state(), init_beliefs=False)
            for seats in (None, np.full(n, t % 4, np.int8)):
                got = env.legal_slots(None if seats is None else torch.from_numpy(seats)).cpu().numpy().astype(bool)
                exp, _ = orc.slot_mask(seats)
                if not np.array_equal(got, exp):
                    e, p, s = np.argwhere(got != exp)[0]
                    raise AssertionError(f"ply {t}: slot mask differs at env {e} pid {p} slot {s}")
        env.ply(env.sample_uniform(seed, t), seed=seed, ply=t)


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_observe_with_caller_beliefs_matches_oracle(mode):
    """jq_observe_beliefs: per-cell float beliefs (zeros, one-hots, random,
    negatives and NaNs, which the reference GPU encoder writes as 0) against
    the oracle, mid-game, for the acting seat and for all four seats."""
    n = 96
    env = JunqiEnvB200(n, show_mode=mode, pool=tables.build_setup_pool(64, seed=9), rules=N.RULES_GAMESTATE)
    env.reset(seed=4)
    for t in range(1, 70):
        env.ply(env.sample_uniform(4, t), seed=4, ply=t)
    rng = np.random.default_rng(mode)
    bel = rng.random((n, 4, 12, 289)).astype(np.float32)
    bel[bel < 0.25] = 0.0
    bel[rng.random(bel.shape) < 0.02] = -0.5
    bel[rng.random(bel.shape) < 0.01] = np.nan
    bel[:, :, 3] = 1.0
    orc = O.OracleBatch(n, mode, rules=1)
    O.load_state(orc, env.state(), init_beliefs=False)
    dbel = torch.from_numpy(bel).cuda()
    sp, gl = env.observe(None, seats_per_env=1, beliefs=dbel)
    o_sp, o_gl = orc.obs_beliefs(bel)
    assert np.array_equal(sp.cpu().numpy().view(np.int32), o_sp.view(np.int32))
    # a NaN belief makes its enemy sum NaN; NaN payloads differ between CPU and GPU adds
    assert np.array_equal(gl.cpu().numpy(), o_gl, equal_nan=True)
    sp4, gl4 = env.observe(None, seats_per_env=4, beliefs=dbel)
    sp4, gl4 = sp4.cpu().numpy().reshape(n, 4, 317, 17, 17), gl4.cpu().numpy().reshape(n, 4, 28)
    for s in range(4):
        o_sp, o_gl = orc.obs_beliefs(bel, np.full(n, s, np.int8))
        assert np.array_equal(sp4[:, s], o_sp) and np.array_equal(gl4[:, s], o_gl, equal_nan=True), s
    # the env's own beliefs are untouched
    sp0, gl0 = env.observe(None, seats_per_env=1)
    o_sp0, o_gl0 = orc.obs()
    assert np.array_equal(sp0.cpu().numpy(), o_sp0) and np.array_equal(gl0.cpu().numpy(), o_gl0)
