"""Parity at the benchmark's full sizes: sampled envs plus whole-batch properties.

The oracle cannot replay 65,536 envs in seconds, so at the benchmark's full
shapes every check is one of:

* sampled parity -- at checkpoint plies a random sample of envs is copied to
  the CPU oracle before the ply (state, beliefs, history) and stepped there
  with the same actions; MoveResult, the whole post-ply state (auto-reset
  included), the legal CSR rows, the canonical masks and the observations of
  the sampled envs must equal the device's bit for bit;
* size-independent properties over every env -- the incremental Zobrist
  hash equals a from-scratch recompute (state.py:1761); CSR rows are
  ascending, duplicate-free and sized like the mask rows; episode
  statistics add up.

Shapes (the benchmark's configurations, GameState rules, HALF_DARK):

* configs[1], the headline: 4,096 envs, acting-seat observation, uniform
  policy, pool of 10,000, 1,000 plies;
* 65,536 envs, observations of all 4 seats, masked softmax;
* 32,768 envs, 512 plies, pool of 8,192, masked softmax;
* 32,768 late-game starts (``workloads.late_game_starts``),
  2,000 uniform plies.
At every checkpoint the sampled envs' observations of their acting seat
(of all four seats at configs[2]'s last checkpoint) are compared too.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N
from junqi_b200 import tables
from junqi_b200.env import HALF_DARK, JunqiEnvB200
from oracle import oracle as O
from tests import _golden as G

pytestmark = pytest.mark.gpu

SAMPLE = 48
BELIEF_KEYS = ["hist_src", "hist_dst", "hist_count", "bel_code", "remaining", "rem_tracked"]


def _oracle_from(env: JunqiEnvB200, idx: np.ndarray) -> O.OracleBatch:
    orc = O.OracleBatch(len(idx), env.show_mode, rules=env.batch.rules)
    O.load_state(orc, env.batch.to_host(envs=idx), init_beliefs=False)
    return orc


def _check_state(env, orc, idx, t):
    got = env.batch.to_host(envs=idx)
    for k in G.STATE_KEYS + BELIEF_KEYS:
        a, b = np.asarray(got[k]), np.asarray(orc.a[k])
        if not np.array_equal(a.reshape(b.shape).astype(b.dtype), b):
            bad = np.nonzero((a.reshape(b.shape) != b).reshape(b.shape[0], -1).any(1))[0]
            raise AssertionError(f"ply {t}: {k} differs in sampled envs {idx[bad[:6]]}")


def _check_legal(env, orc, idx, t):
    off, val = env.csr()
    off = off.cpu().numpy()
    o_off, o_val = orc.legal()
    for i, e in enumerate(idx):
        row = val[off[e]:off[e + 1]].cpu().numpy()
        assert np.array_equal(row, o_val[o_off[i]:o_off[i + 1]]), f"ply {t}: CSR row of env {e} differs"
        m = env.mask[e].cpu().numpy().astype(bool)
        assert np.array_equal(m, orc.canonical_mask(row, int(orc["turn"][i]))), f"ply {t}: mask of env {e} differs"


def _check_properties(env, t):
    st = env.state()
    bad = np.nonzero(O.zobrist_recompute(st, env.show_mode) != st["zobrist"])[0]
    assert bad.size == 0, f"ply {t}: incremental Zobrist differs from a recompute in envs {bad[:8]}"
    off, val = env.csr()
    off = off.cpu()
    counts = env.counts.cpu()
    assert torch.equal(off[1:] - off[:-1], counts), f"ply {t}: CSR offsets do not match counts"
    n_tot = int(off[-1])
    v = val[:n_tot].cpu().numpy().astype(np.int64)
    row = np.repeat(np.arange(env.n), counts.numpy())
    key = row * (289 * 289) + v
    assert np.all(np.diff(key) > 0), f"ply {t}: CSR rows are not strictly ascending"
    if env.mask is not None:
        pop = env.mask.sum(dim=1, dtype=torch.int32).cpu()
        assert torch.equal(pop, counts), f"ply {t}: mask popcount differs from the legal count"
    s = env.stats.cpu().numpy()
    assert s[0] + s[1] + s[2] == s[3]


def _free_bytes() -> int:
    free, _ = torch.cuda.mem_get_info()
    return free


@pytest.mark.parametrize("name,envs,seats,pool_n,plies,policy,late,checks", [
    ("configs[1]", 4096, 1, 10_000, 1000, "uniform", False, (1, 250, 500, 750, 1000)),
    ("configs[2]", 65536, 4, 10_000, 40, "softmax", False, (1, 20, 40)),
    ("configs[3]", 32768, 1, 8192, 512, "softmax", False, (1, 256, 511)),
    ("configs[4]", 32768, 1, 10_000, 2000, "uniform", True, (1, 700, 1400, 2000)),
])
def test_full_size_rollout_sampled_parity(name, envs, seats, pool_n, plies, policy, late, checks):
    seed = 900 + envs // 4096 + 7 * late
    pool = tables.build_setup_pool(pool_n, seed=seed)
    env = JunqiEnvB200(envs, show_mode=HALF_DARK, pool=pool, obs_seats=seats, with_obs=seats == 1,
                       rules=N.RULES_GAMESTATE)
    L = N.lib()
    rng = np.random.default_rng(seed)
    if late:
        from junqi_b200.workloads import late_game_starts
        late_game_starts(env, seed)
    else:
        env.reset(seed=seed)
    sampler = env.sample_uniform if policy == "uniform" else env.sample_softmax
    for t in range(1, plies + 1):
        acts = sampler(seed, t)
        if t not in checks:
            env.ply(acts, seed=seed, ply=t)
            continue
        idx = np.sort(rng.choice(envs, SAMPLE, replace=False))
        orc = _oracle_from(env, idx)
        acts_s = acts.cpu().numpy()[idx].copy()
        out = env.ply(acts, seed=seed, ply=t)
        r = orc.step(acts_s)
        for k in ("valid", "event", "terminated", "winner", "draw", "flag_captured", "reward"):
            got = out[k].cpu().numpy()[idx]
            assert np.array_equal(got.astype(r[k].dtype), r[k]), f"{name} ply {t}: MoveResult.{k} differs"
        for i in np.nonzero(r["terminated"])[0]:
            orc.reset_env(int(i), pool[L.jq_pool_index(seed, t, int(idx[i]), pool.shape[0])])
        _check_state(env, orc, idx, t)
        _check_legal(env, orc, idx, t)
        _check_properties(env, t)
        if seats == 1:  # the acting seat's observation, as the benchmark's ply loop builds it
            sp, gl = env.observe()
            osp, ogl = orc.obs()
            got_sp = sp[torch.from_numpy(idx).to(sp.device)].cpu().numpy()
            got_gl = gl[torch.from_numpy(idx).to(gl.device)].cpu().numpy()
            bad = [int(idx[i]) for i in range(len(idx))
                   if not np.array_equal(got_sp[i].view(np.uint32), osp[i].view(np.uint32))
                   or not np.array_equal(got_gl[i].view(np.uint32), ogl[i].view(np.uint32))]
            assert not bad, f"{name} ply {t}: acting-seat observation differs in envs {bad[:6]}"
        if seats == 4 and t == checks[-1]:
            need = envs * 4 * (317 * 289 * 4 + 28 * 4)
            if _free_bytes() < need + (4 << 30):
                pytest.skip(f"{need / 2**30:.0f} GiB of observations do not fit next to the batch")
            sp, gl = env.observe(seats_per_env=4)  # the full-size launch: unit index * 91,613 > 2^31
            for i, e in enumerate(idx[:12]):
                for s in range(4):
                    osp, ogl = orc.obs_one(i, s)
                    u = int(e) * 4 + s
                    assert np.array_equal(sp[u].cpu().numpy().view(np.uint32), osp.view(np.uint32)), \
                        f"{name}: observation of env {e} seat {s} differs"
                    assert np.array_equal(gl[u].cpu().numpy(), ogl)
            del sp, gl
            env.spatial = env.global_ = None
            torch.cuda.empty_cache()
    s = env.stats.cpu().numpy()
    if plies >= 1000:  # long rollouts finish games and reset them from the pool
        assert s[3] > 0, f"{name}: no episode finished in {plies} plies"
