"""The device rollout collector (gpu_collector.py:673-1003 semantics).

* The rollout captured as one CUDA graph and replayed equals the same
  rollout run eagerly, tensor for tensor and byte for byte in the history
  and the final env state -- on the first rollout and on a second replay
  that continues from where the first ended.
* Every ply applies a move in every env (the policy only picks legal
  actions through the mask), done plies carry the terminal rewards and
  the shaping penalties land on the plies the reference shapes.
* The compact history records the pre-action state of the acting seat:
  rebuilding (t, env) gives exactly the observation and mask the policy saw.
* With a random opponent (torch generator inside the graph) seats 1 and 3
  still only play legal moves.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N
from junqi_b200 import tables
from junqi_b200.batch import FIELDS
from junqi_b200.collector import RolloutCollector
from junqi_b200.env import HALF_DARK, JunqiEnvB200
from junqi_b200.workloads import late_game_starts

pytestmark = pytest.mark.gpu


class HashPolicy:
    """Deterministic stand-in for a policy network: per-env pseudo-random
    logits keyed on the observation, masked argmax."""

    def __init__(self):
        self.idx = torch.arange(16641, device="cuda", dtype=torch.float32)
        self.seen = {}
        self.calls = 0
        self.keep = set()

    def __call__(self, sp, gl, mask):
        key = (sp[:, :27].sum(dim=(1, 2, 3)) * 0.37 + gl.sum(1) * 0.11)[:, None]
        logits = torch.frac(torch.sin(self.idx[None, :] * 0.0127 + key) * 4375.5453)
        logits = logits.masked_fill(~mask, float("-inf"))
        a = logits.argmax(1)
        lp = torch.log_softmax(logits, 1).gather(1, a[:, None]).squeeze(1)
        if self.calls in self.keep:
            self.seen[self.calls] = (sp.clone(), gl.clone(), mask.clone())
        self.calls += 1
        return a, lp, torch.tanh(key.squeeze(1) * 0.01)


def _env(n=128, seed=5, late=False):
    env = JunqiEnvB200(n, show_mode=HALF_DARK, pool=tables.build_setup_pool(48, seed=2), rules=N.RULES_GAMESTATE)
    env.reset(seed=seed)
    if late:  # thinned boards, so that games end inside a short rollout
        late_game_starts(env, seed)
    return env


def _same_state(a: JunqiEnvB200, b: JunqiEnvB200):
    for name, *_ in FIELDS:
        assert torch.equal(a.batch[name], b.batch[name]), name


def test_graph_replay_equals_eager_rollout():
    T = 48
    ea, eb = _env(late=True), _env(late=True)
    ca = RolloutCollector(ea, HashPolicy(), T, seed=9, graph=False)
    cb = RolloutCollector(eb, HashPolicy(), T, seed=9, graph=True)
    for rnd in range(2):
        ca.ply0 = 0  # the graph replays its first rollout's (seed, ply) draws
        ra, rb = ca.collect(), cb.collect()
        for k in ("seats", "actions", "log_probs", "values", "rewards", "dones", "last_values"):
            assert torch.equal(getattr(ra, k), getattr(rb, k)), (rnd, k)
        assert torch.equal(ra.history.buf, rb.history.buf), rnd
        _same_state(ea, eb)
        assert torch.equal(ea.stats, eb.stats)


def test_every_ply_applies_and_rewards_follow_the_reference():
    T, n = 64, 128
    env = _env(n, seed=8, late=True)
    col = RolloutCollector(env, HashPolicy(), T, seed=3, graph=True)
    done_total, shaped = 0, 0
    for _ in range(24):
        s0 = env.stats.clone()
        r = col.collect()
        ds = (env.stats - s0).cpu().numpy()
        assert ds[5] == T * n, "a policy action was not applied"
        rew, done = r.rewards.cpu().numpy(), r.dones.cpu().numpy()
        assert int(done.sum()) == ds[3]
        assert set(np.unique(rew[done]).tolist()) <= {-1.0, 0.0, 1.0}
        assert np.isin(rew[~done], np.float32([0.0, -0.05, -0.02])).all()
        done_total += int(done.sum())
        shaped += int((rew[~done] != 0).sum())
        if done_total >= 10 and shaped:
            break
    assert done_total >= 10 and shaped > 0, (done_total, shaped)


def test_history_holds_what_the_policy_saw():
    T, n = 24, 64
    env = _env(n, seed=4)
    pol = HashPolicy()
    pol.keep = {0, 7, 23}
    col = RolloutCollector(env, pol, T, seed=1, graph=False)
    r = col.collect()
    rng = np.random.default_rng(0)
    for t in sorted(pol.keep):
        envs = rng.choice(n, 16, replace=False)
        out = r.history.reconstruct(t * n + envs)
        sp, gl, mask = pol.seen[t]
        for j, e in enumerate(envs):
            assert torch.equal(out["spatial"][j], sp[e]) and torch.equal(out["global"][j], gl[e]), (t, e)
            assert torch.equal(out["mask"][j].view(torch.bool), mask[e]), (t, e)
            assert int(out["observers"][j]) == int(r.seats[t, e])


def test_random_opponent_in_the_graph_plays_legal_moves():
    T, n = 40, 96
    env = _env(n, seed=6)
    s0 = env.stats.clone()
    col = RolloutCollector(env, HashPolicy(), T, seed=2, random_opponent=True, history=False, graph=True)
    a1 = col.collect().actions.clone()
    a2 = col.collect().actions
    assert int((env.stats - s0)[5]) == 2 * T * n
    assert not torch.equal(a1, a2)
