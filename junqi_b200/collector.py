"""Device rollout collector, with the whole rollout captured as one CUDA graph.

The reference's ``collect_rollout_gpu_v2`` (junqi_rl/training/gpu_collector.py:
673-1003) runs, per ply and with no host round trip: the acting seat's
observation, its canonical legal mask, the policy, the step, the reward
(with shaping), the belief update and the reset of finished games; it
compiles the policy with ``torch.compile(mode="reduce-overhead")`` so only
the policy runs as a CUDA graph.  Here the env side is a handful of
library launches on the same stream as the policy, so the whole T-ply
rollout -- env kernels, policy, sampling, buffer writes, history records
and the final value estimate -- is captured once and replayed with one
launch per rollout.

Per ply t, for every env:

* seat = the env's turn (the reference clamps terminated envs to seat 0;
  with auto-reset inside ``jq_ply`` no env is terminated at this point);
* spatial, global = ``jq_observe`` of that seat; mask = the canonical
  legal mask ``jq_ply`` left for that seat;
* ``policy(spatial, global, mask) -> (canonical action, log_prob, value)``
  -- the signature of the reference's ``policy.act`` (``mask`` is bool);
* with ``random_opponent`` seats 1 and 3 play a uniform legal action
  instead (gpu_collector.py:757-770);
* the pre-action state is recorded in the compact history
  (``buffer.snapshot_history``, gpu_collector.py:830);
* ``jq_canonical_to_world`` then ``jq_ply``: step, beliefs, reward, reset
  of finished games from the pool (seed ``seed``, ply ``ply0 + t + 1``),
  legal mask of the next turn;
* reward = the step reward, plus -0.05 when the mover was killed and
  -0.02 for a mutual kill on plies that did not end the game
  (gpu_collector.py:860-874); done = the ply ended the game.

After T plies the policy's value of the final positions is kept as
``last_values`` (0 for terminated envs, gpu_collector.py:980-1000).

A graph bakes its launch arguments: each replay resets finished games with
the same (seed, ply) draws as the first one.  Successive rollouts still
differ because each continues from the positions the previous one ended
in, and a policy that samples with torch's generator draws new noise on
every replay (torch registers its generator with the captured graph).
Host callbacks (``on_termination`` / ``on_reset``) are not supported; the
per-ply ``dones`` carry the same information.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable

import torch

from . import _native as N
from .env import JunqiEnvB200, _stream_ptr
from .history import RolloutHistory

Policy = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], tuple[torch.Tensor, torch.Tensor, torch.Tensor]]

EVENT_MUTUAL = 3   # both pieces removed (rules.py Event)
EVENT_KILLED = 4   # the moving piece was removed


@dataclass
class Rollout:
    """(T, N) per-ply tensors of one rollout, plus the final values.  Views
    of the collector's buffers: the next ``collect`` overwrites them."""
    seats: torch.Tensor        # int8, acting seat
    actions: torch.Tensor      # int32, compact canonical action (cs*129+cd)
    log_probs: torch.Tensor    # float32
    values: torch.Tensor       # float32
    rewards: torch.Tensor      # float32, with shaping
    dones: torch.Tensor        # bool, the ply ended the game
    last_values: torch.Tensor  # (N,) float32
    history: RolloutHistory | None


class RolloutCollector:
    def __init__(self, env: JunqiEnvB200, policy: Policy, steps: int, *, seed: int = 0, ply0: int = 0,
                 reward_shaping: bool = True, random_opponent: bool = False, history: bool = True,
                 graph: bool = True):
        if env.mask is None:
            raise ValueError("the collector needs the env's canonical legal mask (with_mask=True)")
        self.env, self.policy, self.T = env, policy, int(steps)
        self.seed, self.ply0 = int(seed), int(ply0)
        self.reward_shaping, self.random_opponent = bool(reward_shaping), bool(random_opponent)
        n, T, dev = env.n, self.T, env.device
        self.seats = torch.zeros((T, n), dtype=torch.int8, device=dev)
        self.actions = torch.zeros((T, n), dtype=torch.int32, device=dev)
        self.log_probs = torch.zeros((T, n), dtype=torch.float32, device=dev)
        self.values = torch.zeros((T, n), dtype=torch.float32, device=dev)
        self.rewards = torch.zeros((T, n), dtype=torch.float32, device=dev)
        self.dones = torch.zeros((T, n), dtype=torch.bool, device=dev)
        self.last_values = torch.zeros(n, dtype=torch.float32, device=dev)
        self.world = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.history = RolloutHistory(T, n, dev.index) if history else None
        env.observe(None, seats_per_env=1)  # allocate the observation buffers before any capture
        self.graph_mode = bool(graph)
        self._graph: torch.cuda.CUDAGraph | None = None

    # ------------------------------------------------------------------
    def _act(self):
        env = self.env
        sp, gl = env.observe(None, seats_per_env=1)
        return self.policy(sp, gl, env.mask.view(torch.bool))

    def _ply(self, t: int, ply0: int) -> None:
        env = self.env
        seats = self.seats[t]
        seats.copy_(env.batch["turn"])
        a, lp, v = self._act()
        a = a.to(torch.int32)
        if self.random_opponent:
            # Gumbel-max over the legal set with flat logits: a uniform legal action.
            g = -torch.log(-torch.log(torch.rand(env.mask.shape, device=env.device).clamp_(1e-10, 1.0)))
            rnd = torch.where(env.mask.view(torch.bool), g, float("-inf")).argmax(dim=1).to(torch.int32)
            a = torch.where((seats == 1) | (seats == 3), rnd, a)
        self.actions[t].copy_(a)
        self.log_probs[t].copy_(lp.reshape(-1))
        self.values[t].copy_(v.reshape(-1))
        if self.history is not None:
            self.history.snapshot(env.batch, t)
        N.check(N.lib().jq_canonical_to_world(ctypes.byref(env.batch.struct), self.actions[t].data_ptr(), None,
                                              self.world.data_ptr(), _stream_ptr()), "jq_canonical_to_world")
        out = env.ply(self.world, seed=self.seed, ply=ply0 + t + 1, autoreset=True)
        term = out["terminated"] != 0
        r = out["reward"]
        if self.reward_shaping:
            live = ~term
            ev = out["event"]
            r = r - 0.05 * (live & (ev == EVENT_KILLED)).float() - 0.02 * (live & (ev == EVENT_MUTUAL)).float()
        self.rewards[t].copy_(r)
        self.dones[t].copy_(term)

    def _final(self) -> None:
        _, _, v = self._act()
        self.last_values.copy_(v.reshape(-1) * (self.env.batch["terminated"] == 0).float())

    def _rollout(self, ply0: int) -> None:
        for t in range(self.T):
            self._ply(t, ply0)
        self._final()

    def _capture(self) -> None:
        side = torch.cuda.Stream(device=self.env.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():  # warm the policy's libraries up outside the capture
            for _ in range(3):
                self._act()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(g):
            self._rollout(self.ply0)
        self._graph = g

    def collect(self) -> Rollout:
        """Run T plies from the env's current positions and return them."""
        if self.graph_mode:
            if self._graph is None:
                self._capture()
            self._graph.replay()
        else:
            with torch.no_grad():
                self._rollout(self.ply0)
            self.ply0 += self.T
        return Rollout(self.seats, self.actions, self.log_probs, self.values, self.rewards, self.dones,
                       self.last_values, self.history)
