"""Game records of device rollouts, and replay validation on the device.

A :class:`Trajectory` is one game in junqi_core's replay format
(junqi_core/replay.py:1-30, 83-225): the four 30-slot lineups as piece-type
names, an ``int16 (T, 5)`` action log of ``(seat, src_x, src_y, dst_x,
dst_y)`` rows, and the Zobrist hash of the final position as a determinism
self-check.  Files written by :meth:`Trajectory.save` load with
``junqi_core.replay.Trajectory.load`` and the reverse.

:class:`ReplayRecorder` records every env of a :class:`JunqiEnvB200`
rollout on the device (five small device copies per ply) and cuts the log
into one trajectory per game on the host.  :func:`validate_on_device`
replays many trajectories at once -- one env per game, one ``jq_step`` per
ply -- and checks each final hash, which is ``Trajectory.validate``
(replay.py:243-260) for a whole batch of games in one pass.

Replays follow ``GameState.step_inplace``, so recorders and validation use
the GameState rule set (``RULES_GAMESTATE``).
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import _native as N
from .env import JunqiEnvB200, _stream_ptr

RULES_VERSION = "1.1.0"   # junqi_core/rules.py:34
STATE_VERSION = "2.0"     # junqi_core/replay.py:118
# PieceType member names by value (junqi_core/rules.py:49-70).
PIECE_NAMES = ("NONE", "DARK", "JUNQI", "DILEI", "ZHADAN", "SILING", "JUNZH", "SHIZH", "LVZH", "TUANZH",
               "YINGZH", "LIANZH", "PAIZH", "GONGB")
_NAME_TO_TYPE = {n: i for i, n in enumerate(PIECE_NAMES)}

_on_board_cache: np.ndarray | None = None


def _on_board() -> np.ndarray:
    """(289,) bool: playable cells, from the library's own board tables."""
    global _on_board_cache
    if _on_board_cache is None:
        bufs = [np.zeros(s, np.int32) for s in (289, 289, 289, (289, 4), (289, 4, 12), (289, 2, 11), 129, 289)]
        N.check(N.lib().jq_topology_dump(*[b.ctypes.data for b in bufs]), "jq_topology_dump")
        _on_board_cache = bufs[0].astype(bool)
    return _on_board_cache


@dataclass
class Trajectory:
    """One recorded game (junqi_core/replay.py:83-160).

    ``setups`` is ``(4, 30)`` int8 piece types (camp slots 0), ``actions``
    ``(T, 5)`` int16 rows ``(seat, src_x, src_y, dst_x, dst_y)``."""

    setups: np.ndarray
    actions: np.ndarray
    rng_seed: int
    final_state_hash: int
    first_seat: int = 0
    show_mode: int = 2
    rules_version: str = RULES_VERSION
    state_version: str = STATE_VERSION
    meta: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        # The same file-boundary checks as replay.py:126-156.
        self.setups = np.asarray(self.setups, dtype=np.int8).reshape(4, 30)
        self.actions = np.asarray(self.actions, dtype=np.int16)
        if self.actions.ndim != 2 or self.actions.shape[1] != 5:
            raise ValueError(f"actions must have shape (T, 5), got {self.actions.shape}")
        if self.actions.size:
            rows = self.actions.astype(np.int64)
            if np.any((rows[:, 0] < 0) | (rows[:, 0] > 3)):
                raise ValueError("action seat must be in [0, 3]")
            if np.any((rows[:, 1:] < 0) | (rows[:, 1:] >= 17)):
                raise ValueError("action coordinates must be in [0, 16]")
            if np.any((rows[:, 1] == rows[:, 3]) & (rows[:, 2] == rows[:, 4])):
                raise ValueError("action src and dst must differ")
            ob = _on_board()
            if not (ob[rows[:, 2] * 17 + rows[:, 1]].all() and ob[rows[:, 4] * 17 + rows[:, 3]].all()):
                raise ValueError("action points off playable board")
        if int(self.first_seat) not in (0, 1, 2, 3):
            raise ValueError(f"invalid first_seat: {self.first_seat!r}")
        if int(self.show_mode) not in (0, 1, 2):
            raise ValueError(f"invalid show_mode: {self.show_mode!r}")
        self.first_seat, self.show_mode = int(self.first_seat), int(self.show_mode)
        self.final_state_hash = int(self.final_state_hash)

    @property
    def num_steps(self) -> int:
        return int(self.actions.shape[0])

    def world_actions(self) -> np.ndarray:
        """(T,) int32 world action ids ``src_flat * 289 + dst_flat``."""
        a = self.actions.astype(np.int32)
        return (a[:, 2] * 17 + a[:, 1]) * 289 + a[:, 4] * 17 + a[:, 3]

    def save(self, path: str | os.PathLike[str]) -> None:
        """Uncompressed .npz with the keys of replay.py:171-183."""
        p = Path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        names = np.asarray([[PIECE_NAMES[int(t)] for t in lineup] for lineup in self.setups], dtype=np.str_)
        np.savez(str(p), setups=names, action_log=self.actions.astype(np.int16),
                 rng_seed=np.int64(self.rng_seed), rules_version=np.array(self.rules_version),
                 state_version=np.array(self.state_version), final_state_hash=np.int64(self.final_state_hash),
                 first_seat=np.int8(self.first_seat), show_mode=np.int8(self.show_mode),
                 meta_json=np.array(json.dumps(self.meta, ensure_ascii=False, default=str)))

    @classmethod
    def load(cls, path: str | os.PathLike[str]) -> "Trajectory":
        """Read a file written by :meth:`save` or by junqi_core (replay.py:185-216)."""
        with np.load(str(path), allow_pickle=False) as d:
            rv = str(d["rules_version"])
            if not rv.startswith("1."):
                raise ValueError(f"incompatible replay rules_version {rv!r} (expect 1.x)")
            try:
                setups = np.array([[_NAME_TO_TYPE[str(nm)] for nm in lineup] for lineup in d["setups"].tolist()],
                                  np.int8)
            except KeyError as exc:
                raise ValueError(f"unknown piece name {exc}") from None
            meta: dict[str, Any] = {}
            if "meta_json" in d.files:
                try:
                    m = json.loads(str(d["meta_json"]))
                except (TypeError, ValueError):
                    raise ValueError("invalid replay meta_json") from None
                if isinstance(m, dict):
                    meta = m
            return cls(setups=setups, actions=np.asarray(d["action_log"], np.int16), rng_seed=int(d["rng_seed"]),
                       final_state_hash=int(d["final_state_hash"]), first_seat=int(d["first_seat"]),
                       show_mode=int(d["show_mode"]), rules_version=rv, state_version=str(d["state_version"]),
                       meta=meta)


def _rows_from_world(seats: np.ndarray, acts: np.ndarray) -> np.ndarray:
    src, dst = acts // 289, acts % 289
    return np.stack([seats, src % 17, src // 17, dst % 17, dst // 17], axis=1).astype(np.int16)


class ReplayRecorder:
    """Records the plies of every env of `env` for up to `max_plies` calls.

    Use ``reset`` once, then ``ply`` in place of ``env.ply``; ``trajectories``
    returns the games.  Games start from the pool rows the resets drew
    (``jq_pool_index``), so the recorder needs the same (seed, ply) the
    resets used, which ``reset`` and ``ply`` take as arguments."""

    def __init__(self, env: JunqiEnvB200, max_plies: int):
        if env.batch.rules != N.RULES_GAMESTATE:
            raise ValueError("replays follow GameState.step_inplace: use rules=RULES_GAMESTATE")
        self.env, self.max_plies = env, int(max_plies)
        n, dev = env.n, env.device
        self.seat = torch.empty((self.max_plies, n), dtype=torch.int8, device=dev)
        self.action = torch.empty((self.max_plies, n), dtype=torch.int32, device=dev)
        self.valid = torch.empty((self.max_plies, n), dtype=torch.uint8, device=dev)
        self.terminated = torch.empty((self.max_plies, n), dtype=torch.uint8, device=dev)
        self.zobrist = torch.empty((self.max_plies, n), dtype=torch.int64, device=dev)
        self.t = 0
        self._calls: list[tuple[int, int]] = []
        self._start: tuple[int, int] | None = None

    def reset(self, seed: int, ply: int = 0) -> None:
        self.env.reset(seed=seed, ply=ply, all_envs=True)
        self._start, self._calls, self.t = (int(seed), int(ply)), [], 0

    def ply(self, actions: torch.Tensor, seed: int, ply: int) -> dict[str, torch.Tensor]:
        if self._start is None:
            raise RuntimeError("call reset() first")
        if self.t >= self.max_plies:
            raise RuntimeError(f"recorder is full ({self.max_plies} plies)")
        t, env = self.t, self.env
        self.seat[t].copy_(env.batch["turn"])
        a = actions.to(device=env.device, dtype=torch.int32)
        self.action[t].copy_(a)
        out = env.ply(a, seed=seed, ply=ply, autoreset=True)
        self.valid[t].copy_(out["valid"])
        self.terminated[t].copy_(out["terminated"])
        self.zobrist[t].copy_(out["zobrist"])
        self._calls.append((int(seed), int(ply)))
        self.t += 1
        return out

    def trajectories(self, include_unfinished: bool = False) -> list[Trajectory]:
        """One trajectory per game, env by env in order of completion.  A game
        still running at the end of the log is included when asked, with the
        hash of its last recorded position."""
        T, n, env = self.t, self.env.n, self.env
        if self._start is None or T == 0:
            return []
        h = {k: getattr(self, k)[:T].cpu().numpy() for k in ("seat", "action", "valid", "terminated", "zobrist")}
        pool, P = env.pool_host, env.pool_host.shape[0]
        L = N.lib()
        out: list[Trajectory] = []
        for e in range(n):
            row = L.jq_pool_index(self._start[0], self._start[1], e, P)
            t0, start = 0, self._start
            valid = h["valid"][:, e].astype(bool)
            ends = np.flatnonzero(valid & (h["terminated"][:, e] != 0))
            for t_end in list(ends) + ([T - 1] if include_unfinished else []):
                if t_end < t0:
                    continue
                sel = np.arange(t0, t_end + 1)[valid[t0:t_end + 1]]
                if sel.size == 0:
                    break
                rows = _rows_from_world(h["seat"][sel, e].astype(np.int64), h["action"][sel, e].astype(np.int64))
                out.append(Trajectory(setups=pool[row].reshape(4, 30), actions=rows, rng_seed=-1,
                                      final_state_hash=int(h["zobrist"][sel[-1], e]), first_seat=0,
                                      show_mode=env.show_mode,
                                      meta={"env": e, "reset": list(start), "finished": bool(t_end in ends)}))
                # The game that ended at t_end was replaced by a reset inside the same ply call.
                start = self._calls[t_end]
                row = L.jq_pool_index(start[0], start[1], e, P)
                t0 = t_end + 1
        return out


def validate_on_device(trajectories: list[Trajectory], device: int = 0) -> np.ndarray:
    """Replay every trajectory on the device and return, per trajectory,
    whether each action was a legal move of the seat its row names, played
    on that seat's turn, and the final hash matches -- what
    ``Trajectory.validate`` (replay.py:243-260) establishes through
    ``GameState.step_inplace``, for a whole batch of games at once."""
    ok = np.zeros(len(trajectories), dtype=bool)
    by_mode: dict[int, list[int]] = {}
    for i, tr in enumerate(trajectories):
        by_mode.setdefault(tr.show_mode, []).append(i)
    for mode, idx in by_mode.items():
        ok[idx] = _validate_group([trajectories[i] for i in idx], mode, device)
    return ok


def _validate_group(trs: list[Trajectory], mode: int, device: int) -> np.ndarray:
    n = len(trs)
    pool = np.stack([tr.setups.reshape(120) for tr in trs]).astype(np.int8)
    env = JunqiEnvB200(n, device=device, show_mode=mode, pool=pool, with_obs=False, with_mask=False,
                       rules=N.RULES_GAMESTATE)
    dev = env.device
    env.reset_rows(torch.arange(n, dtype=torch.int32, device=dev))
    first = np.array([tr.first_seat for tr in trs], np.int8)
    if first.any():  # GameState.new_game(first_seat=...) differs only in the turn and its key
        env.batch["turn"].copy_(torch.from_numpy(first).to(dev))
        N.check(N.lib().jq_rehash(ctypes.byref(env.batch.struct), mode, _stream_ptr()), "jq_rehash")
    T = max((tr.num_steps for tr in trs), default=0)
    acts = np.full((max(T, 1), n), -1, np.int32)
    seats = np.full((max(T, 1), n), -1, np.int8)
    for i, tr in enumerate(trs):
        acts[:tr.num_steps, i] = tr.world_actions()
        seats[:tr.num_steps, i] = tr.actions[:, 0]
    acts_d, seats_d = torch.from_numpy(acts).to(dev), torch.from_numpy(seats).to(dev)
    col = torch.arange(env.cap, device=dev)
    good = torch.ones(n, dtype=torch.bool, device=dev)
    env.legal(with_mask=False)
    for t in range(T):
        a, live = acts_d[t], acts_d[t] >= 0
        listed = ((env.ids == a[:, None]) & (col[None, :] < env.counts[:, None])).any(1)
        good &= ~live | (listed & (env.batch["turn"] == seats_d[t]))
        out = env.ply(a, autoreset=False, stats=False)  # step, then the legal moves of the next turn
        good &= ~live | (out["valid"] != 0)
    final = torch.tensor([tr.final_state_hash for tr in trs], dtype=torch.int64, device=dev)
    return (good & (env.batch["zobrist"] == final)).cpu().numpy()
