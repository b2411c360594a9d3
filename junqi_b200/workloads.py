"""Start positions of the benchmark configurations that need more than a reset.

``late_game_starts`` builds the stress configuration's positions (configs[4]
of the benchmark: late-game starts from seeded random setups, 0-60 % of the
pieces removed, engineers placed on the railway so legal generation runs
long rail flood-fills, combat-dense contact).  It starts from
``GameState.new_game`` positions drawn from the setup pool (``jq_reset``),
edits them on the host with numpy, writes them back and lets the device
rebuild the Zobrist hashes (``jq_rehash``, the counterpart of
``_recompute_zobrist``, state.py:1761) and the initial beliefs
(``jq_init_beliefs``).  The edit, per env, seeded by ``seed``:

* draw a removal fraction f ~ U(0, 0.6) and remove every piece except the
  flag with probability f; a removed piece looks like an empty camp slot
  (alive 0, type / seat / position / zero cell / death fields -1);
* move each remaining engineer, with probability 0.7, onto a distinct empty
  rail cell (its zero cell is unchanged);
* rebuild ``cell_pid``.
A seat left without movable pieces loses on its first turn by Q12, as in
the rules.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N

JUNQI, GONGB = 2, 13


def rail_cells() -> np.ndarray:
    """Flat indices of the 73 railway cells (board.py rail layout)."""
    o = {k: np.zeros(s, np.int32) for k, s in (("on", 289), ("rail", 289), ("curve", 289), ("adj", 289 * 4),
                                                ("sr", 289 * 48), ("cr", 289 * 22), ("c2f", 129), ("fl", 289))}
    N.lib().jq_topology_dump(*[o[k].ctypes.data for k in ("on", "rail", "curve", "adj", "sr", "cr", "c2f", "fl")])
    return np.nonzero(o["rail"])[0].astype(np.int64)


def thin_positions(st: dict, seed: int, remove_max: float = 0.6, engineer_move_p: float = 0.7) -> dict:
    """The host edit described in the module docstring, on a state dict of
    new_game positions (field names of ``DeviceBatch``); returns it edited."""
    rng = np.random.default_rng(seed)
    alive = st["alive"].astype(bool)
    n = alive.shape[0]
    typ = st["piece_type"].astype(np.int64)
    frac = rng.uniform(0.0, remove_max, n)
    remove = alive & (typ != JUNQI) & (rng.random((n, 120)) < frac[:, None])
    for k in ("piece_type", "piece_seat", "pos_x", "pos_y", "zero_x", "zero_y", "death_reason", "death_step",
              "death_loc"):
        st[k][remove] = -1
    st["alive"][remove] = 0
    alive &= ~remove
    # engineers onto distinct empty rail cells, in a random order per env
    rails = rail_cells()
    flat = st["pos_y"].astype(np.int64) * 17 + st["pos_x"].astype(np.int64)
    occ = np.zeros((n, 289), bool)
    ei, pi = np.nonzero(alive)
    occ[ei, flat[ei, pi]] = True
    keys = rng.random((n, rails.size))
    keys[occ[:, rails]] = 2.0  # occupied rail cells sort last
    order = np.argsort(keys, axis=1)
    n_empty = (~occ[:, rails]).sum(1)
    moving = alive & (typ == GONGB) & (rng.random((n, 120)) < engineer_move_p)
    rank = np.cumsum(moving, axis=1) - 1
    moving &= rank < n_empty[:, None]
    ei, pi = np.nonzero(moving)
    dst = rails[order[ei, rank[ei, pi]]]
    st["pos_x"][ei, pi] = (dst % 17).astype(st["pos_x"].dtype)
    st["pos_y"][ei, pi] = (dst // 17).astype(st["pos_y"].dtype)
    # cell -> piece index
    cell = np.full((n, 289), -1, np.int16)
    ei, pi = np.nonzero(alive)
    cell[ei, st["pos_y"][ei, pi].astype(np.int64) * 17 + st["pos_x"][ei, pi].astype(np.int64)] = pi
    st["cell_pid"] = cell
    return st


def late_game_starts(env, seed: int) -> None:
    """Replace every env of ``env`` (a JunqiEnvB200) by a late-game start."""
    env.reset(seed=seed, ply=0, all_envs=True)
    st = env.batch.to_host()
    env.batch.load(thin_positions(st, seed))
    L = N.lib()
    s = ctypes.byref(env.batch.struct)
    stream = torch.cuda.current_stream().cuda_stream
    N.check(L.jq_rehash(s, env.show_mode, stream), "jq_rehash")
    N.check(L.jq_init_beliefs(s, env.show_mode, stream), "jq_init_beliefs")
    env.legal()
