"""CPU oracle wrapper (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/libjq_oracle.so`` (the scalar C restatement of junqi_core's
batched rules, see ``jq_oracle.c``) through ctypes and keeps a numpy SoA
batch in the same field-major layout as the device batch.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU arms of
``bench.py`` may import this module; the product path never does.

Host tables are generated here, independently of the product package, with
the same numpy calls the reference uses:

* Zobrist: ``junqi_core/_zobrist.py:80-122`` (PCG64 seeded with
  ``0x4A554E51495F5A4F``, ten draws in a fixed order);
* per-slot belief prior: ``junqi_core/info_model.py:64-146``;
* recency LUT: ``junqi_core/observation.py:1549-1562``
  (``np.exp(-max(elapsed,0)/tau, dtype=float32)`` for elapsed in [0, 4096]).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libjq_oracle.so"

NP_ = 120
NC_ = 289
OBS_CH = 317
OBS_GL = 28
HIST = 32
COMPACT_ACTIONS = 16641

# (name, dtype, per-env shape, fill value at allocation)
FIELDS = [
    ("alive", np.uint8, (120,), 0),
    ("piece_type", np.int8, (120,), -1),
    ("piece_seat", np.int8, (120,), -1),
    ("pos_x", np.int8, (120,), -1),
    ("pos_y", np.int8, (120,), -1),
    ("zero_x", np.int8, (120,), -1),
    ("zero_y", np.int8, (120,), -1),
    ("move_count", np.int16, (120,), 0),
    ("active_eat", np.int16, (120,), 0),
    ("passive_surv", np.int16, (120,), 0),
    ("death_reason", np.int8, (120,), -1),
    ("death_step", np.int16, (120,), -1),
    ("death_loc", np.int16, (120,), -1),
    ("cell_pid", np.int16, (289,), -1),
    ("seat_dead", np.uint8, (4,), 0),
    ("seat_flag", np.uint8, (4,), 0),
    ("turn", np.int8, (), 0),
    ("zobrist", np.int64, (), 0),
    ("move_counter", np.int32, (), 0),
    ("mslc", np.int32, (), 0),
    ("terminated", np.uint8, (), 0),
    ("winner", np.int8, (), -1),
    ("draw", np.uint8, (), 0),
    ("cm_direct_lo", np.uint64, (4, 120), 0),
    ("cm_direct_hi", np.uint64, (4, 120), 0),
    ("cm_direct_type", np.uint16, (4, 120), 0),
    ("cm_last_direct_step", np.int16, (4, 120), -1),
    ("cm_direct_other", np.int16, (4, 120), 0),
    ("cm_chain_lo", np.uint64, (4, 120), 0),
    ("cm_chain_hi", np.uint64, (4, 120), 0),
    ("cm_chain_type", np.uint16, (4, 120), 0),
    ("cm_last_chain_step", np.int16, (4, 120), -1),
    ("cm_eaten_lo", np.uint64, (4, 120), 0),
    ("cm_eaten_hi", np.uint64, (4, 120), 0),
    ("cm_rank_floor", np.int8, (4, 120), 0),
    ("cm_rank_floor_step", np.int16, (4, 120), -1),
    ("cm_is_gongb", np.uint8, (4, 120), 0),
    ("cm_not_gongb", np.uint8, (4, 120), 0),
    ("cm_atk_gongb", np.uint8, (4, 120), 0),
    ("hist_src", np.int16, (32,), -1),
    ("hist_dst", np.int16, (32,), -1),
    ("hist_count", np.int32, (), 0),
    ("bel_code", np.uint8, (4, 120), 0),
    ("remaining", np.int16, (4, 4, 12), 0),
    ("rem_tracked", np.uint8, (4, 4), 0),
]

_CTYPE = {
    np.uint8: ctypes.c_uint8, np.int8: ctypes.c_int8, np.int16: ctypes.c_int16,
    np.uint16: ctypes.c_uint16, np.int32: ctypes.c_int32, np.int64: ctypes.c_int64,
    np.uint64: ctypes.c_uint64,
}


class _CBatch(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32)] + [
        (name, ctypes.POINTER(_CTYPE[dt])) for name, dt, _, _ in FIELDS
    ] + [("rules", ctypes.c_int32), ("max_moves", ctypes.c_int32)]


class _CStepOut(ctypes.Structure):
    _fields_ = [
        ("valid", ctypes.POINTER(ctypes.c_uint8)),
        ("event", ctypes.POINTER(ctypes.c_int8)),
        ("terminated", ctypes.POINTER(ctypes.c_uint8)),
        ("winner", ctypes.POINTER(ctypes.c_int8)),
        ("draw", ctypes.POINTER(ctypes.c_uint8)),
        ("flag_captured", ctypes.POINTER(ctypes.c_uint8)),
        ("reward", ctypes.POINTER(ctypes.c_float)),
    ]


def build(force: bool = False) -> Path:
    """Compile the oracle library with its Makefile (idempotent)."""
    src = _HERE / "jq_oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        _set_tables(_lib)
    return _lib


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


# ---------------------------------------------------------------------------
# Host tables (restated from the reference's numpy generators)
# ---------------------------------------------------------------------------

def zobrist_tables() -> dict[str, np.ndarray]:
    """junqi_core/_zobrist.py:80-122: ten PCG64 draws in this exact order."""
    rng = np.random.default_rng(0x4A554E51495F5A4F)

    def draw(shape):
        return rng.integers(0, np.iinfo(np.uint64).max, size=shape, dtype=np.uint64,
                            endpoint=True).astype(np.int64)

    return {
        "piece": draw((120, 14, 289)),
        "turn": draw((4,)),
        "mc": draw((4096,)),
        "mslc": draw((512,)),
        "terminated": draw((1,)),
        "winner": draw((3,)),
        "draw": draw((1,)),
        "seat_dead": draw((4,)),
        "seat_flag": draw((4,)),
        "show_mode": draw((4,)),
    }


_COUNTS = [1, 3, 2, 1, 1, 2, 2, 2, 2, 3, 3, 3]  # JUNQI..GONGB, rules.py:131-144


def prior_table() -> np.ndarray:
    """info_model.py:64-146 per-slot prior P(type | slot), float32 (30, 12)."""
    out = np.zeros((30, 12), dtype=np.float32)
    for slot in range(30):
        if slot in (6, 8, 12, 16, 18):
            continue
        vec = np.zeros(12, dtype=np.float32)
        for ti in range(12):
            t = ti + 2
            if slot not in (26, 28):
                if t == 2:
                    continue
                if t == 3 and slot < 20:
                    continue
                if t == 4 and slot < 5:
                    continue
            vec[ti] = float(_COUNTS[ti])
        s = vec.sum()
        out[slot] = np.asarray(vec / s, dtype=np.float32)
    return out


def uniform12() -> np.ndarray:
    return np.full(12, 1.0 / 12, dtype=np.float32)


def recency_lut() -> np.ndarray:
    """observation.py:1549-1562 freshness planes, one row per (step kind, tau)."""
    el = np.arange(4097).astype(np.float32)
    rows = [np.exp(-np.maximum(el, 0.0) / tau, dtype=np.float32) for tau in (32.0, 256.0, 64.0, 128.0)]
    return np.ascontiguousarray(np.stack(rows).astype(np.float32))


def _set_tables(L):
    z = zobrist_tables()
    keep = [z["piece"], z["turn"], z["mc"], z["mslc"], z["winner"], z["seat_dead"], z["seat_flag"],
            z["show_mode"]]
    pr, un, rc = prior_table(), uniform12(), recency_lut()
    L._keep = keep + [pr, un, rc]
    i64 = ctypes.c_int64
    L.jqo_set_tables(
        _ptr(z["piece"], i64), _ptr(z["turn"], i64), _ptr(z["mc"], i64), _ptr(z["mslc"], i64),
        i64(int(z["terminated"][0])), _ptr(z["winner"], i64), i64(int(z["draw"][0])),
        _ptr(z["seat_dead"], i64), _ptr(z["seat_flag"], i64), _ptr(z["show_mode"], i64),
        _ptr(pr, ctypes.c_float), _ptr(un, ctypes.c_float), _ptr(rc, ctypes.c_float),
    )


def topology() -> dict[str, np.ndarray]:
    L = lib()
    out = {
        "on_board": np.zeros(289, np.int32), "rail": np.zeros(289, np.int32),
        "curve": np.zeros(289, np.int32), "rail_adj": np.zeros((289, 4), np.int32),
        "srays": np.zeros((289, 4, 12), np.int32), "crays": np.zeros((289, 2, 11), np.int32),
        "compact_to_flat": np.zeros(129, np.int32),
    }
    i32 = ctypes.c_int32
    L.jqo_topology(*[_ptr(out[k], i32) for k in
                     ("on_board", "rail", "curve", "rail_adj", "srays", "crays", "compact_to_flat")])
    return out


# ---------------------------------------------------------------------------
# Batch
# ---------------------------------------------------------------------------

class OracleBatch:
    """N environments in the device's field-major layout, stepped on the CPU."""

    def __init__(self, n: int, show_mode: int = 2, rules: int = 0):
        """rules: 0 = BatchedGameState rules, 1 = GameState rules (state.py)."""
        self.n = int(n)
        self.show_mode = int(show_mode)
        self.rules = int(rules)
        self.a: dict[str, np.ndarray] = {}
        for name, dt, shape, fill in FIELDS:
            self.a[name] = np.full((self.n,) + shape, fill, dtype=dt)
        self._c = _CBatch()
        self._c.n = self.n
        self._c.rules = self.rules
        for name, dt, _, _ in FIELDS:
            setattr(self._c, name, _ptr(self.a[name], _CTYPE[dt]))
        self.threads = int(os.environ.get("JQ_ORACLE_THREADS", "1"))

    def __getitem__(self, k):
        return self.a[k]

    def reset_env(self, env: int, lineup120: np.ndarray) -> None:
        lu = np.ascontiguousarray(lineup120, dtype=np.int8)
        assert lu.shape == (120,)
        lib().jqo_reset_env(ctypes.byref(self._c), int(env), _ptr(lu, ctypes.c_int8), self.show_mode)

    def reset_all(self, lineups: np.ndarray) -> None:
        for e in range(self.n):
            self.reset_env(e, lineups[e])

    def step(self, actions: np.ndarray) -> dict[str, np.ndarray]:
        acts = np.ascontiguousarray(actions, dtype=np.int32)
        assert acts.shape == (self.n,)
        out = {
            "valid": np.zeros(self.n, np.uint8), "event": np.zeros(self.n, np.int8),
            "terminated": np.zeros(self.n, np.uint8), "winner": np.zeros(self.n, np.int8),
            "draw": np.zeros(self.n, np.uint8), "flag_captured": np.zeros(self.n, np.uint8),
            "reward": np.zeros(self.n, np.float32),
        }
        so = _CStepOut()
        so.valid = _ptr(out["valid"], ctypes.c_uint8)
        so.event = _ptr(out["event"], ctypes.c_int8)
        so.terminated = _ptr(out["terminated"], ctypes.c_uint8)
        so.winner = _ptr(out["winner"], ctypes.c_int8)
        so.draw = _ptr(out["draw"], ctypes.c_uint8)
        so.flag_captured = _ptr(out["flag_captured"], ctypes.c_uint8)
        so.reward = _ptr(out["reward"], ctypes.c_float)
        lib().jqo_step(ctypes.byref(self._c), _ptr(acts, ctypes.c_int32), self.show_mode,
                       ctypes.byref(so), self.threads)
        return out

    def legal(self, seats: np.ndarray | None = None, cap: int = 512):
        """Per-env ascending legal ids (CSR offsets, values) for ``seats``."""
        seats = self.a["turn"] if seats is None else np.ascontiguousarray(seats, dtype=np.int8)
        counts = np.zeros(self.n, np.int32)
        ids = np.zeros((self.n, cap), np.int32)
        lib().jqo_legal_batch(ctypes.byref(self._c), _ptr(seats, ctypes.c_int8),
                              _ptr(counts, ctypes.c_int32), _ptr(ids, ctypes.c_int32), cap,
                              self.threads)
        if (counts > cap).any():
            raise RuntimeError("legal action list exceeded capacity")
        offsets = np.zeros(self.n + 1, np.int32)
        np.cumsum(counts, out=offsets[1:])
        values = np.concatenate([ids[e, :counts[e]] for e in range(self.n)]) if self.n else ids[:0, 0]
        return offsets, values.astype(np.int32)

    def canonical_mask(self, ids: np.ndarray, seat: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        m = np.zeros(COMPACT_ACTIONS, np.uint8)
        lib().jqo_canonical_mask(_ptr(ids, ctypes.c_int32), int(ids.size), int(seat),
                                 _ptr(m, ctypes.c_uint8))
        return m.astype(bool)

    def slot_mask(self, seats: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
        """Per-piece 80-slot legal mask of the reference GPU format
        (game_state.cu:1985-2197): (n, 120, 80) bool and the destination flat
        cell of every set slot (n, 120, 80) int16, -1 elsewhere."""
        seats = self["turn"] if seats is None else np.asarray(seats, np.int8)
        mask = np.zeros((self.n, 120, 80), np.uint8)
        dst = np.zeros((self.n, 120, 80), np.int16)
        for e in range(self.n):
            lib().jqo_slot_mask(ctypes.byref(self._c), e, int(seats[e]), _ptr(mask[e], ctypes.c_uint8),
                                _ptr(dst[e], ctypes.c_int16))
        return mask.astype(bool), dst

    def obs(self, observers: np.ndarray | None = None):
        """(n, 317, 17, 17) float32 + (n, 28) float32 for one observer per env."""
        obsv = self.a["turn"] if observers is None else np.ascontiguousarray(observers, dtype=np.int8)
        sp = np.zeros((self.n, OBS_CH, 17, 17), np.float32)
        gl = np.zeros((self.n, OBS_GL), np.float32)
        lib().jqo_obs_batch(ctypes.byref(self._c), _ptr(obsv, ctypes.c_int8), self.show_mode,
                            _ptr(sp, ctypes.c_float), _ptr(gl, ctypes.c_float), self.threads)
        return sp, gl

    def obs_beliefs(self, beliefs: np.ndarray, observers: np.ndarray | None = None):
        """As ``obs`` with caller-given float beliefs (N, 4, 12, 289) [env,
        observer, type, world cell]: the reference GPU encoder's belief
        input (observation.cu:246-253, 330-370, 417-424, 533-544); the
        enemy sums of global[0:24] are added in ascending pid order."""
        obsv = self.a["turn"] if observers is None else np.ascontiguousarray(observers, dtype=np.int8)
        bel = np.ascontiguousarray(beliefs, dtype=np.float32)
        assert bel.shape == (self.n, 4, 12, 289)
        sp = np.zeros((self.n, OBS_CH, 17, 17), np.float32)
        gl = np.zeros((self.n, OBS_GL), np.float32)
        lib().jqo_obs_ext_batch(ctypes.byref(self._c), _ptr(obsv, ctypes.c_int8), self.show_mode,
                                _ptr(bel, ctypes.c_float), _ptr(sp, ctypes.c_float), _ptr(gl, ctypes.c_float),
                                self.threads)
        return sp, gl

    def cellbel_init(self, prior: np.ndarray, bel: np.ndarray, envs=None) -> None:
        """Per-cell float beliefs of the reference GPU rollout, initialised in
        place in ``bel`` (N, 4, 12, 289) for ``envs`` (default all):
        belief_init_kernel, belief.cu:172-248."""
        pr = np.ascontiguousarray(prior, dtype=np.float32).reshape(30 * 12)
        assert bel.dtype == np.float32 and bel.shape == (self.n, 4, 12, 289) and bel.flags.c_contiguous
        for e in range(self.n) if envs is None else envs:
            lib().jqo_cellbel_init(ctypes.byref(self._c), int(e), _ptr(pr, ctypes.c_float), _ptr(bel, ctypes.c_float))

    def cellbel_update(self, event, flag_captured, world_actions, prev_dead, strongholds, bel: np.ndarray) -> None:
        """belief_update_kernel (belief.cu:255-565) on this batch's post-step
        state, in place in ``bel``; prev_dead (N, 4) is the seat_dead
        snapshot taken before the step, strongholds the 4 x 2 flat cells."""
        assert bel.dtype == np.float32 and bel.shape == (self.n, 4, 12, 289) and bel.flags.c_contiguous
        ev = np.asarray(event).astype(np.int64).reshape(self.n)
        fc = np.asarray(flag_captured).astype(np.int64).reshape(self.n)
        wa = np.asarray(world_actions).astype(np.int64).reshape(self.n)
        pd = np.ascontiguousarray(prev_dead, dtype=np.uint8).reshape(self.n, 4)
        sh = np.ascontiguousarray(strongholds, dtype=np.int16).reshape(8)
        for e in range(self.n):
            lib().jqo_cellbel_update(ctypes.byref(self._c), e, int(ev[e]), int(fc[e]), ctypes.c_int32(int(wa[e])),
                                     _ptr(pd[e], ctypes.c_uint8), _ptr(sh, ctypes.c_int16),
                                     _ptr(bel, ctypes.c_float))

    def obs_one(self, env: int, observer: int):
        sp = np.zeros((OBS_CH, 17, 17), np.float32)
        gl = np.zeros(OBS_GL, np.float32)
        lib().jqo_obs(ctypes.byref(self._c), int(env), int(observer), self.show_mode,
                      _ptr(sp, ctypes.c_float), _ptr(gl, ctypes.c_float))
        return sp, gl


def zobrist_recompute(a: dict[str, np.ndarray], show_mode: int) -> np.ndarray:
    """Zobrist hash of every env rebuilt from scratch (state.py:1761-1815,
    ``_recompute_zobrist``), vectorised over envs.  ``a`` holds the batch
    fields (oracle names); returns int64 (N,)."""
    z = zobrist_tables()
    alive = np.asarray(a["alive"]).astype(bool)
    n = alive.shape[0]
    t = np.asarray(a["piece_type"]).astype(np.int64)
    flat = np.asarray(a["pos_y"]).astype(np.int64) * 17 + np.asarray(a["pos_x"]).astype(np.int64)
    live = alive & (t >= 0) & (flat >= 0)
    pid = np.broadcast_to(np.arange(120), alive.shape)
    keys = np.where(live, z["piece"][pid, np.clip(t, 0, 13), np.clip(flat, 0, 288)], 0).view(np.uint64)
    h = np.bitwise_xor.reduce(keys, axis=1)
    u = lambda x: np.asarray(x, np.int64).view(np.uint64)  # noqa: E731
    h ^= u(z["turn"][np.asarray(a["turn"]).astype(np.int64) & 3])
    h ^= u(z["mc"][np.asarray(a["move_counter"]).astype(np.int64) & 0xFFF])
    h ^= u(z["mslc"][np.asarray(a["mslc"]).astype(np.int64) & 0x1FF])
    h ^= u(z["winner"][np.asarray(a["winner"]).astype(np.int64) + 1])
    h ^= u(np.full(n, z["show_mode"][show_mode]))
    h ^= np.where(np.asarray(a["terminated"]).astype(bool), u(z["terminated"][0]), np.uint64(0))
    h ^= np.where(np.asarray(a["draw"]).astype(bool), u(z["draw"][0]), np.uint64(0))
    sd = np.asarray(a["seat_dead"]).astype(bool).reshape(n, 4)
    sf = np.asarray(a["seat_flag"]).astype(bool).reshape(n, 4)
    for s in range(4):
        h ^= np.where(sd[:, s], u(z["seat_dead"][s]), np.uint64(0))
        h ^= np.where(sf[:, s], u(z["seat_flag"][s]), np.uint64(0))
    return h.view(np.int64)


def slot_tables() -> dict[str, np.ndarray]:
    """The 80-slot mask's tables as the oracle rebuilds them (tables.cu:176-350)."""
    adj8 = np.zeros((289, 8), np.int32)
    sr = np.zeros((289, 4, 12), np.int32)
    ra = np.zeros((289, 8), np.int32)
    lib().jqo_slot_tables(_ptr(adj8, ctypes.c_int32), _ptr(sr, ctypes.c_int32), _ptr(ra, ctypes.c_int32))
    return {"adj8": adj8, "srays": sr, "rail_adj": ra}


def load_state(batch: OracleBatch, arrays: dict[str, np.ndarray], init_beliefs: bool = True) -> None:
    """Copy state fields (oracle names) into ``batch`` and seed beliefs."""
    for k, v in arrays.items():
        if k in batch.a:
            batch.a[k][...] = np.asarray(v).reshape(batch.a[k].shape).astype(batch.a[k].dtype)
    if init_beliefs:
        for e in range(batch.n):
            lib().jqo_init_beliefs(ctypes.byref(batch._c), e, batch.show_mode)
