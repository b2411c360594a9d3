"""Device batch: torch-owned device memory described to the C ABI.

Every field of ``jq_batch`` (include/jq.h) is a contiguous CUDA tensor with
the env index outermost.  Unsigned 16/64-bit fields are stored in
same-width signed torch tensors (torch's unsigned support is partial); the
kernels read the bits, and ``to_host`` returns them with their declared
numpy dtypes.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as N

# (name, numpy dtype, per-env shape, fill)  -- order and names follow jq_batch
FIELDS = [
    ("alive", np.uint8, (120,), 0), ("piece_type", np.int8, (120,), -1),
    ("piece_seat", np.int8, (120,), -1), ("pos_x", np.int8, (120,), -1),
    ("pos_y", np.int8, (120,), -1), ("zero_x", np.int8, (120,), -1),
    ("zero_y", np.int8, (120,), -1), ("move_count", np.int16, (120,), 0),
    ("active_eat", np.int16, (120,), 0), ("passive_surv", np.int16, (120,), 0),
    ("death_reason", np.int8, (120,), -1), ("death_step", np.int16, (120,), -1),
    ("death_loc", np.int16, (120,), -1), ("cell_pid", np.int16, (289,), -1),
    ("seat_dead", np.uint8, (4,), 0), ("seat_flag", np.uint8, (4,), 0),
    ("turn", np.int8, (), 0), ("zobrist", np.int64, (), 0), ("move_counter", np.int32, (), 0),
    ("mslc", np.int32, (), 0), ("terminated", np.uint8, (), 0), ("winner", np.int8, (), -1),
    ("draw", np.uint8, (), 0),
    ("cm_direct_lo", np.uint64, (4, 120), 0), ("cm_direct_hi", np.uint64, (4, 120), 0),
    ("cm_direct_type", np.uint16, (4, 120), 0), ("cm_last_direct_step", np.int16, (4, 120), -1),
    ("cm_direct_other", np.int16, (4, 120), 0), ("cm_chain_lo", np.uint64, (4, 120), 0),
    ("cm_chain_hi", np.uint64, (4, 120), 0), ("cm_chain_type", np.uint16, (4, 120), 0),
    ("cm_last_chain_step", np.int16, (4, 120), -1), ("cm_eaten_lo", np.uint64, (4, 120), 0),
    ("cm_eaten_hi", np.uint64, (4, 120), 0), ("cm_rank_floor", np.int8, (4, 120), 0),
    ("cm_rank_floor_step", np.int16, (4, 120), -1), ("cm_is_gongb", np.uint8, (4, 120), 0),
    ("cm_not_gongb", np.uint8, (4, 120), 0), ("cm_atk_gongb", np.uint8, (4, 120), 0),
    ("hist_src", np.int16, (32,), -1), ("hist_dst", np.int16, (32,), -1),
    ("hist_count", np.int32, (), 0), ("bel_code", np.uint8, (4, 120), 0),
    ("remaining", np.int16, (4, 4, 12), 0), ("rem_tracked", np.uint8, (4, 4), 0),
]
assert [f[0] for f in FIELDS] == [f[0] for f in N.BATCH_FIELDS]

_STORAGE = {np.uint8: torch.uint8, np.int8: torch.int8, np.int16: torch.int16,
            np.uint16: torch.int16, np.int32: torch.int32, np.int64: torch.int64,
            np.uint64: torch.int64}
_SIGNED_VIEW = {np.uint16: np.int16, np.uint64: np.int64}

BYTES_PER_ENV = sum(int(np.dtype(dt).itemsize * np.prod(sh, dtype=np.int64)) for _, dt, sh, _ in FIELDS)


class DeviceBatch:
    """N envs of device state in the jq_batch layout."""

    def __init__(self, n: int, device: torch.device | str | int = "cuda", rules: int = N.RULES_BATCHED,
                 max_moves: int = 0):
        if n <= 0:
            raise ValueError(f"num_envs must be positive, got {n}")
        self.n = int(n)
        self.device = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        self.t: dict[str, torch.Tensor] = {}
        for name, dt, shape, fill in FIELDS:
            self.t[name] = torch.full((self.n,) + shape, fill, dtype=_STORAGE[dt], device=self.device)
        self._struct = N.JqBatch()
        self._struct.n = self.n
        self._struct.rules = int(rules)
        self._pool = None
        self.max_moves = max_moves
        for name, _, _, _ in FIELDS:
            setattr(self._struct, name, self.t[name].data_ptr())

    @property
    def rules(self) -> int:
        return int(self._struct.rules)

    @rules.setter
    def rules(self, r: int) -> None:
        if r not in (N.RULES_BATCHED, N.RULES_GAMESTATE):
            raise ValueError(f"unknown rule set {r}")
        self._struct.rules = int(r)

    @property
    def max_moves(self) -> int:
        """Episode cap in plies (a draw when reached), 0 for none beyond the rules' own."""
        return int(self._struct.max_moves)

    @max_moves.setter
    def max_moves(self, m: int) -> None:
        if int(m) < 0:
            raise ValueError(f"max_moves must be >= 0, got {m}")
        self._struct.max_moves = int(m)

    def set_pool(self, pool: torch.Tensor | None) -> None:
        """Setup pool ((P, 120) int8 device tensor) the resets of this batch
        draw from; None: the device-wide pool of jq_set_setup_pool.  The
        batch keeps a reference, so the memory outlives every launch."""
        if pool is None:
            self._pool = None
            self._struct.pool = None
            self._struct.pool_size = 0
            return
        if pool.dtype != torch.int8 or pool.dim() != 2 or pool.shape[1] != 120 or not pool.is_contiguous():
            raise ValueError("pool must be a contiguous (P, 120) int8 tensor")
        if pool.device.type != "cuda" or (self.device.index is not None and pool.device.index != self.device.index):
            raise ValueError(f"pool is on {pool.device}, the batch on {self.device}")
        self._pool = pool
        self._struct.pool = pool.data_ptr()
        self._struct.pool_size = int(pool.shape[0])

    @property
    def struct(self) -> N.JqBatch:
        return self._struct

    def view(self, start: int, count: int) -> N.JqBatch:
        """jq_batch describing envs [start, start + count) of this batch (no copy)."""
        if not (0 <= start and count > 0 and start + count <= self.n):
            raise ValueError(f"env range [{start}, {start + count}) outside [0, {self.n})")
        s = N.JqBatch()
        s.n = int(count)
        s.rules = self._struct.rules
        s.max_moves = self._struct.max_moves
        s.pool = self._struct.pool
        s.pool_size = self._struct.pool_size
        for name, _, _, _ in FIELDS:
            t = self.t[name]
            setattr(s, name, t.data_ptr() + start * t.stride(0) * t.element_size())
        return s

    def __getitem__(self, k: str) -> torch.Tensor:
        return self.t[k]

    def load(self, arrays: dict) -> None:
        """Copy host arrays (names as in FIELDS) into the device batch."""
        for name, dt, shape, _ in FIELDS:
            if name not in arrays:
                continue
            a = np.ascontiguousarray(np.asarray(arrays[name]).reshape((self.n,) + shape).astype(dt))
            if dt in _SIGNED_VIEW:
                a = a.view(_SIGNED_VIEW[dt])
            self.t[name].copy_(torch.from_numpy(a))

    def to_host(self, names=None, envs=None) -> dict[str, np.ndarray]:
        """Host copies of the fields (all, or `names`), for all envs or the index list `envs`."""
        idx = None if envs is None else torch.as_tensor(np.asarray(envs, np.int64), device=self.device)
        out = {}
        for name, dt, _, _ in FIELDS:
            if names is not None and name not in names:
                continue
            t = self.t[name] if idx is None else self.t[name].index_select(0, idx)
            a = t.cpu().numpy()
            out[name] = a.view(dt) if dt in _SIGNED_VIEW else a.astype(dt, copy=False)
        return out
