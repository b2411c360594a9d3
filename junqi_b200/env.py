"""High-level batched environment over the C ABI.

``JunqiEnvB200`` owns a :class:`DeviceBatch` plus every output buffer of the
hot path (step results, legal CSR + canonical mask, observations, episode
stats) as torch CUDA tensors, and issues the C-ABI calls on torch's current
stream.  One ply of the GPU rollout loop (``gpu_collector.py:770-978`` in the
reference) is::

    env.ply(actions)      # step + auto-reset + legal CSR/mask for the new turn
    env.observe()         # 317-channel observation of each env's acting seat
    actions = env.sample_uniform(seed, t)   # stand-in policy

All of it stays on the device; nothing synchronises the host.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N
from . import tables
from .batch import DeviceBatch

BRIGHT, DARK, HALF_DARK = 0, 1, 2
OBS_CHANNELS, OBS_GLOBAL, MASK_BYTES, MAX_LEGAL = 317, 28, 16641, 512

_ready_devices: set[int] = set()


def _stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def ensure_device(device: int) -> None:
    """jq_init + table uploads, once per device per process."""
    if device in _ready_devices:
        return
    if not torch.cuda.is_available():
        raise RuntimeError("junqi_b200 needs a CUDA device; none is available")
    torch.cuda.set_device(device)
    L = N.lib()
    N.check(L.jq_init(device), "jq_init")
    z = tables.zobrist_tables()
    p = lambda a: a.ctypes.data  # noqa: E731
    N.check(L.jq_upload_zobrist(p(z["piece"]), p(z["turn"]), p(z["move_counter"]), p(z["mslc"]),
                                p(z["winner"]), int(z["terminated"][0]), int(z["draw"][0]),
                                p(z["seat_dead"]), p(z["seat_flag"]), p(z["show_mode"])), "jq_upload_zobrist")
    pr, un, rc = tables.prior_table(), tables.uniform12(), tables.recency_lut()
    N.check(L.jq_upload_obs_tables(p(pr), p(un), p(rc)), "jq_upload_obs_tables")
    _ready_devices.add(device)


class JunqiEnvB200:
    def __init__(self, num_envs: int, *, device: int = 0, show_mode: int = HALF_DARK,
                 pool: np.ndarray | None = None, pool_size: int = 10_000, pool_seed: int = 42,
                 obs_seats: int = 1, legal_cap: int = MAX_LEGAL, with_mask: bool = True,
                 with_obs: bool = True, rules: int = N.RULES_BATCHED, max_moves: int = 0):
        ensure_device(device)
        self.device = torch.device("cuda", device)
        self.n = int(num_envs)
        self.show_mode = int(show_mode)
        self.cap = int(legal_cap)
        self.obs_seats = int(obs_seats)
        self.batch = DeviceBatch(self.n, self.device, rules=rules, max_moves=max_moves)
        if pool is None:
            pool = tables.build_setup_pool(pool_size, seed=pool_seed)
        self.set_pool(pool)
        dev = self.device
        n = self.n
        # The step results, then the legal CSR (offsets, values), as views of
        # one device buffer: a host that reads the results and the CSR after
        # every ply does it with one copy of a prefix of this buffer.
        fields = (("valid", torch.uint8), ("event", torch.int8), ("terminated", torch.uint8),
                  ("winner", torch.int8), ("draw", torch.uint8), ("flag_captured", torch.uint8),
                  ("reward", torch.float32), ("world_action", torch.int32), ("zobrist", torch.int64))
        layout, pos = [], 0
        for k, dt in fields + (("offsets", torch.int32),):
            layout.append((k, dt, pos))
            pos += -(-(n + (k == "offsets")) * dt.itemsize // 16) * 16
        self.values_byte_offset = pos
        self.io = torch.zeros(pos + n * self.cap * 4, dtype=torch.uint8, device=dev)
        views = {k: self.io[o:o + (n + (k == "offsets")) * dt.itemsize].view(dt) for k, dt, o in layout}
        self.offsets = views.pop("offsets")
        self.values = self.io[pos:].view(torch.int32)
        self.out = views
        self._out = N.JqStepOut(**{k: v.data_ptr() for k, v in self.out.items()})
        self.counts = torch.zeros(n, dtype=torch.int32, device=dev)
        self.ids = torch.zeros((n, self.cap), dtype=torch.int32, device=dev)
        self.mask = torch.zeros((n, MASK_BYTES), dtype=torch.uint8, device=dev) if with_mask else None
        self.csr_scratch = torch.zeros(max(1, N.lib().jq_csr_scratch_ints(n)), dtype=torch.int32, device=dev)
        self.actions = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.compact_actions = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.stats = torch.zeros(6, dtype=torch.int64, device=dev)  # see sharding.STAT_NAMES
        if with_obs:
            u = n * self.obs_seats
            self.spatial = torch.empty((u, OBS_CHANNELS, 17, 17), dtype=torch.float32, device=dev)
            self.global_ = torch.empty((u, OBS_GLOBAL), dtype=torch.float32, device=dev)
        else:
            self.spatial = self.global_ = None

    # ------------------------------------------------------------------
    def set_pool(self, pool: np.ndarray) -> None:
        pool = np.ascontiguousarray(pool, dtype=np.int8)
        tables.validate_pool(pool)
        self.pool_host = pool
        self.pool = torch.from_numpy(pool).to(self.device)
        # the batch's own pool: other envs in the process keep theirs
        self.batch.set_pool(self.pool)

    def _ptr(self, t):
        return None if t is None else t.data_ptr()

    def reset(self, seed: int = 0, ply: int = 0, all_envs: bool = True) -> None:
        """Reset envs from the pool (all, or only terminated ones) and refresh legal moves."""
        N.check(N.lib().jq_reset(ctypes.byref(self.batch.struct), seed, ply, int(all_envs), self.show_mode,
                                 _stream_ptr()), "jq_reset")
        self.legal()

    def reset_rows(self, rows) -> None:
        """Reset env e from pool row rows[e] (rows[e] < 0: leave env e as it is); no legal refresh."""
        r = torch.as_tensor(np.asarray(rows, np.int32) if not torch.is_tensor(rows) else rows, dtype=torch.int32)
        r = r.to(self.device).contiguous()
        if r.numel() != self.n:
            raise ValueError(f"rows: expected {self.n} entries, got {r.numel()}")
        N.check(N.lib().jq_reset_rows(ctypes.byref(self.batch.struct), r.data_ptr(), self.show_mode, _stream_ptr()),
                "jq_reset_rows")

    def load_state(self, arrays: dict, init_beliefs: bool = True) -> None:
        self.batch.load(arrays)
        if init_beliefs:
            N.check(N.lib().jq_init_beliefs(ctypes.byref(self.batch.struct), self.show_mode, _stream_ptr()),
                    "jq_init_beliefs")

    def step(self, actions: torch.Tensor) -> dict[str, torch.Tensor]:
        a = actions.to(device=self.device, dtype=torch.int32).contiguous()
        N.check(N.lib().jq_step(ctypes.byref(self.batch.struct), a.data_ptr(), self.show_mode,
                                ctypes.byref(self._out), _stream_ptr()), "jq_step")
        return self.out

    def ply(self, actions: torch.Tensor | None, seed: int = 0, ply: int = 0, autoreset: bool = True,
            stats: bool = True) -> dict[str, torch.Tensor]:
        """Step (if actions given), auto-reset terminated envs, legal CSR + mask of the new turn."""
        a = None if actions is None else actions.to(device=self.device, dtype=torch.int32).contiguous()
        N.check(N.lib().jq_ply(ctypes.byref(self.batch.struct), self._ptr(a), self.show_mode,
                               ctypes.byref(self._out), int(autoreset), seed, ply, self.counts.data_ptr(),
                               self.ids.data_ptr(), self.cap, self._ptr(self.mask),
                               self.stats.data_ptr() if stats else None, _stream_ptr()), "jq_ply")
        return self.out

    def legal(self, seats: torch.Tensor | None = None, with_mask: bool = True):
        s = None if seats is None else seats.to(device=self.device, dtype=torch.int8).contiguous()
        N.check(N.lib().jq_legal(ctypes.byref(self.batch.struct), self._ptr(s), self.counts.data_ptr(),
                                 self.ids.data_ptr(), self.cap, self._ptr(self.mask) if with_mask else None,
                                 _stream_ptr()), "jq_legal")
        return self.counts, self.ids

    def legal_slots(self, seats: torch.Tensor | None = None) -> torch.Tensor:
        """Per-piece 80-slot legal mask (N, 120, 80) uint8 of each env's turn (or `seats`)."""
        s = None if seats is None else seats.to(device=self.device, dtype=torch.int8).contiguous()
        out = torch.empty((self.n, 120, 80), dtype=torch.uint8, device=self.device)
        N.check(N.lib().jq_legal_slots(ctypes.byref(self.batch.struct), self._ptr(s), out.data_ptr(),
                                       _stream_ptr()), "jq_legal_slots")
        return out

    def io_prefix_bytes(self, values: int) -> int:
        """Bytes of ``io`` that hold the step results, the CSR offsets and the
        first ``values`` CSR values."""
        return self.values_byte_offset + 4 * min(int(values), self.n * self.cap)

    def csr(self):
        """(offsets (N+1,), values (N*cap,)) of the last legal generation."""
        N.check(N.lib().jq_csr(self.n, self.counts.data_ptr(), self.ids.data_ptr(), self.cap,
                               self.offsets.data_ptr(), self.values.data_ptr(), self.csr_scratch.data_ptr(),
                               _stream_ptr()), "jq_csr")
        return self.offsets, self.values

    def observe(self, observers: torch.Tensor | None = None, seats_per_env: int | None = None,
                beliefs: torch.Tensor | None = None):
        """Observations of `observers` (default: each env's turn, or seats 0..3).  With `beliefs`
        ((N, 4, 12, 289) float32 per-cell beliefs, e.g. a belief network's output) the belief
        planes and global[0:24] come from them instead of the env's own beliefs."""
        s = self.obs_seats if seats_per_env is None else int(seats_per_env)
        if self.spatial is None or self.spatial.shape[0] < self.n * s:
            self.spatial = torch.empty((self.n * s, OBS_CHANNELS, 17, 17), dtype=torch.float32, device=self.device)
            self.global_ = torch.empty((self.n * s, OBS_GLOBAL), dtype=torch.float32, device=self.device)
        o = None if observers is None else observers.to(device=self.device, dtype=torch.int8).contiguous()
        if beliefs is None:
            N.check(N.lib().jq_observe(ctypes.byref(self.batch.struct), self._ptr(o), s, self.show_mode,
                                       self.spatial.data_ptr(), self.global_.data_ptr(), _stream_ptr()), "jq_observe")
        else:
            bel = beliefs.to(device=self.device, dtype=torch.float32).contiguous()
            if tuple(bel.shape) != (self.n, 4, 12, 289):
                raise ValueError(f"beliefs must be ({self.n}, 4, 12, 289), got {tuple(bel.shape)}")
            N.check(N.lib().jq_observe_beliefs(ctypes.byref(self.batch.struct), self._ptr(o), s, self.show_mode,
                                               bel.data_ptr(), self.spatial.data_ptr(), self.global_.data_ptr(),
                                               _stream_ptr()), "jq_observe_beliefs")
        return self.spatial[: self.n * s], self.global_[: self.n * s]

    # -- per-cell float beliefs of the reference GPU rollout (belief.cu) --------
    def cell_beliefs_init(self, beliefs: torch.Tensor, prior: torch.Tensor,
                          env_mask: torch.Tensor | None = None) -> torch.Tensor:
        """Seed ``beliefs`` ((N, 4, 12, 289) float32 on this device) for the envs
        with env_mask[e] != 0 (default all): one-hot rows for each observer's own
        pieces, the slot's row of ``prior`` (30 x 12) for every other piece."""
        self._check_cell_beliefs(beliefs)
        pr = prior.to(device=self.device, dtype=torch.float32).contiguous()
        if pr.numel() != 360:
            raise ValueError("prior must hold 30 x 12 floats")
        m = None if env_mask is None else env_mask.to(device=self.device, dtype=torch.uint8).contiguous()
        N.check(N.lib().jq_cell_beliefs_init(ctypes.byref(self.batch.struct), self._ptr(m), pr.data_ptr(),
                                             beliefs.data_ptr(), _stream_ptr()), "jq_cell_beliefs_init")
        return beliefs

    def cell_beliefs_snapshot(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(seat_dead (N, 4), terminated (N,)) as uint8 copies, taken before a step."""
        dead = torch.empty((self.n, 4), dtype=torch.uint8, device=self.device)
        term = torch.empty(self.n, dtype=torch.uint8, device=self.device)
        N.check(N.lib().jq_cell_beliefs_snapshot(ctypes.byref(self.batch.struct), dead.data_ptr(), term.data_ptr(),
                                                 _stream_ptr()), "jq_cell_beliefs_snapshot")
        return dead, term

    def cell_beliefs_update(self, beliefs: torch.Tensor, world_actions: torch.Tensor, prev_dead: torch.Tensor,
                            strongholds: torch.Tensor) -> torch.Tensor:
        """Apply the last step (its event and flag capture in ``self.out``) to
        ``beliefs``; ``prev_dead`` from cell_beliefs_snapshot before the step,
        ``strongholds`` (4 x 2) each seat's stronghold flat cells."""
        self._check_cell_beliefs(beliefs)
        wa = world_actions.to(device=self.device, dtype=torch.int32).contiguous()
        pd = prev_dead.to(device=self.device, dtype=torch.uint8).contiguous()
        sh = strongholds.to(device=self.device, dtype=torch.int16).contiguous()
        if wa.numel() != self.n or pd.numel() != 4 * self.n or sh.numel() != 8:
            raise ValueError("world_actions (N,), prev_dead (N, 4) and strongholds (4, 2) expected")
        N.check(N.lib().jq_cell_beliefs_update(ctypes.byref(self.batch.struct), self.out["event"].data_ptr(),
                                               self.out["flag_captured"].data_ptr(), wa.data_ptr(), pd.data_ptr(),
                                               sh.data_ptr(), beliefs.data_ptr(), _stream_ptr()),
                "jq_cell_beliefs_update")
        return beliefs

    def _check_cell_beliefs(self, beliefs: torch.Tensor) -> None:
        if (beliefs.dtype != torch.float32 or tuple(beliefs.shape) != (self.n, 4, 12, 289)
                or not beliefs.is_contiguous() or beliefs.device != torch.device(self.device)):
            raise ValueError(f"beliefs must be a contiguous ({self.n}, 4, 12, 289) float32 tensor on {self.device}")

    def sample_uniform(self, seed: int, ply: int) -> torch.Tensor:
        N.check(N.lib().jq_sample_uniform(self.n, self.counts.data_ptr(), self.ids.data_ptr(), self.cap, seed, ply,
                                          self.actions.data_ptr(), _stream_ptr()), "jq_sample_uniform")
        return self.actions

    def sample_softmax(self, seed: int, ply: int) -> torch.Tensor:
        N.check(N.lib().jq_sample_softmax(ctypes.byref(self.batch.struct), self.counts.data_ptr(),
                                          self.ids.data_ptr(), self.cap, seed, ply, self.compact_actions.data_ptr(),
                                          self.actions.data_ptr(), _stream_ptr()), "jq_sample_softmax")
        return self.actions

    def state(self) -> dict[str, np.ndarray]:
        return self.batch.to_host()
