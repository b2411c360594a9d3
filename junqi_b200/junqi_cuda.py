"""Drop-in replacement for the reference's ``junqi_cuda`` extension module.

Same names, argument order and return shapes as
``src/env/cuda/src/bindings.cpp:458-1311`` of freezeng123456/JunQi, served by
the sm_100a kernels of ``libjq.so``.  Differences a caller can observe:

* Beliefs are part of the device state and follow ``BeliefTensor`` exactly
  (info_model.py), updated inside the step.  ``update_beliefs_after_step``,
  ``record_move_history``, ``snapshot_pre_step_flags`` and
  ``init_beliefs_for_reset_envs`` are therefore no-ops.
* Per-cell float beliefs given to ``upload_beliefs`` /
  ``build_observation_batch`` (e.g. a belief network's output) are used as
  given by every observation built afterwards (``jq_observe_beliefs``) until
  ``init_all_beliefs`` or ``gpu_scratch_reset``; steps do not apply the
  reference's per-cell float update rules to them (belief.cu:255-568), and
  ``DeviceRolloutHistory`` records the library's own beliefs.
* Resets reproduce ``GameState.new_game`` exactly (full initial Zobrist
  hash, -1 in unused slots); the pool entry is ``jq_pool_index(seed, k, env)``
  where k counts reset calls.
* Legal ids are returned ascending per env (the CPU order).
* Errors raise ``RuntimeError``; nothing calls ``exit()``.

Device pointers returned by ``step_device`` / ``legal_mask_canonical_batch``
alias buffers owned by the state object and are overwritten by the next call,
as in the reference.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N
from . import tables
from .batch import DeviceBatch
from .env import ensure_device

NUM_ENVS_MAX = 1 << 20
NUM_PIECES = 120
NUM_CELLS = 289
BOARD_SIZE = 17
NUM_SEATS = 4
NUM_OBS_CHANNELS = 317
NUM_GLOBAL_DIMS = 28
FLAT_ACTION_SPACE = 16641
NUM_TRACKED_TYPES = 12
SLOTS_PER_PIECE = 80
COMPACT_ACTION_SPACE = NUM_PIECES * SLOTS_PER_PIECE
MAX_ACTIONS_PER_ENV = 512

_device = 0
_pool: torch.Tensor | None = None
_zobrist_show = None


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def get_gpu_count() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def set_device(device_id: int) -> None:
    global _device
    _device = int(device_id)
    torch.cuda.set_device(_device)


def init_tables() -> None:
    ensure_device(_device)


def cleanup_tables() -> None:
    pass


def upload_zobrist_tables(piece, turn, move_counter, mslc, winner, terminated, draw, seat_dead, seat_flag) -> None:
    """bindings.cpp:485-517.  The show-mode table is not part of the reference
    upload; the one matching junqi_core/_zobrist.py is generated here."""
    ensure_device(_device)
    z = tables.zobrist_tables()
    arrs = [np.ascontiguousarray(a, dtype=np.int64) for a in (piece, turn, move_counter, mslc, winner,
                                                               seat_dead, seat_flag)]
    sizes = [120 * 14 * 289, 4, 4096, 512, 3, 4, 4]
    for a, s in zip(arrs, sizes):
        if a.size != s:
            raise RuntimeError(f"upload_zobrist_tables: expected {s} entries, got {a.size}")
    N.check(N.lib().jq_upload_zobrist(arrs[0].ctypes.data, arrs[1].ctypes.data, arrs[2].ctypes.data,
                                      arrs[3].ctypes.data, arrs[4].ctypes.data, int(terminated), int(draw),
                                      arrs[5].ctypes.data, arrs[6].ctypes.data, z["show_mode"].ctypes.data),
            "jq_upload_zobrist")


def upload_compact_cell_maps(flat_to_compact, compact_to_flat) -> None:
    """Accepted for compatibility; the kernels build the same maps themselves."""
    f2c = np.asarray(flat_to_compact).reshape(-1)
    c2f = np.asarray(compact_to_flat).reshape(-1)
    if f2c.size != 289 or c2f.size != 129:
        raise RuntimeError("upload_compact_cell_maps: expected (289,) and (129,)")


def upload_reset_tables(pos_x, pos_y, piece_seat, camp_slot) -> None:
    for a, s, nm in ((pos_x, 120, "pos_x"), (pos_y, 120, "pos_y"), (piece_seat, 120, "piece_seat"),
                     (camp_slot, 30, "camp_slot")):
        if np.asarray(a).size != s:
            raise RuntimeError(f"upload_reset_tables: {nm} must have {s} entries")


def upload_setup_pool(piece_types) -> None:
    global _pool
    pool = np.ascontiguousarray(piece_types, dtype=np.int8)
    if pool.ndim != 2 or pool.shape[1] != 120:
        raise RuntimeError("upload_setup_pool: piece_types must be (pool_size, 120) int8")
    tables.validate_pool(pool)
    ensure_device(_device)
    _pool = torch.from_numpy(pool).to(f"cuda:{_device}")
    N.check(N.lib().jq_set_setup_pool(_pool.data_ptr(), int(pool.shape[0])), "jq_set_setup_pool")


def upload_belief_prior_table(prior) -> None:
    global _cell_prior
    p = np.ascontiguousarray(prior, dtype=np.float32).reshape(-1)
    if p.size != 360:
        raise RuntimeError("upload_belief_prior_table: expected 360 floats")
    _cell_prior = torch.from_numpy(p.copy()).to(f"cuda:{_device}")
    # the host tables stay referenced until the upload returns: a pointer
    # taken from a temporary array would point at freed (and reused) memory
    uni, rec = tables.uniform12(), tables.recency_lut()
    N.check(N.lib().jq_upload_obs_tables(p.ctypes.data, uni.ctypes.data, rec.ctypes.data), "jq_upload_obs_tables")


def upload_seat_strongholds(strongholds) -> None:
    global _cell_strongholds
    if np.asarray(strongholds).size != 8:
        raise RuntimeError("upload_seat_strongholds: expected 8 entries")
    _cell_strongholds = torch.from_numpy(np.ascontiguousarray(strongholds, dtype=np.int16).reshape(8).copy()).to(
        f"cuda:{_device}")


# Per-cell float beliefs of the reference's GPU rollout (belief.cu), opt-in.
# By default the belief calls below are no-ops and observations use the
# beliefs the step maintains with the CPU BeliefTensor rules; after
# use_reference_gpu_beliefs(True) they run the reference GPU kernels' rules
# (jq_cell_beliefs_*) on a resident (N, 4, 12, 289) tensor that
# build_observation_batch_resident then reads, as the reference does.
_cell_mode = False
_cell_prior: torch.Tensor | None = None
_cell_strongholds: torch.Tensor | None = None
_cell_prev_dead: torch.Tensor | None = None
_cell_prev_term: torch.Tensor | None = None


def use_reference_gpu_beliefs(enabled: bool = True) -> None:
    """Select the reference GPU rollout's per-cell belief rules for the
    init / snapshot / update belief calls (default: off).  Switching the
    mode off drops the resident per-cell tensor, so later observations use
    the library's own beliefs again rather than a tensor no step updates."""
    global _cell_mode, _beliefs, _cell_prev_dead, _cell_prev_term
    if _cell_mode and not enabled:
        _beliefs = None
        _cell_prev_dead = _cell_prev_term = None
    _cell_mode = bool(enabled)


_beliefs: torch.Tensor | None = None  # uploaded per-cell beliefs (N, 4, 12, 289) float32
_observer_seats: torch.Tensor | None = None


def upload_beliefs(num_envs: int, beliefs) -> None:
    """bindings.cpp:1136-1149: per-cell beliefs [env][observer][type][world cell]."""
    global _beliefs
    if torch.is_tensor(beliefs):
        t = beliefs.detach().to(device=f"cuda:{_device}", dtype=torch.float32)
    else:
        t = torch.from_numpy(np.ascontiguousarray(beliefs, dtype=np.float32)).to(f"cuda:{_device}")
    if t.numel() != num_envs * 4 * 12 * 289:
        raise RuntimeError("beliefs: expected (N, 4, 12, 289) float32")
    _beliefs = t.reshape(num_envs, 4, 12, 289).contiguous()


def upload_observer_seats(num_envs: int, observer_seats) -> None:
    global _observer_seats
    a = np.ascontiguousarray(observer_seats, dtype=np.int8)
    if a.size != num_envs * 4:
        raise RuntimeError("observer_seats: expected (N, 4) int8")
    _observer_seats = torch.from_numpy(a.reshape(-1)).to(f"cuda:{_device}")


def gpu_scratch_reset() -> None:
    """Forget uploaded beliefs, observer seats and belief snapshots, and
    leave the reference per-cell belief mode."""
    global _beliefs, _observer_seats, _cell_prev_dead, _cell_prev_term, _cell_mode
    _beliefs = None
    _observer_seats = None
    _cell_prev_dead = _cell_prev_term = None
    _cell_mode = False


def device_synchronize() -> None:
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# State
# ---------------------------------------------------------------------------
_REF_TO_MINE = [
    ("piece_seat_arr", "piece_seat"), ("piece_type_arr", "piece_type"), ("alive", "alive"), ("pos_x", "pos_x"),
    ("pos_y", "pos_y"), ("zero_x", "zero_x"), ("zero_y", "zero_y"), ("move_count_arr", "move_count"),
    ("active_eat_arr", "active_eat"), ("passive_surv_arr", "passive_surv"), ("death_reason_arr", "death_reason"),
    ("death_step_arr", "death_step"), ("death_loc_flat_arr", "death_loc"), ("cell_piece_id", "cell_pid"),
    ("seat_dead_arr", "seat_dead"), ("seat_flag_revealed_arr", "seat_flag"), ("turn", "turn"),
    ("zobrist", "zobrist"), ("move_counter", "move_counter"), ("moves_since_last_combat", "mslc"),
]
_CM_REF = [("direct_lo", "cm_direct_lo"), ("direct_hi", "cm_direct_hi"), ("direct_type", "cm_direct_type"),
           ("last_direct_step", "cm_last_direct_step"), ("direct_other_count", "cm_direct_other"),
           ("chain_lo", "cm_chain_lo"), ("chain_hi", "cm_chain_hi"), ("chain_type", "cm_chain_type"),
           ("last_chain_step", "cm_last_chain_step"), ("eaten_by_pid_lo", "cm_eaten_lo"),
           ("eaten_by_pid_hi", "cm_eaten_hi"), ("rank_floor", "cm_rank_floor"),
           ("rank_floor_step", "cm_rank_floor_step"), ("is_gongb", "cm_is_gongb"), ("not_gongb", "cm_not_gongb"),
           ("attacked_by_known_gongb", "cm_atk_gongb")]


class DeviceGameStateBatch:
    """junqi_cuda.h:48-111; bindings.cpp:519-679."""

    def __init__(self, num_envs: int, max_num_moves: int = 4000, show_mode: int = 2,
                 rules: int = N.RULES_BATCHED):
        if num_envs <= 0 or num_envs > NUM_ENVS_MAX:
            raise RuntimeError(f"num_envs must be in [1, {NUM_ENVS_MAX}]")
        if max_num_moves <= 0:
            raise RuntimeError("max_num_moves must be positive")
        ensure_device(_device)
        self.num_envs = int(num_envs)
        self.show_mode = int(show_mode)
        # the rules draw at move 4000 by themselves; a shorter cap ends games as draws earlier
        self.b = DeviceBatch(self.num_envs, f"cuda:{_device}", rules=rules,
                             max_moves=0 if max_num_moves >= 4000 else int(max_num_moves))
        n, dev = self.num_envs, self.b.device
        self._out = {k: torch.zeros(n, dtype=dt, device=dev) for k, dt in
                     (("valid", torch.uint8), ("event", torch.int8), ("terminated", torch.uint8),
                      ("winner", torch.int8), ("draw", torch.uint8), ("flag_captured", torch.uint8),
                      ("reward", torch.float32), ("world_action", torch.int32), ("zobrist", torch.int64))}
        self._out_s = N.JqStepOut(**{k: v.data_ptr() for k, v in self._out.items()})
        self._counts = torch.zeros(n, dtype=torch.int32, device=dev)
        self._ids = torch.zeros((n, MAX_ACTIONS_PER_ENV), dtype=torch.int32, device=dev)
        self._mask = torch.zeros((n, FLAT_ACTION_SPACE), dtype=torch.uint8, device=dev)
        self._offsets = torch.zeros(n + 1, dtype=torch.int32, device=dev)
        self._values = torch.zeros(n * MAX_ACTIONS_PER_ENV, dtype=torch.int32, device=dev)
        self._csr_scratch = torch.zeros(max(1, N.lib().jq_csr_scratch_ints(n)), dtype=torch.int32, device=dev)
        self._reset_calls = 0

    @property
    def struct(self):
        return self.b.struct

    # ---- pointers (bindings.cpp:526-565) ----
    d_turn_ptr = property(lambda s: s.b["turn"].data_ptr())
    d_terminated_ptr = property(lambda s: s.b["terminated"].data_ptr())
    d_winner_team_ptr = property(lambda s: s.b["winner"].data_ptr())
    d_draw_ptr = property(lambda s: s.b["draw"].data_ptr())
    d_piece_seat_arr_ptr = property(lambda s: s.b["piece_seat"].data_ptr())
    d_piece_type_arr_ptr = property(lambda s: s.b["piece_type"].data_ptr())
    d_alive_ptr = property(lambda s: s.b["alive"].data_ptr())
    d_pos_x_ptr = property(lambda s: s.b["pos_x"].data_ptr())
    d_pos_y_ptr = property(lambda s: s.b["pos_y"].data_ptr())
    d_cell_piece_id_ptr = property(lambda s: s.b["cell_pid"].data_ptr())

    # ---- host <-> device ----
    def copy_from_host(self, arrays: dict) -> None:
        """bindings.cpp:73-110.  Beliefs are re-initialised from the uploaded
        position (BeliefTensor.initial) and the move history is cleared."""
        mine = {}
        for ref, m in _REF_TO_MINE:
            if ref not in arrays:
                raise RuntimeError(f"copy_from_host: missing {ref}")
            mine[m] = np.asarray(arrays[ref])
        self.b.load(mine)
        N.check(N.lib().jq_init_beliefs(ctypes.byref(self.b.struct), self.show_mode, _stream()), "jq_init_beliefs")

    def copy_from_host_legal_lite(self, piece_seat_arr, piece_type_arr, alive, pos_x, pos_y, cell_piece_id) -> None:
        self.b.load({"piece_seat": piece_seat_arr, "piece_type": piece_type_arr, "alive": alive, "pos_x": pos_x,
                     "pos_y": pos_y, "cell_pid": cell_piece_id})

    def copy_to_host(self) -> dict:
        h = self.b.to_host()
        out = {ref: h[m].reshape(-1) for ref, m in _REF_TO_MINE}
        alive = h["alive"].astype(bool)
        out["alive"] = alive.reshape(-1)
        out["seat_dead_arr"] = h["seat_dead"].astype(bool).reshape(-1)
        out["seat_flag_revealed_arr"] = h["seat_flag"].astype(bool).reshape(-1)
        out["cell_piece_id_per_piece"] = np.where(
            alive, h["pos_y"].astype(np.int16) * 17 + h["pos_x"].astype(np.int16), -1).astype(np.int16).reshape(-1)
        return out

    def copy_turn_to_host(self) -> np.ndarray:
        return self.b["turn"].cpu().numpy().copy()

    def copy_termination_from_host(self, terminated, winner_team, draw) -> None:
        n = self.num_envs
        for a, nm in ((terminated, "terminated"), (winner_team, "winner_team"), (draw, "draw")):
            if np.asarray(a).size != n:
                raise RuntimeError(f"{nm} size mismatch")
        self.b.load({"terminated": np.asarray(terminated, bool), "winner": np.asarray(winner_team, np.int8),
                     "draw": np.asarray(draw, bool)})

    def copy_termination_to_host(self) -> dict:
        h = self.b.to_host(["terminated", "winner", "draw"])
        return {"terminated": h["terminated"].astype(bool), "winner_team": h["winner"],
                "draw": h["draw"].astype(bool)}

    def cm_copy_from_host(self, *arrays) -> None:
        if len(arrays) != 16:
            raise RuntimeError("cm_copy_from_host: expected 16 arrays")
        cm_n = self.num_envs * 4 * 120
        d = {}
        for (ref, m), a in zip(_CM_REF, arrays):
            a = np.asarray(a)
            if a.size != cm_n:
                raise RuntimeError(f"cm size mismatch: {ref}")
            d[m] = a
        self.b.load(d)

    def cm_copy_to_host(self) -> dict:
        h = self.b.to_host([m for _, m in _CM_REF])
        out = {ref: h[m].reshape(-1) for ref, m in _CM_REF}
        for k in ("is_gongb", "not_gongb", "attacked_by_known_gongb"):
            out[k] = out[k].astype(bool)
        return out

    # ---- step (bindings.cpp:385-438) ----
    def step_batch(self, action_ids) -> dict:
        a = np.ascontiguousarray(action_ids, dtype=np.int32)
        if a.size != self.num_envs:
            raise RuntimeError("action_ids size must equal num_envs")
        d = torch.from_numpy(a).to(self.b.device)
        N.check(N.lib().jq_step(ctypes.byref(self.b.struct), d.data_ptr(), self.show_mode,
                                ctypes.byref(self._out_s), _stream()), "jq_step")
        o = {k: v.cpu().numpy() for k, v in self._out.items()}
        return {"valid": o["valid"].astype(bool), "event": o["event"], "terminated": o["terminated"].astype(bool),
                "winner_team": o["winner"], "draw": o["draw"].astype(bool),
                "flag_captured": o["flag_captured"].astype(bool)}

    # ---- helpers used by the module functions ----
    def _legal(self, seats_ptr, mask: bool):
        N.check(N.lib().jq_legal(ctypes.byref(self.b.struct), seats_ptr, self._counts.data_ptr(),
                                 self._ids.data_ptr(), MAX_ACTIONS_PER_ENV,
                                 self._mask.data_ptr() if mask else None, _stream()), "jq_legal")


class DeviceObservationBatch:
    """(N, 4, 317, 17, 17) + (N, 4, 28) float32 (junqi_cuda.h obs buffers)."""

    def __init__(self, num_envs: int):
        ensure_device(_device)
        self.num_envs = int(num_envs)
        dev = f"cuda:{_device}"
        self.spatial = torch.zeros((num_envs, 4, NUM_OBS_CHANNELS, 17, 17), dtype=torch.float32, device=dev)
        self.global_ = torch.zeros((num_envs, 4, NUM_GLOBAL_DIMS), dtype=torch.float32, device=dev)

    d_spatial_ptr = property(lambda s: s.spatial.data_ptr())
    d_global_ptr = property(lambda s: s.global_.data_ptr())

    def copy_to_host(self):
        return self.spatial.cpu().numpy(), self.global_.cpu().numpy()


class DeviceObservationSingleBatch:
    def __init__(self, num_envs: int):
        ensure_device(_device)
        self.num_envs = int(num_envs)
        dev = f"cuda:{_device}"
        self.spatial = torch.zeros((num_envs, NUM_OBS_CHANNELS, 17, 17), dtype=torch.float32, device=dev)
        self.global_ = torch.zeros((num_envs, NUM_GLOBAL_DIMS), dtype=torch.float32, device=dev)

    d_spatial_ptr = property(lambda s: s.spatial.data_ptr())
    d_global_ptr = property(lambda s: s.global_.data_ptr())

    def copy_to_host(self):
        return self.spatial.cpu().numpy(), self.global_.cpu().numpy()


def _seats_dev(state: DeviceGameStateBatch, acting_seats) -> torch.Tensor:
    a = np.ascontiguousarray(acting_seats, dtype=np.int8)
    if a.size != state.num_envs:
        raise RuntimeError(f"acting_seats: expected {state.num_envs} elements, got {a.size}")
    return torch.from_numpy(a).to(state.b.device)


def legal_action_ids_batch(state: DeviceGameStateBatch, acting_seats):
    """bindings.cpp:831-890 -> (ids (N, 512) int32, counts (N,) int32)."""
    s = _seats_dev(state, acting_seats)
    state._legal(s.data_ptr(), mask=False)
    return state._ids.cpu().numpy(), state._counts.cpu().numpy()


def legal_action_ids_batch_csr(state: DeviceGameStateBatch, acting_seats):
    """bindings.cpp:892-950 -> (offsets (N+1,), values (sum,))."""
    s = _seats_dev(state, acting_seats)
    state._legal(s.data_ptr(), mask=False)
    N.check(N.lib().jq_csr(state.num_envs, state._counts.data_ptr(), state._ids.data_ptr(), MAX_ACTIONS_PER_ENV,
                           state._offsets.data_ptr(), state._values.data_ptr(), state._csr_scratch.data_ptr(),
                           _stream()), "jq_csr")
    off = state._offsets.cpu().numpy()
    return off, state._values[: int(off[-1])].cpu().numpy()


def legal_action_mask_batch(state: DeviceGameStateBatch, acting_seats) -> np.ndarray:
    """bindings.cpp:951-1000: per-piece 80-slot mask, (N, 120, 80) bool on the host."""
    s = _seats_dev(state, acting_seats)
    out = torch.empty((state.num_envs, NUM_PIECES, SLOTS_PER_PIECE), dtype=torch.uint8, device=state.b.device)
    N.check(N.lib().jq_legal_slots(ctypes.byref(state.struct), s.data_ptr(), out.data_ptr(), _stream()),
            "jq_legal_slots")
    return out.cpu().numpy().astype(bool)


def legal_mask_canonical_batch(state: DeviceGameStateBatch, acting_seats) -> int:
    """bindings.cpp:1004-1027: device pointer to an (N, 16641) bool mask."""
    s = _seats_dev(state, acting_seats)
    state._legal(s.data_ptr(), mask=True)
    return state._mask.data_ptr()


def legal_mask_canonical_batch_from_device(state: DeviceGameStateBatch, d_acting_seats_ptr: int) -> int:
    state._legal(d_acting_seats_ptr, mask=True)
    return state._mask.data_ptr()


def step_device(state: DeviceGameStateBatch, d_canonical_actions_ptr: int, d_acting_seats_ptr: int) -> dict:
    """bindings.cpp:1044-1074: rotate + step + reward (+ history and beliefs)."""
    N.check(N.lib().jq_step_canonical(ctypes.byref(state.b.struct), d_canonical_actions_ptr, d_acting_seats_ptr,
                                      state.show_mode, ctypes.byref(state._out_s), _stream()), "jq_step_canonical")
    o = state._out
    return {"d_valid_ptr": o["valid"].data_ptr(), "d_event_ptr": o["event"].data_ptr(),
            "d_terminated_ptr": o["terminated"].data_ptr(), "d_winner_team_ptr": o["winner"].data_ptr(),
            "d_draw_ptr": o["draw"].data_ptr(), "d_flag_captured_ptr": o["flag_captured"].data_ptr(),
            "d_rewards_ptr": o["reward"].data_ptr(), "d_world_actions_ptr": o["world_action"].data_ptr(),
            "N": state.num_envs}


def record_move_history(state, d_world_actions_ptr, d_valid_ptr) -> None:
    """The move history is recorded inside the step."""


def _cell_ready(state, what: str) -> None:
    if _cell_prior is None or _cell_strongholds is None:
        raise RuntimeError(f"{what}: call upload_belief_prior_table and upload_seat_strongholds first")
    if _beliefs is None or _beliefs.shape[0] != state.num_envs:
        raise RuntimeError(f"{what}: call init_all_beliefs first")


def snapshot_pre_step_flags(state) -> None:
    """bindings.cpp:1272-1278.  Default mode: nothing to do (the step updates
    its own beliefs); reference GPU beliefs: seat_dead and terminated now."""
    global _cell_prev_dead, _cell_prev_term
    if not _cell_mode:
        return
    n = state.num_envs
    if _cell_prev_dead is None or _cell_prev_dead.shape[0] != n:
        _cell_prev_dead = torch.zeros((n, 4), dtype=torch.uint8, device=f"cuda:{_device}")
        _cell_prev_term = torch.zeros(n, dtype=torch.uint8, device=f"cuda:{_device}")
    N.check(N.lib().jq_cell_beliefs_snapshot(ctypes.byref(state.b.struct), _cell_prev_dead.data_ptr(),
                                             _cell_prev_term.data_ptr(), _stream()), "jq_cell_beliefs_snapshot")


def update_beliefs_after_step(state, d_event_ptr=0, d_flag_captured_ptr=0, d_world_actions_ptr=0) -> None:
    """bindings.cpp:1280-1300.  Default mode: beliefs were updated inside the
    step with the BeliefTensor rules; reference GPU beliefs: belief.cu's
    update from the step's event / flag capture / world action."""
    if not _cell_mode:
        return
    _cell_ready(state, "update_beliefs_after_step")
    if _cell_prev_dead is None or _cell_prev_dead.shape[0] != state.num_envs:
        raise RuntimeError("update_beliefs_after_step: call snapshot_pre_step_flags first")
    N.check(N.lib().jq_cell_beliefs_update(ctypes.byref(state.b.struct), int(d_event_ptr), int(d_flag_captured_ptr),
                                           int(d_world_actions_ptr), _cell_prev_dead.data_ptr(),
                                           _cell_strongholds.data_ptr(), _beliefs.data_ptr(), _stream()),
            "jq_cell_beliefs_update")


def init_beliefs_for_reset_envs(state) -> None:
    """bindings.cpp:1252-1260.  Default mode: resets initialise beliefs
    themselves; reference GPU beliefs: re-seed the envs the last snapshot
    saw terminated."""
    if not _cell_mode:
        return
    _cell_ready(state, "init_beliefs_for_reset_envs")
    if _cell_prev_term is None or _cell_prev_term.shape[0] != state.num_envs:
        raise RuntimeError("init_beliefs_for_reset_envs: call snapshot_pre_step_flags first")
    N.check(N.lib().jq_cell_beliefs_init(ctypes.byref(state.b.struct), _cell_prev_term.data_ptr(),
                                         _cell_prior.data_ptr(), _beliefs.data_ptr(), _stream()),
            "jq_cell_beliefs_init")


def init_all_beliefs(state: DeviceGameStateBatch) -> None:
    """bindings.cpp:1262-1270.  Default mode: prior beliefs for every env, and
    observations use the library's beliefs again; reference GPU beliefs: a
    resident per-cell tensor seeded for every env."""
    global _beliefs
    _beliefs = None
    N.check(N.lib().jq_init_beliefs(ctypes.byref(state.b.struct), state.show_mode, _stream()), "jq_init_beliefs")
    if _cell_mode:
        if _cell_prior is None:
            raise RuntimeError("init_all_beliefs: call upload_belief_prior_table first")
        _beliefs = torch.zeros((state.num_envs, 4, 12, 289), dtype=torch.float32, device=f"cuda:{_device}")
        N.check(N.lib().jq_cell_beliefs_init(ctypes.byref(state.b.struct), None, _cell_prior.data_ptr(),
                                             _beliefs.data_ptr(), _stream()), "jq_cell_beliefs_init")


def reset_terminated_envs(state: DeviceGameStateBatch, seed: int) -> None:
    """bindings.cpp:1224-1232."""
    if _pool is None:
        raise RuntimeError("reset_terminated_envs: call upload_setup_pool first")
    state._reset_calls += 1
    N.check(N.lib().jq_reset(ctypes.byref(state.b.struct), int(seed) & (2**64 - 1), state._reset_calls, 0,
                             state.show_mode, _stream()), "jq_reset")


def _observe(state, observers_ptr, seats, show_mode, sp_ptr, gl_ptr):
    if _beliefs is None:
        N.check(N.lib().jq_observe(ctypes.byref(state.b.struct), observers_ptr, seats, int(show_mode), sp_ptr,
                                   gl_ptr, _stream()), "jq_observe")
        return
    if _beliefs.shape[0] != state.num_envs:
        raise RuntimeError(f"uploaded beliefs are for {_beliefs.shape[0]} envs, the state has {state.num_envs}; "
                           "upload matching beliefs or call init_all_beliefs / gpu_scratch_reset")
    N.check(N.lib().jq_observe_beliefs(ctypes.byref(state.b.struct), observers_ptr, seats, int(show_mode),
                                       _beliefs.data_ptr(), sp_ptr, gl_ptr, _stream()), "jq_observe_beliefs")


def build_observation_batch(state, beliefs, observer_seats, obs_out: DeviceObservationBatch, show_mode=2) -> None:
    """bindings.cpp:1091-1134: observations of the given observers from the given per-cell beliefs."""
    upload_beliefs(state.num_envs, beliefs)
    upload_observer_seats(state.num_envs, observer_seats)
    _observe(state, _observer_seats.data_ptr(), 4, show_mode, obs_out.d_spatial_ptr, obs_out.d_global_ptr)


def build_observation_batch_resident(state, obs_out: DeviceObservationBatch, show_mode=2) -> None:
    obs_ptr = _observer_seats.data_ptr() if _observer_seats is not None else None
    _observe(state, obs_ptr, 4, show_mode, obs_out.d_spatial_ptr, obs_out.d_global_ptr)


def build_observation_single_seat(state, obs_out: DeviceObservationSingleBatch, d_acting_seats_ptr: int,
                                  show_mode=2) -> None:
    _observe(state, d_acting_seats_ptr, 1, show_mode, obs_out.d_spatial_ptr, obs_out.d_global_ptr)


# ---------------------------------------------------------------------------
# Rollout history (junqi_cuda.h:186-277, bindings.cpp:728-800)
# ---------------------------------------------------------------------------
class DeviceRolloutHistory:
    """Compact device history that rebuilds PPO minibatches on the device.

    Each record holds what the recorded seat's observation and legal mask
    read: 12,000 bytes (the reference's record, float beliefs plus all four
    observers' combat memory, is 47,243 B: rollout_storage.py:48-52).  The
    observer of a rebuilt record is the seat recorded by ``snapshot``;
    ``reconstruct``'s acting seats are accepted for compatibility."""

    def __init__(self, num_steps: int, num_envs: int):
        from .history import RolloutHistory
        self._h = RolloutHistory(num_steps, num_envs, _device)
        self.num_steps, self.num_envs = int(num_steps), int(num_envs)
        self.history_bytes = self._h.history_bytes
        self.replay_capacity = 0

    def snapshot(self, state: DeviceGameStateBatch, d_acting_seats_ptr: int, step: int) -> None:
        seats = None
        if d_acting_seats_ptr:
            seats = _device_view(d_acting_seats_ptr, state.num_envs, torch.int8, state.b.device)
        self._h.snapshot(state.b, step, seats)

    def reconstruct(self, d_flat_indices_ptr: int, d_acting_seats_ptr: int, batch_size: int,
                    show_mode: int = 2) -> dict:
        idx = _device_view(d_flat_indices_ptr, batch_size, torch.int64, self._h.device).clone()
        out = self._h.reconstruct(idx, show_mode)
        self.replay_capacity = max(self.replay_capacity, self._h._cap)
        return {"d_spatial_ptr": out["spatial"].data_ptr(), "d_global_ptr": out["global"].data_ptr(),
                "d_legal_mask_ptr": out["mask"].data_ptr(), "batch_size": int(batch_size)}


def _device_view(ptr: int, shape, dtype: torch.dtype, device) -> torch.Tensor:
    """A tensor over caller-owned device memory at `ptr` (no copy)."""
    shape = (int(shape),) if isinstance(shape, (int, np.integer)) else tuple(int(d) for d in shape)
    typestr = {torch.int8: "|i1", torch.uint8: "|u1", torch.bool: "|b1", torch.int32: "<i4", torch.int64: "<i8",
               torch.float32: "<f4"}[dtype]

    class _Arr:
        __cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (int(ptr), False), "version": 3,
                                    "strides": None}
    return torch.as_tensor(_Arr(), device=device)
