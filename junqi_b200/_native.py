"""ctypes binding of ``libjq.so`` (the C ABI declared in ``include/jq.h``).

The library is built in-tree (``junqi_b200/libjq.so``) by ``build()``.  There
is no fallback: if the library is missing or a call returns a non-zero
status, a ``RuntimeError`` carrying ``jq_last_error()`` is raised.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libjq.so"
TRACE_LIB_PATH = _PKG / "libjq_trace.so"  # the same library with kernel timestamps (make -C csrc trace)
CSRC = _PKG / "csrc"

JQ_OK = 0
STATUS_NAMES = {1: "JQ_ERR_ARG", 2: "JQ_ERR_CUDA", 3: "JQ_ERR_NOT_READY", 4: "JQ_ERR_CAPACITY"}

# jq_batch field order (include/jq.h); (name, ctypes element type)
BATCH_FIELDS = [
    ("alive", ctypes.c_uint8), ("piece_type", ctypes.c_int8), ("piece_seat", ctypes.c_int8),
    ("pos_x", ctypes.c_int8), ("pos_y", ctypes.c_int8), ("zero_x", ctypes.c_int8),
    ("zero_y", ctypes.c_int8), ("move_count", ctypes.c_int16), ("active_eat", ctypes.c_int16),
    ("passive_surv", ctypes.c_int16), ("death_reason", ctypes.c_int8),
    ("death_step", ctypes.c_int16), ("death_loc", ctypes.c_int16), ("cell_pid", ctypes.c_int16),
    ("seat_dead", ctypes.c_uint8), ("seat_flag", ctypes.c_uint8), ("turn", ctypes.c_int8),
    ("zobrist", ctypes.c_int64), ("move_counter", ctypes.c_int32), ("mslc", ctypes.c_int32),
    ("terminated", ctypes.c_uint8), ("winner", ctypes.c_int8), ("draw", ctypes.c_uint8),
    ("cm_direct_lo", ctypes.c_uint64), ("cm_direct_hi", ctypes.c_uint64),
    ("cm_direct_type", ctypes.c_uint16), ("cm_last_direct_step", ctypes.c_int16),
    ("cm_direct_other", ctypes.c_int16), ("cm_chain_lo", ctypes.c_uint64),
    ("cm_chain_hi", ctypes.c_uint64), ("cm_chain_type", ctypes.c_uint16),
    ("cm_last_chain_step", ctypes.c_int16), ("cm_eaten_lo", ctypes.c_uint64),
    ("cm_eaten_hi", ctypes.c_uint64), ("cm_rank_floor", ctypes.c_int8),
    ("cm_rank_floor_step", ctypes.c_int16), ("cm_is_gongb", ctypes.c_uint8),
    ("cm_not_gongb", ctypes.c_uint8), ("cm_atk_gongb", ctypes.c_uint8),
    ("hist_src", ctypes.c_int16), ("hist_dst", ctypes.c_int16), ("hist_count", ctypes.c_int32),
    ("bel_code", ctypes.c_uint8), ("remaining", ctypes.c_int16), ("rem_tracked", ctypes.c_uint8),
]


class JqBatch(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32)] + [(n, ctypes.c_void_p) for n, _ in BATCH_FIELDS] + \
        [("rules", ctypes.c_int32), ("max_moves", ctypes.c_int32), ("pool", ctypes.c_void_p),
         ("pool_size", ctypes.c_int32)]


RULES_BATCHED, RULES_GAMESTATE = 0, 1


class JqStepOut(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("valid", "event", "terminated", "winner", "draw", "flag_captured", "reward", "world_action",
                 "zobrist")]


# exported name -> (restype, argtypes)
_vp, _i32, _i64, _u64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64
_PB = ctypes.POINTER(JqBatch)
_PO = ctypes.POINTER(JqStepOut)
SIGNATURES = {
    "jq_abi_version": (ctypes.c_int, []),
    "jq_last_error": (ctypes.c_char_p, []),
    "jq_topology_dump": (ctypes.c_int, [_vp] * 8),
    "jq_init": (ctypes.c_int, [ctypes.c_int]),
    "jq_upload_zobrist": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "jq_upload_obs_tables": (ctypes.c_int, [_vp, _vp, _vp]),
    "jq_set_setup_pool": (ctypes.c_int, [_vp, _i32]),
    "jq_pool_index": (_i32, [_u64, _u64, _i32, _i32]),
    "jq_reset": (ctypes.c_int, [_PB, _u64, _u64, _i32, _i32, _vp]),
    "jq_reset_rows": (ctypes.c_int, [_PB, _vp, _i32, _vp]),
    "jq_canonical_to_world": (ctypes.c_int, [_PB, _vp, _vp, _vp, _vp]),
    "jq_init_beliefs": (ctypes.c_int, [_PB, _i32, _vp]),
    "jq_rehash": (ctypes.c_int, [_PB, _i32, _vp]),
    "jq_legal_slots": (ctypes.c_int, [_PB, _vp, _vp, _vp]),
    "jq_history_record_bytes": (_i32, []),
    "jq_history_snapshot": (ctypes.c_int, [_PB, _vp, _vp, ctypes.c_int64, ctypes.c_int64, _vp]),
    "jq_history_restore": (ctypes.c_int, [_vp, ctypes.c_int64, _vp, _PB, _vp, _vp]),
    "jq_step": (ctypes.c_int, [_PB, _vp, _i32, _PO, _vp]),
    "jq_step_canonical": (ctypes.c_int, [_PB, _vp, _vp, _i32, _PO, _vp]),
    "jq_ply": (ctypes.c_int, [_PB, _vp, _i32, _PO, _i32, _u64, _u64, _vp, _vp, _i32, _vp, _vp, _vp]),
    "jq_legal": (ctypes.c_int, [_PB, _vp, _vp, _vp, _i32, _vp, _vp]),
    "jq_csr_scratch_ints": (_i32, [_i32]),
    "jq_csr": (ctypes.c_int, [_i32, _vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "jq_csr_noalloc": (ctypes.c_int, [_i32, _vp, _vp, _i32, _vp, _vp, _vp]),
    "jq_observe": (ctypes.c_int, [_PB, _vp, _i32, _i32, _vp, _vp, _vp]),
    "jq_observe_beliefs": (ctypes.c_int, [_PB, _vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "jq_cell_beliefs_init": (ctypes.c_int, [_PB, _vp, _vp, _vp, _vp]),
    "jq_cell_beliefs_snapshot": (ctypes.c_int, [_PB, _vp, _vp, _vp]),
    "jq_cell_beliefs_update": (ctypes.c_int, [_PB, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "jq_sample_uniform": (ctypes.c_int, [_i32, _vp, _vp, _i32, _u64, _u64, _vp, _vp]),
    "jq_sample_softmax": (ctypes.c_int, [_PB, _vp, _vp, _i32, _u64, _u64, _vp, _vp, _vp]),
    "jq_trace_read": (ctypes.c_int, [_i32, _vp, _i32]),
}


def build(force: bool = False, trace: bool = False) -> Path:
    """Compile libjq.so (or, with ``trace``, libjq_trace.so) for sm_100a with
    nvcc (csrc/Makefile)."""
    path = TRACE_LIB_PATH if trace else LIB_PATH
    srcs = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + \
        [_PKG.parent / "include" / "jq.h"]
    stale = not path.exists() or any(p.stat().st_mtime > path.stat().st_mtime for p in srcs)
    if force or stale:
        subprocess.run(["make", "-s", "-C", str(CSRC)] + (["trace"] if trace else []), check=True)
    return path


_lib = None
_lib_path = LIB_PATH


def use_trace_library() -> None:
    """Load libjq_trace.so instead of libjq.so (before the first call into
    the library): the same kernels plus per-CTA timestamps (jq_trace_read)."""
    global _lib_path
    if _lib is not None and _lib_path != TRACE_LIB_PATH:
        raise RuntimeError("libjq.so is already loaded in this process")
    _lib_path = TRACE_LIB_PATH


def lib():
    """Load libjq.so (raising if it is absent) and declare every signature."""
    global _lib
    if _lib is None:
        if not _lib_path.exists():
            raise RuntimeError(f"{_lib_path.name} not built at {_lib_path}; run junqi_b200._native.build()")
        L = ctypes.CDLL(str(_lib_path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != JQ_OK:
        err = lib().jq_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed: {STATUS_NAMES.get(status, status)}: {err}")


def call(name: str, *args):
    """Call an int-status entry point and raise on failure."""
    st = getattr(lib(), name)(*args)
    check(st, name)
    return st
