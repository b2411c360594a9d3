"""Replay harness for the reference golden trajectories (tests/golden/ref_*).

A driver adapts an implementation (the CPU oracle, or the CUDA batch through
the C-ABI) to five calls:

    load(init: dict[str, ndarray], show_mode, rules)   # oracle field names
    legal() -> (offsets, values)                 # CSR for the current turns
    masks() -> (N, 16641) bool                   # canonical masks, current turns
    step(actions) -> dict                        # MoveResultBatch arrays
    state() -> dict[str, ndarray]                # oracle field names
    obs(env, observer) -> (spatial, global)

``replay`` walks a fixture ply by ply and asserts bit-equality of every
recorded artefact: CSR, canonical masks, Zobrist, MoveResult, combat memory,
observation digests and the final SoA state.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
# batched trajectories (BatchedGameState.step_batch) and GameState trajectories
# (GameState.step, the single-env rules); the latter carry ``rules == 1``
TRAJECTORIES = ("cfg1", "combat_dark", "long_bright", "late_game", "gs_uniform", "gs_combat_dark", "gs_late")

CM_ORDER = ["cm_direct_lo", "cm_direct_hi", "cm_direct_type", "cm_last_direct_step",
            "cm_direct_other", "cm_chain_lo", "cm_chain_hi", "cm_chain_type",
            "cm_last_chain_step", "cm_eaten_lo", "cm_eaten_hi", "cm_rank_floor",
            "cm_rank_floor_step", "cm_is_gongb", "cm_not_gongb", "cm_atk_gongb"]
STATE_KEYS = ["alive", "piece_type", "piece_seat", "pos_x", "pos_y", "zero_x", "zero_y",
              "move_count", "active_eat", "passive_surv", "death_reason", "death_step",
              "death_loc", "cell_pid", "seat_dead", "seat_flag", "turn", "zobrist",
              "move_counter", "mslc", "terminated", "winner", "draw"] + CM_ORDER


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load(name: str) -> dict:
    with np.load(GOLDEN / f"ref_traj_{name}.npz") as z:
        return {k: z[k] for k in z.files}


def manifest() -> dict:
    return json.loads((GOLDEN / "ref_manifest.json").read_text())


def tables() -> dict:
    with np.load(GOLDEN / "ref_tables.npz") as z:
        return {k: z[k] for k in z.files}


def init_state(fx: dict) -> dict:
    return {k[len("init_"):]: v for k, v in fx.items() if k.startswith("init_")}


def _as_u8(a):
    a = np.asarray(a)
    return a.astype(np.uint8) if a.dtype == bool else a


# every state field an observation reads, including the ones no fixture
# digest covers (belief codes, inventories, move history)
SHADOW_KEYS = STATE_KEYS + ["hist_src", "hist_dst", "hist_count", "bel_code", "remaining", "rem_tracked"]


def _obs_diff(sp, gl, osp, ogl, limit=12) -> str:
    sp = np.asarray(sp, np.float32).reshape(317, 17, 17)
    osp = np.asarray(osp, np.float32).reshape(317, 17, 17)
    d = np.argwhere(sp.view(np.uint32) != osp.view(np.uint32))
    parts = [f"ch{c} y{y} x{x}: {sp[c, y, x]!r} vs {osp[c, y, x]!r}" for c, y, x in d[:limit]]
    g = np.nonzero(np.asarray(gl, np.float32).view(np.uint32) != np.asarray(ogl, np.float32).view(np.uint32))[0]
    if g.size:
        parts.append(f"global {g[:limit].tolist()}")
    return f"{len(d)} planes floats differ; " + "; ".join(parts)


def replay(fx: dict, drv, plies: int | None = None, check_obs: bool = True,
           check_every_cm: bool = True, shadow=None) -> int:
    """Replay ``fx`` through ``drv``; returns the number of plies checked.

    ``shadow``: a second driver (the oracle) stepped in lockstep.  After every
    ply each field of SHADOW_KEYS must equal the shadow's, so a divergence in
    a field no fixture digest covers is caught at the ply it happens; an
    observation that misses its digest is reported as its differing
    (channel, cell) list against the shadow's."""
    T = fx["actions"].shape[0] if plies is None else min(plies, fx["actions"].shape[0])
    show, rules = int(fx["show_mode"]), int(fx["rules"]) if "rules" in fx else 0
    drv.load(init_state(fx), show, rules)
    if shadow is not None:
        shadow.load(init_state(fx), show, rules)
    obs_at: dict[int, list] = {}
    for (t, e, s), h in zip(fx["obs_keys"].tolist(), fx["obs_sha"].tolist()):
        obs_at.setdefault(int(t), []).append((int(e), int(s), h))

    def check_obs_at(t):
        for e, s, h in obs_at.get(t, []):
            sp, gl = drv.obs(e, s)
            if sha(np.asarray(sp, np.float32), np.asarray(gl, np.float32)) != h:
                detail = "" if shadow is None else ": " + _obs_diff(sp, gl, *shadow.obs(e, s))
                raise AssertionError(f"observation digest differs at ply {t} env {e} observer {s}{detail}")

    def check_shadow(t, got):
        exp = shadow.state()
        for k in SHADOW_KEYS:
            a, b = np.asarray(got[k]), np.asarray(exp[k])
            a = a.reshape(b.shape).astype(b.dtype)
            if not np.array_equal(a, b):
                envs = np.nonzero((a != b).reshape(b.shape[0], -1).any(1))[0]
                raise AssertionError(f"after ply {t}: state field {k} differs from the oracle in envs {envs[:8]}")

    for t in range(T):
        if check_obs:
            check_obs_at(t)
        off, val = drv.legal()
        assert sha(np.asarray(off, np.int32), np.asarray(val, np.int32)) == fx["csr_sha"][t], \
            f"legal CSR differs at ply {t}"
        assert sha(np.asarray(drv.masks(), bool)) == fx["mask_sha"][t], f"canonical mask differs at ply {t}"
        r = drv.step(fx["actions"][t])
        if shadow is not None:
            shadow.step(fx["actions"][t])
        for k, rk in (("valid", "res_valid"), ("event", "res_event"), ("terminated", "res_terminated"),
                      ("winner", "res_winner"), ("draw", "res_draw"), ("flag_captured", "res_flag")):
            got = np.asarray(r[k]).astype(np.int8)
            assert np.array_equal(got, fx[rk][t]), f"MoveResult.{k} differs at ply {t}: " \
                f"envs {np.nonzero(got != fx[rk][t])[0][:8]}"
        st = drv.state()
        bad = np.nonzero(np.asarray(st["zobrist"]) != fx["zobrist"][t])[0]
        assert bad.size == 0, f"zobrist differs at ply {t}, envs {bad[:8]}"
        if check_every_cm or t == T - 1:
            assert sha(*[_as_u8(st[k]) for k in CM_ORDER]) == fx["cm_sha"][t], f"combat memory differs at ply {t}"
        if shadow is not None:
            check_shadow(t, st)
    if check_obs and T == fx["actions"].shape[0]:
        check_obs_at(T)
    if T == fx["actions"].shape[0]:
        st = drv.state()
        for k in STATE_KEYS:
            exp = fx[f"final_{k}"]
            got = np.asarray(st[k]).reshape(exp.shape)
            assert np.array_equal(_as_u8(got), _as_u8(exp)), f"final state field {k} differs"
    return T
