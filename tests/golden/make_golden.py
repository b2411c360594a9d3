"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is importable, e.g.::

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py

Writes ``tests/golden/ref_*.npz`` and ``tests/golden/ref_manifest.json``.
Nothing here runs during the test suite; the suite only reads the files.

What is recorded (all produced by junqi_core itself):

* ``ref_tables.npz`` -- board/rail topology tables (``_movegen_tables.py``,
  ``board.py``), the per-slot belief prior (``info_model.py``), SHA-256
  digests of the ten Zobrist tables (``_zobrist.py``), and the first 64
  entries of the default setup pool (``gpu_rollout._build_setup_pool``) plus
  32 ``generate_random_setup(random.Random(s))`` lineups.
* ``ref_traj_gs_<name>.npz`` -- the same records for trajectories stepped
  with ``GameState.step`` (state.py, the single-env rules JunqiEnv uses),
  beliefs from ``BeliefTensor.update`` on those states and observations
  from ``ObservationBuilder`` -- exactly the JunqiEnv path.
* ``ref_traj_<name>.npz`` -- a batched trajectory through
  ``BatchedGameState.step_batch`` (the state contract): initial state, the
  action stream, per-ply Zobrist hashes and MoveResultBatch arrays,
  per-ply SHA-256 of the legal CSR and of the canonical masks
  (``action_lut`` rotation), per-ply SHA-256 of the 16 combat-memory arrays,
  the final SoA state, and SHA-256 digests of observations built by the
  reference ``ObservationBuilder`` with beliefs maintained by the reference
  ``BeliefTensor.update`` on GameState views of the batched states.
"""
from __future__ import annotations

import hashlib
import json
import random
import sys
from pathlib import Path

import numpy as np

from junqi_core import _movegen_tables as T
from junqi_core import _zobrist as Z
from junqi_core.batched_state import BatchedGameState
from junqi_core.board import COMPACT_TO_FLAT, FLAT_TO_COMPACT
from junqi_core.combat_memory import CombatMemoryState
from junqi_core.info_model import _INITIAL_PRIOR_TABLE, BeliefTensor
from junqi_core.move_gen import PieceRef
from junqi_core.observation import ObservationBuilder
from junqi_core.rail_topology import CURVE_ARC_CELLS, RAIL_ADJ
from junqi_core.rules import (
    DeathReason, Event, PieceType, Seat, ShowMode, siling_reveals_dst, siling_reveals_src,
)
from junqi_core.setup import generate_random_setup
from junqi_core.state import DeathInfo, GameState, MoveResult, SeatInfo
from junqi_rl.action_lut import ROTATE_LUT
from junqi_rl.gpu_rollout import _build_setup_pool

OUT = Path(__file__).resolve().parent

CM_FIELDS = [
    ("cm_direct_lo", "direct_ate_my_pid_lo"), ("cm_direct_hi", "direct_ate_my_pid_hi"),
    ("cm_direct_type", "direct_ate_my_type_mask"), ("cm_last_direct_step", "last_direct_step"),
    ("cm_direct_other_count", "direct_other_count"), ("cm_chain_lo", "chain_pid_lo"),
    ("cm_chain_hi", "chain_pid_hi"), ("cm_chain_type", "chain_ate_my_type_mask"),
    ("cm_last_chain_step", "last_chain_step"), ("cm_eaten_by_pid_lo", "eaten_by_pid_lo"),
    ("cm_eaten_by_pid_hi", "eaten_by_pid_hi"), ("cm_rank_floor", "rank_floor"),
    ("cm_rank_floor_step", "rank_floor_step"), ("cm_is_gongb", "is_gongb"),
    ("cm_not_gongb", "not_gongb"), ("cm_attacked_by_known_gongb", "attacked_by_known_gongb"),
]
# BatchedGameState field -> fixture key (fixture keys use the oracle's names)
STATE_FIELDS = [
    ("alive", "alive"), ("piece_type_arr", "piece_type"), ("piece_seat_arr", "piece_seat"),
    ("pos_x", "pos_x"), ("pos_y", "pos_y"), ("zero_x", "zero_x"), ("zero_y", "zero_y"),
    ("move_count_arr", "move_count"), ("active_eat_arr", "active_eat"),
    ("passive_surv_arr", "passive_surv"), ("death_reason_arr", "death_reason"),
    ("death_step_arr", "death_step"), ("death_loc_flat_arr", "death_loc"),
    ("cell_piece_id", "cell_pid"), ("seat_dead_arr", "seat_dead"),
    ("seat_flag_revealed_arr", "seat_flag"), ("turn", "turn"), ("zobrist", "zobrist"),
    ("move_counter", "move_counter"), ("moves_since_last_combat", "mslc"),
    ("terminated", "terminated"), ("winner_team", "winner"), ("draw", "draw"),
    ("cm_direct_lo", "cm_direct_lo"), ("cm_direct_hi", "cm_direct_hi"),
    ("cm_direct_type", "cm_direct_type"), ("cm_last_direct_step", "cm_last_direct_step"),
    ("cm_direct_other_count", "cm_direct_other"), ("cm_chain_lo", "cm_chain_lo"),
    ("cm_chain_hi", "cm_chain_hi"), ("cm_chain_type", "cm_chain_type"),
    ("cm_last_chain_step", "cm_last_chain_step"), ("cm_eaten_by_pid_lo", "cm_eaten_lo"),
    ("cm_eaten_by_pid_hi", "cm_eaten_hi"), ("cm_rank_floor", "cm_rank_floor"),
    ("cm_rank_floor_step", "cm_rank_floor_step"), ("cm_is_gongb", "cm_is_gongb"),
    ("cm_not_gongb", "cm_not_gongb"), ("cm_attacked_by_known_gongb", "cm_atk_gongb"),
]


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def state_dict(b: BatchedGameState) -> dict[str, np.ndarray]:
    return {dst: np.array(getattr(b, src), copy=True) for src, dst in STATE_FIELDS}


# ---------------------------------------------------------------------------
# GameState view of one batched env (for BeliefTensor and ObservationBuilder)
# ---------------------------------------------------------------------------

def gs_view(b: BatchedGameState, i: int, hist: list, show_mode: ShowMode) -> GameState:
    pieces = {}
    for pid in range(120):
        if b.alive[i, pid]:
            pieces[(int(b.pos_x[i, pid]), int(b.pos_y[i, pid]))] = PieceRef(
                seat=Seat(int(b.piece_seat_arr[i, pid])),
                piece_type=PieceType(int(b.piece_type_arr[i, pid])), alive=True, piece_id=pid)
    deaths = {}
    for pid in range(120):
        if not b.alive[i, pid] and int(b.death_step_arr[i, pid]) != -1:
            r = int(b.death_reason_arr[i, pid])
            deaths[pid] = DeathInfo(piece_id=pid, reason=DeathReason(r if r in (0, 1, 2) else 0),
                                    death_loc=(0, 0), step=int(b.death_step_arr[i, pid]))
    cm = CombatMemoryState(**{ref: np.array(getattr(b, mine)[i], copy=True) for mine, ref in CM_FIELDS})
    info = {Seat(s): SeatInfo(dead=bool(b.seat_dead_arr[i, s]),
                              flag_revealed=bool(b.seat_flag_revealed_arr[i, s])) for s in range(4)}
    w = int(b.winner_team[i])
    return GameState(
        pieces=pieces, turn=Seat(int(b.turn[i])), move_counter=int(b.move_counter[i]),
        moves_since_last_combat=int(b.moves_since_last_combat[i]), info=info,
        terminated=bool(b.terminated[i]), winner_team=None if w < 0 else w, draw=bool(b.draw[i]),
        show_mode=show_mode, deaths=deaths, combat_memory=cm,
        alive=b.alive[i].copy(), piece_type_arr=b.piece_type_arr[i].copy(),
        piece_seat_arr=b.piece_seat_arr[i].copy(), pos_x=b.pos_x[i].copy(), pos_y=b.pos_y[i].copy(),
        zero_x=b.zero_x[i].copy(), zero_y=b.zero_y[i].copy(),
        move_count_arr=b.move_count_arr[i].copy(), active_eat_arr=b.active_eat_arr[i].copy(),
        passive_surv_arr=b.passive_surv_arr[i].copy(), death_reason_arr=b.death_reason_arr[i].copy(),
        death_step_arr=b.death_step_arr[i].copy(), death_loc_flat_arr=b.death_loc_flat_arr[i].copy(),
        cell_piece_id=b.cell_piece_id[i].copy(), seat_dead_arr=b.seat_dead_arr[i].copy(),
        seat_flag_revealed_arr=b.seat_flag_revealed_arr[i].copy(),
        move_history=list(hist), zobrist=int(b.zobrist[i]),
    )


def canonical_mask(ids: np.ndarray, seat: int) -> np.ndarray:
    """action_lut.build_legal_mask_batch restated per env via ROTATE_LUT."""
    m = np.zeros(129 * 129, dtype=bool)
    if ids.size:
        sf, df = ids // 289, ids % 289
        world_compact = FLAT_TO_COMPACT[sf].astype(np.int64) * 129 + FLAT_TO_COMPACT[df]
        m[ROTATE_LUT[seat][world_compact]] = True
    return m


# ---------------------------------------------------------------------------
# Trajectory recorder
# ---------------------------------------------------------------------------

def record(name: str, b: BatchedGameState, plies: int, policy, show_mode: ShowMode,
           obs_plies: tuple[int, ...], obs_envs: int, full_obs: tuple = ()) -> dict:
    N = b.num_envs
    init = state_dict(b)
    hists = [[] for _ in range(N)]
    beliefs = [[BeliefTensor.initial(gs_view(b, i, [], show_mode), Seat(s)) for s in range(4)]
               for i in range(N)]
    builder = ObservationBuilder()
    sp = np.zeros((317, 17, 17), np.float32)
    gl = np.zeros(28, np.float32)
    acts_all = np.zeros((plies, N), np.int32)
    zob = np.zeros((plies, N), np.int64)
    res = {k: np.zeros((plies, N), np.int8) for k in ("valid", "event", "terminated", "winner", "draw", "flag")}
    csr_sha, mask_sha, cm_sha = [], [], []
    obs_keys, obs_sha, obs_full = [], [], {}

    def snap_obs(t: int):
        for i in range(min(obs_envs, N)):
            view = gs_view(b, i, hists[i], show_mode)
            for s in range(4):
                builder.build_into(view, beliefs[i][s], Seat(s), sp, gl)
                obs_keys.append((t, i, s))
                obs_sha.append(sha(sp, gl))
                if (t, i, s) in full_obs:
                    obs_full[f"obs_{t}_{i}_{s}_sp"] = sp.copy()
                    obs_full[f"obs_{t}_{i}_{s}_gl"] = gl.copy()

    for t in range(plies):
        if t in obs_plies:
            snap_obs(t)
        ids = b.legal_action_ids_batch()
        offsets = np.zeros(N + 1, np.int32)
        np.cumsum([len(x) for x in ids], out=offsets[1:])
        values = np.concatenate(ids).astype(np.int32) if any(len(x) for x in ids) else np.zeros(0, np.int32)
        csr_sha.append(sha(offsets, values))
        masks = np.stack([canonical_mask(ids[i], int(b.turn[i])) for i in range(N)])
        mask_sha.append(sha(masks))
        acts = policy(b, ids)
        acts_all[t] = acts
        pre = [gs_view(b, i, hists[i], show_mode) if not b.terminated[i] else None for i in range(N)]
        pre_dead = b.seat_dead_arr.copy()
        pre_types = [(int(b.piece_type_arr[i, b.cell_piece_id[i, a // 289]]) if b.cell_piece_id[i, a // 289] >= 0 else 0,
                      int(b.piece_type_arr[i, b.cell_piece_id[i, a % 289]]) if b.cell_piece_id[i, a % 289] >= 0 else 0)
                     for i, a in enumerate(acts)]
        acting = b.turn.copy()
        r = b.step_batch(acts)
        for k, src in (("valid", r.valid), ("event", r.event), ("terminated", r.terminated),
                       ("winner", r.winner_team), ("draw", r.draw), ("flag", r.flag_captured)):
            res[k][t] = src.astype(np.int8)
        zob[t] = b.zobrist
        cm_sha.append(sha(*[getattr(b, f) for f, _ in CM_FIELDS]))
        for i in range(N):
            if not r.valid[i]:
                continue
            a = int(acts[i])
            sf, df = a // 289, a % 289
            hists[i].append((sf, df))
            if len(hists[i]) > 32:
                hists[i] = hists[i][-32:]
            post = gs_view(b, i, hists[i], show_mode)
            ev = Event(int(r.event[i]))
            at, dt = pre_types[i]
            frs = ev is not Event.MOVE and siling_reveals_src(PieceType(at), PieceType(dt), ev)
            frd = ev is not Event.MOVE and siling_reveals_dst(PieceType(at), PieceType(dt), ev)
            died = tuple(Seat(s) for s in range(4) if b.seat_dead_arr[i, s] and not pre_dead[i, s])
            mr = MoveResult(seat=Seat(int(acting[i])), src=(sf % 17, sf // 17), dst=(df % 17, df // 17),
                            event=ev, flag_reveal_src=frs, flag_reveal_dst=frd,
                            flag_captured=bool(r.flag_captured[i]), seats_died_this_step=died)
            for s in range(4):
                beliefs[i][s].update(pre[i], post, mr)
    if plies in obs_plies:
        snap_obs(plies)
    events = res["event"][res["valid"] == 1]
    stats = {
        "plies": plies, "envs": N, "valid_steps": int((res["valid"] == 1).sum()),
        "moves": int((events == 1).sum()), "eat": int((events == 2).sum()),
        "bomb": int((events == 3).sum()), "killed": int((events == 4).sum()),
        "flag_captured": int(res["flag"].sum()), "terminated_final": int(b.terminated.sum()),
        "draws": int(b.draw.sum()), "seat_deaths": int(b.seat_dead_arr.sum()),
        "is_gongb_bits": int(b.cm_is_gongb.sum()),
    }
    out = {f"init_{k}": v for k, v in init.items()}
    out.update({f"final_{k}": v for k, v in state_dict(b).items()})
    out.update({"actions": acts_all, "zobrist": zob, **{f"res_{k}": v for k, v in res.items()},
                "csr_sha": np.array(csr_sha), "mask_sha": np.array(mask_sha), "cm_sha": np.array(cm_sha),
                "obs_keys": np.array(obs_keys, np.int32).reshape(-1, 3), "obs_sha": np.array(obs_sha),
                "show_mode": np.int32(show_mode.value)})
    out.update(obs_full)
    np.savez_compressed(OUT / f"ref_traj_{name}.npz", **out)
    print(name, stats, flush=True)
    return stats


# ---------------------------------------------------------------------------
# GameState trajectories (the single-env rules JunqiEnv steps, state.py)
# ---------------------------------------------------------------------------
_GS_FIELDS = [("alive", "alive"), ("piece_type_arr", "piece_type"), ("piece_seat_arr", "piece_seat"),
              ("pos_x", "pos_x"), ("pos_y", "pos_y"), ("zero_x", "zero_x"), ("zero_y", "zero_y"),
              ("move_count_arr", "move_count"), ("active_eat_arr", "active_eat"),
              ("passive_surv_arr", "passive_surv"), ("death_reason_arr", "death_reason"),
              ("death_step_arr", "death_step"), ("death_loc_flat_arr", "death_loc"),
              ("cell_piece_id", "cell_pid"), ("seat_dead_arr", "seat_dead"),
              ("seat_flag_revealed_arr", "seat_flag")]
_CM_MINE = {"cm_direct_lo": "cm_direct_lo", "cm_direct_hi": "cm_direct_hi", "cm_direct_type": "cm_direct_type",
            "cm_last_direct_step": "cm_last_direct_step", "cm_direct_other_count": "cm_direct_other",
            "cm_chain_lo": "cm_chain_lo", "cm_chain_hi": "cm_chain_hi", "cm_chain_type": "cm_chain_type",
            "cm_last_chain_step": "cm_last_chain_step", "cm_eaten_by_pid_lo": "cm_eaten_lo",
            "cm_eaten_by_pid_hi": "cm_eaten_hi", "cm_rank_floor": "cm_rank_floor",
            "cm_rank_floor_step": "cm_rank_floor_step", "cm_is_gongb": "cm_is_gongb",
            "cm_not_gongb": "cm_not_gongb", "cm_attacked_by_known_gongb": "cm_atk_gongb"}


def gs_state(games: list) -> dict[str, np.ndarray]:
    out = {mine: np.stack([np.asarray(getattr(g, ref)) for g in games]) for ref, mine in _GS_FIELDS}
    out["turn"] = np.array([g.turn.value for g in games], np.int8)
    out["zobrist"] = np.array([np.int64(np.uint64(g.zobrist & (2**64 - 1)).astype(np.int64)) for g in games], np.int64)
    out["move_counter"] = np.array([g.move_counter for g in games], np.int32)
    out["mslc"] = np.array([g.moves_since_last_combat for g in games], np.int32)
    out["terminated"] = np.array([g.terminated for g in games], bool)
    out["winner"] = np.array([-1 if g.winner_team is None else g.winner_team for g in games], np.int8)
    out["draw"] = np.array([g.draw for g in games], bool)
    for ref_field, (batched_name, _) in zip([f for _, f in CM_FIELDS], CM_FIELDS):
        out[_CM_MINE[batched_name]] = np.stack([np.asarray(getattr(g.combat_memory, ref_field)) for g in games])
    return out


def record_gamestate(name: str, games: list, plies: int, seed: int, combat_bias: bool, show_mode: ShowMode,
                     obs_plies: tuple[int, ...], obs_envs: int) -> dict:
    from junqi_core.state import Action
    rng = random.Random(seed)
    N = len(games)
    init = gs_state(games)
    beliefs = [[BeliefTensor.initial(g, Seat(s)) for s in range(4)] for g in games]
    builder = ObservationBuilder()
    sp = np.zeros((317, 17, 17), np.float32)
    gl = np.zeros(28, np.float32)
    acts_all = np.zeros((plies, N), np.int32)
    zob = np.zeros((plies, N), np.int64)
    res = {k: np.zeros((plies, N), np.int8) for k in ("valid", "event", "terminated", "winner", "draw", "flag")}
    csr_sha, mask_sha, cm_sha, obs_keys, obs_sha = [], [], [], [], []
    cm_order = [_CM_MINE[b] for b, _ in CM_FIELDS]

    def snap(t):
        for i in range(min(obs_envs, N)):
            for s in range(4):
                builder.build_into(games[i], beliefs[i][s], Seat(s), sp, gl)
                obs_keys.append((t, i, s))
                obs_sha.append(sha(sp, gl))

    for t in range(plies):
        if t in obs_plies:
            snap(t)
        ids = [g.legal_action_ids() for g in games]
        offsets = np.zeros(N + 1, np.int32)
        np.cumsum([len(x) for x in ids], out=offsets[1:])
        values = np.concatenate(ids).astype(np.int32) if any(len(x) for x in ids) else np.zeros(0, np.int32)
        csr_sha.append(sha(offsets, values))
        mask_sha.append(sha(np.stack([canonical_mask(np.asarray(ids[i]), games[i].turn.value) for i in range(N)])))
        for i, g in enumerate(games):
            w = -1 if g.winner_team is None else g.winner_team
            if g.terminated or len(ids[i]) == 0:
                res["terminated"][t, i], res["winner"][t, i], res["draw"][t, i] = g.terminated, w, g.draw
                continue
            pool = ids[i]
            if combat_bias:
                occ = g.cell_piece_id[np.asarray(pool) % 289] >= 0
                if occ.any():
                    pool = np.asarray(pool)[occ]
            a = int(rng.choice(list(pool)))
            acts_all[t, i] = a
            sf, df = a // 289, a % 289
            new, mr = g.step(Action(seat=g.turn, src=(sf % 17, sf // 17), dst=(df % 17, df // 17)))
            for s in range(4):
                beliefs[i][s].update(g, new, mr)
            games[i] = new
            res["valid"][t, i] = 1
            res["event"][t, i] = mr.event.value
            res["terminated"][t, i] = new.terminated
            res["winner"][t, i] = -1 if new.winner_team is None else new.winner_team
            res["draw"][t, i] = new.draw
            res["flag"][t, i] = mr.flag_captured
        st = gs_state(games)
        zob[t] = st["zobrist"]
        cm_sha.append(sha(*[st[k] for k in cm_order]))
    if plies in obs_plies:
        snap(plies)
    events = res["event"][res["valid"] == 1]
    stats = {"plies": plies, "envs": N, "valid_steps": int((res["valid"] == 1).sum()),
             "eat": int((events == 2).sum()), "bomb": int((events == 3).sum()), "killed": int((events == 4).sum()),
             "flag_captured": int(res["flag"].sum()), "terminated_final": int(sum(g.terminated for g in games)),
             "seat_deaths": int(sum(int(np.asarray(g.seat_dead_arr).sum()) for g in games))}
    out = {f"init_{k}": v for k, v in init.items()}
    out.update({f"final_{k}": v for k, v in gs_state(games).items()})
    out.update({"actions": acts_all, "zobrist": zob, **{f"res_{k}": v for k, v in res.items()},
                "csr_sha": np.array(csr_sha), "mask_sha": np.array(mask_sha), "cm_sha": np.array(cm_sha),
                "obs_keys": np.array(obs_keys, np.int32).reshape(-1, 3), "obs_sha": np.array(obs_sha),
                "show_mode": np.int32(show_mode.value), "rules": np.int32(1)})
    np.savez_compressed(OUT / f"ref_traj_{name}.npz", **out)
    print(name, stats, flush=True)
    return stats


def uniform_policy(seed: int):
    rng = random.Random(seed)

    def pol(b, ids):
        a = np.zeros(b.num_envs, np.int32)
        for i in range(b.num_envs):
            if not b.terminated[i] and ids[i].size:
                a[i] = int(rng.choice(ids[i]))
        return a
    return pol


def combat_policy(seed: int):
    rng = random.Random(seed)

    def pol(b, ids):
        a = np.zeros(b.num_envs, np.int32)
        for i in range(b.num_envs):
            if b.terminated[i] or not ids[i].size:
                continue
            occ = b.cell_piece_id[i, ids[i] % 289] >= 0
            pool = ids[i][occ] if occ.any() else ids[i]
            a[i] = int(rng.choice(pool))
        return a
    return pol


def late_game_states(n: int, seed: int, show_mode: ShowMode) -> list[GameState]:
    """Seeded setups thinned by 0-60 % and with engineers moved onto empty rail."""
    rng = random.Random(seed)
    states = []
    for i in range(n):
        g = GameState.new_game(generate_random_setup(random.Random(seed * 1000 + i)), show_mode=show_mode)
        frac = rng.uniform(0.0, 0.6)
        pieces = {}
        for pos, ref in g.pieces.items():
            if ref.piece_type is not PieceType.JUNQI and rng.random() < frac:
                continue
            pieces[pos] = ref
        rails = [int(f) for f in np.nonzero(T.IS_RAIL_FLAT)[0] if (int(f) % 17, int(f) // 17) not in pieces]
        for pos, ref in list(pieces.items()):
            if ref.piece_type is PieceType.GONGB and rails and rng.random() < 0.7:
                f = rails.pop(rng.randrange(len(rails)))
                del pieces[pos]
                pieces[(f % 17, f // 17)] = ref
        st = GameState(pieces=pieces, turn=Seat.SOUTH, move_counter=0, moves_since_last_combat=0,
                       info={s: SeatInfo() for s in Seat}, show_mode=show_mode)
        states.append(st)
    return states


def tables():
    srays = T.STRAIGHT_RAIL_RAYS_PAD.astype(np.int32)
    adj = np.full((289, 4), -1, np.int32)
    for f in range(289):
        for k, n in enumerate(RAIL_ADJ[f]):
            adj[f, k] = n
    zd = {k: sha(np.asarray(getattr(Z, k))) for k in
          ("ZOB_PIECE", "ZOB_TURN", "ZOB_MOVE_COUNTER", "ZOB_MOVES_SINCE_COMBAT", "ZOB_WINNER",
           "ZOB_SEAT_DEAD", "ZOB_SEAT_FLAG_REVEALED", "ZOB_SHOW_MODE")}
    zd["ZOB_TERMINATED"] = str(int(Z.ZOB_TERMINATED))
    zd["ZOB_DRAW"] = str(int(Z.ZOB_DRAW))
    setups = np.array([[int(p) for lu in generate_random_setup(random.Random(s)) for p in lu]
                       for s in range(32)], np.int8)
    np.savez_compressed(
        OUT / "ref_tables.npz",
        on_board=T.IS_ON_BOARD_FLAT.astype(np.int32), rail=T.IS_RAIL_FLAT.astype(np.int32),
        curve=T.CURVE_ID_OF.astype(np.int32), rail_adj=adj, srays=srays,
        crays=T.CURVE_CHAIN_RAYS_PAD.astype(np.int32), compact_to_flat=COMPACT_TO_FLAT.astype(np.int32),
        camp=T.IS_CAMP_FLAT.astype(np.int32), stronghold=T.IS_STRONGHOLD_FLAT.astype(np.int32),
        nine=T.IS_NINE_GRID_FLAT.astype(np.int32), arc=CURVE_ARC_CELLS.astype(np.int32),
        prior=_INITIAL_PRIOR_TABLE.astype(np.float32), pool64=_build_setup_pool(64, seed=42),
        setups_seed0_31=setups, rotate_lut=np.stack(ROTATE_LUT).astype(np.int32),
    )
    return zd


def main() -> None:
    zd = tables()
    manifest = {"zobrist": zd, "trajectories": {}}
    N = int(sys.argv[1]) if len(sys.argv) > 1 else 64
    b = BatchedGameState.from_game_states(
        [GameState.new_game(generate_random_setup(random.Random(1000 + i))) for i in range(N)])
    manifest["trajectories"]["cfg1"] = record(
        "cfg1", b, 300, uniform_policy(7), ShowMode.HALF_DARK, obs_plies=(0, 50, 150, 300), obs_envs=12,
        full_obs=((150, 0, 0), (300, 1, 2)))
    b = BatchedGameState.from_game_states(
        [GameState.new_game(generate_random_setup(random.Random(2000 + i)), show_mode=ShowMode.DARK)
         for i in range(32)])
    manifest["trajectories"]["combat_dark"] = record(
        "combat_dark", b, 400, combat_policy(11), ShowMode.DARK, obs_plies=(100, 400), obs_envs=8)
    b = BatchedGameState.from_game_states(
        [GameState.new_game(generate_random_setup(random.Random(3000 + i)), show_mode=ShowMode.BRIGHT)
         for i in range(24)])
    manifest["trajectories"]["long_bright"] = record(
        "long_bright", b, 1500, combat_policy(13), ShowMode.BRIGHT, obs_plies=(750, 1500), obs_envs=8)
    b = BatchedGameState.from_game_states(late_game_states(32, 5, ShowMode.HALF_DARK))
    manifest["trajectories"]["late_game"] = record(
        "late_game", b, 600, uniform_policy(17), ShowMode.HALF_DARK, obs_plies=(0, 300, 600), obs_envs=8)
    games = [GameState.new_game(generate_random_setup(random.Random(4000 + i))) for i in range(48)]
    manifest["trajectories"]["gs_uniform"] = record_gamestate(
        "gs_uniform", games, 400, 21, False, ShowMode.HALF_DARK, obs_plies=(0, 200, 400), obs_envs=8)
    games = [GameState.new_game(generate_random_setup(random.Random(5000 + i)), show_mode=ShowMode.DARK)
             for i in range(32)]
    manifest["trajectories"]["gs_combat_dark"] = record_gamestate(
        "gs_combat_dark", games, 500, 23, True, ShowMode.DARK, obs_plies=(250, 500), obs_envs=8)
    games = late_game_states(32, 6, ShowMode.HALF_DARK)
    manifest["trajectories"]["gs_late"] = record_gamestate(
        "gs_late", games, 500, 29, True, ShowMode.HALF_DARK, obs_plies=(0, 250, 500), obs_envs=8)
    (OUT / "ref_manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
