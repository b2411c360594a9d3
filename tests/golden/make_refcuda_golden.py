"""Golden vectors from the reference's own CUDA extension for the two formats
junqi_core does not define.

1. The per-piece 80-slot legal mask, ``legal_action_mask_batch`` (slot order
   defined only by game_state.cu:1985-2197 and tables.cu:176-350).
2. Observations built from caller-given per-cell beliefs,
   ``build_observation_batch`` (observation.cu:330-370 for the belief planes,
   417-424 and 533-544 for global[0:24], which sums belief values over the
   enemy cells with float atomics).  The beliefs given are multiples of 1/16
   with at most 30 terms per sum, so every partial sum is exact in float32
   and the atomics' order cannot change the result.

Positions: seeded fresh setups, positions after 40-1500 uniform plies under
GameState rules (combat memory, deaths, finished games), and late-game
thinned positions with engineers on the railway, all built with the CPU
oracle (inputs only; every recorded output is the reference's).  For each
position the mask is recorded for the side to move and for the next seat
(the reference kernel checks neither termination nor dead seats), and the
observation of all four seats, in a rotated seat order, under DARK and
HALF_DARK.

Runs on a B200 with the reference extension built into baseline/_ref
(baseline/build_ref_cuda.py):

    python tests/golden/make_refcuda_golden.py tests/golden/ref_cuda_slots_beliefs.npz
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
SEED = 5150
N_FRESH, N_MID, N_LATE = 16, 48, 32
BEL_CH = list(range(12, 24)) + list(range(27, 51))
REF_KEYS = {"piece_seat_arr": "piece_seat", "piece_type_arr": "piece_type", "alive": "alive", "pos_x": "pos_x",
            "pos_y": "pos_y", "zero_x": "zero_x", "zero_y": "zero_y", "move_count_arr": "move_count",
            "active_eat_arr": "active_eat", "passive_surv_arr": "passive_surv", "death_reason_arr": "death_reason",
            "death_step_arr": "death_step", "death_loc_flat_arr": "death_loc", "cell_piece_id": "cell_pid",
            "seat_dead_arr": "seat_dead", "seat_flag_revealed_arr": "seat_flag", "turn": "turn",
            "zobrist": "zobrist", "move_counter": "move_counter", "moves_since_last_combat": "mslc"}


def positions():
    """Oracle batch of N_FRESH + N_MID + N_LATE positions."""
    from junqi_b200 import tables, workloads
    from oracle import oracle as O
    n = N_FRESH + N_MID + N_LATE
    pool = tables.build_setup_pool(n, seed=SEED)
    out = O.OracleBatch(n, 2, rules=1)
    for e in range(n):
        out.reset_env(e, pool[e])
    rng = np.random.default_rng(SEED)
    # mid-game: each env its own number of uniform plies (finished games stay finished)
    plies = rng.integers(40, 1501, N_MID)
    mid = slice(N_FRESH, N_FRESH + N_MID)
    b = O.OracleBatch(N_MID, 2, rules=1)
    for i in range(N_MID):
        b.reset_env(i, pool[N_FRESH + i])
    for t in range(int(plies.max())):
        off, val = b.legal()
        cnt = np.diff(off)
        acts = np.full(N_MID, -1, np.int32)
        for i in np.nonzero((cnt > 0) & (plies > t))[0]:
            acts[i] = val[off[i] + rng.integers(cnt[i])]
        b.step(acts)
    for k in out.a:
        out.a[k][mid] = b.a[k]
    # late game: thinned setups, engineers on the railway
    late = slice(N_FRESH + N_MID, n)
    st = {k: v[late].copy() for k, v in out.a.items()}
    st = workloads.thin_positions(st, SEED + 1)
    c = O.OracleBatch(N_LATE, 2, rules=1)
    O.load_state(c, st, init_beliefs=True)
    c.a["zobrist"][:] = O.zobrist_recompute(c.a, 2)
    for k in out.a:
        out.a[k][late] = c.a[k]
    return out


def beliefs_x16(n: int) -> np.ndarray:
    """(n, 4, 12, 289) uint8 belief inputs in sixteenths: an integer hash of
    (env, observer, type, cell), about half of them zero.  Empty cells get
    values too, so a sum over cells rather than over pieces would show."""
    i = np.arange(n * 4 * 12 * 289, dtype=np.uint64)
    h = (i + np.uint64(SEED)) * np.uint64(0x9E3779B97F4A7C15)
    h ^= h >> np.uint64(29)
    h *= np.uint64(0xBF58476D1CE4E5B9)
    h ^= h >> np.uint64(32)
    v = (h % np.uint64(17)).astype(np.uint8)
    v[((h >> np.uint64(40)) & np.uint64(1)) == 0] = 0
    return v.reshape(n, 4, 12, 289)


def pack(orc) -> dict:
    d = {ref: np.ascontiguousarray(orc.a[m].reshape(-1)) for ref, m in REF_KEYS.items()}
    for k in ("alive", "seat_dead_arr", "seat_flag_revealed_arr"):
        d[k] = d[k].astype(bool)
    alive = orc.a["alive"].astype(bool).reshape(-1)
    flat = orc.a["pos_y"].astype(np.int16).reshape(-1) * 17 + orc.a["pos_x"].astype(np.int16).reshape(-1)
    d["cell_piece_id_per_piece"] = np.where(alive, flat, -1).astype(np.int16)
    return d


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_refcuda_golden.py <output.npz>")
    orc = positions()
    n = orc.n
    sys.path.insert(0, str(ROOT / "baseline" / "_ref" / "junqi_rl"))
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    from junqi_core.rules import ShowMode
    from junqi_rl import gpu_rollout
    _cuda = gpu_rollout._cuda
    gpu_rollout.GpuRollout(num_envs=n, show_mode=ShowMode.HALF_DARK, device_id=0)  # uploads every table
    state = _cuda.DeviceGameStateBatch(n)
    state.copy_from_host(pack(orc))
    state.copy_termination_from_host(orc.a["terminated"].astype(bool), orc.a["winner"].astype(np.int8),
                                     orc.a["draw"].astype(bool))
    turn = orc.a["turn"].astype(np.int8)
    seats = np.stack([turn, (turn + 1) % 4]).astype(np.int8)
    masks = np.stack([np.asarray(_cuda.legal_action_mask_batch(state, s)) for s in seats])

    beliefs = beliefs_x16(n).astype(np.float32) / 16.0
    observers = np.stack([(np.arange(4) + e) % 4 for e in range(n)]).astype(np.int8)
    obs = _cuda.DeviceObservationBatch(n)
    planes, glob = [], []
    for mode in (1, 2):
        _cuda.build_observation_batch(state, beliefs, observers, obs, mode)
        sp, gl = obs.copy_to_host()
        planes.append(np.ascontiguousarray(np.asarray(sp).reshape(n, 4, 317, 289)[:, :, BEL_CH]))
        glob.append(np.asarray(gl).reshape(n, 4, 28).astype(np.float32))
    planes = np.stack(planes)
    idx = np.flatnonzero(planes)
    out = {"init_" + k: v for k, v in orc.a.items()}
    out.update({"slot_seats": seats, "ref_slot_mask": np.packbits(masks.astype(bool), axis=-1),
                "observers": observers, "show_modes": np.array([1, 2], np.int8),
                "bel_channels": np.array(BEL_CH, np.int32), "ref_global": np.stack(glob),
                "ref_bel_index": idx.astype(np.int32), "ref_bel_value": planes.reshape(-1)[idx].astype(np.float32)})
    np.savez_compressed(sys.argv[1], **out)
    print("wrote", sys.argv[1], "positions", n, "mask bits set", int(masks.sum()),
          "terminated", int(orc.a["terminated"].sum()), "belief floats", idx.size)


if __name__ == "__main__":
    main()
