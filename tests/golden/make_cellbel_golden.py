"""Golden vectors for the per-cell float beliefs of the reference's GPU rollout.

The reference keeps these beliefs only on the device and has no call that
reads them back, so they are captured through what it does expose: the
belief planes of its all-seat observation (channels 12-23 teammate, 27-38
left enemy, 39-50 right enemy: the belief value at each such piece's cell
where it is > 0, observation.cu:330-370), built from the resident beliefs
by build_observation_batch_resident.

Runs on a B200 with the reference's own junqi_cuda extension built into
baseline/_ref (baseline/build_ref_cuda.py).  A GpuRollout of ENVS envs in
HALF_DARK is reset from its setup pool (which seeds the beliefs with
init_beliefs_for_reset_envs) and played PLIES plies with deterministic legal
actions (argmax over the canonical mask times a seeded key vector, rolled
each ply); each ply is step_device_torch (pre-step snapshot, step) then
update_beliefs_device.  Terminated envs are not reset.  Recorded: the
uploaded prior table and stronghold cells; the state fields the update
reads, after the reset and after every ply; each ply's pre-step seat_dead,
event, flag capture and world action; the belief planes after the reset and
every SNAP plies, sparse (flat index into (ENVS, 4, 36, 17, 17), stored as
the difference from the previous index of the same snapshot, and value).

    python tests/golden/make_cellbel_golden.py <output.npz>
    python tests/golden/make_cellbel_golden.py --late <output.npz>

With --late the envs start from late-game positions instead (ENVS_LATE
seeded setups thinned by junqi_b200.workloads.thin_positions, built with
the CPU oracle, uploaded with copy_from_host and seeded with
init_all_beliefs), where captures come within the recorded plies: the
script checks that at least one flag capture and at least one eat of a
non-flag piece on a stronghold happened, so the rules that only those
fire (belief.cu R4, R6) are pinned to the reference's own output too.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
ENVS, PLIES, SNAP, SEED = 5, 600, 30, 4242
ENVS_LATE, SEED_LATE = 16, 5151
BEL_CH = list(range(12, 24)) + list(range(27, 51))
STATE_KEYS = {"piece_seat_arr": (np.int8, 120), "piece_type_arr": (np.int8, 120), "alive": (np.uint8, 120),
              "pos_x": (np.int8, 120), "pos_y": (np.int8, 120), "cell_piece_id": (np.int16, 289),
              "seat_dead_arr": (np.uint8, 4), "terminated": (np.uint8, 1)}


def late_positions(n: int, seed: int) -> dict:
    """Reference-named state arrays of n thinned late-game positions (CPU oracle)."""
    sys.path.insert(0, str(ROOT))
    from junqi_b200 import tables, workloads
    from oracle import oracle as O
    pool = tables.build_setup_pool(n, seed=seed)
    orc = O.OracleBatch(n, 2, rules=1)
    for e in range(n):
        orc.reset_env(e, pool[e])
    st = workloads.thin_positions({k: v.copy() for k, v in orc.a.items()}, seed)
    O.load_state(orc, st, init_beliefs=True)
    orc.a["zobrist"][:] = O.zobrist_recompute(orc.a, 2)
    names = {"piece_seat_arr": "piece_seat", "piece_type_arr": "piece_type", "alive": "alive", "pos_x": "pos_x",
             "pos_y": "pos_y", "zero_x": "zero_x", "zero_y": "zero_y", "move_count_arr": "move_count",
             "active_eat_arr": "active_eat", "passive_surv_arr": "passive_surv",
             "death_reason_arr": "death_reason", "death_step_arr": "death_step",
             "death_loc_flat_arr": "death_loc", "cell_piece_id": "cell_pid", "seat_dead_arr": "seat_dead",
             "seat_flag_revealed_arr": "seat_flag", "turn": "turn", "zobrist": "zobrist",
             "move_counter": "move_counter", "moves_since_last_combat": "mslc"}
    d = {ref: np.ascontiguousarray(orc.a[m].reshape(-1)) for ref, m in names.items()}
    for k in ("alive", "seat_dead_arr", "seat_flag_revealed_arr"):
        d[k] = d[k].astype(bool)
    alive = orc.a["alive"].astype(bool).reshape(-1)
    flat = orc.a["pos_y"].astype(np.int16).reshape(-1) * 17 + orc.a["pos_x"].astype(np.int16).reshape(-1)
    d["cell_piece_id_per_piece"] = np.where(alive, flat, -1).astype(np.int16)
    return d


def main() -> None:
    args = [a for a in sys.argv[1:] if a != "--late"]
    late = "--late" in sys.argv[1:]
    if len(args) != 1:
        raise SystemExit("usage: python tests/golden/make_cellbel_golden.py [--late] <output.npz>")
    envs = ENVS_LATE if late else ENVS
    sys.path.insert(0, str(ROOT / "baseline" / "_ref" / "junqi_rl"))
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    import torch
    from junqi_core.rules import ShowMode
    from junqi_rl import gpu_rollout
    from junqi_rl.gpu_rollout import (GpuRollout, _build_belief_prior_table, _build_seat_strongholds,
                                      _CudaArrayInterfaceView)

    ro = GpuRollout(num_envs=envs, show_mode=ShowMode.HALF_DARK, device_id=0)
    assert ro._beliefs_enabled, "the reference build has no device beliefs"
    if late:
        ro.state.copy_from_host(late_positions(envs, SEED_LATE))
        ro.state.copy_termination_from_host(np.zeros(envs, bool), np.full(envs, -1, np.int8), np.zeros(envs, bool))
        gpu_rollout._cuda.init_all_beliefs(ro.state)
    else:
        ro.reset_from_setup_pool(seed=SEED)
    n_envs = envs

    def state() -> dict[str, np.ndarray]:
        h = dict(ro.state.copy_to_host())
        h["terminated"] = ro.state.copy_termination_to_host()["terminated"]
        return {k: np.asarray(h[k]).reshape(n_envs, n).astype(dt) for k, (dt, n) in STATE_KEYS.items()}

    def planes() -> tuple[np.ndarray, np.ndarray]:
        sp, _ = ro.build_all_seat_observations()
        b = np.ascontiguousarray(np.asarray(sp)[:, :, BEL_CH])
        idx = np.flatnonzero(b)
        return idx.astype(np.int32), b.reshape(-1)[idx].astype(np.float32)

    g = torch.Generator(device="cuda").manual_seed(SEED)
    keys = torch.randint(1, 32000, (16641,), device="cuda", dtype=torch.int32, generator=g)
    rec = {k: [] for k in STATE_KEYS}
    s0 = state()
    snaps_i, snaps_v, snap_ply = [], [], []
    i, v = planes()
    snaps_i.append(i), snaps_v.append(v), snap_ply.append(0)
    prev_dead, events, flags, actions = [], [], [], []
    for t in range(1, PLIES + 1):
        acting = ro.turn_torch().clone()
        mask = ro.legal_mask_canonical_torch_device(acting)
        acts = (mask.to(torch.int32) * torch.roll(keys, t)).argmax(dim=1).to(torch.int32)
        prev_dead.append(state()["seat_dead_arr"])
        res = ro.step_device_torch(acts, acting)
        ro.update_beliefs_device(res, acting)
        p = ro._last_step_ptrs
        wa = torch.as_tensor(_CudaArrayInterfaceView(p["d_world_actions_ptr"], (n_envs,), "<i4"), device="cuda")
        fc = torch.as_tensor(_CudaArrayInterfaceView(p["d_flag_captured_ptr"], (n_envs,), "|b1"), device="cuda")
        events.append(res["event"].cpu().numpy().astype(np.int8).reshape(n_envs))
        flags.append(fc.cpu().numpy().astype(np.uint8))
        actions.append(wa.cpu().numpy().astype(np.int32))
        for k, a in state().items():
            rec[k].append(a)
        if t % SNAP == 0:
            i, v = planes()
            snaps_i.append(i), snaps_v.append(v), snap_ply.append(t)
    ev = np.stack(events)
    fc = np.stack(flags)
    sh = _build_seat_strongholds().astype(np.int64).reshape(-1)
    wa = np.stack(actions)
    sh_eats = int(((ev == 2) & (fc == 0) & np.isin(wa % 289, sh) & (wa >= 0)).sum())
    print("plies", PLIES, "events", {int(k): int((ev == k).sum()) for k in range(5)},
          "flag captures", int(fc.sum()), "non-flag stronghold eats", sh_eats,
          "terminated", int(rec["terminated"][-1].sum()))
    if late and (fc.sum() == 0 or sh_eats == 0):
        raise SystemExit("the late-game capture needs a flag capture and a non-flag stronghold eat")
    out = {"prior": _build_belief_prior_table().astype(np.float32).reshape(30, 12),
           "strongholds": _build_seat_strongholds().astype(np.int16).reshape(8),
           "prev_dead": np.stack(prev_dead), "event": ev, "flag_captured": np.stack(flags),
           "world_action": np.stack(actions), "snap_ply": np.array(snap_ply, np.int32),
           "snap_len": np.array([len(x) for x in snaps_i], np.int64),
           "snap_index_delta": np.concatenate([np.diff(i, prepend=0) for i in snaps_i]).astype(np.int32),
           "snap_value": np.concatenate(snaps_v),
           "bel_channels": np.array(BEL_CH, np.int32)}
    for k in STATE_KEYS:
        out["init_" + k] = s0[k]
        out["post_" + k] = np.stack(rec[k])
    np.savez_compressed(args[0], **out)
    print("wrote", args[0])


if __name__ == "__main__":
    main()
