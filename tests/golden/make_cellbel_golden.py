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
every SNAP plies, sparse (flat index into (ENVS, 4, 36, 17, 17), value).

    python tests/golden/make_cellbel_golden.py <output.npz>
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
ENVS, PLIES, SNAP, SEED = 5, 600, 30, 4242
BEL_CH = list(range(12, 24)) + list(range(27, 51))
STATE_KEYS = {"piece_seat_arr": (np.int8, 120), "piece_type_arr": (np.int8, 120), "alive": (np.uint8, 120),
              "pos_x": (np.int8, 120), "pos_y": (np.int8, 120), "cell_piece_id": (np.int16, 289),
              "seat_dead_arr": (np.uint8, 4), "terminated": (np.uint8, 1)}


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_cellbel_golden.py <output.npz>")
    sys.path.insert(0, str(ROOT / "baseline" / "_ref" / "junqi_rl"))
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    import torch
    from junqi_core.rules import ShowMode
    from junqi_rl.gpu_rollout import (GpuRollout, _build_belief_prior_table, _build_seat_strongholds,
                                      _CudaArrayInterfaceView)

    ro = GpuRollout(num_envs=ENVS, show_mode=ShowMode.HALF_DARK, device_id=0)
    assert ro._beliefs_enabled, "the reference build has no device beliefs"
    ro.reset_from_setup_pool(seed=SEED)

    def state() -> dict[str, np.ndarray]:
        h = dict(ro.state.copy_to_host())
        h["terminated"] = ro.state.copy_termination_to_host()["terminated"]
        return {k: np.asarray(h[k]).reshape(ENVS, n).astype(dt) for k, (dt, n) in STATE_KEYS.items()}

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
        wa = torch.as_tensor(_CudaArrayInterfaceView(p["d_world_actions_ptr"], (ENVS,), "<i4"), device="cuda")
        fc = torch.as_tensor(_CudaArrayInterfaceView(p["d_flag_captured_ptr"], (ENVS,), "|b1"), device="cuda")
        events.append(res["event"].cpu().numpy().astype(np.int8).reshape(ENVS))
        flags.append(fc.cpu().numpy().astype(np.uint8))
        actions.append(wa.cpu().numpy().astype(np.int32))
        for k, a in state().items():
            rec[k].append(a)
        if t % SNAP == 0:
            i, v = planes()
            snaps_i.append(i), snaps_v.append(v), snap_ply.append(t)
    ev = np.stack(events)
    print("plies", PLIES, "events", {int(k): int((ev == k).sum()) for k in range(5)},
          "flag captures", int(np.stack(flags).sum()), "terminated", int(rec["terminated"][-1].sum()))
    out = {"prior": _build_belief_prior_table().astype(np.float32).reshape(30, 12),
           "strongholds": _build_seat_strongholds().astype(np.int16).reshape(8),
           "prev_dead": np.stack(prev_dead), "event": ev, "flag_captured": np.stack(flags),
           "world_action": np.stack(actions), "snap_ply": np.array(snap_ply, np.int32),
           "snap_len": np.array([len(x) for x in snaps_i], np.int64),
           "snap_index": np.concatenate(snaps_i), "snap_value": np.concatenate(snaps_v),
           "bel_channels": np.array(BEL_CH, np.int32)}
    for k in STATE_KEYS:
        out["init_" + k] = s0[k]
        out["post_" + k] = np.stack(rec[k])
    np.savez_compressed(sys.argv[1], **out)
    print("wrote", sys.argv[1])


if __name__ == "__main__":
    main()
