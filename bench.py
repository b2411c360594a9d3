#!/usr/bin/env python
"""Benchmark: env plies/s for step + legal mask + 317-channel observation.

One "step" is one ply over the whole batch: observation of every env's
acting seat, a stand-in policy (uniform-random legal action, or a masked
softmax over seeded N(0,1) logits), then the fused ply kernel (step, combat
memory, beliefs, auto-reset from the setup pool, legal CSR + canonical mask
of the new turn).  ``value`` counts plies actually applied (MoveResult
valid) summed over ranks, divided by the max over ranks of the device time
of the timed steps.  Inputs are device resident; every step writes
>1.5 GB (observations), far above the 126 MB L2, so no flush is needed.

``--impl reference`` times the CPU restatement of the reference rules (the
oracle port; the reference itself is Python and does not travel to the GPU
host) on the host cores, same metric and config, bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: envs per GPU, observer seats per env, policy, pool size, plies, show mode
    "cfg2": dict(envs=4096, seats=1, policy="uniform", pool=10_000, plies=1000, mode=2,
                 workload="configs[1]: 4096 envs/GPU, step + CSR legal mask + 317-ch obs (acting seat), "
                          "uniform-random legal policy, auto-reset from a seeded 10,000-setup pool"),
    "cfg3": dict(envs=65536, seats=4, policy="softmax", pool=10_000, plies=100, mode=2,
                 workload="configs[2]: 65536 envs, obs for all 4 seats, masked softmax over seeded N(0,1) logits"),
    "cfg4": dict(envs=32768, seats=1, policy="softmax", pool=8192, plies=512, mode=2,
                 workload="configs[3]: 32768 envs/GPU, 512-ply rollout, pool of 8192, masked softmax, "
                          "episode stats all-reduced once per rollout"),
    "cfg5": dict(envs=32768, seats=1, policy="uniform", pool=10_000, plies=2000, mode=2, start="late",
                 workload="configs[4]: 32768 envs/GPU late-game starts (seeded setups, 0-60% of pieces removed, "
                          "engineers on the railway), 2000 plies, uniform-random legal policy"),
}

OBS_WRITE = 317 * 289 * 4 + 28 * 4  # bytes written per (env, seat) observation
EVENT_EVERY = 8  # timed plies between plies that carry per-kernel CUDA events

# jq_batch.rules: 1 = GameState.step (state.py; Q12 "no legal move -> seat
# dies" on every ply, as the single-env JunqiEnv and the reference GPU kernel
# do), 0 = BatchedGameState.step_batch (batched_state.py; plain moves test Q12
# only when the next seat is already dead, so a seat left without moves can
# stall its env for good).  Both are pinned bit-exactly to junqi_core.
RULES = {"gamestate": 1, "batched": 0}
RULES_TEXT = {"gamestate": "GameState.step (state.py:638)", "batched": "BatchedGameState.step_batch (batched_state.py:417)"}


def obs_read_bytes() -> int:
    """Bytes the observation kernel must read per (env, observer) unit."""
    piece = 120 * (1 + 1 + 1 + 1 + 1 + 1 + 1 + 2 + 2 + 2 + 1 + 2 + 2)      # piece SoA fields read
    cm_obs = 120 * (8 + 8 + 2 + 2 + 2 + 8 + 8 + 2 + 2 + 1 + 2 + 1 + 1 + 1)  # observer's CM row
    cm_opp = 30 * 2 * (8 + 8 + 2 + 1 + 1) + 30 * 16                    # opponents' view of own pieces, eaten_by
    other = 120 + 2 * 24 + 8 + 2 * 32 * 2 + 4 + 4 + 4                  # belief codes, remaining, flags, history
    return piece + cm_obs + cm_opp + other


def pipeline_roofline(plies_per_gpu: float, seats: int, k_avg: float, peak: float) -> dict:
    """Whole step + mask + obs pipeline against HBM: the compulsory bytes of
    one env-ply of the API tensors (obs written, canonical mask written, CSR
    written, game SoA read + written, combat memory read, the observer's
    belief slice read, the action read) times plies/s per GPU."""
    b_ply = seats * (OBS_WRITE + 13_872) + 16_641 + 4 * (k_avg + 1) + 2 * 3_142 + 30_720 + 4
    achieved = plies_per_gpu * b_ply / 1e9
    return {"bytes_per_ply": b_ply, "legal_per_env": k_avg, "achieved": achieved, "unit": "GB/s per GPU",
            "peak": peak, "frac": achieved / peak}


def sample_clocks(dev: int, stop: threading.Event, rows: list) -> None:
    q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    try:
        p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-i", str(dev),
                              "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return
    try:
        while not stop.is_set():
            line = p.stdout.readline()
            if not line:
                break
            rows.append([x.strip() for x in line.split(",")])
    finally:
        p.terminate()
        try:
            p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            p.kill()


def summarize_clocks(rows: list) -> dict:
    sm = [float(r[0]) for r in rows if len(r) >= 8 and r[0].replace(".", "").isdigit()]
    mx = [float(r[1]) for r in rows if len(r) >= 8 and r[1].replace(".", "").isdigit()]
    reasons = set()
    for r in rows:
        if len(r) < 8:
            continue
        for name, v in (("hw_slowdown", r[4]), ("hw_thermal_slowdown", r[5]), ("sw_thermal_slowdown", r[6]),
                        ("sw_power_cap", r[7])):
            if v.strip().lower() == "active":
                reasons.add(name)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons), "samples": len(sm)}


def peak_hbm() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profiled_traffic(cfg: str) -> float | None:
    """DRAM bytes per observation unit from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "obs_kernel_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return float(d["dram_bytes_per_unit"])
    except Exception:
        return None


# ---------------------------------------------------------------------------
# CPU arms (oracle = CPU restatement of the reference rules)
# ---------------------------------------------------------------------------

def cpu_rollout(envs: int, plies: int, seats: int, seed: int, threads: int, budget_s: float, rules: int = 1,
                late: bool = False, burn_in: int = 0):
    """Step + legal + observation on the CPU oracle; returns (plies/s, plies, seconds, sample text).
    ``burn_in`` untimed plies (step + legal, no observation) come first, as in the GPU arm."""
    os.environ["JQ_ORACLE_THREADS"] = str(threads)
    from junqi_b200 import tables
    from oracle import oracle as O
    pool = tables.build_setup_pool(256, seed=42)
    b = O.OracleBatch(envs, 2, rules=rules)
    b.threads = threads
    rng = np.random.default_rng(seed)
    for e in range(envs):
        b.reset_env(e, pool[e % len(pool)])
    if late:  # the same host edit the GPU arm applies (junqi_b200/workloads.py)
        from junqi_b200 import workloads
        O.load_state(b, workloads.thin_positions({k: v.copy() for k, v in b.a.items()}, seed), init_beliefs=True)
        b.a["zobrist"][:] = O.zobrist_recompute(b.a, 2)
    def pick_actions():
        off, val = b.legal()
        cnt = np.diff(off)
        pick = (rng.random(envs) * np.maximum(cnt, 1)).astype(np.int64)
        return np.where(cnt > 0, val[np.minimum(off[:-1] + pick, max(len(val) - 1, 0))] if len(val) else -1, -1)

    for _ in range(burn_in):
        r = b.step(pick_actions().astype(np.int32))
        for e in np.nonzero(r["terminated"])[0]:
            b.reset_env(int(e), pool[int(rng.integers(len(pool)))])
    done = 0
    t0 = time.perf_counter()
    t = 0
    for t in range(plies):
        if seats == 1:
            b.obs()
        else:
            for s in range(4):
                b.obs(np.full(envs, s, np.int8))
        r = b.step(pick_actions().astype(np.int32))
        done += int(r["valid"].sum())
        for e in np.nonzero(r["terminated"])[0]:
            b.reset_env(int(e), pool[int(rng.integers(len(pool)))])
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    sample = (f"{envs} envs x {t + 1} plies after a {burn_in}-ply burn-in, step + legal + obs ({seats} seat/env), "
              f"{threads} threads")
    return done / dt, done, dt, sample


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_arm(args, cfg: dict) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = host_cores()
    from oracle import oracle as O
    O.build()
    envs = min(cfg["envs"], 256 * threads)
    for _ in range(args.warmup if args.warmup < 3 else 2):
        cpu_rollout(min(envs, 64), 1, cfg["seats"], args.seed, threads, 5.0, RULES[args.rules])
    rate, done, dt, sample = cpu_rollout(envs, args.steps, cfg["seats"], args.seed, threads, 120.0,
                                         RULES[args.rules], late=cfg.get("start") == "late", burn_in=args.burn_in)
    line = {"impl": "reference", "metric": "env plies/s (step + legal mask + 317-ch obs)", "value": rate,
            "unit": "plies/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/int16/f32",
            "data": "synthetic (seeded setup pool of random legal lineups, seeded policy)",
            "config": arm_config(cfg, args, args.gpus),
            "cpu_baseline": {"value": rate, "unit": "plies/s", "cores": threads, "kind": "port",
                             "sample": sample + f", {dt:.1f} s"},
            "e2e": {"value": rate, "unit": "plies/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _batched_worker(rank: int, envs: int, budget_s: float, seed: int, q) -> None:
    """junqi_core's vectorised path on one core: BatchedGameState.step_batch
    (batched_state.py:417) + legal_action_ids_batch (:370) over `envs` games,
    a uniform legal action each.  The batch has no per-env reset, so games
    are played in windows: a fresh batch, 50 untimed plies, then 300 timed
    plies; windows repeat until the timed plies add up to budget_s."""
    import random
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    from junqi_core.batched_state import BatchedGameState
    from junqi_core.setup import generate_random_setup
    from junqi_core.state import GameState
    rng = random.Random(seed + 7919 * rank)

    def ply(b) -> int:
        ids = b.legal_action_ids_batch()
        acts = np.array([int(x[rng.randrange(len(x))]) if len(x) else 0 for x in ids], np.int32)
        return int(np.asarray(b.step_batch(acts).valid).sum())

    done, secs = 0, 0.0
    while secs < budget_s:
        b = BatchedGameState.from_game_states(
            [GameState.new_game(generate_random_setup(random.Random(rng.getrandbits(32)))) for _ in range(envs)])
        for _ in range(50):
            ply(b)
        t0 = time.perf_counter()
        for _ in range(300):
            done += ply(b)
        secs += time.perf_counter() - t0
    q.put((done, secs, 0))


def _junqi_core_worker(rank: int, envs: int, burn_in: int, budget_s: float, seed: int, q, seats: int = 1) -> None:
    """One host core's slice: the reference's own CPU path for one ply of the
    single-env rules (the JunqiEnv ply, GameState.step, state.py:626):
    acting-seat observation (ObservationBuilder.build_into, observation.py:
    510), legal ids, a uniform action, the step and the four seats'
    BeliefTensor.update (info_model.py:271), with finished games reset from
    seeded setups (GameState.new_game, setup.py:162 lineups)."""
    import random
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    from junqi_core.info_model import BeliefTensor
    from junqi_core.observation import ObservationBuilder
    from junqi_core.rules import Seat
    from junqi_core.setup import generate_random_setup
    from junqi_core.state import Action, GameState
    rng = random.Random(seed + 7919 * rank)

    def fresh():
        g = GameState.new_game(generate_random_setup(random.Random(rng.getrandbits(32))))
        return g, [BeliefTensor.initial(g, Seat(k)) for k in range(4)]

    games = [fresh() for _ in range(envs)]
    builder = ObservationBuilder()
    sp = np.zeros((317, 17, 17), np.float32)
    gl = np.zeros(28, np.float32)

    def ply(obs: bool) -> int:
        done = 0
        for i, (g, bel) in enumerate(games):
            if obs:
                for s in ([g.turn] if seats == 1 else [Seat(k) for k in range(4)]):
                    builder.build_into(g, bel[s.value], s, sp, gl)
            ids = g.legal_action_ids()
            if g.terminated or len(ids) == 0:
                games[i] = fresh()
                continue
            a = int(ids[rng.randrange(len(ids))])
            sf, df = a // 289, a % 289
            new, mr = g.step(Action(seat=g.turn, src=(sf % 17, sf // 17), dst=(df % 17, df // 17)))
            for b in bel:
                b.update(g, new, mr)
            games[i] = (new, bel) if not new.terminated else fresh()
            done += 1
        return done

    for _ in range(burn_in):
        ply(False)
    done, plies = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        done += ply(True)
        plies += 1
    q.put((done, time.perf_counter() - t0, plies))


def reference_python_arm(args, cfg: dict) -> None:
    """The reference's own Python implementation of the path (junqi_core,
    staged into baseline/_ref by baseline/build_ref_cuda.py), timed on all
    host cores, one process per core each playing its own slice of envs:
    a reported baseline beside the oracle port of --impl reference."""
    import multiprocessing as mp
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if not (ROOT / "baseline" / "_ref" / "junqi_core").exists():
        print(json.dumps({"impl": "reference-python", "unavailable": "baseline/_ref has no junqi_core; run "
                          "baseline/build_ref_cuda.py where the reference checkout exists"}), flush=True)
        return
    cores = host_cores()
    per = 8
    burn = min(args.burn_in, 50)
    seats = cfg["seats"]
    ctx = mp.get_context("spawn")

    def run(target, nproc, head, tail=()):
        """nproc processes of target(rank, *head, queue, *tail); (plies, seconds, per-process results)."""
        q = ctx.Queue()
        procs = [ctx.Process(target=target, args=(r, *head, q, *tail)) for r in range(nproc)]
        for p in procs:
            p.start()
        res = [q.get(timeout=600) for _ in procs]
        for p in procs:
            p.join(timeout=60)
        return sum(r[0] for r in res), max(r[1] for r in res), res

    done, secs, res = run(_junqi_core_worker, cores, (per, burn, 20.0, args.seed), (seats,))
    rate = done / secs
    what = "acting-seat observation" if seats == 1 else "observations of all 4 seats"
    sample = (f"{cores} processes x {per} envs, {min(r[2] for r in res)}-{max(r[2] for r in res)} plies each after "
              f"a {burn}-ply burn-in, {what} + legal ids + step + 4-seat belief update, {secs:.1f} s")
    # the vectorised step + legal path alone (no observation, no beliefs), 64 envs per process
    one, one_s, _ = run(_batched_worker, 1, (64, 10.0, args.seed))
    allc, all_s, _ = run(_batched_worker, cores, (64, 10.0, args.seed))
    print(json.dumps({"impl": "reference-python", "metric": "env plies/s (step + legal mask + 317-ch obs)",
                      "value": rate, "unit": "plies/s", "n_gpus": 1, "higher_is_better": True,
                      "config": arm_config(cfg, args, 1),
                      "cpu_baseline": {"value": rate, "unit": "plies/s", "cores": cores, "kind": "reference",
                                       "sample": sample},
                      "step_legal_only": {"unit": "plies/s", "one_core": one / one_s, "all_cores": allc / all_s,
                                          "cores": cores,
                                          "sample": "BatchedGameState.step_batch + legal_action_ids_batch, 64 envs "
                                                    "per process, uniform legal actions, plies 50-349 of "
                                                    "fresh games, >= 10 s timed"},
                      "source": "junqi_core (GameState.step, ObservationBuilder.build_into, BeliefTensor.update) "
                                "from baseline/_ref"}), flush=True)


def reference_cuda_arm(args, cfg: dict) -> None:
    """The reference's own CUDA extension on this GPU -- a reported baseline,
    not part of the driver contract.  Built by baseline/build_ref_cuda.py
    into baseline/_ref; times the reference ``GpuRollout`` per-ply chain
    (gpu_collector.py:770-978: acting-seat observation, canonical mask,
    step_device, belief update, reset of finished games) with CUDA events
    around those calls only, the action choice (a masked argmax with keys
    that change every ply) left out."""
    import glob
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    so = glob.glob(str(ROOT / "baseline" / "_ref" / "junqi_rl" / "junqi_cuda*.so"))
    if not so:
        print(json.dumps({"impl": "reference-cuda", "unavailable": "baseline/_ref has no junqi_cuda build; "
                          "run baseline/build_ref_cuda.py where the reference checkout exists"}), flush=True)
        return
    sys.path.insert(0, str(ROOT / "baseline" / "_ref" / "junqi_rl"))
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    import torch
    from junqi_core.rules import ShowMode
    from junqi_rl.gpu_rollout import GpuRollout, _CudaArrayInterfaceView
    n, plies = args.envs or cfg["envs"], args.steps or cfg["plies"]
    if cfg["seats"] != 1:
        print(json.dumps({"impl": "reference-cuda", "unavailable": "only the acting-seat configs are timed"}))
        return
    ro = GpuRollout(num_envs=n, show_mode=ShowMode(cfg["mode"]), device_id=0)
    ro.reset_from_setup_pool(seed=args.seed)
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    keys = torch.randint(1, 32000, (16641,), device="cuda", dtype=torch.int32, generator=g)
    applied = torch.zeros((), dtype=torch.int64, device="cuda")
    evs = []
    for t in range(args.warmup + plies):
        acting = ro.turn_torch().clone()
        a = torch.cuda.Event(enable_timing=True)
        b1 = torch.cuda.Event(enable_timing=True)
        a.record()
        ro.build_acting_seat_observation_torch(acting)
        lm = ro.legal_mask_canonical_torch_device(acting)
        b1.record()
        acts = (lm.to(torch.int32) * torch.roll(keys, t)).argmax(dim=1).to(torch.int32)
        c = torch.cuda.Event(enable_timing=True)
        d = torch.cuda.Event(enable_timing=True)
        c.record()
        res = ro.step_device_torch(acts, acting)
        ro.update_beliefs_device(res, acting)
        ro.reset_terminated_device(seed=args.seed + 1_000_003 * (t + 1))
        d.record()
        if t >= args.warmup:
            valid = torch.as_tensor(_CudaArrayInterfaceView(ro._last_step_ptrs["d_valid_ptr"], (n,), "|b1"),
                                    device="cuda")
            applied += valid.sum()
            evs.append((a, b1, c, d))
    torch.cuda.synchronize()
    ms_obs = sum(a.elapsed_time(b1) for a, b1, c, d in evs)
    ms_step = sum(c.elapsed_time(d) for a, b1, c, d in evs)
    ms = ms_obs + ms_step
    done = int(applied)
    print(json.dumps({"impl": "reference-cuda", "metric": "env plies/s (step + legal mask + 317-ch obs)",
                      "value": done / (ms / 1e3), "unit": "plies/s", "n_gpus": 1, "steps": plies,
                      "warmup": args.warmup, "ms_per_step": ms / plies, "higher_is_better": True,
                      "split_ms_per_step": {"observation + canonical mask": ms_obs / plies,
                                            "step + beliefs + reset": ms_step / plies},
                      "config": {"workload": cfg["workload"], "envs_per_gpu": n, "plies_applied": done,
                                 "policy": "masked argmax over keys rotated every ply (not timed)",
                                 "chain": "build_acting_seat_observation_torch, legal_mask_canonical_torch_device, "
                                          "step_device_torch, update_beliefs_device, reset_terminated_device"},
                      "source": "reference junqi_cuda built for sm_100a by baseline/build_ref_cuda.py"}), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def arm_config(cfg: dict, args, world: int) -> dict:
    """The workload description both arms print (the reference arm times a
    bounded sample of this same workload; its sample is in cpu_baseline)."""
    return {"workload": cfg["workload"], "envs_per_gpu": cfg["envs"], "seats_per_env": cfg["seats"],
            "policy": cfg["policy"], "show_mode": "HALF_DARK", "rules": RULES_TEXT[args.rules],
            "burn_in_plies": args.burn_in,
            "l2": "per-step output (obs) > 1.5 GB >> 126 MB L2; no flush needed",
            "parallelism": f"env-sharded x{world} (weak)"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed plies (default: the config's plies)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--burn-in", type=int, default=200,
                    help="untimed plies played before the warm-up, so the timed plies sample a rollout's steady "
                         "mix of openings, combat, finished games and resets rather than only fresh games")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-cuda", "reference-python"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--envs", type=int, default=None, help="envs per GPU (default: the config's)")
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-pin", action="store_true", help="do not restrict each rank to its share of host cores")
    ap.add_argument("--collector", action="store_true",
                    help="time RolloutCollector (eager vs one CUDA graph per rollout) instead; one line per case")
    ap.add_argument("--rules", default="gamestate", choices=sorted(RULES),
                    help="turn-advance rules: GameState.step (default) or BatchedGameState.step_batch")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.envs:
        cfg["envs"] = args.envs
    if args.steps is None:
        args.steps = cfg["plies"]
    if args.impl == "reference-cuda":
        reference_cuda_arm(args, cfg)
        return
    if args.impl == "reference-python":
        reference_python_arm(args, cfg)
        return
    if args.impl == "reference":
        reference_arm(args, cfg)
        return
    if args.collector:
        collector_bench(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    from junqi_b200 import sharding
    cores = sharding.pin_rank_cores(local, local_world) if world > 1 and not args.no_pin else None
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    from junqi_b200 import _native
    from junqi_b200 import tables
    from junqi_b200.env import JunqiEnvB200
    _native.build()

    n, seats = cfg["envs"], cfg["seats"]
    seed = sharding.rank_seed(args.seed, rank)
    pool = tables.build_setup_pool(cfg["pool"], seed=42)
    env = JunqiEnvB200(n, device=local, show_mode=cfg["mode"], pool=pool, obs_seats=seats,
                       rules=RULES[args.rules])
    sampler = env.sample_uniform if cfg["policy"] == "uniform" else env.sample_softmax
    if cfg.get("start") == "late":
        from junqi_b200 import workloads
        workloads.late_game_starts(env, seed)
    else:
        env.reset(seed=seed)
    stream = torch.cuda.current_stream()

    def one_ply(t, ev=None):
        if ev is not None:
            ev[0].record(stream)
        env.observe()
        if ev is not None:
            ev[1].record(stream)
        acts = sampler(seed, t)
        if ev is not None:
            ev[2].record(stream)
        env.ply(acts, seed=seed, ply=t)
        if ev is not None:
            ev[3].record(stream)

    # clocks are sampled from the burn-in on, so the GPU never idles between
    # the warm-up and the timed plies (an idle gap lets it leave its loaded
    # state and slows the first timed plies)
    clock_rows, stop = [], threading.Event()
    th = threading.Thread(target=sample_clocks, args=(local, stop, clock_rows), daemon=True)
    th.start()
    t = 0
    for t in range(1, args.burn_in + 1):
        one_ply(t)
    for t in range(args.burn_in + 1, args.burn_in + args.warmup + 1):  # the timed loop's ops, events included
        one_ply(t, [torch.cuda.Event(enable_timing=True) for _ in range(4)] if t % EVENT_EVERY == 0 else None)
    t0_ply = t + 1
    env.stats.zero_()  # jq_ply counts plies applied and episode statistics on the device
    # Per-kernel CUDA events on every EVENT_EVERY-th timed ply (an event between
    # two kernels keeps the next launch from overlapping the previous one's
    # tail), from the 4th on: the first timed plies follow the synchronize
    # above, so their events would also time the host submitting the kernels
    # to an idle GPU.
    evs = {k: [torch.cuda.Event(enable_timing=True) for _ in range(4)]
           for k in range(min(EVENT_EVERY // 2, args.steps - 1), args.steps, EVENT_EVERY)}
    start, end, ar0 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        # Leave the barrier on the device: every GPU starts its timed plies
        # when this all-reduce completes on all of them, not when its host
        # got there, so host launch skew stays out of the max over ranks.
        align = torch.zeros(1, dtype=torch.int64, device=env.device)
        dist.all_reduce(align)
    t_wall = time.perf_counter()
    start.record(stream)
    for k in range(args.steps):
        one_ply(t0_ply + k, evs.get(k))
    ar0.record(stream)
    if world > 1:
        sharding.reduce_episode_stats(env.stats)  # one collective per rollout: episode statistics
    end.record(stream)
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    if world > 1:
        dist.barrier()
    ms_total = start.elapsed_time(end)
    obs_ms = [e[0].elapsed_time(e[1]) for e in evs.values()]
    ply_ms = [e[2].elapsed_time(e[3]) for e in evs.values()]
    stats = env.stats.cpu().numpy().tolist()  # summed over ranks inside the timed region
    ms_max = sharding.max_over_ranks(ms_total, env.device)
    plies_all = int(stats[5])
    value = plies_all / (ms_max / 1e3)

    k_avg = float(env.counts.sum(dtype=torch.int64).item()) / n  # legal actions per env, last ply

    # e2e through the public API with host buffers: H2D actions, D2H results + CSR, host policy
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(env, args, seed, stream)
    stop.set()
    th.join(timeout=10)
    mine = {"rank": rank, "device_ms": round(ms_total, 4), "plies_ms": round(start.elapsed_time(ar0), 4),
            "allreduce_ms": round(ar0.elapsed_time(end), 4),
            "obs_kernel_ms": round(statistics.mean(obs_ms), 4), "ply_kernel_ms": round(statistics.mean(ply_ms), 4),
            "host_cores": None if cores is None else len(cores)}
    if e2e is not None:
        mine.update({k: e2e.pop(k) for k in ("e2e_ms_per_step", "host_ms_per_step", "wait_ms_per_step")})
    per_rank = sharding.gather_over_ranks(mine)
    if rank == 0:
        peak, peak_kind = peak_hbm()
        units = n * seats
        obs_bytes = units * (OBS_WRITE + obs_read_bytes())
        obs_avg = statistics.mean(obs_ms)
        achieved = obs_bytes / (obs_avg / 1e3) / 1e9
        traffic_unit = profiled_traffic(args.config)
        config = arm_config(cfg, args, world)
        config["timed_plies"] = f"{t0_ply}..{t0_ply + args.steps - 1} of each env batch's rollout"
        line = {
            "metric": "env plies/s (step + legal mask + 317-ch obs)", "value": value, "unit": "plies/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/int16/f32",
            "data": "synthetic (seeded setup pool of random legal lineups, seeded policy)",
            "config": config,
            "plies_applied": plies_all, "plies_offered": n * world * args.steps,
            "roofline": {"bound": "hbm", "kernel": "obs_kernel", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": None if traffic_unit is None else traffic_unit * units,
                         "algorithmic_bytes_per_launch": obs_bytes, "avg_launch_ms": obs_avg,
                         "ply_kernel_avg_ms": statistics.mean(ply_ms)},
            "pipeline": pipeline_roofline(value / world, seats, k_avg, peak),
            "clocks": summarize_clocks(clock_rows),
            "gpu_launches": 3 * args.steps,  # obs_kernel + sample kernel + rules_kernel per ply
            "kernel_timing": f"CUDA events around each kernel on every {EVENT_EVERY}th timed ply from the "
                             f"{min(EVENT_EVERY // 2, args.steps - 1)}th ({len(obs_ms)} plies)",
            "episode_stats": {"wins_team0": stats[0], "wins_team1": stats[1], "draws": stats[2],
                              "episodes": stats[3], "sum_len": stats[4]},
            "per_rank": per_rank,
            "wall_s": t_wall,
        }
        if e2e is not None:
            line["e2e"] = e2e
        if not args.no_cpu_baseline:
            threads = host_cores()
            rate, done, dt, sample = cpu_rollout(min(n, 64 * threads), 400, seats, args.seed, threads, 15.0,
                                                 RULES[args.rules], late=cfg.get("start") == "late",
                                                 burn_in=min(args.burn_in, 100))
            line["cpu_baseline"] = {"value": rate, "unit": "plies/s", "cores": threads, "kind": "port",
                                    "sample": sample + f", {dt:.1f} s"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(env, args, seed, stream) -> dict:
    """Same metric through the public API with host buffers every step.

    Per ply the host picks actions from the previous ply's CSR, uploads them
    from pinned memory, launches ply + CSR + observation, and reads back the
    MoveResult and the CSR -- one copy of a prefix of the env's io buffer,
    which holds the results, the offsets and the values in that order -- on
    a side stream as soon as the CSR is built, while the observation kernel
    keeps running on the main stream.  The values are read up to a bound
    that grows with the largest CSR seen, so the host blocks once per ply; a
    CSR beyond the bound costs a second, rare, read."""
    import torch
    n = env.n
    np_type = {torch.uint8: np.uint8, torch.int8: np.int8, torch.int32: np.int32, torch.int64: np.int64,
               torch.float32: np.float32}
    acts_h = torch.empty(n, dtype=torch.int32, pin_memory=True)
    io_h = torch.empty(env.io.numel(), dtype=torch.uint8, pin_memory=True)
    io_np = io_h.numpy()

    def view(t):  # the host image of a view of env.io
        o = t.data_ptr() - env.io.data_ptr()
        return io_np[o:o + t.numel() * t.element_size()].view(np_type[t.dtype])

    off_np, val_np, valid_np = view(env.offsets), view(env.values), view(env.out["valid"])
    acts_d = torch.empty(n, dtype=torch.int32, device=env.device)
    rng = np.random.default_rng(seed)
    env.legal()
    env.csr()
    torch.cuda.synchronize()
    io_h[: env.io_prefix_bytes(0)].copy_(env.io[: env.io_prefix_bytes(0)])
    tot = int(off_np[-1])
    io_h[: env.io_prefix_bytes(tot)].copy_(env.io[: env.io_prefix_bytes(tot)])
    bound = min(n * env.cap, max(4 * n, tot + tot // 4))
    applied, h2d, d2h, extra_reads = 0, 0, 0, 0
    steps = args.e2e_steps
    host_s = wait_s = 0.0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    copy_stream = torch.cuda.Stream(device=env.device)
    csr_done, acts_up, copies_done = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
    torch.cuda.synchronize()
    import torch.distributed as dist
    if dist.is_initialized():
        dist.barrier()
    start.record(stream)
    for t in range(steps):
        h0 = time.perf_counter()
        cnt = np.diff(off_np)
        pick = (rng.random(n) * np.maximum(cnt, 1)).astype(np.int64)
        acts_h.numpy()[:] = np.where(cnt > 0, val_np[np.minimum(off_np[:-1] + pick, max(int(off_np[-1]) - 1, 0))],
                                     -1)
        with torch.cuda.stream(copy_stream):  # upload under the observation kernel still running
            acts_d.copy_(acts_h, non_blocking=True)
            acts_up.record(copy_stream)
        h2d += n * 4
        stream.wait_event(acts_up)
        env.ply(acts_d, seed=seed, ply=100_000 + t)
        env.csr()
        csr_done.record(stream)
        env.observe()
        nb = env.io_prefix_bytes(bound)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(csr_done)
            io_h[:nb].copy_(env.io[:nb], non_blocking=True)
            copies_done.record(copy_stream)
        d2h += nb
        h1 = time.perf_counter()
        copies_done.synchronize()  # the one blocking wait of the ply
        h2 = time.perf_counter()
        tot = int(off_np[-1])
        if tot > bound:  # a CSR larger than any seen so far
            nt = env.io_prefix_bytes(tot)
            with torch.cuda.stream(copy_stream):
                io_h[nb:nt].copy_(env.io[nb:nt], non_blocking=True)
            copy_stream.synchronize()
            d2h += nt - nb
            extra_reads += 1
            bound = min(n * env.cap, tot + tot // 4)
        applied += int(valid_np.sum(dtype=np.int64))
        host_s += (h1 - h0) + (time.perf_counter() - h2)
        wait_s += h2 - h1
    end.record(stream)
    torch.cuda.synchronize()
    from junqi_b200 import sharding
    ms_own = start.elapsed_time(end)
    ms = sharding.max_over_ranks(ms_own, env.device)
    applied = sharding.sum_over_ranks(applied, env.device)
    return {"value": applied / (ms / 1e3), "unit": "plies/s", "h2d_bytes_per_step": h2d // steps,
            "d2h_bytes_per_step": d2h // steps, "steps": steps, "extra_csr_reads": extra_reads,
            "e2e_ms_per_step": round(ms_own / steps, 4), "host_ms_per_step": round(host_s * 1e3 / steps, 4),
            "wait_ms_per_step": round(wait_s * 1e3 / steps, 4),
            "api": "JunqiEnvB200.ply/csr/observe with pinned host actions in; MoveResult + CSR out as one read "
                   "per ply on a side stream, overlapping the observation kernel"}


class _ArgmaxPolicy:
    """Stand-in for a network: masked argmax over fixed random per-action
    scores (one pass over the canonical mask), so the collector's own cost
    shows."""

    def __init__(self, device):
        import torch
        g = torch.Generator(device="cpu").manual_seed(0)
        self.score = torch.rand(16641, generator=g).to(device)

    def __call__(self, sp, gl, mask):
        import torch
        v, a = torch.where(mask, self.score, -1.0).max(1)
        return a, v, gl[:, 0]


def collector_bench(args) -> None:
    """RolloutCollector throughput, eager against one CUDA graph per
    rollout (GameState rules, HALF_DARK, compact history on): one JSON line
    per (envs, mode).  --envs sets the batch (default 256 and 4096), --steps
    the plies per rollout (default 64)."""
    import torch
    from junqi_b200 import _native as N
    from junqi_b200 import tables
    from junqi_b200.collector import RolloutCollector
    from junqi_b200.env import HALF_DARK, JunqiEnvB200
    N.build()
    pool = tables.build_setup_pool(1024, seed=2)
    plies = args.steps if args.steps and args.steps != CONFIGS[args.config]["plies"] else 64
    for n in ([args.envs] if args.envs else [256, 4096]):
        for graph in (False, True):
            env = JunqiEnvB200(n, show_mode=HALF_DARK, pool=pool, rules=N.RULES_GAMESTATE)
            env.reset(seed=1)
            col = RolloutCollector(env, _ArgmaxPolicy(env.device), plies, seed=3, graph=graph)
            for _ in range(max(1, args.warmup // 5)):
                col.collect()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(3):
                col.collect()
            t1.record()
            torch.cuda.synchronize()
            ms = t0.elapsed_time(t1) / 3
            print(json.dumps({"collector": True, "envs": n, "plies": plies, "graph": graph,
                              "ms_per_rollout": round(ms, 3), "plies_per_s": round(plies * n / ms * 1e3)}),
                  flush=True)


if __name__ == "__main__":
    main()
