"""Per-CTA timelines of the observation and rules kernels (tracing build).

    python -m junqi_b200.trace [--envs 4096] [--plies 200]
    python -m junqi_b200.trace --sweep

builds libjq_trace.so (the library compiled with JQ_TRACE: one %globaltimer
store per CTA at a few points of each kernel, jq_trace.cuh), plays a
configs[1]-style rollout (acting-seat observation, uniform policy, GameState
rules) and prints, for the last ply's observation and rules launches, where
their time goes: CTA start spread, wait for the previous kernel, the first
unit's staging before any store, the streaming span and the tail.  With
--sweep it times instead (CUDA events, plain libjq.so) one observation and
one ply launch at 1,024 ... 32,768 envs after a 200-ply burn-in, the median
of 20 launches each, so the fixed and per-unit parts of each kernel's time
can be separated.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import _native as N

OBS, RULES = 0, 1


POINTS = 20


def read(kernel: int, ctas: int) -> np.ndarray:
    """(ctas, POINTS) uint64 timestamps (and counts) of the last launch of `kernel`."""
    out = np.zeros((ctas, POINTS), np.uint64)
    N.check(N.lib().jq_trace_read(kernel, out.ctypes.data, ctas), "jq_trace_read")
    return out


def obs_timeline(t: np.ndarray) -> dict:
    """Observation-kernel phases in microseconds from the first CTA's entry."""
    t = t.astype(np.int64)
    t0 = t[:, 0].min()
    us = lambda a: (a - t0) / 1e3  # noqa: E731
    end = t[:, 5].max()
    return {"ctas": int(len(t)), "span_us": (end - t0) / 1e3,
            "entry_spread_us": float(us(t[:, 0]).max()),
            "waited_us_median": float(np.median(us(t[:, 1]))),
            "first_staged_us_median": float(np.median(us(t[:, 2]))),
            "first_stream_us_median": float(np.median(us(t[:, 3]))),
            "first_stream_us_max": float(us(t[:, 3]).max()),
            "last_streamed_us_min": float(us(t[:, 4]).min()),
            "last_streamed_us_median": float(np.median(us(t[:, 4]))),
            "exit_us_min": float(us(t[:, 5]).min()), "exit_us_max": float(us(t[:, 5]).max()),
            "units_per_cta_min": int(t[:, 6].min()), "units_per_cta_max": int(t[:, 6].max()),
            # units 1 and 2 of every CTA (us, median over CTAs and the two units): streaming warp 0
            # waiting for the staged buffer, streaming; staging one unit (start to staged)
            "steady_unit_us": _steady(t),
            # the tail: exits after the last ticket was taken (T0), split by whether the CTA
            # still had a staged unit waiting behind the one it was streaming at T0
            "tail_after_last_ticket_us": _tail(t)}


def _steady(t: np.ndarray) -> dict:
    """Per-unit phases of the CTAs' units 1 and 2 from the raw stamps."""
    ok = t[:, 6] >= 4
    u = t[ok].astype(np.int64)
    wait = np.concatenate([u[:, 11] - u[:, 10], u[:, 13] - u[:, 12]]) / 1e3
    stream = np.concatenate([u[:, 12] - u[:, 11], u[:, 14] - u[:, 13]]) / 1e3
    stage = (u[:, 17] - u[:, 18]) / 1e3  # unit 2: began after its free-buffer barrier, staged
    return {"stream_wait": round(float(np.median(wait)), 2), "stream": round(float(np.median(stream)), 2),
            "stage_unit2": round(float(np.median(stage)), 2), "ctas": int(ok.sum())}


def _tail(t: np.ndarray) -> dict:
    """Exits after T0, the moment the last unit's ticket was taken; for the
    CTAs that exit last, when they took their own last ticket and finished
    staging it, relative to T0 (us)."""
    took = t[:, 7] > 0
    t0 = t[took, 7].max() if took.any() else t[:, 5].min()
    rel = lambda a: (a - t0) / 1e3  # noqa: E731
    after = rel(t[:, 5])
    last = np.argsort(after)[-6:]
    return {"exit_after_t0_p10_p50_max": [round(float(np.percentile(after, 10)), 1),
                                          round(float(np.median(after)), 1), round(float(after.max()), 1)],
            "latest_exits": [{"exit": round(float(after[i]), 1), "last_ticket": round(float(rel(t[i, 7])), 1),
                              "last_staged": round(float(rel(t[i, 8])), 1), "units": int(t[i, 6])} for i in last]}


def rules_timeline(t: np.ndarray) -> dict:
    """Rules-kernel CTA exits, and the phases of each CTA's warp-0 env (us,
    median / p90 / max over CTAs)."""
    t = t.astype(np.int64)
    t0 = t[:, 0].min()
    us = lambda a: (a - t0) / 1e3  # noqa: E731
    out = {"ctas": int(len(t)), "span_us": float(us(t[:, 7]).max()),
           "waited_us_median": float(np.median(us(t[:, 1]))),
           "exit_us_min": float(us(t[:, 7]).min()), "exit_us_median": float(np.median(us(t[:, 7]))),
           "exit_us_p90": float(np.percentile(us(t[:, 7]), 90)), "exit_us_max": float(us(t[:, 7]).max())}
    for name, a, b in (("load", 1, 2), ("step", 2, 3), ("step_scalar", 2, 8), ("step_combat", 8, 9),
                       ("step_q12", 9, 10), ("step_commit", 10, 11), ("step_beliefs", 11, 3), ("reset", 3, 4),
                       ("legal_ids", 4, 5), ("legal_dsts", 4, 14), ("legal_rank", 14, 15), ("legal_store", 15, 5),
                       ("mask", 5, 6), ("env_total", 1, 6)):
        d = (t[:, b] - t[:, a]) / 1e3
        out[name + "_us"] = [round(float(np.median(d)), 2), round(float(np.percentile(d, 90)), 2),
                             round(float(d.max()), 2)]
    # the slowest envs: their phases, event and Q12 full scans
    slow = np.argsort((t[:, 6] - t[:, 1]))[-5:]
    out["slowest"] = [{"total": round((t[i, 6] - t[i, 1]) / 1e3, 1), "load": round((t[i, 2] - t[i, 1]) / 1e3, 1),
                       "scalar": round((t[i, 8] - t[i, 2]) / 1e3, 1), "combat": round((t[i, 9] - t[i, 8]) / 1e3, 1),
                       "q12": round((t[i, 10] - t[i, 9]) / 1e3, 1), "commit": round((t[i, 11] - t[i, 10]) / 1e3, 1),
                       "beliefs": round((t[i, 3] - t[i, 11]) / 1e3, 1), "ids": round((t[i, 5] - t[i, 4]) / 1e3, 1),
                       "dsts": round((t[i, 14] - t[i, 4]) / 1e3, 1), "rank": round((t[i, 15] - t[i, 14]) / 1e3, 1),
                       "mask": round((t[i, 6] - t[i, 5]) / 1e3, 1), "event": int(t[i, 12]),
                       "q12_scans": int(t[i, 13]), "path": round((t[i, 16] - t[i, 2]) / 1e3, 1),
                       "path_rounds": int(t[i, 17]), "piece_type": int(t[i, 18]),
                       "legal": _legal_shape(t[i, 19])} for i in slow]
    # destination-set time against the legal set's shape
    dst = (t[:, 14] - t[:, 4]) / 1e3
    shape = [_legal_shape(v) for v in t[:, 19]]
    tot = np.array([s["total"] for s in shape])
    eng = np.array([s["engineer_max"] for s in shape])
    out["legal_dsts_by_shape"] = {
        "total_moves_p50_max": [int(np.median(tot)), int(tot.max())],
        "corr_dsts_total": _corr(dst, tot),
        "corr_dsts_engineer_max": _corr(dst, eng),
        "dsts_us_p50_by_total_quartile": [round(float(np.median(dst[(tot >= a) & (tot <= b)])), 2)
                                          for a, b in zip(np.percentile(tot, [0, 25, 50, 75]),
                                                          np.percentile(tot, [25, 50, 75, 100]))],
        "dsts_us_p50_engineer_max_ge_20_vs_lt": [round(float(np.median(dst[eng >= 20])), 2) if (eng >= 20).any() else None,
                                                 round(float(np.median(dst[eng < 20])), 2) if (eng < 20).any() else None]}
    # the engineer path check: how many envs ran it, its rounds and time, and
    # the scalar part with and without it
    ran = t[:, 17] > 0
    path = (t[:, 16] - t[:, 2]) / 1e3
    scal = (t[:, 8] - t[:, 2]) / 1e3
    out["path_check"] = {"envs": int(ran.sum()), "of": int(len(t)),
                         "rounds_p50_max": [int(np.median(t[ran, 17])), int(t[ran, 17].max())] if ran.any() else [],
                         "us_p50_max": [round(float(np.median(path[ran])), 2), round(float(path[ran].max()), 2)]
                         if ran.any() else [],
                         "scalar_us_with_p50_max": [round(float(np.median(scal[ran])), 2), round(float(scal[ran].max()), 2)]
                         if ran.any() else [],
                         "scalar_us_without_p50_max": [round(float(np.median(scal[~ran])), 2),
                                                       round(float(scal[~ran].max()), 2)]}
    return out


def _corr(a: np.ndarray, b: np.ndarray):
    """Pearson correlation rounded to 0.01, None when either side is constant."""
    if a.std() == 0 or b.std() == 0:
        return None
    return round(float(np.corrcoef(a, b)[0, 1]), 2)


def _legal_shape(v) -> dict:
    """The packed legal-set shape of one traced env (tracing build)."""
    v = int(v)
    return {"engineers": v >> 48, "engineer_max": (v >> 32) & 0xFFFF, "piece_max": (v >> 16) & 0xFFFF,
            "total": v & 0xFFFF}


def sweep() -> None:
    import torch

    from . import tables
    from .env import JunqiEnvB200
    N.build()
    pool = tables.build_setup_pool(10_000, seed=42)
    for n in (1024, 2048, 4096, 8192, 16384, 32768):
        env = JunqiEnvB200(n, pool=pool, rules=N.RULES_GAMESTATE)
        env.reset(seed=5)
        for t in range(1, 201):
            env.ply(env.sample_uniform(5, t), seed=5, ply=t)
        s = torch.cuda.current_stream()
        res = {}
        for what in ("obs", "ply"):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(42)]
            for i in range(21):
                a = env.sample_uniform(5, 300 + i) if what == "ply" else None
                ev[2 * i].record(s)
                env.observe() if what == "obs" else env.ply(a, seed=5, ply=300 + i)
                ev[2 * i + 1].record(s)
            torch.cuda.synchronize()
            res[what] = sorted(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(1, 21))[10]
        print(json.dumps({"envs": n, "obs_ms": round(res["obs"], 4), "ply_ms": round(res["ply"], 4),
                          "obs_GBps": round(n * 376_480 / (res["obs"] / 1e3) / 1e9, 1)}), flush=True)
        del env
        torch.cuda.empty_cache()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--envs", type=int, default=4096)
    ap.add_argument("--plies", type=int, default=200)
    ap.add_argument("--sweep", action="store_true", help="time both kernels over a range of batch sizes")
    args = ap.parse_args()
    if args.sweep:
        sweep()
        return
    N.build(trace=True)
    N.use_trace_library()
    import torch

    from . import tables
    from .env import JunqiEnvB200
    env = JunqiEnvB200(args.envs, pool=tables.build_setup_pool(10_000, seed=42), rules=N.RULES_GAMESTATE)
    env.reset(seed=7)
    for t in range(1, args.plies + 1):
        env.observe()
        env.ply(env.sample_uniform(7, t), seed=7, ply=t)
    torch.cuda.synchronize()
    env.observe()
    torch.cuda.synchronize()
    dev = torch.cuda.current_device()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    obs_ctas = min(2 * sms, args.envs)
    rule_ctas = min((args.envs + 7) // 8, 1024)
    print(json.dumps({"kernel": "obs_kernel", "units": args.envs, **obs_timeline(read(OBS, obs_ctas))}))
    print(json.dumps({"kernel": "rules_kernel", "envs": args.envs, **rules_timeline(read(RULES, rule_ctas))}))


if __name__ == "__main__":
    main()
