"""Host-side analysis of the tracing build's stamp tables (junqi_b200/trace.py),
on synthetic tables: the phase arithmetic, the per-unit stamps of the
observation kernel and the packed legal-set shape.  No GPU."""
import json

import numpy as np

from junqi_b200 import trace


def _obs_table(ctas=6, units=5):
    t = np.zeros((ctas, trace.POINTS), np.uint64)
    base = 1_000_000
    for c in range(ctas):
        t[c, 0] = base + 10 * c              # entry
        t[c, 1] = base + 2_000               # wait passed
        t[c, 2] = base + 9_000               # first unit staged
        t[c, 3] = base + 9_500               # first store
        t[c, 4] = base + 9_500 + units * 18_000  # last unit streamed
        t[c, 5] = int(t[c, 4]) + 100         # exit
        t[c, 6] = units
        t[c, 7] = base + 80_000 + c          # last ticket
        t[c, 8] = base + 90_000 + c          # last unit staged
        # units 0..2: passed the staged-buffer barrier, streamed (18 us each, 1 us wait)
        for k in range(3):
            t[c, 9 + 2 * k] = base + 9_500 + k * 19_000
            t[c, 10 + 2 * k] = base + 9_500 + k * 19_000 + 18_000
        for k in range(3):
            t[c, 15 + k] = base + 9_000 + k * 19_000
        t[c, 18] = base + 9_000 + 2 * 19_000 - 17_000  # unit 2 began: staged 17 us later
        t[c, 19] = base + 9_000 + 3 * 19_000 - 17_000
    return t


def test_obs_timeline_phases():
    out = trace.obs_timeline(_obs_table())
    json.dumps(out)  # the tool prints it as one JSON line
    assert out["ctas"] == 6
    assert abs(out["waited_us_median"] - 2.0) < 0.1
    assert abs(out["first_staged_us_median"] - 9.0) < 0.1
    assert out["units_per_cta_min"] == out["units_per_cta_max"] == 5
    st = out["steady_unit_us"]
    assert st["ctas"] == 6
    assert abs(st["stream"] - 18.0) < 1e-6 and abs(st["stream_wait"] - 1.0) < 1e-6
    assert abs(st["stage_unit2"] - 17.0) < 1e-6


def test_legal_shape_unpacks_the_packed_counts():
    v = (3 << 48) | (41 << 32) | (41 << 16) | 117
    assert trace._legal_shape(np.uint64(v)) == {"engineers": 3, "engineer_max": 41, "piece_max": 41, "total": 117}


def test_rules_timeline_phases_and_slowest_envs():
    ctas = 8
    t = np.zeros((ctas, trace.POINTS), np.uint64)
    for c in range(ctas):
        b = 5_000_000 + c
        # entry, waited, loaded, stepped, reset, ids, masked, exit
        for i, us in enumerate([0, 26, 33, 41, 42, 52, 57, 60]):
            t[c, i] = b + us * 1000 + (c * 100 if i >= 6 else 0)
        t[c, 8] = b + 35_000   # scalar part done
        t[c, 9] = b + 36_000   # combat memory done
        t[c, 10] = b + 38_000  # Q12 done
        t[c, 11] = b + 38_500  # commit done
        t[c, 12] = 1 + c % 4   # event
        t[c, 13] = 0
        t[c, 14] = b + 49_000  # destination sets done
        t[c, 15] = b + 50_000  # ranked
        t[c, 16] = b + 34_000  # path check done
        t[c, 17] = 7 if c % 2 else 0  # path-check rounds
        t[c, 18] = 13
        t[c, 19] = (1 << 48) | ((10 + 10 * c) << 32) | (30 << 16) | (60 + c)
    out = trace.rules_timeline(t)
    json.dumps(out)
    assert out["ctas"] == ctas
    assert out["load_us"][0] == 7.0 and out["legal_dsts_us"][0] == 7.0
    assert len(out["slowest"]) == 5 and out["slowest"][-1]["legal"]["engineer_max"] == 80
    assert out["path_check"]["envs"] == ctas // 2 and out["path_check"]["rounds_p50_max"] == [7, 7]
    assert out["legal_dsts_by_shape"]["total_moves_p50_max"][1] == 60 + ctas - 1
    assert out["legal_dsts_by_shape"]["corr_dsts_total"] is None  # every env took the same 7 us
