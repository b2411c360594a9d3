"""CPU-side checks of the product library and host code (no GPU needed).

* libjq.so loads and exports every entry point include/jq.h declares;
* the board tables the kernels use equal junqi_core's;
* host-generated tables (Zobrist, belief prior, setups, pool) equal the
  reference's, so hashes and resets can match bit for bit.
"""
from __future__ import annotations

import random
import re
from pathlib import Path

import numpy as np
import pytest

from junqi_b200 import _native as N
from junqi_b200 import tables
from tests import _golden as G

ROOT = Path(__file__).resolve().parent.parent


def header_symbols() -> list[str]:
    text = (ROOT / "include" / "jq.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(jq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    N.build()
    L = N.lib()
    syms = header_symbols()
    assert len(syms) >= 18
    for s in syms:
        assert hasattr(L, s), f"libjq.so does not export {s}"
    assert set(syms) <= set(N.SIGNATURES), "binding lacks a declared entry point"
    assert L.jq_abi_version() == 7


def test_kernel_board_tables_match_reference():
    L = N.lib()
    o = {k: np.zeros(s, np.int32) for k, s in [("on", 289), ("rail", 289), ("curve", 289), ("adj", (289, 4)),
                                               ("sr", (289, 4, 12)), ("cr", (289, 2, 11)), ("c2f", 129),
                                               ("fl", 289)]}
    L.jq_topology_dump(*[o[k].ctypes.data for k in ("on", "rail", "curve", "adj", "sr", "cr", "c2f", "fl")])
    ref = G.tables()
    for mine, r in (("on", "on_board"), ("rail", "rail"), ("curve", "curve"), ("adj", "rail_adj"),
                    ("sr", "srays"), ("cr", "crays"), ("c2f", "compact_to_flat")):
        assert np.array_equal(o[mine], ref[r]), r
    assert np.array_equal(o["fl"] & 1, ref["camp"])
    assert np.array_equal((o["fl"] >> 1) & 1, ref["stronghold"])
    assert np.array_equal((o["fl"] >> 3) & 1, ref["nine"])
    assert np.array_equal((o["fl"] >> 4) & 1, ref["arc"])


def test_host_tables_match_reference():
    ref = G.tables()
    assert np.array_equal(tables.prior_table(), ref["prior"])
    z = tables.zobrist_tables()
    man = G.manifest()["zobrist"]
    for mine, r in (("piece", "ZOB_PIECE"), ("turn", "ZOB_TURN"), ("move_counter", "ZOB_MOVE_COUNTER"),
                    ("mslc", "ZOB_MOVES_SINCE_COMBAT"), ("winner", "ZOB_WINNER"), ("seat_dead", "ZOB_SEAT_DEAD"),
                    ("seat_flag", "ZOB_SEAT_FLAG_REVEALED"), ("show_mode", "ZOB_SHOW_MODE")):
        assert G.sha(z[mine]) == man[r], r
    assert str(int(z["terminated"][0])) == man["ZOB_TERMINATED"]


def test_setup_generator_and_pool_match_reference():
    ref = G.tables()
    assert np.array_equal(tables.build_setup_pool(64, 42), ref["pool64"])
    got = np.stack([tables.random_setup(random.Random(s)) for s in range(32)])
    assert np.array_equal(got, ref["setups_seed0_31"])
    tables.validate_pool(got)


@pytest.mark.parametrize("slot,t,code", [(6, 5, "C1"), (0, 3, "C3"), (1, 4, "C4")])
def test_pool_validation_rejects_illegal_lineups(slot, t, code):
    pool = tables.build_setup_pool(2, 3)
    bad = pool.copy()
    bad[1, slot] = t
    with pytest.raises(ValueError, match=code):
        tables.validate_pool(bad)


def test_pool_index_is_deterministic_and_in_range():
    L = N.lib()
    idx = [L.jq_pool_index(7, 3, e, 97) for e in range(200)]
    assert all(0 <= i < 97 for i in idx)
    assert idx == [L.jq_pool_index(7, 3, e, 97) for e in range(200)]
    assert len(set(idx)) > 50
    assert L.jq_pool_index(7, 3, 0, 0) == -1


def test_entry_points_reject_bad_arguments_without_a_gpu():
    L = N.lib()
    assert L.jq_init(-1) == 1
    assert L.jq_csr(0, None, None, 0, None, None, None, None) == 1
    assert L.jq_sample_uniform(0, None, None, 0, 0, 0, None, None) == 1
    assert b"bad" in L.jq_last_error() or len(L.jq_last_error()) > 0


def test_history_record_is_compact_and_aligned():
    """One rollout-history record per (step, env): 16-byte aligned, and far
    smaller than the 366 KB observation it rebuilds."""
    size = N.lib().jq_history_record_bytes()
    assert size % 16 == 0 and 8_000 <= size <= 16_384


def test_no_host_pointer_is_taken_from_a_temporary_array():
    """``f(make_table().ctypes.data)`` hands the library a pointer into an
    array CPython frees before the call runs (only the integer survives);
    the C side then copies freed, possibly reused, heap memory -- a device
    table uploaded that way is corrupt for the rest of the process.  Host
    code must keep every array it passes by pointer in a named variable."""
    import re
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    bad = []
    for p in [*sorted((root / "junqi_b200").glob("*.py")), root / "bench.py", root / "__graft_entry__.py"]:
        for i, line in enumerate(p.read_text().splitlines(), 1):
            if re.search(r"\)\s*\.ctypes\.data\b", line):
                bad.append(f"{p.name}:{i}: {line.strip()}")
    assert not bad, "pointers taken from temporaries:\n" + "\n".join(bad)


def test_trace_points_hold_no_warp_collectives():
    """The rules kernel's trace points run on lane 0 of one warp only
    (`traced`); a warp barrier, ballot or shuffle inside such a block would
    wait for 31 lanes that never arrive and hang the kernel -- in the
    normal build too, where only the stores are compiled out."""
    import re
    from pathlib import Path
    csrc = Path(__file__).resolve().parent.parent / "junqi_b200" / "csrc"
    collective = re.compile(r"__syncwarp|__ballot_sync|__shfl|__any_sync|__all_sync|__reduce_|bar_sync|bar_arrive|"
                            r"__syncthreads")
    bad = []
    for p in sorted(csrc.glob("*.cu*")):
        lines = p.read_text().splitlines()
        for i, line in enumerate(lines):
            if not re.search(r"\bif \(traced\)", line):
                continue
            body = [line]
            if line.rstrip().endswith("{"):
                depth, j = 1, i + 1
                while depth and j < len(lines):
                    depth += lines[j].count("{") - lines[j].count("}")
                    body.append(lines[j])
                    j += 1
            if any(collective.search(b) for b in body):
                bad.append(f"{p.name}:{i + 1}")
    assert not bad, "warp collectives inside lane-0 trace blocks: " + ", ".join(bad)
