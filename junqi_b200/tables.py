"""Host-side tables and setup generation.

These reproduce, with the same library calls in the same order, the
numbers the reference derives on the host, so hashes, observations and
setups match bit for bit:

* ``zobrist_tables`` -- junqi_core/_zobrist.py:80-122 (numpy PCG64 seeded
  with the ASCII of "JUNQI_ZO", ten draws in a fixed order);
* ``prior_table`` -- info_model.py:64-146, the per-slot belief prior
  ``counts / counts.sum()`` in float32;
* ``recency_lut`` -- observation.py:1549-1562, ``exp(-elapsed/tau)`` in
  float32 for elapsed in [0, 4096] and tau in (32, 256, 64, 128);
* ``random_lineup`` / ``random_setup`` -- setup.py:162-263, driven by a
  ``random.Random`` exactly as the reference drives it;
* ``build_setup_pool`` -- gpu_rollout.py:255-275, (P, 120) int8 piece types
  per pid.
"""
from __future__ import annotations

import random

import numpy as np

ZOBRIST_SEED = 0x4A554E51495F5A4F

# rules.py:131-144 counts in tracked-type order JUNQI..GONGB (types 2..13)
PIECE_COUNTS = (1, 3, 2, 1, 1, 2, 2, 2, 2, 3, 3, 3)
CAMP_SLOTS = (6, 8, 12, 16, 18)
STRONGHOLD_SLOTS = (26, 28)


def zobrist_tables() -> dict:
    rng = np.random.default_rng(ZOBRIST_SEED)

    def draw(shape):
        return rng.integers(0, np.iinfo(np.uint64).max, size=shape, dtype=np.uint64,
                            endpoint=True).astype(np.int64)

    names = [("piece", (120, 14, 289)), ("turn", (4,)), ("move_counter", (4096,)),
             ("mslc", (512,)), ("terminated", (1,)), ("winner", (3,)), ("draw", (1,)),
             ("seat_dead", (4,)), ("seat_flag", (4,)), ("show_mode", (4,))]
    return {k: np.ascontiguousarray(draw(s)) for k, s in names}


def prior_table() -> np.ndarray:
    out = np.zeros((30, 12), np.float32)
    for slot in range(30):
        if slot in CAMP_SLOTS:
            continue
        vec = np.zeros(12, np.float32)
        for ti, cnt in enumerate(PIECE_COUNTS):
            t = ti + 2
            if slot not in STRONGHOLD_SLOTS:
                if t == 2 or (t == 3 and slot < 20) or (t == 4 and slot < 5):
                    continue
            vec[ti] = float(cnt)
        out[slot] = np.asarray(vec / vec.sum(), dtype=np.float32)
    return out


def uniform12() -> np.ndarray:
    return np.full(12, 1.0 / 12, dtype=np.float32)


def recency_lut() -> np.ndarray:
    el = np.arange(4097).astype(np.float32)
    return np.ascontiguousarray(np.stack(
        [np.exp(-np.maximum(el, 0.0) / tau, dtype=np.float32) for tau in (32.0, 256.0, 64.0, 128.0)]
    ).astype(np.float32))


# ---------------------------------------------------------------------------
# Setups
# ---------------------------------------------------------------------------
_INVENTORY_ORDER = tuple(range(2, 14))  # PIECE_COUNTS iteration order (rules.py:131-144)


def random_lineup(rng: random.Random) -> list[int]:
    """One seat's 30-slot lineup (piece type per slot, 0 on camps)."""
    flag_slot = rng.choice(sorted(STRONGHOLD_SLOTS))
    inventory = dict(zip(_INVENTORY_ORDER, PIECE_COUNTS))
    inventory[2] -= 1
    free = [i for i in range(30) if i not in CAMP_SLOTS and i != flag_slot]
    rng.shuffle(free)
    dilei_ok = [i for i in free if i >= 20]
    zhadan_ok = [i for i in free if i >= 5]
    place = {flag_slot: 2}
    rng.shuffle(dilei_ok)
    chosen_d = dilei_ok[:inventory[3]]
    for i in chosen_d:
        place[i] = 3
    inventory[3] = 0
    used = set(chosen_d)
    zhadan_ok = [i for i in zhadan_ok if i not in used]
    rng.shuffle(zhadan_ok)
    chosen_z = zhadan_ok[:inventory[4]]
    for i in chosen_z:
        place[i] = 4
    inventory[4] = 0
    used.update(chosen_z)
    rest = [i for i in free if i not in used]
    rng.shuffle(rest)
    pieces = []
    for t, c in inventory.items():
        pieces.extend([t] * c)
    rng.shuffle(pieces)
    for s, t in zip(rest, pieces, strict=True):
        place[s] = t
    for i in CAMP_SLOTS:
        place[i] = 0
    return [place[i] for i in range(30)]


def random_setup(rng: random.Random) -> np.ndarray:
    """Four lineups flattened to piece types per pid (seat*30 + slot)."""
    return np.array([t for _ in range(4) for t in random_lineup(rng)], dtype=np.int8)


def build_setup_pool(pool_size: int, seed: int = 42) -> np.ndarray:
    rng = random.Random(seed)
    return np.stack([random_setup(rng) for _ in range(pool_size)]).astype(np.int8)


def validate_lineup(lineup) -> list[str]:
    """C1-C5 of setup.py:56-137; returns the violated codes."""
    lu = [int(x) for x in lineup]
    v = []
    if len(lu) != 30:
        return ["LENGTH"]
    if any(lu[i] != 0 for i in CAMP_SLOTS):
        v.append("C1")
    flags = [i for i, t in enumerate(lu) if t == 2]
    if len(flags) != 1 or flags[0] not in STRONGHOLD_SLOTS:
        v.append("C2")
    if any(t == 3 and i < 20 for i, t in enumerate(lu)):
        v.append("C3")
    if any(t == 4 and i < 5 for i, t in enumerate(lu)):
        v.append("C4")
    counts = [lu.count(t) for t in range(2, 14)]
    if tuple(counts) != PIECE_COUNTS or lu.count(0) != 5 or any(t < 0 or t > 13 or t == 1 for t in lu):
        v.append("C5")
    return v


def validate_pool(pool: np.ndarray) -> None:
    pool = np.asarray(pool)
    if pool.ndim != 2 or pool.shape[1] != 120:
        raise ValueError(f"setup pool must be (P, 120), got {pool.shape}")
    for i, row in enumerate(pool):
        for s in range(4):
            bad = validate_lineup(row[s * 30:(s + 1) * 30])
            if bad:
                raise ValueError(f"setup pool entry {i} seat {s} violates {bad}")
