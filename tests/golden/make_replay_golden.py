"""Generate the replay-format fixtures that pin junqi_b200.replay.

Run in a container where the reference checkout is importable, e.g.::

    PYTHONPATH=<reference checkout> python tests/golden/make_replay_golden.py

Writes ``tests/golden/replay/ref_game_<name>.npz``: games recorded by
junqi_core's own ``record_trajectory`` (junqi_core/replay.py:296-370) and
saved with ``Trajectory.save``, so the files carry the reference's exact
keys, dtypes and final Zobrist hashes.  Nothing here runs during the test
suite; the suite only reads the files.
"""
from __future__ import annotations

from pathlib import Path

from junqi_core.replay import Trajectory, record_trajectory
from junqi_core.rules import Seat, ShowMode

OUT = Path(__file__).resolve().parent / "replay"

GAMES = {
    # name: (rng_seed, show_mode, first_seat, max_steps)
    "half_dark_s3": (3, ShowMode.HALF_DARK, Seat.SOUTH, 1000),
    "dark_s11": (11, ShowMode.DARK, Seat.SOUTH, 600),
    "bright_west_s5": (5, ShowMode.BRIGHT, Seat.WEST, 400),
}


def main() -> None:
    OUT.mkdir(parents=True, exist_ok=True)
    for name, (seed, mode, first, steps) in GAMES.items():
        tr = record_trajectory(rng_seed=seed, show_mode=mode, first_seat=first, max_steps=steps)
        tr.validate()
        path = OUT / f"ref_game_{name}.npz"
        tr.save(path)
        back = Trajectory.load(path)
        back.validate()
        print(name, tr.num_steps, "plies, final hash", tr.final_state_hash)


if __name__ == "__main__":
    main()
