"""Writes tests/golden/astar_costs.txt: the reference's optimal A* plan costs (search::astar_eager, h^max, unit costs)
on the logistics configs, from the compiled reference in oracle/_ref (built by make -C oracle). The 3-package config
takes the reference about 13 minutes on one core, so the tests read the file instead of rerunning it.

    python tests/golden/make_astar_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from mymyr_b200 import tasks  # noqa: E402
from oracle import ref  # noqa: E402

CONFIGS = [(8, 4, 6, 2, 2, 0), (8, 4, 6, 2, 3, 0)]


def main() -> None:
    lines = ["# cities locs_per_city trucks airplanes packages seed | cost expanded generated seconds"]
    for cfg in CONFIGS:
        r = ref.RefTask(tasks.logistics(*cfg)).astar()
        lines.append(" ".join(map(str, cfg)) + f" | {int(r['cost'])} {r['expanded']} {r['generated']} "
                     f"{r['seconds']:.1f}")
        print(lines[-1], flush=True)
    (HERE / "astar_costs.txt").write_text("\n".join(lines) + "\n")


if __name__ == "__main__":
    main()
