"""Writes tests/golden/tile4x4_brfs.json: the reference's BrFS of the 4x4 sliding-tile workload (60 seeded blank
moves from the solved layout, seed 0; witness pruning and canonical order on, stop_at_goal off, deterministic ids) at
every depth from 12 to 25: stored states, expanded, generated, per-layer counts and the BrFS fingerprint, from the
compiled reference in oracle/_ref (mymyr::brfs with its concurrent store on every host thread, built by
make -C oracle). bench.py checks each search it times against this file at the depth it runs (22 + log2 N GPUs, or
--depth), so every bench line, also at 2, 4 and 8 GPUs, is the throughput of a search whose results match the
reference's.

    python tests/golden/make_brfs_golden.py [max_depth]
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from mymyr_b200 import tasks  # noqa: E402
from oracle import ref  # noqa: E402


def main() -> None:
    top = int(sys.argv[1]) if len(sys.argv) > 1 else 25
    rt = ref.RefTask(tasks.sliding_tile(4, 4, 60, 0))
    out = {"workload": "sliding_tile(4, 4, 60, seed=0), witness pruning on, stop_at_goal off", "depths": {}}
    threads = os.cpu_count() or 1
    for d in range(12, top + 1):
        r = rt.brfs(threads=threads, max_depth=d, stop_at_goal=False, fingerprint=True, store="concurrent")
        out["depths"][str(d)] = {"states": r["states"], "expanded": r["expanded"], "generated": r["generated"],
                                 "layers": r["layers"], "fingerprint": f"{r['fingerprint']:#018x}",
                                 "layer_counts": [list(x) for x in r["layer_counts"]]}
        print(d, r["states"], r["expanded"], f"{r['fingerprint']:#x}", f"{r['search_s']:.1f}s", flush=True)
    (HERE / "tile4x4_brfs.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
