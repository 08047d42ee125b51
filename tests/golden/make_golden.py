"""Regenerate tests/golden/c1_top10.json: the oracle's exact top-10 for config C1.

C1 is the reference's quickstart workload (examples/quickstart.rs:25-36):
5,000 x 64 cosine, queries = every 50th vector, k = 10. The ids and f32
distances come from the CPU oracle (oracle/pxo.cpp), which restates
FlatIndex::search (crates/proxima-index/src/flat.rs:153-169) and is pinned by
tests/test_oracle_core.py. Run from the repository root:
    python tests/golden/make_golden.py
"""
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import pxo  # noqa: E402
from proxima_b200 import fixtures  # noqa: E402

data = fixtures.quickstart()
prepared = pxo.prepare(pxo.COSINE, data)
queries = prepared[::50]
ids, dist, lens = pxo.flat_search(prepared, queries, 10, pxo.COSINE)
out = {
    "_about": "oracle top-10 for the quickstart workload (C1); see make_golden.py",
    "ids": [list(map(int, r)) for r in ids],
    "distances": [[float(x) for x in r] for r in dist],
}
(Path(__file__).parent / "c1_top10.json").write_text(json.dumps(out))
print("wrote", len(out["ids"]), "queries")
