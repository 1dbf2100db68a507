"""Regenerate the smoke-tier golden fixture (run once, in the build container).

Inputs: the reference's smoke corpus recipe (ultravec-ann
scripts/generate_smoke_data.py:13-24) restated with numpy: default_rng(42),
128x32 N(0,1) base rows normalized, 16 queries = base[:16] + N(0, 0.02)
noise, normalized.

Expected outputs: the reference's own retained run of that corpus
(results/generated/smoke-synthetic/per-query.csv, `trellis` rows: per-query
Recall@1/10/100 of the 2-bit, M=12 trellis under the cosine harness) and the
reconstruction MSE it printed (stdout.txt).  The files written here are
committed; nothing reads the reference at test time.

Usage: python tests/golden/make_smoke_fixture.py [reference_root]
"""
from __future__ import annotations

import csv
import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def corpus():
    rng = np.random.default_rng(42)
    base = rng.normal(size=(128, 32)).astype(np.float32)
    base /= np.linalg.norm(base, axis=1, keepdims=True)
    query = base[:16] + rng.normal(scale=0.02, size=(16, 32)).astype(np.float32)
    query /= np.linalg.norm(query, axis=1, keepdims=True)
    return base.astype("<f4"), query.astype("<f4")


def main() -> int:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
    bundle = ref / "results" / "generated" / "smoke-synthetic"
    base, query = corpus()
    (HERE / "smoke_base.f32").write_bytes(base.tobytes())
    (HERE / "smoke_query.f32").write_bytes(query.tobytes())
    rows = []
    with open(bundle / "per-query.csv") as fh:
        for r in csv.DictReader(fh):
            if r["quantizer"] == "trellis":
                rows.append([float(r["recall_at_1"]), float(r["recall_at_10"]),
                             float(r["recall_at_100"])])
    text = (bundle / "stdout.txt").read_text()
    m = re.search(r"^\| trellis \| 2 \| ([0-9.]+) \| ([0-9.]+) \| ([0-9.]+) \| ([0-9.]+) \|",
                  text, re.M)
    assert m, "trellis row not found"
    expected = {
        "source": "results/generated/smoke-synthetic (reference retained bundle)",
        "config": {"dim": 32, "bits": 2, "mem": 12, "seed": 42, "rounds": 3,
                   "n_base": 128, "n_query": 16, "harness": "cosine, top-100"},
        "per_query_recall_1_10_100": rows,
        "mean_recall_1_10_100": [float(m.group(1)), float(m.group(2)), float(m.group(3))],
        "recon_mse": m.group(4),
    }
    (HERE / "smoke_expected.json").write_text(json.dumps(expected, indent=1) + "\n")
    print(f"wrote smoke fixture: {base.shape} base, {query.shape} query, "
          f"{len(rows)} expected rows, mse {m.group(4)}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
