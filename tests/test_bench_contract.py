"""bench.py's contract pieces that need no GPU: its copy of the library's scan rule, the parity
object of its CPU baseline, and the reference arm's JSON line on a tiny workload."""
import io
import json
import os
import sys
import types
from contextlib import redirect_stdout

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _cfg(**kw):
    base = dict(n=3000, d=64, centres=40, sigma=0.3, nq=60, qsigma=0.05, nlist=16, nprobe=4, k=5, rerank=20,
                seed=11, config=2, aniso=0, query_bits=4, device_data=False, gt_sample=60)
    base.update(kw)
    return base


@pytest.mark.parametrize("nq,nprobe,nlist,n,R,qb,d,kind", [
    (10000, 32, 1024, 1_000_000, 200, 4, 256, 0),   # config 2: the list scan
    (1024, 32, 1024, 1_000_000, 200, 4, 256, 0),    # 32 pairs per list: the tile scan
    (200000, 48, 2048, 200_000, 800, 4, 256, 0),    # config 3: lists shorter than R
    (10000, 32, 1024, 1_000_000, 200, 16, 256, 0),  # LUT16: no list scan
    (10000, 32, 1024, 1_000_000, 200, 8, 800, 0),   # padded dim above 768
    (10000, 32, 1024, 1_000_000, 200, 4, 256, 1),   # forced tile scan
    (64, 4, 1024, 1000, 10, 4, 128, 2),             # forced list scan
])
def test_bench_scan_rule_matches_the_library_rule(oracle, nq, nprobe, nlist, n, R, qb, d, kind):
    cfg = _cfg(nq=nq, nprobe=nprobe, nlist=nlist, n=n, query_bits=qb, d=d, scan_kind=kind, k=10)
    dp = (d + 31) // 32 * 32
    try:
        lib = oracle.uses_list_scan(kind, qb, 1, dp, nq, nprobe, nlist, n, max(R, 10))
    except ValueError:
        lib = False
    assert bench.list_scan_used(cfg, 1, R) == lib


def test_parity_object_counts_ties_and_differences():
    d = np.array([[0.1, 0.2, 0.2, 0.5]], np.float32)
    i = np.array([[3, 7, 9, 1]])
    p = bench.parity_of(d, i, d.copy(), i.copy())
    assert p["ids_equal"] and p["dist_bits_equal"] and p["rows_differing"] == 0
    # two ids swapped at equal distance: a tie, not a difference
    p = bench.parity_of(d, np.array([[3, 9, 7, 1]]), d, i)
    assert not p["ids_equal"] and p["ids_differing_outside_ties"] == 0
    # a different neighbour at a different distance
    d2 = d.copy()
    d2[0, 3] = 0.6
    p = bench.parity_of(d2, np.array([[3, 7, 9, 4]]), d, i)
    assert not p["dist_bits_equal"] and p["ids_differing_outside_ties"] == 1 and p["rows_differing"] == 1


def test_reference_arm_line(oracle):
    """The reference arm on a tiny mixture: one JSON line with the contract's keys, the tile scan
    timed, rank 0 only."""
    args = types.SimpleNamespace(rerank=0, steps=2, warmup=1, gpus=1, kmeans="balanced")
    cfg = _cfg()
    out = io.StringIO()
    with redirect_stdout(out):
        assert bench.run_reference(args, cfg) == 0
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "queries/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["timed_scan"].startswith("tile")
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["config"]["rerank"] in bench.rerank_ladder(cfg)
    # other ranks of a torchrun launch print nothing and succeed
    os.environ["RANK"] = "1"
    try:
        out = io.StringIO()
        with redirect_stdout(out):
            assert bench.run_reference(args, cfg) == 0
        assert out.getvalue() == ""
    finally:
        del os.environ["RANK"]
