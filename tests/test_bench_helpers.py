"""Host-side pieces of bench.py that feed its JSON line: the algorithmic-byte
count behind roofline.achieved, the measured DRAM traffic read from the
committed ncu summary, and the workload descriptions."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_search_algorithmic_bytes_formula():
    rep = {"search_evals": 1000, "expansions": 10}
    # per eval one row; per expansion an adjacency row + degree + 8-byte record;
    # per vertex and round its row, own ids + distances and degree
    got = bench.search_algorithmic_bytes(rep, n=5, row_bytes=128, R=64, iters=4)
    assert got == 1000 * 128 + 10 * (64 * 4 + 4 + 8) + 4 * 5 * (128 + 64 * 8 + 4 + 4)


def test_traffic_read_from_profile_summary():
    t = bench.traffic_per_launch("search_kernel", bench.WORKLOAD["name"], bench.WORKLOAD["N"])
    text = (ROOT / "profiles" / f"search_kernel_traffic_{bench.WORKLOAD['name']}.md").read_text()
    assert t is not None and str(t) in text
    # the capture covers the full workload only: smaller N reports no traffic
    assert bench.traffic_per_launch("search_kernel", bench.WORKLOAD["name"], 1000) is None
    assert bench.traffic_per_launch("no_such_kernel", bench.WORKLOAD["name"], bench.WORKLOAD["N"]) is None


@pytest.mark.parametrize("fn,n,name", [("config_dict", 123, "cfg1_u8_10M"), ("cfg0_config", 77, "cfg0_f32_1M_fp16")])
def test_workload_configs_name_the_workload(fn, n, name):
    cfg = getattr(bench, fn)(n)
    assert cfg["workload"] == name and cfg["N"] == n
    assert {"R", "L", "C", "STEPS"} <= set(cfg) and "model" not in cfg


def test_read_graph_padded_matches_file(tmp_path):
    import numpy as np
    import bench
    from dance_b200 import formats
    rng = np.random.default_rng(0)
    n, R = 400, 12
    deg = rng.integers(0, R + 1, n).astype(np.uint32)
    g = np.full((n, R), 0xFFFFFFFF, np.uint32)
    for i in range(n):
        g[i, :deg[i]] = rng.integers(0, n, deg[i])
    formats.write_graph(tmp_path / "g.idx", g, deg, 7)
    g2, d2, start = bench.read_graph_padded(tmp_path / "g.idx", R)
    assert np.array_equal(g, g2) and np.array_equal(deg, d2) and start == 7
