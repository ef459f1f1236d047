"""The drop-in claim, checked with the reference's own caller.

DANCE's standard app (apps/utils/gpu_vamana_memory_index.cpp, unmodified) is
compiled against this repository's include/ and linked to libdance_b200.so
only (oracle/ref/Makefile targets gpu_vamana_memory_index and its copy
gpu_vamana_app, which the app lets use --builder v8).  CPU: the compile and
link step, and that the binary needs our library and nothing of the
reference's.  GPU: the binary builds an index from a .u8bin / .fbin file; the
files it writes pass the graph audit, hold the input vectors, and carry
exactly the graph that gpu_vamana_vnew2_build gives through ctypes.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
APP = ROOT / "oracle" / "_ref" / "gpu_vamana_memory_index"
APP_ANY = ROOT / "oracle" / "_ref" / "gpu_vamana_app"


def _reference_tree():
    sys.path.insert(0, str(ROOT))
    import __graft_entry__
    return __graft_entry__.reference_tree()


def test_reference_app_compiles_and_links_against_our_library(dance_lib):
    ref = _reference_tree()
    if ref is None:
        if not APP.exists():
            pytest.skip("DANCE sources not on this machine and the app was not prebuilt")
    else:
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle" / "ref"), f"REF={ref}", "../_ref/gpu_vamana_app"],
                       check=True)
    assert APP.exists() and APP_ANY.exists()
    needed = subprocess.run(["readelf", "-d", str(APP)], capture_output=True, text=True, check=True).stdout
    assert "libdance_b200.so" in needed
    assert "libref_" not in needed
    # every builder symbol the app calls is one our library exports
    undef = subprocess.run(["nm", "-D", "--undefined-only", str(APP)], capture_output=True, text=True,
                           check=True).stdout
    wanted = {ln.split()[-1] for ln in undef.splitlines() if "gpu_vamana" in ln}
    assert wanted >= {"gpu_vamana_vnew2_build", "gpu_vamana_vnew2_build_float", "gpu_vamana_build",
                      "gpu_vamana_build_float", "gpu_vamana_vnew2_get_last_medoid", "gpu_vamana_get_last_stats"}
    exported = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "dance_b200" / "libdance_b200.so")],
                              capture_output=True, text=True, check=True).stdout
    have = {ln.split()[-1] for ln in exported.splitlines()}
    assert wanted <= have, wanted - have


def _run_app(app, data_path, prefix, dtype, R, L, C, S, builder="vnew2"):
    cmd = [str(app), "--data_path", str(data_path), "--data_type", dtype, "--index_prefix", str(prefix),
           "--R", str(R), "--L", str(L), "--C", str(C), "--STEPS", str(S), "--builder", builder]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    report = json.loads(res.stdout[res.stdout.index("{\n"):])
    return report


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["uint8", "float"])
def test_reference_app_builds_our_graph(tmp_path, dance_lib, dtype):
    from dance_b200 import formats, vamana, workloads
    if not APP.exists():
        pytest.skip("reference app not built (make -C oracle/ref REF=...)")
    n, R, L, C, S = 4000, 32, 64, 48, 32
    if dtype == "uint8":
        x = workloads.clustered_u8(n, 128, centroids=30, seed=11).numpy()
        path = tmp_path / "base.u8bin"
    else:
        x = workloads.gaussian_mixture_f32(n, 96, centroids=30, seed=11).numpy()
        path = tmp_path / "base.fbin"
    formats.write_bin(path, x)
    prefix = tmp_path / "index"
    report = _run_app(APP, path, prefix, dtype, R, L, C, S)
    assert report["graph_valid"] and report["memory_index_serialized"] and report["return_code"] == 0
    rows, _, start, frozen = formats.read_graph(prefix)
    assert start == report["medoid"] and len(rows) == n and frozen == 0
    deg = np.array([len(r) for r in rows], np.uint32)
    stored = formats.read_bin(str(prefix) + ".data", x.dtype)
    assert np.array_equal(stored, x)
    # the same graph as the library's reference-ABI build through ctypes
    build = vamana.gpu_vamana_vnew2_build if dtype == "uint8" else vamana.gpu_vamana_vnew2_build_float
    g, d = build(x, R, L, C, S)
    assert start == vamana.gpu_vamana_vnew2_get_last_medoid()
    assert np.array_equal(deg, d)
    for v in range(n):
        assert list(rows[v]) == list(g[v, :d[v]])
    audit = formats.audit_graph(g, d, R, start)
    assert audit == {"invalid": 0, "self": 0, "duplicate": 0, "overflow": 0, "medoid_out_of_range": 0}


@pytest.mark.gpu
def test_reference_app_v8_builder_entry_point(tmp_path, dance_lib):
    from dance_b200 import formats, workloads
    if not APP_ANY.exists():
        pytest.skip("reference app not built (make -C oracle/ref REF=...)")
    x = workloads.clustered_u8(3000, 64, centroids=20, seed=12).numpy()
    path = tmp_path / "b.u8bin"
    formats.write_bin(path, x)
    report = _run_app(APP_ANY, path, tmp_path / "v8index", "uint8", 24, 48, 32, 24, builder="v8")
    assert report["graph_valid"] and report["builder"] == "v8"
    rows, _, start, _ = formats.read_graph(tmp_path / "v8index")
    assert len(rows) == 3000 and max(len(r) for r in rows) <= 24 and start < 3000
