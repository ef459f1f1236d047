"""DiskANN on-disk formats: byte layout, round trips, atomic refuse-to-overwrite."""
import struct

import numpy as np
import pytest

from dance_b200 import formats

INVALID = 0xFFFFFFFF


def _graph():
    g = np.full((5, 4), INVALID, np.uint32)
    deg = np.array([2, 0, 4, 1, 3], np.uint32)
    g[0, :2] = [1, 2]
    g[2, :4] = [0, 1, 3, 4]
    g[3, :1] = [2]
    g[4, :3] = [0, 2, 3]
    return g, deg


def test_graph_layout_bytes(tmp_path):
    g, deg = _graph()
    p = tmp_path / "idx"
    formats.write_graph(p, g, deg, start=2)
    blob = p.read_bytes()
    size, max_degree, start, frozen = struct.unpack_from("<QIIQ", blob, 0)
    assert size == len(blob) == 24 + 4 * 5 + 4 * int(deg.sum())
    assert (max_degree, start, frozen) == (4, 2, 0)
    words = np.frombuffer(blob[24:], np.uint32)
    assert list(words[:3]) == [2, 1, 2] and words[3] == 0 and list(words[4:9]) == [4, 0, 1, 3, 4]
    rows, md, st, fr = formats.read_graph(p)
    assert [list(r) for r in rows] == [[1, 2], [], [0, 1, 3, 4], [2], [0, 2, 3]]


def test_refuse_overwrite_and_no_temp_left(tmp_path):
    g, deg = _graph()
    p = tmp_path / "idx"
    formats.write_graph(p, g, deg, 0)
    with pytest.raises(FileExistsError):
        formats.write_graph(p, g, deg, 0)
    assert not (tmp_path / "idx.tmp").exists()


def test_memory_index_and_bins(tmp_path):
    rng = np.random.default_rng(0)
    x = rng.integers(0, 256, (5, 8), dtype=np.uint8)
    g, deg = _graph()
    formats.save_memory_index(tmp_path / "mem", x, g, deg, 3)
    assert np.array_equal(formats.read_bin(tmp_path / "mem.data", np.uint8), x)
    assert formats.read_graph(tmp_path / "mem")[2] == 3
    f = rng.normal(size=(7, 3)).astype(np.float32)
    formats.write_bin(tmp_path / "v.fbin", f)
    assert np.array_equal(formats.read_bin(tmp_path / "v.fbin", np.float32), f)
    (tmp_path / "bad.fbin").write_bytes(struct.pack("<II", 7, 3) + b"\0" * 10)
    with pytest.raises(ValueError):
        formats.read_bin(tmp_path / "bad.fbin", np.float32)


def test_groundtruth_roundtrip(tmp_path):
    ids = np.arange(20, dtype=np.uint32).reshape(2, 10)
    d = np.linspace(0, 1, 20, dtype=np.float32).reshape(2, 10)
    formats.write_groundtruth(tmp_path / "gt", ids, d)
    i2, d2 = formats.read_groundtruth(tmp_path / "gt")
    assert np.array_equal(i2, ids) and np.array_equal(d2, d)


def test_audit_counts_violations():
    g, deg = _graph()
    assert formats.audit_graph(g, deg, 4, 0) == {"invalid": 0, "self": 0, "duplicate": 0, "overflow": 0,
                                                 "medoid_out_of_range": 0}
    g2 = g.copy()
    g2[2, 0] = 2  # self loop
    g2[4, 2] = 0  # duplicate
    g2[0, 1] = 99  # invalid
    bad = formats.audit_graph(g2, deg, 4, 7)
    assert bad["self"] == 1 and bad["duplicate"] == 1 and bad["invalid"] == 1 and bad["medoid_out_of_range"] == 1
