"""The quantized-weights cache file format (QuantSink / read_manifest /
iter_tensors), CPU only: the schema and commit protocol of _makeQuantSink and
loadQuantCache (models/qwen3.js:3626-3717) -- 16-byte-aligned segments in one
global stream cut into chunks, the manifest written last and deleted first,
every invalidating field honoured, segments reassembled across chunk edges."""
import json
import os

import numpy as np
import pytest

from tabinfer_b200 import qcache

CFG = dict(layers=2, hidden=64, n_heads=2, n_kv_heads=1, head_dim=64, intermediate=128, vocab=50)


def _segments(rng):
    t = {}
    for i, n in enumerate((33, 1000, 7, 4096, 1)):
        t["model.layers.%d.mlp.up_proj.weight" % i] = (rng.integers(0, 2**32, n, dtype=np.uint32),
                                                       rng.integers(0, 2**16, (n + 3) // 4, dtype=np.uint16))
    t["model.norm.weight"] = (rng.integers(0, 2**16, 77, dtype=np.uint16), None)
    return t


def _write(root, chunk):
    rng = np.random.default_rng(1)
    t = _segments(rng)
    sink = qcache.QuantSink(root, "tiny", CFG, chunk)
    for name, (a, b) in t.items():
        if b is None:
            sink.add(name, "buf", a, {"kind": "f16", "shape": [a.size], "numel": a.size})
        else:
            meta = {"kind": "int4", "shape": [a.size // 1, 8], "numel": a.size * 8, "N": a.size, "K": 8}
            sink.add(name, "pack", a, meta)
            sink.add(name, "scales", b, meta)
    sink.finalize()
    return t


@pytest.mark.parametrize("chunk", [256, 4096, qcache.QCHUNK])
def test_round_trip_across_chunk_edges(tmp_path, chunk):
    t = _write(str(tmp_path), chunk)
    m = qcache.read_manifest(str(tmp_path), "tiny", CFG, chunk)
    assert m is not None and m["ver"] == 1 and m["qgroup"] == 32 and m["chunkSize"] == chunk
    assert m["config"] == qcache.cfg_key(CFG)
    assert all(s["off"] % 16 == 0 for s in m["segs"])
    assert m["nChunks"] == -(-m["totalBytes"] // chunk)
    got = {name: roles for name, roles, _ in qcache.iter_tensors(str(tmp_path), "tiny", m)}
    assert set(got) == set(t)
    for name, (a, b) in t.items():
        if b is None:
            np.testing.assert_array_equal(got[name]["buf"].view(np.uint16), a)
        else:
            np.testing.assert_array_equal(got[name]["pack"].view(np.uint32), a)
            np.testing.assert_array_equal(got[name]["scales"].view(np.uint16), b)


def test_invalidations(tmp_path):
    root = str(tmp_path)
    _write(root, 4096)
    assert qcache.read_manifest(root, "tiny", CFG, 4096) is not None
    assert qcache.read_manifest(root, "other", CFG, 4096) is None                 # no such variant
    assert qcache.read_manifest(root, "tiny", CFG, qcache.QCHUNK) is None         # chunkSize differs
    assert qcache.read_manifest(root, "tiny", dict(CFG, vocab=51), 4096) is None  # layout-defining dim differs
    man = os.path.join(root, "v1", "tiny", "manifest")
    m = json.load(open(man))
    for field, val in (("ver", 2), ("qgroup", 64)):
        json.dump(dict(m, **{field: val}), open(man, "w"))
        assert qcache.read_manifest(root, "tiny", CFG, 4096) is None
    open(man, "w").write("{broken")
    assert qcache.read_manifest(root, "tiny", CFG, 4096) is None


def test_manifest_is_the_commit_point(tmp_path):
    root = str(tmp_path)
    _write(root, 4096)
    sink = qcache.QuantSink(root, "tiny", CFG, 4096)       # a new write invalidates at once
    assert qcache.read_manifest(root, "tiny", CFG, 4096) is None
    sink.add("model.norm.weight", "buf", np.zeros(8, np.uint16), {"kind": "f16", "shape": [8], "numel": 8})
    sink.finalize()
    m = qcache.read_manifest(root, "tiny", CFG, 4096)
    assert m is not None and [s["name"] for s in m["segs"]] == ["model.norm.weight"]


def test_missing_chunk_raises(tmp_path):
    root = str(tmp_path)
    _write(root, 256)
    m = qcache.read_manifest(root, "tiny", CFG, 256)
    os.remove(os.path.join(root, "v1", "tiny", "c3"))
    with pytest.raises(IOError, match="missing chunk 3"):
        list(qcache.iter_tensors(root, "tiny", m))
