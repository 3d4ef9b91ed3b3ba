"""`.cpu.bin` containers loaded onto the device (tb_bin_open).

* The golden container (written by the reference's own native/tools/pack_bin.py)
  loads with every tensor's device bytes equal to the file's blob, in the
  reference's BTreeMap (name) order, and the Q2_0_g64 GEMV run straight on the
  loaded codes and scales is bit-exact with gemv_tern_scalar (tern.rs:79-119).
* A ~100 MB container (several of the loader's 32 MB staging chunks, odd sizes)
  round-trips byte for byte.
* A malformed container is refused before any device memory is touched."""
import json
import os
import struct

import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from tabinfer_b200 import binfmt
from helpers import host

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden", "tiny.cpu.bin")


def _parse(path):
    raw = open(path, "rb").read()
    (hl,) = struct.unpack("<I", raw[:4])
    return json.loads(raw[4:4 + hl]), raw[4 + hl:]


def test_golden_loads_byte_exact_and_feeds_the_gemv(cuda):
    header, blob = _parse(GOLD)
    with binfmt.Container.open(GOLD) as c:
        assert c.blob_bytes() == len(blob)
        assert c.names() == sorted(header["tensors"])
        for name, t in header["tensors"].items():
            if t["kind"] == "tern":
                codes, scales = c.ternary(name)
                np.testing.assert_array_equal(host(codes).ravel(),
                                              np.frombuffer(blob, np.uint8, t["codesLen"], t["codesOff"]))
                np.testing.assert_array_equal(host(scales).ravel(),
                                              np.frombuffer(blob, np.float32, t["scalesLen"] // 4, t["scalesOff"]))
                # the Q2_0_g64 GEMV on the loaded tensors, bit-exact with the scalar reference
                x = np.random.default_rng(t["N"]).normal(0, 1, t["K"]).astype(np.float32)
                act, xsum, _ = oracle.quantize_act(x[None, :])
                out = tb.gemv_tern(codes, scales, torch.from_numpy(act).cuda(), torch.from_numpy(xsum).cuda())
                ref = oracle.gemv_tern_scalar(host(codes), host(scales), act[0], xsum[0])
                np.testing.assert_array_equal(host(out).ravel(), np.asarray(ref).ravel())
            elif t["kind"] == "embed_f16":
                e = c.embed(name)
                assert list(e.shape) == t["shape"]
                np.testing.assert_array_equal(host(e).view(np.uint16).ravel(),
                                              np.frombuffer(blob, np.uint16, t["len"] // 2, t["off"]))
            else:
                f = c.f32s(name)
                np.testing.assert_array_equal(host(f).ravel(), np.frombuffer(blob, np.float32, t["len"] // 4, t["off"]))
        with pytest.raises(tb.TabInferError):
            c.ternary("model.norm.weight")
        with pytest.raises(tb.TabInferError):
            c.info("no.such.tensor")


def _write(path, tensors):
    header, blob = {"G": 64, "tensors": {}}, bytearray()

    def put(a):
        off = len(blob)
        b = np.ascontiguousarray(a).tobytes()
        blob.extend(b)
        blob.extend(b"\0" * ((-len(blob)) % 16))
        return off, len(b)

    for name, (kind, arrs) in tensors.items():
        if kind == "tern":
            codes, scales = arrs
            co, cl = put(codes)
            so, sl = put(scales)
            header["tensors"][name] = {"kind": "tern", "N": codes.shape[0], "K": codes.shape[1] * 4,
                                       "codesOff": co, "codesLen": cl, "scalesOff": so, "scalesLen": sl}
        else:
            off, ln = put(arrs)
            header["tensors"][name] = {"kind": kind, "shape": list(arrs.shape), "off": off, "len": ln}
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<I", len(h)) + h + bytes(blob))
    return header, bytes(blob)


def test_large_container_round_trips(cuda, tmp_path):
    rng = np.random.default_rng(3)
    N, K = 6144, 12288          # 18 MB of codes, 4.5 MB of scales per matrix
    t = {}
    for i in range(4):
        t["m%d" % i] = ("tern", (rng.integers(0, 256, (N, K // 4), dtype=np.uint8),
                                 rng.uniform(0.01, 0.05, (N, K // 64)).astype(np.float32)))
    t["embed"] = ("embed_f16", rng.uniform(-1, 1, (3001, 777)).astype(np.float16).view(np.uint16))
    t["norm"] = ("f32", rng.uniform(0.5, 1.5, 2053).astype(np.float32))
    p = str(tmp_path / "big.cpu.bin")
    header, blob = _write(p, t)
    assert len(blob) > 2 * (32 << 20)      # three staging chunks, the last one partial
    assert binfmt.check(p) is None
    with binfmt.Container.open(p) as c:
        for name, (kind, arrs) in t.items():
            if kind == "tern":
                codes, scales = c.ternary(name)
                np.testing.assert_array_equal(host(codes), arrs[0])
                np.testing.assert_array_equal(host(scales), arrs[1])
            elif kind == "embed_f16":
                np.testing.assert_array_equal(host(c.embed(name)).view(np.uint16), arrs)
            else:
                np.testing.assert_array_equal(host(c.f32s(name)), arrs)


def test_malformed_is_refused(cuda, tmp_path):
    header, blob = _parse(GOLD)
    header["tensors"]["lm_head.weight"]["scalesLen"] += 4
    h = json.dumps(header).encode()
    p = tmp_path / "bad.cpu.bin"
    p.write_bytes(struct.pack("<I", len(h)) + h + blob)
    with pytest.raises(tb.TabInferError, match="scalesLen"):
        binfmt.Container.open(str(p))
