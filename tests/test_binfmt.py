"""The `.cpu.bin` container reader (tb_bin_check), CPU only, through the C ABI.

Pinned on tests/golden/tiny.cpu.bin, written by the reference's own writer
(native/tools/pack_bin.py) from a seeded synthetic checkpoint: an independent
numpy parse of the file must match the format spec (native/docs/FORMAT.md), its
codes must equal the oracle packer's on the stored weights, and every malformed
variant the reference reader rejects (Container::open / assemble / validate,
native/crates/n2-core/src/binfmt.rs:104-257) must be rejected with its wording."""
import json
import os
import struct

import numpy as np
import pytest

import oracle
from tabinfer_b200 import binfmt

GOLD = os.path.join(os.path.dirname(__file__), "golden", "tiny.cpu.bin")
WEIGHTS = os.path.join(os.path.dirname(__file__), "golden", "tiny_bin_weights.npz")


def parse(path):
    raw = open(path, "rb").read()
    (hl,) = struct.unpack("<I", raw[:4])
    return json.loads(raw[4:4 + hl]), raw[4 + hl:]


def write(path, header, blob):
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<I", len(h)) + h + blob)


def test_golden_container_matches_the_spec_and_the_oracle():
    assert binfmt.check(GOLD) is None
    header, blob = parse(GOLD)
    assert header["G"] == 64
    w = np.load(WEIGHTS)
    for name, t in header["tensors"].items():
        u16 = w[name.replace(".", "__")]
        if t["kind"] == "tern":
            assert t["codesOff"] % 16 == 0 and t["scalesOff"] % 16 == 0
            codes = np.frombuffer(blob, np.uint8, t["codesLen"], t["codesOff"]).reshape(t["N"], t["K"] // 4)
            scales = np.frombuffer(blob, np.float32, t["scalesLen"] // 4, t["scalesOff"]).reshape(t["N"], -1)
            rc, rs = oracle.pack_ternary(oracle.bf16_to_f32(u16).reshape(t["N"], t["K"]))
            np.testing.assert_array_equal(codes, rc)
            np.testing.assert_array_equal(scales, rs)
        elif t["kind"] == "embed_f16":
            np.testing.assert_array_equal(np.frombuffer(blob, np.uint16, t["len"] // 2, t["off"]), u16.ravel())
        else:
            got = np.frombuffer(blob, np.float32, t["len"] // 4, t["off"])
            np.testing.assert_array_equal(got, u16.view(np.float16).astype(np.float32).ravel())


def _mutated(tmp_path, fn):
    header, blob = parse(GOLD)
    header = json.loads(json.dumps(header))
    fn(header, blob)
    p = tmp_path / "m.cpu.bin"
    write(str(p), header, blob)
    return str(p)


def _q(h):
    return h["tensors"]["model.layers.0.self_attn.q_proj.weight"]


@pytest.mark.parametrize("mutate,msg", [
    (lambda h, b: h.__setitem__("G", 32), "container group size G=32 but the kernels are built for G=64"),
    (lambda h, b: h.pop("tensors"), "header has no `tensors` object"),
    (lambda h, b: _q(h).pop("kind"), "q_proj.weight: missing `kind`"),
    (lambda h, b: _q(h).__setitem__("kind", "int4"), "q_proj.weight: unknown kind `int4`"),
    (lambda h, b: _q(h).__setitem__("codesLen", _q(h)["codesLen"] + 4), "codesLen=4100 but N*K/4=4096"),
    (lambda h, b: _q(h).__setitem__("scalesLen", 4), "scalesLen=4 but N*(K/G)*4=1024"),
    (lambda h, b: _q(h).__setitem__("K", 96), "K=96 is not a multiple of G=64"),
    (lambda h, b: _q(h).__setitem__("codesOff", len(b)), "overruns the"),
    (lambda h, b: _q(h).pop("N"), "missing field `N`"),
])
def test_rejects_what_the_reference_rejects(tmp_path, mutate, msg):
    p = _mutated(tmp_path, mutate)
    err = binfmt.check(p)
    assert err is not None and msg in err, err


def test_absent_group_size_means_64(tmp_path):
    assert binfmt.check(_mutated(tmp_path, lambda h, b: h.pop("G"))) is None


def test_truncated_files(tmp_path):
    p = tmp_path / "short.cpu.bin"
    p.write_bytes(b"\x01\x00")
    assert "too short" in binfmt.check(str(p))
    p.write_bytes(struct.pack("<I", 1000) + b"{}")
    assert "overruns the file" in binfmt.check(str(p))
    p.write_bytes(struct.pack("<I", 5) + b"{nope")
    assert "header JSON" in binfmt.check(str(p))
