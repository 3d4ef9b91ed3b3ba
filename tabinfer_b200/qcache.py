"""The quantized-weights cache of the reference loader, on a file system.

models/qwen3.js:3626-3717 streams the GPU-ready bytes of every tensor (int4 or
ternary pack + f16 scales of the projections and lm_head, f16 copies of the rest)
into 64 MiB chunks plus a JSON manifest, so a later load skips the bf16 download
and the re-quantization.  The browser keeps them in Cache Storage under
`https://tabinfer.quant/v1/<variant>/<part>`; here the same parts are files
`<root>/v1/<variant>/<part>` (`manifest`, `c0`, `c1`, ...), with the same
manifest schema (ver, variant, qgroup, chunkSize, nChunks, totalBytes, config,
segs [{name, role, off, len, kind, shape, numel, N, K}]), the same 16-byte
alignment of every segment in the global byte stream, and the same commit
protocol: the manifest is deleted first and written last, so a partial write is
never read.

QuantSink mirrors _makeQuantSink (:3633-3663); write_quant_cache mirrors what
_uploadTensor (:3503-3545) hands the sink; load_quant_cache mirrors
loadQuantCache (:3671-3717) and sets each tensor on a Qwen3 model shard as soon
as its segments are complete (peak host memory: one chunk plus the tensors in
flight, not the model).
"""
import json
import os

import numpy as np
import torch

from . import _lib
from .ops import quantize_int4_bf16, quantize_tern_bf16, convert_bf16_f16

QCACHE_VER = 1
QCHUNK = 64 * 1024 * 1024
QGROUP = 32


def _ceil16(n):
    return (n + 15) & ~15


def cfg_key(cfg):
    """_cfgKey (qwen3.js:3629): the dims that define the quantized layout."""
    return {"numLayers": cfg["layers"], "hidden": cfg["hidden"], "nHeads": cfg["n_heads"],
            "nKvHeads": cfg["n_kv_heads"], "headDim": cfg["head_dim"], "intermediate": cfg["intermediate"],
            "vocab": cfg["vocab"]}


def is_quant_weight(name):
    """isQuantWeight (qwen3.js:3470)."""
    return "_proj.weight" in name or name == "lm_head.weight"


def _dir(root, variant):
    return os.path.join(root, "v%d" % QCACHE_VER, variant)


class QuantSink:
    """_makeQuantSink (qwen3.js:3633-3663): segments appended to a global byte
    stream (each 16-aligned) cut into chunk files; finalize() writes the manifest."""

    def __init__(self, root, variant, cfg, chunk_size=QCHUNK):
        self.dir = _dir(root, variant)
        os.makedirs(self.dir, exist_ok=True)
        man = os.path.join(self.dir, "manifest")
        if os.path.exists(man):
            os.remove(man)                       # invalidate any prior cache up-front
        self.variant, self.cfg, self.chunk = variant, cfg, chunk_size
        self.buf = bytearray()
        self.chunk_idx = 0
        self.global_off = 0
        self.segs = []

    def _flush(self):
        if not self.buf:
            return
        with open(os.path.join(self.dir, "c%d" % self.chunk_idx), "wb") as f:
            f.write(self.buf)
        self.chunk_idx += 1
        self.buf = bytearray()

    def _write(self, b):
        mv = memoryview(b).cast("B")
        src = 0
        while src < len(mv):
            if len(self.buf) == self.chunk:
                self._flush()
            n = min(self.chunk - len(self.buf), len(mv) - src)
            self.buf += mv[src:src + n]
            src += n

    def add(self, name, role, data, meta):
        pad = _ceil16(self.global_off) - self.global_off
        if pad:
            self._write(bytes(pad))
            self.global_off += pad
        data = np.ascontiguousarray(data).view(np.uint8).ravel()
        self.segs.append({"name": name, "role": role, "off": self.global_off, "len": int(data.size),
                          "kind": meta["kind"], "shape": list(meta["shape"]), "numel": int(meta["numel"]),
                          "N": meta.get("N"), "K": meta.get("K")})
        self._write(data)
        self.global_off += int(data.size)

    def finalize(self):
        self._flush()
        manifest = {"ver": QCACHE_VER, "variant": self.variant, "qgroup": QGROUP, "chunkSize": self.chunk,
                    "nChunks": self.chunk_idx, "totalBytes": self.global_off, "config": cfg_key(self.cfg),
                    "segs": self.segs}
        with open(os.path.join(self.dir, "manifest"), "w") as f:
            json.dump(manifest, f)


def write_quant_cache(root, variant, cfg, tensors, ternary=True, chunk_size=QCHUNK):
    """Quantize checkpoint tensors exactly as the loader does and cache them.
    tensors: iterable of (name, bf16 tensor on a CUDA device).  Projections and
    lm_head: the ternary record when the tensor is ternary (and `ternary`), else
    int4 G32; everything else: bf16ToF16bits."""
    sink = QuantSink(root, variant, cfg, chunk_size)
    for name, w in tensors:
        shape = list(w.shape)
        numel = w.numel()
        if is_quant_weight(name):
            N, K = shape
            t = quantize_tern_bf16(w.view(torch.int16)) if ternary else None
            kind = "tern" if t is not None else "int4"
            pack, sc = t if t is not None else quantize_int4_bf16(w.view(torch.int16))
            meta = {"kind": kind, "shape": shape, "numel": numel, "N": N, "K": K}
            sink.add(name, "pack", pack.cpu().numpy(), meta)
            sink.add(name, "scales", sc.cpu().numpy(), meta)
        else:
            sink.add(name, "buf", convert_bf16_f16(w.view(torch.int16)).cpu().numpy(),
                     {"kind": "f16", "shape": shape, "numel": numel})
    sink.finalize()


def read_manifest(root, variant, cfg, chunk_size=QCHUNK):
    """The manifest when it is valid for this variant and config, else None
    (loadQuantCache's checks, qwen3.js:3673-3678)."""
    path = os.path.join(_dir(root, variant), "manifest")
    if not os.path.exists(path):
        return None
    try:
        m = json.load(open(path))
    except ValueError:
        return None
    if not m or m.get("ver") != QCACHE_VER or m.get("variant") != variant or m.get("qgroup") != QGROUP or \
            m.get("chunkSize") != chunk_size:
        return None
    want = cfg_key(cfg)
    if any(m.get("config", {}).get(k) != v for k, v in want.items()):
        return None
    return m


def iter_tensors(root, variant, m):
    """Reads the chunks in order and yields (name, {role: uint8 array}, seg) as
    soon as every segment of a tensor is complete."""
    segs = sorted(m["segs"], key=lambda s: s["off"])
    need = {}
    for s in segs:
        need.setdefault(s["name"], set()).add(s["role"])
    bufs = {}
    filled = {}
    first = 0
    for ci in range(m["nChunks"]):
        path = os.path.join(_dir(root, variant), "c%d" % ci)
        if not os.path.exists(path):
            raise IOError("quant cache missing chunk %d" % ci)
        u8 = np.fromfile(path, np.uint8)
        c0, c1 = ci * m["chunkSize"], ci * m["chunkSize"] + u8.size
        while first < len(segs) and segs[first]["off"] + _ceil16(segs[first]["len"]) <= c0:
            first += 1
        for i in range(first, len(segs)):
            s = segs[i]
            if s["off"] >= c1:
                break
            lo, hi = max(s["off"], c0), min(s["off"] + s["len"], c1)
            if hi <= lo:
                continue
            key = (s["name"], s["role"])
            if key not in bufs:
                bufs[key] = np.empty(s["len"], np.uint8)
                filled[key] = 0
            bufs[key][lo - s["off"]:hi - s["off"]] = u8[lo - c0:hi - c0]
            filled[key] += hi - lo
            if filled[key] == s["len"]:
                roles = {r: bufs.get((s["name"], r)) for r in need[s["name"]]}
                if all(v is not None and filled[(s["name"], r)] == len(v) for r, v in roles.items()):
                    yield s["name"], roles, s
                    for r in roles:
                        del bufs[(s["name"], r)]
                        del filled[(s["name"], r)]


def load_quant_cache(model, root, variant, chunk_size=QCHUNK):
    """loadQuantCache onto a Qwen3 model shard: False (cold) when there is no
    valid cache for this variant and config, else sets every cached tensor and
    returns True."""
    m = read_manifest(root, variant, model.cfg, chunk_size)
    if m is None:
        return False
    for name, roles, seg in iter_tensors(root, variant, m):
        shape = seg["shape"]
        rows, cols = (1, shape[0]) if len(shape) == 1 else (shape[0], shape[1])
        if seg["kind"] in ("int4", "tern"):
            fmt = _lib.QW_FMT_TERN if seg["kind"] == "tern" else _lib.QW_FMT_INT4
            model.load_quantized(name, fmt, roles["pack"], roles["scales"], (rows, cols))
        else:
            model.load_quantized(name, _lib.QW_FMT_F16, roles["buf"], None, (rows, cols))
    return True
