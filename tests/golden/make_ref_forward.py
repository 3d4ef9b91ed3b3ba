"""Golden logits from the REFERENCE'S OWN numpy forward pass.

Run in the build container, where the TabInfer checkout is mounted:

    python tests/golden/make_ref_forward.py /path/to/TabInfer

native/tools/ref_forward.py:50-112 is the reference's full-precision Qwen3 /
Bonsai forward (RMSNorm, q/k head norms, split-half RoPE at theta 1e6, GQA
softmax attention over an f32 cache, SwiGLU, untied lm_head), run token by token
over a prompt.  Its model sizes, prompt and checkpoint directory are module
globals, so this script imports it from the checkout, points it at a small
synthetic Bonsai-style checkpoint written here as safetensors (ternary bf16
projections and lm_head with one magnitude per 32-group, bf16 norms, the
embedding as the f16 bits the engine's bf16ToF16bits gives, which is how the
reference script reads it), calls its own main(), and keeps the logits of the
last prompt token (the product of its own `lin('lm_head.weight', xf)`) and the
top-10 ids it prints.

The checkpoint itself is not stored: tests regenerate it with
tests/qwen3_oracle.make_weights(CFG, SEED, ternary=True), and the sha256 of the
regenerated bits is kept in the fixture so a generator drift is caught.
"""
import contextlib
import hashlib
import importlib.util
import io
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TESTS = os.path.dirname(HERE)
sys.path.insert(0, TESTS)
sys.path.insert(0, os.path.dirname(TESTS))

CFG = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, vocab=1000,
           rope_theta=1e6, rms_eps=1e-6)
SEED = 0x5EF0
IDS = [17, 401, 998, 3, 250, 77, 640, 12, 905, 331, 58, 712, 129]
OUT = os.path.join(HERE, "ref_forward_bonsai.npz")


def weights_digest(W):
    h = hashlib.sha256()
    for name in sorted(W):
        h.update(name.encode())
        h.update(np.ascontiguousarray(W[name], np.uint16).tobytes())
    return h.hexdigest()


def _write_safetensors(path, tensors):
    hdr, off, blobs = {}, 0, []
    for name, (dt, shape, u16) in tensors.items():
        b = np.ascontiguousarray(u16, np.uint16).tobytes()
        hdr[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def checkpoint_tensors(W):
    """name -> (safetensors dtype, shape, u16 bits) as ref_forward.load_all reads them."""
    from qwen3_oracle import f16_of_bf16
    out = {}
    for name, u16 in W.items():
        if name == "model.embed_tokens.weight":
            out[name] = ("F16", u16.shape, f16_of_bf16(u16))     # ref_forward reads the embedding as f16
        else:
            out[name] = ("BF16", u16.shape, u16)
    return out


def run_reference(ref_root, W):
    path = os.path.join(ref_root, "native", "tools", "ref_forward.py")
    spec = importlib.util.spec_from_file_location("ref_forward", path)
    rf = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rf)
    c = CFG
    with tempfile.TemporaryDirectory() as d:
        _write_safetensors(os.path.join(d, "model.safetensors"), checkpoint_tensors(W))
        json.dump({"weight_map": {n: "model.safetensors" for n in W}},
                  open(os.path.join(d, "model.safetensors.index.json"), "w"))
        rf.ROOT = d
        rf.L, rf.H, rf.NH, rf.NKV, rf.HD, rf.I = c["layers"], c["hidden"], c["n_heads"], c["n_kv_heads"], \
            c["head_dim"], c["intermediate"]
        rf.THETA, rf.EPS, rf.VOCAB = c["rope_theta"], c["rms_eps"], c["vocab"]
        rf.IDS = list(IDS)
        rf.PARIS = 0
        captured = []

        class _Rec(np.ndarray):
            """the lm_head matrix: records the script's own product lin('lm_head.weight', xf)"""
            def __matmul__(self, other):
                r = np.asarray(self) @ other
                captured.append(np.array(r, np.float32))
                return r

        deq = rf.deq

        def deq_rec(Wd, name):
            a = deq(Wd, name)
            return a.view(_Rec) if name == "lm_head.weight" else a

        rf.deq = deq_rec
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            rf.main()
    text = buf.getvalue()
    top = [ln for ln in text.splitlines() if ln.startswith("top10 ids:")]
    top10 = json.loads(top[-1].split(":", 1)[1]) if top else []
    return captured[-1], np.array(top10, np.int64), text


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TABINFER_REF", "")
    if not os.path.exists(os.path.join(ref, "native", "tools", "ref_forward.py")):
        sys.exit("usage: make_ref_forward.py <TabInfer checkout>  (native/tools/ref_forward.py not found)")
    from qwen3_oracle import make_weights
    W = make_weights(CFG, SEED, ternary=True)
    logits, top10, text = run_reference(ref, W)
    assert logits.shape == (CFG["vocab"],)
    assert np.array_equal(np.argsort(-logits)[:10], top10), "captured logits differ from the printed top 10"
    np.savez_compressed(OUT, logits=logits, top10=top10, ids=np.array(IDS, np.int64),
                        cfg=json.dumps(CFG), seed=SEED, weights_sha256=weights_digest(W),
                        printed=text)
    print(text)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
