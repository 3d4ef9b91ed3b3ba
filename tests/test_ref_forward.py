"""Pin of the decode-step structure against the reference's own forward pass.

tests/golden/ref_forward_bonsai.npz holds the logits that the reference's numpy
forward (native/tools/ref_forward.py:50-112, executed by
tests/golden/make_ref_forward.py) computed for a 13-token prompt on a small
synthetic Bonsai-style checkpoint (ternary bf16 projections and lm_head).  The
reference runs in f32 throughout; the engine quantizes activations to int8
(QUANTQ8) before every GEMV and keeps the cache in int8 per-32 groups, so the
logits agree within REF_TOL max-abs, not exactly, and the top token must agree
wherever the reference's top-2 margin exceeds twice that.

Here (CPU): the checkpoint regenerates bit for bit, and the CPU composition of
the engine's step (tests/qwen3_oracle.py, which the GPU parity tests use) meets
that bar against the reference's logits.  test_gpu_ref_forward.py runs the CUDA
step itself against the same fixture.
"""
import json
import os

import numpy as np

from golden.make_ref_forward import weights_digest
from qwen3_oracle import OracleModel, make_weights

HERE = os.path.dirname(os.path.abspath(__file__))
REF_TOL = 5e-2      # int8 activations + int8 KV vs the reference's f32 forward


def load_fixture():
    f = np.load(os.path.join(HERE, "golden", "ref_forward_bonsai.npz"))
    cfg = json.loads(str(f["cfg"]))
    return cfg, int(f["seed"]), [int(t) for t in f["ids"]], f["logits"].astype(np.float64), f["top10"], \
        str(f["weights_sha256"])


def check_logits(got, ref, tol=REF_TOL):
    got = np.asarray(got, np.float64)
    err = float(np.max(np.abs(got - ref)))
    assert err <= tol, "logits max-abs err %.4g > %.3g" % (err, tol)
    order = np.argsort(-ref)
    if ref[order[0]] - ref[order[1]] > 2 * tol:
        assert int(np.argmax(got)) == int(order[0]), "top-1 id differs from the reference forward"
    # every reference top-5 token stays in the engine's top 10
    assert set(order[:5].tolist()) <= set(np.argsort(-got)[:10].tolist())
    return err


def test_fixture_checkpoint_regenerates():
    cfg, seed, _, ref, top10, digest = load_fixture()
    W = make_weights(cfg, seed, ternary=True)
    assert weights_digest(W) == digest
    assert np.array_equal(np.argsort(-ref)[:10], top10)


def test_composed_step_oracle_matches_reference_forward():
    cfg, seed, ids, ref, _, _ = load_fixture()
    om = OracleModel(cfg, make_weights(cfg, seed, ternary=True), ternary=True)
    assert all(om.tern.values())
    ms, row = 64, cfg["n_kv_heads"] * cfg["head_dim"]
    cache = [(np.zeros((ms, row), np.int8), np.zeros((ms, row // 32), np.float32),
              np.zeros((ms, row), np.int8), np.zeros((ms, row // 32), np.float32)) for _ in range(cfg["layers"])]
    for pos, tok in enumerate(ids):
        logits = om.step(tok, pos, cache)
    check_logits(logits, ref)
