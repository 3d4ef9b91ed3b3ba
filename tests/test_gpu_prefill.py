"""The prefill forward (tb_qwen3_prefill: forward(ids, posBase) at T > 1,
models/qwen3.js:3938-4069) against the composed oracle run token by token.

The oracle runs the prefill tokens one by one with the reference's prefill
arithmetic: the GEMMs' exact int8 group sums (gemmDP4A / gemmTern, as the
kernels compute them) and the attention at the operand precision of the
reference's f16 prefill kernel (Q, K, V, P rounded to f16 -- the kernel sums in
f32, the oracle exactly).  The last row's logits are within 5e-2 max-abs (see
LOGIT_TOL), the
returned token is the oracle's argmax where its top-2 margin is clear, the
dequantized cache rows match within 1e-2 of each row's largest magnitude at
layer 0 (the RMSNorm's f32 reduction order can flip an int8 activation code at a
tie) and 5e-2 deeper (the attention's f32 sums flip codes of each layer's input,
and every re-quantization carries them on), the position advances, and decode steps continue from the prefilled state.  (Against an
f32-attention oracle the int8 re-quantization of every layer amplifies the f16
rounding -- a perturbation that moves a value across a rounding boundary shifts
it by 1/127 of its group maximum -- to ~1e-2 on these small models' logits.)"""
import numpy as np
import pytest

import tabinfer_b200 as tb
from helpers import u16_dev
from qwen3_oracle import OracleModel, make_weights
from test_gpu_qwen3 import SMALL, _check_step

pytestmark = pytest.mark.gpu

# Two exact-arithmetic oracles that differ only in the attention's operand
# precision (f32 vs the reference's f16 prefill kernel) already differ by 1.2e-2 to
# 2.5e-2 on these small models' logits: every layer re-quantizes its input to int8,
# so any last-bit difference in the attention (here: f32 sums against exact sums)
# that moves a value across a rounding boundary is carried on.  The prefill is held
# to twice that spread.
LOGIT_TOL = 5e-2


def _model(cfg, W):
    m = tb.Qwen3(cfg)
    for name, w in W.items():
        assert m.load(name, u16_dev(w))
    return m


def _oracle_run(om, cfg, toks, cache, start=0):
    """the prefill tokens through the oracle one by one, attention at the
    reference's f16 prefill-kernel operand precision"""
    ref = None
    for p, t in enumerate(toks):
        ref = om.step(t, start + p, cache, attn_f16ops=True)
    return ref


def _empty_cache(cfg):
    row = cfg["n_kv_heads"] * cfg["head_dim"]
    S = cfg["max_seq"]
    return [(np.zeros((S, row), np.int8), np.zeros((S, row // 32), np.float32), np.zeros((S, row), np.int8),
             np.zeros((S, row // 32), np.float32)) for _ in range(cfg["layers"])]


def _compare(m, seq, cfg, ref, cache, T):
    got = m.logits().numpy()[seq]
    err = float(np.max(np.abs(got - ref)))
    assert err <= LOGIT_TOL, "logits max-abs err %.3g" % err
    ids, pos = m.tokens()
    assert pos[seq] == T
    top2 = np.sort(ref)[-2:]
    if top2[1] - top2[0] > 2 * LOGIT_TOL:
        assert ids[seq] == int(np.argmax(ref))
    for l in range(cfg["layers"]):
        Kq, Ks, Vq, Vs = (a[seq] for a in m.kv_host(l))
        rK, rKs, rV, rVs = cache[l]
        for got, ref, sg, sr, what in ((Kq, rK, Ks, rKs, "K"), (Vq, rV, Vs, rVs, "V")):
            deq = [q[:T].astype(np.float64) / 127 * np.repeat(sc[:T].astype(np.float64), 32, axis=1)
                   for q, sc in ((got, sg), (ref, sr))]
            rel = np.max(np.abs(deq[0] - deq[1]), axis=1) / np.max(np.abs(deq[1]), axis=1)
            bound = 1e-2 if l == 0 else 5e-2
            assert float(np.max(rel)) < bound, "layer %d %s: %.3g" % (l, what, float(np.max(rel)))


@pytest.mark.parametrize("ternary", [False, True])
def test_prefill_then_decode_matches_oracle(cuda, ternary):
    cfg = dict(SMALL, batch=2, max_seq=256)
    W = make_weights(cfg, 51, ternary=ternary)
    m = _model(cfg, W)
    om = OracleModel(cfg, W)
    rng = np.random.default_rng(52)
    toks = [rng.integers(0, cfg["vocab"], n).tolist() for n in (37, 140)]
    caches = []
    for seq, tk in enumerate(toks):
        nxt = m.prefill(seq, tk, 0)
        cache = _empty_cache(cfg)
        ref = _oracle_run(om, cfg, tk, cache)
        _compare(m, seq, cfg, ref, cache, len(tk))
        assert nxt == m.tokens()[0][seq]
        caches.append(cache)
    # decode continues from the prefilled caches (the step reads the GPU's own state)
    ids, pos = m.tokens()
    ids2, pos2 = _check_step(m, om, cfg, ids, pos, route_f32=False)
    _check_step(m, om, cfg, ids2, pos2, route_f32=False)
    m.close()


def test_chunked_prefill_crosses_tiles(cuda):
    """Two prefills of one sequence (positions 0..99 then 100..229): the second
    attends to the first chunk's cache rows; the result equals one long run."""
    cfg = dict(SMALL, batch=1, max_seq=256)
    W = make_weights(cfg, 61)
    m = _model(cfg, W)
    om = OracleModel(cfg, W)
    tk = np.random.default_rng(62).integers(0, cfg["vocab"], 230).tolist()
    m.prefill(0, tk[:100], 0)
    m.prefill(0, tk[100:], 100)
    cache = _empty_cache(cfg)
    ref = _oracle_run(om, cfg, tk, cache)
    _compare(m, 0, cfg, ref, cache, 230)
    m.close()


def test_prefill_rejects_what_does_not_fit(cuda):
    cfg = dict(SMALL, batch=1, max_seq=64)
    m = _model(cfg, make_weights(cfg, 71))
    with pytest.raises(tb.TabInferError):
        m.prefill(0, list(range(60)), 10)          # 70 > 64 cache rows
    with pytest.raises(tb.TabInferError):
        m.prefill(1, [1, 2, 3], 0)                 # no sequence 1
    m.close()
