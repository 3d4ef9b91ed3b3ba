"""int8-KV prefill attention (tb_attn_prefill_q8) against the CPU restatement of
attentionQ8 at T > 1 (models/qwen3.js:2534-2577): causal over the cache, GQA,
positions S-T .. S-1.

Tolerance: each (query, head) output row within 2e-3 of that row's largest
magnitude (the kernel rounds Q, K, V and P to f16, unit roundoff 2^-11, and sums
in f32; the reference's own f16 kernel rounds the same operands and sums in f16)."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import host

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _case(seed, T, S, nHq, nKv, hd):
    rng = np.random.default_rng(seed)
    K = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    V = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    Kq, Ks = oracle.kv_quant_q8(K)
    Vq, Vs = oracle.kv_quant_q8(V)
    q = rng.normal(0, 1.5, (T, nHq * hd)).astype(np.float32)
    return q, Kq, Ks.reshape(S, -1), Vq, Vs.reshape(S, -1)


def _dev(*a):
    return [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in a]


def _row_err(got, ref, hd):
    g = np.asarray(got, np.float64).reshape(-1, hd)
    r = np.asarray(ref, np.float64).reshape(-1, hd)
    return float(np.max(np.max(np.abs(g - r), axis=1) / np.max(np.abs(r), axis=1)))


@pytest.mark.parametrize("T,S,nHq,nKv,hd", [(1, 1, 16, 8, 128), (5, 40, 4, 2, 64), (128, 128, 16, 8, 128),
                                            (200, 700, 16, 8, 128), (64, 300, 8, 1, 64), (77, 77, 8, 8, 128),
                                            (33, 1000, 16, 4, 128), (300, 300, 16, 8, 64)])
def test_prefill_matches_oracle(cuda, T, S, nHq, nKv, hd):
    q, Kq, Ks, Vq, Vs = _case(T * 7 + S, T, S, nHq, nKv, hd)
    qd, Kqd, Ksd, Vqd, Vsd = _dev(q, Kq, Ks, Vq, Vs)
    out = tb.attention_prefill_q8(qd, (Kqd, Ksd, Vqd, Vsd), S, nHq, nKv, hd)
    ref = oracle.attn_prefill_q8(q, Kq, Ks, Vq, Vs, T, S, nHq, nKv, hd)
    assert _row_err(host(out), ref, hd) < TOL
    # the last query of a prefill is the decode step at the same position
    dec = tb.attention_decode_q8(qd[-1].contiguous(), (Kqd, Ksd, Vqd, Vsd), S, nHq, nKv, hd, 0)
    assert _row_err(host(out)[-1], host(dec), hd) < TOL


def test_prefill_2048_tokens_sampled(cuda):
    """Config-4-sized prefill (2048 tokens of Qwen3-1.7B attention, one layer):
    a seeded sample of query rows against the oracle."""
    T = S = 2048
    nHq, nKv, hd = 16, 8, 128
    q, Kq, Ks, Vq, Vs = _case(2048, T, S, nHq, nKv, hd)
    out = host(tb.attention_prefill_q8(*_dev(q)[:1], tuple(_dev(Kq, Ks, Vq, Vs)), S, nHq, nKv, hd))
    for i in np.sort(np.random.default_rng(1).choice(T, 12, replace=False)):
        ref = oracle.attn_decode_q8(q[i], Kq, Ks, Vq, Vs, i + 1, nHq, nKv, hd)
        assert _row_err(out[i], ref, hd) < TOL, i


def test_prefill_rejects_bad_shapes(cuda):
    q, Kq, Ks, Vq, Vs = _case(0, 8, 8, 4, 2, 64)
    kv = tuple(_dev(Kq, Ks, Vq, Vs))
    with pytest.raises(tb.TabInferError):
        tb.attention_prefill_q8(_dev(q)[0], kv, 4, 4, 2, 64)      # T > S
    with pytest.raises(tb.TabInferError):
        tb.attention_prefill_q8(torch.zeros(8, 6 * 64, device="cuda"), kv, 8, 6, 2, 64)   # GQA group 3
