"""GPU parity: int8 KV cache + split-KV GQA decode attention and decode glue
(models/qwen3.js:2048-2308, 2625-2690, 60-88, 1621-1675).

Bars: V quantize-write bit-exact (raw input); K (after norm+RoPE) within one
int8 step, only at rounding ties; q RoPE output within 1e-5 of the f64 oracle;
attention output of each q head within 1e-4 of that head row's largest
magnitude (max|got-ref| / max|ref|, f32 accumulation over S keys) against the
f64 oracle, for every split count (uneven and empty splits included); argmax
ids exact."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import host, u16_dev

pytestmark = pytest.mark.gpu


def _cache(S, nKv, hd, dev="cuda"):
    Kq = torch.zeros(S, nKv * hd, dtype=torch.int8, device=dev)
    Vq = torch.zeros_like(Kq)
    Ks = torch.zeros(S, nKv * hd // 32, dtype=torch.float32, device=dev)
    Vs = torch.zeros_like(Ks)
    return Kq, Ks, Vq, Vs


def _filled_cache(S, nKv, hd, seed):
    rng = np.random.default_rng(seed)
    K = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    V = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    Kq, Ks = oracle.kv_quant_q8(K)
    Vq, Vs = oracle.kv_quant_q8(V)
    return Kq, Ks.reshape(S, -1), Vq, Vs.reshape(S, -1)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def head_rel_err(got, ref, hd):
    got = np.asarray(got, np.float64).reshape(-1, hd)
    ref = np.asarray(ref, np.float64).reshape(-1, hd)
    return float(np.max(np.abs(got - ref).max(1) / np.abs(ref).max(1)))


@pytest.mark.parametrize("pos", [0, 17, 4095, 32767])
def test_attn_prep(cuda, pos):
    nHq, nKv, hd, S = 16, 8, 128, pos + 1
    rng = np.random.default_rng(pos)
    q = rng.normal(0, 1, nHq * hd).astype(np.float32)
    k = rng.normal(0, 1, nKv * hd).astype(np.float32)
    v = rng.normal(0, 1, nKv * hd).astype(np.float32)
    qw = np.float16(rng.uniform(0.5, 1.5, hd)).view(np.uint16)
    kw = np.float16(rng.uniform(0.5, 1.5, hd)).view(np.uint16)
    kv = _cache(S, nKv, hd)
    qr = tb.attn_prep_q8(_dev(q), _dev(k), _dev(v), u16_dev(qw), u16_dev(kw), kv, nHq, nKv, hd, pos, 1e6, 1e-6)
    qref = oracle.head_norm_rope(q.reshape(nHq, hd), qw, pos).reshape(-1)
    assert np.max(np.abs(host(qr) - qref)) < 1e-5
    Kq, Ks, Vq, Vs = [host(t) for t in kv]
    # V: raw -> bit-exact snorm quantization
    vq, vs = oracle.kv_quant_q8(v)
    np.testing.assert_array_equal(Vq[pos], vq)
    np.testing.assert_array_equal(Vs[pos], vs)
    # K: norm + RoPE in f64 on the oracle side; scales agree to f32 rounding,
    # codes to one step at ties
    kref = oracle.head_norm_rope(k.reshape(nKv, hd), kw, pos).reshape(-1).astype(np.float32)
    kq, ks = oracle.kv_quant_q8(kref)
    np.testing.assert_allclose(Ks[pos], ks, rtol=1e-5)
    assert np.max(np.abs(Kq[pos].astype(int) - kq.astype(int))) <= 1
    assert np.all(Kq[:pos] == 0) and np.all(Vq[:pos] == 0)   # other rows untouched


def test_kv_quant_write_bit_exact(cuda):
    T, nKv, hd, base = 5, 8, 128, 3
    rng = np.random.default_rng(1)
    kr = rng.normal(0, 2, (T, nKv * hd)).astype(np.float32)
    v = rng.normal(0, 2, (T, nKv * hd)).astype(np.float32)
    kv = _cache(base + T, nKv, hd)
    tb.kv_quant_write(_dev(kr), _dev(v), kv, T, nKv, hd, base)
    Kq, Ks, Vq, Vs = [host(t) for t in kv]
    kq, ks = oracle.kv_quant_q8(kr)
    vq, vs = oracle.kv_quant_q8(v)
    np.testing.assert_array_equal(Kq[base:], kq)
    np.testing.assert_array_equal(Vq[base:], vq)
    np.testing.assert_array_equal(Ks[base:].reshape(-1), ks)
    np.testing.assert_array_equal(Vs[base:].reshape(-1), vs)


@pytest.mark.parametrize("S", [1, 7, 128, 300, 4096])
@pytest.mark.parametrize("nsplit", [0, 1, 3, 16, 64])
def test_decode_attention_splits(cuda, S, nsplit):
    nHq, nKv, hd = 16, 8, 128
    Kq, Ks, Vq, Vs = _filled_cache(S, nKv, hd, S)
    q = np.random.default_rng(S + 1).normal(0, 1, nHq * hd).astype(np.float32)
    out = tb.attention_decode_q8(_dev(q), (_dev(Kq), _dev(Ks), _dev(Vq), _dev(Vs)), S, nHq, nKv, hd, nsplit)
    ref = oracle.attn_decode_q8(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd)
    assert head_rel_err(host(out), ref, hd) < 1e-4


@pytest.mark.parametrize("nHq,nKv,hd", [(8, 8, 64), (16, 4, 128), (32, 4, 64), (8, 1, 128)])
def test_decode_attention_head_layouts(cuda, nHq, nKv, hd):
    S = 777
    Kq, Ks, Vq, Vs = _filled_cache(S, nKv, hd, nHq)
    q = np.random.default_rng(2).normal(0, 1, nHq * hd).astype(np.float32)
    out = tb.attention_decode_q8(_dev(q), (_dev(Kq), _dev(Ks), _dev(Vq), _dev(Vs)), S, nHq, nKv, hd)
    ref = oracle.attn_decode_q8(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd)
    assert head_rel_err(host(out), ref, hd) < 1e-4


def test_decode_attention_32k_context(cuda):
    """Config 3 at S = 32768 (1.7B heads), sampled against the oracle."""
    nHq, nKv, hd, S = 16, 8, 128, 32768
    Kq, Ks, Vq, Vs = _filled_cache(S, nKv, hd, 99)
    q = np.random.default_rng(5).normal(0, 1, nHq * hd).astype(np.float32)
    out = tb.attention_decode_q8(_dev(q), (_dev(Kq), _dev(Ks), _dev(Vq), _dev(Vs)), S, nHq, nKv, hd)
    ref = oracle.attn_decode_q8(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd)
    assert head_rel_err(host(out), ref, hd) < 1e-4


def test_argmax_reference_selftests(cuda):
    """qwen3.js:3159-3178: max at 3712 of 5000; two-stage vocab case max at 98765 of 151936
    written at outPos 2."""
    a = np.sin(np.arange(5000) * 0.017).astype(np.float32)
    a[3712] = 99.0
    assert host(tb.argmax(_dev(a)))[0] == 3712
    b = (np.sin(np.arange(151936) * 0.0007) * 3).astype(np.float32)
    b[98765] = 99.0
    out = torch.zeros(4, dtype=torch.int32, device="cuda")
    tb.argmax(_dev(b), out=out, offset=2)
    assert list(host(out)) == [0, 0, 98765, 0]


def test_argmax_ties_rows_and_nan(cuda):
    x = np.random.default_rng(0).normal(0, 1, (3, 151936)).astype(np.float32)
    x[0, [10, 20000, 150000]] = 50.0       # ties -> lowest index
    x[1, 5] = np.nan                       # NaN never wins
    got = host(tb.argmax(_dev(x)))
    assert got[0] == 10
    assert got[1] == oracle.argmax(np.where(np.isnan(x[1]), -np.inf, x[1]))
    assert got[2] == oracle.argmax(x[2])


def test_rmsnorm_and_embed(cuda):
    rng = np.random.default_rng(8)
    T, H = 3, 2048
    x = rng.normal(0, 2, (T, H)).astype(np.float32)
    w = np.float16(rng.uniform(0.5, 1.5, H))
    y = host(tb.rmsnorm(_dev(x), u16_dev(w.view(np.uint16)), 1e-6))
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * w.astype(np.float64)
    np.testing.assert_allclose(y, ref, rtol=2e-6, atol=1e-6)
    emb = np.float16(rng.normal(0, 1, (1000, 64)))
    ids = np.array([0, 5, 999, 5, 7], np.uint32)
    out = host(tb.embed_gather(_dev(ids.view(np.int32)), _dev(emb.view(np.int16)), 3, idoff=1))
    np.testing.assert_array_equal(out, emb[ids[1:4]].astype(np.float32))
