"""Parity of the recorded Qwen3 decode step (tb_qwen3_*) with the CPU oracle of
models/qwen3.js forward (T = 1, int8 KV): logits within 2e-2 max-abs, argmax
ids equal wherever the top-2 margin exceeds that tolerance, positions advanced,
the cache rows the step wrote equal to the oracle's (int8 within 1, scales
2e-3 rel: one RMSNorm tie flip), and a replay of the recorded step continuing from the GPU's state."""
import numpy as np
import pytest
import torch

from helpers import u16_dev
from qwen3_oracle import OracleModel, make_weights

LOGIT_TOL = 2e-2

SMALL = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, vocab=1000,
             rope_theta=1e6, rms_eps=1e-6, max_seq=64)


def _build(cfg, seed, prefill, ternary=False):
    import tabinfer_b200 as tb
    W = make_weights(cfg, seed, ternary=ternary)
    m = tb.Qwen3(cfg)
    for name, w in W.items():
        assert m.load(name, u16_dev(w))
    rng = np.random.default_rng(seed + 1)
    row = cfg["n_kv_heads"] * cfg["head_dim"]
    for l in range(cfg["layers"]):
        for b, n in enumerate(prefill):
            if n == 0:
                continue
            k = torch.from_numpy(rng.standard_normal((n, row)).astype(np.float32)).cuda()
            v = torch.from_numpy(rng.standard_normal((n, row)).astype(np.float32)).cuda()
            m.kv_fill(l, b, k, v, 0)
    return W, m


def _check_step(m, om, cfg, ids, pos, route_f32):
    B, L = cfg["batch"], cfg["layers"]
    before = [m.kv_host(l) for l in range(L)]
    m.step()
    got = m.logits().numpy()
    new_ids, new_pos = m.tokens()
    after = [m.kv_host(l) for l in range(L)]
    assert new_pos == [p + 1 for p in pos]
    for b in range(B):
        cache = [tuple(a[b].copy() for a in before[l]) for l in range(L)]
        ref = om.step(ids[b], pos[b], cache, route_f32)
        err = float(np.max(np.abs(got[b] - ref)))
        assert err <= LOGIT_TOL, "seq %d: logits max-abs err %.3g" % (b, err)
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 2 * LOGIT_TOL:
            assert new_ids[b] == int(np.argmax(ref)), "seq %d: argmax" % b
        for l in range(L):
            for i, (g, r) in enumerate(zip((a[b][pos[b]] for a in after[l]), (c[pos[b]] for c in cache[l]))):
                if i in (0, 2):
                    assert np.max(np.abs(g.astype(np.int32) - r.astype(np.int32))) <= 1, "layer %d int8 row" % l
                else:
                    # f32 scales of the row: a one-LSB RMSNorm tie flip in the int8
                    # activation (the quantizers agree up to ties) moves every output
                    # of a 256-wide dot product by about 1/(127*16)
                    np.testing.assert_allclose(g, r, rtol=2e-3)
    return new_ids, new_pos


@pytest.mark.gpu
@pytest.mark.parametrize("batch,hd,heads,max_seq,layers", [(2, 128, (4, 2), 64, 2), (9, 64, (8, 2), 64, 2),
                                                           (1, 128, (8, 8), 64, 2), (2, 128, (4, 2), 1024, 1),
                                                           (3, 128, (16, 8), 4096, 1), (1, 64, (8, 1), 2000, 1),
                                                           (16, 128, (4, 2), 64, 1)])
def test_decode_step_matches_oracle(cuda, batch, hd, heads, max_seq, layers):
    """max_seq sets the attention's split count (the automatic rule at S_max =
    max_seq), so the larger cases combine many splits."""
    cfg = dict(SMALL, batch=batch, head_dim=hd, n_heads=heads[0], n_kv_heads=heads[1], max_seq=max_seq,
               layers=layers)
    prefill = [(5 + 7 * b) % 40 if max_seq <= 64 else (max_seq * (b + 1)) // (batch + 2) + 3 * b
               for b in range(batch)]
    W, m = _build(cfg, 11 + batch, prefill)
    om = OracleModel(cfg, W)
    ids = [(17 + 131 * b) % cfg["vocab"] for b in range(batch)]
    m.set_tokens(ids, prefill)
    ids2, pos2 = _check_step(m, om, cfg, ids, prefill, route_f32=False)
    # second token: replay of the recorded step from the state the first left
    _check_step(m, om, cfg, ids2, pos2, route_f32=False)
    kernels, coll = m.launches_per_step()
    assert coll == 0 and kernels > 0
    m.close()


@pytest.mark.gpu
def test_decode_step_lm_head_f32_route(cuda):
    """batch 1 with vocab >= 16384: the lm_head runs as gemvQ on the f32 row
    (linearQ's routing, qwen3.js:1588-1608)."""
    cfg = dict(SMALL, layers=1, vocab=16384, batch=1)
    W, m = _build(cfg, 5, [12])
    om = OracleModel(cfg, W)
    m.set_tokens([4321], [12])
    _check_step(m, om, cfg, [4321], [12], route_f32=True)
    m.close()


@pytest.mark.gpu
def test_decode_step_position_out_of_cache_sets_error(cuda):
    """A device position past the cache is refused on the device: the error word
    is set and nothing is written outside the cache."""
    import tabinfer_b200 as tb
    cfg = dict(SMALL, layers=1, batch=1, max_seq=16)
    W, m = _build(cfg, 3, [0])
    m.set_tokens([1], [16])
    m.step()
    m.ctx.synchronize()
    code = m.ctx.device_error()
    assert code == 0x6a01, hex(code)
    assert tb.default_context(0).device_error() == 0   # reading cleared it
    m.close()


@pytest.mark.gpu
def test_generate_greedy_tokens_follow_oracle(cuda):
    """Four greedy tokens through generate(): each step's input id is the
    previous step's argmax (the reference's GPU token history)."""
    cfg = dict(SMALL, layers=1, batch=1)
    W, m = _build(cfg, 21, [6])
    om = OracleModel(cfg, W)
    m.set_tokens([99], [6])
    cache = [tuple(a[0].copy() for a in m.kv_host(0))]
    toks = m.generate(4)
    tok, pos = 99, 6
    for t in toks:
        ref = om.step(tok, pos, cache)
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] <= 2 * LOGIT_TOL:
            break          # a near-tie: later tokens may legitimately differ
        assert t[0] == int(np.argmax(ref))
        tok, pos = t[0], pos + 1
    m.close()


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [4, 12])
def test_batched_ternary_step_matches_oracle(cuda, batch):
    """A ternary (WebGPU layout) checkpoint at 2..16 sequences: the tensor-core GEMVs on
    the ternary codes, with the attention and the gate/up epilogue writing the next
    GEMV's rows in the ternary fragment order, against the composed oracle."""
    cfg = dict(SMALL, batch=batch, layers=2)
    prefill = [(5 + 7 * b) % 40 for b in range(batch)]
    W, m = _build(cfg, 61 + batch, prefill, ternary=True)
    om = OracleModel(cfg, W)
    assert all(om.tern.values())
    ids = [(17 + 131 * b) % cfg["vocab"] for b in range(batch)]
    m.set_tokens(ids, prefill)
    ids2, pos2 = _check_step(m, om, cfg, ids, prefill, route_f32=False)
    _check_step(m, om, cfg, ids2, pos2, route_f32=False)
    m.close()
