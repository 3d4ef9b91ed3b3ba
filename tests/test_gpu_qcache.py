"""Bonsai-style ternary checkpoints through the Qwen3 decode step, and the
quantized-weights cache round trip.

* A checkpoint whose projections are ternary loads, as the reference loader does
  (_uploadTensor, models/qwen3.js:3503-3523), as ternary WebGPU-layout records;
  the recorded decode step then runs gemvTern / gateupTern and matches the
  composed oracle (logits within 2e-2 max-abs, argmax where the margin allows).
* A mixed checkpoint (some ternary tensors, some not -- q/k/v of one layer of
  different kinds) written to the cache (QuantSink / write_quant_cache) and
  loaded from it (load_quant_cache) gives a model whose weight kinds equal the
  quantize-on-arrival model's and whose decode steps are bit-identical to it."""
import numpy as np
import pytest

import tabinfer_b200 as tb
from tabinfer_b200 import qcache, _lib
from helpers import tern_bf16, u16_dev
from qwen3_oracle import OracleModel, make_weights
from test_gpu_qwen3 import SMALL, _check_step

pytestmark = pytest.mark.gpu


def _model(cfg, W):
    m = tb.Qwen3(cfg)
    for name, w in W.items():
        assert m.load(name, u16_dev(w))
    return m


@pytest.mark.parametrize("batch", [1, 3])
def test_ternary_checkpoint_decode_matches_oracle(cuda, batch):
    cfg = dict(SMALL, batch=batch, max_seq=64)
    W = make_weights(cfg, 21, ternary=True)
    m = _model(cfg, W)
    for name in W:
        if qcache.is_quant_weight(name):
            assert m.weight_format(name) == _lib.QW_FMT_TERN, name
    om = OracleModel(cfg, W)
    assert all(om.tern.values())
    ids = [(5 + 101 * b) % cfg["vocab"] for b in range(batch)]
    pos = [0] * batch
    m.set_tokens(ids, pos)
    ids2, pos2 = _check_step(m, om, cfg, ids, pos, route_f32=False)
    _check_step(m, om, cfg, ids2, pos2, route_f32=False)
    m.close()


def _mixed_weights(cfg):
    W = make_weights(cfg, 33)
    T = make_weights(cfg, 34, ternary=True)
    rng = np.random.default_rng(35)
    for name in ("model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.v_proj.weight",
                 "model.layers.1.mlp.gate_proj.weight", "model.layers.1.mlp.up_proj.weight",
                 "model.layers.1.mlp.down_proj.weight", "lm_head.weight"):
        W[name] = T[name]
    # a tensor that is ternary but for one group 3 ulps off: int4
    w = tern_bf16(rng, *W["model.layers.0.self_attn.o_proj.weight"].shape)
    g = w[0, :32]
    i = int(np.flatnonzero(g & 0x7FFF)[0])
    w[0, i] = (int(np.max(g & 0x7FFF)) - 3) | (int(g[i]) & 0x8000)
    W["model.layers.0.self_attn.o_proj.weight"] = w
    return W


def test_quant_cache_round_trip_is_bit_identical(cuda, tmp_path):
    cfg = dict(SMALL, batch=2, max_seq=64)
    W = _mixed_weights(cfg)
    a = _model(cfg, W)
    qcache.write_quant_cache(str(tmp_path), "small", cfg, ((n, u16_dev(w)) for n, w in W.items()),
                             chunk_size=1 << 20)
    m = qcache.read_manifest(str(tmp_path), "small", cfg, 1 << 20)
    assert m is not None and m["nChunks"] > 1
    kinds = {s["name"]: s["kind"] for s in m["segs"]}
    assert kinds["lm_head.weight"] == "tern" and kinds["model.layers.0.self_attn.o_proj.weight"] == "int4"
    assert kinds["model.layers.0.self_attn.k_proj.weight"] == "int4" and kinds["model.norm.weight"] == "f16"
    b = tb.Qwen3(cfg)
    assert not qcache.load_quant_cache(b, str(tmp_path), "other")
    assert qcache.load_quant_cache(b, str(tmp_path), "small", chunk_size=1 << 20)
    for name in W:
        assert a.weight_format(name) == b.weight_format(name), name
    ids, pos = [7, 900], [0, 0]
    for mm in (a, b):
        mm.set_tokens(ids, pos)
    for _ in range(3):
        a.step()
        b.step()
        np.testing.assert_array_equal(a.logits().numpy(), b.logits().numpy())
        assert a.tokens() == b.tokens()
    # and the mixed model against the oracle (mixed q/k/v kinds take per-matrix launches)
    om = OracleModel(cfg, W)
    c = _model(cfg, W)
    c.set_tokens(ids, pos)
    _check_step(c, om, cfg, ids, pos, route_f32=False)
    for mm in (a, b, c):
        mm.close()
