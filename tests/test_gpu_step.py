"""The persistent decode step (tb_step.cu: embed and every layer in one kernel,
grid barriers between the phases) against the multi-kernel step on identical
models: logits bit-identical, the same ids, positions and cache rows, over
several consecutive steps (graph replays), at the small test shapes and at
Qwen3-1.7B width (context 4096, the bench's attention split), with int4 and
with Bonsai-style ternary layer weights, plus the oracle check of the
persistent path at batch 1."""
import numpy as np
import pytest

import tabinfer_b200 as tb
from tabinfer_b200 import _lib
from qwen3_oracle import OracleModel, make_weights
from test_gpu_qwen3 import SMALL, _build, _check_step

pytestmark = pytest.mark.gpu

WIDE = dict(hidden=2048, layers=2, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=6144, vocab=20000,
            rope_theta=1e6, rms_eps=1e-6, max_seq=4200, batch=1)


def _pair(cfg, seed, prefill, ternary=False):
    out = []
    for mode in (_lib.QW_STEP_KERNELS, _lib.QW_STEP_PERSISTENT):
        W, m = _build(cfg, seed, prefill, ternary)
        m.set_step_mode(mode)
        out.append(m)
    return out


@pytest.mark.parametrize("cfg,prefill,ternary", [(dict(SMALL, batch=1), [23], False),
                                                 (dict(SMALL, batch=1, n_heads=8, n_kv_heads=8), [40], False),
                                                 (dict(SMALL, batch=1, max_seq=1024, layers=3), [700], False),
                                                 (WIDE, [4095], False),
                                                 (dict(SMALL, batch=1), [23], True),
                                                 (dict(SMALL, batch=1, max_seq=1024, layers=3), [700], True),
                                                 (WIDE, [4095], True)])
def test_persistent_step_equals_kernels(cuda, cfg, prefill, ternary):
    mk, mp = _pair(cfg, 31, prefill, ternary)
    if ternary:
        assert mp.weight_format("model.layers.0.mlp.down_proj.weight") == _lib.QW_FMT_TERN
    ids = [777 % cfg["vocab"]]
    for m in (mk, mp):
        m.set_tokens(ids, prefill)
    for step in range(3):
        for m in (mk, mp):
            m.step()
        assert mk.step_kind() == _lib.QW_STEP_KERNELS and mp.step_kind() == _lib.QW_STEP_PERSISTENT
        np.testing.assert_array_equal(mp.logits().numpy(), mk.logits().numpy(), err_msg="step %d" % step)
        assert mp.tokens() == mk.tokens()
    n = prefill[0] + 3                    # rows past these were never written (uninitialised)
    for l in range(cfg["layers"]):
        for a, b in zip(mp.kv_host(l), mk.kv_host(l)):
            np.testing.assert_array_equal(a[:, :n], b[:, :n])
    assert mp.ctx.device_error() == 0
    k, c = mp.launches_per_step()
    assert 0 < k <= 4 and c == 0          # the persistent kernel, lm_head, argmax
    for m in (mk, mp):
        m.close()


def test_persistent_step_matches_oracle(cuda):
    cfg = dict(SMALL, batch=1, layers=2)
    W, m = _build(cfg, 41, [17])
    m.set_step_mode(_lib.QW_STEP_PERSISTENT)
    om = OracleModel(cfg, W)
    m.set_tokens([5], [17])
    ids, pos = _check_step(m, om, cfg, [5], [17], route_f32=False)
    _check_step(m, om, cfg, ids, pos, route_f32=False)
    assert m.step_kind() == _lib.QW_STEP_PERSISTENT
    m.close()


def test_persistent_mode_refused_where_it_does_not_apply(cuda):
    cfg = dict(SMALL, batch=2)
    W, m = _build(cfg, 43, [3, 4])
    m.set_step_mode(_lib.QW_STEP_PERSISTENT)
    with pytest.raises(tb.TabInferError):
        m.step()
    m.set_step_mode(_lib.QW_STEP_AUTO)
    m.step()
    assert m.step_kind() == _lib.QW_STEP_KERNELS
    m.close()


def test_persistent_ternary_step_matches_oracle(cuda):
    cfg = dict(SMALL, batch=1, layers=2)
    W, m = _build(cfg, 45, [11], ternary=True)
    m.set_step_mode(_lib.QW_STEP_PERSISTENT)
    om = OracleModel(cfg, W)
    assert all(om.tern.values())
    m.set_tokens([8], [11])
    ids, pos = _check_step(m, om, cfg, [8], [11], route_f32=False)
    _check_step(m, om, cfg, ids, pos, route_f32=False)
    assert m.step_kind() == _lib.QW_STEP_PERSISTENT
    m.close()


def test_step_follows_weight_format_changes(cuda):
    """The persistent kernel needs one format for every layer matrix: a ternary
    model runs it; with one int4 matrix among ternary ones AUTO records the
    multi-kernel step and PERSISTENT is refused; with every layer matrix int4
    the persistent step is planned again, for the new format, and still matches
    the oracle."""
    from helpers import u16_dev
    cfg = dict(SMALL, batch=1)
    W, m = _build(cfg, 49, [6], ternary=True)
    m.set_tokens([4], [6])
    m.step()
    assert m.step_kind() == _lib.QW_STEP_PERSISTENT
    I4 = make_weights(cfg, 50)
    layer_mats = [n for n in W if ".layers." in n and n.endswith("proj.weight")]
    assert len(layer_mats) == 7 * cfg["layers"]
    m.load(layer_mats[0], u16_dev(I4[layer_mats[0]]))
    assert m.weight_format(layer_mats[0]) == _lib.QW_FMT_INT4
    m.step()
    assert m.step_kind() == _lib.QW_STEP_KERNELS
    m.set_step_mode(_lib.QW_STEP_PERSISTENT)
    with pytest.raises(tb.TabInferError):
        m.step()
    for n in layer_mats[1:]:
        m.load(n, u16_dev(I4[n]))
    W2 = dict(W, **{n: I4[n] for n in layer_mats})
    om = OracleModel(cfg, W2)
    ids, pos = m.tokens()
    ids, pos = _check_step(m, om, cfg, ids, pos, route_f32=False)
    assert m.step_kind() == _lib.QW_STEP_PERSISTENT
    _check_step(m, om, cfg, ids, pos, route_f32=False)
    assert m.ctx.device_error() == 0
    m.close()


def test_phase_trace_stamps_are_ordered(cuda):
    """tb_qwen3_step_trace: every CTA stamps the kernel start and, for each layer
    and phase, weights ready <= phase done <= barrier passed, phases in order."""
    import torch
    cfg = dict(SMALL, batch=1, layers=2)
    W, m = _build(cfg, 47, [9])
    m.set_tokens([3], [9])
    m.step()
    assert m.step_kind() == _lib.QW_STEP_PERSISTENT
    L = cfg["layers"]
    G = torch.cuda.get_device_properties(0).multi_processor_count
    buf = torch.zeros(G, 1 + 38 * L, dtype=torch.int64, device="cuda")
    m.step_trace(buf)
    m.step_layers()
    t = buf.cpu().numpy()
    m.step_trace(None)
    assert (t[:, 0] > 0).all()
    ph = t[:, 1:1 + 25 * L].reshape(G, L, 5, 5)       # ready, loaded, staged, done, out
    ready, done, out = ph[:, :, :, 0], ph[:, :, :, 3], ph[:, :, :, 4]
    last = (slice(None), L - 1, 4)                    # the last phase has no barrier after it
    assert (ready > 0).all() and (done >= ready).all()
    out[last] = done[last]
    assert (out >= done).all()
    flat_ready = ready.reshape(G, -1)
    assert (np.diff(flat_ready, axis=1) >= 0).all()
    assert m.ctx.device_error() == 0
    m.close()
