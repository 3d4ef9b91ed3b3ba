"""The CUDA decode step and prefill against the reference's own forward pass
(native/tools/ref_forward.py, run by tests/golden/make_ref_forward.py on a small
synthetic Bonsai-style checkpoint): the logits of the last prompt token within
REF_TOL max-abs of the reference's f32 logits and the same top token (the engine
runs int8 activations and an int8 cache; the bound is stated in
tests/test_ref_forward.py, where the CPU composition of the step meets it too).
Both step forms (one kernel per operation, and the persistent kernel) and the
prefill-then-decode route are checked."""
import numpy as np
import pytest

from helpers import u16_dev
from qwen3_oracle import make_weights
from test_ref_forward import check_logits, load_fixture


def _model(mode):
    import tabinfer_b200 as tb
    from tabinfer_b200 import _lib
    cfg, seed, ids, ref, _, _ = load_fixture()
    m = tb.Qwen3(dict(cfg, max_seq=64, batch=1))
    for name, w in make_weights(cfg, seed, ternary=True).items():
        assert m.load(name, u16_dev(w))
    m.set_step_mode({"kernels": _lib.QW_STEP_KERNELS, "persistent": _lib.QW_STEP_PERSISTENT}[mode])
    return m, ids, ref


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["kernels", "persistent"])
def test_decode_steps_match_reference_forward(cuda, mode):
    from tabinfer_b200 import _lib
    m, ids, ref = _model(mode)
    for pos, tok in enumerate(ids):
        m.set_tokens([tok], [pos])
        m.step()
    got = m.logits().numpy()[0]
    want_kind = _lib.QW_STEP_KERNELS if mode == "kernels" else _lib.QW_STEP_PERSISTENT
    assert m.step_kind() == want_kind
    err = check_logits(got, ref)
    assert m.tokens()[0][0] == int(np.argmax(got))
    m.close()
    print("decode (%s) vs reference forward: max-abs %.4f" % (mode, err))


@pytest.mark.gpu
def test_prefill_then_decode_matches_reference_forward(cuda):
    m, ids, ref = _model("kernels")
    m.prefill(0, ids[:-1], 0)
    m.set_tokens([ids[-1]], [len(ids) - 1])
    m.step()
    err = check_logits(m.logits().numpy()[0], ref)
    m.close()
    print("prefill + decode vs reference forward: max-abs %.4f" % err)
