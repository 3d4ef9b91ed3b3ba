"""CPU tests: the oracle pinned against the reference's own golden data and
known-answer tests, before it is trusted to judge the CUDA kernels.

* ternary packing: bit-exact against the reference's own numpy packer
  (native/tools/pack_bin.py, executed by tests/golden/make_golden.py);
* ternary GEMV: the tern.rs test suite restated (tern.rs:405-470) and the n2
  selftest shapes (n2-cli main.rs:116-160);
* int4 quantizer: bit-exact against a second, independent restatement of the
  JS (tests/golden/int4_js.npz) and hand-worked known answers from the JS text;
* WGSL self-test fixtures and tolerances (models/qwen3.js:3077-3157).
"""
import numpy as np
import pytest

import oracle


# ---------------------------------------------------------------- ternary

TERN_SHAPES = [("tern_rs_oracle", 0x2026_0805, [(1, 64), (3, 128), (17, 256), (8, 1024)]),
               ("tern_rs_avx2", 0xC0FFEE, [(1, 64), (1, 192), (5, 192), (17, 256), (64, 2048)])]


@pytest.mark.parametrize("tag,base,dims", TERN_SHAPES)
def test_pack_ternary_matches_reference_numpy(golden, tag, base, dims):
    for n, k in dims:
        codes, scales, _, _, w, _ = oracle.tern_fixture(n, k, base + k)
        np.testing.assert_array_equal(codes, golden["tern"][f"{tag}_{n}x{k}_codes"])
        np.testing.assert_array_equal(scales, golden["tern"][f"{tag}_{n}x{k}_scales"])


def test_pack_ternary_config1_matches_reference_numpy(golden):
    w = golden["tern"]["config1_w"]
    codes, scales = oracle.pack_ternary(w)
    np.testing.assert_array_equal(codes, golden["tern"]["config1_codes"])
    np.testing.assert_array_equal(scales, golden["tern"]["config1_scales"])


def _max_rel(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return float(np.max(np.abs(a - b) / np.maximum(np.maximum(np.abs(a), np.abs(b)), 1e-3)))


def test_scalar_matches_dequant_oracle():
    """tern.rs:405-416"""
    for n, k in [(1, 64), (3, 128), (17, 256), (8, 1024)]:
        codes, scales, act, xsum, _, _ = oracle.tern_fixture(n, k, 0x2026_0805 + k)
        got = oracle.gemv_tern_scalar(codes, scales, act, xsum)[0]
        want = oracle.gemv_tern_dequant(codes, scales, act)[0]
        assert _max_rel(got, want) < 1e-5, (n, k)


def test_avx2_transcription_matches_scalar():
    """tern.rs:418-435 (includes an odd block count to hit the scalar tail)"""
    for n, k in [(1, 64), (1, 192), (5, 192), (17, 256), (64, 2048)]:
        codes, scales, act, xsum, _, _ = oracle.tern_fixture(n, k, 0xC0FFEE + k)
        a = oracle.gemv_tern_scalar(codes, scales, act, xsum)[0]
        b = oracle.gemv_tern_avx2(codes, scales, act, xsum)
        assert _max_rel(a, b) < 1e-5, (n, k)
        c = oracle.gemv_tern_avx2(codes, scales, act, xsum, threads=4)
        np.testing.assert_array_equal(b, c)


def test_timed_scalar_baseline_is_the_oracle_scalar():
    """The timed scalar baseline (-O3 build) gives the oracle's gemv_tern_scalar bits."""
    for n, k in [(1, 64), (5, 192), (64, 2048)]:
        codes, scales, act, xsum, _, _ = oracle.tern_fixture(n, k, 0xBEEF + k)
        a = oracle.gemv_tern_scalar(codes, scales, act, xsum)[0]
        np.testing.assert_array_equal(oracle.gemv_tern_scalar_timed(codes, scales, act, xsum), a)
        np.testing.assert_array_equal(oracle.gemv_tern_scalar_timed(codes, scales, act, xsum, threads=3), a)


def test_selftest_shapes():
    """n2 selftest (main.rs:116-160), seed 0x9E3779B97F4A7C15."""
    for n, k in [(1, 64), (3, 192), (17, 256), (64, 2048)]:
        codes, scales, act, xsum, _, _ = oracle.tern_fixture(n, k, 0x9E3779B97F4A7C15)
        got = oracle.gemv_tern_scalar(codes, scales, act, xsum)[0]
        want = oracle.gemv_tern_dequant(codes, scales, act)[0]
        assert _max_rel(got, want) < 1e-5


def test_zero_activations_are_zero_not_nan():
    """tern.rs:437-450"""
    rng = oracle.XorShift64(7)
    u = rng.u32_array(4 * 128)
    w = np.array([-1.0, 1.0, 0.0, 0.2, -0.9], np.float32)[u % 5].reshape(4, 128)
    codes, scales = oracle.pack_ternary(w)
    act, xsum, s = oracle.quantize_act(np.zeros((1, 128), np.float32))
    assert s[0] == 1.0
    out = oracle.gemv_tern_scalar(codes, scales, act, xsum)
    assert np.all(out == 0.0)


def test_packing_places_codes_in_expected_plane():
    """tern.rs:452-470"""
    w = np.zeros((1, 64), np.float32)
    w[0, 0] = 1.0
    w[0, 16] = -1.0
    w[0, 33] = 1.0
    codes, scales = oracle.pack_ternary(w)
    assert scales[0, 0] == 1.0
    assert codes[0, 0] & 3 == 2
    assert (codes[0, 0] >> 2) & 3 == 0
    assert (codes[0, 0] >> 4) & 3 == 1
    assert (codes[0, 1] >> 4) & 3 == 2


def test_quantize_act_rounds_half_away_and_clamps():
    """tern.rs:206-222: scale = 127/amax; f32::round is half-away-from-zero."""
    x = np.zeros((1, 64), np.float32)
    x[0, 0] = 127.0          # amax -> scale 1.0
    x[0, 1] = 2.5            # -> 3 (away from zero, not even)
    x[0, 2] = -2.5           # -> -3
    x[0, 3] = 0.49999997
    act, xsum, s = oracle.quantize_act(x)
    assert s[0] == 1.0
    assert list(act[0, :4]) == [127, 3, -3, 0]
    assert xsum[0, 0] == 127 + 3 - 3


# ---------------------------------------------------------------- int4

def test_f32_to_f16_rounds_half_up_not_even():
    """qwen3.js:3357-3374 increments on the first dropped bit (ties away), unlike RNE."""
    one_plus_half_ulp = np.frombuffer(np.uint32(0x3F801000).tobytes(), np.float32)[0]   # 1 + 2^-11
    assert oracle.f32_to_f16_js(one_plus_half_ulp) == 0x3C01
    assert np.float16(one_plus_half_ulp).view(np.uint16) == 0x3C00   # RNE would round to even
    assert oracle.f32_to_f16_js(1.0) == 0x3C00
    assert oracle.f32_to_f16_js(-2.0) == 0xC000
    assert oracle.f32_to_f16_js(70000.0) == 0x7C00                  # overflow -> Inf
    assert oracle.f32_to_f16_js(float("inf")) == 0x7C00
    assert oracle.f32_to_f16_js(float("nan")) == 0x7E00
    assert oracle.f32_to_f16_js(1e-8) == 0x0000                     # below half the min subnormal
    assert oracle.f32_to_f16_js(2.0 ** -24) == 0x0001               # min subnormal


def test_int4_known_answer_one_seventh():
    """Group [1, 0, 0, ...]: maxabs 1 -> scale 1/7 -> f16 0x3092 (0.142822...) ->
    inv 7.0017 -> q(1) = round(7.0017) = 7 (nibble 15), q(0) = 0 (nibble 8)."""
    w = np.zeros((1, 32), np.float32)
    w[0, 0] = 1.0
    pack, sc = oracle.quant_int4_g32(oracle.f32_to_bf16_trunc(w))
    assert sc[0, 0] == 0x3092
    assert pack[0, 0] == 0x8888888F
    assert all(pack[0, 1:] == 0x88888888)


def test_int4_known_answer_js_round_ties_up():
    """Math.round ties toward +inf: with scale bits for 1.0 (maxabs = 7), w = -2.5 -> -2 (nib 6),
    w = 2.5 -> 3 (nib 11), w = -0.5 -> -0 (nib 8), w = 0.5 -> 1 (nib 9)."""
    w = np.zeros((1, 32), np.float32)
    w[0, :5] = [7.0, -2.5, 2.5, -0.5, 0.5]
    pack, sc = oracle.quant_int4_g32(oracle.f32_to_bf16_trunc(w))
    assert sc[0, 0] == 0x3C00
    nibs = [(int(pack[0, 0]) >> (4 * i)) & 0xF for i in range(8)]
    assert nibs[:5] == [15, 6, 11, 8, 9]


def test_int4_zero_group_and_underflow():
    """All-zero group: scale 1e-8 -> f16 0 -> inv = Inf -> 0*Inf = NaN -> nibble 0.
    Tiny nonzero group: scale underflows to 0 -> +-Inf -> clamp -> 15 / 0."""
    w = np.zeros((2, 32), np.float32)
    w[1, 0] = 1e-30
    w[1, 1] = -1e-30
    pack, sc = oracle.quant_int4_g32(oracle.f32_to_bf16_trunc(w))
    assert sc[0, 0] == 0 and all(pack[0] == 0)
    assert sc[1, 0] == 0
    assert pack[1, 0] & 0xFF == 0x0F   # k0 -> 15, k1 -> 0, the zeros -> 0
    assert (int(pack[1, 0]) >> 8) == 0


@pytest.mark.parametrize("name", ["selftest_gemvQ", "selftest_gemvDP4A", "selftest_up", "normal_002", "edges"])
def test_int4_quantizer_matches_independent_restatement(golden, name):
    g = golden["int4"]
    pack, sc = oracle.quant_int4_g32(g[name + "_w"])
    np.testing.assert_array_equal(sc, g[name + "_scales"])
    np.testing.assert_array_equal(pack, g[name + "_pack"])


def test_gemvq_selftest_fixture():
    """qwen3.js:3077-3091: gemvQ N=130 K=256, x = sin(0.2i), W = cos(0.013i).
    The f64 oracle equals a plain dequant-then-dot in numpy."""
    N, K = 130, 256
    x = np.sin(np.arange(K) * 0.2).astype(np.float32)
    W = np.cos(np.arange(N * K) * 0.013).astype(np.float32).reshape(N, K)
    pack, sc = oracle.quant_int4_g32(oracle.f32_to_bf16_trunc(W))
    wdq = oracle.dequant_int4_g32(pack, sc)
    y = oracle.gemv_int4_f32act(x, pack, sc)[0]
    ref = wdq.astype(np.float64) @ x.astype(np.float64)
    np.testing.assert_allclose(y, ref, rtol=1e-12, atol=1e-12)
    # the dequantized weights stay close to the source (int4: |err| <= scale/2)
    assert np.max(np.abs(wdq - W)) < 0.08


def test_dp4a_math_within_reference_tolerance():
    """qwen3.js:3093-3106: gemvDP4A vs the f32 dequant reference, rel 2e-2."""
    N, K = 200, 320
    x = np.sin(np.arange(K) * 0.2).astype(np.float32)
    W = np.cos(np.arange(N * K) * 0.013).astype(np.float32).reshape(N, K)
    pack, sc = oracle.quant_int4_g32(oracle.f32_to_bf16_trunc(W))
    ref = oracle.gemv_int4_f32act(x, pack, sc)[0]
    xq, xs, _ = oracle.quant_q8(x)
    got = oracle.gemv_int4_q8act(xq, xs, pack, sc)[0]
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) < 2e-2


def test_quant_q8_round_half_even_and_sums():
    """QUANTQ8 (qwen3.js:332-358): WGSL round() is half-to-even."""
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = 127.0   # scale 1, inv 1
    x[0, 1] = 2.5     # -> 2
    x[0, 2] = 3.5     # -> 4
    x[0, 3] = -2.5    # -> -2
    x[0, 20] = 5.0
    xq, xs, xsum = oracle.quant_q8(x)
    assert xs[0, 0] == 1.0
    assert list(xq[0, :4]) == [127, 2, 4, -2]
    assert xsum[0, 0] == 127 + 2 + 4 - 2 and xsum[0, 1] == 5


def test_rmsnorm_q8_is_rmsnorm_then_quant():
    rng = np.random.default_rng(5)
    H = 256
    x = rng.normal(0, 1, (2, H)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, H)).view(np.uint16)
    xq, xs, xsum, inv = oracle.rmsnorm_q8(x, w16, 1e-6)
    normed = (x * inv[:, None]) * w16.view(np.float16).astype(np.float32)
    xq2, xs2, xsum2 = oracle.quant_q8(normed)
    np.testing.assert_array_equal(xq, xq2)
    np.testing.assert_array_equal(xs, xs2)
    np.testing.assert_array_equal(xsum, xsum2)


def test_gateup_selftest_fixture():
    """qwen3.js:3143-3157: gateUpSiluQ I=130 H=256 vs the f32 dequant reference, rel 3e-2."""
    I, H = 130, 256
    x = np.sin(np.arange(H) * 0.2).astype(np.float32)
    gf = np.cos(np.arange(I * H) * 0.013).astype(np.float32).reshape(I, H)
    uf = np.sin(np.arange(I * H) * 0.009).astype(np.float32).reshape(I, H)
    gp, gs = oracle.quant_int4_g32(oracle.f32_to_bf16_trunc(gf))
    up, us = oracle.quant_int4_g32(oracle.f32_to_bf16_trunc(uf))
    g = oracle.gemv_int4_f32act(x, gp, gs)[0]
    u = oracle.gemv_int4_f32act(x, up, us)[0]
    ref = g / (1 + np.exp(-g)) * u
    xq, xs, _ = oracle.quant_q8(x)
    got = oracle.gateup_q8act(xq, xs, gp, gs, up, us)[0]
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) < 3e-2


# ---------------------------------------------------------------- attention

def _split_kv_numpy(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit):
    """Independent restatement with the split / online-softmax / combine
    structure of qwen3.js:2077-2164 + 2048-2069 (128-key tiles)."""
    grp = nHq // nKv
    kd = np.maximum(Kq.astype(np.float64) / 127.0, -1.0) * np.repeat(Ks, 32, axis=1)
    vd = np.maximum(Vq.astype(np.float64) / 127.0, -1.0) * np.repeat(Vs, 32, axis=1)
    out = np.zeros(nHq * hd)
    per = -(-S // nsplit)
    for hq in range(nHq):
        hk = hq // grp
        parts = []
        for sp in range(nsplit):
            c0, c1 = sp * per, min(S, sp * per + per)
            m, l, o = -3e38, 0.0, np.zeros(hd)
            for k0 in range(c0, c1, 128):
                ks = range(k0, min(c1, k0 + 128))
                s = np.array([q[hq * hd:(hq + 1) * hd] @ kd[t, hk * hd:(hk + 1) * hd] for t in ks]) / np.sqrt(hd)
                mn = max(m, s.max())
                corr = np.exp(m - mn)
                p = np.exp(s - mn)
                l = l * corr + p.sum()
                o = o * corr + sum(p[i] * vd[t, hk * hd:(hk + 1) * hd] for i, t in enumerate(ks))
                m = mn
            parts.append((m, l, o))
        M = max(p[0] for p in parts)
        L = sum(p[1] * np.exp(p[0] - M) for p in parts)
        out[hq * hd:(hq + 1) * hd] = sum(p[2] * np.exp(p[0] - M) for p in parts) / L
    return out


def test_attention_oracle_equals_split_kv_structure():
    rng = np.random.default_rng(11)
    nHq, nKv, hd, S = 4, 2, 64, 300
    K = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    V = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    Kq, Ks = oracle.kv_quant_q8(K)
    Vq, Vs = oracle.kv_quant_q8(V)
    Ks = Ks.reshape(S, -1)
    Vs = Vs.reshape(S, -1)
    q = rng.normal(0, 1, nHq * hd).astype(np.float32)
    got = oracle.attn_decode_q8(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd)
    for nsplit in (1, 3, 16):   # 16 splits of 19 keys: uneven, some splits shorter
        ref = _split_kv_numpy(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit)
        np.testing.assert_allclose(got, ref, rtol=1e-9, atol=1e-12)


def test_kv_snorm_round_trip():
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 4096).astype(np.float32)
    q, s = oracle.kv_quant_q8(x)
    deq = np.maximum(q.astype(np.float32) / 127, -1) * np.repeat(s, 32)
    assert np.all(np.abs(deq - x) <= np.repeat(s, 32) / 254 + 1e-6)
    assert q.min() >= -127


def test_dec_nsplit_rule():
    """_decNsplit, qwen3.js:2354."""
    import math
    for S in [1, 100, 128, 129, 512, 1024, 1792, 4096, 7168, 32768]:
        want = max(1, min(16, math.ceil(S / 128), max(4, math.ceil(S / 448))))
        assert oracle.dec_nsplit(S) == want


def test_argmax_lowest_index_on_ties():
    x = np.array([1.0, 5.0, 3.0, 5.0], np.float32)
    assert oracle.argmax(x) == 1


# ---- ternary, WebGPU layout (quantizeTernaryBf16, models/qwen3.js:3435-3469) ----
# The reference holds no fixtures for this path and no JavaScript runtime is
# available to run it, so the restatement is pinned by properties its comments
# state (lossless, the dot4 lane layout, the 2-ulp tolerance) and by decoding to
# the same matrix as the Q2_0_g64 packer, which is pinned on tern.rs's fixtures.

from helpers import tern_bf16, tern_wgsl_codes  # noqa: E402


def _bf16_val(bits):
    return oracle.bf16_to_f32(bits).astype(np.float64)


def test_tern_wgsl_pack_is_lossless():
    rng = np.random.default_rng(1)
    w = tern_bf16(rng, 16, 256)
    pack, sc = oracle.quant_tern_wgsl(w)
    dq = (tern_wgsl_codes(pack, 256) - 1) * np.repeat(oracle.f16_bits_to_f64(sc), 32, axis=1)
    np.testing.assert_array_equal(dq, _bf16_val(w))


def test_tern_wgsl_dot4_lane_layout():
    """(word >> 2s) & 0x03030303 holds the codes of k = 16w+4s .. 16w+4s+3 in byte lanes."""
    rng = np.random.default_rng(2)
    w = tern_bf16(rng, 2, 128)
    pack, _ = oracle.quant_tern_wgsl(w)
    codes = tern_wgsl_codes(pack, 128)
    for wi in range(8):
        for s in range(4):
            v = (int(pack[0, wi]) >> (2 * s)) & 0x03030303
            lanes = [(v >> (8 * b)) & 0xFF for b in range(4)]
            assert lanes == list(codes[0, 16 * wi + 4 * s: 16 * wi + 4 * s + 4])


def test_tern_wgsl_matches_q2g64_decode():
    """The same ternary matrix packed in both layouts decodes to the same weights."""
    rng = np.random.default_rng(3)
    N, K = 8, 512
    s = (rng.uniform(0.01, 0.05, (N, K // 64)).astype(np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)
    t = rng.integers(-1, 2, (N, K)).astype(np.float32)
    w = t * np.repeat(s, 64, axis=1)
    codes, sc64 = oracle.pack_ternary(w)
    pack, sc = oracle.quant_tern_wgsl(oracle.f32_to_bf16_trunc(w))
    # Q2_0_g64: code j of a 64-group in byte j % 16 at bit 2 * (j // 16)
    j = np.arange(K) % 64
    byte = (np.arange(K) // 64) * 16 + (j % 16)
    c64 = (codes[:, byte] >> (2 * (j // 16))) & 3
    dq64 = (c64.astype(np.float64) - 1) * np.repeat(sc64.astype(np.float64), 64, axis=1)
    dqw = (tern_wgsl_codes(pack, K) - 1) * np.repeat(oracle.f16_bits_to_f64(sc), 32, axis=1)
    np.testing.assert_array_equal(dqw, dq64)


def test_tern_wgsl_tolerance_zero_groups_and_rejections():
    rng = np.random.default_rng(4)
    w = tern_bf16(rng, 6, 128, wobble=0.3, negzero=0.5)
    pack, sc = oracle.quant_tern_wgsl(w)
    mag = w & 0x7FFF
    sign = (w >> 15) & 1
    exp_codes = np.where(mag == 0, 1, np.where(sign == 1, 0, 2))
    np.testing.assert_array_equal(tern_wgsl_codes(pack, 128), exp_codes)   # wobble snaps to +-1, -0 is 0
    z = w.copy()
    z[0, 32:64] = 0
    pz, sz = oracle.quant_tern_wgsl(z)
    assert sz[0, 1] == 0 and np.all(pz[0, 2:4] == 0x55555555)
    bad = w.copy()
    g = bad[5, 96:128]
    i = int(np.flatnonzero(g & 0x7FFF)[0])
    bad[5, 96 + i] = (int(np.max(g & 0x7FFF)) - 3) | (int(g[i]) & 0x8000)   # 3 ulps below: not ternary
    assert oracle.quant_tern_wgsl(bad) is None
    assert oracle.quant_tern_wgsl(w[:, :96]) is None                        # K % 64 != 0
    assert oracle.quant_tern_wgsl(oracle.f32_to_bf16_trunc(rng.normal(0, 0.02, (4, 64)).astype(np.float32))) is None


def test_tern_wgsl_scale_is_bf16_to_f16_half_up():
    """scale = bf16ToF16bits(group max) (qwen3.js:3386-3390)."""
    rng = np.random.default_rng(5)
    w = tern_bf16(rng, 4, 64)
    _, sc = oracle.quant_tern_wgsl(w)
    mx = np.max(w.reshape(4, 2, 32) & 0x7FFF, axis=2)
    vals = oracle.bf16_to_f32(mx.astype(np.uint16)).ravel()
    exp = np.array([oracle.f32_to_f16_js(float(v)) for v in vals], np.uint16).reshape(mx.shape)
    np.testing.assert_array_equal(sc, exp)


def test_tern_wgsl_gemv_oracle_is_dequant_dot():
    rng = np.random.default_rng(6)
    w = tern_bf16(rng, 40, 256)
    pack, sc = oracle.quant_tern_wgsl(w)
    xq, xs, _ = oracle.quant_q8(rng.normal(0, 1, (3, 256)).astype(np.float32))
    y = oracle.gemv_tern_wgsl_q8act(xq, xs, pack, sc)
    xd = xq.astype(np.float64) * np.repeat(xs.astype(np.float64), 32, axis=1)
    ref = xd @ _bf16_val(w).T
    # the only rounding is the f32 product f32(s) * xs of each group (~6e-8)
    np.testing.assert_allclose(y, ref, rtol=0, atol=1e-6 * np.max(np.abs(ref)))


def _np_quantize_wasm(x):
    """numpy restatement of cpu/kernel/src/lib.rs:566-606 in f32 arithmetic"""
    x = np.asarray(x, np.float32)
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0)
    asc = np.float32(amax / np.float32(127.0)) if amax > 0 else np.float32(1e-9)
    inv = np.float32(np.float32(1.0) / asc)
    q = np.clip(np.rint((x * inv).astype(np.float32)), -127, 127).astype(np.int8)
    return q, q.reshape(-1, 64).astype(np.int32).sum(1), asc


def test_quantize_wasm_oracle_matches_restatement():
    rng = np.random.default_rng(5)
    rows = [rng.normal(0, 1, 2048), np.zeros(128), rng.normal(0, 3, 6144)]
    r = np.zeros(64, np.float32)
    r[:4] = [127.0, 0.5, -0.5, 1.5]          # x * (1/asc) lands exactly on .5 ties: nearest-even
    rows.append(r)
    for x in rows:
        x = np.asarray(x, np.float32)
        act, xsum, asc = oracle.quantize_act_wasm(x)
        q, s, a = _np_quantize_wasm(x)
        np.testing.assert_array_equal(act[0], q)
        np.testing.assert_array_equal(xsum[0], s)
        assert asc[0] == a
    act, _, asc = oracle.quantize_act_wasm(rows[-1])
    assert asc[0] == 1.0 and list(act[0][:4]) == [127, 0, 0, 2]    # ties to even, unlike tern.rs
    _, _, asc0 = oracle.quantize_act_wasm(np.zeros(64, np.float32))
    assert asc0[0] == np.float32(1e-9)


def test_quant_int3_oracle_matches_restatement():
    """bf16 -> int3 (group 32 / 128): scale = engine f16(max|w|/4), q = clamp(rn(w/scale), -4, 3)."""
    rng = np.random.default_rng(8)
    w = (rng.normal(0, 0.02, (6, 256)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    w[0, :128] = 0
    for group in (32, 128):
        p3, s3 = oracle.quant_int3(w, group)
        wf = (w.astype(np.uint32) << 16).view(np.float32).reshape(6, -1, group)
        for r in range(6):
            for gi in range(256 // group):
                m = np.float32(np.max(np.abs(wf[r, gi])))
                sh = oracle.engine_f32_to_f16(float(np.float32(m / np.float32(4.0))))
                assert s3[r, gi] == sh
                sc = np.float32(oracle.f16_to_f64(int(sh)))
                q = np.zeros(group, np.int64) if sc == 0 else np.clip(np.rint(wf[r, gi] / sc), -4, 3).astype(np.int64)
                st = (q + 4).reshape(-1, 32)
                for j in range(group // 32):
                    for p in range(3):
                        want = int(sum(((int(st[j, i]) >> p) & 1) << i for i in range(32)))
                        assert int(p3[r, gi * (group // 32) + j, p]) == want
