"""GPU parity: ternary Q2_0_g64 path (native/crates/n2-kernels/src/tern.rs).

Bars: codes/scales bit-exact with the reference's numpy packer (golden);
activations/xsum bit-exact with quantize_act; GEMV output BIT-EXACT with
gemv_tern_scalar (tern.rs:79-119), and within the reference's own 1e-5
relative bar of the dequant oracle and the AVX2 backend."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import host

pytestmark = pytest.mark.gpu

FIXTURES = [("tern_rs_oracle", 0x2026_0805, [(1, 64), (3, 128), (17, 256), (8, 1024)]),
            ("tern_rs_avx2", 0xC0FFEE, [(1, 64), (1, 192), (5, 192), (17, 256), (64, 2048)])]


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("T,K", [(1, 64), (1, 2048), (4, 6144), (3, 128)])
def test_quantize_wasm_bit_exact(cuda, T, K):
    """WASM quantize (cpu/kernel/src/lib.rs:566-606): asc = amax/127, nearest-even,
    asc returned; a zero row gives asc 1e-9 and zero codes."""
    rng = np.random.default_rng(K + 7 * T)
    x = rng.normal(0, 1, (T, K)).astype(np.float32)
    if T > 1:
        x[1] = 0.0
    x[0, :4] = [x[0].max() / 127 * 0.5, -x[0].max() / 127 * 1.5, 0.0, x[0].max()]
    dst, xsum, asc = tb.quantize_wasm(_dev(x))
    oa, ox, oasc = oracle.quantize_act_wasm(x)
    np.testing.assert_array_equal(host(dst), oa)
    np.testing.assert_array_equal(host(xsum), ox)
    np.testing.assert_array_equal(host(asc), oasc)


@pytest.mark.parametrize("tag,base,dims", FIXTURES)
def test_pack_bit_exact_with_reference_packer(cuda, golden, tag, base, dims):
    for n, k in dims:
        _, _, _, _, w, _ = oracle.tern_fixture(n, k, base + k)
        codes, scales = tb.pack_ternary(_dev(w))
        np.testing.assert_array_equal(host(codes), golden["tern"][f"{tag}_{n}x{k}_codes"])
        np.testing.assert_array_equal(host(scales), golden["tern"][f"{tag}_{n}x{k}_scales"])


def test_pack_config1_bit_exact(cuda, golden):
    codes, scales = tb.pack_ternary(_dev(golden["tern"]["config1_w"]))
    np.testing.assert_array_equal(host(codes), golden["tern"]["config1_codes"])
    np.testing.assert_array_equal(host(scales), golden["tern"]["config1_scales"])


@pytest.mark.parametrize("T,K", [(1, 64), (1, 2048), (4, 6144), (8, 2048)])
def test_quantize_act_bit_exact(cuda, T, K):
    rng = np.random.default_rng(K + T)
    x = rng.normal(0, 1, (T, K)).astype(np.float32)
    x[0, 5] = 0.5 * x[0].max() / 127 * 127   # exercise ties under the row scale
    act, xsum, sc = tb.quantize_act(_dev(x))
    oa, ox, os_ = oracle.quantize_act(x)
    np.testing.assert_array_equal(host(act), oa)
    np.testing.assert_array_equal(host(xsum), ox)
    np.testing.assert_array_equal(host(sc), os_)


@pytest.mark.parametrize("tag,base,dims", FIXTURES)
def test_gemv_bit_exact_on_tern_rs_fixtures(cuda, tag, base, dims):
    for n, k in dims:
        codes, scales, act, xsum, _, _ = oracle.tern_fixture(n, k, base + k)
        out = tb.gemv_tern(_dev(codes), _dev(scales), _dev(act[None]), _dev(xsum[None]))
        want = oracle.gemv_tern_scalar(codes, scales, act, xsum)
        np.testing.assert_array_equal(host(out), want)
        deq = oracle.gemv_tern_dequant(codes, scales, act)
        rel = np.max(np.abs(host(out) - deq) / np.maximum(np.maximum(np.abs(host(out)), np.abs(deq)), 1e-3))
        assert rel < 1e-5
        avx = oracle.gemv_tern_avx2(codes, scales, act, xsum)
        rel = np.max(np.abs(host(out)[0] - avx) / np.maximum(np.maximum(np.abs(avx), np.abs(host(out)[0])), 1e-3))
        assert rel < 1e-5


CONFIG1 = [("qkv", 4096, 2048), ("o", 2048, 2048), ("gate", 6144, 2048), ("down", 2048, 6144)]


def _config1_weights(seed, N, K):
    """Config 1: codes uniform over {-1,0,+1}, scales U(0.01,0.05) rounded to f16."""
    rng = np.random.default_rng(seed)
    c = rng.integers(0, 3, (N, K), dtype=np.int8).astype(np.float32) - 1.0
    s = rng.uniform(0.01, 0.05, (N, K // 64)).astype(np.float16).astype(np.float32)
    return c * np.repeat(s, 64, axis=1)


@pytest.mark.parametrize("B", [1, 2, 4, 8])
@pytest.mark.parametrize("tag,N,K", CONFIG1)
def test_gemv_bit_exact_config1(cuda, tag, N, K, B):
    w = _config1_weights(N + K, N, K)
    codes, scales = tb.pack_ternary(_dev(w))
    oc, os_ = oracle.pack_ternary(w)
    np.testing.assert_array_equal(host(codes), oc)
    np.testing.assert_array_equal(host(scales), os_)
    rng = np.random.default_rng(B)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    act, xsum, _ = oracle.quantize_act(x)
    out = tb.gemv_tern(codes, scales, _dev(act), _dev(xsum))
    np.testing.assert_array_equal(host(out), oracle.gemv_tern_scalar(oc, os_, act, xsum))


def test_zero_activations_give_zero(cuda):
    rng = oracle.XorShift64(7)
    u = rng.u32_array(4 * 128)
    w = np.array([-1.0, 1.0, 0.0, 0.2, -0.9], np.float32)[u % 5].reshape(4, 128)
    codes, scales = tb.pack_ternary(_dev(w))
    act, xsum, sc = tb.quantize_act(torch.zeros(1, 128, device="cuda"))
    assert host(sc)[0] == 1.0
    out = host(tb.gemv_tern(codes, scales, act, xsum))
    assert np.all(out == 0.0) and not np.any(np.isnan(out))


@pytest.mark.parametrize("T", [1, 3])
def test_linear_tern_matches_model_linear(cuda, T):
    """Model::linear (model.rs:316-339): out = gemv(quantize(x)) * (1/scale), bit-exact."""
    N, K = 2048, 6144
    w = _config1_weights(3, N, K)
    oc, os_ = oracle.pack_ternary(w)
    x = np.random.default_rng(4).normal(0, 1, (T, K)).astype(np.float32)
    y = host(tb.linear_tern(_dev(x), _dev(oc), _dev(os_)))
    act, xsum, sc = oracle.quantize_act(x)
    raw = oracle.gemv_tern_scalar(oc, os_, act, xsum)
    want = raw * (np.float32(1.0) / sc)[:, None]
    np.testing.assert_array_equal(y, want.astype(np.float32))


def test_bad_k_raises(cuda):
    with pytest.raises(tb.TabInferError):
        tb.pack_ternary(torch.zeros(4, 96, device="cuda"))


def _random_q2g64(seed, N, K):
    """valid Q2_0_g64 codes (every 2-bit field in {0,1,2}) and f32 scales, made
    directly (no f32 weight matrix), for large shapes"""
    import itertools
    rng = np.random.default_rng(seed)
    lut = np.array([a | (b << 2) | (c << 4) | (d << 6) for a, b, c, d in itertools.product(range(3), repeat=4)],
                   np.uint8)
    codes = lut[rng.integers(0, 81, (N, K // 4), dtype=np.uint8)]
    scales = np.float16(rng.uniform(0.01, 0.05, (N, K // 64))).astype(np.float32)
    return codes, scales


# Shapes that make the streaming GEMV wrap its stage ring many times (tens of
# tiles per CTA), odd tails whose scales cannot travel by bulk copy, every
# batch its register path takes (1..4) and the largest K it keeps in registers.
@pytest.mark.parametrize("N,K,B", [(60000, 2048, 1), (30000, 6144, 1), (13, 64, 3), (7, 128, 2), (1000, 4096, 2),
                                   (777, 8192, 1), (20000, 2048, 4), (5003, 1024, 3), (9001, 8256, 1)])
def test_gemv_bit_exact_streaming_shapes(cuda, N, K, B):
    codes, scales = _random_q2g64(N + K + B, N, K)
    x = np.random.default_rng(B + 11).normal(0, 1, (B, K)).astype(np.float32)
    act, xsum, _ = oracle.quantize_act(x)
    out = host(tb.gemv_tern(_dev(codes), _dev(scales), _dev(act), _dev(xsum)))
    np.testing.assert_array_equal(out, oracle.gemv_tern_scalar(codes, scales, act, xsum))
