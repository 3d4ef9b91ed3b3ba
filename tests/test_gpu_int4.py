"""GPU parity: int4 G=32 path vs the oracle (models/qwen3.js math).

Bars: bit-exact for packs, scales and int8 activations; per-row relative error
<= 1e-3 (|err| / max(|ref|, 1e-3*rms)) for the GEMV outputs against the f64
oracle in the matching numerics mode (f32-activation gemvQ, int8-activation
gemvDP4A)."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import bf16_normal, host, row_rel_err, u16_dev, u32_dev

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _quant(cuda, wbits):
    pack, sc = tb.quantize_int4_bf16(u16_dev(wbits))
    torch.cuda.synchronize()
    return host(pack, np.uint32), host(sc, np.uint16), pack, sc


@pytest.mark.parametrize("name", ["selftest_gemvQ", "selftest_gemvDP4A", "selftest_up", "normal_002", "edges"])
def test_quantizer_bit_exact_on_golden(cuda, golden, name):
    g = golden["int4"]
    p, s, _, _ = _quant(cuda, g[name + "_w"])
    np.testing.assert_array_equal(s, g[name + "_scales"])
    np.testing.assert_array_equal(p, g[name + "_pack"])


@pytest.mark.parametrize("N,K", [(1024, 1024), (3072, 1024), (1024, 3072), (257, 2048)])
def test_quantizer_bit_exact_random(cuda, N, K):
    rng = np.random.default_rng(N * 7 + K)
    w = bf16_normal(rng, (N, K), 0.02)
    w[0, :32] = 0                      # zero group
    w[1, :64] = w[1, :64] & 0x807F     # tiny magnitudes (scale underflow / subnormal paths)
    p, s, _, _ = _quant(cuda, w)
    op, os_ = oracle.quant_int4_g32(w)
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(p, op)


@pytest.mark.parametrize("T,K", [(1, 32), (1, 1024), (4, 3072), (8, 2048), (3, 6144)])
def test_quant_q8_bit_exact(cuda, T, K):
    rng = np.random.default_rng(T * 100 + K)
    x = rng.normal(0, 1, (T, K)).astype(np.float32)
    x[0, :32] = 0.0                    # all-zero group -> scale 0, inv 0
    xq, xs, xsum = tb.quant_q8(torch.from_numpy(x).cuda())
    oq, os_, osum = oracle.quant_q8(x)
    np.testing.assert_array_equal(host(xq), oq)
    np.testing.assert_array_equal(host(xs), os_)
    np.testing.assert_array_equal(host(xsum), osum)


@pytest.mark.parametrize("T,H", [(1, 1024), (1, 2048), (8, 2048)])
def test_rmsnorm_q8(cuda, T, H):
    rng = np.random.default_rng(H + T)
    x = rng.normal(0, 3, (T, H)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, H)).view(np.uint16)
    xq, xs, xsum = tb.rmsnorm_q8(torch.from_numpy(x).cuda(), u16_dev(w16), 1e-6)
    oq, os_, osum, inv = oracle.rmsnorm_q8(x, w16, 1e-6)
    np.testing.assert_allclose(host(xs), os_, rtol=2e-6)
    d = np.abs(host(xq).astype(int) - oq.astype(int))
    assert d.max() <= 1
    # any 1-LSB difference must sit on a rounding tie of the oracle's value
    if d.max() == 1:
        normed = (x * inv[:, None]) * w16.view(np.float16).astype(np.float32)
        v = normed / np.repeat(os_, 32, axis=1)
        frac = np.abs(np.abs(v - np.floor(v)) - 0.5)
        assert np.all(frac[d == 1] < 1e-3)


SHAPES_06B = [("q", 2048, 1024), ("kv", 1024, 1024), ("o", 1024, 2048), ("gate", 3072, 1024),
              ("down", 1024, 3072), ("odd", 130, 256), ("dp4a_fixture", 200, 320), ("k6144", 96, 6144),
              ("tail", 4099, 1024)]


def _mat(seed, N, K):
    rng = np.random.default_rng(seed)
    w = bf16_normal(rng, (N, K), 0.02)
    pack, sc = oracle.quant_int4_g32(w)
    return pack, sc


@pytest.mark.parametrize("B", [1, 2, 4, 8])
@pytest.mark.parametrize("tag,N,K", SHAPES_06B)
def test_gemv_dp4(cuda, tag, N, K, B):
    pack, sc = _mat(N + K, N, K)
    rng = np.random.default_rng(B)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    xq, xs, _ = oracle.quant_q8(x)
    y = tb.gemv_dp4(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc))
    ref = oracle.gemv_int4_q8act(xq, xs, pack, sc)
    assert row_rel_err(host(y), ref) < TOL


@pytest.mark.parametrize("B", [1, 3, 8])
@pytest.mark.parametrize("tag,N,K", SHAPES_06B)
def test_gemv_q_f32(cuda, tag, N, K, B):
    pack, sc = _mat(N * 3 + K, N, K)
    rng = np.random.default_rng(B + 10)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    y = tb.gemv_q(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc))
    ref = oracle.gemv_int4_f32act(x, pack, sc)
    assert row_rel_err(host(y), ref) < TOL


def test_gemv_selftest_fixtures(cuda):
    """qwen3.js:3077-3106 fixtures through the GPU, against the JS CPU reference math."""
    N, K = 130, 256
    x = np.sin(np.arange(K) * 0.2).astype(np.float32)
    W = np.cos(np.arange(N * K) * 0.013).astype(np.float32).reshape(N, K)
    wb = oracle.f32_to_bf16_trunc(W)
    _, _, pack, sc = _quant(cuda, wb)
    y = host(tb.gemv_q(torch.from_numpy(x).cuda(), pack, sc))[0]
    ref = oracle.gemv_int4_f32act(x, host(pack, np.uint32), host(sc, np.uint16))[0]
    assert np.max(np.abs(y - ref)) < 1e-2 and row_rel_err(y, ref) < TOL
    N, K = 200, 320
    x = np.sin(np.arange(K) * 0.2).astype(np.float32)
    W = np.cos(np.arange(N * K) * 0.013).astype(np.float32).reshape(N, K)
    _, _, pack, sc = _quant(cuda, oracle.f32_to_bf16_trunc(W))
    y = host(tb.linear_q(torch.from_numpy(x[None]).cuda(), pack, sc))[0]
    ref = oracle.gemv_int4_f32act(x, host(pack, np.uint32), host(sc, np.uint16))[0]
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 2e-2


def test_gemv_acc_adds_residual(cuda):
    pack, sc = _mat(5, 1024, 2048)
    rng = np.random.default_rng(6)
    x = rng.normal(0, 1, (1, 2048)).astype(np.float32)
    r = rng.normal(0, 1, (1, 1024)).astype(np.float32)
    xq, xs, _ = oracle.quant_q8(x)
    y = torch.from_numpy(r.copy()).cuda()
    tb.gemv_dp4(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc), y=y, acc=True)
    ref = oracle.gemv_int4_q8act(xq, xs, pack, sc) + r
    assert row_rel_err(host(y), ref) < TOL
    y2 = torch.from_numpy(r.copy()).cuda()
    tb.gemv_q(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc), y=y2, acc=True)
    ref2 = oracle.gemv_int4_f32act(x, pack, sc) + r
    assert row_rel_err(host(y2), ref2) < TOL


@pytest.mark.parametrize("B", [1, 4])
def test_multi_matrix_launch_equals_separate(cuda, B):
    mats = [_mat(i, n, 1024) for i, n in enumerate([2048, 1024, 1024])]
    rng = np.random.default_rng(9)
    x = rng.normal(0, 1, (B, 1024)).astype(np.float32)
    xq, xs, _ = oracle.quant_q8(x)
    ys = tb.gemv_dp4_multi(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(),
                           [(u32_dev(p), u16_dev(s)) for p, s in mats])
    for (p, s), y in zip(mats, ys):
        assert row_rel_err(host(y), oracle.gemv_int4_q8act(xq, xs, p, s)) < TOL


@pytest.mark.parametrize("B", [1, 2, 8])
@pytest.mark.parametrize("I,H", [(3072, 1024), (130, 256), (6144, 2048)])
def test_gateup_silu(cuda, I, H, B):
    gp, gs = _mat(I, I, H)
    up, us = _mat(I + 1, I, H)
    rng = np.random.default_rng(B + I)
    x = rng.normal(0, 1, (B, H)).astype(np.float32)
    xq, xs, _ = oracle.quant_q8(x)
    swi = tb.gate_up_silu_dp4(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(gp), u16_dev(gs),
                              u32_dev(up), u16_dev(us))
    ref = oracle.gateup_q8act(xq, xs, gp, gs, up, us)
    assert row_rel_err(host(swi), ref) < TOL


@pytest.mark.parametrize("B", [1, 4, 8])
@pytest.mark.parametrize("K", [1024, 2048, 3072, 6144])
def test_fused_rmsnorm_quant_gemv(cuda, K, B):
    """rmsnormQ + projGemv fused: the in-kernel int8 rows equal tb_rmsnorm_q8's, and the
    outputs match the oracle on those rows (one launch vs two)."""
    N = 1000
    pack, sc = _mat(K + B, N, K)
    rng = np.random.default_rng(K * B)
    x = rng.normal(0, 2, (B, K)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, K)).view(np.uint16)
    xd, wd = torch.from_numpy(x).cuda(), u16_dev(w16)
    xq, xs, _ = tb.rmsnorm_q8(xd, wd, 1e-6)
    y_fused = tb.gemv_dp4a(xd, u32_dev(pack), u16_dev(sc), norm_w=wd, eps=1e-6)
    y_sep = tb.gemv_dp4(xq, xs, u32_dev(pack), u16_dev(sc))
    np.testing.assert_array_equal(host(y_fused), host(y_sep))
    ref = oracle.gemv_int4_q8act(host(xq), host(xs), pack, sc)
    assert row_rel_err(host(y_fused), ref) < TOL
    # plain quantQ8 prologue (gemvDP4A)
    y2 = tb.gemv_dp4a(xd, u32_dev(pack), u16_dev(sc))
    oq, os_, _ = oracle.quant_q8(x)
    assert row_rel_err(host(y2), oracle.gemv_int4_q8act(oq, os_, pack, sc)) < TOL


@pytest.mark.parametrize("B", [1, 2])
def test_fused_multi_and_gateup(cuda, B):
    H = 2048
    mats = [_mat(10 + i, n, H) for i, n in enumerate([2048, 1024, 1024])]
    gp, gs = _mat(20, 6144, H)
    up, us = _mat(21, 6144, H)
    rng = np.random.default_rng(B)
    x = rng.normal(0, 1, (B, H)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, H)).view(np.uint16)
    xd, wd = torch.from_numpy(x).cuda(), u16_dev(w16)
    xq, xs, _ = tb.rmsnorm_q8(xd, wd, 1e-6)
    ys = tb.gemv_dp4a_multi(xd, [(u32_dev(p), u16_dev(s)) for p, s in mats], norm_w=wd)
    for (p, s), y in zip(mats, ys):
        assert row_rel_err(host(y), oracle.gemv_int4_q8act(host(xq), host(xs), p, s)) < TOL
    swi = tb.gate_up_silu_dp4a(xd, u32_dev(gp), u16_dev(gs), u32_dev(up), u16_dev(us), norm_w=wd)
    ref = oracle.gateup_q8act(host(xq), host(xs), gp, gs, up, us)
    assert row_rel_err(host(swi), ref) < TOL


@pytest.mark.parametrize("B", [1, 8])
def test_fused_norm_lm_head(cuda, B):
    """final rmsnorm + gemvQ lm_head in one launch == tb_rmsnorm then gemvQ."""
    N, K = 20000, 2048
    pack, sc = _mat(33, N, K)
    rng = np.random.default_rng(3)
    x = rng.normal(0, 3, (B, K)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, K)).view(np.uint16)
    xd, wd = torch.from_numpy(x).cuda(), u16_dev(w16)
    normed = tb.rmsnorm(xd, wd, 1e-6)
    y_sep = tb.gemv_q(normed, u32_dev(pack), u16_dev(sc))
    y_fused = tb.gemv_q_norm(xd, wd, 1e-6, u32_dev(pack), u16_dev(sc))
    np.testing.assert_array_equal(host(y_fused), host(y_sep))
    assert row_rel_err(host(y_fused), oracle.gemv_int4_f32act(host(normed), pack, sc)) < TOL


@pytest.mark.parametrize("T,N", [(1, 1024), (1, 20000), (4, 3072), (8, 1024), (12, 1024), (16, 4096), (5, 1001)])
def test_linear_router(cuda, T, N):
    """linearQ routing (qwen3.js:1597-1608): T=1 N<16384 int8; T=1 N>=16384 f32; T>1 per-token
    int8 (the tensor-core GEMV at 2..16 rows, the dp4a GEMV where the rows are not a multiple of 8)."""
    K = 1024
    pack, sc = _mat(T + N, N, K)
    rng = np.random.default_rng(T)
    x = rng.normal(0, 1, (T, K)).astype(np.float32)
    y = host(tb.linear_q(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc)))
    if T == 1 and N >= 16384:
        ref = oracle.gemv_int4_f32act(x, pack, sc)
    else:
        xq, xs, _ = oracle.quant_q8(x)
        ref = oracle.gemv_int4_q8act(xq, xs, pack, sc)
    assert row_rel_err(y, ref) < TOL


def test_lm_head_full_size_sampled_rows_and_linearity(cuda):
    """Config-2 tied lm_head 151936 x 1024 at full size: a seeded sample of rows
    against the oracle, plus linearity of the f32-activation GEMV."""
    N, K = 151936, 1024
    g = torch.Generator(device="cuda").manual_seed(1)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    pack, sc = tb.quantize_int4_bf16(w.view(torch.int16))
    x1 = torch.randn(1, K, device="cuda", generator=g)
    x2 = torch.randn(1, K, device="cuda", generator=g)
    y1 = tb.gemv_q(x1, pack, sc)
    y2 = tb.gemv_q(x2, pack, sc)
    y12 = tb.gemv_q(x1 + x2, pack, sc)
    assert row_rel_err(host(y12), host(y1) + host(y2)) < 1e-3
    rows = np.random.default_rng(2).choice(N, 512, replace=False)
    rows.sort()
    rt = torch.from_numpy(rows).cuda()
    p_s = host(pack[rt], np.uint32)
    s_s = host(sc[rt], np.uint16)
    ref = oracle.gemv_int4_f32act(host(x1), p_s, s_s)[0]
    assert row_rel_err(host(y1)[0, rows], ref) < TOL
    # the packed sample is what the oracle quantizer makes of the same bf16 rows
    wp, ws = oracle.quant_int4_g32(host(w[rt].view(torch.int16), np.uint16))
    np.testing.assert_array_equal(wp, p_s)
    np.testing.assert_array_equal(ws, s_s)


def test_stream_ordering_with_torch(cuda):
    """The library's kernels run on torch's current stream: a torch upload, the
    GEMV and a torch readback issued back to back (no explicit sync) always see
    each other's results, on the default stream and on a side stream."""
    pack, sc = _mat(77, 20000, 2048)
    x = np.random.default_rng(1).normal(0, 1, (8, 2048)).astype(np.float32)
    ref = oracle.gemv_int4_f32act(x, pack, sc)
    for stream in (None, torch.cuda.Stream()):
        ctx_mgr = torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream())
        with ctx_mgr:
            for _ in range(6):
                y = tb.gemv_q(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc))
                assert row_rel_err(host(y), ref) < TOL


def test_bad_shapes_raise(cuda):
    pack, sc = _mat(1, 64, 64)
    x = torch.zeros(1, 48, device="cuda")
    with pytest.raises(tb.TabInferError):
        tb.gemv_q(x, u32_dev(pack), u16_dev(sc))
    with pytest.raises(tb.TabInferError):
        tb.linear_q(torch.zeros(9, 64, device="cuda"), u32_dev(pack), u16_dev(sc))
