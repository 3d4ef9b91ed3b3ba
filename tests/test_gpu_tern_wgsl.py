"""Ternary weights in the WebGPU layout of models/qwen3.js: the lossless detector +
packer (quantizeTernaryBf16, :3435-3469) bit-exact against its CPU restatement,
and the GEMV / fused gate-up / prefill GEMM / linear router against the oracle's
exact per-32-group integer sums (gemvTern2Wgsl :449-503, gateupTern2Wgsl
:747-810, gemmTern :1410-1420, linearQ :1594-1598).

Tolerances: GEMV rows 1e-3 relative (the GEMV tests' form, |err| / max(|ref|,
1e-3 rms)).  The tensor-core GEMM rounds every activation to f16(xs * q) (unit
roundoff 2^-11) and sums in f32, so each token row is held to 1e-3 of its max
|y| and every output to 2^-10 * sum_k |w x| (twice the f16 rounding budget)."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import host, row_rel_err, tern_bf16, tern_wgsl_codes, u16_dev, u32_dev

pytestmark = pytest.mark.gpu

TOL = 1e-3
# Bonsai-1.7B (Qwen3-1.7B shapes): q/o, k/v, gate/up, down
SHAPES = [("q", 2048, 2048), ("kv", 1024, 2048), ("gate", 6144, 2048), ("down", 2048, 6144), ("odd", 1000, 1024)]


def _tern(seed, N, K, **kw):
    w = tern_bf16(np.random.default_rng(seed), N, K, **kw)
    pack, sc = oracle.quant_tern_wgsl(w)
    return w, pack, sc


@pytest.mark.parametrize("N,K", [(300, 2048), (2048, 6144), (7, 64)])
def test_pack_bit_exact(cuda, N, K):
    w, pack, sc = _tern(N + K, N, K, wobble=0.01, negzero=0.1)
    got = tb.quantize_tern_bf16(u16_dev(w))
    assert got is not None
    np.testing.assert_array_equal(host(got[0]).view(np.uint32), pack)
    np.testing.assert_array_equal(host(got[1]).view(np.uint16), sc)


def test_pack_rejects_what_the_reference_rejects(cuda):
    rng = np.random.default_rng(9)
    normal = oracle.f32_to_bf16_trunc(rng.normal(0, 0.02, (64, 256)).astype(np.float32))
    assert oracle.quant_tern_wgsl(normal) is None and tb.quantize_tern_bf16(u16_dev(normal)) is None
    w = tern_bf16(rng, 640, 512)
    g = w[639, 480:512]
    i = int(np.flatnonzero(g & 0x7FFF)[-1])
    w[639, 480 + i] = (int(np.max(g & 0x7FFF)) - 3) | (int(g[i]) & 0x8000)   # last row, last group, 3 ulps
    assert oracle.quant_tern_wgsl(w) is None and tb.quantize_tern_bf16(u16_dev(w)) is None
    w2 = tern_bf16(rng, 8, 96)                                               # K % 64 != 0
    assert tb.quantize_tern_bf16(u16_dev(w2)) is None


@pytest.mark.parametrize("B", [1, 3, 8])
@pytest.mark.parametrize("tag,N,K", SHAPES)
def test_gemv_q8(cuda, tag, N, K, B):
    _, pack, sc = _tern(N * 7 + K, N, K)
    x = np.random.default_rng(B).normal(0, 1, (B, K)).astype(np.float32)
    xq, xs, _ = oracle.quant_q8(x)
    y = tb.gemv_tern_wgsl(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc))
    assert row_rel_err(host(y), oracle.gemv_tern_wgsl_q8act(xq, xs, pack, sc)) < TOL


def test_gemv_acc_adds(cuda):
    N, K = 2048, 2048
    _, pack, sc = _tern(5, N, K)
    rng = np.random.default_rng(5)
    xq, xs, _ = oracle.quant_q8(rng.normal(0, 1, (2, K)).astype(np.float32))
    y0 = rng.normal(0, 1, (2, N)).astype(np.float32)
    y = torch.from_numpy(y0.copy()).cuda()
    tb.gemv_tern_wgsl(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc), y=y,
                      acc=True)
    assert row_rel_err(host(y), oracle.gemv_tern_wgsl_q8act(xq, xs, pack, sc) + y0) < TOL


@pytest.mark.parametrize("B", [1, 4])
def test_fused_norm_multi_and_gateup(cuda, B):
    """rmsnormQ + ternary q/k/v in one launch and the fused gate/up: the in-kernel
    int8 rows are tb_rmsnorm_q8's (outputs equal the pre-quantized launch)."""
    H, I = 2048, 6144
    mats = [_tern(30 + i, n, H)[1:] for i, n in enumerate([2048, 1024, 1024])]
    _, gp, gs = _tern(40, I, H)
    _, up, us = _tern(41, I, H)
    rng = np.random.default_rng(B)
    x = rng.normal(0, 1, (B, H)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, H)).view(np.uint16)
    xd, wd = torch.from_numpy(x).cuda(), u16_dev(w16)
    xq, xs, _ = tb.rmsnorm_q8(xd, wd, 1e-6)
    ys = tb.gemv_tern_wgsl_dp4a_multi(xd, [(u32_dev(p), u16_dev(s)) for p, s in mats], norm_w=wd)
    for (p, s), y in zip(mats, ys):
        np.testing.assert_array_equal(host(y), host(tb.gemv_tern_wgsl(xq, xs, u32_dev(p), u16_dev(s))))
        assert row_rel_err(host(y), oracle.gemv_tern_wgsl_q8act(host(xq), host(xs), p, s)) < TOL
    swi = tb.gate_up_silu_tern_dp4a(xd, u32_dev(gp), u16_dev(gs), u32_dev(up), u16_dev(us), norm_w=wd)
    swi2 = tb.gate_up_silu_tern(xq, xs, u32_dev(gp), u16_dev(gs), u32_dev(up), u16_dev(us))
    np.testing.assert_array_equal(host(swi), host(swi2))
    ref = oracle.gateup_tern_wgsl_q8act(host(xq), host(xs), gp, gs, up, us)
    assert row_rel_err(host(swi), ref) < TOL


def test_lm_head_full_size_sampled_rows(cuda):
    """Bonsai-1.7B lm_head 151936 x 2048, packed on the device; a seeded sample of
    rows against the oracle (pack bit-exact, GEMV within tolerance)."""
    N, K = 151936, 2048
    g = torch.Generator(device="cuda").manual_seed(11)
    mag = (torch.rand(N, K // 32, device="cuda", generator=g) * 0.05 + 0.005).view(torch.int32) >> 16
    t = torch.randint(-1, 2, (N, K), device="cuda", generator=g, dtype=torch.int32)
    bits = torch.where(t == 0, torch.zeros_like(t), mag.repeat_interleave(32, dim=1) | ((t < 0).int() << 15))
    w = torch.where(bits >= 32768, bits - 65536, bits).to(torch.int16)   # the same 16 bits
    del t, bits
    pack, sc = tb.quantize_tern_bf16(w)
    rng = np.random.default_rng(12)
    x = rng.normal(0, 1, (1, K)).astype(np.float32)
    xq, xs, _ = oracle.quant_q8(x)
    y = host(tb.gemv_tern_wgsl(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), pack, sc))
    rows = np.sort(rng.choice(N, 64, replace=False))
    rows_t = torch.from_numpy(rows).cuda()
    wp = host(w[rows_t]).view(np.uint16)
    rp, rs = oracle.quant_tern_wgsl(wp)
    np.testing.assert_array_equal(host(pack[rows_t]).view(np.uint32), rp)
    assert row_rel_err(y[:, rows], oracle.gemv_tern_wgsl_q8act(xq, xs, rp, rs)) < TOL


def _gemm_errs(got, ref, xq, xs, pack, sc):
    """(max over token rows of max|err| / max|ref|, max over outputs of
    |err| / (2^-10 sum_k |w_nk x_mk|))"""
    d = np.abs(np.asarray(got, np.float64) - ref)
    K = xq.shape[1]
    absw = np.abs(tern_wgsl_codes(pack, K) - 1) * np.repeat(sc.view(np.float16).astype(np.float64), 32, axis=1)
    absx = np.abs(xq.astype(np.float64)) * np.repeat(xs.astype(np.float64), 32, axis=1)
    budget = 2.0 ** -10 * (absx @ absw.T) + 1e-30
    return float(np.max(np.max(d, axis=1) / np.max(np.abs(ref), axis=1))), float(np.max(d / budget))


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 2048), (128, 2048, 6144), (384, 768, 1024)])
def test_gemm_tern(cuda, M, N, K):
    _, pack, sc = _tern(M + N + K, N, K)
    x = np.random.default_rng(K).normal(0, 1, (M, K)).astype(np.float32)
    xq, xs, _ = oracle.quant_q8(x)
    y = tb.gemm_tern(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc))
    rel, bud = _gemm_errs(host(y), oracle.gemv_tern_wgsl_q8act(xq, xs, pack, sc), xq, xs, pack, sc)
    assert rel < TOL and bud < 1.0, (rel, bud)


def test_linear_router(cuda):
    """linearQ's ternary branch: T <= 16 takes a GEMV (exact group sums; the
    tensor-core one at 2..16 rows), T > 16 quantizes (QUANTQ8T) and takes the GEMM;
    acc adds."""
    N, K = 512, 2048
    _, pack, sc = _tern(77, N, K)
    rng = np.random.default_rng(77)
    for T in (1, 5, 12, 256):
        x = rng.normal(0, 1, (T, K)).astype(np.float32)
        y0 = rng.normal(0, 1, (T, N)).astype(np.float32)
        y = torch.from_numpy(y0.copy()).cuda()
        tb.linear_tern_wgsl(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc), y=y, acc=True)
        xq, xs, _ = oracle.quant_q8(x)
        ref = oracle.gemv_tern_wgsl_q8act(xq, xs, pack, sc)
        if T <= 16:
            assert row_rel_err(host(y) - y0, ref) < TOL
        else:
            rel, _ = _gemm_errs(host(y) - y0, ref, xq, xs, pack, sc)
            assert rel < TOL, rel
    with pytest.raises(tb.TabInferError):
        tb.linear_tern_wgsl(torch.zeros(100, K, device="cuda"), u32_dev(pack), u16_dev(sc))
