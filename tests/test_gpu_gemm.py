"""Prefill GEMM on tcgen05 (tb_gemm_int4_g32) against the CPU restatement of the
reference's f16 prefill GEMM (gemmQ, models/qwen3.js:964-1026).

Tolerance: every token row of Y within 1e-3 relative of the f64 sum of the same
f16 operands, max_n |y - ref| / max_n |ref|.  (The GEMV tests' per-element form,
|err| / max(|ref|, 1e-3 rms), is not used here: a K = 2048..6144 dot product
summed in f32 -- on the tensor core as in the reference's own f32 gemmQ -- is off
by ~1e-6 of the rms, which that form magnifies 1000x on near-zero outputs.)
The rms-relative error is also held to 1e-4 (measured ~1e-5 at K = 2048: the
tensor core's f32 accumulation keeps slightly fewer low bits than a sequential
f32 sum)."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import bf16_normal, host, u16_dev, u32_dev

TOL = 1e-3


def row_rel_err(got, ref):
    """max over token rows of max|got - ref| / max|ref|"""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.max(np.abs(got - ref), axis=1) / np.max(np.abs(ref), axis=1)))

pytestmark = pytest.mark.gpu


def _weights(rng, N, K):
    w = bf16_normal(rng, (N, K), 0.02)
    pack, sc = oracle.quant_int4_g32(w)
    return pack, sc


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 512), (128, 1024, 2048), (384, 256, 6144),
                                   (256, 768, 1024)])
def test_gemm_f32_activations(cuda, M, N, K):
    rng = np.random.default_rng(M + N + K)
    pack, sc = _weights(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = host(tb.gemm_q(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc)))
    ref = oracle.gemm_int4_f16(x, pack, sc)
    err = row_rel_err(y, ref)
    assert err < TOL, err
    # exact f16 products summed in f32: the error is accumulation rounding only
    rms_err = float(np.max(np.abs(y - ref)) / np.sqrt(np.mean(ref ** 2)))
    assert rms_err < 1e-4, rms_err


def test_gemm_bf16_activations_and_acc(cuda):
    """config 4's bf16 activations; acc adds into y (linearQ's fused residual)."""
    M, N, K = 256, 512, 2048
    rng = np.random.default_rng(4)
    pack, sc = _weights(rng, N, K)
    xb = bf16_normal(rng, (M, K), 1.0)
    y0 = rng.standard_normal((M, N)).astype(np.float32)
    y = torch.from_numpy(y0.copy()).cuda()
    xt = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    tb.gemm_q(xt, u32_dev(pack), u16_dev(sc), y=y, acc=True)
    ref = oracle.gemm_int4_f16(xb, pack, sc) + y0
    assert row_rel_err(host(y), ref) < TOL


def test_gemm_config4_shape_sampled_rows(cuda):
    """Config 4 at full size (M = 2048 tokens x gate 6144 x 2048): a seeded
    sample of token rows against the oracle, plus additivity over acc."""
    M, N, K = 2048, 6144, 2048
    g = torch.Generator(device="cuda").manual_seed(7)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    pack, sc = tb.quantize_int4_bf16(w.view(torch.int16))
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    y = tb.gemm_q(x, pack, sc)
    rows = np.sort(np.random.default_rng(3).choice(M, 16, replace=False))
    xs = host(x[torch.from_numpy(rows).cuda()].view(torch.int16)).view(np.uint16)
    ref = oracle.gemm_int4_f16(xs, host(pack).view(np.uint32), host(sc).view(np.uint16))
    assert row_rel_err(host(y)[rows], ref) < TOL
    y2 = y.clone()
    tb.gemm_q(x, pack, sc, y=y2, acc=True)
    np.testing.assert_allclose(host(y2), 2 * host(y), rtol=1e-6, atol=1e-6)


def _dp4_budget_err(got, ref, xq, xs, pack, sc):
    """max over outputs of |err| / (2^-10 sum_k |w x|): the f16 rounding of xs*q
    (2^-11) is the one difference from gemmDP4A's exact group sums."""
    K = xq.shape[1]
    w = np.abs(oracle.dequant_int4_g32(pack, sc).astype(np.float64))
    absx = np.abs(xq.astype(np.float64)) * np.repeat(xs.astype(np.float64), 32, axis=1)
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref) / (2.0 ** -10 * (absx @ w.T) + 1e-30)))


def _rms_err(got, ref):
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref)) / np.sqrt(np.mean(ref ** 2)))


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 512, 2048), (384, 768, 6144), (128, 2048, 1024)])
def test_gemm_dp4_exact_group_sums(cuda, M, N, K):
    """gemmDP4A with exact per-group int8 sums against the oracle's: only the f32
    accumulation of the per-group terms differs (~1e-6 of the rms)."""
    rng = np.random.default_rng(M * 3 + K)
    pack, sc = _weights(rng, N, K)
    xq, xs, _ = oracle.quant_q8(rng.standard_normal((M, K)).astype(np.float32))
    y = host(tb.gemm_dp4(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc)))
    ref = oracle.gemv_int4_q8act(xq, xs, pack, sc)
    assert _rms_err(y, ref) < 1e-5
    assert row_rel_err(y, ref) < 1e-5


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (256, 768, 2048)])
def test_gemm_dp4_exact_ternary(cuda, M, N, K):
    """gemmTern (qwen3.js:1410-1420) with exact group sums."""
    from helpers import tern_bf16
    rng = np.random.default_rng(M + N + K)
    pack, sc = oracle.quant_tern_wgsl(tern_bf16(rng, N, K))
    xq, xs, _ = oracle.quant_q8(rng.standard_normal((M, K)).astype(np.float32))
    y = host(tb.gemm_dp4(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc),
                         tern=True))
    ref = oracle.gemv_tern_wgsl_q8act(xq, xs, pack, sc)
    assert _rms_err(y, ref) < 1e-5


@pytest.mark.parametrize("tern", [False, True])
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 384, 1024), (640, 2048, 2048), (2048, 1024, 6144),
                                   (1280, 1920, 640)])
def test_gemm_dp4_tcgen05_equals_warp_form(cuda, M, N, K, tern):
    """The tcgen05 kind::i8 kernel (raw nibbles / codes as unsigned bytes, the offset
    removed through kc) and the mma.sync kernel (signed widened weights) compute the
    same group sums and fold them in the same order: every output bit-equal, for
    every epilogue.  (640, 2048) and (2048, 1024) give more tiles than SMs, so a CTA
    runs several tiles through the same stage ring and TMEM slots; (1280, 1920, 640)
    gives 150 tiles, two past one a SM."""
    from helpers import tern_bf16
    rng = np.random.default_rng(M + 7 * N + K + tern)
    pack, sc = oracle.quant_tern_wgsl(tern_bf16(rng, N, K)) if tern else _weights(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[3, :64] = 0.0                       # zero groups: scale 0
    x[5] *= 40.0                          # a row of large activations
    xq, xs, _ = oracle.quant_q8(x)
    args = (torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc))
    y0 = rng.standard_normal((M, N)).astype(np.float32)
    for epi in (0, 1, 2):
        a = host(tb.gemm_dp4(*args, y=torch.from_numpy(y0.copy()).cuda(), epilogue=epi, tern=tern))
        b = host(tb.gemm_dp4(*args, y=torch.from_numpy(y0.copy()).cuda(), epilogue=epi, tern=tern, warp=True))
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    ref = (oracle.gemv_tern_wgsl_q8act if tern else oracle.gemv_int4_q8act)(xq, xs, pack, sc)
    # each row against its own largest output (row 5's outputs are 40x the others')
    y = host(tb.gemm_dp4(*args, tern=tern)).astype(np.float64)
    assert np.max(np.abs(y - ref) / np.max(np.abs(ref), axis=1, keepdims=True)) < 1e-5


def test_gemm_dp4_extreme_group_sums(cuda):
    """Activations and weights at the ends of their ranges (xq = -127/+127, nibbles 0
    and 15): the largest group sums, 32 * 127 * 8, stay exact through the offset
    conversion; checked against the exact integer products in double."""
    M, N, K = 128, 256, 512
    rng = np.random.default_rng(77)
    xq = np.where(rng.random((M, K)) < 0.5, -127, 127).astype(np.int8)
    xq[0] = -127
    xs = np.full((M, K // 32), 0.5, np.float32)
    nib = np.where(rng.random((N, K)) < 0.5, 0, 15).astype(np.uint32)
    nib[0] = 0
    pack = np.zeros((N, K // 8), np.uint32)
    for i in range(8):
        pack |= nib[:, i::8] << (4 * i)
    sc = np.full((N, K // 32), np.float16(0.25).view(np.uint16), np.uint16)
    y = host(tb.gemm_dp4(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc)))
    w = nib.astype(np.float64) - 8.0
    ref = (xq.astype(np.float64) @ w.T) * 0.125
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=0)
    assert y[0, 0] == 127 * 8 * K * 0.125


def test_gemm_dp4_f16_within_rounding_budget(cuda):
    """The tcgen05 f16-operand form: every output within 2^-10 * sum |w x|."""
    M, N, K = 256, 512, 2048
    rng = np.random.default_rng(31)
    pack, sc = _weights(rng, N, K)
    xq, xs, _ = oracle.quant_q8(rng.standard_normal((M, K)).astype(np.float32))
    y = host(tb.gemm_dp4_f16(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc)))
    ref = oracle.gemv_int4_q8act(xq, xs, pack, sc)
    assert row_rel_err(y, ref) < TOL
    assert _dp4_budget_err(y, ref, xq, xs, pack, sc) < 1.0


@pytest.mark.parametrize("f16", [False, True])
def test_gemm_dp4_epilogues(cuda, f16):
    """epilogue 1 adds into y; epilogue 2 is the forward's swiglu, silu(gate) * up."""
    M, N, K = 128, 512, 1024
    rng = np.random.default_rng(12)
    pack, sc = _weights(rng, N, K)
    xq, xs, _ = oracle.quant_q8(rng.standard_normal((M, K)).astype(np.float32))
    args = (torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), u32_dev(pack), u16_dev(sc))
    fn = tb.gemm_dp4_f16 if f16 else tb.gemm_dp4
    base = host(fn(*args))
    y0 = rng.standard_normal((M, N)).astype(np.float32)
    y1 = host(fn(*args, y=torch.from_numpy(y0.copy()).cuda(), epilogue=1))
    np.testing.assert_allclose(y1, y0 + base, rtol=1e-6, atol=1e-6)
    y2 = host(fn(*args, y=torch.from_numpy(y0.copy()).cuda(), epilogue=2))
    g = y0.astype(np.float64)
    np.testing.assert_allclose(y2, g / (1 + np.exp(-g)) * base, rtol=1e-5, atol=1e-6)


def test_linear_router_prefill_goes_to_gemm(cuda):
    """linearQ with T > 8 (prefill) routes to gemmDP4A: QUANTQ8T rows then the exact GEMM."""
    M, N, K = 256, 512, 1024
    rng = np.random.default_rng(9)
    pack, sc = _weights(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = host(tb.linear_q(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc)))
    xq, xs, _ = oracle.quant_q8(x)
    ref = oracle.gemv_int4_q8act(xq, xs, pack, sc)
    assert _rms_err(y, ref) < 1e-5


def test_gemm_rejects_untiled_shapes(cuda):
    rng = np.random.default_rng(1)
    pack, sc = _weights(rng, 256, 128)
    x = torch.zeros(100, 128, device="cuda")
    with pytest.raises(tb.TabInferError):
        tb.gemm_q(x, u32_dev(pack), u16_dev(sc))
