"""GPU parity: the tensor-core decode GEMVs at 2..16 rows (linearQ's T > 1 DP4A
route, models/qwen3.js:1600-1607; gemmdp4Wgsl :1321-1407; gemmTern :1410-1420)
against the oracle's exact per-32-group integer sums in double.

The int8 rows are QUANTQ8T (or RMSNORMQ with a norm weight), bit-identical to
the oracle's, and every group sum is exact, so the only difference is the f32
scaling and summation order: per-row relative error <= 1e-3 (|err| /
max(|ref|, 1e-3 rms)), the GEMV tests' bar."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import bf16_normal, host, row_rel_err, tern_bf16, u16_dev, u32_dev

pytestmark = pytest.mark.gpu
TOL = 1e-3

# Qwen3-1.7B projections (q, k/v, gate/up, down), a multi-item row count, a row
# count that is not a whole number of items, and K = 768 (a last stage of 8 groups)
SHAPES = [(2048, 2048), (1024, 2048), (6144, 2048), (2048, 6144), (8200, 1024), (40, 256), (1032, 768)]


def _mat(seed, N, K):
    w = bf16_normal(np.random.default_rng(seed), (N, K), 0.02)
    return oracle.quant_int4_g32(w)


def _x(seed, B, K):
    x = np.random.default_rng(seed).normal(0, 1, (B, K)).astype(np.float32)
    x[0, :32] = 0.0                     # an all-zero group: scale 0
    return x


@pytest.mark.parametrize("B", [2, 5, 8, 9, 16])
@pytest.mark.parametrize("N,K", SHAPES)
def test_gemv_mma_int4(cuda, N, K, B):
    pack, sc = _mat(N + 3 * K, N, K)
    x = _x(B + N, B, K)
    y = tb.gemv_mma(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc))
    xq, xs, _ = oracle.quant_q8(x)
    assert row_rel_err(host(y), oracle.gemv_int4_q8act(xq, xs, pack, sc)) < TOL


@pytest.mark.parametrize("B", [4, 16])
def test_gemv_mma_rmsnorm_and_residual(cuda, B):
    N, K = 4096, 2048
    pack, sc = _mat(7, N, K)
    rng = np.random.default_rng(8)
    x = rng.normal(0, 3, (B, K)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, K)).view(np.uint16)
    r = rng.normal(0, 1, (B, N)).astype(np.float32)
    y = torch.from_numpy(r.copy()).cuda()
    tb.gemv_mma(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc), norm_w=u16_dev(w16), eps=1e-6, y=y,
                acc=True)
    xq, xs, _, _ = oracle.rmsnorm_q8(x, w16, 1e-6)
    ref = oracle.gemv_int4_q8act(xq, xs, pack, sc) + r
    assert row_rel_err(host(y), ref) < TOL


@pytest.mark.parametrize("B", [3, 8, 16])
@pytest.mark.parametrize("I,H", [(6144, 2048), (3072, 1024), (40, 256)])
def test_gateup_silu_mma_int4(cuda, I, H, B):
    gp, gs = _mat(I, I, H)
    up, us = _mat(I + 1, I, H)
    x = _x(B * 3 + I, B, H)
    swi = tb.gate_up_silu_mma(torch.from_numpy(x).cuda(), u32_dev(gp), u16_dev(gs), u32_dev(up), u16_dev(us))
    xq, xs, _ = oracle.quant_q8(x)
    assert row_rel_err(host(swi), oracle.gateup_q8act(xq, xs, gp, gs, up, us)) < TOL


def _tern(seed, N, K):
    pack, sc = oracle.quant_tern_wgsl(tern_bf16(np.random.default_rng(seed), N, K))
    return pack, sc


@pytest.mark.parametrize("B", [2, 8, 16])
@pytest.mark.parametrize("N,K", [(2048, 2048), (2048, 6144), (1000, 1024), (264, 768)])
def test_gemv_mma_tern_wgsl(cuda, N, K, B):
    pack, sc = _tern(N * 5 + K, N, K)
    x = _x(B + 77, B, K)
    y = tb.gemv_mma(torch.from_numpy(x).cuda(), u32_dev(pack), u16_dev(sc), tern=True)
    xq, xs, _ = oracle.quant_q8(x)
    assert row_rel_err(host(y), oracle.gemv_tern_wgsl_q8act(xq, xs, pack, sc)) < TOL


@pytest.mark.parametrize("B", [4, 16])
def test_gateup_silu_mma_tern_wgsl(cuda, B):
    I, H = 6144, 2048
    gp, gs = _tern(11, I, H)
    up, us = _tern(12, I, H)
    rng = np.random.default_rng(13)
    x = rng.normal(0, 3, (B, H)).astype(np.float32)
    w16 = np.float16(rng.uniform(0.5, 1.5, H)).view(np.uint16)
    swi = tb.gate_up_silu_mma(torch.from_numpy(x).cuda(), u32_dev(gp), u16_dev(gs), u32_dev(up), u16_dev(us),
                              norm_w=u16_dev(w16), eps=1e-6, tern=True)
    xq, xs, _, _ = oracle.rmsnorm_q8(x, w16, 1e-6)
    assert row_rel_err(host(swi), oracle.gateup_tern_wgsl_q8act(xq, xs, gp, gs, up, us)) < TOL


def test_gemv_mma_matches_batched_dp4a(cuda):
    """The same int8 rows and exact group sums as the 8-row dp4a GEMV: the two
    differ only in f32 summation order."""
    N, K, B = 2048, 2048, 8
    pack, sc = _mat(21, N, K)
    x = torch.from_numpy(_x(22, B, K)).cuda()
    a = host(tb.gemv_mma(x, u32_dev(pack), u16_dev(sc)))
    b = host(tb.gemv_dp4a(x, u32_dev(pack), u16_dev(sc)))
    # f32 rounding of 64 group terms per row, against the row's largest output
    assert np.max(np.abs(a - b) / np.max(np.abs(b), axis=1, keepdims=True)) < 1e-5


def test_gemv_mma_rejects_bad_shapes(cuda):
    pack, sc = _mat(1, 64, 256)
    for B, K in ((1, 256), (17, 256)):
        with pytest.raises(tb.TabInferError):
            tb.gemv_mma(torch.zeros((B, K), device="cuda"), u32_dev(pack), u16_dev(sc))
    p2, s2 = _mat(2, 64, 224)                 # K % 256 != 0
    with pytest.raises(tb.TabInferError):
        tb.gemv_mma(torch.zeros((4, 224), device="cuda"), u32_dev(p2), u16_dev(s2))
    p3, s3 = _mat(3, 60, 256)                 # rows % 8 != 0
    with pytest.raises(tb.TabInferError):
        tb.gemv_mma(torch.zeros((4, 256), device="cuda"), u32_dev(p3), u16_dev(s3))


@pytest.mark.parametrize("B", [4, 16])
def test_gemv_mma_multi_equals_separate(cuda, B):
    """The q/k/v triple in one launch over concatenated rows: each matrix equals
    its own launch bit for bit (the same group sums in the same order)."""
    mats = [_mat(30 + i, n, 2048) for i, n in enumerate([2048, 1024, 1024])]
    rng = np.random.default_rng(31)
    x = torch.from_numpy(rng.normal(0, 1, (B, 2048)).astype(np.float32)).cuda()
    w16 = u16_dev(np.float16(rng.uniform(0.5, 1.5, 2048)).view(np.uint16))
    dev = [(u32_dev(p), u16_dev(s)) for p, s in mats]
    ys = tb.gemv_mma_multi(x, dev, norm_w=w16, eps=1e-6)
    xq, xs, _, _ = oracle.rmsnorm_q8(host(x), host(w16).view(np.uint16), 1e-6)
    for (p, s), (pd, sd), y in zip(mats, dev, ys):
        np.testing.assert_array_equal(host(y), host(tb.gemv_mma(x, pd, sd, norm_w=w16, eps=1e-6)))
        assert row_rel_err(host(y), oracle.gemv_int4_q8act(xq, xs, p, s)) < TOL
