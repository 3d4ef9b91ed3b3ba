"""int3 MoE of LFM2.5 (config 5 shapes): _requant43 bit-exact against its CPU
restatement (the engine's f32ToF16 quirk included), the router's expert ids
exact and weights to 1e-6, and the grouped expert FFN per token within 1e-3
relative (max|err| / max|ref| over the token's hidden row) of the f64 oracle."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import host

pytestmark = pytest.mark.gpu

H, I, NE, K = 2048, 1792, 32, 4


def _int4_from_normal(rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    return tb.quantize_int4_bf16(w.view(torch.int16))


def test_requant43_bit_exact(cuda):
    pack, sc = _int4_from_normal(512, 256, 1)
    # groups that exercise the edges: all zero (m = 0), ties (m = 8), every m
    p = host(pack).view(np.uint32).copy()
    p[0, 0:4] = 0x88888888                      # q4 = 0 everywhere -> m = 0
    p[1, 0:4] = 0x0F0F0F0F                      # -8 and 7 -> m = 8, halves
    for m in range(1, 8):                       # q4 = +m, -m alternating -> max |q4| = m
        p[2 + m, 0:4] = np.uint32(((8 + m) | ((8 - m) << 4)) * 0x01010101)
    # random f16 scales over the normal range (hits the engine's OR rounding quirk)
    rng = np.random.default_rng(0)
    s = host(sc).view(np.uint16).copy()
    s[256:] = rng.integers(0x0400, 0x7BFF, s[256:].shape).astype(np.uint16)
    pack_d = torch.from_numpy(p.view(np.int32)).cuda()
    sc_d = torch.from_numpy(s.view(np.int16)).cuda()
    p3, s3 = tb.requant_int3(pack_d, sc_d)
    rp3, rs3 = oracle.requant43(p, s)
    np.testing.assert_array_equal(host(p3).view(np.uint32), rp3)
    np.testing.assert_array_equal(host(s3).view(np.uint16), rs3)


def test_router_matches_oracle(cuda):
    rng = np.random.default_rng(3)
    T = 64
    logits = rng.standard_normal((T, NE)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(NE)).astype(np.float32)
    logits[5, :] = -1.0
    logits[5, 7] = logits[5, 9] = 4.0          # a tie at the top: the lower expert first
    bias[7] = bias[9] = 0.0
    idx, wt = tb.moe_router(torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda(), K)
    ridx, rwt = oracle.moe_router(logits, bias, K)
    np.testing.assert_array_equal(host(idx).view(np.uint32), ridx)
    np.testing.assert_allclose(host(wt), rwt, rtol=1e-6, atol=1e-7)
    assert list(ridx[5][:2]) == [7, 9]


@pytest.fixture(scope="module")
def experts():
    """config 5 experts: N(0, 0.02) -> int4 G32 -> int3 (the reference's path)."""
    ws = []
    for j, (rows, cols) in enumerate(((NE * I, H), (NE * I, H), (NE * H, I))):
        pack, sc = _int4_from_normal(rows, cols, 100 + j)
        ws.append(tb.requant_int3(pack, sc))
    torch.cuda.synchronize()
    return ws


def _host_planes(w):
    return host(w[0]).view(np.uint32), host(w[1]).view(np.uint16)


@pytest.mark.parametrize("T", [1, 8, 64])
def test_moe_ffn_matches_oracle(cuda, experts, T):
    rng = np.random.default_rng(T)
    logits = rng.standard_normal((T, NE)).astype(np.float32)
    bias = np.zeros(NE, np.float32)
    a = rng.standard_normal((T, H)).astype(np.float32)
    x0 = rng.standard_normal((T, H)).astype(np.float32)
    idx, wt = tb.moe_router(torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda(), K)
    x = torch.from_numpy(x0.copy()).cuda()
    w1, w3, w2 = experts
    tb.moe_ffn_int3(x, torch.from_numpy(a).cuda(), idx, wt, w1, w3, w2, NE, H, I)
    got = host(x) - x0
    rows = np.arange(T) if T <= 8 else np.sort(rng.choice(T, 6, replace=False))
    ref = oracle.moe_ffn_int3(a[rows], host(idx).view(np.uint32)[rows], host(wt)[rows], _host_planes(w1),
                              _host_planes(w3), _host_planes(w2), H, I)
    err = np.max(np.abs(got[rows] - ref), axis=1) / np.max(np.abs(ref), axis=1)
    assert float(np.max(err)) < 1e-3, err


def test_moe_many_pairs_one_expert(cuda, experts):
    """Every token routed to the same experts: chunks of pairs per expert."""
    T = 20
    idx = torch.tensor([[3, 17, 0, 31]] * T, dtype=torch.int32, device="cuda")
    wt = torch.full((T, K), 0.25, device="cuda")
    rng = np.random.default_rng(5)
    a = rng.standard_normal((T, H)).astype(np.float32)
    x = torch.zeros(T, H, device="cuda")
    w1, w3, w2 = experts
    tb.moe_ffn_int3(x, torch.from_numpy(a).cuda(), idx, wt, w1, w3, w2, NE, H, I)
    rows = [0, 9, 19]
    ref = oracle.moe_ffn_int3(a[rows], host(idx).view(np.uint32)[rows], host(wt)[rows], _host_planes(w1),
                              _host_planes(w3), _host_planes(w2), H, I)
    err = np.max(np.abs(host(x)[rows] - ref), axis=1) / np.max(np.abs(ref), axis=1)
    assert float(np.max(err)) < 1e-3, err


# ---- group-128 int3 (the LFM2.5 benchmark configuration's format) -------------------
def _bf16_normal(rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).to(torch.bfloat16).view(torch.int16)


@pytest.mark.parametrize("group", [32, 128])
def test_quant_int3_bit_exact(cuda, group):
    w = _bf16_normal(96, 1024, 11 + group)
    w[0, :group] = 0                             # an all-zero group: scale 0, q = 0
    wh = host(w).view(np.uint16)
    p3, s3 = tb.quant_int3(w, group)
    rp3, rs3 = oracle.quant_int3(wh, group)
    np.testing.assert_array_equal(host(p3).view(np.uint32), rp3)
    np.testing.assert_array_equal(host(s3).view(np.uint16), rs3)
    assert rs3[0, 0] == 0 and rp3[0, 0, 2] == 0xFFFFFFFF and rp3[0, 0, 0] == 0


@pytest.fixture(scope="module")
def experts128():
    """config 5 experts as the configuration states them: N(0, 0.02) -> int3, group 128."""
    ws = [tb.quant_int3(_bf16_normal(rows, cols, 200 + j), 128)
          for j, (rows, cols) in enumerate(((NE * I, H), (NE * I, H), (NE * H, I)))]
    torch.cuda.synchronize()
    return ws


@pytest.mark.parametrize("T", [1, 8, 64])
def test_moe_ffn_group128_matches_oracle(cuda, experts128, T):
    rng = np.random.default_rng(T + 40)
    logits = rng.standard_normal((T, NE)).astype(np.float32)
    a = rng.standard_normal((T, H)).astype(np.float32)
    idx, wt = tb.moe_router(torch.from_numpy(logits).cuda(), torch.zeros(NE, device="cuda"), K)
    x = torch.zeros(T, H, device="cuda")
    w1, w3, w2 = experts128
    tb.moe_ffn_int3(x, torch.from_numpy(a).cuda(), idx, wt, w1, w3, w2, NE, H, I, group=128)
    rows = np.arange(T) if T <= 8 else np.sort(rng.choice(T, 6, replace=False))
    ref = oracle.moe_ffn_int3(a[rows], host(idx).view(np.uint32)[rows], host(wt)[rows], _host_planes(w1),
                              _host_planes(w3), _host_planes(w2), H, I, group=128)
    err = np.max(np.abs(host(x)[rows] - ref), axis=1) / np.max(np.abs(ref), axis=1)
    assert float(np.max(err)) < 1e-3, err
