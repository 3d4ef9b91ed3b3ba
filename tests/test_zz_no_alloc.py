"""The allocation-free split-KV decode entry point (tb_attn_decode_q8_noalloc).

It exists for callers that cannot let the library call cudaMalloc — a process
that hands its whole device budget to its own pool at start-up, or a decode loop
that must not let an allocation synchronize the device mid-step.  Its partials
live in a fixed device array inside the library.  Through the C ABI the test
checks that two calls in a row (the second reusing the array with the first
call's contents still in it) give bit-for-bit the output of tb_attn_decode_q8
at the same split count (both run the same kernel, so nothing may differ), that
one case agrees with the CPU oracle within the attention tolerance used
elsewhere (1e-4 of each head row's largest magnitude), that the automatic split
count is capped to what fits the array for a wide model, and that an explicit
request larger than the array is refused.

This file is collected last on purpose; it must pass alone and after the rest.
"""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from tabinfer_b200._lib import LIB, P

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 1 << 18


def _case(seed, S, nHq, nKv, hd):
    rng = np.random.default_rng(seed)
    K = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    V = rng.normal(0, 1, (S, nKv * hd)).astype(np.float32)
    Kq, Ks = oracle.kv_quant_q8(K)
    Vq, Vs = oracle.kv_quant_q8(V)
    q = rng.normal(0, 1, nHq * hd).astype(np.float32)
    host = (q, Kq, Ks.reshape(S, -1), Vq, Vs.reshape(S, -1))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    return dev(q), tuple(dev(a) for a in host[1:]), host


def _noalloc(ctx, qr, kv, S, nHq, nKv, hd, nsplit):
    out = torch.full((nHq * hd,), float("nan"), dtype=torch.float32, device="cuda")
    Kq, Ks, Vq, Vs = kv
    ptr = lambda t: P(t.data_ptr())  # noqa: E731
    rc = LIB.tb_attn_decode_q8_noalloc(ctx.h, ptr(out), ptr(qr), ptr(Kq), ptr(Ks), ptr(Vq), ptr(Vs),
                                       S, nHq, nKv, hd, nsplit)
    return rc, out


def _head_rel(got, ref, hd):
    got = np.asarray(got, np.float64).reshape(-1, hd)
    ref = np.asarray(ref, np.float64).reshape(-1, hd)
    return float(np.max(np.abs(got - ref).max(1) / np.abs(ref).max(1)))


def test_noalloc_decode_matches_scratch_entry_point_twice(cuda):
    ctx = tb.default_context(0)
    nHq, nKv, hd = 16, 8, 128
    # two calls in a row: a long context with many splits, then a short one that
    # uses fewer slots of the same array (stale partials from call 1 remain)
    for seed, S, nsplit in ((1, 4096, 64), (2, 300, 3)):
        qr, kv, host = _case(seed, S, nHq, nKv, hd)
        rc, got = _noalloc(ctx, qr, kv, S, nHq, nKv, hd, nsplit)
        assert rc == 0, LIB.tb_last_error(ctx.h)
        want = tb.attention_decode_q8(qr, kv, S, nHq, nKv, hd, nsplit)
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.isfinite(g))
        np.testing.assert_array_equal(g, w, err_msg="S=%d nsplit=%d" % (S, nsplit))
        if S == 300:
            ref = oracle.attn_decode_q8(*host, S, nHq, nKv, hd)
            assert _head_rel(g, ref, hd) < 1e-4
    assert ctx.device_error() == 0


def test_noalloc_auto_split_fits_wide_models(cuda):
    # 64 q heads over 8 kv heads at 8192 keys: the automatic split count of the
    # scratch entry point (37) would need 64*37*130 floats, more than the array
    ctx = tb.default_context(0)
    nHq, nKv, hd, S = 64, 8, 128, 8192
    fit = SCRATCH_FLOATS // (nHq * (hd + 2))
    qr, kv, _ = _case(4, S, nHq, nKv, hd)
    rc, got = _noalloc(ctx, qr, kv, S, nHq, nKv, hd, 0)
    assert rc == 0, LIB.tb_last_error(ctx.h)
    want = tb.attention_decode_q8(qr, kv, S, nHq, nKv, hd, fit)
    np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())


def test_noalloc_decode_rejects_oversized_requests(cuda):
    ctx = tb.default_context(0)
    nHq, nKv, hd, S = 16, 8, 128, 300
    qr, kv, _ = _case(3, S, nHq, nKv, hd)
    rc, _ = _noalloc(ctx, qr, kv, S, nHq, nKv, hd, 1024)   # 16*1024*130 floats > 262144
    assert rc == 1
    assert b"exceeds the fixed scratch" in LIB.tb_last_error(ctx.h)
