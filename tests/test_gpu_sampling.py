"""The sampling transforms before argmax (models/qwen3.js:2692-2737): the grammar
logit mask bit-exact, the Gumbel noise within 1e-5 of the restatement (u
formed in f32 as the shader does; only the two logs differ in rounding), the fused
mask + noise + argmax identical to the three separate steps, and Gumbel-max
sampling drawing from softmax(logits / T) (a chi-square check over 40000 rows)."""
import numpy as np
import pytest
import torch

import oracle
import tabinfer_b200 as tb
from helpers import host

pytestmark = pytest.mark.gpu


def _words(bits):
    """bit i of a row -> bit i % 32 of word i / 32 (little-endian packing)"""
    rows, n = bits.shape
    pad = np.zeros((rows, (n + 31) // 32 * 32), bool)
    pad[:, :n] = bits
    return np.packbits(pad, axis=1, bitorder="little").view(np.uint32)


def _mask(rng, rows, n, keep=0.3):
    bits = rng.random((rows, n)) < keep
    return bits, torch.from_numpy(_words(bits).view(np.int32)).cuda()


def test_logit_mask_bit_exact(cuda):
    rng = np.random.default_rng(1)
    rows, n = 3, 151936
    x = rng.normal(0, 3, (rows, n)).astype(np.float32)
    bits, m = _mask(rng, rows, n)
    y = host(tb.logit_mask(torch.from_numpy(x).cuda(), m))
    np.testing.assert_array_equal(y, np.where(bits, x, np.float32(-3.0e38)))


def test_gumbel_noise_matches_restatement(cuda):
    rows, n, seed, temp = 2, 151936, 0x1234ABCD, 0.7
    x = np.random.default_rng(2).normal(0, 3, (rows, n)).astype(np.float32)
    y = host(tb.gumbel_noise(torch.from_numpy(x).cuda(), seed, temp))
    ref = x.astype(np.float64) + oracle.gumbel_noise(rows * n, seed, temp).reshape(rows, n)
    fin = np.isfinite(ref)        # u rounds to 1 in f32 at h >> 8 = 2^24 - 1: +inf noise, as the shader
    np.testing.assert_array_equal(y[~fin], ref[~fin])
    assert float(np.max(np.abs(y[fin] - ref[fin]))) < 1e-5


@pytest.mark.parametrize("temp", [0.0, 0.8])
def test_fused_sample_argmax_equals_the_three_steps(cuda, temp):
    rng = np.random.default_rng(3)
    rows, n = 4, 151936
    x = rng.normal(0, 3, (rows, n)).astype(np.float32)
    _, m = _mask(rng, rows, n, keep=0.05)
    seeds = tb.GumbelSeeds()
    seed = seeds.next()
    xd = torch.from_numpy(x).cuda()
    fused = host(tb.sample_argmax(xd, m, seed, temp))
    np.testing.assert_array_equal(host(xd), x)          # logits untouched
    y = tb.logit_mask(xd.clone(), m)
    if temp:
        tb.gumbel_noise(y, seed, temp)
    sep = host(tb.argmax(y)).view(np.uint32)
    np.testing.assert_array_equal(fused.view(np.uint32), sep)
    # and the oracle's choice wherever its top-2 margin is clear of rounding
    w = host(m).view(np.uint32)
    bits = np.unpackbits(w.view(np.uint8), axis=1, bitorder="little")[:, :n].astype(bool)
    ref = np.where(bits, x.astype(np.float64), -3.0e38)
    if temp:
        ref = ref + oracle.gumbel_noise(rows * n, seed, temp).reshape(rows, n)
    for r in range(rows):
        top = np.sort(ref[r])[-2:]
        if top[1] - top[0] > 1e-4:
            assert fused.view(np.uint32)[r] == int(np.argmax(ref[r]))


def test_gumbel_max_samples_softmax(cuda):
    """argmax(logits + T g) ~ softmax(logits / T): 40000 rows of one 8-token
    distribution (each row a different noise draw) against the expected counts."""
    logits = np.array([1.0, 0.5, 0.0, -0.5, 2.0, -1.0, 0.25, 1.5], np.float32)
    temp, rows = 0.9, 40000
    x = torch.from_numpy(np.tile(logits, (rows, 1))).cuda()
    ids = host(tb.sample_argmax(x, None, 0xC0FFEE, temp)).view(np.uint32)
    p = np.exp(logits / temp - np.max(logits / temp))
    p /= p.sum()
    counts = np.bincount(ids, minlength=8)
    chi2 = float(np.sum((counts - rows * p) ** 2 / (rows * p)))
    assert chi2 < 30.0, (chi2, counts, rows * p)    # 7 dof: p(chi2 > 30) ~ 1e-4
