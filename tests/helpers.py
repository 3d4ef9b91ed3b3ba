"""Shared helpers for the GPU parity tests."""
import numpy as np
import torch


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def u16_dev(a):
    """uint16 numpy bit patterns -> int16 device tensor (same bits)."""
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).cuda()


def u32_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).cuda()


def host(t, np_dtype=None):
    a = t.detach().cpu().numpy()
    return a.view(np_dtype) if np_dtype is not None else a


def row_rel_err(got, ref):
    """Per-row relative error |got-ref| / max(|ref|, 1e-3 * rms(ref)) — rows near
    zero are judged against the row population's scale."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2)) if ref.size else 1.0
    den = np.maximum(np.abs(ref), 1e-3 * max(rms, 1e-30))
    return float(np.max(np.abs(got - ref) / den)) if ref.size else 0.0


def bf16_normal(rng, shape, std):
    """f32 N(0, std) truncated to bf16 bits (qwen3.js:3072 f32ToBf16)."""
    x = rng.normal(0, std, shape).astype(np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def bf16_to_f32(u):
    return (u.astype(np.uint32) << 16).view(np.float32)


def tern_bf16(rng, N, K, wobble=0.0, negzero=0.0):
    """Ternary bf16 bits [N,K] in the form quantizeTernaryBf16 accepts: per 32-group
    a bf16 magnitude m, values {-m, 0, +m}; a `wobble` fraction of the nonzeros sit
    1-2 ulps below m (the f16-export wobble the reference tolerates), a `negzero`
    fraction of the zeros are -0."""
    s = rng.uniform(0.004, 0.06, (N, K // 32)).astype(np.float32)
    m = (s.view(np.uint32) >> 16).astype(np.int32) & 0x7FFF
    t = rng.integers(-1, 2, (N, K))
    mag = np.repeat(m, 32, axis=1)
    if wobble:
        mag = mag - (rng.random((N, K)) < wobble) * rng.integers(1, 3, (N, K))
    bits = np.where(t == 0, 0, mag | ((t < 0).astype(np.int32) << 15))
    if negzero:
        bits = np.where((t == 0) & (rng.random((N, K)) < negzero), 0x8000, bits)
    return bits.astype(np.uint16)


def tern_wgsl_codes(pack, K):
    """codes [N,K] of the WebGPU ternary layout: weight k at bits 8(k%4)+2((k/4)%4) of word k/16."""
    pack = np.asarray(pack, np.uint32)
    k = np.arange(K)
    sh = (8 * (k & 3) + 2 * ((k >> 2) & 3)).astype(np.uint32)
    return ((pack[:, k >> 4] >> sh) & 3).astype(np.int32)
