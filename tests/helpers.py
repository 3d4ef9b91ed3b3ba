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
