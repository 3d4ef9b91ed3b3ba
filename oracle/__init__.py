"""CPU oracle for the TabInfer quantized-GEMV hot path (numpy front end).

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU
legs of bench.py may import this package; it is the checker, never the thing
shipped or measured as the product.  The arithmetic lives in tb_oracle.c (each
function there cites the reference file:line it restates); this module loads
it with ctypes and adds the reference's own fixture generators:

* the xorshift64 generator and "ternaryish" weights of
  native/crates/n2-kernels/src/tern.rs:355-389 and n2-cli main.rs:93-114;
* the sin/cos fixtures of the WGSL self-tests, models/qwen3.js:3077-3157,
  including f32ToBf16 by truncation (qwen3.js:3072).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_lib = None
_ref = None

_P = ctypes.c_void_p
_I = ctypes.c_int64


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


def lib():
    global _lib
    if _lib is None:
        from . import build as _b
        _b.build()
        _lib = ctypes.CDLL(os.path.join(HERE, "liboracle.so"))
        _lib.tbo_f32_to_f16_js.restype = ctypes.c_uint16
        _lib.tbo_f32_to_f16_js.argtypes = [ctypes.c_float]
        _lib.tbo_f16_to_f64.restype = ctypes.c_double
        _lib.tbo_f16_to_f64.argtypes = [ctypes.c_uint16]
        _lib.tbo_dec_nsplit.restype = ctypes.c_int
        _lib.tbo_dec_nsplit.argtypes = [_I]
        _lib.tbo_argmax.restype = _I
        _lib.tbo_argmax.argtypes = [_P, _I]
    return _lib


def cpuref():
    """Transcribed CPU baseline (tb_cpu_ref.c)."""
    global _ref
    if _ref is None:
        from . import build as _b
        _b.build()
        _ref = ctypes.CDLL(os.path.join(HERE, "libcpuref.so"))
    return _ref


# --------------------------------------------------------------------------
# fixture generators (the reference's own)
# --------------------------------------------------------------------------

class XorShift64:
    """xorshift64 (13, 7, 17), returning the high 32 bits: tern.rs:356-365."""

    def __init__(self, seed):
        self.s = seed & 0xFFFFFFFFFFFFFFFF

    def next_u32(self):
        x = self.s
        x ^= (x << 13) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 7
        x ^= (x << 17) & 0xFFFFFFFFFFFFFFFF
        self.s = x
        return x >> 32

    def u32_array(self, n):
        """n successive next_u32() values, vectorised in blocks of 64k."""
        out = np.empty(n, np.uint64)
        s = self.s
        M = 0xFFFFFFFFFFFFFFFF
        for i in range(n):
            s ^= (s << 13) & M
            s ^= s >> 7
            s ^= (s << 17) & M
            out[i] = s >> 32
        self.s = s
        return out.astype(np.uint32)


_TERNARYISH = np.array([-1.0, 1.0, 0.0, 0.2, -0.9], np.float32)


def tern_fixture(n, k, seed):
    """(codes, scales, act, xsum) exactly as tern.rs:382-389 builds them."""
    rng = XorShift64(seed)
    u = rng.u32_array(n * k + k)
    w = _TERNARYISH[u[: n * k] % 5].reshape(n, k)
    codes, scales = pack_ternary(w)
    x = ((u[n * k:] % 2001).astype(np.float32) / np.float32(1000.0) - np.float32(1.0)).astype(np.float32)
    act, xsum, _ = quantize_act(x[None, :])
    return codes, scales, act[0], xsum[0], w, x


def f32_to_bf16_trunc(a):
    """f32ToBf16 of the self-tests: bits >> 16 (truncation), qwen3.js:3072."""
    a = np.ascontiguousarray(a, np.float32)
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def bf16_to_f32(u):
    return (np.ascontiguousarray(u, np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------
# int4 path
# --------------------------------------------------------------------------

def f32_to_f16_js(v):
    return lib().tbo_f32_to_f16_js(float(v))


def f16_to_f64(h):
    return lib().tbo_f16_to_f64(int(h))


def f16_bits_to_f64(h):
    """f16 bit patterns (any shape) -> exact float64 values."""
    return np.ascontiguousarray(h, np.uint16).view(np.float16).astype(np.float64)


def quant_int4_g32(w_bf16):
    w = np.ascontiguousarray(w_bf16, np.uint16)
    N, K = w.shape
    assert K % 32 == 0
    pack = np.zeros((N, K // 8), np.uint32)
    scales = np.zeros((N, K // 32), np.uint16)
    lib().tbo_quant_int4_g32(_ptr(w), _I(N), _I(K), _ptr(pack), _ptr(scales))
    return pack, scales


def dequant_int4_g32(pack, scales):
    N = pack.shape[0]
    K = pack.shape[1] * 8
    w = np.zeros((N, K), np.float32)
    lib().tbo_dequant_int4_g32(_ptr(np.ascontiguousarray(pack)), _ptr(np.ascontiguousarray(scales)),
                               _I(N), _I(K), _ptr(w))
    return w


def gemv_int4_f32act(x, pack, scales):
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    B, K = x.shape
    N = pack.shape[0]
    y = np.zeros((B, N), np.float64)
    lib().tbo_gemv_int4_f32act(_ptr(x), _ptr(np.ascontiguousarray(pack)), _ptr(np.ascontiguousarray(scales)),
                               _I(N), _I(K), _I(B), _ptr(y))
    return y


def gemm_int4_f16(x, pack, scales):
    """f16 prefill GEMM (gemmQ): x [M,K] f32 or bf16 bits (uint16) -> y [M,N] f64."""
    x = np.ascontiguousarray(x)
    bf16 = x.dtype == np.uint16
    if not bf16:
        x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    N = pack.shape[0]
    y = np.zeros((M, N), np.float64)
    lib().tbo_gemm_int4_f16(_ptr(x), ctypes.c_int(1 if bf16 else 0), _ptr(np.ascontiguousarray(pack)),
                            _ptr(np.ascontiguousarray(scales)), _I(M), _I(N), _I(K), _ptr(y))
    return y


def quant_q8(x):
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    T, K = x.shape
    xq = np.zeros((T, K), np.int8)
    xs = np.zeros((T, K // 32), np.float32)
    xsum = np.zeros((T, K // 16), np.int32)
    lib().tbo_quant_q8(_ptr(x), _I(T), _I(K), _ptr(xq), _ptr(xs), _ptr(xsum))
    return xq, xs, xsum


def rmsnorm_q8(x, w16, eps):
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    T, H = x.shape
    xq = np.zeros((T, H), np.int8)
    xs = np.zeros((T, H // 32), np.float32)
    xsum = np.zeros((T, H // 16), np.int32)
    inv = np.zeros(T, np.float32)
    lib().tbo_rmsnorm_q8(_ptr(x), _ptr(np.ascontiguousarray(w16, np.uint16)), _I(T), _I(H),
                         ctypes.c_float(eps), _ptr(xq), _ptr(xs), _ptr(xsum), _ptr(inv))
    return xq, xs, xsum, inv


def gemv_int4_q8act(xq, xs, pack, scales):
    xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
    xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
    B, K = xq.shape
    N = pack.shape[0]
    y = np.zeros((B, N), np.float64)
    lib().tbo_gemv_int4_q8act(_ptr(xq), _ptr(xs), _ptr(np.ascontiguousarray(pack)),
                              _ptr(np.ascontiguousarray(scales)), _I(N), _I(K), _I(B), _ptr(y))
    return y


def gateup_q8act(xq, xs, gpack, gscales, upack, uscales):
    xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
    xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
    B, H = xq.shape
    I = gpack.shape[0]
    y = np.zeros((B, I), np.float64)
    lib().tbo_gateup_q8act(_ptr(xq), _ptr(xs), _ptr(np.ascontiguousarray(gpack)),
                           _ptr(np.ascontiguousarray(gscales)), _ptr(np.ascontiguousarray(upack)),
                           _ptr(np.ascontiguousarray(uscales)), _I(I), _I(H), _I(B), _ptr(y))
    return y


# --------------------------------------------------------------------------
# ternary path
# --------------------------------------------------------------------------

def quant_tern_wgsl(w_bf16):
    """quantizeTernaryBf16 (qwen3.js:3435-3469): (pack u32 [N,K/16], scales f16 bits
    [N,K/32]) or None when not ternary."""
    w = np.ascontiguousarray(w_bf16, np.uint16)
    N, K = w.shape
    pack = np.zeros((N, max(K // 16, 1)), np.uint32)
    scales = np.zeros((N, max(K // 32, 1)), np.uint16)
    ok = lib().tbo_quant_tern_wgsl(_ptr(w), _I(N), _I(K), _ptr(pack), _ptr(scales))
    return (pack, scales) if ok else None


def gemv_tern_wgsl_q8act(xq, xs, pack, scales):
    """gemvTern2Wgsl (qwen3.js:449-503) in double over exact per-group int32 dots."""
    xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
    xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
    B, K = xq.shape
    N = pack.shape[0]
    y = np.zeros((B, N), np.float64)
    lib().tbo_gemv_tern_wgsl_q8act(_ptr(xq), _ptr(xs), _ptr(np.ascontiguousarray(pack, np.uint32)),
                                   _ptr(np.ascontiguousarray(scales, np.uint16)), _I(N), _I(K), _I(B), _ptr(y))
    return y


def gateup_tern_wgsl_q8act(xq, xs, gpack, gscales, upack, uscales):
    """gateupTern2Wgsl (qwen3.js:747-810): silu(g) * u in double."""
    xq = np.ascontiguousarray(np.atleast_2d(xq), np.int8)
    xs = np.ascontiguousarray(np.atleast_2d(xs), np.float32)
    B, H = xq.shape
    I = gpack.shape[0]
    y = np.zeros((B, I), np.float64)
    lib().tbo_gateup_tern_wgsl_q8act(_ptr(xq), _ptr(xs), _ptr(np.ascontiguousarray(gpack, np.uint32)),
                                     _ptr(np.ascontiguousarray(gscales, np.uint16)),
                                     _ptr(np.ascontiguousarray(upack, np.uint32)),
                                     _ptr(np.ascontiguousarray(uscales, np.uint16)), _I(I), _I(H), _I(B), _ptr(y))
    return y


def pack_ternary(w):
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    assert K % 64 == 0
    codes = np.zeros((N, K // 4), np.uint8)
    scales = np.zeros((N, K // 64), np.float32)
    lib().tbo_pack_ternary(_ptr(w), _I(N), _I(K), _ptr(codes), _ptr(scales))
    return codes, scales


def quantize_act(x):
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    T, K = x.shape
    act = np.zeros((T, K), np.int8)
    xsum = np.zeros((T, K // 64), np.int32)
    sc = np.zeros(T, np.float32)
    lib().tbo_quantize_act(_ptr(x), _I(T), _I(K), _ptr(act), _ptr(xsum), _ptr(sc))
    return act, xsum, sc


def quantize_act_wasm(x):
    """WASM quantize (cpu/kernel/src/lib.rs:566-606): returns (act, xsum, asc)."""
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    T, K = x.shape
    act = np.zeros((T, K), np.int8)
    xsum = np.zeros((T, K // 64), np.int32)
    asc = np.zeros(T, np.float32)
    lib().tbo_quantize_act_wasm(_ptr(x), _I(T), _I(K), _ptr(act), _ptr(xsum), _ptr(asc))
    return act, xsum, asc


def gemv_tern_scalar(codes, scales, act, xsum):
    act = np.ascontiguousarray(np.atleast_2d(act), np.int8)
    xsum = np.ascontiguousarray(np.atleast_2d(xsum), np.int32)
    B, K = act.shape
    N = codes.shape[0]
    out = np.zeros((B, N), np.float32)
    lib().tbo_gemv_tern_scalar(_ptr(out), _ptr(np.ascontiguousarray(codes)), _ptr(np.ascontiguousarray(scales)),
                               _ptr(act), _ptr(xsum), _I(N), _I(K), _I(B))
    return out


def gemv_tern_dequant(codes, scales, act):
    act = np.ascontiguousarray(np.atleast_2d(act), np.int8)
    B, K = act.shape
    N = codes.shape[0]
    out = np.zeros((B, N), np.float32)
    lib().tbo_gemv_tern_dequant(_ptr(out), _ptr(np.ascontiguousarray(codes)), _ptr(np.ascontiguousarray(scales)),
                                _ptr(act), _I(N), _I(K), _I(B))
    return out


def gemv_tern_scalar_timed(codes, scales, act, xsum, threads=1):
    """The transcribed scalar backend (tern.rs:100-140) of the timed CPU
    baseline, built -O3; single activation row."""
    N = codes.shape[0]
    K = act.shape[-1]
    out = np.zeros(N, np.float32)
    cpuref().tbr_gemv_tern_scalar(_ptr(out), _ptr(np.ascontiguousarray(codes)), _ptr(np.ascontiguousarray(scales)),
                                  _ptr(np.ascontiguousarray(act, np.int8)), _ptr(np.ascontiguousarray(xsum, np.int32)),
                                  _I(N), _I(K), ctypes.c_int(threads))
    return out


def gemv_tern_avx2(codes, scales, act, xsum, threads=1):
    """The transcribed AVX2 backend (tern.rs:268-338), single activation row."""
    N = codes.shape[0]
    K = act.shape[-1]
    out = np.zeros(N, np.float32)
    cpuref().tbr_gemv_tern_avx2(_ptr(out), _ptr(np.ascontiguousarray(codes)), _ptr(np.ascontiguousarray(scales)),
                                _ptr(np.ascontiguousarray(act, np.int8)), _ptr(np.ascontiguousarray(xsum, np.int32)),
                                _I(N), _I(K), ctypes.c_int(threads))
    return out


# --------------------------------------------------------------------------
# attention
# --------------------------------------------------------------------------

def kv_quant_q8(x):
    x = np.ascontiguousarray(x, np.float32)
    n = x.size
    q = np.zeros(n, np.int8)
    s = np.zeros(n // 32, np.float32)
    lib().tbo_kv_quant_q8(_ptr(x), _I(n), _ptr(q), _ptr(s))
    return q.reshape(x.shape), s


def head_norm_rope(x, w16, pos, theta=1e6, eps=1e-6):
    """x [nH, hd] -> per-head RMSNorm(w16) + RoPE split-half at `pos` (f64)."""
    x = np.array(x, np.float64, copy=True, order="C")
    nH, hd = x.shape
    lib().tbo_head_norm_rope(_ptr(x), _ptr(np.ascontiguousarray(w16, np.uint16)), _I(nH), _I(hd),
                             _I(pos), ctypes.c_double(theta), ctypes.c_double(eps))
    return x


def attn_decode_q8(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd):
    out = np.zeros(nHq * hd, np.float64)
    lib().tbo_attn_decode_q8(_ptr(np.ascontiguousarray(q, np.float32)), _ptr(np.ascontiguousarray(Kq, np.int8)),
                             _ptr(np.ascontiguousarray(Ks, np.float32)), _ptr(np.ascontiguousarray(Vq, np.int8)),
                             _ptr(np.ascontiguousarray(Vs, np.float32)), _I(S), _I(nHq), _I(nKv), _I(hd), _ptr(out))
    return out


def attn_decode_q8_f16ops(q, Kq, Ks, Vq, Vs, S, nHq, nKv, hd):
    """decode attention at the reference's f16 prefill-kernel operand precision (q, K, V, p in f16)."""
    out = np.zeros(nHq * hd, np.float64)
    lib().tbo_attn_decode_q8_f16ops(_ptr(np.ascontiguousarray(q, np.float32)), _ptr(np.ascontiguousarray(Kq, np.int8)),
                                    _ptr(np.ascontiguousarray(Ks, np.float32)), _ptr(np.ascontiguousarray(Vq, np.int8)),
                                    _ptr(np.ascontiguousarray(Vs, np.float32)), _I(S), _I(nHq), _I(nKv), _I(hd),
                                    _ptr(out))
    return out


def attn_prefill_q8(q, Kq, Ks, Vq, Vs, T, S, nHq, nKv, hd):
    """attentionQ8 at T > 1 (qwen3.js:2534-2577), causal over the int8 cache, in double."""
    out = np.zeros((T, nHq * hd), np.float64)
    lib().tbo_attn_prefill_q8(_ptr(np.ascontiguousarray(q, np.float32)), _ptr(np.ascontiguousarray(Kq, np.int8)),
                              _ptr(np.ascontiguousarray(Ks, np.float32)), _ptr(np.ascontiguousarray(Vq, np.int8)),
                              _ptr(np.ascontiguousarray(Vs, np.float32)), _I(T), _I(S), _I(nHq), _I(nKv), _I(hd),
                              _ptr(out))
    return out


def gumbel_noise(total, seed, temp):
    """GUMBEL_WGSL noise (qwen3.js:2719-2730) of flat indices 0..total-1, in double."""
    out = np.zeros(total, np.float64)
    lib().tbo_gumbel_noise(_I(total), ctypes.c_uint32(seed & 0xFFFFFFFF), ctypes.c_double(temp), _ptr(out))
    return out


def dec_nsplit(S):
    return lib().tbo_dec_nsplit(int(S))


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().tbo_argmax(_ptr(x), _I(x.size)))


# --------------------------------------------------------------------------
# int3 MoE (lfm25.js)
# --------------------------------------------------------------------------

def requant43(pack4, s4):
    """_requant43: int4 pack [rows][K/8] + f16 scales -> int3 planes [rows][K/32][3], f16 scales."""
    pack4 = np.ascontiguousarray(pack4, np.uint32)
    rows, K = pack4.shape[0], pack4.shape[1] * 8
    p3 = np.zeros((rows, K // 32, 3), np.uint32)
    s3 = np.zeros((rows, K // 32), np.uint16)
    lib().tbo_requant43(_ptr(pack4), _ptr(np.ascontiguousarray(s4, np.uint16)), _I(rows), _I(K), _ptr(p3), _ptr(s3))
    return p3, s3


def engine_f32_to_f16(v):
    lib().tbo_engine_f32_to_f16.restype = ctypes.c_uint16
    return lib().tbo_engine_f32_to_f16(ctypes.c_float(v))


def moe_router(logits, bias, K):
    logits = np.ascontiguousarray(logits, np.float32)
    T, nE = logits.shape
    idx = np.zeros((T, K), np.uint32)
    wt = np.zeros((T, K), np.float32)
    lib().tbo_moe_router(_ptr(logits), _ptr(np.ascontiguousarray(bias, np.float32)), _I(T), _I(nE), _I(K),
                         _ptr(idx), _ptr(wt))
    return idx, wt


def moe_ffn_int3(a, idx, wt, w1, w3, w2, H, I, group=32):
    """sum_k wt * W2_e(silu(W1_e a) * W3_e a) per token (f64); w* = (planes, scales);
    group: weights per f16 scale (32 or 128)."""
    a = np.ascontiguousarray(a, np.float32)
    T = a.shape[0]
    K = idx.shape[1]
    out = np.zeros((T, H), np.float64)
    c = lambda t: np.ascontiguousarray(t)  # noqa: E731
    w1, w3, w2 = [(c(p), c(s)) for p, s in (w1, w3, w2)]
    lib().tbo_moe_ffn_int3_g(_ptr(a), _ptr(np.ascontiguousarray(idx, np.uint32)),
                             _ptr(np.ascontiguousarray(wt, np.float32)),
                             _ptr(w1[0]), _ptr(w1[1]), _ptr(w3[0]), _ptr(w3[1]), _ptr(w2[0]), _ptr(w2[1]),
                             _I(T), _I(K), _I(H), _I(I), _I(group), _ptr(out))
    return out


def quant_int3(w, group):
    """bf16 bits [rows, K] -> int3 planes [rows][K/32][3], f16 scales [rows][K/group]."""
    w = np.ascontiguousarray(w, np.uint16)
    rows, K = w.shape
    p3 = np.zeros((rows, K // 32, 3), np.uint32)
    s3 = np.zeros((rows, K // group), np.uint16)
    lib().tbo_quant_int3(_ptr(w), _I(rows), _I(K), _I(group), _ptr(p3), _ptr(s3))
    return p3, s3
