"""Host-side operator mirror over the C ABI.

Each function follows one reference operator (cited) with the same argument
meaning; device buffers are torch CUDA tensors (contiguous), outputs are
allocated when not supplied.  Every call is ordered on the current torch
stream of the tensor's device.  Shape/alignment errors raise TabInferError
with the library's message (the reference throws / panics).
"""
import ctypes
import threading

import torch

from ._lib import LIB, P

TB_ACT_F32, TB_ACT_Q8 = 0, 1
CUDA_STREAM_LEGACY = 0x1   # cudaStreamLegacy


class TabInferError(RuntimeError):
    pass


class Context:
    """One tb_ctx per (host thread, device): replaces the engine handle of
    engine/webgpu-engine.js:72 and the module scratch of models/qwen3.js."""

    def __init__(self, device=0):
        h = P()
        rc = LIB.tb_ctx_create(int(device), ctypes.byref(h))
        if rc != 0:
            raise TabInferError("tb_ctx_create(%d) failed with status %d" % (device, rc))
        self.h = h
        self.device = int(device)

    def check(self, rc, what):
        if rc != 0:
            msg = LIB.tb_last_error(self.h)
            raise TabInferError("%s: status %d: %s" % (what, rc, msg.decode() if msg else ""))

    def bind_stream(self):
        """Order the library's work on torch's current stream.  torch reports its
        default (legacy NULL) stream as handle 0, which the C ABI reads as "the
        context's own stream", so it is passed as cudaStreamLegacy (0x1)."""
        s = torch.cuda.current_stream(self.device).cuda_stream
        LIB.tb_ctx_set_stream(self.h, P(s if s else CUDA_STREAM_LEGACY))

    def own_stream(self):
        """Handle of the context's own (non-blocking) stream; binds it."""
        LIB.tb_ctx_set_stream(self.h, None)
        return LIB.tb_ctx_get_stream(self.h)

    def set_pdl(self, on):
        LIB.tb_ctx_set_pdl(self.h, 1 if on else 0)

    def synchronize(self):
        self.check(LIB.tb_ctx_synchronize(self.h), "synchronize")

    def device_error(self):
        code = ctypes.c_int(0)
        LIB.tb_ctx_device_error(self.h, ctypes.byref(code))
        return code.value

    def close(self):
        if self.h:
            LIB.tb_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_tls = threading.local()


def default_context(device=None):
    if device is None:
        device = torch.cuda.current_device()
    device = int(device)
    ctxs = getattr(_tls, "ctxs", None)
    if ctxs is None:
        ctxs = _tls.ctxs = {}
    c = ctxs.get(device)
    if c is None:
        c = ctxs[device] = Context(device)
    c.bind_stream()
    return c


def _p(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise TabInferError("tensor must be on a CUDA device")
    if not t.is_contiguous():
        raise TabInferError("tensor must be contiguous")
    return P(t.data_ptr())


def _ctx(t):
    return default_context(t.device.index)


def _u16(t):
    """bf16 / f16 tensors are passed as their 16-bit patterns."""
    return t


# --------------------------------------------------------------------------
# int4 G=32 path (models/qwen3.js)
# --------------------------------------------------------------------------

def quantize_int4_bf16(w, pack=None, scales=None):
    """quantizeInt4Bf16 (qwen3.js:3405-3426): bf16 [N,K] -> (pack u32 [N,K/8] as int32, scales f16 [N,K/32])."""
    N, K = w.shape
    if pack is None:
        pack = torch.empty((N, K // 8), dtype=torch.int32, device=w.device)
    if scales is None:
        scales = torch.empty((N, K // 32), dtype=torch.float16, device=w.device)
    c = _ctx(w)
    c.check(LIB.tb_quant_int4_g32(c.h, _p(w), _p(pack), _p(scales), N, K), "quant_int4_g32")
    return pack, scales


def convert_bf16_f16(w, out=None):
    """bf16ToF16bits (qwen3.js:3386-3390): the loader's f16 copy of a non-projection tensor."""
    out = out if out is not None else torch.empty(w.shape, dtype=torch.int16, device=w.device)
    c = _ctx(w)
    c.check(LIB.tb_convert_bf16_f16(c.h, _p(w.contiguous()), _p(out), w.numel()), "convert_bf16_f16")
    return out


def quant_q8(x, xq=None, xs=None, xsum16=None):
    """quantQ8 / QUANTQ8T (qwen3.js:332-358, 1210-1231): f32 [T,K] -> int8, per-32 scales, per-16 sums."""
    x2 = x.reshape(-1, x.shape[-1])
    T, K = x2.shape
    xq = xq if xq is not None else torch.empty((T, K), dtype=torch.int8, device=x.device)
    xs = xs if xs is not None else torch.empty((T, K // 32), dtype=torch.float32, device=x.device)
    xsum16 = xsum16 if xsum16 is not None else torch.empty((T, K // 16), dtype=torch.int32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_quant_q8(c.h, _p(x2), _p(xq), _p(xs), _p(xsum16), T, K), "quant_q8")
    return xq, xs, xsum16


def rmsnorm_q8(x, w16, eps, xq=None, xs=None, xsum16=None):
    """rmsnormQ (qwen3.js:569-621): fused RMSNorm -> per-32 int8."""
    x2 = x.reshape(-1, x.shape[-1])
    T, H = x2.shape
    xq = xq if xq is not None else torch.empty((T, H), dtype=torch.int8, device=x.device)
    xs = xs if xs is not None else torch.empty((T, H // 32), dtype=torch.float32, device=x.device)
    xsum16 = xsum16 if xsum16 is not None else torch.empty((T, H // 16), dtype=torch.int32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_rmsnorm_q8(c.h, _p(x2), _p(w16), float(eps), _p(xq), _p(xs), _p(xsum16), T, H), "rmsnorm_q8")
    return xq, xs, xsum16


def gemv_dp4(xq, xs, pack, scales, y=None, acc=False):
    """gemvDP4_only (qwen3.js:422-427): int8-activation GEMV, batch = xq rows."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    B, K = xq2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((B, N), dtype=torch.float32, device=xq.device)
    c = _ctx(xq)
    c.check(LIB.tb_gemv_int4_q8(c.h, _p(y), _p(xq2), _p(xs), _p(pack), _p(scales), N, K, B, 1 if acc else 0),
            "gemv_int4_q8")
    return y


def gemv_dp4_multi(xq, xs, mats, ys=None, acc=False):
    """q/k/v projGemv triple on one quantized activation (qwen3.js:3981-3984), one launch.
    mats: list of (pack, scales)."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    B, K = xq2.shape
    n = len(mats)
    if ys is None:
        ys = [torch.zeros((B, p.shape[0]), dtype=torch.float32, device=xq.device) for p, _ in mats]
    arr_y = (P * n)(*[y.data_ptr() for y in ys])
    arr_p = (P * n)(*[p.data_ptr() for p, _ in mats])
    arr_s = (P * n)(*[s.data_ptr() for _, s in mats])
    arr_n = (ctypes.c_int64 * n)(*[p.shape[0] for p, _ in mats])
    c = _ctx(xq)
    c.check(LIB.tb_gemv_int4_q8_multi(c.h, n, ctypes.cast(arr_y, P), ctypes.cast(arr_p, P), ctypes.cast(arr_s, P),
                                      ctypes.cast(arr_n, P), _p(xq2), _p(xs), K, B, 1 if acc else 0),
            "gemv_int4_q8_multi")
    return ys


def gemv_dp4a(x, pack, scales, norm_w=None, eps=1e-6, y=None, acc=False):
    """gemvDP4A (qwen3.js:428-431): quantQ8 + gemvDP4 in one launch; with norm_w it is
    rmsnormQ + gemvDP4_only (forward, qwen3.js:3981-3984)."""
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((B, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_gemv_int4_dp4a(c.h, _p(y), _p(x2), _p(norm_w), float(eps), _p(pack), _p(scales), N, K, B,
                                  1 if acc else 0), "gemv_int4_dp4a")
    return y


def gemv_dp4a_multi(x, mats, norm_w=None, eps=1e-6, ys=None, acc=False):
    """rmsnormQ + q/k/v projGemv (qwen3.js:3981-3984) in one launch.  mats: [(pack, scales)]."""
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    n = len(mats)
    if ys is None:
        ys = [torch.zeros((B, p.shape[0]), dtype=torch.float32, device=x.device) for p, _ in mats]
    arr_y = (P * n)(*[y.data_ptr() for y in ys])
    arr_p = (P * n)(*[p.data_ptr() for p, _ in mats])
    arr_s = (P * n)(*[s.data_ptr() for _, s in mats])
    arr_n = (ctypes.c_int64 * n)(*[p.shape[0] for p, _ in mats])
    c = _ctx(x)
    c.check(LIB.tb_gemv_int4_dp4a_multi(c.h, n, ctypes.cast(arr_y, P), ctypes.cast(arr_p, P), ctypes.cast(arr_s, P),
                                        ctypes.cast(arr_n, P), _p(x2), _p(norm_w), float(eps), K, B,
                                        1 if acc else 0), "gemv_int4_dp4a_multi")
    return ys


def gate_up_silu_dp4a(x, gpack, gscales, upack, uscales, norm_w=None, eps=1e-6, swi=None):
    """rmsnormQ + gateUpSiluDP4_only (qwen3.js:4023-4024) in one launch."""
    x2 = x.reshape(-1, x.shape[-1])
    B, Hd = x2.shape
    I = gpack.shape[0]
    if swi is None:
        swi = torch.empty((B, I), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_gateup_silu_int4_dp4a(c.h, _p(swi), _p(x2), _p(norm_w), float(eps), _p(gpack), _p(gscales),
                                         _p(upack), _p(uscales), I, Hd, B), "gateup_silu_int4_dp4a")
    return swi


def gemv_mma(x, pack, scales, norm_w=None, eps=1e-6, y=None, acc=False, tern=False):
    """linearQ's T > 1 DP4A route (qwen3.js:1600-1607) at 2..16 rows on the tensor
    cores, every weight read once: y (+)= W . quantQ8(rmsnorm?(x)); int4 G32 weights,
    or the ternary WebGPU layout with tern=True."""
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((B, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    fn = LIB.tb_gemv_tern_wgsl_mma if tern else LIB.tb_gemv_int4_mma
    c.check(fn(c.h, _p(y), _p(x2), _p(norm_w), float(eps), _p(pack), _p(scales), N, K, B, 1 if acc else 0),
            "gemv_mma")
    return y


def gemv_mma_multi(x, mats, norm_w=None, eps=1e-6, ys=None, acc=False):
    """rmsnormQ + the q/k/v projGemv triple (qwen3.js:3981-3984) at 2..16 rows on the
    tensor cores: one quantization, one launch.  mats: [(pack, scales)] (<= 3)."""
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    n = len(mats)
    if ys is None:
        ys = [torch.zeros((B, p.shape[0]), dtype=torch.float32, device=x.device) for p, _ in mats]
    arr_y = (P * n)(*[y.data_ptr() for y in ys])
    arr_p = (P * n)(*[p.data_ptr() for p, _ in mats])
    arr_s = (P * n)(*[s.data_ptr() for _, s in mats])
    arr_n = (ctypes.c_int64 * n)(*[p.shape[0] for p, _ in mats])
    c = _ctx(x)
    c.check(LIB.tb_gemv_int4_mma_multi(c.h, n, ctypes.cast(arr_y, P), ctypes.cast(arr_p, P), ctypes.cast(arr_s, P),
                                       ctypes.cast(arr_n, P), _p(x2), _p(norm_w), float(eps), K, B,
                                       1 if acc else 0), "gemv_mma_multi")
    return ys


def gate_up_silu_mma(x, gpack, gscales, upack, uscales, norm_w=None, eps=1e-6, swi=None, tern=False):
    """rmsnormQ + gate/up + silu(gate) * up at 2..16 rows on the tensor cores."""
    x2 = x.reshape(-1, x.shape[-1])
    B, Hd = x2.shape
    I = gpack.shape[0]
    if swi is None:
        swi = torch.empty((B, I), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    fn = LIB.tb_gateup_silu_tern_wgsl_mma if tern else LIB.tb_gateup_silu_int4_mma
    c.check(fn(c.h, _p(swi), _p(x2), _p(norm_w), float(eps), _p(gpack), _p(gscales), _p(upack), _p(uscales), I, Hd,
               B), "gateup_silu_mma")
    return swi


def gemm_q(x, pack, scales, y=None, acc=False):
    """Prefill GEMM on the tensor cores: y[M,N] (+)= f16(x) . f16(deq(W))^T
    (gemmQ, qwen3.js:964-1026).  x [M,K] f32 or bf16."""
    x2 = x.reshape(-1, x.shape[-1])
    M, K = x2.shape
    N = pack.shape[0]
    y = y if y is not None else torch.zeros((M, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_gemm_int4_g32(c.h, _p(y), _p(x2), 1 if x2.dtype == torch.bfloat16 else 0, _p(pack), _p(scales),
                                 M, N, K, 1 if acc else 0), "gemm_int4_g32")
    return y


def requant_int3(pack4, scales4):
    """_requant43 (lfm25.js:833-855): int4 G32 -> int3 bitplanes [rows][K/32][3] + f16 scales."""
    rows, K = pack4.shape[0], pack4.shape[1] * 8
    p3 = torch.empty((rows, K // 32, 3), dtype=torch.int32, device=pack4.device)
    s3 = torch.empty((rows, K // 32), dtype=torch.int16, device=pack4.device)
    c = _ctx(pack4)
    c.check(LIB.tb_requant_int4_int3(c.h, _p(p3), _p(s3), _p(pack4), _p(scales4), rows, K), "requant_int4_int3")
    return p3, s3


def moe_router(logits, bias, K):
    """ROUTER_WGSL (lfm25.js:111-141) -> (idx [T,K] int32, wt [T,K] f32)."""
    T, nE = logits.shape
    idx = torch.empty((T, K), dtype=torch.int32, device=logits.device)
    wt = torch.empty((T, K), dtype=torch.float32, device=logits.device)
    c = _ctx(logits)
    c.check(LIB.tb_moe_router(c.h, _p(idx), _p(wt), _p(logits), _p(bias), T, nE, K), "moe_router")
    return idx, wt


def moe_ffn_int3(x_out, x_in, idx, wt, w1, w3, w2, n_experts, hidden, inter, group=32):
    """x_out += sum_k wt * W2_e(silu(W1_e x_in) * W3_e x_in); w* = (planes, scales);
    group: weights per f16 scale (32, the reference's layout, or 128)."""
    T, K = idx.shape
    c = _ctx(x_in)
    c.check(LIB.tb_moe_ffn_int3_g(c.h, _p(x_out), _p(x_in), _p(idx), _p(wt), _p(w1[0]), _p(w1[1]), _p(w3[0]),
                                  _p(w3[1]), _p(w2[0]), _p(w2[1]), T, K, n_experts, hidden, inter, int(group)),
            "moe_ffn_int3")
    return x_out


def quant_int3(w, group=128):
    """bf16 [rows, K] -> int3 planes [rows][K/32][3] + f16 scales [rows][K/group]
    (scale = f16(max|w|/4), q = clamp(rn(w/scale), -4, 3))."""
    rows, K = w.shape
    p3 = torch.empty((rows, K // 32, 3), dtype=torch.int32, device=w.device)
    s3 = torch.empty((rows, K // group), dtype=torch.int16, device=w.device)
    c = _ctx(w)
    c.check(LIB.tb_quant_int3_bf16(c.h, _p(w), _p(p3), _p(s3), rows, K, int(group)), "quant_int3_bf16")
    return p3, s3


def gemv_q_norm(x, norm_w, eps, pack, scales, y=None, acc=False):
    """rmsnorm + gemvQ (the final norm + lm_head of forward, qwen3.js:4037-4049) in one launch."""
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((B, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_gemv_int4_f32_norm(c.h, _p(y), _p(x2), _p(norm_w), float(eps), _p(pack), _p(scales), N, K, B,
                                      1 if acc else 0), "gemv_int4_f32_norm")
    return y


def gemv_q(x, pack, scales, y=None, acc=False):
    """gemvQ (qwen3.js:314-321): f32-activation int4 GEMV, batch = x rows."""
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((B, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_gemv_int4_f32(c.h, _p(y), _p(x2), _p(pack), _p(scales), N, K, B, 1 if acc else 0),
            "gemv_int4_f32")
    return y


def linear_q(x, pack, scales, y=None, acc=False):
    """linearQ (qwen3.js:1588-1608) for T = x rows (1..8)."""
    x2 = x.reshape(-1, x.shape[-1])
    T, K = x2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((T, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_linear_int4(c.h, _p(y), _p(x2), _p(pack), _p(scales), T, N, K, 1 if acc else 0), "linear_int4")
    return y


def gate_up_silu_dp4(xq, xs, gpack, gscales, upack, uscales, swi=None):
    """gateUpSiluDP4_only (qwen3.js:861-877): swi = silu(W_g x) * (W_u x)."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    B, H = xq2.shape
    I = gpack.shape[0]
    if swi is None:
        swi = torch.empty((B, I), dtype=torch.float32, device=xq.device)
    c = _ctx(xq)
    c.check(LIB.tb_gateup_silu_int4_q8(c.h, _p(swi), _p(xq2), _p(xs), _p(gpack), _p(gscales), _p(upack),
                                       _p(uscales), I, H, B), "gateup_silu_int4_q8")
    return swi


# --------------------------------------------------------------------------
# ternary, WebGPU layout (models/qwen3.js): pack u32 [N,K/16], f16 scales [N,K/32]
# --------------------------------------------------------------------------

def quantize_tern_bf16(w):
    """quantizeTernaryBf16 (qwen3.js:3435-3469): bf16 [N,K] -> (pack int32 [N,K/16],
    scales f16 [N,K/32]), or None when the matrix is not ternary (the reference's
    null, after which its loader quantizes to int4).  Synchronises to read the flag."""
    N, K = w.shape
    pack = torch.empty((N, max(K // 16, 1)), dtype=torch.int32, device=w.device)
    scales = torch.empty((N, max(K // 32, 1)), dtype=torch.float16, device=w.device)
    flag = torch.empty(1, dtype=torch.int32, device=w.device)
    c = _ctx(w)
    c.check(LIB.tb_quant_tern_wgsl_bf16(c.h, _p(w), _p(pack), _p(scales), N, K, _p(flag)), "quant_tern_wgsl_bf16")
    if int(flag.item()) != 0:
        return None
    return pack, scales


def gemv_tern_wgsl(xq, xs, pack, scales, y=None, acc=False):
    """gemvTern_only (qwen3.js:548-556) against a QUANTQ8 activation; batch = xq rows."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    B, K = xq2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((B, N), dtype=torch.float32, device=xq.device)
    c = _ctx(xq)
    c.check(LIB.tb_gemv_tern_wgsl_q8(c.h, _p(y), _p(xq2), _p(xs), _p(pack), _p(scales), N, K, B, 1 if acc else 0),
            "gemv_tern_wgsl_q8")
    return y


def gemv_tern_wgsl_dp4a_multi(x, mats, norm_w=None, eps=1e-6, ys=None, acc=False):
    """quantQ8 (or rmsnormQ) + projGemv of ternary q/k/v (qwen3.js:558-561, 3981-3984),
    one launch.  mats: [(pack, scales)]."""
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    n = len(mats)
    if ys is None:
        ys = [torch.zeros((B, p.shape[0]), dtype=torch.float32, device=x.device) for p, _ in mats]
    arr_y = (P * n)(*[y.data_ptr() for y in ys])
    arr_p = (P * n)(*[p.data_ptr() for p, _ in mats])
    arr_s = (P * n)(*[s.data_ptr() for _, s in mats])
    arr_n = (ctypes.c_int64 * n)(*[p.shape[0] for p, _ in mats])
    c = _ctx(x)
    c.check(LIB.tb_gemv_tern_wgsl_dp4a_multi(c.h, n, ctypes.cast(arr_y, P), ctypes.cast(arr_p, P),
                                             ctypes.cast(arr_s, P), ctypes.cast(arr_n, P), _p(x2), _p(norm_w),
                                             float(eps), K, B, 1 if acc else 0), "gemv_tern_wgsl_dp4a_multi")
    return ys


def gate_up_silu_tern(xq, xs, gpack, gscales, upack, uscales, swi=None):
    """gateUpSiluDP4_only's ternary branch (qwen3.js:861-870, gateupTern2Wgsl :747-810)."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    B, H = xq2.shape
    I = gpack.shape[0]
    if swi is None:
        swi = torch.empty((B, I), dtype=torch.float32, device=xq.device)
    c = _ctx(xq)
    c.check(LIB.tb_gateup_silu_tern_wgsl_q8(c.h, _p(swi), _p(xq2), _p(xs), _p(gpack), _p(gscales), _p(upack),
                                            _p(uscales), I, H, B), "gateup_silu_tern_wgsl_q8")
    return swi


def gate_up_silu_tern_dp4a(x, gpack, gscales, upack, uscales, norm_w=None, eps=1e-6, swi=None):
    """gateUpSiluQ's ternary branch (qwen3.js:730): quantQ8 (or rmsnormQ) + gateupTern2, one launch."""
    x2 = x.reshape(-1, x.shape[-1])
    B, H = x2.shape
    I = gpack.shape[0]
    if swi is None:
        swi = torch.empty((B, I), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_gateup_silu_tern_wgsl_dp4a(c.h, _p(swi), _p(x2), _p(norm_w), float(eps), _p(gpack),
                                              _p(gscales), _p(upack), _p(uscales), I, H, B),
            "gateup_silu_tern_wgsl_dp4a")
    return swi


def attention_prefill_q8(q, kv, S, nHq, nKv, hd, out=None):
    """attentionQ8 at T > 1 (qwen3.js:2534-2577): q [T, nHq*hd] after norm+RoPE at
    positions S-T .. S-1, causal over the int8 cache kv = (Kq, Ks, Vq, Vs)."""
    q2 = q.reshape(-1, nHq * hd)
    T = q2.shape[0]
    Kq, Ks, Vq, Vs = kv
    out = out if out is not None else torch.empty((T, nHq * hd), dtype=torch.float32, device=q.device)
    c = _ctx(q)
    c.check(LIB.tb_attn_prefill_q8(c.h, _p(out), _p(q2), _p(Kq), _p(Ks), _p(Vq), _p(Vs), T, S, nHq, nKv, hd),
            "attn_prefill_q8")
    return out


def gemm_dp4(xq, xs, pack, scales, y=None, epilogue=0, tern=False, warp=False):
    """gemmDP4A / gemmTern (qwen3.js:1321-1420) with exact per-group int8 sums, from
    QUANTQ8T rows.  epilogue 0: y =, 1: y +=, 2: y = silu(y) * (X W^T).  The
    tcgen05 kind::i8 kernel; warp=True runs the warp-level mma.sync form of the
    same arithmetic (bit-equal outputs)."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    M, K = xq2.shape
    N = pack.shape[0]
    y = y if y is not None else torch.zeros((M, N), dtype=torch.float32, device=xq.device)
    c = _ctx(xq)
    fn = LIB.tb_gemm_dp4_warp if warp else LIB.tb_gemm_dp4
    c.check(fn(c.h, _p(y), _p(xq2), _p(xs), _p(pack), _p(scales), M, N, K, int(epilogue), 1 if tern else 0),
            "gemm_dp4_warp" if warp else "gemm_dp4")
    return y


def gemm_dp4_f16(xq, xs, pack, scales, y=None, epilogue=0):
    """gemmDP4A's data flow on tcgen05 with f16 operands f16(xs*q) and f16((nib-8)*s)."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    M, K = xq2.shape
    N = pack.shape[0]
    y = y if y is not None else torch.zeros((M, N), dtype=torch.float32, device=xq.device)
    c = _ctx(xq)
    c.check(LIB.tb_gemm_int4_q8(c.h, _p(y), _p(xq2), _p(xs), _p(pack), _p(scales), M, N, K, int(epilogue)),
            "gemm_int4_q8")
    return y


def gemm_tern(xq, xs, pack, scales, y=None, acc=False):
    """gemmTern (qwen3.js:1410-1420) on the tensor cores from QUANTQ8T rows:
    y[M,N] (+)= f16(xs*xq) . f16((c-1)*s)^T."""
    xq2 = xq.reshape(-1, xq.shape[-1])
    M, K = xq2.shape
    N = pack.shape[0]
    y = y if y is not None else torch.zeros((M, N), dtype=torch.float32, device=xq.device)
    c = _ctx(xq)
    c.check(LIB.tb_gemm_tern_wgsl(c.h, _p(y), _p(xq2), _p(xs), _p(pack), _p(scales), M, N, K, 1 if acc else 0),
            "gemm_tern_wgsl")
    return y


def linear_tern_wgsl(x, pack, scales, y=None, acc=False):
    """linearQ for a ternary weight record (qwen3.js:1594-1598), T = x rows."""
    x2 = x.reshape(-1, x.shape[-1])
    T, K = x2.shape
    N = pack.shape[0]
    if y is None:
        y = torch.zeros((T, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_linear_tern_wgsl(c.h, _p(y), _p(x2), _p(pack), _p(scales), T, N, K, 1 if acc else 0),
            "linear_tern_wgsl")
    return y


# --------------------------------------------------------------------------
# ternary Q2_0_g64 (native/crates/n2-kernels/src/tern.rs)
# --------------------------------------------------------------------------

def pack_ternary(w, codes=None, scales=None):
    """tern::pack_ternary (tern.rs:131-160): f32 [N,K] -> codes u8 [N,K/4], scales f32 [N,K/64]."""
    N, K = w.shape
    codes = codes if codes is not None else torch.empty((N, K // 4), dtype=torch.uint8, device=w.device)
    scales = scales if scales is not None else torch.empty((N, K // 64), dtype=torch.float32, device=w.device)
    c = _ctx(w)
    c.check(LIB.tb_pack_tern_q2g64(c.h, _p(w), _p(codes), _p(scales), N, K), "pack_tern_q2g64")
    return codes, scales


def quantize_act(x, act=None, xsum=None, scale=None):
    """tern::quantize_act (tern.rs:196-222): returns (act i8, xsum i32 per 64, scale per row)."""
    x2 = x.reshape(-1, x.shape[-1])
    T, K = x2.shape
    act = act if act is not None else torch.empty((T, K), dtype=torch.int8, device=x.device)
    xsum = xsum if xsum is not None else torch.empty((T, K // 64), dtype=torch.int32, device=x.device)
    scale = scale if scale is not None else torch.empty((T,), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_quant_act_q8(c.h, _p(x2), _p(act), _p(xsum), _p(scale), T, K), "quant_act_q8")
    return act, xsum, scale


def quantize_wasm(x, dst=None, xsum=None, asc=None):
    """WASM quantize(dst, xsum, x, k) -> asc (cpu/kernel/src/lib.rs:566-606), per
    row of x: returns (dst i8, xsum i32 per 64, asc f32 per row)."""
    x2 = x.reshape(-1, x.shape[-1])
    T, K = x2.shape
    dst = dst if dst is not None else torch.empty((T, K), dtype=torch.int8, device=x.device)
    xsum = xsum if xsum is not None else torch.empty((T, K // 64), dtype=torch.int32, device=x.device)
    asc = asc if asc is not None else torch.empty((T,), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_quantize_wasm(c.h, _p(dst), _p(xsum), _p(x2), K, _p(asc), T), "quantize_wasm")
    return dst, xsum, asc


def gemv_tern(codes, scales, act, xsum, out=None):
    """tern::gemv_tern (tern.rs:56-71) / WASM gemm_tern_b4 (lib.rs:331): batch = act rows."""
    a2 = act.reshape(-1, act.shape[-1])
    B, K = a2.shape
    N = codes.shape[0]
    out = out if out is not None else torch.empty((B, N), dtype=torch.float32, device=act.device)
    c = _ctx(act)
    c.check(LIB.tb_gemv_tern_q2g64(c.h, _p(out), _p(codes), _p(scales), _p(a2), _p(xsum), N, K, B), "gemv_tern_q2g64")
    return out


def linear_tern(x, codes, scales, y=None):
    """Model::linear (model.rs:316-339): quantize_act -> gemv_tern -> *= 1/scale."""
    x2 = x.reshape(-1, x.shape[-1])
    T, K = x2.shape
    N = codes.shape[0]
    y = y if y is not None else torch.empty((T, N), dtype=torch.float32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_linear_tern(c.h, _p(y), _p(x2), _p(codes), _p(scales), T, N, K), "linear_tern")
    return y


# --------------------------------------------------------------------------
# int8 KV attention (qwen3.js:2048-2308)
# --------------------------------------------------------------------------

def attn_prep_q8(q, k, v, qw16, kw16, kv, nHq, nKv, hd, pos, theta, eps, qr=None):
    """attnPrepQ8 (qwen3.js:2297-2308). kv = (Kq, Ks, Vq, Vs) cache tensors."""
    qr = qr if qr is not None else torch.empty((nHq * hd,), dtype=torch.float32, device=q.device)
    Kq, Ks, Vq, Vs = kv
    c = _ctx(q)
    c.check(LIB.tb_attn_prep_q8(c.h, _p(q), _p(k), _p(v), _p(qw16), _p(kw16), _p(qr), _p(Kq), _p(Ks), _p(Vq),
                                _p(Vs), nHq, nKv, hd, int(pos), float(theta), float(eps)), "attn_prep_q8")
    return qr


def kv_quant_write(kr, v, kv, T, nKv, hd, pos_base):
    """kvQuantWrite (qwen3.js:2211-2216)."""
    Kq, Ks, Vq, Vs = kv
    c = _ctx(kr)
    c.check(LIB.tb_kv_quant_write(c.h, _p(kr), _p(v), _p(Kq), _p(Ks), _p(Vq), _p(Vs), T, nKv, hd, int(pos_base)),
            "kv_quant_write")


def attention_decode_q8(qr, kv, S, nHq, nKv, hd, nsplit=0, out=None):
    """attnDecodeStreamQ8 + combine (qwen3.js:2165-2173)."""
    out = out if out is not None else torch.empty((nHq * hd,), dtype=torch.float32, device=qr.device)
    Kq, Ks, Vq, Vs = kv
    c = _ctx(qr)
    c.check(LIB.tb_attn_decode_q8(c.h, _p(out), _p(qr), _p(Kq), _p(Ks), _p(Vq), _p(Vs), int(S), nHq, nKv, hd,
                                  int(nsplit)), "attn_decode_q8")
    return out


# --------------------------------------------------------------------------
# glue
# --------------------------------------------------------------------------

def argmax(x, out=None, offset=0):
    """argmaxKernel (qwen3.js:2681-2690) over each row of x."""
    x2 = x.reshape(-1, x.shape[-1])
    R, n = x2.shape
    out = out if out is not None else torch.empty((R,), dtype=torch.int32, device=x.device)
    c = _ctx(x)
    c.check(LIB.tb_argmax(c.h, _p(x2), n, R, _p(out), int(offset)), "argmax")
    return out


def logit_mask(logits, mask):
    """logitMask (qwen3.js:2706-2710): tokens whose mask bit is clear -> -3e38, in place.
    mask: int32/uint32 words [rows, ceil(n/32)]."""
    x2 = logits.reshape(-1, logits.shape[-1])
    rows, n = x2.shape
    c = _ctx(logits)
    c.check(LIB.tb_logit_mask(c.h, _p(x2), _p(mask), n, rows), "logit_mask")
    return logits


def gumbel_noise(logits, seed, temp):
    """gumbelNoise (qwen3.js:2731-2737) in place with the given seed."""
    x2 = logits.reshape(-1, logits.shape[-1])
    rows, n = x2.shape
    c = _ctx(logits)
    c.check(LIB.tb_gumbel_noise(c.h, _p(x2), n, rows, int(seed) & 0xFFFFFFFF, float(temp)), "gumbel_noise")
    return logits


def sample_argmax(logits, mask=None, seed=0, temp=0.0, out=None):
    """mask + Gumbel noise + argmax fused (logits untouched): one id per row."""
    x2 = logits.reshape(-1, logits.shape[-1])
    rows, n = x2.shape
    out = out if out is not None else torch.empty((rows,), dtype=torch.int32, device=logits.device)
    c = _ctx(logits)
    c.check(LIB.tb_sample_argmax(c.h, _p(x2), n, rows, _p(mask), int(seed) & 0xFFFFFFFF, float(temp), _p(out)),
            "sample_argmax")
    return out


class GumbelSeeds:
    """The reference's per-forward seed stream (_rngSeed, qwen3.js:2730-2733):
    starts at 0x9E3779B9 and advances before every sampled step."""

    def __init__(self, seed=0x9E3779B9):
        self.seed = seed & 0xFFFFFFFF

    def next(self):
        self.seed = (self.seed * 1664525 + 1013904223) & 0xFFFFFFFF
        return self.seed


def rmsnorm(x, w16, eps, y=None):
    """rmsnorm (qwen3.js:81-88)."""
    x2 = x.reshape(-1, x.shape[-1])
    T, H = x2.shape
    y = y if y is not None else torch.empty_like(x2)
    c = _ctx(x)
    c.check(LIB.tb_rmsnorm(c.h, _p(x2), _p(w16), _p(y), T, H, float(eps)), "rmsnorm")
    return y


def embed_gather(ids, embed_f16, T, idoff=0, y=None):
    """embedGather (qwen3.js:1663-1675)."""
    H = embed_f16.shape[1]
    y = y if y is not None else torch.empty((T, H), dtype=torch.float32, device=ids.device)
    c = _ctx(ids)
    c.check(LIB.tb_embed_gather(c.h, _p(ids), int(idoff), _p(embed_f16), _p(y), T, H), "embed_gather")
    return y
