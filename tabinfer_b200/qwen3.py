"""Qwen3 decode on the C ABI's model runner (tb_qwen3_*), the host-side mirror of
models/qwen3.js: the quant-on-arrival loader (_uploadTensor, :3503-3545), the
T = 1 forward (:3938-4069) and the greedy generate loop that feeds each
argmax token back through the GPU token history (:4055-4060).

Weights arrive as bf16 device tensors under the checkpoint's names; the
runner keeps int4 G=32 packs for every `*_proj.weight` and `lm_head.weight`
and f16 copies of the embedding table and the norms, exactly as the
reference's loader does.  One `step()` decodes one token for each of `batch`
sequences and replays a recorded CUDA graph; ids and positions stay on the
device between steps.
"""
import ctypes
import re

import torch

from . import _lib
from .ops import LIB, Context, default_context, _p

_NAMES = {
    "model.embed_tokens.weight": _lib.QW_EMBED,
    "lm_head.weight": _lib.QW_LM_HEAD,
    "model.norm.weight": _lib.QW_FINAL_NORM,
}
_LAYER_NAMES = {
    "self_attn.q_proj.weight": _lib.QW_Q,
    "self_attn.k_proj.weight": _lib.QW_K,
    "self_attn.v_proj.weight": _lib.QW_V,
    "self_attn.o_proj.weight": _lib.QW_O,
    "mlp.gate_proj.weight": _lib.QW_GATE,
    "mlp.up_proj.weight": _lib.QW_UP,
    "mlp.down_proj.weight": _lib.QW_DOWN,
    "input_layernorm.weight": _lib.QW_LN_ATTN,
    "post_attention_layernorm.weight": _lib.QW_LN_MLP,
    "self_attn.q_norm.weight": _lib.QW_Q_NORM,
    "self_attn.k_norm.weight": _lib.QW_K_NORM,
}
_LAYER_RE = re.compile(r"^model\.layers\.(\d+)\.(.+)$")

# Qwen3-1.7B; CONFIG fields of models/qwen3.js
QWEN3_1_7B = dict(hidden=2048, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=6144,
                  vocab=151936, rope_theta=1e6, rms_eps=1e-6)
QWEN3_0_6B = dict(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=3072,
                  vocab=151936, rope_theta=1e6, rms_eps=1e-6)


def weight_kind(name):
    """(kind, layer) of a checkpoint tensor name, or None for names the decode
    path does not use."""
    if name in _NAMES:
        return _NAMES[name], 0
    m = _LAYER_RE.match(name)
    if m and m.group(2) in _LAYER_NAMES:
        return _LAYER_NAMES[m.group(2)], int(m.group(1))
    return None


def shard(cfg, kind):
    """(row0, nrows, col0, ncols): the block of the full tensor `kind` that
    rank cfg['tp_rank'] of cfg['tp_size'] keeps.  Host-only (no GPU)."""
    c = make_config(cfg)
    out = [ctypes.c_int64() for _ in range(4)]
    rc = LIB.tb_qwen3_shard(ctypes.byref(c), kind, *[ctypes.byref(o) for o in out])
    if rc:
        raise ValueError("tb_qwen3_shard: invalid config or kind (status %d)" % rc)
    return tuple(o.value for o in out)


def _hp(t):
    """host tensor -> pointer for tb_copy_h2d / tb_copy_d2h"""
    assert not t.is_cuda and t.is_contiguous()
    return ctypes.c_void_p(t.data_ptr())


def make_config(cfg):
    c = _lib.Qwen3Config()
    for f, _ in _lib.Qwen3Config._fields_:
        default = {"tp_size": 1, "tp_rank": 0, "batch": 1, "ternary": 1}.get(f)
        v = cfg.get(f, default)
        if v is None:
            raise KeyError("qwen3 config needs '%s'" % f)
        setattr(c, f, v)
    return c


def nccl_unique_id():
    """128 bytes for tb_qwen3_tp_init (make on one rank, broadcast to all)."""
    buf = ctypes.create_string_buffer(128)
    rc = LIB.tb_nccl_unique_id(buf)
    if rc:
        raise RuntimeError("tb_nccl_unique_id failed (status %d)" % rc)
    return buf.raw


class Qwen3:
    """One rank's Qwen3 decoder.  cfg: the model sizes (QWEN3_1_7B ...) plus
    max_seq, batch, and tp_size / tp_rank for tensor parallelism."""

    def __init__(self, cfg, device=0, ctx: Context = None):
        self.cfg = dict(cfg)
        self.cfg.setdefault("tp_size", 1)
        self.cfg.setdefault("tp_rank", 0)
        self.cfg.setdefault("batch", 1)
        self.device = torch.device("cuda", device)
        self.ctx = ctx or default_context(device)
        c = make_config(self.cfg)
        h = ctypes.c_void_p()
        self.ctx.check(LIB.tb_qwen3_create(self.ctx.h, ctypes.byref(c), ctypes.byref(h)), "qwen3_create")
        self.h = h
        P = self.cfg["tp_size"]
        self.n_kv_local = self.cfg["n_kv_heads"] // P
        self.vocab_local = self.cfg["vocab"] // P
        ids, pos, logits = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        self.ctx.check(LIB.tb_qwen3_io(self.h, ctypes.byref(ids), ctypes.byref(pos), ctypes.byref(logits)), "io")
        self._io = (ids.value, pos.value, logits.value)

    def close(self):
        if getattr(self, "h", None):
            LIB.tb_qwen3_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- loading (quant on arrival) -------------------------------------------
    def load(self, name, w_bf16):
        """Upload one checkpoint tensor (bf16, on this device)."""
        kl = weight_kind(name)
        if kl is None:
            return False
        kind, layer = kl
        w = w_bf16.contiguous()
        assert w.dtype in (torch.bfloat16, torch.int16, torch.uint16) and w.device == self.device
        rows, cols = (1, w.numel()) if w.dim() == 1 else tuple(w.shape)
        self.ctx.check(LIB.tb_qwen3_set_weight(self.h, kind, layer, _p(w), rows, cols), "set_weight " + name)
        return True

    def load_quantized(self, name, fmt, data, scales=None, shape=None):
        """Set one tensor from its already-quantized FULL form (what the quant
        cache holds, qwen3.js:3671-3717): fmt QW_FMT_INT4 / QW_FMT_TERN with pack
        and f16 scales, or QW_FMT_F16 with the f16 buffer.  data / scales are
        numpy arrays (host) or CUDA tensors; shape = (rows, cols) of the tensor."""
        kl = weight_kind(name)
        if kl is None:
            return False
        kind, layer = kl
        rows, cols = shape

        keep = []

        def ptr(a):
            if a is None:
                return None
            if isinstance(a, torch.Tensor):
                a = a.contiguous()
                keep.append(a)
                return _p(a) if a.is_cuda else ctypes.c_void_p(a.data_ptr())
            import numpy as np
            a = np.ascontiguousarray(a)
            keep.append(a)
            return ctypes.c_void_p(a.ctypes.data)
        self.ctx.check(LIB.tb_qwen3_set_weight_q(self.h, kind, layer, fmt, ptr(data), ptr(scales), rows, cols),
                       "set_weight_q " + name)
        self.ctx.synchronize()   # the host buffers may be reused by the caller
        return True

    def prefill(self, seq, ids, pos0=0):
        """forward(ids, posBase) at T > 1 for sequence `seq` (qwen3.js:3938-4069):
        runs the T tokens, fills their cache rows, and returns the next token id
        (also left in the decode step's ids / pos for `seq`)."""
        import numpy as np
        a = np.ascontiguousarray(ids, np.uint32)
        self.ctx.check(LIB.tb_qwen3_prefill(self.h, int(seq), ctypes.c_void_p(a.ctypes.data), a.size, int(pos0)),
                       "prefill")
        toks, _ = self.tokens()
        return toks[seq]

    def weight_format(self, name):
        """QW_FMT_* the loader chose for a tensor (-1 when unset or unknown)."""
        kl = weight_kind(name)
        if kl is None:
            return -1
        return LIB.tb_qwen3_weight_format(self.h, kl[0], kl[1])

    def tp_init(self, unique_id):
        """NCCL exchange: every rank passes the same 128-byte unique id."""
        self.ctx.check(LIB.tb_qwen3_tp_init(self.h, ctypes.c_char_p(bytes(unique_id))), "tp_init")

    def set_step_mode(self, mode):
        """QW_STEP_AUTO (persistent where it applies), QW_STEP_KERNELS (one kernel
        per operation) or QW_STEP_PERSISTENT (one persistent kernel for embed +
        all layers; batch 1, one GPU, int4 layer weights)."""
        self.ctx.check(LIB.tb_qwen3_set_step_mode(self.h, int(mode)), "set_step_mode")

    def step_layers(self):
        """The persistent kernel alone (embed + every layer) at the current
        position, for timing; needs a recorded persistent step."""
        self.ctx.check(LIB.tb_qwen3_step_layers(self.h), "step_layers")

    def step_trace(self, buf):
        """Phase trace of the persistent kernel into buf (int64 CUDA tensor of
        SMs x (1 + 38 * layers)), or None to stop."""
        self.ctx.check(LIB.tb_qwen3_step_trace(self.h, None if buf is None else _p(buf)), "step_trace")

    def step_kind(self):
        """QW_STEP_KERNELS or QW_STEP_PERSISTENT once the step was recorded, else 0."""
        return int(LIB.tb_qwen3_step_kind(self.h))

    def tp_handle(self):
        """This rank's 64-byte IPC handle of its exchange arena."""
        buf = ctypes.create_string_buffer(64)
        self.ctx.check(LIB.tb_qwen3_tp_handle(self.h, buf), "tp_handle")
        return buf.raw

    def tp_connect(self, handles):
        """Peer-memory exchange: handles = every rank's tp_handle(), rank order."""
        blob = b"".join(bytes(h) for h in handles)
        assert len(blob) == 64 * self.cfg["tp_size"]
        self.ctx.check(LIB.tb_qwen3_tp_connect(self.h, ctypes.c_char_p(blob)), "tp_connect")

    def tp_reset(self):
        """Clear this rank's exchange state after a device-side wait gave up
        (tb_qwen3_tp_reset): call it on every rank with every rank idle, behind
        a barrier, and step again only after every rank returned."""
        self.ctx.check(LIB.tb_qwen3_tp_reset(self.h), "tp_reset")

    # ---- cache and I/O ----------------------------------------------------------
    def kv_pointers(self, layer):
        p = [ctypes.c_void_p() for _ in range(4)]
        self.ctx.check(LIB.tb_qwen3_kv(self.h, layer, *[ctypes.byref(x) for x in p]), "kv")
        return tuple(x.value for x in p)

    def kv_fill(self, layer, seq, k_rows, v_rows, pos_base=0):
        """Quantize-write rows [pos_base, pos_base+T) of sequence `seq`'s cache
        (k_rows already RoPE'd, both f32 [T][n_kv_local*hd]) -- kvQuantWrite."""
        Kq, Ks, Vq, Vs = self.kv_pointers(layer)
        hd = self.cfg["head_dim"]
        row = self.n_kv_local * hd
        base = seq * self.cfg["max_seq"] * row
        T = k_rows.shape[0]
        self.ctx.check(LIB.tb_kv_quant_write(self.ctx.h, _p(k_rows), _p(v_rows), Kq + base, Ks + base // 32 * 4,
                                             Vq + base, Vs + base // 32 * 4, T, self.n_kv_local, hd, pos_base),
                       "kv_fill")

    def kv_host(self, layer):
        """Host copies (numpy) of this rank's cache of a layer: Kq int8, Ks f32,
        Vq int8, Vs f32, each [batch][max_seq][...]."""
        import numpy as np
        Kq, Ks, Vq, Vs = self.kv_pointers(layer)
        B, S, hd = self.cfg["batch"], self.cfg["max_seq"], self.cfg["head_dim"]
        row = self.n_kv_local * hd
        out = []
        self.ctx.synchronize()
        for ptr, dt, n in ((Kq, np.int8, row), (Ks, np.float32, row // 32), (Vq, np.int8, row),
                           (Vs, np.float32, row // 32)):
            a = np.empty((B, S, n), dt)
            self.ctx.check(LIB.tb_copy_d2h(self.ctx.h, a.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(ptr),
                                           a.nbytes), "copy_d2h")
            out.append(a)
        self.ctx.synchronize()
        return tuple(out)

    def set_tokens(self, ids, pos):
        """ids, pos: int sequences of length batch (written to the device)."""
        B = self.cfg["batch"]
        ids_t = torch.tensor(list(ids), dtype=torch.int32).reshape(B)
        pos_t = torch.tensor(list(pos), dtype=torch.int32).reshape(B)
        self._copy_in(self._io[0], ids_t)
        self._copy_in(self._io[1], pos_t)

    def _copy_in(self, dev_ptr, host_t):
        host_t = host_t.contiguous()
        self.ctx.check(LIB.tb_copy_h2d(self.ctx.h, ctypes.c_void_p(dev_ptr), _hp(host_t),
                                       host_t.numel() * host_t.element_size()), "copy_h2d")
        self.ctx.synchronize()

    def tokens(self):
        B = self.cfg["batch"]
        ids = torch.empty(B, dtype=torch.int32)
        pos = torch.empty(B, dtype=torch.int32)
        self.ctx.synchronize()
        self.ctx.check(LIB.tb_copy_d2h(self.ctx.h, _hp(ids), ctypes.c_void_p(self._io[0]), 4 * B), "copy_d2h")
        self.ctx.check(LIB.tb_copy_d2h(self.ctx.h, _hp(pos), ctypes.c_void_p(self._io[1]), 4 * B), "copy_d2h")
        self.ctx.synchronize()
        return ids.tolist(), pos.tolist()

    def logits(self):
        B = self.cfg["batch"]
        out = torch.empty((B, self.vocab_local), dtype=torch.float32)
        self.ctx.synchronize()
        self.ctx.check(LIB.tb_copy_d2h(self.ctx.h, _hp(out), ctypes.c_void_p(self._io[2]), out.numel() * 4),
                       "copy_d2h")
        self.ctx.synchronize()
        return out

    # ---- decode -------------------------------------------------------------------
    def step(self):
        """One token for every sequence (forward, T = 1): replays the recorded step."""
        self.ctx.check(LIB.tb_qwen3_decode_step(self.h), "decode_step")

    def generate(self, n):
        """n greedy tokens per sequence; returns them as [n][batch] ids."""
        out = []
        for _ in range(n):
            self.step()
            out.append(self.tokens()[0])
        return out

    def launches_per_step(self):
        k, c = ctypes.c_int(), ctypes.c_int()
        self.ctx.check(LIB.tb_qwen3_launches_per_step(self.h, ctypes.byref(k), ctypes.byref(c)), "launches")
        return k.value, c.value
