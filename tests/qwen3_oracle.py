"""CPU oracle of one Qwen3 decode step (models/qwen3.js forward :3938-4069, the
T = 1 int8-KV branch), composed from the per-op restatements in oracle/ — test
infrastructure only.  Each op follows the reference routine named beside it;
intermediate rows are rounded to f32 where the reference stores f32 buffers.
"""
import numpy as np

import oracle

from helpers import bf16_normal, bf16_to_f32, tern_bf16


def f16_of_bf16(u16):
    """bf16ToF16bits (qwen3.js:3386-3390) then f16 -> f64, elementwise."""
    flat = bf16_to_f32(np.ascontiguousarray(u16, np.uint16).ravel())
    bits = np.array([oracle.f32_to_f16_js(float(v)) for v in flat], np.uint16)
    return bits.reshape(np.shape(u16))


def f16_to_f32(bits):
    return np.array([oracle.f16_to_f64(int(b)) for b in np.ravel(bits)], np.float64).reshape(np.shape(bits)) \
        .astype(np.float32)


def make_weights(cfg, seed, ternary=False):
    """Checkpoint-named bf16 bit arrays: projections/lm_head/embed N(0, 0.02),
    norms 1 + N(0, 0.1) (configs 2-4 of the benchmark).  ternary: projections and
    lm_head are Bonsai-style ternary bf16 ({-m, 0, +m} per 32-group)."""
    rng = np.random.default_rng(seed)
    H, hd, nHq, nKv, I, V = (cfg[k] for k in ("hidden", "head_dim", "n_heads", "n_kv_heads", "intermediate", "vocab"))
    proj = (lambda shape: tern_bf16(rng, *shape)) if ternary else (lambda shape: bf16_normal(rng, shape, 0.02))
    W = {"model.embed_tokens.weight": bf16_normal(rng, (V, H), 0.02), "model.norm.weight": _norm(rng, H)}
    W["lm_head.weight"] = proj((V, H))
    for l in range(cfg["layers"]):
        p = "model.layers.%d." % l
        W[p + "self_attn.q_proj.weight"] = proj((nHq * hd, H))
        W[p + "self_attn.k_proj.weight"] = proj((nKv * hd, H))
        W[p + "self_attn.v_proj.weight"] = proj((nKv * hd, H))
        W[p + "self_attn.o_proj.weight"] = proj((H, nHq * hd))
        W[p + "mlp.gate_proj.weight"] = proj((I, H))
        W[p + "mlp.up_proj.weight"] = proj((I, H))
        W[p + "mlp.down_proj.weight"] = proj((H, I))
        W[p + "input_layernorm.weight"] = _norm(rng, H)
        W[p + "post_attention_layernorm.weight"] = _norm(rng, H)
        W[p + "self_attn.q_norm.weight"] = _norm(rng, hd)
        W[p + "self_attn.k_norm.weight"] = _norm(rng, hd)
    return W


def _norm(rng, n):
    x = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


class OracleModel:
    """Quantized weights as the loader's _uploadTensor makes them (the lossless
    ternary record of quantizeTernaryBf16 when a tensor is ternary and `ternary`
    is on, else quantizeInt4Bf16) and f16 norms of a checkpoint dict, for
    oracle decode steps."""

    def __init__(self, cfg, W, ternary=True):
        self.cfg = cfg
        self.W = W
        self.q = {}
        self.tern = {}
        for name, w in W.items():
            if name.endswith("_proj.weight") or name == "lm_head.weight":
                t = oracle.quant_tern_wgsl(w) if ternary else None
                self.tern[name] = t is not None
                self.q[name] = t if t is not None else oracle.quant_int4_g32(w)
        self.f16 = {name: f16_of_bf16(w) for name, w in W.items()
                    if name.endswith("norm.weight") or name.endswith("layernorm.weight")}

    def _gemv(self, name, xq, xs):
        """projGemv / linearQ at one row: gemvTern or gemvDP4 by weight kind."""
        f = oracle.gemv_tern_wgsl_q8act if self.tern[name] else oracle.gemv_int4_q8act
        return f(xq, xs, *self.q[name])

    def embed_row(self, tok):
        return f16_to_f32(f16_of_bf16(self.W["model.embed_tokens.weight"][tok]))

    def step(self, tok, pos, cache, route_f32=False, attn_f16ops=False):
        """One decode step of one sequence.  cache: per layer (Kq, Ks, Vq, Vs)
        numpy arrays [max_seq][...] holding rows < pos; row `pos` is written
        into them (as attnPrepQ8 does).  route_f32: the lm_head runs as gemvQ on
        the f32 row (linearQ's route for one row with vocab >= 16384), else as
        the int8 DP4A GEMV.  attn_f16ops: the attention at the operand precision
        of the reference's f16 prefill kernel (a prefill token).  Returns f64 logits."""
        c = self.cfg
        H, hd, nHq, nKv, eps, theta = (c[k] for k in ("hidden", "head_dim", "n_heads", "n_kv_heads", "rms_eps",
                                                      "rope_theta"))
        x = self.embed_row(tok).astype(np.float64)
        for l in range(c["layers"]):
            p = "model.layers.%d." % l
            Kq, Ks, Vq, Vs = cache[l]
            xq, xs, _, _ = oracle.rmsnorm_q8(x.astype(np.float32), self.f16[p + "input_layernorm.weight"], eps)
            q = self._gemv(p + "self_attn.q_proj.weight", xq, xs)[0].astype(np.float32)
            k = self._gemv(p + "self_attn.k_proj.weight", xq, xs)[0].astype(np.float32)
            v = self._gemv(p + "self_attn.v_proj.weight", xq, xs)[0].astype(np.float32)
            qr = oracle.head_norm_rope(q.reshape(nHq, hd), self.f16[p + "self_attn.q_norm.weight"], pos, theta, eps)
            kr = oracle.head_norm_rope(k.reshape(nKv, hd), self.f16[p + "self_attn.k_norm.weight"], pos, theta, eps)
            kq_row, ks_row = oracle.kv_quant_q8(kr.astype(np.float32).ravel())
            vq_row, vs_row = oracle.kv_quant_q8(v.ravel())
            Kq[pos], Ks[pos], Vq[pos], Vs[pos] = kq_row, ks_row, vq_row, vs_row
            S = pos + 1
            att = oracle.attn_decode_q8_f16ops if attn_f16ops else oracle.attn_decode_q8
            attn = att(qr.astype(np.float32).ravel(), Kq[:S], Ks[:S], Vq[:S], Vs[:S], S, nHq, nKv,
                       hd).astype(np.float32)
            aq, as_, _ = oracle.quant_q8(attn)
            x = x + self._gemv(p + "self_attn.o_proj.weight", aq, as_)[0]
            x = x.astype(np.float32).astype(np.float64)
            xq, xs, _, _ = oracle.rmsnorm_q8(x.astype(np.float32), self.f16[p + "post_attention_layernorm.weight"],
                                             eps)
            gate = p + "mlp.gate_proj.weight"
            f = oracle.gateup_tern_wgsl_q8act if self.tern[gate] else oracle.gateup_q8act
            swi = f(xq, xs, *self.q[gate], *self.q[p + "mlp.up_proj.weight"])[0].astype(np.float32)
            sq, ss, _ = oracle.quant_q8(swi)
            x = x + self._gemv(p + "mlp.down_proj.weight", sq, ss)[0]
            x = x.astype(np.float32).astype(np.float64)
        return self.head(x.astype(np.float32), route_f32)

    def head(self, x, route_f32):
        """final norm + lm_head (qwen3.js:4037-4049)."""
        c = self.cfg
        fn = self.f16["model.norm.weight"]
        if route_f32 and not self.tern["lm_head.weight"]:
            _, _, _, inv = oracle.rmsnorm_q8(x, fn, c["rms_eps"])
            xn = (x.astype(np.float32) * np.float32(inv[0])) * f16_to_f32(fn)
            return oracle.gemv_int4_f32act(xn.astype(np.float32), *self.q["lm_head.weight"])[0]
        xq, xs, _, _ = oracle.rmsnorm_q8(x, fn, c["rms_eps"])
        return self._gemv("lm_head.weight", xq, xs)[0]
