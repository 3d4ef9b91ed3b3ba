"""bench.py -- Qwen3-1.7B int4 decode on B200, with the
int4 GEMV roofline of its kernels.

One step = one decode token for each of `batch` sequences through the recorded
Qwen3 decode step of libtabinfer_b200 (tb_qwen3_decode_step: the forward of
models/qwen3.js:3938-4069 at T = 1 with the int8 KV cache): embedding gather,
28 x (fused RMSNorm+int8+q/k/v GEMV, attention prep (q/k norm, RoPE, int8 K/V
write), split-KV GQA decode attention over the context, o GEMV + residual,
fused RMSNorm+int8+gate/up+SiLU, down GEMV + residual), final norm + tied
lm_head (151936 x 2048) and GPU argmax that feeds the next step.  With N GPUs
the step is tensor-parallel (q/k/v, gate/up, lm_head rows and kv heads split,
o/down columns split, NCCL allreduce after o and down): strong scaling, the
same tokens per step on 1..8 GPUs.

Weights: bf16 N(0, 0.02) (norms 1 + N(0, 0.1)) generated on the GPU from a
fixed seed and quantized on arrival with the reference's int4 G=32 scheme;
the KV cache holds `context - 1` rows of N(0, 1) keys/values quantized with the
reference's int8 per-32 scheme; each step appends one row.  The weights
(0.97 GB) and the cache exceed the 126 MB L2, so every step streams from HBM.

value = tokens per second (batch x steps / device time, max over ranks).
e2e = the same through the public API with host buffers: per step the pinned
host ids and positions are copied in (tb_copy_h2d), the step runs, and the new
token ids are read back (tb_copy_d2h), all inside the timed region.

--impl reference times the reference's CPU path for the same step (the C
transcription of the JS int4 linearQ math in oracle/tb_cpu_ref.c over all host
threads) on a bounded sample of the matrices.
"""
import argparse
import ctypes
import json
import os
import statistics
import numpy as np
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

# Qwen3-1.7B
Q17 = dict(hidden=2048, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=6144, vocab=151936,
           rope_theta=1e6, rms_eps=1e-6)
# Qwen3-0.6B GEMV chain, reported beside the decode step
H6, NHQ6, NKV6, HD6, INTER6, VOCAB6, LAYERS6 = 1024, 16, 8, 128, 3072, 151936, 28
MATS6 = [("q", NHQ6 * HD6, H6), ("k", NKV6 * HD6, H6), ("v", NKV6 * HD6, H6), ("o", H6, NHQ6 * HD6),
         ("gate", INTER6, H6), ("up", INTER6, H6), ("down", H6, INTER6)]


def wbytes(N, K, tern=False):
    """int4 G32 weight bytes (packed nibbles + f16 scales), or ternary WebGPU-layout
    bytes (2-bit codes + f16 scales)."""
    return N * K // (4 if tern else 2) + N * (K // 32) * 2


def gemv_bytes(N, K, B, act_bytes, tern=False):
    """packed weights + scales read once, B activation rows in, B output rows out."""
    return wbytes(N, K, tern) + B * K * act_bytes + B * N * 4


def step_matrices(cfg, P):
    """(name, N, K, launches-per-step) of one rank's int4 matrices."""
    H, hd, I, V = cfg["hidden"], cfg["head_dim"], cfg["intermediate"], cfg["vocab"]
    q, kv = cfg["n_heads"] * hd // P, cfg["n_kv_heads"] * hd // P
    L = cfg["layers"]
    return [("q", q, H, L), ("k", kv, H, L), ("v", kv, H, L), ("o", H, cfg["n_heads"] * hd // P, L),
            ("gate", I // P, H, L), ("up", I // P, H, L), ("down", H, I // P, L), ("lm_head", V // P, H, 1)]


def kv_bytes(cfg, P, S):
    """int8 K and V + f32 per-32 scales read by one attention launch (one layer,
    one sequence, S context rows)."""
    row = cfg["n_kv_heads"] // P * cfg["head_dim"]
    return 2 * S * row * (1 + 4 / 32)


def step_bytes(cfg, P, B, S, tern=False):
    """Algorithmic HBM bytes of one rank's step: every weight once, the KV
    context of every sequence, activations in/out of the GEMVs."""
    tot = 0
    q8 = 1 + 4 / 32
    for name, N, K, n in step_matrices(cfg, P):
        act = 4 if (name == "lm_head" and B == 1 and not tern) else q8
        tot += n * gemv_bytes(N, K, B, act, tern)
    tot += cfg["layers"] * B * kv_bytes(cfg, P, S)
    return int(tot)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples (100 ms) of SM clock, power and throttle reasons while
    the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        pw = [num(r[3]) for r in rows]
        good = [p for p in pw if p is not None]
        lo, hi = (min(good), max(good)) if good else (0.0, 0.0)
        load = [num(r[1]) for r, p in zip(rows, pw) if p is not None and p >= (lo + hi) / 2 and num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(load or sm) if (load or sm) else None,
                "sm_max_mhz": max(num(r[2]) or 0 for r in rows), "reasons": reasons, "samples": len(rows),
                "power_w_max": hi}


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# the decode model
# ---------------------------------------------------------------------------

def build_model(cfg, dev, batch, context, extra_rows, P, rank, seed=1234, ternary=False):
    """A Qwen3 rank with random weights (same full tensors on every rank; each
    keeps its shard) and a cache prefilled to context - 1 rows.  ternary: the
    projections and lm_head are Bonsai-style ternary bf16 ({-m, 0, +m} per
    32-group, m U(0.005, 0.055)), which the loader stores as ternary records."""
    import torch
    import tabinfer_b200 as tb
    full = dict(cfg, max_seq=context + extra_rows, batch=batch, tp_size=P, tp_rank=rank)
    m = tb.Qwen3(full, device=dev.index)
    H, hd, I, V = cfg["hidden"], cfg["head_dim"], cfg["intermediate"], cfg["vocab"]
    nq, nkv = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    g = torch.Generator(device=dev)

    def load(name, shape, std, k):
        g.manual_seed(seed * 1000 + k)
        if std is None:
            w = (1.0 + 0.1 * torch.randn(shape, device=dev, generator=g)).to(torch.bfloat16)
        elif ternary and ("_proj." in name or name == "lm_head.weight"):
            N, K = shape
            mag = (torch.rand(N, K // 32, device=dev, generator=g) * 0.05 + 0.005).view(torch.int32) >> 16
            t = torch.randint(-1, 2, (N, K), device=dev, generator=g, dtype=torch.int32)
            bits = torch.where(t == 0, torch.zeros_like(t), mag.repeat_interleave(32, dim=1) | ((t < 0).int() << 15))
            w = torch.where(bits >= 32768, bits - 65536, bits).to(torch.int16)
            del t, bits, mag
        else:
            w = (torch.randn(shape, device=dev, generator=g) * std).to(torch.bfloat16)
        m.load(name, w.view(torch.int16))

    load("model.embed_tokens.weight", (V, H), 0.02, 0)
    load("lm_head.weight", (V, H), 0.02, 0)          # tied: the same bf16 table (int4); ternary: its own
    load("model.norm.weight", (H,), None, 1)
    k = 2
    for l in range(cfg["layers"]):
        p = "model.layers.%d." % l
        for name, shape, std in (("self_attn.q_proj.weight", (nq, H), 0.02), ("self_attn.k_proj.weight", (nkv, H), 0.02),
                                 ("self_attn.v_proj.weight", (nkv, H), 0.02), ("self_attn.o_proj.weight", (H, nq), 0.02),
                                 ("mlp.gate_proj.weight", (I, H), 0.02), ("mlp.up_proj.weight", (I, H), 0.02),
                                 ("mlp.down_proj.weight", (H, I), 0.02), ("input_layernorm.weight", (H,), None),
                                 ("post_attention_layernorm.weight", (H,), None),
                                 ("self_attn.q_norm.weight", (hd,), None), ("self_attn.k_norm.weight", (hd,), None)):
            load(p + name, shape, std, k)
            k += 1
    # cache: rows [0, context-1) of N(0,1) keys/values, int8 per-32 (kvQuantWrite);
    # one random block serves every layer and sequence
    rows = context - 1
    if rows > 0:
        g.manual_seed(seed + 7 + rank)
        kr = torch.randn(rows, m.n_kv_local * hd, device=dev, generator=g)
        vr = torch.randn(rows, m.n_kv_local * hd, device=dev, generator=g)
        for l in range(cfg["layers"]):
            for b in range(batch):
                m.kv_fill(l, b, kr, vr, 0)
        del kr, vr
    torch.cuda.synchronize(dev)
    return m


def time_steps(m, K, stream):
    """Device time (ms) of K replays of the recorded step (CUDA events on the
    stream the step is launched on)."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        m.step()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


def time_e2e(m, K, stream, ids0, pos0):
    """K steps through the public API with host buffers: pinned ids/positions in,
    the step, the new ids out (tb_copy_h2d / tb_qwen3_decode_step / tb_copy_d2h)."""
    import torch
    from tabinfer_b200._lib import LIB
    B = m.cfg["batch"]
    hin = torch.tensor(list(ids0) + list(pos0), dtype=torch.int32).pin_memory()
    hout = torch.zeros(B, dtype=torch.int32).pin_memory()
    ids_dev, pos_dev, _ = m._io
    c = m.ctx
    P = ctypes.c_void_p
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        c.check(LIB.tb_copy_h2d(c.h, P(ids_dev), P(hin.data_ptr()), 4 * B), "h2d ids")
        c.check(LIB.tb_copy_h2d(c.h, P(pos_dev), P(hin.data_ptr() + 4 * B), 4 * B), "h2d pos")
        m.step()
        c.check(LIB.tb_copy_d2h(c.h, P(hout.data_ptr()), P(ids_dev), 4 * B), "d2h ids")
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1), 8 * B, 4 * B


def kernel_kinds(cfg, dev, P, context, peak):
    """Per-launch device time of each kernel kind of one rank's multi-kernel step at
    batch 1: one recorded batch of back-to-back launches of the kind, each on its own
    copy of the weights (or KV cache), the copies together at least twice the L2, so
    every launch streams from HBM; CUDA events around replays on the launching
    stream, divided by the launches.  Returns {kind: {...}} with algorithmic bytes
    and GB/s."""
    import math
    import torch
    import tabinfer_b200 as tb
    g = torch.Generator(device=dev).manual_seed(99)
    H, hd, I, V, L = cfg["hidden"], cfg["head_dim"], cfg["intermediate"], cfg["vocab"], cfg["layers"]
    nHq, nKv = cfg["n_heads"] // P, cfg["n_kv_heads"] // P
    ctx = tb.default_context(dev.index)

    def mat(N, K):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        return tb.quantize_int4_bf16(w.view(torch.int16))

    ln = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half().view(torch.int16)
    x = torch.randn(1, H, device=dev, generator=g)
    xa = torch.randn(1, nHq * hd, device=dev, generator=g)
    xs = torch.randn(1, I // P, device=dev, generator=g)
    S = context
    row = nKv * hd
    qr = torch.randn(nHq * hd, device=dev, generator=g)

    def kv():
        return (torch.randint(-127, 128, (S, row), device=dev, generator=g, dtype=torch.int8),
                torch.rand(S, row // 32, device=dev, generator=g) + 0.5,
                torch.randint(-127, 128, (S, row), device=dev, generator=g, dtype=torch.int8),
                torch.rand(S, row // 32, device=dev, generator=g) + 0.5)

    outs = {n: torch.zeros(1, N, device=dev) for n, N in (("q", nHq * hd), ("k", nKv * hd), ("v", nKv * hd),
                                                             ("o", H), ("swi", I // P), ("lm", V // P))}
    att = torch.zeros(nHq * hd, device=dev)
    # kind: (one copy's tensors, the launch on a copy, algorithmic bytes a launch, launches a step)
    kinds = {
        "gemv rmsnorm+qkv": (lambda: (mat(nHq * hd, H), mat(nKv * hd, H), mat(nKv * hd, H)),
                             lambda c: tb.gemv_dp4a_multi(x, list(c), norm_w=ln, ys=[outs["q"], outs["k"], outs["v"]]),
                             sum(wbytes(N, H) + N * 4 for N in (nHq * hd, nKv * hd, nKv * hd)) + H * 4, L),
        "gemv o": (lambda: mat(H, nHq * hd), lambda c: tb.gemv_dp4a(xa, *c, y=outs["o"], acc=True),
                   gemv_bytes(H, nHq * hd, 1, 4), L),
        "gemv rmsnorm+gate+up+silu": (lambda: (mat(I // P, H), mat(I // P, H)),
                                      lambda c: tb.gate_up_silu_dp4a(x, *c[0], *c[1], norm_w=ln, swi=outs["swi"]),
                                      2 * wbytes(I // P, H) + H * 4 + (I // P) * 4, L),
        "gemv down": (lambda: mat(H, I // P), lambda c: tb.gemv_dp4a(xs, *c, y=outs["o"], acc=True),
                      gemv_bytes(H, I // P, 1, 4), L),
        "gemv rmsnorm+lm_head (f32)": (lambda: mat(V // P, H), lambda c: tb.gemv_q_norm(x, ln, 1e-6, *c, y=outs["lm"]),
                                       gemv_bytes(V // P, H, 1, 4), 1),
        "attn decode S=%d" % S: (kv, lambda c: tb.attention_decode_q8(qr, c, S, nHq, nKv, hd, out=att),
                                 kv_bytes(cfg, P, S) + 2 * nHq * hd * 4, L),
    }
    from tabinfer_b200._lib import LIB
    res = {}
    l2 = 126 << 20
    for name, (make, fn, nbytes, per_step) in kinds.items():
        nc = max(4, int(math.ceil(2 * l2 / nbytes)))
        copies = [make() for _ in range(nc)]
        h, stream = _record_batch(ctx, dev, lambda: [fn(c) for c in copies])
        ms = _replay_ms(ctx, h, stream, 5)
        LIB.tb_batch_destroy(h)
        us = ms * 1e3 / nc
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"us_per_launch": round(us, 3), "bytes_per_launch": int(nbytes), "launches_per_step": per_step,
                     "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4), "us_per_step": round(us * per_step, 2),
                     "timing": "%d back-to-back launches on %d weight copies (> 2x L2), recorded, CUDA events" % (nc, nc)}
        del copies
        torch.cuda.synchronize(dev)
    torch.cuda.synchronize(dev)
    return res


# ---------------------------------------------------------------------------
# Qwen3-0.6B GEMV chain: int4 GEMV HBM GB/s without attention
# ---------------------------------------------------------------------------

class Chain:
    """Weights of the 0.6B decode GEMV chain, quantized on the GPU."""

    def __init__(self, dev, seed):
        import torch
        import tabinfer_b200 as tb
        self.dev = dev
        g = torch.Generator(device=dev).manual_seed(seed)
        self.layers = []
        for _ in range(LAYERS6):
            L = {}
            for name, N, K in MATS6:
                w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
                L[name] = tb.quantize_int4_bf16(w.view(torch.int16))
            L["ln1"] = (1.0 + 0.1 * torch.randn(H6, device=dev, generator=g)).half().view(torch.int16)
            L["ln2"] = (1.0 + 0.1 * torch.randn(H6, device=dev, generator=g)).half().view(torch.int16)
            self.layers.append(L)
        w = (torch.randn(VOCAB6, H6, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.lm_head = tb.quantize_int4_bf16(w.view(torch.int16))
        self.norm = (1.0 + 0.1 * torch.randn(H6, device=dev, generator=g)).half().view(torch.int16)
        del w
        torch.cuda.synchronize(dev)


def chain_bytes(B):
    q8 = 1 + 4 / 32
    tot = sum(gemv_bytes(N, K, B, q8) for _, N, K in MATS6) * LAYERS6
    return int(tot + gemv_bytes(VOCAB6, H6, B, 4 if B == 1 else q8))


def chain_gbs(dev, ctx, B, steps):
    """GB/s of the 0.6B GEMV chain (4 fused GEMV launches per layer + lm_head +
    argmax, attention left out), recorded with tb_batch and replayed."""
    import torch
    import tabinfer_b200 as tb
    from tabinfer_b200._lib import LIB, P
    c = Chain(dev, 1000)
    z = lambda *s: torch.zeros(*s, dtype=torch.float32, device=dev)  # noqa: E731
    x, q, k, v, swi, logits = z(B, H6), z(B, NHQ6 * HD6), z(B, NKV6 * HD6), z(B, NKV6 * HD6), z(B, INTER6), z(B, VOCAB6)
    tok = torch.zeros(B, dtype=torch.int32, device=dev)

    # batch >= 2: the tensor-core GEMVs (one weight read for all rows; a
    # quantization launch before each), the route the decode step takes
    mma = B >= 2

    def step():
        for L in c.layers:
            if mma:
                tb.gemv_mma_multi(x, [L["q"], L["k"], L["v"]], norm_w=L["ln1"], eps=1e-6, ys=[q, k, v])
                tb.gemv_mma(q, *L["o"], y=x, acc=True)
                tb.gate_up_silu_mma(x, *L["gate"], *L["up"], norm_w=L["ln2"], eps=1e-6, swi=swi)
                tb.gemv_mma(swi, *L["down"], y=x, acc=True)
            else:
                tb.gemv_dp4a_multi(x, [L["q"], L["k"], L["v"]], norm_w=L["ln1"], eps=1e-6, ys=[q, k, v])
                tb.gemv_dp4a(q, *L["o"], y=x, acc=True)
                tb.gate_up_silu_dp4a(x, *L["gate"], *L["up"], norm_w=L["ln2"], eps=1e-6, swi=swi)
                tb.gemv_dp4a(swi, *L["down"], y=x, acc=True)
        if B == 1:
            tb.gemv_q_norm(x, c.norm, 1e-6, *c.lm_head, y=logits)
        elif mma:
            tb.gemv_mma(x, *c.lm_head, norm_w=c.norm, eps=1e-6, y=logits)
        else:
            tb.gemv_dp4a(x, *c.lm_head, norm_w=c.norm, eps=1e-6, y=logits)
        tb.argmax(logits, out=tok)

    torch.cuda.synchronize(dev)     # the context's own stream does not wait for torch's
    stream = torch.cuda.ExternalStream(ctx.own_stream(), device=dev)
    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        ctx.check(LIB.tb_batch_begin(ctx.h), "batch_begin")
        step()
        h = P()
        ctx.check(LIB.tb_batch_end(ctx.h, ctypes.byref(h)), "batch_end")
        for _ in range(5):
            ctx.check(LIB.tb_batch_submit(ctx.h, h), "submit")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            ctx.check(LIB.tb_batch_submit(ctx.h, h), "submit")
        e1.record(stream)
        e1.synchronize()
    LIB.tb_batch_destroy(h)
    ms = e0.elapsed_time(e1) / steps
    del c
    torch.cuda.synchronize(dev)
    return {"gbs": round(chain_bytes(B) / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms, 4), "batch": B,
            "bytes_per_step": chain_bytes(B), "launches_per_step": (8 * LAYERS6 + 4) if mma else (4 * LAYERS6 + 3),
            "gemv": "mma_s8u8" if mma else "dp4a"}


# ---------------------------------------------------------------------------
# prefill GEMM and int3 MoE beside the decode step
# ---------------------------------------------------------------------------

def _cold_time(fn, flush, stream, reps=5):
    """median CUDA-event time (ms) of fn() after an L2-evicting write"""
    import torch
    fn()
    ts = []
    for r in range(reps + 1):
        flush.fill_(r & 0xff)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        if r:
            ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def prefill_extra(dev, peak_tf, stream):
    """The seven Qwen3-1.7B layer matrices as prefill GEMMs (tcgen05, f16 math of
    gemmQ) on M = 512 / 2048 / 8192 bf16 activation rows: TFLOP/s of 2*M*N*K."""
    import torch
    import tabinfer_b200 as tb
    g = torch.Generator(device=dev).manual_seed(5)
    H, I = Q17["hidden"], Q17["intermediate"]
    shapes = [(2048, H), (1024, H), (1024, H), (H, 2048), (I, H), (I, H), (H, I)]
    mats = []
    for N, K in shapes:
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        mats.append(tb.quantize_int4_bf16(w.view(torch.int16)))
        del w
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    for M in (512, 2048, 8192):
        ms = 0.0
        flop = 0
        for (N, K), (pk, sc) in zip(shapes, mats):
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            y = torch.empty(M, N, device=dev)
            ms += _cold_time(lambda: tb.gemm_q(x, pk, sc, y=y), flush, stream)
            flop += 2 * M * N * K
        tf = flop / (ms * 1e-3) / 1e12
        out["M%d" % M] = {"us_7_matrices": round(ms * 1e3, 1), "tflops": round(tf, 1),
                          "frac_of_bf16_peak": round(tf / peak_tf, 4)}
    del flush
    torch.cuda.synchronize(dev)
    return out


def prefill_exact_extra(dev, peak_tf, stream):
    """The seven Qwen3-1.7B layer matrices as the exact-sum prefill GEMM
    (gemmDP4A, the product's prefill route) on M = 512 / 2048 / 8192 QUANTQ8T rows:
    int8 TOP/s of 2*M*N*K for the tcgen05 kind::i8 kernel and for the warp-level
    mma.sync form of the same arithmetic, cold L2 per launch."""
    import torch
    import tabinfer_b200 as tb
    g = torch.Generator(device=dev).manual_seed(6)
    H, I = Q17["hidden"], Q17["intermediate"]
    shapes = [(2048, H), (1024, H), (1024, H), (H, 2048), (I, H), (I, H), (H, I)]
    mats = []
    for N, K in shapes:
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        mats.append(tb.quantize_int4_bf16(w.view(torch.int16)))
        del w
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    for M in (512, 2048, 8192):
        row = {}
        for form, warp in (("tcgen05", False), ("mma_sync", True)):
            ms = 0.0
            ops = 0
            for (N, K), (pk, sc) in zip(shapes, mats):
                xq = torch.randint(-127, 128, (M, K), device=dev, dtype=torch.int32, generator=g).to(torch.int8)
                xs = torch.rand(M, K // 32, device=dev, generator=g) * 0.01
                y = torch.empty(M, N, device=dev)
                ms += _cold_time(lambda: tb.gemm_dp4(xq, xs, pk, sc, y=y, warp=warp), flush, stream)
                ops += 2 * M * N * K
            tops = ops / (ms * 1e-3) / 1e12
            row[form] = {"us_7_matrices": round(ms * 1e3, 1), "tops": round(tops, 1),
                         "frac_of_bf16_peak": round(tops / peak_tf, 4)}
        row["speedup"] = round(row["mma_sync"]["us_7_matrices"] / row["tcgen05"]["us_7_matrices"], 3)
        out["M%d" % M] = row
    del flush
    torch.cuda.synchronize(dev)
    return out


def moe_extra(dev, peak_gbs, stream, group=32):
    """One LFM2.5-8B-A1B-shaped int3 MoE FFN (hidden 2048, 32 experts, I 1792,
    top-4) over 1 / 8 / 64 tokens: router + grouped expert GEMVs + combine.
    group 32: the reference's _requant43 path (bf16 -> int4 G32 -> int3); group
    128: the configuration's group-128 int3 quantized from bf16 directly.
    Algorithmic bytes = the int3 planes and scales of every expert routed to +
    activations."""
    import torch
    import tabinfer_b200 as tb
    H, I, NE, K = 2048, 1792, 32, 4
    g = torch.Generator(device=dev).manual_seed(11)
    ws = []
    for rows, cols in ((NE * I, H), (NE * I, H), (NE * H, I)):
        w = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        if group == 32:
            pk, sc = tb.quantize_int4_bf16(w.view(torch.int16))
            del w
            ws.append(tb.requant_int3(pk, sc))
            del pk, sc
        else:
            ws.append(tb.quant_int3(w.view(torch.int16), group))
            del w
    per_expert = (2 * I * H + H * I) * 12 // 32 + (2 * I * H + H * I) * 2 // group
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(dev)
    out = {"group": group}
    for T in (1, 8, 64):
        logits = torch.randn(T, NE, device=dev, generator=g)
        bias = torch.zeros(NE, device=dev)
        a = torch.randn(T, H, device=dev, generator=g)
        x = torch.zeros(T, H, device=dev)

        def step():
            idx, wt = tb.moe_router(logits, bias, K)
            tb.moe_ffn_int3(x, a, idx, wt, ws[0], ws[1], ws[2], NE, H, I, group=group)
        step()
        idx, _ = tb.moe_router(logits, bias, K)
        used = len(set(idx.flatten().tolist()))
        ms = _cold_time(step, flush, stream)
        nbytes = used * per_expert + T * H * 4 * 2 + T * K * (I + H) * 4 * 2
        gbs = nbytes / (ms * 1e-3) / 1e9
        out["T%d" % T] = {"us": round(ms * 1e3, 1), "experts_used": used, "bytes": int(nbytes),
                          "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak_gbs, 4)}
    del flush
    torch.cuda.synchronize(dev)
    return out


def moe_ep_extra(dev, world, rank, stream, peak_gbs, dist):
    """Config 5 expert-parallel: the LFM2.5-8B-A1B-shaped int3 MoE FFN (hidden
    2048, 32 experts, I 1792, top-4) with 32/world experts per GPU, every rank
    routing its own 1 / 8 / 64 tokens (tb_moe_ep_forward: dispatch over NVLink
    peer memory, grouped expert GEMVs, outputs written back into the origin,
    combine).  Per forward: median of cold-L2 CUDA-event times on each rank,
    max over ranks.  expert_gbs = int3 planes + scales of the experts this rank
    ran / time (max-loaded rank)."""
    import torch
    import tabinfer_b200 as tb
    H, I, NE, K = 2048, 1792, 32, 4
    El = NE // world
    ws = []
    for j, (rows, cols) in enumerate(((I, H), (I, H), (H, I))):
        g = torch.Generator(device=dev).manual_seed(40 + j)
        w = (torch.randn(NE * rows, cols, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        pk, sc = tb.quantize_int4_bf16(w.view(torch.int16))
        del w
        p3, s3 = tb.requant_int3(pk, sc)
        del pk, sc
        ws.append((p3[rank * El * rows:(rank + 1) * El * rows].clone(), s3[rank * El * rows:(rank + 1) * El * rows].clone()))
        del p3, s3
    per_expert = (2 * I * H + H * I) * 14 // 32
    ep = tb.MoeEP(world, rank, NE, K, H, I, 64, device=dev.index)
    if world > 1:
        mine = torch.frombuffer(bytearray(ep.handle()), dtype=torch.uint8).to(dev)
        allh = [torch.zeros(64, dtype=torch.uint8, device=dev) for _ in range(world)]
        dist.all_gather(allh, mine)
        ep.connect([bytes(h.cpu().numpy().tobytes()) for h in allh])
    ep.set_experts(*ws)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {"experts_per_gpu": El, "gpus": world}
    for T in (1, 8, 64):
        g = torch.Generator(device=dev).manual_seed(1000 + 17 * rank + T)
        logits = torch.randn(T, NE, device=dev, generator=g)
        a = torch.randn(T, H, device=dev, generator=g)
        x = torch.zeros(T, H, device=dev)
        idx, wt = tb.moe_router(logits, torch.zeros(NE, device=dev), K)
        ids = idx.flatten().tolist()
        mine_used = len({e for e in ids if e // El == rank})
        ts = []
        for r in range(25):
            flush.fill_(r & 0xff)
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ep.forward(x, a, idx, wt)
            e1.record(stream)
            e1.synchronize()
            if r >= 5:
                ts.append(e0.elapsed_time(e1))
        ms = statistics.median(ts)
        ms_max, used_max = ms, mine_used
        if world > 1:
            t = torch.tensor([ms, float(mine_used)], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_max, used_max = float(t[0]), int(t[1])
        gbs = used_max * per_expert / (ms_max * 1e-3) / 1e9
        out["T%d_per_gpu" % T] = {"us": round(ms_max * 1e3, 1), "tokens_per_s": round(world * T / (ms_max * 1e-3), 1),
                                  "experts_on_busiest_gpu": used_max, "expert_gbs": round(gbs, 1),
                                  "frac_of_peak": round(gbs / peak_gbs, 4)}
    err = ep.ctx.device_error()
    assert err == 0, "moe ep device error 0x%x" % err
    ep.close()
    del flush, ws
    torch.cuda.synchronize(dev)
    return out


def _tern_weights(dev, g, N, K):
    """A ternary bf16 matrix (per 32-group {-m, 0, +m}) packed on the device in the
    WebGPU layout (quantizeTernaryBf16)."""
    import torch
    import tabinfer_b200 as tb
    mag = (torch.rand(N, K // 32, device=dev, generator=g) * 0.05 + 0.005).view(torch.int32) >> 16
    t = torch.randint(-1, 2, (N, K), device=dev, generator=g, dtype=torch.int32)
    bits = torch.where(t == 0, torch.zeros_like(t), mag.repeat_interleave(32, dim=1) | ((t < 0).int() << 15))
    w = torch.where(bits >= 32768, bits - 65536, bits).to(torch.int16)
    del t, bits, mag
    r = tb.quantize_tern_bf16(w)
    assert r is not None
    return r


def tern_extra(dev, peak_gbs, peak_tf, stream):
    """Ternary weights in the WebGPU layout at Bonsai-1.7B shapes (Qwen3-1.7B
    architecture): the batch-1 decode GEMVs (quantQ8 fused, weights from HBM) with their
    algorithmic bytes (codes K/4 + f16 scales K/16 bytes a row, f32 activation in,
    f32 out), and the prefill GEMM on 2048 rows (2*M*N*K flops)."""
    import torch
    import tabinfer_b200 as tb
    g = torch.Generator(device=dev).manual_seed(21)
    H, I, V = Q17["hidden"], Q17["intermediate"], Q17["vocab"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    mats = {n: _tern_weights(dev, g, N, K) for n, (N, K) in
            {"q": (2048, H), "k": (1024, H), "v": (1024, H), "o": (H, 2048), "gate": (I, H), "up": (I, H),
             "down": (H, I), "lm_head": (V, H)}.items()}

    def tb_bytes(N, K, nact=1):
        return N * K // 4 + N * K // 16 + nact * K * 4 + N * 4

    x = torch.randn(1, H, device=dev, generator=g)
    xi = torch.randn(1, I, device=dev, generator=g)
    ys = {n: torch.empty(1, p.shape[0], device=dev) for n, (p, _) in mats.items()}
    swi = torch.empty(1, I, device=dev)
    # case: (matrix shapes of one copy, the launch on a copy, algorithmic bytes a launch)
    cases = {
        "qkv": ([(2048, H), (1024, H), (1024, H)],
                lambda c: tb.gemv_tern_wgsl_dp4a_multi(x, c, ys=[ys["q"], ys["k"], ys["v"]]),
                tb_bytes(2048, H) + 2 * tb_bytes(1024, H)),
        "o": ([(H, 2048)], lambda c: tb.linear_tern_wgsl(x, *c[0], y=ys["o"]), tb_bytes(H, 2048)),
        "gateup": ([(I, H), (I, H)], lambda c: tb.gate_up_silu_tern_dp4a(x, *c[0], *c[1], swi=swi),
                   2 * tb_bytes(I, H)),
        "down": ([(H, I)], lambda c: tb.linear_tern_wgsl(xi, *c[0], y=ys["down"]), tb_bytes(H, I)),
        "lm_head": ([(V, H)], lambda c: tb.linear_tern_wgsl(x, *c[0], y=ys["lm_head"]), tb_bytes(V, H)),
    }
    # one recorded batch of back-to-back launches, each on its own copy of the
    # weights, the copies together at least twice the L2 (every launch streams from
    # HBM, as in decode); CUDA events around replays, divided by the launches
    import math
    from tabinfer_b200._lib import LIB
    ctx = tb.default_context(dev.index)
    tot_ms = tot_b = 0.0
    for name, (shp, fn, nbytes) in cases.items():
        nc = max(4, int(math.ceil(2 * (126 << 20) / nbytes)))
        copies = [[_tern_weights(dev, g, N, K) for N, K in shp] for _ in range(nc)]
        fn(copies[0])                       # any first-call set-up happens before recording
        torch.cuda.synchronize(dev)
        h, st = _record_batch(ctx, dev, lambda: [fn(c) for c in copies])
        ms = _replay_ms(ctx, h, st, 5) / nc
        LIB.tb_batch_destroy(h)
        del copies
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"us": round(ms * 1e3, 3), "bytes": int(nbytes), "gbs": round(gbs, 1),
                     "frac_of_peak": round(gbs / peak_gbs, 4),
                     "timing": "%d back-to-back launches on %d weight copies (> 2x L2), recorded, CUDA events" % (nc, nc)}
        if name != "lm_head":
            tot_ms += ms
            tot_b += nbytes
    out["layer_gemvs"] = {"us": round(tot_ms * 1e3, 2), "gbs": round(tot_b / (tot_ms * 1e-3) / 1e9, 1),
                          "frac_of_peak": round(tot_b / (tot_ms * 1e-3) / 1e9 / peak_gbs, 4)}
    M = 2048
    ms = flop = 0.0
    for n in ("q", "k", "v", "o", "gate", "up", "down"):
        pk, sc = mats[n]
        N, K = pk.shape[0], pk.shape[1] * 16
        xq = torch.randint(-127, 128, (M, K), device=dev, generator=g, dtype=torch.int32).to(torch.int8)
        xs = torch.rand(M, K // 32, device=dev, generator=g) * 0.01
        y = torch.empty(M, N, device=dev)
        ms += _cold_time(lambda: tb.gemm_tern(xq, xs, pk, sc, y=y), flush, stream)
        flop += 2 * M * N * K
    tf = flop / (ms * 1e-3) / 1e12
    out["prefill_M2048"] = {"us_7_matrices": round(ms * 1e3, 1), "tflops": round(tf, 1),
                            "frac_of_bf16_peak": round(tf / peak_tf, 4)}
    del flush, mats
    torch.cuda.synchronize(dev)
    return out


# ---------------------------------------------------------------------------
# ternary Q2_0_g64 decode GEMV: the Bonsai-1.7B layer matrices in the
# n2-core binfmt layout, on the B200 and on the host cores
# ---------------------------------------------------------------------------
BONSAI_MATS = [("qkv", 4096, 2048), ("o", 2048, 2048), ("gate", 6144, 2048), ("up", 6144, 2048),
               ("down", 2048, 6144)]
BONSAI_LAYERS = 28


def q2g64_bytes(N, K, B=1):
    """Q2_0_g64 GEMV algorithmic bytes: 2-bit codes (K/4 bytes a row) and one f32
    scale per 64 read once, B int8 activation rows with their i32 sums per 64 in,
    B f32 rows out (0.3125 B a weight + activations)."""
    return N * K // 4 + N * (K // 64) * 4 + B * (K + (K // 64) * 4 + N * 4)


def _q2g64_pack(dev, g, N, K):
    """configs[0] weights: t in {-1, 0, +1} with p = 1/3 each times a per-64-group
    scale U(0.01, 0.05) rounded to f16, packed by the product's tb_pack_tern_q2g64
    (tern.rs pack_ternary): codes t + 1, scales s exactly."""
    import torch
    import tabinfer_b200 as tb
    t = torch.randint(0, 3, (N, K), device=dev, generator=g, dtype=torch.int32).float() - 1.0
    s = (torch.rand(N, K // 64, device=dev, generator=g) * 0.04 + 0.01).half().float()
    w = t * s.repeat_interleave(64, dim=1)
    del t
    return tb.pack_ternary(w)


def _record_batch(ctx, dev, fn):
    """fn's launches recorded once as a replayable tb_batch on the context's own
    stream (so the timed replays are not bound by Python launch overhead)."""
    import torch
    from tabinfer_b200._lib import LIB, P
    # the context's own stream does not wait for torch's: inputs made there
    # (weights, activations) must be complete before anything is recorded or timed
    torch.cuda.synchronize(dev)
    stream = torch.cuda.ExternalStream(ctx.own_stream(), device=dev)
    with torch.cuda.stream(stream):
        fn()
        stream.synchronize()
        ctx.check(LIB.tb_batch_begin(ctx.h), "batch_begin")
        fn()
        h = P()
        ctx.check(LIB.tb_batch_end(ctx.h, ctypes.byref(h)), "batch_end")
    return h, stream


def _replay_ms(ctx, h, stream, reps):
    """ms per replay of a recorded batch: CUDA events on its stream around `reps`
    back-to-back replays, after three untimed ones."""
    import torch
    from tabinfer_b200._lib import LIB
    for _ in range(3):
        ctx.check(LIB.tb_batch_submit(ctx.h, h), "submit")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        ctx.check(LIB.tb_batch_submit(ctx.h, h), "submit")
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def q2g64_extra(dev, ctx, peak_gbs):
    """configs[0] on the B200: tb_gemv_tern_q2g64 (batch 1) over the Bonsai-1.7B
    layer matrices.  28 layer copies (440 MB, > 3x L2) are swept in order, each
    matrix one launch, recorded once and replayed; a launch therefore reads its
    weights from HBM, as in decode.  Also the kernel alone on a 151936 x 2048
    (lm_head-sized) matrix, rotated over three copies."""
    import torch
    import tabinfer_b200 as tb
    from tabinfer_b200._lib import LIB
    g = torch.Generator(device=dev).manual_seed(31)
    layers = [{n: _q2g64_pack(dev, g, N, K) for n, N, K in BONSAI_MATS} for _ in range(BONSAI_LAYERS)]
    acts = {}
    for K in sorted({K for _, _, K in BONSAI_MATS} | {Q17["hidden"]}):
        x = torch.randn(1, K, device=dev, generator=g)
        acts[K] = tb.quantize_act(x)[:2]
    outs = {n: torch.empty(1, N, device=dev) for n, N, _ in BONSAI_MATS}
    dims = {n: (N, K) for n, N, K in BONSAI_MATS}
    torch.cuda.synchronize(dev)

    def gemv(name, L):
        codes, scales = L[name]
        act, xsum = acts[dims[name][1]]
        tb.gemv_tern(codes, scales, act, xsum, out=outs[name])

    res = {}
    reps = 30
    h, stream = _record_batch(ctx, dev, lambda: [gemv(n, L) for L in layers for n, _, _ in BONSAI_MATS])
    ms = _replay_ms(ctx, h, stream, reps)
    LIB.tb_batch_destroy(h)
    lb = sum(q2g64_bytes(N, K) for _, N, K in BONSAI_MATS)
    gbs = lb * BONSAI_LAYERS / (ms * 1e-3) / 1e9
    macs = sum(N * K for _, N, K in BONSAI_MATS)
    res["layer_sweep"] = {"us_per_layer": round(ms * 1e3 / BONSAI_LAYERS, 3), "bytes_per_layer": lb,
                          "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak_gbs, 4),
                          "gmacs": round(macs * BONSAI_LAYERS / (ms * 1e-3) / 1e9, 1),
                          "launches_per_layer": len(BONSAI_MATS)}
    per = {}
    for n, N, K in BONSAI_MATS:
        h, stream = _record_batch(ctx, dev, lambda: [gemv(n, L) for L in layers])
        msn = _replay_ms(ctx, h, stream, reps) / BONSAI_LAYERS
        LIB.tb_batch_destroy(h)
        b = q2g64_bytes(N, K)
        per[n] = {"N": N, "K": K, "us": round(msn * 1e3, 3), "bytes": b, "gbs": round(b / (msn * 1e-3) / 1e9, 1),
                  "frac_of_peak": round(b / (msn * 1e-3) / 1e9 / peak_gbs, 4),
                  "gmacs": round(N * K / (msn * 1e-3) / 1e9, 1)}
    res["per_matrix"] = per
    del layers
    torch.cuda.synchronize(dev)
    V, H = Q17["vocab"], Q17["hidden"]
    big = [_q2g64_pack(dev, g, V, H) for _ in range(3)]
    yb = torch.empty(1, V, device=dev)
    act, xsum = acts[H]
    torch.cuda.synchronize(dev)
    h, stream = _record_batch(ctx, dev, lambda: [tb.gemv_tern(c, s, act, xsum, out=yb) for c, s in big])
    msb = _replay_ms(ctx, h, stream, 20) / 3
    LIB.tb_batch_destroy(h)
    b = q2g64_bytes(V, H)
    res["lm_head_151936x2048"] = {"us": round(msb * 1e3, 2), "bytes": b, "gbs": round(b / (msb * 1e-3) / 1e9, 1),
                                  "frac_of_peak": round(b / (msb * 1e-3) / 1e9 / peak_gbs, 4)}
    del big
    torch.cuda.synchronize(dev)
    res["timing"] = ("recorded launches replayed back to back (PDL on), CUDA events on the launching stream; weights "
                     "rotated over > 2x L2 (28 layer copies, 3 lm_head copies); bytes = 0.3125 B a weight + int8 "
                     "activation, i32 sums and f32 output")
    return res


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _llc_bytes():
    try:
        v = os.sysconf("SC_LEVEL3_CACHE_SIZE")
        if v and v > 0:
            return int(v)
    except (ValueError, OSError):
        pass
    return 64 << 20


def cpu_q2g64(budget_s=12.0):
    """configs[0] on the host cores: the reference's ternary GEMV backends,
    transcribed to C (oracle/tb_cpu_ref.c: tern.rs scalar :100-140 and AVX2
    :268-338), over the same Bonsai-1.7B layer matrices.  The weight copies
    together exceed 4x the last-level cache (DRAM-streaming, the regime
    native/docs/ROADMAP.md:11-27 says predicts decode).  Discipline of
    n2-kernels/src/timing.rs: warm-up, alternating order every repetition, min
    over repetitions, and a base-vs-base control whose ratio must read ~1.000."""
    import itertools
    import oracle
    lib = oracle.cpuref()
    rng = np.random.default_rng(0x9E3779B9)
    lut = np.array([a | (b << 2) | (c << 4) | (d << 6) for a, b, c, d in itertools.product(range(3), repeat=4)],
                   np.uint8)
    layer_b = sum(q2g64_bytes(N, K) for _, N, K in BONSAI_MATS)
    ws = min(max(256 << 20, 4 * _llc_bytes()), 640 << 20)
    nl = max(2, -(-ws // layer_b))
    mats = []
    for _ in range(nl):
        for n, N, K in BONSAI_MATS:
            codes = lut[rng.integers(0, 81, N * K // 4, dtype=np.uint8)]
            scales = np.float16(rng.uniform(0.01, 0.05, N * (K // 64))).astype(np.float32)
            mats.append((N, K, codes, scales))
    acts = {}
    for K in {K for _, _, K in BONSAI_MATS}:
        acts[K] = (rng.integers(-127, 128, K).astype(np.int8), rng.integers(-2000, 2000, K // 64).astype(np.int32))
    outs = {N: np.zeros(N, np.float32) for _, N, _ in BONSAI_MATS}
    P = ctypes.c_void_p
    threads_all = os.cpu_count() or 1

    def sweep(fn, threads):
        t0 = time.perf_counter()
        for N, K, codes, scales in mats:
            act, xsum = acts[K]
            fn(P(outs[N].ctypes.data), P(codes.ctypes.data), P(scales.ctypes.data), P(act.ctypes.data),
               P(xsum.ctypes.data), ctypes.c_int64(N), ctypes.c_int64(K), ctypes.c_int(threads))
        return time.perf_counter() - t0

    variants = [("avx2_1t", lib.tbr_gemv_tern_avx2, 1), ("avx2_1t_control", lib.tbr_gemv_tern_avx2, 1),
                ("scalar_1t", lib.tbr_gemv_tern_scalar, 1), ("avx2_all", lib.tbr_gemv_tern_avx2, threads_all)]
    for _, fn, th in variants:          # warm-up
        sweep(fn, th)
    best = {v[0]: float("inf") for v in variants}
    reps = 0
    t0 = time.perf_counter()
    while reps < 3 or (time.perf_counter() - t0 < budget_s and reps < 50):
        order = variants if reps % 2 == 0 else variants[::-1]
        for name, fn, th in order:
            best[name] = min(best[name], sweep(fn, th))
        reps += 1
    macs = sum(N * K for N, K, _, _ in mats)
    nbytes = sum(q2g64_bytes(N, K) for N, K, _, _ in mats)
    out = {}
    for name, _, th in variants:
        if name == "avx2_1t_control":
            continue
        out[name] = {"threads": th, "gmacs": round(macs / best[name] / 1e9, 2),
                     "gbs": round(nbytes / best[name] / 1e9, 2), "ms_per_layer": round(best[name] * 1e3 / nl, 3)}
    out["control_ratio"] = round(best["avx2_1t"] / best["avx2_1t_control"], 3)
    out.update({"kind": "port", "reps": reps, "layer_copies": nl, "working_set_mb": round(nbytes / 2 ** 20, 1),
                "cpu_model": _cpu_model(), "nproc": threads_all,
                "reference_published": "AVX2 1 thread DRAM-streaming 15.32 GMAC/s ~ 4.8 GB/s, scalar 2.69 GMAC/s "
                                       "(i5-1235U, native/docs/ROADMAP.md:17-25)",
                "sample": "the 5 Bonsai-1.7B layer GEMVs over %d layer copies per repetition, min of %d "
                          "alternating-order repetitions" % (nl, reps)})
    return out


# ---------------------------------------------------------------------------
# profiling cases (for ncu on a small case)
# ---------------------------------------------------------------------------

def profile_case():
    """One cold-L2 launch of each kernel kind of the 1.7B step at batch 1 (TP 1):
    the four per-layer GEMV kinds, the f32 lm_head, the config-1 ternary qkv
    GEMV (4096 x 2048) and decode attention at S=4096.  Every launch is preceded
    by a 256 MB write that evicts L2; two passes."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    H, hd, I, V = Q17["hidden"], Q17["head_dim"], Q17["intermediate"], Q17["vocab"]

    def q(N, K):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        return tb.quantize_int4_bf16(w.view(torch.int16))

    qm, km, vm, om = q(2048, H), q(1024, H), q(1024, H), q(H, 2048)
    gm, um, dm, lm = q(I, H), q(I, H), q(H, I), q(V, H)
    ln = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half().view(torch.int16)
    tw = (torch.randint(0, 3, (4096, 2048), device=dev, generator=g).float() - 1.0) * 0.03
    codes, tsc = tb.pack_ternary(tw)
    S, nHq, nKv = 4096, 16, 8
    Kq = torch.randint(-127, 128, (S, nKv * hd), device=dev, generator=g, dtype=torch.int8)
    Vq = torch.randint(-127, 128, (S, nKv * hd), device=dev, generator=g, dtype=torch.int8)
    Ks = torch.rand(S, nKv * hd // 32, device=dev, generator=g) + 0.5
    Vs = torch.rand(S, nKv * hd // 32, device=dev, generator=g) + 0.5
    qr = torch.randn(nHq * hd, device=dev, generator=g)
    x1, x2, x3 = (torch.randn(1, k, device=dev, generator=g) for k in (H, 2048, I))
    xt = torch.randn(1, 2048, device=dev, generator=g)
    act, xsum, _ = tb.quantize_act(xt)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    launches = [
        lambda: tb.gemv_dp4a_multi(x1, [qm, km, vm], norm_w=ln),
        lambda: tb.gemv_dp4a(x2, *om),
        lambda: tb.gate_up_silu_dp4a(x1, *gm, *um, norm_w=ln),
        lambda: tb.gemv_dp4a(x3, *dm),
        lambda: tb.gemv_q_norm(x1, ln, 1e-6, *lm),
        lambda: tb.gemv_tern(codes, tsc, act, xsum),
        lambda: tb.attention_decode_q8(qr, (Kq, Ks, Vq, Vs), S, nHq, nKv, hd),
    ]
    torch.cuda.synchronize()
    for it in range(2):
        for fn in launches:
            flush.fill_(it)
            fn()
    torch.cuda.synchronize()
    assert tb.default_context(0).device_error() == 0
    print("profile case done", flush=True)


def profile_attn(S):
    """Three cold-L2 launches of int8-KV decode attention at context S (Qwen3-1.7B
    heads: 16 q / 8 kv, hd 128; auto split count), for an ncu capture of one."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    nHq, nKv, hd = 16, 8, 128
    Kq = torch.randint(-127, 128, (S, nKv * hd), device=dev, generator=g, dtype=torch.int8)
    Vq = torch.randint(-127, 128, (S, nKv * hd), device=dev, generator=g, dtype=torch.int8)
    Ks = torch.rand(S, nKv * hd // 32, device=dev, generator=g) + 0.5
    Vs = torch.rand(S, nKv * hd // 32, device=dev, generator=g) + 0.5
    qr = torch.randn(nHq * hd, device=dev, generator=g)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for it in range(3):
        flush.fill_(it)
        tb.attention_decode_q8(qr, (Kq, Ks, Vq, Vs), S, nHq, nKv, hd)
    torch.cuda.synchronize()
    err = tb.default_context(0).device_error()
    assert err == 0, err
    print("profile attn done", flush=True)


def profile_decode(context, batch=1):
    """Three recorded Qwen3-1.7B decode steps (`batch` sequences) at the given
    context on one GPU, for an ncu launch list of one step."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    m = build_model(Q17, dev, batch, context, 16, 1, 0)
    m.set_tokens([(1000 + 7919 * b) % Q17["vocab"] for b in range(batch)], [context - 1] * batch)
    for _ in range(3):
        m.step()
    torch.cuda.synchronize()
    kernels, _ = m.launches_per_step()
    err = tb.default_context(0).device_error()
    assert err == 0, err
    m.close()
    print("profile decode done: %d kernels per step" % kernels, flush=True)


def profile_step(layers):
    """The persistent decode step of a Qwen3-1.7B-width model with `layers` layers
    (context 4096, batch 1): one recorded step, then three launches of the
    persistent kernel alone, for an ncu capture of one of them."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    m = build_model(dict(Q17, layers=layers), dev, 1, 4096, 16, 1, 0)
    m.set_tokens([1000], [4095])
    m.step()
    assert m.step_kind() == 2, "the persistent step does not apply"
    for _ in range(3):
        m.step_layers()
    torch.cuda.synchronize()
    err = tb.default_context(0).device_error()
    assert err == 0, err
    m.close()
    print("profile step done", flush=True)


def profile_moe(T):
    """Three int3 MoE layers (config 5 shapes: router, grouping, grouped gate/up
    and down GEMVs, combine) over T tokens, for an ncu launch list."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    H, I, NE, K = 2048, 1792, 32, 4
    ws = []
    for j, (rows, cols) in enumerate(((NE * I, H), (NE * I, H), (NE * H, I))):
        g = torch.Generator(device=dev).manual_seed(11 + j)
        w = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        pk, sc = tb.quantize_int4_bf16(w.view(torch.int16))
        del w
        ws.append(tb.requant_int3(pk, sc))
    g = torch.Generator(device=dev).manual_seed(5)
    logits = torch.randn(T, NE, device=dev, generator=g)
    bias = torch.zeros(NE, device=dev)
    a = torch.randn(T, H, device=dev, generator=g)
    x = torch.zeros(T, H, device=dev)
    for _ in range(3):
        idx, wt = tb.moe_router(logits, bias, K)
        tb.moe_ffn_int3(x, a, idx, wt, ws[0], ws[1], ws[2], NE, H, I)
    torch.cuda.synchronize()
    print("profile moe done", flush=True)


def profile_gemm(M, N, K):
    """Three cold-L2 launches of the tcgen05 prefill GEMM (bf16 activations) at
    M x N x K (config 4: M in {512, 2048, 8192}), for an ncu capture of one."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    pack, sc = tb.quantize_int4_bf16(w.view(torch.int16))
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty(M, N, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for it in range(3):
        flush.fill_(it)
        tb.gemm_q(x, pack, sc, y=y)
    torch.cuda.synchronize()
    err = tb.default_context(0).device_error()
    assert err == 0, err
    print("profile gemm done", flush=True)


def bonsai_extra(dev, peak_gbs, stream, context=4096):
    """Bonsai-1.7B (the Qwen3-1.7B architecture with ternary projections and
    lm_head, loaded as ternary WebGPU-layout records) through the recorded
    decode step: tok/s at batch 1, context 4096."""
    import torch
    from tabinfer_b200 import _lib as _tl
    steps = 50
    m = build_model(Q17, dev, 1, context, steps + 16, 1, 0, seed=77, ternary=True)
    for _ in range(5):
        m.set_tokens([1000], [context - 1])
        m.step()
    m.set_tokens([1000], [context - 1])        # every timed step inside the cache
    torch.cuda.synchronize(dev)
    ms = time_steps(m, steps, stream) / steps
    err = m.ctx.device_error()
    assert err == 0, "bonsai decode device error 0x%x" % err
    kind = {_tl.QW_STEP_KERNELS: "kernels", _tl.QW_STEP_PERSISTENT: "persistent"}.get(m.step_kind(), "?")
    # the same step as one kernel per operation, for comparison
    m.set_step_mode(_tl.QW_STEP_KERNELS)
    for _ in range(3):
        m.set_tokens([1000], [context - 1])
        m.step()
    m.set_tokens([1000], [context - 1])
    torch.cuda.synchronize(dev)
    ms_k = time_steps(m, steps, stream) / steps
    err = m.ctx.device_error()
    assert err == 0, "bonsai decode (kernels) device error 0x%x" % err
    nb = step_bytes(Q17, 1, 1, context, tern=True)
    kinds = sorted({m.weight_format(n) for n in ("lm_head.weight", "model.layers.0.mlp.down_proj.weight")})
    m.close()
    torch.cuda.synchronize(dev)
    return {"tok_per_s": round(1e3 / ms, 1), "ms_per_step": round(ms, 4), "step_kind": kind,
            "tok_per_s_one_kernel_per_op": round(1e3 / ms_k, 1), "bytes_per_step": int(nb),
            "step_hbm_gbs": round(nb / (ms * 1e-3) / 1e9, 1), "frac_of_peak": round(nb / (ms * 1e-3) / 1e9 / peak_gbs, 4),
            "weight_formats": kinds, "reference_webgpu_tok_per_s": "21.7 (Iris Xe)"}


def prefill_forward_extra(dev, stream, T=2048):
    """forward(ids, 0) at T tokens (tb_qwen3_prefill) of Qwen3-1.7B, int4 weights:
    prompt tokens per second, one sequence (exact-sum GEMMs, int8-KV prefill
    attention, T-row KV writes, last-row lm_head)."""
    import torch
    m = build_model(Q17, dev, 1, T + 16, 16, 1, 0, seed=91)
    ids = list(np.random.default_rng(3).integers(0, Q17["vocab"], T))
    m.prefill(0, ids, 0)                       # buffers, warm-up
    ts = []
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.prefill(0, ids, 0)
        e1.record(stream)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    m.close()
    torch.cuda.synchronize(dev)
    ms = statistics.median(ts)
    return {"tokens": T, "ms": round(ms, 3), "tok_per_s": round(T / (ms * 1e-3), 1)}


def prefill_forward_tp_extra(dev, stream, world, rank, dist, T=2048):
    """forward(ids, 0) at T tokens of Qwen3-1.7B tensor-parallel over the world
    (column-split q/k/v and gate/up, row-split o/down with an NCCL allreduce of
    the prompt rows after each, vocab-split lm_head): prompt tokens per second,
    device time max over ranks.  Every rank runs every step."""
    import torch
    from tabinfer_b200.qwen3 import nccl_unique_id
    m = build_model(Q17, dev, 1, T + 16, 16, world, rank, seed=91)
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    m.tp_init(bytes(uid.cpu().numpy().tobytes()))
    ids = list(np.random.default_rng(3).integers(0, Q17["vocab"], T))
    m.prefill(0, ids, 0)
    torch.cuda.synchronize(dev)
    ts = []
    for _ in range(3):
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.prefill(0, ids, 0)
        e1.record(stream)
        e1.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ts.append(float(t.item()))
    err = m.ctx.device_error()
    m.close()
    del m
    torch.cuda.synchronize(dev)
    ms = statistics.median(ts)
    return {"tokens": T, "tp": world, "ms": round(ms, 3), "tok_per_s": round(T / (ms * 1e-3), 1),
            "device_error": err, "timing": "CUDA events per rank, max over ranks, median of 3"}


def prefill_attn_extra(dev, peak_tf, stream):
    """int8-KV prefill attention of one Qwen3-1.7B layer (16 q / 8 kv heads of
    128) over T = S = 512 / 2048 / 8192: TFLOP/s of the causal 4 * pairs * hd * heads."""
    import torch
    import tabinfer_b200 as tb
    g = torch.Generator(device=dev).manual_seed(9)
    nHq, nKv, hd = Q17["n_heads"], Q17["n_kv_heads"], Q17["head_dim"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    for T in (512, 2048, 8192):
        S = T
        Kq = torch.randint(-127, 128, (S, nKv * hd), device=dev, dtype=torch.int32, generator=g).to(torch.int8)
        Vq = torch.randint(-127, 128, (S, nKv * hd), device=dev, dtype=torch.int32, generator=g).to(torch.int8)
        Ks = torch.rand(S, nKv * hd // 32, device=dev, generator=g) * 0.02
        Vs = torch.rand(S, nKv * hd // 32, device=dev, generator=g) * 0.02
        q = torch.randn(T, nHq * hd, device=dev, generator=g)
        o = torch.empty(T, nHq * hd, device=dev)
        ms = _cold_time(lambda: tb.attention_prefill_q8(q, (Kq, Ks, Vq, Vs), S, nHq, nKv, hd, out=o), flush, stream)
        fl = 4 * (T * (T + 1) / 2) * hd * nHq
        tf = fl / (ms * 1e-3) / 1e12
        out["T%d" % T] = {"us": round(ms * 1e3, 1), "tflops": round(tf, 1), "frac_of_bf16_peak": round(tf / peak_tf, 4)}
    del flush
    torch.cuda.synchronize(dev)
    return out


def profile_prefill_attn(T):
    """Three launches of the int8-KV prefill attention of one Qwen3-1.7B layer at
    T = S tokens (cold L2 before each), for an ncu capture of one."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    nHq, nKv, hd = Q17["n_heads"], Q17["n_kv_heads"], Q17["head_dim"]
    Kq = torch.randint(-127, 128, (T, nKv * hd), device=dev, dtype=torch.int32, generator=g).to(torch.int8)
    Vq = torch.randint(-127, 128, (T, nKv * hd), device=dev, dtype=torch.int32, generator=g).to(torch.int8)
    Ks = torch.rand(T, nKv * hd // 32, device=dev, generator=g) * 0.02
    Vs = torch.rand(T, nKv * hd // 32, device=dev, generator=g) * 0.02
    q = torch.randn(T, nHq * hd, device=dev, generator=g)
    o = torch.empty(T, nHq * hd, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for it in range(3):
        flush.fill_(it)
        tb.attention_prefill_q8(q, (Kq, Ks, Vq, Vs), T, nHq, nKv, hd, out=o)
    torch.cuda.synchronize()
    assert tb.default_context(0).device_error() == 0
    print("profile prefill attention done", flush=True)


def profile_gemm_dp4(M, N, K):
    """Three launches of the exact-sum prefill GEMM (gemmDP4A) at M x N x K."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    pack, sc = tb.quantize_int4_bf16(w.view(torch.int16))
    xq = torch.randint(-127, 128, (M, K), device=dev, dtype=torch.int32, generator=g).to(torch.int8)
    xs = torch.rand(M, K // 32, device=dev, generator=g) * 0.01
    y = torch.empty(M, N, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for it in range(3):
        flush.fill_(it)
        tb.gemm_dp4(xq, xs, pack, sc, y=y)
    torch.cuda.synchronize()
    assert tb.default_context(0).device_error() == 0
    print("profile gemm_dp4 done", flush=True)


def profile_prefill(T):
    """Two T-token prefill forwards of Qwen3-1.7B (random int4 weights), for an ncu
    launch list of the second (the first also sizes every buffer)."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    m = build_model(Q17, dev, 1, T + 16, 16, 1, 0, seed=91)
    ids = list(np.random.default_rng(3).integers(0, Q17["vocab"], T))
    for _ in range(2):
        m.prefill(0, ids, 0)
        torch.cuda.synchronize(dev)
    m.close()
    print("profile prefill done", flush=True)


def profile_lm_head(kind):
    """Three cold-L2 lm_head GEMVs (151936 x 2048, RMSNorm fused) of one weight
    kind -- int4_f32 (gemvQ, batch 1), int4_dp4a (rmsnormQ + gemvDP4, batch 1),
    tern (ternary WebGPU layout, batch 1) or int4_mma16 (16 rows on the tensor
    cores: one quantization launch, then the GEMV) -- for an ncu capture of one."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    N, K = Q17["vocab"], Q17["hidden"]
    if kind == "tern":
        pack, sc = _tern_weights(dev, g, N, K)
    else:
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        pack, sc = tb.quantize_int4_bf16(w.view(torch.int16))
        del w
    nw = (1 + 0.1 * torch.randn(K, device=dev, generator=g)).half().view(torch.int16)
    B = 16 if kind == "int4_mma16" else 1
    x = torch.randn(B, K, device=dev, generator=g)
    y = torch.empty(B, N, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for it in range(3):
        flush.fill_(it)
        if kind == "int4_f32":
            tb.gemv_q_norm(x, nw, 1e-6, pack, sc, y=y)
        elif kind == "int4_dp4a":
            tb.gemv_dp4a(x, pack, sc, norm_w=nw, y=y)
        elif kind == "int4_mma16":
            tb.gemv_mma(x, pack, sc, norm_w=nw, y=y)
        else:
            tb.gemv_tern_wgsl_dp4a_multi(x, [(pack, sc)], norm_w=nw, ys=[y])
    torch.cuda.synchronize()
    err = tb.default_context(0).device_error()
    assert err == 0, err
    print("profile lm_head %s done" % kind, flush=True)


# ---------------------------------------------------------------------------
# CPU path (the reference's int4 linearQ math, C transcription)
# ---------------------------------------------------------------------------

def cpu_step_seconds(threads, budget_s, cfg=Q17):
    """Seconds per decode token of the transcribed CPU GEMV path
    (oracle/tb_cpu_ref.c: linearQ's DP4A math for N < 16384, gemvQ's f32 math
    for the lm_head), measured on a bounded sample -- 2 of the 28 layers' seven
    matrices and 1/16 of the lm_head rows, repeated for `budget_s` -- and scaled
    to the whole step.  Attention is not included (the reference has no CPU
    int8-KV attention on this path), so the CPU rate is an upper bound."""
    import numpy as np
    import oracle
    lib = oracle.cpuref()
    rng = np.random.default_rng(7)
    H, I, V = cfg["hidden"], cfg["intermediate"], cfg["vocab"]
    nq, nkv = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    shapes = [(nq, H), (nkv, H), (nkv, H), (H, nq), (I, H), (I, H), (H, I)]
    mats = []
    for _ in range(2):
        for N, K in shapes:
            mats.append((N, K, rng.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint32),
                         np.float16(rng.uniform(0.001, 0.004, (N, K // 32))).view(np.uint16), False))
    Nl = V // 16
    mats.append((Nl, H, rng.integers(0, 2 ** 32, (Nl, H // 8), dtype=np.uint32),
                 np.float16(rng.uniform(0.001, 0.004, (Nl, H // 32))).view(np.uint16), True))
    P = ctypes.c_void_p
    Kmax = max(m[1] for m in mats)
    xs = {m[1]: rng.normal(0, 1, m[1]).astype(np.float32) for m in mats}
    xq = np.zeros(Kmax, np.int8)
    xsc = np.zeros(Kmax // 32, np.float32)
    ys = [np.zeros(m[0], np.float32) for m in mats]
    t_layers = t_lm = 0.0
    reps = 0
    t0 = time.perf_counter()
    while True:
        for (N, K, pk, sc, is_lm), y in zip(mats, ys):
            ta = time.perf_counter()
            if is_lm:
                lib.tbr_gemv_int4_f32(P(y.ctypes.data), P(xs[K].ctypes.data), P(pk.ctypes.data), P(sc.ctypes.data),
                                      ctypes.c_int64(N), ctypes.c_int64(K), ctypes.c_int(0), ctypes.c_int(threads))
                t_lm += time.perf_counter() - ta
            else:
                lib.tbr_linear_int4(P(y.ctypes.data), P(xs[K].ctypes.data), P(pk.ctypes.data), P(sc.ctypes.data),
                                    ctypes.c_int64(N), ctypes.c_int64(K), ctypes.c_int(0), P(xq.ctypes.data),
                                    P(xsc.ctypes.data), ctypes.c_int(threads))
                t_layers += time.perf_counter() - ta
        reps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    per_step = (t_layers / reps) * (cfg["layers"] / 2) + (t_lm / reps) * 16
    return per_step, reps, time.perf_counter() - t0


def run_reference(args, rank, world):
    """The reference's CPU path for the same decode step on all host threads."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    vals = []
    budget = max(0.25, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    for i in range(args.warmup + args.steps):
        sec, reps, dt = cpu_step_seconds(threads, budget)
        if i >= args.warmup:
            vals.append(args.batch / sec)
    v = statistics.median(vals)
    sample = ("2 of 28 Qwen3-1.7B decoder layers (q,k,v,o,gate,up,down) + 1/16 of the lm_head rows per repetition, "
              "%.1f s per step, scaled to the full step; attention excluded" % budget)
    line = {"metric": "Qwen3-1.7B int4 decode tok/s (context %d, batch %d)" % (args.context, args.batch),
            "impl": "reference", "value": round(v, 4), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * args.batch / v, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4xint8->int32,f32", "data": "synthetic",
            "config": {"workload": "qwen3-1.7b int4 decode step", "batch": args.batch, "context": args.context},
            "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference CPU path = C transcription of the JS linearQ int4 math (no node/cargo in this "
                    "image), row-partitioned over all host threads as cpu/kernel/cpuengine-mt.js does"}
    print(json.dumps(line), flush=True)


def profile_q2g64():
    """Three tb_gemv_tern_q2g64 launches, batch 1, each on its own 151936 x 2048
    matrix (117 MB; the three together exceed L2), for an ncu capture of one."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(31)
    V, H = Q17["vocab"], Q17["hidden"]
    mats = [_q2g64_pack(dev, g, V, H) for _ in range(3)]
    act, xsum, _ = tb.quantize_act(torch.randn(1, H, device=dev, generator=g))
    y = torch.empty(1, V, device=dev)
    torch.cuda.synchronize(dev)
    for c, s in mats:
        tb.gemv_tern(c, s, act, xsum, out=y)
    torch.cuda.synchronize(dev)
    assert tb.default_context(0).device_error() == 0


def decode_extra(dev, stream, B, S):
    """Qwen3-1.7B decode steps of B sequences at context S (recorded step, 50 timed)."""
    import torch
    mx = build_model(Q17, dev, B, S, 64 + 16, 1, 0)
    mx.set_tokens([(3 + 101 * b) % Q17["vocab"] for b in range(B)], [S - 1] * B)
    for _ in range(5):
        mx.step()
    torch.cuda.synchronize(dev)
    msx = time_steps(mx, 50, stream) / 50
    errx = mx.ctx.device_error()
    assert errx == 0, "decode extra device error 0x%x" % errx
    out = {"tok_per_s": round(B * 1e3 / msx, 1), "ms_per_step": round(msx, 4),
           "step_hbm_gbs": round(step_bytes(Q17, 1, B, S) / (msx * 1e-3) / 1e9, 1),
           "kernels_per_step": mx.launches_per_step()[0]}
    mx.close()
    del mx
    torch.cuda.synchronize(dev)
    return out


def run_only(name, steps):
    """One extra block alone (a development run; not the benchmark line)."""
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ctx = tb.default_context(0)
    peak, _ = load_peaks()
    if name == "q2g64":
        out = q2g64_extra(dev, ctx, peak)
    elif name == "moe":
        stream = torch.cuda.current_stream(dev)
        out = {"group32": moe_extra(dev, peak, stream), "group128": moe_extra(dev, peak, stream, group=128)}
    elif name == "decode":
        stream = torch.cuda.current_stream(dev)     # the stream main() times the model steps on
        out = {"batch%d_context%d" % (B, S): decode_extra(dev, stream, B, S)
               for B, S in ((16, 4096), (4, 4096), (8, 4096), (1, 32768))}
    elif name == "prefill":
        stream = torch.cuda.current_stream(dev)
        mp = os.path.join(REPO, "MEASURED_PEAKS.json")
        bf16 = json.load(open(mp)).get("bf16_tflops", 1590.0) if os.path.exists(mp) else 1590.0
        out = {"gemm_f16": prefill_extra(dev, bf16, stream), "gemm_exact": prefill_exact_extra(dev, bf16, stream),
               "forward": prefill_forward_extra(dev, stream)}
    elif name == "tern":
        stream = torch.cuda.current_stream(dev)
        mp = os.path.join(REPO, "MEASURED_PEAKS.json")
        bf16 = json.load(open(mp)).get("bf16_tflops", 1590.0) if os.path.exists(mp) else 1590.0
        out = tern_extra(dev, peak, bf16, stream)
    elif name == "chain":
        out = {}
        for B in (1, 4, 8):
            ch = chain_gbs(dev, ctx, B, max(100, steps))
            ch["frac_of_peak"] = round(ch["gbs"] / peak, 4)
            out["batch%d" % B] = ch
    else:
        out = kernel_kinds(Q17, dev, 1, 4096, peak)
    assert ctx.device_error() == 0
    print(json.dumps({"only": name, name: out}), flush=True)


# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--tp-exchange", default="p2p", choices=["p2p", "nccl"],
                    help="tensor-parallel sums: this library's peer-memory kernels, or NCCL")
    ap.add_argument("--profile-case", action="store_true",
                    help="one cold-L2 launch per kernel kind (for ncu), then exit")
    ap.add_argument("--profile-attn", type=int, default=0, metavar="S",
                    help="three cold-L2 decode-attention launches at context S (for ncu), then exit")
    ap.add_argument("--profile-gemm", type=int, nargs=3, default=None, metavar=("M", "N", "K"),
                    help="three cold-L2 prefill-GEMM launches at M x N x K (for ncu), then exit")
    ap.add_argument("--profile-prefill-attn", type=int, default=0, metavar="T",
                    help="three cold-L2 prefill-attention launches at T = S tokens (for ncu), then exit")
    ap.add_argument("--profile-prefill", type=int, default=None, metavar="T",
                    help="two T-token prefill forwards (for an ncu launch list)")
    ap.add_argument("--profile-gemm-dp4", type=int, nargs=3, default=None, metavar=("M", "N", "K"),
                    help="three cold-L2 exact-sum prefill GEMM launches (for ncu), then exit")
    ap.add_argument("--profile-lm-head", default=None, choices=("int4_f32", "int4_dp4a", "tern", "int4_mma16"),
                    help="three cold-L2 batch-1 lm_head GEMVs of one weight kind (for ncu), then exit")
    ap.add_argument("--step-mode", default="auto", choices=("auto", "kernels", "persistent"),
                    help="decode step as one persistent kernel (auto: where it applies) or one kernel per op")
    ap.add_argument("--profile-step", type=int, default=0, metavar="LAYERS",
                    help="persistent decode step of a LAYERS-layer 1.7B-width model, launched alone (for ncu)")
    ap.add_argument("--profile-moe", type=int, default=0, metavar="T",
                    help="three int3 MoE layers over T tokens (for an ncu launch list), then exit")
    ap.add_argument("--profile-decode", type=int, default=0, metavar="S",
                    help="three recorded decode steps at context S (for an ncu launch list), then exit")
    ap.add_argument("--profile-q2g64", action="store_true",
                    help="three Q2_0_g64 GEMV launches on 151936 x 2048 matrices (for an ncu capture), then exit")
    ap.add_argument("--only", default=None, choices=("q2g64", "chain", "kinds", "decode", "moe", "prefill", "tern"),
                    help="run one extra block alone on GPU 0 and print its JSON (development runs)")
    args = ap.parse_args()
    if args.only:
        run_only(args.only, args.steps)
        return
    if args.profile_q2g64:
        profile_q2g64()
        return
    if args.profile_decode:
        profile_decode(args.profile_decode, args.batch)
        return
    if args.profile_moe:
        profile_moe(args.profile_moe)
        return
    if args.profile_step:
        profile_step(args.profile_step)
        return
    if args.profile_lm_head:
        profile_lm_head(args.profile_lm_head)
        return
    if args.profile_prefill_attn:
        profile_prefill_attn(args.profile_prefill_attn)
        return
    if args.profile_prefill:
        profile_prefill(args.profile_prefill)
        return
    if args.profile_gemm_dp4:
        profile_gemm_dp4(*args.profile_gemm_dp4)
        return
    if args.profile_gemm:
        profile_gemm(*args.profile_gemm)
        return
    if args.profile_case:
        profile_case()
        return
    if args.profile_attn:
        profile_attn(args.profile_attn)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    import tabinfer_b200 as tb
    from tabinfer_b200.qwen3 import nccl_unique_id
    ctx = tb.default_context(local)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def tp_setup(m):
        if world == 1:
            return
        if args.tp_exchange == "nccl":
            uid = torch.zeros(128, dtype=torch.uint8, device=dev)
            if rank == 0:
                uid.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
            dist.broadcast(uid, 0)
            m.tp_init(bytes(uid.cpu().numpy().tobytes()))
            return
        mine = torch.frombuffer(bytearray(m.tp_handle()), dtype=torch.uint8).to(dev)
        allh = [torch.zeros(64, dtype=torch.uint8, device=dev) for _ in range(world)]
        dist.all_gather(allh, mine)
        m.tp_connect([bytes(h.cpu().numpy().tobytes()) for h in allh])

    B, S = args.batch, args.context
    K2 = max(50, args.steps // 4)
    extra = args.warmup + args.steps + K2 + 16
    m = build_model(Q17, dev, B, S, extra, world, rank)
    tp_setup(m)
    from tabinfer_b200 import _lib as _tl
    m.set_step_mode({"auto": _tl.QW_STEP_AUTO, "kernels": _tl.QW_STEP_KERNELS,
                     "persistent": _tl.QW_STEP_PERSISTENT}[args.step_mode])
    ids0 = [(1000 + 7919 * b) % Q17["vocab"] for b in range(B)]
    pos0 = [S - 1] * B
    m.set_tokens(ids0, pos0)
    for _ in range(args.warmup):
        m.step()
    torch.cuda.synchronize(dev)
    m.set_tokens(ids0, pos0)
    barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ms = time_steps(m, args.steps, stream) / args.steps
    clocks_info = clocks.stop()
    torch.cuda.synchronize(dev)
    barrier()
    ms_max = max_over_ranks(ms)
    kernels, colls = m.launches_per_step()
    # e2e through the public API with host buffers
    m.set_tokens(ids0, pos0)
    barrier()
    e2e_total, h2d, d2h = time_e2e(m, K2, stream, ids0, pos0)
    e2e_ms = max_over_ranks(e2e_total / K2)
    step_kind = {_tl.QW_STEP_KERNELS: "kernels", _tl.QW_STEP_PERSISTENT: "persistent"}.get(m.step_kind(), "?")
    pers_us = None
    kernels_alt = None
    if step_kind == "persistent":
        # the persistent kernel alone (embed + all layers), for its roofline
        for _ in range(3):
            m.step_layers()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(K2):
            m.step_layers()
        e1.record(stream)
        e1.synchronize()
        pers_us = e0.elapsed_time(e1) * 1e3 / K2
        if not args.no_extras:
            # the same model as one kernel per operation (identical results), for
            # comparison; every rank takes the same steps
            m.set_step_mode(_tl.QW_STEP_KERNELS)
            m.set_tokens(ids0, pos0)
            for _ in range(args.warmup):
                m.step()
            m.set_tokens(ids0, pos0)
            torch.cuda.synchronize(dev)
            barrier()
            msk = max_over_ranks(time_steps(m, args.steps, stream) / args.steps)
            kernels_alt = {"tok_per_s": round(B * 1e3 / msk, 2), "ms_per_step": round(msk, 4),
                           "launches_per_step": m.launches_per_step()[0]}
    err = ctx.device_error()
    assert err == 0, "device error word 0x%x" % err
    m.close()
    del m
    torch.cuda.synchronize(dev)

    value = B * 1e3 / ms_max
    peak, peak_src = load_peaks()
    nbytes = step_bytes(Q17, world, B, S)
    extras = {"step_hbm_gbs_per_rank": round(nbytes / (ms_max * 1e-3) / 1e9, 1),
              "step_hbm_frac_per_rank": round(nbytes / (ms_max * 1e-3) / 1e9 / peak, 4)}
    roof = None
    cpu = None
    if pers_us is not None:
        lm_bytes = gemv_bytes(Q17["vocab"] // world, Q17["hidden"], B, 4 if B == 1 else 1 + 4 / 32)
        body = nbytes - int(lm_bytes)
        gbs = body / (pers_us * 1e-6) / 1e9
        tp = os.path.join(REPO, "profiles", "traffic.json")
        traffic = json.load(open(tp)).get("k_decode_step") if os.path.exists(tp) else None
        roof = {"bound": "hbm", "kernel": "k_decode_step (persistent: embed + %d layers)" % Q17["layers"],
                "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                "traffic": traffic, "peak_source": peak_src + " hbm_gbs (burst copy)",
                "algorithmic_bytes_per_launch": body, "us_per_launch": round(pers_us, 2),
                "timing": "CUDA events on the launching stream over %d back-to-back launches (weights 0.97 GB "
                          "> L2)" % K2}
        extras["step_kind"] = step_kind
        if kernels_alt:
            extras["decode_step_one_kernel_per_op"] = kernels_alt
    if rank == 0 and not args.no_extras:
        kinds = kernel_kinds(Q17, dev, world, S, peak)
        dom = max(kinds, key=lambda k: kinds[k]["us_per_step"])
        d = kinds[dom]
        traffic = None
        tp = os.path.join(REPO, "profiles", "traffic.json")
        if os.path.exists(tp) and world == 1:
            traffic = json.load(open(tp)).get(dom)
        if roof is None:
            roof = {"bound": "hbm", "kernel": dom, "achieved": d["gbs"], "peak": peak, "unit": "GB/s",
                    "frac": d["frac_of_peak"], "traffic": traffic,
                    "peak_source": peak_src + " hbm_gbs (burst copy)",
                    "algorithmic_bytes_per_launch": d["bytes_per_launch"], "us_per_launch": d["us_per_launch"],
                    "timing": d["timing"]}
        extras["kernels"] = kinds
    if world == 1 and rank == 0 and not args.no_extras:
        extras["gemv_chain_0.6b"] = chain_gbs(dev, ctx, 1, max(100, args.steps))
        extras["gemv_chain_0.6b"]["frac_of_peak"] = round(extras["gemv_chain_0.6b"]["gbs"] / peak, 4)
        for (Bx, Sx) in ((16, 4096), (1, 32768)):
            if (Bx, Sx) == (B, S):
                continue
            extras["batch%d_context%d" % (Bx, Sx)] = decode_extra(dev, stream, Bx, Sx)
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) if os.path.exists(
            os.path.join(REPO, "MEASURED_PEAKS.json")) else {}
        extras["prefill_gemm_1.7b"] = prefill_extra(dev, peaks.get("bf16_tflops", 1590.0), stream)
        extras["prefill_gemm_1.7b"]["peak"] = "bf16_tflops %s (cuBLAS burst)" % (
            "measured" if peaks else "fallback 1590")
        extras["prefill_gemm_exact_1.7b"] = prefill_exact_extra(dev, peaks.get("bf16_tflops", 1590.0), stream)
        extras["moe_int3_lfm2.5"] = moe_extra(dev, peak, stream)
        extras["moe_int3_lfm2.5_group128"] = moe_extra(dev, peak, stream, group=128)
        extras["ternary_wgsl_bonsai_1.7b"] = tern_extra(dev, peak, peaks.get("bf16_tflops", 1590.0), stream)
        extras["ternary_wgsl_bonsai_1.7b"]["decode_step_context4096"] = bonsai_extra(dev, peak, stream)
        extras["prefill_attention_1.7b"] = prefill_attn_extra(dev, peaks.get("bf16_tflops", 1590.0), stream)
        extras["prefill_forward_1.7b"] = prefill_forward_extra(dev, stream)
        sec, reps, dt = cpu_step_seconds(1, 12.0)
        cpu = {"value": round(B / sec, 4), "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": "2 of 28 decoder layers (7 matrices each) + 1/16 of the lm_head rows, %d repetitions in "
                         "%.1f s, scaled to the full step; C transcription of the JS linearQ int4 math, 1 thread; "
                         "attention excluded" % (reps, dt)}

    if world == 1 and rank == 0 and not args.no_extras:
        for Bc in (4, 8):
            ch = chain_gbs(dev, ctx, Bc, max(100, args.steps))
            ch["frac_of_peak"] = round(ch["gbs"] / peak, 4)
            ch["tok_per_s"] = round(Bc * 1e3 / ch["ms_per_step"], 1)
            extras["gemv_chain_0.6b_batch%d" % Bc] = ch
        q2 = q2g64_extra(dev, ctx, peak)
        q2["cpu_baseline"] = cpu_q2g64(12.0)
        extras["ternary_q2g64_bonsai_1.7b"] = q2

    if not args.no_extras:          # every rank: the expert-parallel exchange needs all of them
        ep_out = moe_ep_extra(dev, world, rank, stream, peak, dist)
        if rank == 0:
            extras["moe_ep_lfm2.5"] = ep_out
        if world > 1:
            pf = prefill_forward_tp_extra(dev, stream, world, rank, dist)
            if rank == 0:
                extras["prefill_forward_1.7b_tp"] = pf

    if rank == 0:
        line = {"metric": "Qwen3-1.7B int4 decode tok/s (context %d, batch %d)" % (S, B), "value": round(value, 2),
                "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int4xint8->int32,f32", "data": "synthetic",
                "config": {"workload": "qwen3-1.7b int4 decode step (28 layers, int8 KV, tied lm_head)",
                           "batch": B, "context": S, "hidden": Q17["hidden"], "layers": Q17["layers"],
                           "heads": "%d q / %d kv x %d" % (Q17["n_heads"], Q17["n_kv_heads"], Q17["head_dim"]),
                           "intermediate": Q17["intermediate"], "vocab": Q17["vocab"],
                           "bytes_per_step_per_rank": nbytes,
                           "l2": "weights 0.97 GB + KV cache > 126 MB L2 (no flush needed)",
                           "parallelism": "tp%d" % world if world > 1 else "single"},
                "roofline": roof, "cpu_baseline": cpu,
                "e2e": {"value": round(B * 1e3 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)},
                "gpu_launches": kernels * args.steps, "nccl_collectives_per_step": colls,
                "tp_exchange": args.tp_exchange if world > 1 else None,
                "clocks": clocks_info}
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
