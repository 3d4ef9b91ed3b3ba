"""bench.py -- int4 decode-GEMV throughput on B200.

One step = the int4 GEMV chain of one Qwen3-0.6B decode token at batch B, in
the order models/qwen3.js:forward (3938-4069) issues it, attention left out:
per layer (x28) fused RMSNorm->int8, q/k/v GEMVs in one launch, int8 of the
q row (standing in for the attention output, same shape) -> o GEMV (+residual),
fused RMSNorm->int8, gate+up+SiLU, int8 of swi -> down GEMV (+residual); then
RMSNorm and the tied lm_head (151936 x 1024; f32-activation gemvQ at B=1 as
linearQ routes it, the int8 DP4A math at B>1) and a GPU argmax.
Weights: bf16 N(0, 0.02) quantized on the GPU with the reference's int4 G=32
scheme; activations N(0,1) rows.  The packed weights (335 MB) exceed the
126 MB L2, so every step streams them from HBM.

value = algorithmic bytes per step (packed weights + f16 scales + activations in
and outputs out of every GEMV) / device time per step, summed over ranks
(weak scaling: every rank runs its own replica; there is no data-path
collective).  e2e = the same bytes per step measured through the C ABI with
host buffers: tb_copy_h2d of the input rows from pinned memory, tb_batch_submit
of the recorded step, tb_copy_d2h of the token ids, all inside the timed region.

--impl reference times the reference's CPU path for the same chain (the scalar
transcription of the JS linearQ math in oracle/tb_cpu_ref.c, all host
threads) on a bounded sample of the layers.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

H, NHQ, NKV, HD, INTER, VOCAB, LAYERS = 1024, 16, 8, 128, 3072, 151936, 28
MATS = [("q", NHQ * HD, H), ("k", NKV * HD, H), ("v", NKV * HD, H), ("o", H, NHQ * HD),
        ("gate", INTER, H), ("up", INTER, H), ("down", H, INTER)]


def wbytes(N, K):
    return N * K // 2 + N * (K // 32) * 2


def gemv_bytes(N, K, B, act_bytes):
    """packed weights + scales read once, B activation rows in, B output rows out."""
    return wbytes(N, K) + B * K * act_bytes + B * N * 4


def step_bytes(B):
    tot = 0
    q8 = 1 + 4 / 32   # int8 activation + one f32 scale per 32
    for _, N, K in MATS:
        tot += gemv_bytes(N, K, B, q8)
    tot *= LAYERS
    tot += gemv_bytes(VOCAB, H, B, 4 if B == 1 else q8)
    return int(tot)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
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
        # samples "under load": power above the midpoint of the observed range
        lo, hi = min(p for p in pw if p is not None), max(p for p in pw if p is not None)
        load = [num(r[1]) for r, p in zip(rows, pw) if p is not None and p >= (lo + hi) / 2 and num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(load or sm), "sm_max_mhz": max(num(r[2]) or 0 for r in rows),
                "reasons": reasons, "samples": len(rows), "power_w_max": hi}


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# GPU workload
# ---------------------------------------------------------------------------

class Chain:
    """Weights of the 0.6B decode GEMV chain, quantized on the GPU."""

    def __init__(self, dev, seed):
        import torch
        import tabinfer_b200 as tb
        self.dev = dev
        g = torch.Generator(device=dev).manual_seed(seed)
        self.layers = []
        for _ in range(LAYERS):
            L = {}
            for name, N, K in MATS:
                w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
                L[name] = tb.quantize_int4_bf16(w.view(torch.int16))
            L["ln1"] = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).half().view(torch.int16)
            L["ln2"] = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).half().view(torch.int16)
            self.layers.append(L)
        w = (torch.randn(VOCAB, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.lm_head = tb.quantize_int4_bf16(w.view(torch.int16))
        self.norm = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).half().view(torch.int16)
        del w
        torch.cuda.synchronize(dev)


class ChainRun:
    """Activation buffers for batch B and the recorded step."""

    def __init__(self, chain, B, ctx):
        import torch
        dev = chain.dev
        self.chain, self.B, self.ctx = chain, B, ctx
        z = lambda *s, dt=torch.float32: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
        self.x = z(B, H)
        self.q, self.k, self.v = z(B, NHQ * HD), z(B, NKV * HD), z(B, NKV * HD)
        self.swi = z(B, INTER)
        self.logits = z(B, VOCAB)
        self.tok = torch.zeros(B, dtype=torch.int32, device=dev)
        self.batch = None
        self.launches = 0

    def step(self):
        """Issue one step's calls (eager, or under recording): 4 fused launches per layer."""
        import tabinfer_b200 as tb
        c = self.chain
        n = 0
        for L in c.layers:
            tb.gemv_dp4a_multi(self.x, [L["q"], L["k"], L["v"]], norm_w=L["ln1"], eps=1e-6, ys=[self.q, self.k, self.v])
            tb.gemv_dp4a(self.q, *L["o"], y=self.x, acc=True)
            tb.gate_up_silu_dp4a(self.x, *L["gate"], *L["up"], norm_w=L["ln2"], eps=1e-6, swi=self.swi)
            tb.gemv_dp4a(self.swi, *L["down"], y=self.x, acc=True)
            n += 4
        if self.B == 1:
            tb.gemv_q_norm(self.x, c.norm, 1e-6, *c.lm_head, y=self.logits)
        else:
            tb.gemv_dp4a(self.x, *c.lm_head, norm_w=c.norm, eps=1e-6, y=self.logits)
        tb.argmax(self.logits, out=self.tok)
        self.launches = n + 3

    def record(self):
        import torch
        from tabinfer_b200._lib import LIB, P
        stream = torch.cuda.ExternalStream(self.ctx.own_stream(), device=self.chain.dev)
        self.stream = stream
        with torch.cuda.stream(stream):
            self.step()                      # eager warm-up (sizes any scratch)
            stream.synchronize()
            self.ctx.check(LIB.tb_batch_begin(self.ctx.h), "batch_begin")
            self.step()
            h = P()
            self.ctx.check(LIB.tb_batch_end(self.ctx.h, ctypes.byref(h)), "batch_end")
        self.batch = h

    def submit(self):
        from tabinfer_b200._lib import LIB
        self.ctx.check(LIB.tb_batch_submit(self.ctx.h, self.batch), "batch_submit")

    def close(self):
        from tabinfer_b200._lib import LIB
        if self.batch is not None:
            LIB.tb_batch_destroy(self.batch)
            self.batch = None


def time_replays(run, K):
    import torch
    s = run.stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(K):
        run.submit()
    e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / K


def time_e2e(run, K):
    """Same step through the C ABI with host buffers: pinned H2D of the input
    rows, one recorded-batch submit, D2H of the token ids."""
    import torch
    from tabinfer_b200._lib import LIB, P
    s = run.stream
    hx = torch.randn(run.B, H).pin_memory()
    htok = torch.zeros(run.B, dtype=torch.int32).pin_memory()
    h2d = hx.numel() * 4
    d2h = htok.numel() * 4
    c = run.ctx
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(K):
        c.check(LIB.tb_copy_h2d(c.h, P(run.x.data_ptr()), P(hx.data_ptr()), h2d), "h2d")
        run.submit()
        c.check(LIB.tb_copy_d2h(c.h, P(htok.data_ptr()), P(run.tok.data_ptr()), d2h), "d2h")
    e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / K, h2d, d2h


def dominant_kernel_roofline(chain, ctx, peak, reps=3):
    """Per-launch device time of each GEMV kind, cold L2 (a 256 MB buffer is
    written between launches), with CUDA events on the launching stream.
    Returns the kind with the largest share of the step and all kinds."""
    import torch
    import tabinfer_b200 as tb
    from tabinfer_b200._lib import LIB
    dev = chain.dev
    s = torch.cuda.ExternalStream(ctx.own_stream(), device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    B = 1
    x1 = torch.randn(B, H, device=dev)
    x2 = torch.randn(B, NHQ * HD, device=dev)
    x3 = torch.randn(B, INTER, device=dev)
    ln = chain.layers[0]["ln1"]
    with torch.cuda.stream(s):
        outs = {n: torch.zeros(B, N, device=dev) for n, N, _ in MATS}
        logits = torch.zeros(B, VOCAB, device=dev)
        swi = torch.zeros(B, INTER, device=dev)
        kinds = {
            "gemv_dp4a rmsnorm+qkv (4096x1024)": (lambda L: tb.gemv_dp4a_multi(x1, [L["q"], L["k"], L["v"]], norm_w=ln,
                                                                                ys=[outs["q"], outs["k"], outs["v"]]),
                                                  gemv_bytes(4096, H, B, 1.125), LAYERS),
            "gemv_dp4a o (1024x2048)": (lambda L: tb.gemv_dp4a(x2, *L["o"], y=outs["o"]),
                                        gemv_bytes(H, 2048, B, 1.125), LAYERS),
            "gemv_dp4a rmsnorm+gate+up+silu (2x3072x1024)": (
                lambda L: tb.gate_up_silu_dp4a(x1, *L["gate"], *L["up"], norm_w=ln, swi=swi),
                2 * wbytes(INTER, H) + B * H * 1.125 + B * INTER * 4, LAYERS),
            "gemv_dp4a down (1024x3072)": (lambda L: tb.gemv_dp4a(x3, *L["down"], y=outs["down"]),
                                           gemv_bytes(H, INTER, B, 1.125), LAYERS),
            "gemv_f32 rmsnorm+lm_head (151936x1024)": (lambda L: tb.gemv_q_norm(x1, chain.norm, 1e-6, *chain.lm_head, y=logits),
                                                       gemv_bytes(VOCAB, H, B, 4), 1),
        }
        res = {}
        for name, (fn, nbytes, per_step) in kinds.items():
            ts = []
            for r in range(reps):
                for li, L in enumerate(chain.layers if per_step > 1 else chain.layers[:1]):
                    flush.fill_(r & 0xff)
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(s)
                    fn(L)
                    e1.record(s)
                    e1.synchronize()
                    ts.append(e0.elapsed_time(e1))
            us = statistics.median(ts) * 1e3
            res[name] = {"us_per_launch": us, "bytes_per_launch": int(nbytes), "launches_per_step": per_step,
                         "gbs": nbytes / (us * 1e-6) / 1e9, "us_per_step": us * per_step}
    dom = max(res, key=lambda k: res[k]["us_per_step"])
    return dom, res


def profile_case():
    """One cold-L2 launch of each kernel kind, for `ncu --set full` on a small
    case (a few hundred MB on the device): the five GEMV kinds of the 0.6B chain
    at batch 1, the config-1 ternary qkv GEMV (4096 x 2048) and int8-KV decode
    attention at S = 4096 (1.7B heads).  Every launch is preceded by a 256 MB
    write that evicts L2."""
    import numpy as np
    import torch
    import tabinfer_b200 as tb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)

    def q(N, K):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        return tb.quantize_int4_bf16(w.view(torch.int16))

    qm, km, vm, om = q(2048, H), q(1024, H), q(1024, H), q(H, 2048)
    gm, um, dm, lm = q(INTER, H), q(INTER, H), q(H, INTER), q(VOCAB, H)
    ln = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).half().view(torch.int16)
    tw = (torch.randint(0, 3, (4096, 2048), device=dev, generator=g).float() - 1.0) * 0.03
    codes, tsc = tb.pack_ternary(tw)
    S, nHq, nKv, hd = 4096, 16, 8, 128
    Kq = torch.randint(-127, 128, (S, nKv * hd), device=dev, generator=g, dtype=torch.int8)
    Vq = torch.randint(-127, 128, (S, nKv * hd), device=dev, generator=g, dtype=torch.int8)
    Ks = torch.rand(S, nKv * hd // 32, device=dev, generator=g) + 0.5
    Vs = torch.rand(S, nKv * hd // 32, device=dev, generator=g) + 0.5
    qr = torch.randn(nHq * hd, device=dev, generator=g)
    x1, x2, x3 = (torch.randn(1, k, device=dev, generator=g) for k in (H, 2048, INTER))
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


def cpu_baseline_sample(threads, budget_s=12.0):
    """The transcribed CPU path (oracle/tb_cpu_ref.c, linearQ math) on a bounded
    sample: 2 decoder layers' 7 matrices + 1/16 of the lm_head rows, repeated
    until `budget_s` of CPU work.  Returns GB/s of the same algorithmic bytes."""
    import numpy as np
    import oracle
    lib = oracle.cpuref()
    rng = np.random.default_rng(7)
    mats = []
    for _ in range(2):
        for _, N, K in MATS:
            mats.append((N, K, rng.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint32),
                         np.float16(rng.uniform(0.001, 0.004, (N, K // 32))).view(np.uint16)))
    Nl = VOCAB // 16
    mats.append((Nl, H, rng.integers(0, 2 ** 32, (Nl, H // 8), dtype=np.uint32),
                 np.float16(rng.uniform(0.001, 0.004, (Nl, H // 32))).view(np.uint16)))
    P = ctypes.c_void_p
    xs = {K: rng.normal(0, 1, K).astype(np.float32) for K in (H, 2048, INTER)}
    xq = np.zeros(INTER, np.int8)
    xsc = np.zeros(INTER // 32, np.float32)
    ys = [np.zeros(N, np.float32) for N, *_ in mats]
    nbytes = 0
    t0 = time.perf_counter()
    reps = 0
    while True:
        for (N, K, pk, sc), y in zip(mats, ys):
            if N == Nl:   # lm_head rows keep linearQ's f32 (gemvQ) route, as at N >= 16384
                lib.tbr_gemv_int4_f32(P(y.ctypes.data), P(xs[K].ctypes.data), P(pk.ctypes.data), P(sc.ctypes.data),
                                      ctypes.c_int64(N), ctypes.c_int64(K), ctypes.c_int(0), ctypes.c_int(threads))
            else:
                lib.tbr_linear_int4(P(y.ctypes.data), P(xs[K].ctypes.data), P(pk.ctypes.data), P(sc.ctypes.data),
                                    ctypes.c_int64(N), ctypes.c_int64(K), ctypes.c_int(0), P(xq.ctypes.data),
                                    P(xsc.ctypes.data), ctypes.c_int(threads))
            nbytes += gemv_bytes(N, K, 1, 1.125 if N != Nl else 4)
        reps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return nbytes / dt / 1e9, reps, dt


# ---------------------------------------------------------------------------

def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    vals = []
    budget = max(1.0, min(20.0, 150.0 / max(1, args.steps + args.warmup)))
    for i in range(args.warmup + args.steps):
        gbs, reps, dt = cpu_baseline_sample(threads, budget_s=budget)
        if i >= args.warmup:
            vals.append(gbs)
    v = statistics.median(vals)
    sample = ("2 of 28 Qwen3-0.6B decoder layers (q,k,v,o,gate,up,down) + 1/16 of the lm_head rows per "
              "repetition, repeated for %.1f s per step" % budget)
    line = {"metric": "int4 decode GEMV HBM GB/s (Qwen3-0.6B chain, batch 1)", "impl": "reference",
            "value": round(v, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic", "config": {"workload": "qwen3-0.6b int4 decode GEMV chain", "batch": 1},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference CPU path = C transcription of the JS linearQ int4 math (no node/cargo in this "
                    "image); row-partitioned over all host threads as cpu/kernel/cpuengine-mt.js does"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--profile-case", action="store_true",
                    help="one cold-L2 launch per kernel kind (for ncu), then exit")
    ap.add_argument("--profile-attn", type=int, default=0, metavar="S",
                    help="three cold-L2 decode-attention launches at context S (for ncu), then exit")
    args = ap.parse_args()
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
    ctx = tb.default_context(local)
    ctx.own_stream()
    chain = Chain(dev, seed=1000 + rank)
    run = ChainRun(chain, args.batch, ctx)
    run.record()
    for _ in range(args.warmup):
        run.submit()
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    barrier()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ms = time_replays(run, args.steps)
    clocks_info = clocks.stop()
    torch.cuda.synchronize(dev)
    barrier()
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())

    B = args.batch
    nbytes = step_bytes(B)
    value = nbytes * world / (ms_max * 1e-3) / 1e9

    # e2e through the C ABI with host buffers
    e2e_ms, h2d, d2h = time_e2e(run, max(50, args.steps // 4))
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(nbytes * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)}

    peak, peak_src = load_peaks()
    extras = {}
    roof = None
    if rank == 0 and not args.no_extras:
        dom, kinds = dominant_kernel_roofline(chain, ctx, peak)
        d = kinds[dom]
        traffic = None
        tp = os.path.join(REPO, "profiles", "traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get(dom)
        roof = {"bound": "hbm", "kernel": dom, "achieved": round(d["gbs"], 1), "peak": peak, "unit": "GB/s",
                "frac": round(d["gbs"] / peak, 4), "traffic": traffic, "peak_source": peak_src + " hbm_gbs (burst copy)",
                "algorithmic_bytes_per_launch": d["bytes_per_launch"], "us_per_launch": round(d["us_per_launch"], 3)}
        extras["kernels"] = {k: {kk: round(vv, 3) if isinstance(vv, float) else vv for kk, vv in v.items()}
                             for k, v in kinds.items()}
        for Bx in (4, 8):
            if Bx == B:
                continue
            r2 = ChainRun(chain, Bx, ctx)
            r2.record()
            for _ in range(5):
                r2.submit()
            ms2 = time_replays(r2, max(50, args.steps // 4))
            extras["batch%d" % Bx] = {"gbs": round(step_bytes(Bx) / (ms2 * 1e-3) / 1e9, 1), "ms_per_step": round(ms2, 4),
                                      "tok_per_s_gemv_only": round(Bx * 1e3 / ms2, 1)}
            r2.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_extras:
        gbs, reps, dt = cpu_baseline_sample(1, budget_s=12.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": "2 of 28 decoder layers (7 matrices each) + 1/16 of the lm_head rows, %d repetitions in %.1f s, "
                         "C transcription of the JS linearQ int4 math, 1 thread" % (reps, dt)}

    if rank == 0:
        line = {"metric": "int4 decode GEMV HBM GB/s (Qwen3-0.6B chain, batch %d)" % B, "value": round(value, 2),
                "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "u8", "data": "synthetic",
                "config": {"workload": "qwen3-0.6b int4 decode GEMV chain (28 layers + tied lm_head)", "batch": B,
                           "hidden": H, "intermediate": INTER, "vocab": VOCAB, "layers": LAYERS,
                           "bytes_per_step": nbytes, "l2": "weights 335 MB > 126 MB L2 (no flush needed)",
                           "parallelism": "replicas" if world > 1 else "single"},
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": run.launches * args.steps,
                "clocks": clocks_info}
        line.update(extras)
        print(json.dumps(line), flush=True)
    run.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
