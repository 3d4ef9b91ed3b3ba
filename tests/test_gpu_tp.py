"""Tensor-parallel decode step on 2 GPUs (one process per GPU, NCCL): the two
ranks' vocab shards of the logits, concatenated, match the single-GPU step on
the same weights and cache, and both ranks produce the same argmax ids and
advanced positions.  Needs 2 GPUs (skipped on a 1-GPU box)."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from qwen3_oracle import make_weights

CFG = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, intermediate=512, vocab=1000,
           rope_theta=1e6, rms_eps=1e-6, max_seq=64, batch=3)
PREFILL = [9, 0, 30]
IDS = [17, 400, 999]


def _kv_rows(cfg, seed):
    rng = np.random.default_rng(seed)
    row = cfg["n_kv_heads"] * cfg["head_dim"]
    return [[(rng.standard_normal((n, row)).astype(np.float32), rng.standard_normal((n, row)).astype(np.float32))
             for n in PREFILL] for _ in range(cfg["layers"])]


def _run(cfg, rank, P, uid=None, exchange=None):
    """Build rank `rank` of P on cuda:rank, one step; returns logits, ids, pos.
    exchange: (handle queue in, handles queue out) for the peer-memory path."""
    import tabinfer_b200 as tb
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    W = make_weights(cfg, 5)
    m = tb.Qwen3(dict(cfg, tp_size=P, tp_rank=rank), device=rank)
    for name, w in W.items():
        m.load(name, torch.from_numpy(np.ascontiguousarray(w).view(np.int16)).to(dev))
    w = cfg["n_kv_heads"] // P * cfg["head_dim"]
    for l, per_seq in enumerate(_kv_rows(cfg, 8)):
        for b, (k, v) in enumerate(per_seq):
            if k.shape[0]:
                ks = torch.from_numpy(np.ascontiguousarray(k[:, rank * w:(rank + 1) * w])).to(dev)
                vs = torch.from_numpy(np.ascontiguousarray(v[:, rank * w:(rank + 1) * w])).to(dev)
                m.kv_fill(l, b, ks, vs, 0)
    if P > 1 and exchange is None:
        m.tp_init(uid)
    elif P > 1:
        hq, allq = exchange
        hq.put((rank, m.tp_handle()))
        m.tp_connect(allq.get(timeout=120))
    m.set_tokens(IDS, PREFILL)
    m.step()
    out = (m.logits().numpy(), *m.tokens())
    m.step()                          # a replay: the graph holds the collectives
    out2 = m.tokens()
    m.close()
    return out, out2


def _rank(rank, P, uid, q, exchange):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        q.put((rank, _run(CFG, rank, P, uid, exchange)))
    except Exception as e:          # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_tp2_step_matches_single_gpu(cuda, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from tabinfer_b200.qwen3 import nccl_unique_id
    single, single2 = _run(CFG, 0, 1)
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    exch = [None, None]
    if mode == "p2p":
        hq = ctx.Queue()
        outs = [ctx.Queue() for _ in range(2)]
        exch = [(hq, outs[r]) for r in range(2)]
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, q, exch[r])) for r in range(2)]
    for p in procs:
        p.start()
    if mode == "p2p":
        hs = dict(hq.get(timeout=240) for _ in range(2))
        for o in outs:
            o.put([hs[0], hs[1]])
    res = {}
    for _ in range(2):
        r, v = q.get(timeout=240)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    logits = np.concatenate([res[0][0][0], res[1][0][0]], axis=1)
    np.testing.assert_allclose(logits, single[0], atol=2e-2, rtol=0)
    for r in range(2):
        assert res[r][0][1] == single[1], "rank %d ids" % r
        assert res[r][0][2] == single[2] == [p + 1 for p in PREFILL]
        assert res[r][1] == single2, "rank %d second step" % r


# The prefill's residual sums differ in order between one GPU (x + s) and two
# (x + s0, then + s1 over the allreduce); every layer re-quantizes its input to
# int8, which carries a last-bit difference on as a 1/127 step of a group's
# maximum, so the two runs are held to the prefill's own logit budget.
PF_TOL = 5e-2
PF_TOKENS = {0: 40, 2: 150}


def _run_prefill(cfg, rank, P, uid=None):
    """Rank `rank` of P: prefill sequences 0 and 2, then one decode step.
    Returns (logits, ids, pos) after the prefills, this rank's cache columns of
    every layer, and (logits, ids, pos) after the step."""
    import tabinfer_b200 as tb
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    W = make_weights(cfg, 15)
    m = tb.Qwen3(dict(cfg, tp_size=P, tp_rank=rank), device=rank)
    for name, w in W.items():
        m.load(name, torch.from_numpy(np.ascontiguousarray(w).view(np.int16)).to(dev))
    if P > 1:
        m.tp_init(uid)
    rng = np.random.default_rng(16)
    for seq, n in PF_TOKENS.items():
        m.prefill(seq, rng.integers(0, cfg["vocab"], n).tolist(), 0)
    after = (m.logits().numpy(), *m.tokens())
    kv = [m.kv_host(l) for l in range(cfg["layers"])]
    m.step()
    stepped = (m.logits().numpy(), *m.tokens())
    m.close()
    return after, kv, stepped


def _rank_prefill(rank, P, uid, q):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        q.put((rank, _run_prefill(PF_CFG, rank, P, uid)))
    except Exception as e:
        q.put((rank, repr(e)))


PF_CFG = dict(CFG, max_seq=256)


def _deq(q, s):
    return q.astype(np.float64) / 127 * np.repeat(s.astype(np.float64), 32, axis=-1)


@pytest.mark.gpu
def test_tp2_prefill_matches_single_gpu(cuda):
    """Tensor-parallel prefill (column-split q/k/v/gate/up, row-split o/down
    with an allreduce of the T rows after each, vocab-split lm_head with the
    argmax merged over ranks) against the single-GPU prefill on the same
    weights: the concatenated logits, each rank's cache columns, the next
    tokens, and a decode step continuing from the prefilled state."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from tabinfer_b200.qwen3 import nccl_unique_id
    single = _run_prefill(PF_CFG, 0, 1)
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_prefill, args=(r, 2, uid, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    for k in (0, 2):            # after the prefills, after the step
        logits = np.concatenate([res[0][k][0], res[1][k][0]], axis=1)
        ref = single[k][0]
        rows = list(PF_TOKENS) if k == 0 else range(PF_CFG["batch"])
        for b in rows:
            assert float(np.max(np.abs(logits[b] - ref[b]))) <= PF_TOL, (k, b)
            top2 = np.sort(ref[b])[-2:]
            if top2[1] - top2[0] > 2 * PF_TOL:
                assert res[0][k][1][b] == res[1][k][1][b] == single[k][1][b], (k, b)
        assert res[0][k][2] == res[1][k][2] == single[k][2]
    assert single[0][2] == [PF_TOKENS.get(b, 0) for b in range(PF_CFG["batch"])]
    # rank r's cache holds kv heads [r*nKv/2, (r+1)*nKv/2) of the single GPU's rows
    w = PF_CFG["n_kv_heads"] // 2 * PF_CFG["head_dim"]
    for l in range(PF_CFG["layers"]):
        for r in range(2):
            for i in (0, 2):                # K, V
                for b, n in PF_TOKENS.items():      # rows past a prefill are never written
                    got = _deq(res[r][1][l][i][b, :n], res[r][1][l][i + 1][b, :n])
                    full = _deq(single[1][l][i][b, :n], single[1][l][i + 1][b, :n])[:, r * w:(r + 1) * w]
                    rel = np.max(np.abs(got - full), axis=1) / np.max(np.abs(full), axis=1)
                    assert float(np.max(rel)) < 5e-2, (l, r, i, b)


# ---- the persistent decode step under tensor parallelism ---------------------------
# (the o / down rows' exchange inside the kernel, per CTA over the peer-mapped
# exchange arenas) against the multi-kernel TP step on the same rank: same bits.
WIDE1 = dict(hidden=2048, layers=2, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=6144, vocab=20000,
             rope_theta=1e6, rms_eps=1e-6, max_seq=4200, batch=1)
KIND_CASES = [(dict(CFG, batch=1), 9, False), (dict(CFG, batch=1, max_seq=1024, layers=3), 700, False),
              (dict(CFG, batch=1), 9, True), (WIDE1, 4095, False)]


def _run_kinds(rank, P, exchange, case):
    """Rank `rank` of P over peer memory: three steps as one kernel per op,
    then the same three steps (same start) as the persistent kernel."""
    import tabinfer_b200 as tb
    from tabinfer_b200 import _lib
    cfg, n, ternary = KIND_CASES[case]
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    W = make_weights(cfg, 23, ternary=ternary)
    m = tb.Qwen3(dict(cfg, tp_size=P, tp_rank=rank), device=rank)
    for name, w in W.items():
        m.load(name, torch.from_numpy(np.ascontiguousarray(w).view(np.int16)).to(dev))
    rng = np.random.default_rng(29)
    row = cfg["n_kv_heads"] * cfg["head_dim"]
    w = row // P
    for l in range(cfg["layers"]):
        k = rng.standard_normal((n, row)).astype(np.float32)
        v = rng.standard_normal((n, row)).astype(np.float32)
        m.kv_fill(l, 0, torch.from_numpy(np.ascontiguousarray(k[:, rank * w:(rank + 1) * w])).to(dev),
                  torch.from_numpy(np.ascontiguousarray(v[:, rank * w:(rank + 1) * w])).to(dev), 0)
    hq, allq = exchange
    hq.put((rank, m.tp_handle()))
    m.tp_connect(allq.get(timeout=120))
    out = {}
    for mode in (_lib.QW_STEP_KERNELS, _lib.QW_STEP_PERSISTENT):
        m.set_step_mode(mode)
        m.set_tokens([321 % cfg["vocab"]], [n])
        runs = []
        for _ in range(3):
            m.step()
            runs.append((m.logits().numpy().copy(), *m.tokens()))
        out[mode] = (m.step_kind(), runs)
    err = m.ctx.device_error()
    m.close()
    return out, err


def _rank_kinds(rank, P, q, exchange, case):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        q.put((rank, _run_kinds(rank, P, exchange, case)))
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(len(KIND_CASES)))
def test_tp2_persistent_step_equals_kernels(cuda, case):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from tabinfer_b200 import _lib
    ctx = mp.get_context("spawn")
    q, hq = ctx.Queue(), ctx.Queue()
    outs = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=_rank_kinds, args=(r, 2, q, (hq, outs[r]), case)) for r in range(2)]
    for p in procs:
        p.start()
    hs = dict(hq.get(timeout=300) for _ in range(2))
    for o in outs:
        o.put([hs[0], hs[1]])
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        out, err = res[r]
        assert err == 0, "rank %d device error 0x%x" % (r, err)
        kk, runs_k = out[_lib.QW_STEP_KERNELS]
        kp, runs_p = out[_lib.QW_STEP_PERSISTENT]
        assert kk == _lib.QW_STEP_KERNELS and kp == _lib.QW_STEP_PERSISTENT
        for i, (a, b) in enumerate(zip(runs_k, runs_p)):
            np.testing.assert_array_equal(b[0], a[0], err_msg="rank %d step %d" % (r, i))
            assert b[1:] == a[1:], (r, i)
    assert [x[1:] for x in res[0][0][_lib.QW_STEP_PERSISTENT][1]] == \
        [x[1:] for x in res[1][0][_lib.QW_STEP_PERSISTENT][1]]


# ---- a peer that never arrives: bounded wait, poison, reset -------------------------
def _run_poison(rank, P, exchange, mine, other):
    """Rank 0 runs one persistent TP step while rank 1 launches nothing: the
    in-kernel exchange wait runs out (ERR_STEP_TP), the rank is poisoned and
    its next step refuses to run.  Then both ranks, idle, reset behind a
    queue barrier and step together; the persistent steps must equal the
    multi-kernel TP steps from the same start."""
    import tabinfer_b200 as tb
    from tabinfer_b200 import _lib
    cfg, n = dict(CFG, batch=1), 9
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    W = make_weights(cfg, 23)
    m = tb.Qwen3(dict(cfg, tp_size=P, tp_rank=rank), device=rank)
    for name, w in W.items():
        m.load(name, torch.from_numpy(np.ascontiguousarray(w).view(np.int16)).to(dev))
    hq, allq = exchange
    hq.put((rank, m.tp_handle()))
    m.tp_connect(allq.get(timeout=120))
    m.set_step_mode(_lib.QW_STEP_PERSISTENT)
    codes = []
    if rank == 0:
        import time
        t0 = time.time()
        m.set_tokens([321], [n])
        m.step()
        codes.append(m.ctx.device_error())      # synchronizes: the wait gave up
        codes.append(time.time() - t0)
        m.step()
        codes.append(m.ctx.device_error())      # poisoned: refused
        other.put("alone done")
    else:
        assert mine.get(timeout=120) == "alone done"
    # barrier (both idle), reset, barrier
    other.put("idle")
    assert mine.get(timeout=120) == "idle"
    m.tp_reset()
    other.put("reset")
    assert mine.get(timeout=120) == "reset"
    out = {}
    for mode in (_lib.QW_STEP_PERSISTENT, _lib.QW_STEP_KERNELS):
        m.set_step_mode(mode)
        m.set_tokens([321], [n])
        runs = []
        for _ in range(2):
            m.step()
            runs.append((m.logits().numpy().copy(), *m.tokens()))
        out[mode] = runs
    err = m.ctx.device_error()
    m.close()
    return codes, out, err


def _rank_poison(rank, P, q, exchange, mine, other):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        q.put((rank, _run_poison(rank, P, exchange, mine, other)))
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.gpu
def test_tp2_exchange_timeout_poisons_until_reset(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from tabinfer_b200 import _lib
    ctx = mp.get_context("spawn")
    q, hq = ctx.Queue(), ctx.Queue()
    outs = [ctx.Queue() for _ in range(2)]
    boxes = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=_rank_poison, args=(r, 2, q, (hq, outs[r]), boxes[r], boxes[1 - r]))
             for r in range(2)]
    for p in procs:
        p.start()
    hs = dict(hq.get(timeout=300) for _ in range(2))
    for o in outs:
        o.put([hs[0], hs[1]])
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    codes = res[0][0]
    # the first bounded wait to run out: ERR_STEP_TP (0x5103) in a CTA waiting for the
    # peer's packets, or ERR_STEP_BARRIER (0x5101) in a CTA that owns no residual rows
    # (it skips the exchange) waiting at the next grid barrier for the others
    assert codes[0] in (0x5103, 0x5101), "first step: 0x%x" % codes[0]
    assert codes[1] < 20.0, "the bounded wait took %.1f s" % codes[1]
    assert codes[2] == 0x5104, "poisoned step: 0x%x" % codes[2]     # refused until the reset
    for r in range(2):
        _, out, err = res[r]
        assert err == 0, "rank %d device error 0x%x after the reset" % (r, err)
        for a, b in zip(out[_lib.QW_STEP_KERNELS], out[_lib.QW_STEP_PERSISTENT]):
            np.testing.assert_array_equal(b[0], a[0])
            assert b[1:] == a[1:]
    assert [x[1:] for x in res[0][1][_lib.QW_STEP_PERSISTENT]] == [x[1:] for x in res[1][1][_lib.QW_STEP_PERSISTENT]]
