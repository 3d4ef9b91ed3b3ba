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
