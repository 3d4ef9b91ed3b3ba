"""Expert-parallel MoE dataflow on CPU (no GPU): world_size-2 gloo ranks each
route their own tokens, send every token row once to each rank owning one of
its experts (the dispatch plan of tb_moe_ep_forward: one slot per token and
destination in token order, per top-k slot the code (local expert << 24) |
t*K + k or ~0), the owners run their experts on what they received (the
oracle's int3 expert FFN on the rank's own slice of the expert tensors), the
outputs travel back to their (token, k) slots and the origin combines in k
order.  The result equals the single-device oracle FFN exactly (same f64
operations in the same order)."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle

H, I, NE, K, P = 64, 64, 8, 3, 2


def _experts(seed):
    rng = np.random.default_rng(seed)
    out = []
    for rows, cols in ((NE * I, H), (NE * I, H), (NE * H, I)):
        pack = rng.integers(0, 2**32, (rows, cols // 8), dtype=np.uint64).astype(np.uint32)
        s4 = (rng.uniform(0.5, 2.0, (rows, cols // 32)) * 1e-2).astype(np.float16).view(np.uint16)
        out.append(oracle.requant43(pack, s4))
    return out


def dispatch_plan(idx, El, P):
    """Per destination rank: the token rows it receives (token order) and the
    K meta codes of each."""
    T, Kk = idx.shape
    plan = []
    for d in range(P):
        toks = [t for t in range(T) if any(int(e) // El == d for e in idx[t])]
        meta = np.full((len(toks), Kk), 0xFFFFFFFF, np.uint32)
        for j, t in enumerate(toks):
            for k in range(Kk):
                if int(idx[t, k]) // El == d:
                    meta[j, k] = ((int(idx[t, k]) % El) << 24) | (t * Kk + k)
        plan.append((toks, meta))
    return plan


def _tokens(rank):
    rng = np.random.default_rng(100 + rank)
    T = 5 + 4 * rank
    logits = rng.standard_normal((T, NE)).astype(np.float32)
    if rank == 1:
        logits[:, :NE // 2] += 6.0            # rank 1's tokens all routed to rank 0's experts
    idx, wt = oracle.moe_router(logits, np.zeros(NE, np.float32), K)
    a = rng.standard_normal((T, H)).astype(np.float32)
    return a, idx, wt


def _a2a_obj(objs):
    """all-to-all of picklable objects over gloo (counts, then byte payloads)."""
    import pickle
    blobs = [np.frombuffer(pickle.dumps(o), np.uint8) for o in objs]
    send_n = torch.tensor([len(b) for b in blobs], dtype=torch.int64)
    recv_n = torch.empty_like(send_n)
    dist.all_to_all_single(recv_n, send_n)
    send = torch.from_numpy(np.concatenate(blobs).copy())
    recv = torch.empty(int(recv_n.sum()), dtype=torch.uint8)
    dist.all_to_all_single(recv, send, recv_n.tolist(), send_n.tolist())
    out, off = [], 0
    for n in recv_n.tolist():
        out.append(pickle.loads(recv[off:off + n].numpy().tobytes()))
        off += n
    return out


def _rank(rank, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=P)
        El = NE // P
        w = _experts(7)
        local = [(p[rank * El * (p.shape[0] // NE):(rank + 1) * El * (p.shape[0] // NE)],
                  s[rank * El * (s.shape[0] // NE):(rank + 1) * El * (s.shape[0] // NE)]) for p, s in w]
        a, idx, wt = _tokens(rank)
        plan = dispatch_plan(idx, El, P)
        # dispatch: rows + meta to every destination
        recv = _a2a_obj([(a[toks], meta) for toks, meta in plan])
        # owner: every received (row, k) whose expert is here
        back = [[] for _ in range(P)]
        for s, (rows, meta) in enumerate(recv):
            for j in range(rows.shape[0]):
                for k in range(meta.shape[1]):
                    code = int(meta[j, k])
                    if code == 0xFFFFFFFF:
                        continue
                    el, pair = code >> 24, code & 0xFFFFFF
                    o = oracle.moe_ffn_int3(rows[j:j + 1], np.array([[el]], np.uint32), np.ones((1, 1), np.float32),
                                            local[0], local[1], local[2], H, I)
                    back[s].append((pair, o[0]))
        ret = _a2a_obj(back)
        T = a.shape[0]
        outs = {}
        for lst in ret:
            for pair, o in lst:
                assert pair not in outs
                outs[pair] = o
        assert sorted(outs) == list(range(T * K))       # every (token, k) computed exactly once
        x = np.zeros((T, H), np.float64)
        for t in range(T):
            for k in range(K):
                x[t] += np.float64(wt[t, k]) * outs[t * K + k]
        ref = oracle.moe_ffn_int3(a, idx, wt, w[0], w[1], w[2], H, I)
        q.put((rank, float(np.max(np.abs(x - ref))), [len(toks) for toks, _ in plan]))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e), None))


def test_ep_dataflow_matches_single_device():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(P)]
    for p in procs:
        p.start()
    res = dict((r, (err, sent)) for r, err, sent in (q.get(timeout=300) for _ in range(P)))
    for p in procs:
        p.join(timeout=60)
    for r in range(P):
        assert not isinstance(res[r][0], str), res[r][0]
        assert res[r][0] == 0.0
    assert res[1][1][1] == 0          # the skewed rank sends nothing to rank 1


def test_dispatch_plan_codes():
    idx = np.array([[0, 5, 3], [6, 7, 1], [2, 1, 0]], np.uint32)
    plan = dispatch_plan(idx, 4, 2)
    assert plan[0][0] == [0, 1, 2] and plan[1][0] == [0, 1]
    assert plan[0][1][0].tolist() == [0 << 24 | 0, 0xFFFFFFFF, 3 << 24 | 2]
    assert plan[1][1][1].tolist() == [2 << 24 | 3, 3 << 24 | 4, 0xFFFFFFFF]
