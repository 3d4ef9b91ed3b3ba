"""Expert-parallel int3 MoE FFN (tb_moe_ep_*) against the single-device MoE
FFN (tb_moe_ffn_int3, itself checked against the oracle in test_gpu_moe.py):
bit-identical outputs, since the owner ranks run the same grouped GEMVs per
(token, expert) pair and the origin combines in the same k order.

* P = 1 on one GPU: the whole exchange path (dispatch into the arena, plan,
  GEMVs writing into the return slots, signal, combine) with all 32 experts.
* P = every visible GPU up to 8 (skipped on one; 8 GPUs is config 5's 4 experts
  per GPU): each rank routing its own tokens, rank 1's routing skewed onto rank
  0's experts, several forwards with different token counts (epochs), no device
  errors."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from helpers import host

pytestmark = pytest.mark.gpu

H, I, NE, K = 2048, 1792, 32, 4


def _experts(dev):
    """config-5 experts, N(0, 0.02) -> int4 G32 -> int3, identical on any device."""
    import tabinfer_b200 as tb
    ws = []
    for j, (rows, cols) in enumerate(((NE * I, H), (NE * I, H), (NE * H, I))):
        g = torch.Generator(device=dev).manual_seed(300 + j)
        w = (torch.randn(rows, cols, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        pk, sc = tb.quantize_int4_bf16(w.view(torch.int16))
        del w
        ws.append(tb.requant_int3(pk, sc))
    return ws


def _local(ws, P, r):
    El = NE // P
    out = []
    for (p3, s3), n in zip(ws, (I, I, H)):
        out.append((p3[r * El * n:(r + 1) * El * n].contiguous(), s3[r * El * n:(r + 1) * El * n].contiguous()))
    return out


def _tokens(rank, it, T, dev):
    rng = np.random.default_rng(1000 * rank + it)
    logits = rng.standard_normal((T, NE)).astype(np.float32)
    if rank == 1 and it == 0:
        logits[:, :NE // 2] += 8.0            # all of rank 1's tokens to rank 0's experts
    a = rng.standard_normal((T, H)).astype(np.float32)
    x0 = rng.standard_normal((T, H)).astype(np.float32)
    return [torch.from_numpy(v).to(dev) for v in (logits, a, x0)]


def _single(ws, logits, a, x0):
    import tabinfer_b200 as tb
    idx, wt = tb.moe_router(logits, torch.zeros(NE, device=logits.device), K)
    x = x0.clone()
    tb.moe_ffn_int3(x, a, idx, wt, ws[0], ws[1], ws[2], NE, H, I)
    return host(x)


def _runs(rank):
    """tokens per forward of a rank"""
    return [[64, 1, 37], [50, 8, 64]][rank] if rank < 2 else [1 + 9 * rank, 64, 3 + rank]


def _ep_run(rank, P, ws, exchange=None):
    import tabinfer_b200 as tb
    dev = torch.device("cuda", rank)
    ep = tb.MoeEP(P, rank, NE, K, H, I, 64, device=rank)
    if P > 1:
        hq, mine = exchange
        hq.put((rank, ep.handle()))
        ep.connect(mine.get(timeout=120))
    ep.set_experts(*_local(ws, P, rank))
    outs = []
    for it, T in enumerate(_runs(rank)):
        logits, a, x0 = _tokens(rank, it, T, dev)
        idx, wt = tb.moe_router(logits, torch.zeros(NE, device=dev), K)
        x = x0.clone()
        ep.forward(x, a, idx, wt)
        outs.append(host(x))
    err = ep.ctx.device_error()
    ep.close()
    return outs, err


def test_ep1_matches_single_device(cuda):
    ws = _experts(torch.device("cuda", 0))
    outs, err = _ep_run(0, 1, ws)
    assert err == 0
    for it, T in enumerate(_runs(0)):
        ref = _single(ws, *_tokens(0, it, T, torch.device("cuda", 0)))
        np.testing.assert_array_equal(outs[it], ref)


def _rank(rank, P, q, exchange):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        torch.cuda.set_device(rank)
        ws = _experts(torch.device("cuda", rank))
        q.put((rank, _ep_run(rank, P, ws, exchange)))
    except Exception as e:
        q.put((rank, repr(e)))


def test_ep_matches_single_device(cuda):
    n = min(8, torch.cuda.device_count())
    P = 1 << (n.bit_length() - 1) if n > 0 else 0      # 32 experts split evenly: 2, 4 or 8 ranks
    if P < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q, hq = ctx.Queue(), ctx.Queue()
    mine = [ctx.Queue() for _ in range(P)]
    procs = [ctx.Process(target=_rank, args=(r, P, q, (hq, mine[r]))) for r in range(P)]
    for p in procs:
        p.start()
    hs = dict(hq.get(timeout=300) for _ in range(P))
    for m in mine:
        m.put([hs[r] for r in range(P)])
    res = dict(q.get(timeout=300) for _ in range(P))
    for p in procs:
        p.join(timeout=60)
    for r in range(P):
        assert not isinstance(res[r], str), res[r]
        assert res[r][1] == 0, "rank %d device error %#x" % (r, res[r][1])
    ws = _experts(torch.device("cuda", 0))
    for r in range(P):
        for it, T in enumerate(_runs(r)):
            ref = _single(ws, *_tokens(r, it, T, torch.device("cuda", 0)))
            np.testing.assert_array_equal(res[r][0][it], ref, err_msg="rank %d forward %d" % (r, it))
