"""Tensor-parallel host logic on CPU (no GPU): the shard plan the model runner
uses (tb_qwen3_shard), and a world_size-2 gloo emulation of the two exchanges
of the TP decode step — the allreduce of row-split o/down partial products and
the cross-rank argmax merge — checked against the single-device oracle."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from helpers import bf16_normal

Q17 = dict(hidden=2048, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=6144, vocab=151936,
           rope_theta=1e6, rms_eps=1e-6, max_seq=4096, batch=1)


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_shard_plan_partitions_every_tensor(P):
    from tabinfer_b200 import _lib, qwen3
    full = {_lib.QW_Q: (2048, 2048), _lib.QW_K: (1024, 2048), _lib.QW_V: (1024, 2048), _lib.QW_O: (2048, 2048),
            _lib.QW_GATE: (6144, 2048), _lib.QW_UP: (6144, 2048), _lib.QW_DOWN: (2048, 6144),
            _lib.QW_LM_HEAD: (151936, 2048)}
    for kind, (R, C) in full.items():
        blocks = [qwen3.shard(dict(Q17, tp_size=P, tp_rank=r), kind) for r in range(P)]
        rows_split = any(b[1] != R for b in blocks)
        cols_split = any(b[3] != C for b in blocks)
        assert not (rows_split and cols_split)
        # the split dimension is cut into consecutive, non-overlapping pieces in
        # rank order; a column (K) cut also lands on a 32-group boundary
        lo, hi = (0, 1) if not cols_split else (2, 3)
        edge = 0
        for b in blocks:
            assert b[lo] == edge
            edge += b[hi]
            if cols_split:
                assert b[2] % 32 == 0 and b[3] % 32 == 0
            assert (b[0], b[1]) == (b[0], R) or rows_split
        assert edge == (C if cols_split else R), "kind %d at P=%d" % (kind, P)
    # kv heads are sharded whole and q heads follow their kv group (GQA 2:1)
    for r in range(P):
        cfg = dict(Q17, tp_size=P, tp_rank=r)
        q0, qn, _, _ = qwen3.shard(cfg, _lib.QW_Q)
        k0, kn, _, _ = qwen3.shard(cfg, _lib.QW_K)
        assert qn == 2 * kn and q0 == 2 * k0 and k0 % 128 == 0


def test_shard_plan_rejects_bad_splits():
    from tabinfer_b200 import _lib, qwen3
    with pytest.raises(ValueError):
        qwen3.shard(dict(Q17, tp_size=3, tp_rank=0), _lib.QW_Q)      # 8 kv heads over 3 ranks
    with pytest.raises(ValueError):
        qwen3.shard(dict(Q17, tp_size=16, tp_rank=0), _lib.QW_Q)


def test_activation_groups_survive_the_split():
    """Per-32 int8 quantization of a rank's attn/swi slice equals the matching
    groups of the full row's quantization: every slice starts on a group."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal(6144).astype(np.float32)
    fq, fs, _ = oracle.quant_q8(x)
    for P in (2, 4, 8):
        w = 6144 // P
        for r in range(P):
            q, s, _ = oracle.quant_q8(x[r * w:(r + 1) * w])
            assert (q == fq[:, r * w:(r + 1) * w]).all()
            assert (s == fs[:, r * w // 32:(r + 1) * w // 32]).all()


def _rank(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tabinfer_b200 import _lib, qwen3
        cfg = dict(hidden=256, layers=1, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512, vocab=96,
                   rope_theta=1e6, rms_eps=1e-6, max_seq=8, batch=1, tp_size=world, tp_rank=rank)
        rng = np.random.default_rng(42)                      # same full tensors on every rank
        Wo = bf16_normal(rng, (256, 256), 0.02)
        Wd = bf16_normal(rng, (256, 512), 0.02)
        attn = rng.standard_normal(256).astype(np.float32)
        swi = rng.standard_normal(512).astype(np.float32)
        x = rng.standard_normal(256)
        out = {}
        for name, W, a, kind in (("o", Wo, attn, _lib.QW_O), ("down", Wd, swi, _lib.QW_DOWN)):
            r0, nr, c0, nc = qwen3.shard(cfg, kind)
            pack, sc = oracle.quant_int4_g32(np.ascontiguousarray(W[r0:r0 + nr, c0:c0 + nc]))
            aq, as_, _ = oracle.quant_q8(a[c0:c0 + nc])
            part = oracle.gemv_int4_q8act(aq, as_, pack, sc)[0]
            y = torch.from_numpy(part + (x if rank == 0 else 0.0))   # rank 0 carries the residual
            dist.all_reduce(y)
            out[name] = y.numpy()
        # argmax merge: ranks hold vocab rows [r*V/P, ...); the winner is the
        # largest value, then the lowest global index (a tie across ranks)
        V = cfg["vocab"]
        logits = rng.standard_normal(V).astype(np.float32)
        logits[5] = logits[V - 7] = np.float32(9.0)
        r0, nr, _, _ = qwen3.shard(cfg, _lib.QW_LM_HEAD)
        loc = logits[r0:r0 + nr]
        i = int(np.argmax(loc))
        key = torch.tensor([float(loc[i]), -(r0 + i)], dtype=torch.float64)
        keys = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(keys, key)
        best = max(keys, key=lambda k: (k[0].item(), k[1].item()))
        out["argmax"] = int(-best[1].item())
        if rank == 0:
            ret.put(out)
    finally:
        dist.destroy_process_group()


def test_tp_exchanges_match_single_device_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(42)
    Wo = bf16_normal(rng, (256, 256), 0.02)
    Wd = bf16_normal(rng, (256, 512), 0.02)
    attn = rng.standard_normal(256).astype(np.float32)
    swi = rng.standard_normal(512).astype(np.float32)
    x = rng.standard_normal(256)
    for name, W, a in (("o", Wo, attn), ("down", Wd, swi)):
        pack, sc = oracle.quant_int4_g32(W)
        aq, as_, _ = oracle.quant_q8(a)
        ref = x + oracle.gemv_int4_q8act(aq, as_, pack, sc)[0]
        np.testing.assert_allclose(got[name], ref, rtol=1e-12, atol=1e-12)
    assert got["argmax"] == 5
