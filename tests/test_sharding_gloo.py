"""Host logic of the multi-GPU partitions, on CPU ranks over gloo (world size 2
and 4). The per-rank compute is the CPU oracle here; on GPUs it is the d2sd
kernels and the transport is NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from d2sd_b200 import sharding as S


def test_head_ranges_partition_the_heads():
    for Hq, Hk in ((32, 8), (64, 8)):
        for world in (1, 2, 4, 8):
            seen_k, seen_q = [], []
            for r in range(world):
                a, b = S.kv_head_range(Hk, world, r)
                c, d = S.qo_head_range(Hq, Hk, world, r)
                seen_k += list(range(a, b))
                seen_q += list(range(c, d))
                assert all(h // (Hq // Hk) in range(a, b) for h in range(c, d))
            assert seen_k == list(range(Hk)) and seen_q == list(range(Hq))
    with pytest.raises(ValueError):
        S.kv_head_range(8, 3, 0)


def test_lpt_partition_balanced_and_deterministic():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 8193, 64)
    costs = S.request_costs(lens, [64] * 64)
    bins = S.lpt_partition(costs, 8)
    assert sorted(sum(bins, [])) == list(range(64))
    loads = [sum(costs[i] for i in b) for b in bins]
    assert max(loads) <= min(loads) * 1.10
    assert bins == S.lpt_partition(costs, 8)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, kn, vn, kp, vp, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import attention as AT
        B, T, Hq, D = q.shape
        Hk = kn.shape[2]

        def compute(ql, kl, vl, layer):
            # ql [B*T, hq, D]: the rank's heads of the cascade attention
            hq, hk = ql.shape[1], kl.shape[1]
            a, b = S.kv_head_range(Hk, world, rank)
            o, _ = AT.cascade_attention(ql.reshape(B, T, hq, D), kl.reshape(B, T, hk, D),
                                        vl.reshape(B, T, hk, D), kp[:, a:b], vp[:, a:b])
            return torch.from_numpy(o).float().reshape(B * T, hq, D)

        att = S.KVHeadShardedAttention(None, Hq, Hk, D, B * T, torch.float32, "cpu", compute)
        ql, kl, vl = att.local_slices(q.reshape(B * T, Hq, D), kn.reshape(B * T, Hk, D),
                                      vn.reshape(B * T, Hk, D))
        full = att.forward(ql, kl, vl, 0)
        if rank == 0:
            ret.put(full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_kv_head_sharded_equals_unsharded(world):
    g = torch.Generator().manual_seed(world)
    B, T, Hq, Hk, D, P = 2, 4, 8, 4, 16, 40
    q = torch.randn(B, T, Hq, D, generator=g)
    kn = torch.randn(B, T, Hk, D, generator=g)
    vn = torch.randn(B, T, Hk, D, generator=g)
    kp = torch.randn(P, Hk, D, generator=g)
    vp = torch.randn(P, Hk, D, generator=g)
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, kn, vn, kp, vp, ret))
             for r in range(world)]
    for p in procs:
        p.start()
    full = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from oracle import attention as AT
    ref, _ = AT.cascade_attention(q, kn, vn, kp, vp)
    np.testing.assert_allclose(full, ref.reshape(B * T, Hq, D), atol=1e-5)


def test_vocab_ranges_partition_the_vocabulary():
    for V in (151936, 201088, 1000, 7):
        for world in (1, 2, 3, 4, 8):
            cols = [S.vocab_range(V, world, r) for r in range(world)]
            assert cols[0][0] == 0 and cols[-1][1] == V
            assert all(cols[r][1] == cols[r + 1][0] for r in range(world - 1))
            widths = [b - a for a, b in cols]
            assert max(widths) - min(widths) <= 1


def _better(va, ia, vb, ib):
    """The total order kernel (c) keeps: NaN above every number, larger value
    first, equal values -> smaller index (accept.cu, better())."""
    na, nb = va != va, vb != vb
    if na or nb:
        return ia < ib if (na and nb) else na
    if va != vb:
        return va > vb
    return ia < ib


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_sharded_argmax_combine_equals_torch_argmax(world):
    """Vocabulary-sharded acceptance: each rank's (max, first index) over its
    slice, combined over the ranks in rank order with the kernel's order, is
    torch.argmax of the whole row -- ties across a slice boundary and NaNs
    included."""
    g = torch.Generator().manual_seed(world)
    V = 997
    rows = torch.randn(64, V, generator=g).to(torch.bfloat16).float()
    rows[1, [10, 500, 900]] = 9.0                       # ties in three slices
    rows[2, :] = -float("inf")                          # all -inf: index 0
    rows[3, [700, 20]] = float("nan")                   # first NaN wins
    lo, hi = S.vocab_range(V, world, 1)
    rows[4, [lo - 1, lo]] = 7.5                         # tie across a boundary
    for r in range(rows.shape[0]):
        best_v, best_i = -float("inf"), None
        for k in range(world):
            a, b = S.vocab_range(V, world, k)
            sl = rows[r, a:b]
            if b > a:
                i = int(torch.argmax(sl))              # the slice's first maximal index
                v, i = float(sl[i]), a + i
                if best_i is None or _better(v, i, best_v, best_i):
                    best_v, best_i = v, i
        assert best_i == int(torch.argmax(rows[r])), r
