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
