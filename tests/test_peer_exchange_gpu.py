"""The NVLink exchanges fused into kernels (b) and (c).

1 GPU: each exchange's bounded wait runs out (a peer slot that nothing
signals) and the kernel returns with status 3 instead of hanging; the context
stays usable.

2, 4 and 8 GPUs (skipped when fewer are present), one process per GPU:
* KV-head sharding: kernel (b)'s epilogue stores each rank's rows into every
  rank's output; the gathered [tokens, Hq, D] output of every call is compared
  with the float64 oracle of the whole attention. The calls change their number
  of blocks (so the grid changes between calls) and one rank lags on the host
  before reading each output, so a peer that ran ahead would overwrite an
  unread buffer if the double buffering were wrong.
* Vocabulary-sharded acceptance: each rank scans 1/world of [8, 32, V] logits;
  every rank's acceptance length, ids and branch equal the oracle's bit for bit.
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _LocalExchange:
    """A two-rank exchange whose 'peer' is a second buffer on the same GPU
    that no kernel ever signals: the wait must run out."""

    def __init__(self, tokens, hq, d, dev):
        self.world, self.rank, self.head_offset, self.epoch = 2, 0, 0, 0
        self.buffers = torch.zeros(2, tokens, 2 * hq, d, dtype=torch.bfloat16, device=dev)
        self.peer = torch.zeros_like(self.buffers)
        self.control = torch.zeros(2, 8, dtype=torch.int64, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        par = self.buffers[0].numel() * 2
        self.out_ptrs = torch.tensor([self.buffers.data_ptr(), self.peer.data_ptr(),
                                      self.buffers.data_ptr() + par, self.peer.data_ptr() + par],
                                     dtype=torch.int64, device=dev)
        self.counter_ptrs = torch.tensor([self.control[0].data_ptr(), self.control[1].data_ptr()],
                                         dtype=torch.int64, device=dev)

    def next_epoch(self):
        self.epoch += 1
        return self.epoch


def test_exchange_wait_times_out_with_status(cuda_device):
    import d2sd_b200 as d
    from d2sd_b200 import ops
    dev = cuda_device
    B, T, Hq, Hk, D, P = 2, 16, 8, 2, 128, 300
    g = torch.Generator().manual_seed(1)
    bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).to(dev)  # noqa: E731
    q, kn, vn, kp, vp = bf(B * T, Hq, D), bf(B * T, Hk, D), bf(B * T, Hk, D), bf(P, Hk, D), bf(P, Hk, D)
    plan = d.CascadePlan([d.Request(B * T, 0, 0, P)], Hq, Hk, D, dev)
    plan.run_prefix(q, kp, vp, "nhd", D ** -0.5)
    x = _LocalExchange(B * T, Hq, D, dev)
    out = torch.empty(B * T, Hq, D, dtype=torch.bfloat16, device=dev)
    t0 = time.time()
    ops.suffix_merge(q, kn, vn, out, None, num_blocks=B, block_len=T, num_qo_heads=Hq,
                     num_kv_heads=Hk, sm_scale=D ** -0.5, partial=plan.partial,
                     plan_dev=plan.plan, exchange=x)
    torch.cuda.synchronize()
    assert int(x.status.item()) == 3
    assert time.time() - t0 < 30
    # this rank's own signal arrived, the missing peer's did not; the ticket is free again
    assert int(x.control[0, 1].item()) == 1 and int(x.control[0, 2].item()) == 0
    # the rows were stored into both 'ranks' buffers of the odd parity
    assert torch.equal(x.buffers[1, :, :Hq], x.peer[1, :, :Hq])
    assert x.buffers[1, :, :Hq].abs().sum() > 0
    # the context is still usable
    assert float(torch.ones(4, device=dev).sum().item()) == 4.0


def test_sharded_accept_wait_times_out_with_status(cuda_device):
    from d2sd_b200 import ops
    dev = cuda_device
    B, T, V = 4, 8, 4096
    g = torch.Generator().manual_seed(2)
    logits = torch.randn(1, B, T, V // 2, generator=g).to(torch.bfloat16).to(dev)
    ids = torch.randint(0, V, (1, B, T), generator=g).to(dev)
    rows = B * T

    class X:
        world, rank, epoch, rows_ = 2, 0, 0, rows
        records = torch.zeros(2, 2, 2, rows, 4, dtype=torch.int32, device=dev)  # [rank-local][...]
        control = torch.zeros(2, 8, dtype=torch.int64, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)

        def next_epoch(self):
            self.epoch += 1

    x = X()
    x.rows = rows
    par = x.records[0, 0].numel() * 4
    x.record_ptrs = torch.tensor([x.records[0].data_ptr(), x.records[1].data_ptr(),
                                  x.records[0].data_ptr() + par, x.records[1].data_ptr() + par],
                                 dtype=torch.int64, device=dev)
    x.control_ptrs = torch.tensor([x.control[0].data_ptr(), x.control[1].data_ptr()],
                                  dtype=torch.int64, device=dev)
    ws = torch.zeros(ops.accept_batch_workspace_bytes(1, B, T, V // 2), dtype=torch.uint8,
                     device=dev)
    result = torch.zeros(1, 2, dtype=torch.int32, device=dev)
    acc = torch.zeros(1, T, dtype=torch.int64, device=dev)
    ops.verify_accept_sharded(logits, 0, ids, result, acc, ws, x)
    torch.cuda.synchronize()
    assert int(x.status.item()) == 3
    assert 1 <= int(result[0, 0].item()) <= T  # the walk still ran and wrote a result
    assert float(torch.ones(4, device=dev).sum().item()) == 4.0


def _worker(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    import d2sd_b200 as d
    from d2sd_b200 import ops
    from d2sd_b200.sharding import kv_head_range, qo_head_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    px = sv = None
    try:
        T, Hq, Hk, D, P = 16, 32, 8, 128, 4096
        blocks = [8, 3, 8, 5]  # the grid changes from call to call
        k0, k1 = kv_head_range(Hk, world, rank)
        h0, h1 = qo_head_range(Hq, Hk, world, rank)
        hk, hq = k1 - k0, h1 - h0
        px = d.PeerExchange(max(blocks) * T, Hq, Hk, D, torch.bfloat16, dev)
        outs = []
        for e, B in enumerate(blocks):
            N = B * T
            g = torch.Generator().manual_seed(100 + e)  # same inputs on every rank
            bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
            q, kn, vn, kp, vp = bf(N, Hq, D), bf(N, Hk, D), bf(N, Hk, D), bf(P, Hk, D), bf(P, Hk, D)
            cache = d.PagedKVCache(1, hk, D, P + 64, device=dev,
                                   page_order=torch.randperm(-(-(P + 64) // 16), generator=g))
            cache.write(0, kp[:, k0:k1].to(dev), vp[:, k0:k1].to(dev))
            plan = d.CascadePlan([d.Request(N, 0, 0, P)], hq, hk, D, dev)
            ql = q[:, h0:h1].contiguous().to(dev)
            plan.run_prefix(ql, cache.k[0], cache.v[0], cache.kv_layout, D ** -0.5,
                            page_table=cache.page_table)
            out = torch.empty(N, hq, D, dtype=torch.bfloat16, device=dev)
            ops.suffix_merge(ql, kn[:, k0:k1].contiguous().to(dev),
                             vn[:, k0:k1].contiguous().to(dev), out, None, num_blocks=B,
                             block_len=T, num_qo_heads=hq, num_kv_heads=hk, sm_scale=D ** -0.5,
                             partial=plan.partial, plan_dev=plan.plan, exchange=px)
            if rank == 1:
                time.sleep(0.3)  # this rank reads its output late; the others run ahead
            outs.append(px.buffer[:N].float().cpu().numpy())
            assert int(plan.status.item()) == 0
        torch.cuda.synchronize()
        stats = px.wait_stats()

        # vocabulary-sharded acceptance over [1, 8, 32, V]
        B, T, V = 8, 32, 151936
        sv = d.ShardedVerifier(1, B, T, V, dev)
        c0, c1 = sv.columns
        accs = []
        for e in range(3):
            gz = torch.Generator(device=dev).manual_seed(200 + e)
            z = torch.randn(1, B, T, V, generator=gz, device=dev).to(torch.bfloat16)
            if e == 2:  # ties across slice boundaries: the first maximal index must win
                z[0, :, :, c0] = 9.0
                z[0, :, :, 0] = 9.0
            x = torch.randint(0, V, (1, B, T), generator=gz, device=dev)
            keep = torch.rand(1, B, T, generator=gz, device=dev) < 0.7
            x[:, :, 1:] = torch.where(keep[:, :, 1:], z.float().argmax(-1)[:, :, :-1], x[:, :, 1:])
            x[:, :, 0] = x[:, 0:1, 0]
            sv.launch(z[..., c0:c1], x)
            accs.append((sv.result.cpu().numpy().copy(), sv.accepted.cpu().numpy().copy(),
                         z[0].float().cpu().numpy() if rank == 0 else None,
                         x[0].cpu().numpy()))
        torch.cuda.synchronize()
        results[rank] = {"outs": outs, "status": int(px.status.item()), "stats": stats,
                         "acc": accs, "acc_status": int(sv.status.item())}
        dist.barrier()
    finally:
        if px is not None:
            px.close()
        if sv is not None:
            sv.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_sharded_exchange_matches_oracle(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    from oracle import accept as OA
    from oracle import attention as AT
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    T, Hq, Hk, D, P = 16, 32, 8, 128, 4096
    for e, B in enumerate([8, 3, 8, 5]):
        N = B * T
        g = torch.Generator().manual_seed(100 + e)
        bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
        q, kn, vn, kp, vp = bf(N, Hq, D), bf(N, Hk, D), bf(N, Hk, D), bf(P, Hk, D), bf(P, Hk, D)
        ro, _ = AT.cascade_attention(q.double().view(B, T, Hq, D), kn.double().view(B, T, Hk, D),
                                     vn.double().view(B, T, Hk, D), kp.double(), vp.double(),
                                     causal=True)
        for r in range(world):
            got = results[r]["outs"][e].reshape(B, T, Hq, D)
            np.testing.assert_allclose(got, ro, atol=ATOL, rtol=RTOL, err_msg=f"rank {r} call {e}")
            assert np.array_equal(got, results[0]["outs"][e].reshape(B, T, Hq, D))
    for r in range(world):
        assert results[r]["status"] == 0, f"rank {r}: the output exchange timed out"
        assert results[r]["acc_status"] == 0, f"rank {r}: the acceptance exchange timed out"
        assert results[r]["stats"]["waits"] == 4
    for e in range(3):
        _, _, z, x = results[0]["acc"][e]
        racc, rids, rbranch = OA.verify_accept(z, x)
        for r in range(world):
            res, acc_ids, _, _ = results[r]["acc"][e]
            assert (int(res[0, 0]), int(res[0, 1])) == (racc, rbranch), (r, e)
            np.testing.assert_array_equal(acc_ids[0, :racc], rids)
