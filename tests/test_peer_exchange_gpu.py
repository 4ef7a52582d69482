"""KV-head sharding on 2 GPUs: the output all-gather fused into kernel (b)
(peer stores over NVLink + arrival counters) equals NCCL's all_gather of the
same kernel's local output, bit for bit, over several calls (epochs). Needs two
GPUs; skipped otherwise."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    import d2sd_b200 as d
    from d2sd_b200 import ops
    from d2sd_b200.sharding import assemble_heads, kv_head_range, qo_head_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    px = None
    try:
        B, T, Hq, Hk, D, P = 4, 16, 32, 8, 128, 777
        N = B * T
        g = torch.Generator().manual_seed(3)
        bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
        q, kn, vn, kp, vp = bf(N, Hq, D), bf(N, Hk, D), bf(N, Hk, D), bf(P, Hk, D), bf(P, Hk, D)
        k0, k1 = kv_head_range(Hk, world, rank)
        h0, h1 = qo_head_range(Hq, Hk, world, rank)
        hk, hq = k1 - k0, h1 - h0
        cache = d.PagedKVCache(1, hk, D, P + 64, device=dev)
        cache.write(0, kp[:, k0:k1].to(dev), vp[:, k0:k1].to(dev))
        cache.length = P
        ql = q[:, h0:h1].contiguous().to(dev)
        knl = kn[:, k0:k1].contiguous().to(dev)
        vnl = vn[:, k0:k1].contiguous().to(dev)
        plan = d.CascadePlan([d.Request(N, 0, 0, P)], hq, hk, D, dev)
        out = torch.empty(N, hq, D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(N, hq, dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        px = d.PeerExchange(N, Hq, Hk, D, torch.bfloat16, dev)
        gathered = torch.empty(world * N, hq, D, dtype=torch.bfloat16, device=dev)
        worst = 0.0
        for epoch in range(3):
            scale = D ** -0.5 * (1.0 + 0.1 * epoch)
            plan.run_prefix(ql, cache.k[0], cache.v[0], cache.kv_layout, scale,
                            page_table=cache.page_table)
            kw = dict(num_blocks=B, block_len=T, num_qo_heads=hq, num_kv_heads=hk, sm_scale=scale,
                      partial=plan.partial, plan_dev=plan.plan)
            ops.suffix_merge(ql, knl, vnl, out, lse, **kw)
            dist.all_gather_into_tensor(gathered, out)
            ref = assemble_heads(gathered.view(world, N, hq, D))
            ops.suffix_merge(ql, knl, vnl, out, lse, status=status, exchange=px, **kw)
            torch.cuda.synchronize()
            worst = max(worst, float((px.buffer.float() - ref.float()).abs().max()))
        results[rank] = (worst, int(status.item()))
        dist.barrier()
    finally:
        if px is not None:
            px.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_peer_exchange_matches_nccl_all_gather():
    import torch.multiprocessing as mp
    world = 2
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    for r in range(world):
        worst, status = results[r]
        assert status == 0, f"rank {r}: exchange wait ran out of time"
        assert worst == 0.0, f"rank {r}: gathered rows differ by {worst}"
