"""Kernels (a)-(d) at the exact shapes the benchmark reports, against the
float64 CPU oracle on identical seeded inputs.

* Config 3 (the north-star shape): prefix 32768 in 16-key UMMA pages with a
  shuffled page table, 8 branches x 32 tokens, 32/8 heads, D 128, tree trunks
  k in {0, 4, 8}; and every per-rank KV-head shard the multi-GPU benchmark
  runs (hk = 4, 2, 1 kv heads with their 4*hk query heads and pages).
* Config 5 (GPT-OSS-20B shapes): prefix 16384, 6 x 16 tokens, 64/8 heads,
  D 64, full and 128-token sliding layers, sinks in both modes.
* Config 4 (batched serving): 64 requests with seeded prefix lengths in
  [512, 8192] in one page pool, 4 x 16 tokens each: one kernel (a) launch over
  all requests, one kernel (b) launch, batched acceptance over [64, 4, 16,
  151936] bf16 logits and the batched commit.

Tolerances (north star): attention outputs within 2e-2 abs / 1e-2 rel of the
oracle, base-2 LSEs within 1e-2; acceptance and committed KV bit-exact. Every
kernel's status word must read 0.
"""
import numpy as np
import pytest
import torch

from oracle import accept as OA
from oracle import attention as AT

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-2, 1e-2, 1e-2


def f64(t):
    return t.detach().double().cpu().numpy()


def close(a, b, atol=ATOL, rtol=RTOL):
    np.testing.assert_allclose(f64(a) if torch.is_tensor(a) else a, b, atol=atol, rtol=rtol)


def bf(gen, *shape):
    return torch.randn(*shape, generator=gen).to(torch.bfloat16)


# ---------------------------------------------------------------------------
# config 3
# ---------------------------------------------------------------------------
C3 = dict(P=32768, B=8, T=32, Hq=32, Hk=8, D=128)


@pytest.fixture(scope="module")
def cfg3():
    g = torch.Generator().manual_seed(3)
    c = C3
    data = {
        "q": bf(g, c["B"], c["T"], c["Hq"], c["D"]),
        "kn": bf(g, c["B"], c["T"], c["Hk"], c["D"]),
        "vn": bf(g, c["B"], c["T"], c["Hk"], c["D"]),
        "kp": bf(g, c["P"], c["Hk"], c["D"]),
        "vp": bf(g, c["P"], c["Hk"], c["D"]),
        "order": torch.randperm(-(-(c["P"] + c["T"] + 16) // 16), generator=g),
    }
    data["oracle"] = AT.cascade_attention(f64(data["q"]), f64(data["kn"]), f64(data["vn"]),
                                          f64(data["kp"]), f64(data["vp"]), causal=True)
    return data


def run_cascade(dev, q, kn, vn, kp, vp, order, shared=0, window=None, sinks=None,
                sink_mode="reference"):
    """The benchmark's path: a paged UMMA cache with the given page order, one
    plan, kernel (a) then kernel (b); returns (out, lse) after checking both
    kernels' status words."""
    import d2sd_b200 as d
    B, T, Hq, D = q.shape
    Hk, P = kn.shape[2], kp.shape[0]
    cache = d.PagedKVCache(1, Hk, D, P + T + 16, device=dev, layout="umma", page_order=order)
    cache.write(0, kp.to(dev), vp.to(dev))
    cache.length = P
    kv_start = max(0, P - window) if window is not None else 0
    n_u = shared + B * (T - shared) if shared else B * T
    plan = d.CascadePlan([d.Request(n_u, 0, kv_start, P)], Hq, Hk, D, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out, lse = d.cascade_attention(q.to(dev), kn.to(dev), vn.to(dev), cache.k[0], cache.v[0],
                                   cache.kv_layout, P, page_table=cache.page_table,
                                   sliding_window=window, shared_tokens=shared, plan=plan,
                                   sinks=None if sinks is None else sinks.to(dev),
                                   sink_mode=sink_mode, status=status)
    torch.cuda.synchronize()
    assert int(plan.status.item()) == 0, "kernel (a) reported a wait time-out"
    assert int(status.item()) == 0, "kernel (b) reported a wait time-out"
    return out, lse


@pytest.mark.parametrize("shared", [0, 4, 8])
def test_cfg3_north_star_shape(cuda_device, cfg3, shared):
    q, kn, vn = cfg3["q"].clone(), cfg3["kn"].clone(), cfg3["vn"].clone()
    if shared:
        q[:, :shared] = q[0:1, :shared]
        kn[:, :shared] = kn[0:1, :shared]
        vn[:, :shared] = vn[0:1, :shared]
        ro, rl = AT.cascade_attention(f64(q), f64(kn), f64(vn), f64(cfg3["kp"]), f64(cfg3["vp"]),
                                      causal=True)
    else:
        ro, rl = cfg3["oracle"]
    out, lse = run_cascade(cuda_device, q, kn, vn, cfg3["kp"], cfg3["vp"], cfg3["order"], shared)
    close(out, ro)
    close(lse, rl, atol=LSE_ATOL)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_cfg3_kv_head_shards(cuda_device, cfg3, world):
    """What each rank of bench.py --gpus N computes: its kv heads' pages, its
    query heads, its own plan over the full grid of one GPU."""
    Hk, Hq = C3["Hk"], C3["Hq"]
    hk, G = Hk // world, Hq // Hk
    ro, rl = cfg3["oracle"]
    for rank in sorted({0, world - 1}):
        k0, k1 = rank * hk, (rank + 1) * hk
        h0, h1 = k0 * G, k1 * G
        out, lse = run_cascade(cuda_device, cfg3["q"][:, :, h0:h1].contiguous(),
                               cfg3["kn"][:, :, k0:k1].contiguous(),
                               cfg3["vn"][:, :, k0:k1].contiguous(),
                               cfg3["kp"][:, k0:k1].contiguous(), cfg3["vp"][:, k0:k1].contiguous(),
                               cfg3["order"])
        close(out, ro[:, :, h0:h1])
        close(lse, rl[:, :, h0:h1], atol=LSE_ATOL)


# ---------------------------------------------------------------------------
# config 5
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg5():
    g = torch.Generator().manual_seed(5)
    P, B, T, Hq, Hk, D = 16384, 6, 16, 64, 8, 64
    return {"q": bf(g, B, T, Hq, D), "kn": bf(g, B, T, Hk, D), "vn": bf(g, B, T, Hk, D),
            "kp": bf(g, P, Hk, D), "vp": bf(g, P, Hk, D), "sinks": torch.randn(Hq, generator=g),
            "order": torch.randperm(-(-(P + T + 16) // 16), generator=g)}


@pytest.mark.parametrize("window", [None, 128])
@pytest.mark.parametrize("sink_mode", ["reference", "exact"])
def test_cfg5_gptoss_shape(cuda_device, cfg5, window, sink_mode):
    c = cfg5
    out, lse = run_cascade(cuda_device, c["q"], c["kn"], c["vn"], c["kp"], c["vp"], c["order"],
                           window=window, sinks=c["sinks"], sink_mode=sink_mode)
    ro, rl = AT.cascade_attention(f64(c["q"]), f64(c["kn"]), f64(c["vn"]), f64(c["kp"]),
                                  f64(c["vp"]), causal=True, sliding_window=window,
                                  sinks=f64(c["sinks"]), sink_mode=sink_mode)
    close(out, ro)
    close(lse, rl, atol=LSE_ATOL)


# ---------------------------------------------------------------------------
# config 4
# ---------------------------------------------------------------------------
def test_cfg4_batched_serving(cuda_device):
    import d2sd_b200 as d
    from d2sd_b200 import ops
    dev = cuda_device
    R, B, T, Hq, Hk, D, V, L = 64, 4, 16, 32, 8, 128, 151936, 2
    lens = np.random.default_rng(4).integers(512, 8193, R).tolist()
    g = torch.Generator().manual_seed(44)
    pool = d.PagedKVPool(L, Hk, D, [p + T + 16 for p in lens], device=dev, shuffle_seed=7)
    kps, vps = [], []
    for r, P in enumerate(lens):
        kp, vp = bf(g, P, Hk, D), bf(g, P, Hk, D)
        for l in range(L):
            pool.write_seq(l, r, kp.to(dev), vp.to(dev))
        kps.append(kp)
        vps.append(vp)
    pool.set_lengths(lens)
    N = R * B * T
    q, kn, vn = bf(g, N, Hq, D), bf(g, N, Hk, D), bf(g, N, Hk, D)
    reqs = [d.Request(B * T, r * B * T, 0, P, pool.page_offsets_host[r])
            for r, P in enumerate(lens)]
    plan = d.CascadePlan(reqs, Hq, Hk, D, dev)
    qd, knd, vnd = q.to(dev), kn.to(dev), vn.to(dev)
    plan.run_prefix(qd, pool.k[0], pool.v[0], pool.kv_layout, D ** -0.5,
                    page_table=pool.page_table)
    out = torch.empty(N, Hq, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(N, Hq, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.suffix_merge(qd, knd, vnd, out, lse, num_blocks=R * B, block_len=T, num_qo_heads=Hq,
                     num_kv_heads=Hk, sm_scale=D ** -0.5, partial=plan.partial,
                     plan_dev=plan.plan, status=status)

    # acceptance over every request's logits in one launch, then the batched commit
    gz = torch.Generator(device=dev).manual_seed(45)
    logits = torch.randn(R, B, T, V, generator=gz, device=dev).to(torch.bfloat16)
    ids = torch.randint(0, V, (R, B, T), generator=gz, device=dev)
    keep = torch.rand(R, B, T, generator=gz, device=dev) < 0.7
    ids[:, :, 1:] = torch.where(keep[:, :, 1:], logits.float().argmax(-1)[:, :, :-1],
                                ids[:, :, 1:])
    ids[:, :, 0] = ids[:, 0:1, 0]
    ver = d.BatchVerifier(R, B, T, V, dev)
    argmax = torch.empty(R, B, T, dtype=torch.int64, device=dev)
    ver.launch(logits, ids, argmax)
    new_k = torch.stack([kn.view(R * B, T, Hk, D).transpose(1, 2)] * L).to(dev)  # [L, R*B, Hk, T, D]
    new_v = torch.stack([vn.view(R * B, T, Hk, D).transpose(1, 2)] * L).to(dev)
    pool.commit_batch(new_k, new_v, ver.result, num_branches=B)
    torch.cuda.synchronize()
    assert int(plan.status.item()) == 0 and int(status.item()) == 0

    for r, P in enumerate(lens):
        sl = slice(r * B * T, (r + 1) * B * T)
        ro, rl = AT.cascade_attention(f64(q[sl]).reshape(B, T, Hq, D),
                                      f64(kn[sl]).reshape(B, T, Hk, D),
                                      f64(vn[sl]).reshape(B, T, Hk, D), f64(kps[r]), f64(vps[r]),
                                      causal=True)
        close(out[sl].reshape(B, T, Hq, D), ro)
        close(lse[sl].reshape(B, T, Hq), rl, atol=LSE_ATOL)

    res = ver.result.cpu().numpy()
    acc_ids = ver.accepted.cpu().numpy()
    am = argmax.cpu().numpy()
    ids_c = ids.cpu()
    for r in range(R):
        sl = slice(r * B * T, (r + 1) * B * T)
        z = logits[r].float().cpu()
        racc, rids, rbranch = OA.verify_accept(z, ids_c[r])
        assert (int(res[r, 0]), int(res[r, 1])) == (racc, rbranch), r
        np.testing.assert_array_equal(acc_ids[r, :racc], rids)
        assert (acc_ids[r, racc:] == -1).all()
        np.testing.assert_array_equal(am[r], z.argmax(-1).numpy())
        # committed rows: block positions 0..acc-1 of the winning branch, every layer
        for l in range(L):
            gk, gv = pool.gather_seq(l, r, lens[r] + racc)
            exp_k = torch.cat([kps[r], kn[sl].view(B, T, Hk, D)[rbranch, :racc]], 0)
            exp_v = torch.cat([vps[r], vn[sl].view(B, T, Hk, D)[rbranch, :racc]], 0)
            assert torch.equal(gk.cpu(), exp_k) and torch.equal(gv.cpu(), exp_v), (r, l)
