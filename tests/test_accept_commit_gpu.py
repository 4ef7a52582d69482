"""Kernels (c) acceptance and (d) KV commit: bit-exact against the golden
vectors of the reference and the CPU oracle."""
import numpy as np
import pytest
import torch

from conftest import decode_logits, load_cases
from oracle import accept as OA
from oracle import commit as OC

pytestmark = pytest.mark.gpu


def test_accept_golden(cuda_device):
    import d2sd_b200 as d
    for c in load_cases("accept_cases.npz"):
        logits = decode_logits(c).to(cuda_device)
        ids = torch.from_numpy(c["block_ids"]).to(cuda_device)
        acc, got, branch = d.verify(logits, ids)
        assert acc == int(c["acc"]), (c["block_ids"].shape, c["dtype"])
        assert branch == int(c["branch"])
        np.testing.assert_array_equal(got.cpu().numpy(), c["ids"])


def test_accept_argmax_matches_torch(cuda_device):
    import d2sd_b200 as d
    for c in load_cases("accept_cases.npz")[::7]:
        logits = decode_logits(c).to(cuda_device)
        ids = torch.from_numpy(c["block_ids"]).to(cuda_device)
        ver = d.Verifier(*logits.shape, cuda_device)
        ver.launch(logits, ids)
        torch.cuda.synchronize()
        ref = logits.float().argmax(-1).reshape(-1)
        assert torch.equal(ver.argmax, ref)


@pytest.mark.parametrize("B,T,V,dtype", [
    (8, 32, 151936, torch.bfloat16),   # north-star shape, Qwen3 vocab
    (4, 16, 151936, torch.float32),
    (6, 16, 201088, torch.bfloat16),   # GPT-OSS vocab
    (3, 5, 1001, torch.float16),       # odd vocab: unaligned rows, scalar tails
    (64, 2, 333, torch.float32),       # maximum branch count
    (1, 32, 151936, torch.bfloat16),   # DFlash single branch
])
def test_accept_full_size_vs_oracle(cuda_device, B, T, V, dtype):
    import d2sd_b200 as d
    g = torch.Generator().manual_seed(B * 100 + T)
    for trial in range(3):
        z = torch.randn(B, T, V, generator=g).to(dtype)
        amax = z.float().argmax(-1)
        x = torch.randint(0, V, (B, T), generator=g)
        x[:, 0] = x[0, 0]
        keep = torch.rand(B, T, generator=g) < (0.7 + 0.15 * trial)
        x[:, 1:] = torch.where(keep[:, 1:], amax[:, :-1], x[:, 1:])
        acc, ids, branch = d.verify(z.to(cuda_device), x.to(cuda_device))
        racc, rids, rbranch = OA.verify_accept(z.float(), x)
        assert (acc, branch) == (racc, rbranch)
        np.testing.assert_array_equal(ids.cpu().numpy(), rids)
        if B == 1:
            dacc, dids, _ = OA.dflash_accept(z.float(), x)
            assert acc == dacc
            np.testing.assert_array_equal(ids.cpu().numpy(), dids)


def test_accept_strided_logits_and_repeat(cuda_device):
    """A non-contiguous branch/position layout and back-to-back launches on the
    same workspace (the ticket must reset)."""
    import d2sd_b200 as d
    from d2sd_b200 import ops
    g = torch.Generator().manual_seed(7)
    B, T, V = 4, 8, 4096
    big = torch.randn(T, B, V, generator=g).to(torch.bfloat16).to(cuda_device)
    z = big.transpose(0, 1)  # [B, T, V] with branch stride V, position stride B*V
    x = torch.randint(0, V, (B, T), generator=g).to(cuda_device)
    ver = d.Verifier(B, T, V, cuda_device)
    for _ in range(5):
        ops.verify_accept(z, x, ver.result, ver.accepted, ver.workspace, ver.argmax)
    acc, ids, branch = ver.read()
    racc, rids, rbranch = OA.verify_accept(z.float().cpu(), x.cpu())
    assert (acc, branch) == (racc, rbranch)
    np.testing.assert_array_equal(ids.cpu().numpy(), rids)


def test_commit_golden_paged(cuda_device):
    import d2sd_b200 as d
    for i, c in enumerate(load_cases("commit_cases.npz")):
        L = int(c["L"])
        cache_k, cache_v = c["cache_k"], c["cache_v"]  # [L, 1, Hk, P, D]
        _, _, Hk, P, D = cache_k.shape
        B, T = c["new_k"].shape[1], c["new_k"].shape[3]
        npages = -(-(P + T) // 16) + 2
        g = torch.Generator().manual_seed(i)
        cache = d.PagedKVCache(L, Hk, D, npages * 16, dtype=torch.float32, device=cuda_device,
                               page_order=torch.randperm(npages, generator=g), layout="hnd")
        for l in range(L):
            cache.write(l, torch.from_numpy(cache_k[l, 0]).transpose(0, 1).to(cuda_device),
                        torch.from_numpy(cache_v[l, 0]).transpose(0, 1).to(cuda_device))
        cache.length = P
        new_k = torch.from_numpy(c["new_k"]).to(cuda_device)
        new_v = torch.from_numpy(c["new_v"]).to(cuda_device)
        res = torch.tensor([int(c["acc"]), int(c["branch"])], dtype=torch.int32,
                           device=cuda_device)
        cache.commit(new_k, new_v, res, advance_by=int(c["acc"]))
        torch.cuda.synchronize()
        for l in range(L):
            gk, gv = cache.gather(l)
            np.testing.assert_array_equal(gk.transpose(0, 1).cpu().numpy(), c["out_k"][l, 0])
            np.testing.assert_array_equal(gv.transpose(0, 1).cpu().numpy(), c["out_v"][l, 0])


@pytest.mark.parametrize("layout", ["umma", "hnd"])
def test_verify_then_commit_device_chain(cuda_device, layout):
    """Acceptance result consumed on the device by the commit (no host sync in
    between), all layers in one launch, bf16, strided [B, T, Hk, D] new K/V."""
    import d2sd_b200 as d
    g = torch.Generator().manual_seed(4)
    L, B, T, Hk, D, V, P = 36, 8, 32, 8, 128, 151936, 1000
    cache = d.PagedKVCache(L, Hk, D, P + T + 16, device=cuda_device, layout=layout,
                           page_order=torch.randperm(-(-(P + T + 16) // 16), generator=g))
    base_k = [torch.randn(P, Hk, D, generator=g).to(torch.bfloat16) for _ in range(L)]
    for l in range(L):
        cache.write(l, base_k[l].to(cuda_device), base_k[l].to(cuda_device))
    cache.length = P
    # new K/V produced as [L, B, T, Hk, D] and viewed as [L, B, Hk, T, D]
    nk = torch.randn(L, B, T, Hk, D, generator=g).to(torch.bfloat16).to(cuda_device).transpose(2, 3)
    nv = torch.randn(L, B, T, Hk, D, generator=g).to(torch.bfloat16).to(cuda_device).transpose(2, 3)
    z = torch.randn(B, T, V, generator=g).to(torch.bfloat16)
    x = torch.randint(0, V, (B, T), generator=g)
    x[:, 1:] = torch.where(torch.rand(B, T - 1, generator=g) < 0.8, z.float().argmax(-1)[:, :-1],
                           x[:, 1:])
    ver = d.Verifier(B, T, V, cuda_device)
    ver.launch(z.to(cuda_device), x.to(cuda_device))
    cache.commit(nk, nv, ver.result)
    acc, ids, branch = ver.read()
    racc, _, rbranch = OA.verify_accept(z.float(), x)
    assert (acc, branch) == (racc, rbranch)
    cache.length = P + acc
    for l in (0, 17, 35):
        gk, gv = cache.gather(l)
        ok, ov = OC.commit_contiguous([base_k[l].transpose(0, 1)[None].float().numpy()],
                                      [base_k[l].transpose(0, 1)[None].float().numpy()],
                                      [(nk[l].float().cpu().numpy(), nv[l].float().cpu().numpy())],
                                      branch, acc)
        np.testing.assert_array_equal(gk.float().transpose(0, 1).cpu().numpy(), ok[0][0])
        np.testing.assert_array_equal(gv.float().transpose(0, 1).cpu().numpy(), ov[0][0])


def test_commit_with_context_feature_golden(cuda_device):
    """The context-feature gather fused into the commit launch against the
    reference's extract_context_feature(...)[valid_block, :acceptance_length]
    (generation/d3_generator.py:239), fp32 hidden states, bit for bit; the KV
    commit of the same launch is checked against the oracle."""
    import d2sd_b200 as d
    g = torch.Generator().manual_seed(12)
    for c in load_cases("hidden_cases.npz"):
        hidden = torch.from_numpy(c["hidden"])  # [L + 2, B, T, H]
        ids = [int(i) for i in c["layer_ids"]]
        branch, acc = int(c["branch"]), int(c["acc"])
        _, B, T, H = hidden.shape
        Hk, D, P = 2, 16, 40
        cache = d.PagedKVCache(1, Hk, D, P + T + 16, dtype=torch.float32, device=cuda_device,
                               layout="hnd")
        base = torch.randn(P, Hk, D, generator=g)
        cache.write(0, base.to(cuda_device), base.to(cuda_device))
        cache.length = P
        nk = torch.randn(1, B, Hk, T, D, generator=g)
        src = [hidden[i + 1].to(cuda_device) for i in ids]
        out = torch.full((T, len(ids) * H), -7.0, device=cuda_device)
        res = torch.tensor([acc, branch], dtype=torch.int32, device=cuda_device)
        cache.commit(nk.to(cuda_device), nk.to(cuda_device), res, advance_by=acc,
                     target_hidden=(src, out))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out[:acc].cpu().numpy(), c["out"][0])
        assert bool((out[acc:] == -7.0).all())
        gk, gv = cache.gather(0)
        ok, _ = OC.commit_contiguous([base.transpose(0, 1)[None].numpy()],
                                     [base.transpose(0, 1)[None].numpy()],
                                     [(nk[0].numpy(), nk[0].numpy())], branch, acc)
        np.testing.assert_array_equal(gk.transpose(0, 1).cpu().numpy(), ok[0][0])


def test_verify_commit_context_feature_chain(cuda_device):
    """bf16 hidden states [B, T, H] at Qwen3-8B width (H 4096) and three draft
    layers, acc and branch read on the device from kernel (c)."""
    import d2sd_b200 as d
    g = torch.Generator().manual_seed(13)
    L, B, T, Hk, D, V, P, H = 2, 8, 16, 8, 128, 4096, 256, 4096
    cache = d.PagedKVCache(L, Hk, D, P + T + 16, device=cuda_device)
    cache.length = P
    nk = torch.randn(L, B, Hk, T, D, generator=g).to(torch.bfloat16).to(cuda_device)
    z = torch.randn(B, T, V, generator=g).to(torch.bfloat16)
    x = torch.randint(0, V, (B, T), generator=g)
    x[:, 1:] = torch.where(torch.rand(B, T - 1, generator=g) < 0.8, z.float().argmax(-1)[:, :-1],
                           x[:, 1:])
    hs = [torch.randn(B, T, H, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(5)]
    ids = [0, 2, 3]
    out = torch.zeros(T, len(ids) * H, dtype=torch.bfloat16, device=cuda_device)
    ver = d.Verifier(B, T, V, cuda_device)
    ver.launch(z.to(cuda_device), x.to(cuda_device))
    cache.commit(nk, nk, ver.result, target_hidden=([hs[i + 1] for i in ids], out))
    acc, _, branch = ver.read()
    ref = OC.context_feature([h.float().cpu().numpy() for h in hs], ids, branch, acc)
    np.testing.assert_array_equal(out[:acc].float().cpu().numpy(), ref)
