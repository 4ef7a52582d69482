"""The CPU oracle against the golden vectors produced by running the reference
(tests/golden/make_golden.py). CPU only."""
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, decode_logits, load_cases
from oracle import accept as OA
from oracle import attention as AT
from oracle import commit as OC


def test_reference_pin_summary():
    pin = json.loads((GOLDEN / "reference_pin.json").read_text())
    # the reference's cascade path (with the oracle in FlashInfer's place) equals
    # its plain HF-sdpa path on the tiny Qwen3
    assert pin["qwen3"]["max_abs_logit_diff_cascade_vs_plain"] < 1e-4
    assert pin["accept_cases"] >= 100 and pin["commit_cases"] >= 5


def test_accept_oracle_matches_reference():
    cases = load_cases("accept_cases.npz")
    assert len(cases) >= 100
    for c in cases:
        logits = decode_logits(c).float()
        acc, ids, branch = OA.verify_accept(logits, c["block_ids"])
        assert acc == int(c["acc"])
        assert branch == int(c["branch"])
        np.testing.assert_array_equal(ids, c["ids"])
        # output_ids[start+1 : start+acc+1] = accepted ids (d3_generator.py:222)
        np.testing.assert_array_equal(c["output_ids"][4:4 + acc], ids)


def test_dflash_oracle_matches_reference():
    for c in load_cases("dflash_cases.npz"):
        acc, ids, _ = OA.dflash_accept(c["logits"], c["block_ids"])
        assert acc == int(c["acc"])
        # output_ids[start:start+a+1] = block[:a+1]; output_ids[start+a+1] = bonus
        np.testing.assert_array_equal(c["output_ids"][2 + 1:2 + acc + 1], ids)
        # the single-branch walk is the multi-branch walk with B = 1
        acc2, ids2, _ = OA.verify_accept(c["logits"], c["block_ids"])
        assert acc2 == acc
        np.testing.assert_array_equal(ids2, ids)


def test_commit_oracle_matches_reference():
    for c in load_cases("commit_cases.npz"):
        L = int(c["L"])
        ck = [c["cache_k"][l] for l in range(L)]
        cv = [c["cache_v"][l] for l in range(L)]
        new = [(c["new_k"][l], c["new_v"][l]) for l in range(L)]
        ok, ov = OC.commit_contiguous(ck, cv, new, int(c["branch"]), int(c["acc"]))
        for l in range(L):
            np.testing.assert_array_equal(ok[l], c["out_k"][l])
            np.testing.assert_array_equal(ov[l], c["out_v"][l])


def test_commit_paged_equals_contiguous():
    rng = np.random.default_rng(0)
    Hk, D, ps, B, T = 2, 8, 16, 3, 32
    for P in (0, 5, 16, 31):
        for acc in (1, 7, 32):
            n_pages = (P + T + ps - 1) // ps + 1
            table = rng.permutation(n_pages + 3)[:n_pages]
            pool_k = np.zeros((n_pages + 3, Hk, ps, D), np.float32)
            pool_v = np.zeros_like(pool_k)
            ck = rng.standard_normal((1, Hk, P, D)).astype(np.float32)
            cv = rng.standard_normal((1, Hk, P, D)).astype(np.float32)
            for p in range(P):
                pool_k[table[p // ps], :, p % ps] = ck[0, :, p]
                pool_v[table[p // ps], :, p % ps] = cv[0, :, p]
            nk = rng.standard_normal((B, Hk, T, D)).astype(np.float32)
            nv = rng.standard_normal((B, Hk, T, D)).astype(np.float32)
            OC.commit_paged(pool_k, pool_v, table, P, nk, nv, 1, acc)
            ok, ov = OC.commit_contiguous([ck], [cv], [(nk, nv)], 1, acc)
            for p in range(P + acc):
                np.testing.assert_array_equal(pool_k[table[p // ps], :, p % ps], ok[0][0, :, p])
                np.testing.assert_array_equal(pool_v[table[p // ps], :, p % ps], ov[0][0, :, p])


@pytest.mark.parametrize("kind", ["qwen3", "gptoss"])
def test_cascade_oracle_matches_reference_attention(kind):
    layers = load_cases(f"attention_{kind}.npz")
    for lay in layers:
        window = int(lay["window"])
        sinks = lay.get("sinks")
        out, _ = AT.cascade_attention(lay["q"], lay["k_new"], lay["v_new"], lay["k_prefix"],
                                      lay["v_prefix"], causal=True,
                                      sliding_window=None if window < 0 else window,
                                      sinks=sinks, sink_mode="reference")
        # golden = what the reference fed o_proj (fp32 model, fp32 rounding)
        np.testing.assert_allclose(out, lay["out"], atol=2e-5, rtol=1e-5)


def test_single_prefill_matches_torch_sdpa():
    g = torch.Generator().manual_seed(3)
    for (N, P, Hq, Hk, D, causal) in ((7, 33, 4, 2, 16, False), (9, 9, 8, 8, 32, True),
                                      (5, 12, 6, 2, 8, True)):
        q = torch.randn(N, Hq, D, generator=g, dtype=torch.float64)
        k = torch.randn(P, Hk, D, generator=g, dtype=torch.float64)
        v = torch.randn(P, Hk, D, generator=g, dtype=torch.float64)
        out, lse = AT.single_prefill(q, k, v, causal=causal, sm_scale=D ** -0.5)
        kk = k.repeat_interleave(Hq // Hk, 1).transpose(0, 1)
        vv = v.repeat_interleave(Hq // Hk, 1).transpose(0, 1)
        qq = q.transpose(0, 1)
        mask = torch.ones(N, P, dtype=torch.bool)
        if causal:
            mask = torch.arange(P)[None] <= torch.arange(N)[:, None] + (P - N)
        ref = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask)
        np.testing.assert_allclose(out, ref.transpose(0, 1).numpy(), atol=1e-6)
        sc = (qq @ kk.transpose(-1, -2)) * D ** -0.5
        ref_lse = torch.logsumexp(sc.masked_fill(~mask, float("-inf")), -1) / np.log(2)
        np.testing.assert_allclose(lse, ref_lse.T.numpy(), atol=1e-6)


def test_merge_state_is_exact_split():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((6, 4, 16))
    k = rng.standard_normal((40, 2, 16))
    v = rng.standard_normal((40, 2, 16))
    full, lf = AT.single_prefill(q, k, v)
    a, la = AT.single_prefill(q, k[:17], v[:17])
    b, lb = AT.single_prefill(q, k[17:], v[17:])
    m, lm = AT.merge_state(a, la, b, lb)
    np.testing.assert_allclose(m, full, atol=1e-12)
    np.testing.assert_allclose(lm, lf, atol=1e-12)


def test_torch_masked_sdpa_matches_cascade():
    g = torch.Generator().manual_seed(5)
    B, T, Hq, Hk, D, P = 3, 6, 4, 2, 16, 20
    q = torch.randn(B, T, Hq, D, generator=g)
    kn = torch.randn(B, T, Hk, D, generator=g)
    vn = torch.randn(B, T, Hk, D, generator=g)
    kp = torch.randn(P, Hk, D, generator=g)
    vp = torch.randn(P, Hk, D, generator=g)
    o1, l1 = AT.torch_masked_sdpa(q, kn, vn, kp, vp, causal=True)
    o2, l2 = AT.cascade_attention(q, kn, vn, kp, vp, causal=True)
    np.testing.assert_allclose(o1.numpy(), o2, atol=1e-5)
    np.testing.assert_allclose(l1.numpy(), l2, atol=1e-5)


def test_context_feature_oracle_matches_reference():
    cases = load_cases("hidden_cases.npz")
    assert len(cases) >= 10
    for c in cases:
        got = OC.context_feature(list(c["hidden"]), [int(i) for i in c["layer_ids"]],
                                 int(c["branch"]), int(c["acc"]))
        np.testing.assert_array_equal(got[None], c["out"])


def test_rope_oracle_matches_reference():
    import torch
    from oracle import rope as OR
    cases = load_cases("rope_cases.npz")
    assert len(cases) >= 3
    bf = lambda a: torch.from_numpy(a).view(torch.bfloat16)  # noqa: E731
    for c in cases:
        gpt = str(c["kind"]) == "gptoss"
        ch, sh = bf(c["cos_half"]), bf(c["sin_half"])
        cos = ch[None] if gpt else torch.cat([ch, ch], -1)[None]
        sin = sh[None] if gpt else torch.cat([sh, sh], -1)[None]
        qw = None if gpt else bf(c["q_weight"])
        kw = None if gpt else bf(c["k_weight"])
        q, k = OR.qk_norm_rope(bf(c["q"]), bf(c["k"]), cos, sin, qw, kw, 1e-6, gpt_oss=gpt)
        assert torch.equal(q.contiguous().view(torch.int16), torch.from_numpy(c["q_out"]))
        assert torch.equal(k.contiguous().view(torch.int16), torch.from_numpy(c["k_out"]))
