"""CPU restatement of the verify attention (TEST INFRASTRUCTURE ONLY).

float64 numpy, FlashInfer conventions: q [N, Hq, D] / k, v [P, Hk, D] (NHD),
query head h reads kv head h // G, and the returned log-sum-exp is base 2,
lse = log2(sum_j 2^(s_j * sm_scale * log2(e))), the value FlashInfer's
single_prefill_with_kv_cache(return_lse=True) returns (flashinfer
include/flashinfer/attention/state.cuh:45, prefill.cuh:1855-1858: m + log2(d)
with m in scale*log2e units).
"""
from __future__ import annotations

import math

import numpy as np

LOG2E = 1.0 / math.log(2.0)


def _to64(x) -> np.ndarray:
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().float().cpu().numpy()
    return np.asarray(x, dtype=np.float64)


def single_prefill(q, k, v, causal: bool = False, sm_scale: float | None = None,
                   kv_start: int = 0):
    """flashinfer.single_prefill_with_kv_cache(q, k, v, causal, return_lse=True, sm_scale).

    Call sites: generation/verification.py:145-148 (causal=False, the shared
    prefix) and model/cascade_graph.py:54-57 (causal per runner, one branch).
    causal follows FlashInfer's bottom-right alignment: query i of N sees keys
    j <= i + (P - N). Keys before kv_start are invisible (a sliding window).
    Returns (out [N, Hq, D] float64, lse [N, Hq] float64 base 2); a row with no
    visible key gets out = 0 and lse = -inf.
    Computed one kv head (its G query heads) and one block of query rows at a
    time with float64 matrix products on the CPU (torch, multi-threaded), so
    that long prefixes (32768 keys) fit and finish in seconds.
    """
    q, k, v = _to64(q), _to64(k), _to64(v)
    N, Hq, D = q.shape
    P, Hk, _ = k.shape
    G = Hq // Hk
    scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    out = np.zeros((N, Hq, D))
    lse = np.full((N, Hq), -np.inf)
    if P == 0 or N == 0:
        return out, lse
    import torch
    rows = max(1, (1 << 22) // max(P, 1))  # query tokens per block (~32 MB of scores per head)
    keys = torch.arange(P)
    qt, kt, vt = (torch.from_numpy(np.ascontiguousarray(a)) for a in (q, k, v))
    for h in range(Hk):
        kh, vh = kt[:, h, :], vt[:, h, :]
        for n0 in range(0, N, rows):
            n1 = min(N, n0 + rows)
            qb = qt[n0:n1, h * G:(h + 1) * G, :].reshape(-1, D)  # [n*G, D]
            s = (qb @ kh.T).view(n1 - n0, G, P) * scale
            visible = torch.ones(n1 - n0, P, dtype=torch.bool)
            if causal:
                visible &= keys[None, :] <= (torch.arange(n0, n1)[:, None] + (P - N))
            if kv_start > 0:
                visible &= keys[None, :] >= kv_start
            s = s.masked_fill(~visible[:, None, :], -math.inf)
            m = s.amax(dim=-1, keepdim=True)
            has = torch.isfinite(m)
            m_safe = torch.where(has, m, torch.zeros_like(m))
            p = torch.exp(s - m_safe)
            l = p.sum(dim=-1, keepdim=True)
            o = (p.view(-1, P) @ vh).view(n1 - n0, G, D) / torch.where(l > 0, l, torch.ones_like(l))
            out[n0:n1, h * G:(h + 1) * G] = o.numpy()
            lse_b = torch.where(has[..., 0],
                                (m_safe[..., 0] + torch.log(torch.where(l[..., 0] > 0, l[..., 0],
                                                                        torch.ones_like(l[..., 0]))))
                                * LOG2E, torch.full_like(l[..., 0], -math.inf))
            lse[n0:n1, h * G:(h + 1) * G] = lse_b.numpy()
    return out, lse


def merge_state(v, s, v_other, s_other):
    """flashinfer.merge_state_in_place(v, s, v_other, s_other) (base-2 states).

    Call sites: model/cascade_graph.py:58-60, generation/verification.py:163-165.
    Returns the merged (v, s); FlashInfer's formula: with M = max(s, s_o),
    a = 2^(s-M), b = 2^(s_o-M): v = (a v + b v_o)/(a+b), s = M + log2(a+b).
    """
    v, s, vo, so = _to64(v), _to64(s), _to64(v_other), _to64(s_other)
    M = np.maximum(s, so)
    Mz = np.where(np.isfinite(M), M, 0.0)
    a = np.where(np.isfinite(s), np.exp2(s - Mz), 0.0)
    b = np.where(np.isfinite(so), np.exp2(so - Mz), 0.0)
    den = a + b
    safe = np.where(den > 0, den, 1.0)
    out_v = (a[..., None] * v + b[..., None] * vo) / safe[..., None]
    out_s = np.where(den > 0, Mz + np.log2(safe), -np.inf)
    return out_v, out_s


def _round(x, dtype):
    if dtype is None:
        return x
    import torch
    return torch.from_numpy(np.asarray(x, dtype=np.float32)).to(dtype).double().numpy()


def runner_local_merge(q_local, k_local, v_local, out_shared, lse_shared, causal: bool,
                       sm_scale: float, round_dtype=None):
    """CascadeGraphRunner.run (model/cascade_graph.py:52-60,76-112).

    For each branch i: out_l, lse_l = single_prefill(q[i], k[i], v[i], causal);
    merge_state_in_place(out_shared[i], lse_shared[i], out_l, lse_l).
    q_local [B, T, Hq, D], k/v_local [B, T, Hk, D], out_shared [B, T, Hq, D],
    lse_shared [B, T, Hq]. round_dtype (a torch dtype) rounds the FlashInfer
    outputs (out_l and the merged v) the way the reference's bf16 kernels do.
    """
    q_local = _to64(q_local)
    out = _to64(out_shared).copy()
    lse = _to64(lse_shared).copy()
    for i in range(q_local.shape[0]):
        o_l, s_l = single_prefill(q_local[i], k_local[i], v_local[i], causal=causal,
                                  sm_scale=sm_scale)
        o_l = _round(o_l, round_dtype)
        mv, ms = merge_state(out[i], lse[i], o_l, s_l)
        out[i] = _round(mv, round_dtype)
        lse[i] = ms
    return out, lse


def cascade_attention(q, k_new, v_new, k_prefix, v_prefix, causal: bool = True,
                      sm_scale: float | None = None, sliding_window: int | None = None,
                      sinks=None, sink_mode: str = "reference", round_dtype=None):
    """The attention of one layer of cascade_verify_forward.

    generation/verification.py:127-176: the shared prefix is truncated to its
    last sliding_window keys when longer (:130-135); level 1 attends every
    query token of every branch to the prefix with causal=False (:139-150);
    level 2 runs the per-branch local attention and merges (:152-165); GPT-OSS
    sinks rescale out by sigmoid(lse - sink) with the base-2 merged lse
    (:173-176, sink_mode="reference") or by the HF softmax-with-sink factor
    sigmoid(lse*ln2 - sink) (sink_mode="exact").
    q [B, T, Hq, D], k_new/v_new [B, T, Hk, D] (the block tokens' own K/V),
    k_prefix/v_prefix [P, Hk, D]. Returns (out [B, T, Hq, D], lse [B, T, Hq]).
    """
    q = _to64(q)
    B, T, Hq, D = q.shape
    kp, vp = _to64(k_prefix), _to64(v_prefix)
    if sliding_window is not None and kp.shape[0] > sliding_window:
        kp, vp = kp[-sliding_window:], vp[-sliding_window:]
    scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    if kp.shape[0] > 0:
        o_s, l_s = single_prefill(q.reshape(B * T, Hq, D), kp, vp, causal=False, sm_scale=scale)
    else:
        o_s, l_s = np.zeros((B * T, Hq, D)), np.full((B * T, Hq), -np.inf)
    o_s = _round(o_s, round_dtype).reshape(B, T, Hq, D)
    l_s = l_s.reshape(B, T, Hq)
    out, lse = runner_local_merge(q, _to64(k_new), _to64(v_new), o_s, l_s, causal, scale,
                                  round_dtype)
    if sinks is not None:
        sk = _to64(sinks).reshape(1, 1, Hq)
        x = lse * math.log(2.0) - sk if sink_mode == "exact" else lse - sk
        out = out * (1.0 / (1.0 + np.exp(-x)))[..., None]
    return out, lse


def torch_masked_sdpa(q, k_new, v_new, k_prefix, v_prefix, causal: bool = True,
                      sm_scale: float | None = None, kv_start: int = 0, threads: int | None = None):
    """The reference's torch.sdpa masked path on the CPU (the timed CPU baseline).

    Per branch b, the queries q[b] [T, Hq, D] attend cat(prefix, k_new[b]) with a
    [T, P+T] boolean mask (prefix visible from kv_start on, causal within the
    branch) -- what HF sdpa computes for the plain verify forward of
    generation/verification.py:204-220 -- and the base-2 LSE is
    torch.logsumexp of the masked scores times log2(e).
    Inputs are torch CPU tensors; returns (out [B, T, Hq, D], lse [B, T, Hq]).
    """
    import torch
    import torch.nn.functional as F
    if threads:
        torch.set_num_threads(threads)
    B, T, Hq, D = q.shape
    P, Hk = k_prefix.shape[0], k_prefix.shape[1]
    scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    mask = torch.ones(T, P + T, dtype=torch.bool)
    if kv_start:
        mask[:, :kv_start] = False
    if causal:
        mask[:, P:] = torch.ones(T, T, dtype=torch.bool).tril()
    outs, lses = [], []
    for b in range(B):
        kk = torch.cat([k_prefix, k_new[b]], 0).transpose(0, 1).unsqueeze(0)  # [1,Hk,P+T,D]
        vv = torch.cat([v_prefix, v_new[b]], 0).transpose(0, 1).unsqueeze(0)
        qq = q[b].transpose(0, 1).unsqueeze(0)  # [1,Hq,T,D]
        o = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=scale,
                                           enable_gqa=True)
        kr = kk.repeat_interleave(Hq // Hk, dim=1)
        sc = (qq @ kr.transpose(-1, -2)) * scale
        sc = sc.masked_fill(~mask, float("-inf"))
        lse = torch.logsumexp(sc, dim=-1) * LOG2E  # [1,Hq,T]
        outs.append(o[0].transpose(0, 1))
        lses.append(lse[0].transpose(0, 1))
    return torch.stack(outs), torch.stack(lses)


def torch_tree_sdpa(q, k_new, v_new, k_prefix, v_prefix, causal: bool = True,
                    sm_scale: float | None = None, kv_start: int = 0):
    """The torch.sdpa masked path for all branches in ONE call (the timed CPU
    baseline): the B*T block queries attend [prefix | all branches' block
    tokens] under a [B*T, P + B*T] boolean tree mask -- the prefix from
    kv_start on, and within the blocks only the query's own branch (causal:
    its tokens 0..t). Per branch this is what HF sdpa computes for the plain
    verify forward of generation/verification.py:204-220.
    Torch CPU tensors q [B, T, Hq, D], k/v_new [B, T, Hk, D], k/v_prefix
    [P, Hk, D]; returns out [B, T, Hq, D]."""
    import torch
    import torch.nn.functional as F
    B, T, Hq, D = q.shape
    P, Hk = k_prefix.shape[0], k_prefix.shape[1]
    scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    n = B * T
    mask = torch.zeros(n, P + n, dtype=torch.bool)
    mask[:, kv_start:P] = True
    blk = torch.arange(n) // T
    pos = torch.arange(n) % T
    same = blk[:, None] == blk[None, :]
    if causal:
        same &= pos[None, :] <= pos[:, None]
    mask[:, P:] = same
    kk = torch.cat([k_prefix, k_new.reshape(n, Hk, D)], 0).transpose(0, 1).unsqueeze(0)
    vv = torch.cat([v_prefix, v_new.reshape(n, Hk, D)], 0).transpose(0, 1).unsqueeze(0)
    qq = q.reshape(n, Hq, D).transpose(0, 1).unsqueeze(0)
    o = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=scale, enable_gqa=True)
    return o[0].transpose(0, 1).reshape(B, T, Hq, D)
