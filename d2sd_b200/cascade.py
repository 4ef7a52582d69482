"""Two-level cascade verify attention: plan once, run per layer.

The reference runs, per layer (generation/verification.py:127-176):
  1. a transpose copy of the whole prefix KV to NHD (:139-140),
  2. flashinfer.single_prefill_with_kv_cache over the prefix for all B*T
     query tokens (:145-148),
  3. per branch a causal single_prefill over the block + merge_state_in_place
     (:152-165, or the CascadeGraphRunner graph, model/cascade_graph.py:52-60),
  4. the GPT-OSS sink rescale (:173-176).
Here step 1 disappears (kernel (a) reads the cache in place: a DynamicCache
layer, a contiguous NHD prefix or a paged pool), step 2 is kernel (a) over a
persistent grid, and steps 3-4 are one launch of kernel (b).

``CascadePlan`` is the host-side plan (the shapes, prefix lengths and the
work partition) plus its device copy and workspace; it is rebuilt only when the
request shapes or prefix lengths change, like FlashInfer's plan/run split.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, ops


@dataclass
class Request:
    q_tokens: int        # query tokens attending this request's prefix
    q_token_offset: int  # first row of those tokens in the Q tensor
    kv_start: int        # first visible prefix position (sliding window), usually 0
    kv_end: int          # prefix length
    page_offset: int = 0  # offset into the page table (paged) or token offset (contiguous)


class CascadePlan:
    """Plan + device state of kernel (a) for one batch of requests."""

    def __init__(self, requests: list[Request], num_qo_heads: int, num_kv_heads: int,
                 head_dim: int, device: torch.device | str, num_ctas: int | None = None):
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("CascadePlan needs a CUDA device")
        self.device = device
        self.requests = list(requests)
        self.num_qo_heads, self.num_kv_heads, self.head_dim = num_qo_heads, num_kv_heads, head_dim
        sms = num_ctas or ops.num_sms(device)
        plan, nslots = ops.prefix_plan([r.q_tokens for r in requests],
                                       [r.q_token_offset for r in requests],
                                       [r.kv_start for r in requests],
                                       [r.kv_end for r in requests], num_qo_heads, num_kv_heads,
                                       sms)
        self.host_plan = plan
        self.num_ctas = int(plan[1])
        self.num_slots = nslots
        self.plan = torch.from_numpy(plan).to(device)
        slot_bytes = ops.partial_slot_bytes(head_dim)
        self.partial = torch.empty(max(1, nslots) * slot_bytes // 4, dtype=torch.float32,
                                   device=device)
        self.page_offsets = torch.tensor([r.page_offset for r in requests], dtype=torch.int32,
                                         device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)

    def key(self):
        return tuple((r.q_tokens, r.q_token_offset, r.kv_start, r.kv_end, r.page_offset)
                     for r in self.requests)

    def run_prefix(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_layout: str,
                   sm_scale: float, page_table: torch.Tensor | None = None) -> None:
        """Kernel (a): every planned query row against its request's prefix."""
        if self.num_ctas == 0:
            return
        ops.prefix_attention(q, k, v, kv_layout, self.plan, self.num_ctas, self.partial, sm_scale,
                             page_table=page_table, page_table_offset=self.page_offsets,
                             status=self.status)

    def finalize(self, out: torch.Tensor, lse: torch.Tensor | None, sm_scale: float) -> None:
        """Prefix-only result (no level 2): merge the partial slots into out [N, Hq, D]
        and lse [N, Hq] for the N planned query tokens."""
        ops.suffix_merge(None, None, None, out, lse, num_blocks=out.shape[0], block_len=1,
                         num_qo_heads=self.num_qo_heads, num_kv_heads=self.num_kv_heads,
                         sm_scale=sm_scale, mask_mode=_lib.MASK_NONE,
                         partial=self.partial if self.num_ctas else None,
                         plan_dev=self.plan)


_MASKS = {"none": _lib.MASK_NONE, "causal": _lib.MASK_CAUSAL, "custom": _lib.MASK_CUSTOM}
_SINKS = {"reference": _lib.SINK_REFERENCE, "exact": _lib.SINK_EXACT}


def shared_trunk_map(num_branches: int, block_len: int, shared: int, device) -> torch.Tensor:
    """Block token (b, t) -> row of the de-duplicated query list when every
    branch shares its first `shared` tokens (a tree whose trunk is common)."""
    b = torch.arange(num_branches).view(-1, 1)
    t = torch.arange(block_len).view(1, -1)
    idx = torch.where(t < shared, t, shared + b * (block_len - shared) + (t - shared))
    return idx.reshape(-1).to(torch.int32).to(device)


def cascade_attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                      k_cache: torch.Tensor, v_cache: torch.Tensor, kv_layout: str,
                      kv_len: int, *, causal: bool = True, sm_scale: float | None = None,
                      page_table: torch.Tensor | None = None, sliding_window: int | None = None,
                      sinks: torch.Tensor | None = None, sink_mode: str = "reference",
                      shared_tokens: int = 0, custom_mask: torch.Tensor | None = None,
                      plan: CascadePlan | None = None, out: torch.Tensor | None = None,
                      lse: torch.Tensor | None = None, status: torch.Tensor | None = None):
    """One layer of the cascade verify attention for one request.

    q [B, T, Hq, D] bf16 (the block tokens' queries), k_new/v_new [B, T, Hk, D]
    (their own K/V), the prefix K/V in ``k_cache``/``v_cache`` per ``kv_layout``
    (see ops.kv_view) holding ``kv_len`` positions. ``sliding_window`` keeps only
    the last window prefix keys (generation/verification.py:130-135);
    ``shared_tokens`` > 0 declares that all branches share their first tokens,
    so their prefix attention is computed once. fp32 q/k/v (a contiguous
    "nhd" or "hnd" prefix) take the fp32 kernel (d2sd_cascade_attention_f32). Returns (out [B, T, Hq, D],
    lse [B, T, Hq] base 2), written into ``out``/``lse`` when given. Kernel (a)
    reports a wait time-out in ``plan.status``, kernel (b) in ``status`` (an
    int32 device tensor, optional).
    """
    B, T, Hq, D = q.shape
    Hk = k_new.shape[2]
    scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    kv_start = max(0, kv_len - sliding_window) if sliding_window is not None else 0
    if q.dtype == torch.float32:
        return _cascade_f32(q, k_new, v_new, k_cache, v_cache, kv_layout, kv_len, kv_start,
                            causal, scale, sinks, sink_mode, custom_mask, out, lse)
    if shared_tokens:
        n_u = shared_tokens + B * (T - shared_tokens)
        q_pref = torch.cat([q[0, :shared_tokens], q[:, shared_tokens:].reshape(-1, Hq, D)], 0)
        ptok = shared_trunk_map(B, T, shared_tokens, q.device)
    else:
        n_u = B * T
        q_pref = q.reshape(B * T, Hq, D)
        ptok = None
    if plan is None:
        plan = CascadePlan([Request(n_u, 0, kv_start, kv_len)], Hq, Hk, D, q.device)
    plan.run_prefix(q_pref, k_cache, v_cache, kv_layout, scale, page_table=page_table)
    if out is None:
        out = torch.empty(B, T, Hq, D, dtype=q.dtype, device=q.device)
    if lse is None:
        lse = torch.empty(B, T, Hq, dtype=torch.float32, device=q.device)
    mode = _MASKS["custom" if custom_mask is not None else ("causal" if causal else "none")]
    ops.suffix_merge(q.reshape(B * T, Hq, D), k_new.reshape(B * T, Hk, D),
                     v_new.reshape(B * T, Hk, D), out.view(B * T, Hq, D), lse.view(B * T, Hq),
                     num_blocks=B, block_len=T, num_qo_heads=Hq, num_kv_heads=Hk, sm_scale=scale,
                     mask_mode=mode, custom_mask=custom_mask,
                     partial=plan.partial if plan.num_ctas else None, plan_dev=plan.plan,
                     prefix_token=ptok, sinks=sinks,
                     sink_mode=_SINKS[sink_mode] if sinks is not None else _lib.SINK_NONE,
                     status=status)
    return out, lse


def _cascade_f32(q, k_new, v_new, k_cache, v_cache, kv_layout, kv_len, kv_start, causal, scale,
                 sinks, sink_mode, custom_mask, out, lse):
    """The fp32 form of ``cascade_attention`` (one launch of the SIMT fp32
    kernel: prefix keys, the block's own keys and the sinks in fp32)."""
    B, T, Hq, D = q.shape
    Hk = k_new.shape[2]
    if kv_layout == "nhd":
        kp, vp = k_cache[:kv_len], v_cache[:kv_len]
    elif kv_layout == "hnd":
        kp, vp = k_cache[:, :kv_len].transpose(0, 1), v_cache[:, :kv_len].transpose(0, 1)
    else:
        raise NotImplementedError("the fp32 cascade reads a contiguous nhd/hnd prefix")
    if out is None:
        out = torch.empty(B, T, Hq, D, dtype=torch.float32, device=q.device)
    if lse is None:
        lse = torch.empty(B, T, Hq, dtype=torch.float32, device=q.device)
    mode = _MASKS["custom" if custom_mask is not None else ("causal" if causal else "none")]
    ops.cascade_attention_f32(
        q.reshape(B * T, Hq, D), out.view(B * T, Hq, D), lse.view(B * T, Hq), num_blocks=B,
        block_len=T, num_kv_heads=Hk, sm_scale=scale, k_prefix=kp if kv_len else None,
        v_prefix=vp if kv_len else None, kv_start=kv_start, k_local=k_new.reshape(B * T, Hk, D),
        v_local=v_new.reshape(B * T, Hk, D), mask_mode=mode, custom_mask=custom_mask, sinks=sinks,
        sink_mode=_SINKS[sink_mode] if sinks is not None else _lib.SINK_NONE)
    return out, lse
