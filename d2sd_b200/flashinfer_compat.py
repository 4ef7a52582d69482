"""FlashInfer-signature replacements for the two calls D2-SD makes.

``single_prefill_with_kv_cache`` and ``merge_state_in_place`` keep FlashInfer's
argument meaning and conventions (NHD tensors, GQA by head grouping, base-2
LSE, bottom-right causal alignment), so the call sites of
generation/verification.py:145-165, model/cascade_graph.py:54-60 and
model/dflash.py:112-133 can switch by changing the import. They route to the
two kernels of this package by shape:
  * the level-2 case (q and kv of one block, q_len == kv_len <= 64) runs kernel
    (b) with a causal or full mask;
  * the level-1 case (causal=False, any prefix length) runs kernel (a) over a
    persistent grid and kernel (b) to finalise the partial states.
A causal call with q_len != kv_len or a block longer than 64 tokens is not part
of D2-SD's path and raises NotImplementedError.
"""
from __future__ import annotations

import torch

from . import _lib, ops
from .cascade import CascadePlan, Request

_plans: dict = {}


def _plan_for(n: int, p: int, hq: int, hk: int, d: int, device) -> CascadePlan:
    key = (n, p, hq, hk, d, str(device))
    plan = _plans.get(key)
    if plan is None:
        if len(_plans) > 64:
            _plans.clear()
        plan = CascadePlan([Request(n, 0, 0, p)], hq, hk, d, device)
        _plans[key] = plan
    return plan


def single_prefill_with_kv_cache(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                 causal: bool = False, kv_layout: str = "NHD",
                                 sm_scale: float | None = None, return_lse: bool = False,
                                 **unused):
    """q [qo_len, Hq, D]; k, v [kv_len, Hk, D] (NHD) or [Hk, kv_len, D] (HND).
    Returns out [qo_len, Hq, D] (q's dtype), plus lse [qo_len, Hq] fp32 base 2
    when ``return_lse``."""
    layout = kv_layout.lower()
    if layout not in ("nhd", "hnd"):
        raise ValueError("kv_layout must be NHD or HND")
    N, Hq, D = q.shape
    if layout == "nhd":
        P, Hk = k.shape[0], k.shape[1]
    else:
        Hk, P = k.shape[0], k.shape[1]
    scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    out = torch.empty(N, Hq, D, dtype=q.dtype, device=q.device)
    lse = torch.empty(N, Hq, dtype=torch.float32, device=q.device)
    kk = k if layout == "nhd" else k.transpose(0, 1)
    vv = v if layout == "nhd" else v.transpose(0, 1)
    if q.dtype == torch.float32:  # fp32 end to end (d2sd_cascade_attention_f32)
        if N == P and N <= 64:
            ops.cascade_attention_f32(q, out, lse, num_blocks=1, block_len=N, num_kv_heads=Hk,
                                      sm_scale=scale, k_local=kk, v_local=vv,
                                      mask_mode=_lib.MASK_CAUSAL if causal else _lib.MASK_NONE)
        elif not causal:
            ops.cascade_attention_f32(q, out, lse, num_blocks=1, block_len=N, num_kv_heads=Hk,
                                      sm_scale=scale, k_prefix=kk if P else None,
                                      v_prefix=vv if P else None)
        else:
            raise NotImplementedError("causal prefill with qo_len != kv_len is outside D2-SD's path")
        return (out, lse) if return_lse else out
    if N == P and N <= 64:
        ops.suffix_merge(q, kk, vv, out, lse, num_blocks=1, block_len=N, num_qo_heads=Hq,
                         num_kv_heads=Hk, sm_scale=scale,
                         mask_mode=_lib.MASK_CAUSAL if causal else _lib.MASK_NONE)
    elif not causal:
        plan = _plan_for(N, P, Hq, Hk, D, q.device)
        plan.run_prefix(q, k, v, layout, scale)
        plan.finalize(out, lse, scale)
    else:
        raise NotImplementedError("causal prefill with qo_len != kv_len is outside D2-SD's path")
    return (out, lse) if return_lse else out


def merge_state_in_place(v: torch.Tensor, s: torch.Tensor, v_other: torch.Tensor,
                         s_other: torch.Tensor, mask=None) -> None:
    """(v, s) <- merge((v, s), (v_other, s_other)); v [n, H, D], s [n, H] fp32."""
    if mask is not None:
        raise NotImplementedError("merge_state_in_place: mask is not used by D2-SD")
    ops.merge_state(v, s, v_other, s_other)
