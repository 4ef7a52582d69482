"""CPU restatement of the QK-norm + RoPE step of the verify forward
(TEST INFRASTRUCTURE ONLY: used by tests/ and as the checker, never by the
product).

generation/verification.py:113-124: for Qwen3, q = attn.q_norm(q) and
k = attn.k_norm(k) (transformers' Qwen3RMSNorm: x.float() * rsqrt(mean(x^2) +
eps), cast back to the input dtype, times the weight); then
q, k = rope_apply(q, k, cos, sin) with _apply_rotary_pos_emb_qwen3 (:21-28,
q*cos + rotate_half(q)*sin with full-width tables) or, for GPT-OSS,
_apply_rotary_pos_emb_gpt_oss (:31-43, half-width tables, no norm). Restated
on torch CPU tensors of the data dtype so that every rounding of the eager
expressions is the same.
"""
from __future__ import annotations

import torch


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    return weight * h.to(dt)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def qk_norm_rope(q, k, cos, sin, q_weight=None, k_weight=None, eps: float = 1e-6,
                 gpt_oss: bool = False):
    """q [B, T, Hq, D], k [B, T, Hk, D] (the projections viewed per head);
    cos/sin [1, T, D] (Qwen3) or [1, T, D/2] (GPT-OSS). Returns q, k as
    [B, T, H, D] (the reference transposes to [B, H, T, D] before RoPE; the
    values are the same)."""
    if q_weight is not None:
        q = rms_norm(q, q_weight, eps)
        k = rms_norm(k, k_weight, eps)
    q = q.transpose(1, 2)
    k = k.transpose(1, 2)
    c = cos.unsqueeze(1)
    s = sin.unsqueeze(1)
    if gpt_oss:
        def _apply(x):
            first, second = torch.chunk(x, 2, dim=-1)
            return torch.cat([first * c - second * s, second * c + first * s], dim=-1)
        q, k = _apply(q), _apply(k)
    else:
        q = (q * c) + (rotate_half(q) * s)
        k = (k * c) + (rotate_half(k) * s)
    return q.transpose(1, 2), k.transpose(1, 2)
