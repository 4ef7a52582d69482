"""``cascade_verify_forward`` on the d2sd kernels.

Same signature and results as generation/verification.py:49-201 of the
reference: a manual layer-by-layer forward of a HuggingFace Qwen3 or GPT-OSS
target over B candidate blocks that share one cached prefix. The projections,
norms, RoPE, MLP and lm_head stay PyTorch (cuBLAS); the attention of every
layer is one launch of kernel (a) over the cache in place -- the DynamicCache
layer [1, Hk, P, D] read as an HND tensor, so the reference's per-layer
transpose copy of the whole prefix (:139-140) is gone -- and one launch of
kernel (b) for the per-branch causal attention, the LSE merge and, for GPT-OSS,
the sink rescale (:152-176). The GPT-OSS sliding layers see the last
`sliding_window` prefix keys, as in the reference (:130-135).

``cascade_graph_runner`` is accepted for call compatibility; the fused kernel
(b) already does what the runner's graph did.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch

from .cascade import CascadePlan, Request, cascade_attention


def _rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def _rope_qwen3(q, k, cos, sin):
    """cos/sin [bsz, seq, head_dim] with duplicated halves (verification.py:21-28)."""
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


def _rope_gpt_oss(q, k, cos, sin):
    """cos/sin [bsz, seq, head_dim/2] applied to the two halves (verification.py:31-42)."""
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)

    def ap(x):
        a, b = torch.chunk(x, 2, dim=-1)
        return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)

    return ap(q), ap(k)


def _layer_kv(past_key_values, idx):
    layer = past_key_values.layers[idx]
    return layer.keys, layer.values


@torch.no_grad()
def cascade_verify_forward(target_model, input_ids: torch.Tensor, position_ids: torch.Tensor,
                           past_key_values, output_hidden_states: bool = True,
                           cascade_graph_runner=None):
    """Returns (logits [bsz, block, vocab], hidden states (L+2 entries) or None,
    new_kv_list [(k_new, v_new) per layer, each [bsz, Hk, block, D]])."""
    model = target_model.model
    bsz, seq_len = input_ids.shape
    is_gpt_oss = type(model.layers[0].self_attn).__name__ == "GptOssAttention"
    rope = _rope_gpt_oss if is_gpt_oss else _rope_qwen3

    hidden = model.embed_tokens(input_ids)
    cos, sin = model.rotary_emb(hidden, position_ids)
    all_hidden = [hidden] if output_hidden_states else None
    new_kv_list = []
    plans: dict = {}

    for layer_idx, layer in enumerate(model.layers):
        residual = hidden
        h = layer.input_layernorm(hidden)
        attn = layer.self_attn
        Hq = attn.config.num_attention_heads
        Hk = attn.config.num_key_value_heads
        D = attn.head_dim
        q = attn.q_proj(h).view(bsz, seq_len, Hq, D)
        k_new = attn.k_proj(h).view(bsz, seq_len, Hk, D)
        v_new = attn.v_proj(h).view(bsz, seq_len, Hk, D)
        if not is_gpt_oss:
            q = attn.q_norm(q)
            k_new = attn.k_norm(k_new)
        q, k_new = rope(q.transpose(1, 2), k_new.transpose(1, 2), cos, sin)
        v_new = v_new.transpose(1, 2)
        new_kv_list.append((k_new, v_new))

        keys, values = _layer_kv(past_key_values, layer_idx)  # [1, Hk, P, D]
        P = keys.shape[2]
        window = getattr(attn, "sliding_window", None)
        kv_start = P - window if (window is not None and P > window) else 0
        key = (P, kv_start, Hq, Hk, D)
        plan = plans.get(key)
        if plan is None:
            plan = CascadePlan([Request(bsz * seq_len, 0, kv_start, P)], Hq, Hk, D, q.device)
            plans[key] = plan
        sinks = attn.sinks.float() if is_gpt_oss else None
        out, _ = cascade_attention(q.transpose(1, 2), k_new.transpose(1, 2),
                                   v_new.transpose(1, 2), keys[0], values[0], "hnd", P,
                                   causal=True, sm_scale=D ** -0.5,
                                   sliding_window=None if kv_start == 0 else P - kv_start,
                                   sinks=sinks, sink_mode="reference", plan=plan)
        hidden = residual + attn.o_proj(out.reshape(bsz, seq_len, -1))

        residual = hidden
        mlp_out = layer.mlp(layer.post_attention_layernorm(hidden))
        if isinstance(mlp_out, tuple):
            mlp_out = mlp_out[0]
        hidden = residual + mlp_out
        if output_hidden_states:
            all_hidden.append(hidden)

    hidden = model.norm(hidden)
    if output_hidden_states:
        all_hidden.append(hidden)
    logits = target_model.lm_head(hidden)
    return logits, all_hidden, new_kv_list


def plain_verify_forward(target_model, input_ids, position_ids, past_key_values,
                         output_hidden_states: bool = True):
    """The reference's single-branch path (verification.py:204-220), unchanged:
    the HF forward. Kept so callers can import both from one place."""
    output = target_model(input_ids, position_ids=position_ids, past_key_values=past_key_values,
                          use_cache=True, output_hidden_states=output_hidden_states)
    return SimpleNamespace(logits=output.logits, hidden_states=output.hidden_states)
