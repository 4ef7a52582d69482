"""``cascade_verify_forward`` on the d2sd kernels.

Same signature and results as generation/verification.py:49-201 of the
reference: a manual layer-by-layer forward of a HuggingFace Qwen3 or GPT-OSS
target over B candidate blocks that share one cached prefix. The projections,
MLP and lm_head stay PyTorch (cuBLAS); the QK-norm and RoPE of each layer's
block q and k are one launch of d2sd_qk_norm_rope (:113-124); the attention of
every layer is one launch of kernel (a) over the cache in place -- the DynamicCache
layer [1, Hk, P, D] read as an HND tensor, so the reference's per-layer
transpose copy of the whole prefix (:139-140) is gone -- and one launch of
kernel (b) for the per-branch causal attention, the LSE merge and, for GPT-OSS,
the sink rescale (:152-176). The GPT-OSS sliding layers see the last
`sliding_window` prefix keys, as in the reference (:130-135).

``past_key_values`` is the reference's DynamicCache or a ``PagedKVCache``
holding the same prefix (its ``length`` positions of every layer); with the
paged cache the whole D3 step -- this forward, ``verify`` and
``PagedKVCache.commit`` -- runs without the reference's per-step
reallocation of the cache.

``cascade_graph_runner`` is accepted for call compatibility; the fused kernel
(b) already does what the runner's graph did.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch

from . import ops
from .cascade import CascadePlan, Request, cascade_attention
from .kv_cache import PagedKVCache


def _prefix(past_key_values, idx):
    """(k, v, kv_layout, prefix length, page table) of layer idx. A
    ``PagedKVCache`` is read through its page table (the D3 loop then commits
    the accepted rows with ``PagedKVCache.commit`` instead of the reference's
    torch.cat, generation/d3_generator.py:227-232); a DynamicCache layer
    [1, Hk, P, D] is read in place as an HND tensor."""
    if isinstance(past_key_values, PagedKVCache):
        c = past_key_values
        return c.k[idx], c.v[idx], c.kv_layout, c.length, c.page_table
    layer = past_key_values.layers[idx]
    return layer.keys[0], layer.values[0], "hnd", layer.keys.shape[2], None


# Plans by shape, kept across calls: a decode loop (or a CUDA graph capture
# after one warm-up call) then builds no plan and copies nothing to the device.
_plans: dict = {}


@torch.no_grad()
def cascade_verify_forward(target_model, input_ids: torch.Tensor, position_ids: torch.Tensor,
                           past_key_values, output_hidden_states: bool = True,
                           cascade_graph_runner=None):
    """Returns (logits [bsz, block, vocab], hidden states (L+2 entries) or None,
    new_kv_list [(k_new, v_new) per layer, each [bsz, Hk, block, D]])."""
    model = target_model.model
    bsz, seq_len = input_ids.shape
    is_gpt_oss = type(model.layers[0].self_attn).__name__ == "GptOssAttention"
    hidden = model.embed_tokens(input_ids)
    cos, sin = model.rotary_emb(hidden, position_ids)  # [1, block, D] (GPT-OSS: D/2)
    cos_t, sin_t = cos[0].contiguous(), sin[0].contiguous()
    all_hidden = [hidden] if output_hidden_states else None
    new_kv_list = []

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
        # QK-norm (Qwen3) and RoPE in place on the token-major [B*T, H, D] views
        norm = not is_gpt_oss
        ops.qk_norm_rope(q.view(bsz * seq_len, Hq, D), k_new.view(bsz * seq_len, Hk, D), cos_t,
                         sin_t, q_weight=attn.q_norm.weight if norm else None,
                         k_weight=attn.k_norm.weight if norm else None,
                         eps=attn.q_norm.variance_epsilon if norm else 1e-6, block_len=seq_len)
        q = q.transpose(1, 2)
        k_new = k_new.transpose(1, 2)
        v_new = v_new.transpose(1, 2)
        new_kv_list.append((k_new, v_new))

        keys, values, kv_layout, P, page_table = _prefix(past_key_values, layer_idx)
        window = getattr(attn, "sliding_window", None)
        kv_start = P - window if (window is not None and P > window) else 0
        key = (bsz * seq_len, P, kv_start, Hq, Hk, D, str(q.device))
        plan = _plans.get(key)
        if plan is None:
            plan = CascadePlan([Request(bsz * seq_len, 0, kv_start, P)], Hq, Hk, D, q.device)
            if len(_plans) > 256:
                _plans.clear()
            _plans[key] = plan
        sinks = attn.sinks.float() if is_gpt_oss else None
        out, _ = cascade_attention(q.transpose(1, 2), k_new.transpose(1, 2),
                                   v_new.transpose(1, 2), keys, values, kv_layout, P,
                                   page_table=page_table, causal=True, sm_scale=D ** -0.5,
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
