"""cascade_verify_forward on the kernels against the same forward with the
float64 oracle as its attention, on tiny random bf16 Qwen3 / GPT-OSS targets,
and the DFlash/D3-style decode loop pieces (verify -> commit) end to end."""
import copy

import numpy as np
import pytest
import torch

from oracle import attention as AT

pytestmark = pytest.mark.gpu


def tiny(kind, dev):
    torch.manual_seed(0)
    if kind == "qwen3":
        from transformers import Qwen3Config, Qwen3ForCausalLM
        cfg = Qwen3Config(vocab_size=512, hidden_size=512, intermediate_size=512,
                          num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                          head_dim=128, rope_theta=1e6, max_position_embeddings=4096)
        m = Qwen3ForCausalLM(cfg)
    else:
        from transformers import GptOssConfig, GptOssForCausalLM
        cfg = GptOssConfig(vocab_size=512, hidden_size=512, intermediate_size=256,
                           num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                           head_dim=64, num_local_experts=4, num_experts_per_tok=2,
                           sliding_window=128, layer_types=["sliding_attention", "full_attention"],
                           max_position_embeddings=4096, attn_implementation="eager")
        m = GptOssForCausalLM(cfg)
        with torch.no_grad():
            for layer in m.model.layers:
                layer.self_attn.sinks.normal_()
    return m.to(dev).to(torch.bfloat16).eval()


def oracle_forward(model, ids, pos, cache, is_gpt_oss):
    """The reference's layer loop (generation/verification.py:96-201) with the
    attention computed by the float64 oracle of the same cascade."""
    from oracle import rope as OR
    m = model.model
    B, T = ids.shape
    h = m.embed_tokens(ids)
    cos, sin = m.rotary_emb(h, pos)
    for li, layer in enumerate(m.layers):
        res = h
        x = layer.input_layernorm(h)
        at = layer.self_attn
        Hq, Hk, D = at.config.num_attention_heads, at.config.num_key_value_heads, at.head_dim
        q = at.q_proj(x).view(B, T, Hq, D)
        k = at.k_proj(x).view(B, T, Hk, D)
        v = at.v_proj(x).view(B, T, Hk, D)
        qw = None if is_gpt_oss else at.q_norm.weight
        kw = None if is_gpt_oss else at.k_norm.weight
        q, k = OR.qk_norm_rope(q, k, cos, sin, qw, kw, 1e-6 if is_gpt_oss else at.q_norm.variance_epsilon,
                               gpt_oss=is_gpt_oss)
        q, k = q.transpose(1, 2), k.transpose(1, 2)
        v = v.transpose(1, 2)
        kp = cache.layers[li].keys[0].transpose(0, 1)
        vp = cache.layers[li].values[0].transpose(0, 1)
        sw = getattr(at, "sliding_window", None)
        o, _ = AT.cascade_attention(q.transpose(1, 2).double().cpu(), k.transpose(1, 2).double().cpu(),
                                    v.transpose(1, 2).double().cpu(), kp.double().cpu(),
                                    vp.double().cpu(), causal=True, sliding_window=sw,
                                    sinks=at.sinks.double().cpu().numpy() if is_gpt_oss else None)
        o = torch.from_numpy(o).to(h.dtype).to(h.device)
        h = res + at.o_proj(o.reshape(B, T, -1))
        res = h
        mo = layer.mlp(layer.post_attention_layernorm(h))
        if isinstance(mo, tuple):
            mo = mo[0]
        h = res + mo
    return model.lm_head(m.norm(h))


@pytest.mark.parametrize("kind", ["qwen3", "gptoss"])
def test_cascade_verify_forward_matches_oracle(cuda_device, kind):
    from transformers import DynamicCache

    import d2sd_b200 as d
    model = tiny(kind, cuda_device)
    g = torch.Generator().manual_seed(1)
    P, B, T = 700, 4, 16
    prompt = torch.randint(0, 512, (1, P), generator=g).to(cuda_device)
    cache = DynamicCache()
    with torch.no_grad():
        model(prompt, past_key_values=cache, use_cache=True)
    block = torch.randint(0, 512, (B, T), generator=g).to(cuda_device)
    block[:, 0] = block[0, 0]
    pos = torch.arange(P, P + T, device=cuda_device).unsqueeze(0)
    logits, hidden, new_kv = d.cascade_verify_forward(model, block, pos, cache,
                                                      output_hidden_states=True)
    assert len(hidden) == len(model.model.layers) + 2
    assert new_kv[0][0].shape == (B, model.config.num_key_value_heads, T,
                                  model.model.layers[0].self_attn.head_dim)
    with torch.no_grad():
        ref = oracle_forward(model, block, pos, copy.deepcopy(cache), kind == "gptoss")
    err = (logits.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item()
    assert err <= 2e-2 * scale + 2e-2, (err, scale)
    agree = (logits.argmax(-1) == ref.argmax(-1)).float().mean().item()
    assert agree > 0.95
