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


def oracle_forward(model, ids, pos, cache, is_gpt_oss, new_kv=None):
    """The reference's layer loop (generation/verification.py:96-201) with the
    attention computed by the float64 oracle of the same cascade; appends each
    layer's post-RoPE (k, v) [B, Hk, T, D] to ``new_kv`` when given."""
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
        if new_kv is not None:
            new_kv.append((k, v))
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


def test_d3_loop_on_the_paged_cache(cuda_device):
    """Three D3 steps (generation/d3_generator.py:186-239): verify forward ->
    acceptance -> commit -> next block at the advanced positions, run on the
    paged cache with the kernels, beside the reference loop (DynamicCache +
    torch.cat commit) with the float64 oracle as its attention, fed the same
    commits. Each step: logits within tolerance, acceptance bit-exact against
    the oracle walk of the same logits, and the paged cache equal to the
    reference's concatenated cache bit for bit."""
    from transformers import DynamicCache

    import d2sd_b200 as d
    from oracle import accept as OA
    dev = cuda_device
    model = tiny("qwen3", dev)
    nl = len(model.model.layers)
    Hk, D = model.config.num_key_value_heads, model.model.layers[0].self_attn.head_dim
    g = torch.Generator().manual_seed(5)
    P, B, T, steps = 300, 4, 16, 3
    prompt = torch.randint(0, 512, (1, P), generator=g).to(dev)
    ref_cache = DynamicCache()
    with torch.no_grad():
        model(prompt, past_key_values=ref_cache, use_cache=True)
    paged = d.PagedKVCache(nl, Hk, D, P + steps * T + 16, device=dev,
                           page_order=torch.randperm(-(-(P + steps * T + 16) // 16), generator=g))
    for l in range(nl):
        paged.write(l, ref_cache.layers[l].keys[0].transpose(0, 1),
                    ref_cache.layers[l].values[0].transpose(0, 1))
    paged.length = P
    ver = d.Verifier(B, T, 512, dev)
    anchor = int(prompt[0, -1])
    for step in range(steps):
        L0 = paged.length
        pos = torch.arange(L0, L0 + T, device=dev).unsqueeze(0)
        block = torch.randint(0, 512, (B, T), generator=g).to(dev)
        block[:, 0] = anchor
        # drafts that agree with the target for a few positions (first pass)
        first, _, _ = d.cascade_verify_forward(model, block, pos, paged, output_hidden_states=False)
        pred = first.argmax(-1)
        for b in range(B):
            block[b, 1:1 + 2 * b] = pred[b, :2 * b]
        logits, _, new_kv = d.cascade_verify_forward(model, block, pos, paged,
                                                     output_hidden_states=False)
        with torch.no_grad():
            ref = oracle_forward(model, block, pos, copy.deepcopy(ref_cache), False)
        err = (logits.float() - ref.float()).abs().max().item()
        assert err <= 2e-2 * ref.float().abs().max().item() + 2e-2, (step, err)
        ver.launch(logits, block)
        paged.commit([k for k, _ in new_kv], [v for _, v in new_kv], ver.result)
        acc, ids, branch = ver.read()
        racc, rids, rbranch = OA.verify_accept(logits.float().cpu(), block.cpu())
        assert (acc, branch) == (racc, rbranch), step
        np.testing.assert_array_equal(ids.cpu().numpy(), rids)
        # the reference's commit (generation/d3_generator.py:227-232) of the same rows
        for l, (k, v) in enumerate(new_kv):
            lay = ref_cache.layers[l]
            lay.keys = torch.cat([lay.keys, k[branch:branch + 1, :, :acc]], dim=2)
            lay.values = torch.cat([lay.values, v[branch:branch + 1, :, :acc]], dim=2)
        paged.length = L0 + acc
        for l in range(nl):
            gk, gv = paged.gather(l)
            assert torch.equal(gk, ref_cache.layers[l].keys[0].transpose(0, 1)), (step, l)
            assert torch.equal(gv, ref_cache.layers[l].values[0].transpose(0, 1)), (step, l)
        anchor = int(ids[-1])
