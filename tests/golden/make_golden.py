"""Generate the golden fixtures of tests/golden/ by running the reference itself.

Runs only where a checkout of the reference exists, named by the environment
variable $D2SD_REFERENCE (the directory holding generation/ and model/); the committed .npz/.json outputs travel, this script does not
need to. Nothing here is imported by the product or by the GPU tests.

What is executed from the reference (catnanami/D2-SD), unmodified:
  * acceptance: the block generation/d3_generator.py:204-222 (greedy walk and the
    output_ids write), executed from the reference file's own text with the
    reference's model/utils.py:sample;
  * single-branch acceptance: generation/dflash_generator.py:110-120;
  * KV commit: generation/d3_generator.py:227-232 on a transformers DynamicCache;
  * draft context feature: the assignment at generation/d3_generator.py:239
    (state.target_hidden = extract_context_feature(...)[valid_block,
    :acceptance_length, :].unsqueeze(0)) with the reference's
    model/utils.py:extract_context_feature (written to hidden_cases.npz;
    `--only hidden` regenerates that file alone);
  * QK-norm + RoPE: generation/verification.py:113-124 restated with the
    reference's own _apply_rotary_pos_emb_qwen3 / _apply_rotary_pos_emb_gpt_oss
    and transformers' Qwen3RMSNorm on bf16 tensors (rope_cases.npz;
    `--only rope` regenerates that file alone);
  * attention: generation/verification.py:cascade_verify_forward on tiny random
    Qwen3 and GPT-OSS models, with flashinfer's two kernels (which need a GPU)
    replaced by the float64 oracle, and the Qwen3 logits checked against the
    reference's plain_verify_forward (HF sdpa, an independent attention). The
    attention output each layer feeds o_proj is recorded as the golden value.

Usage: python tests/golden/make_golden.py [--only hidden|rope]
"""
from __future__ import annotations

import copy
import json
import os
import sys
import textwrap
from pathlib import Path
from types import SimpleNamespace
from typing import List

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if "D2SD_REFERENCE" not in os.environ:
    raise SystemExit("set D2SD_REFERENCE to the reference checkout (generation/, model/)")
REF = Path(os.environ["D2SD_REFERENCE"])
sys.path.insert(0, str(REPO))


def ref_block(rel: str, first: str, last: str) -> str:
    """Source lines of a reference file from the line containing `first` to the
    line containing `last` (inclusive), dedented."""
    lines = (REF / rel).read_text().splitlines()
    i = next(k for k, l in enumerate(lines) if first in l)
    j = next(k for k in range(i, len(lines)) if last in lines[k])
    return textwrap.dedent("\n".join(lines[i:j + 1]))


def import_reference():
    sys.path.insert(0, str(REF))
    from transformers import DynamicCache
    if not hasattr(DynamicCache, "__getitem__") or True:
        # transformers 5 dropped tuple indexing; the reference indexes
        # past_key_values[layer][0|1] (verification.py:127-128).
        DynamicCache.__getitem__ = lambda s, i: (s.layers[i].keys, s.layers[i].values)
    import generation.verification as ver  # noqa: E402
    from model.utils import sample  # noqa: E402
    return ver, sample


# --------------------------------------------------------------------------
# acceptance
# --------------------------------------------------------------------------
def gen_accept_cases(sample, rng: np.random.Generator):
    block = ref_block("generation/d3_generator.py", "output_logits = output.logits",
                      "state.output_ids[:, start + 1:start + acceptance_length + 1]")
    cases = []
    specs = []
    for B in (1, 2, 3, 5, 8):
        for T in (1, 2, 5, 16, 32):
            for V in (37, 129):
                for dt in ("f32", "bf16"):
                    specs.append((B, T, V, dt, "random"))
    for B, T in ((4, 16), (8, 32), (64, 4)):
        specs.append((B, T, 200, "bf16", "all_match"))
        specs.append((B, T, 200, "bf16", "ties"))
        specs.append((B, T, 200, "f32", "nan"))
        specs.append((B, T, 200, "f32", "neginf"))
        specs.append((B, T, 200, "bf16", "late_branch"))
    for (B, T, V, dt, kind) in specs:
        z = rng.standard_normal((B, T, V)).astype(np.float32)
        if kind == "ties":
            z = np.round(z * 2) / 2  # many equal maxima
        if kind == "nan":
            z[rng.integers(0, B), rng.integers(0, T), rng.integers(0, V, 3)] = np.nan
            z[0, 0, V // 2] = np.nan
        if kind == "neginf":
            z[:, :, :] = np.where(rng.random((B, T, V)) < 0.5, -np.inf, z)
            z[0, 0, :] = -np.inf
        zt = torch.from_numpy(z)
        if dt == "bf16":
            zt = zt.to(torch.bfloat16)
        amax = zt.float().argmax(-1).numpy()
        x = rng.integers(0, V, (B, T)).astype(np.int64)
        x[:, 0] = rng.integers(0, V)
        p = {"random": 0.7, "all_match": 1.0, "ties": 0.8, "nan": 0.7, "neginf": 0.7,
             "late_branch": 0.9}[kind]
        for b in range(B):
            for t in range(1, T):
                if rng.random() < p:
                    x[b, t] = amax[b, t - 1]
        if kind == "late_branch" and B > 1:
            # only the last branch survives past position 1
            x[:-1, 1] = (amax[0, 0] + 1) % V
            x[-1, 1:] = amax[-1, :-1]
        start = 3
        ns = dict(torch=torch, sample=sample, List=List, device="cpu", temperature=0.0,
                  block_size_2=T, block_output_ids=torch.from_numpy(x.copy()),
                  output=SimpleNamespace(logits=zt),
                  state=SimpleNamespace(output_ids=torch.full((1, start + T + 2), -7,
                                                              dtype=torch.long)),
                  start=start)
        exec(block, ns)
        # bf16 logits are stored as their raw 16-bit patterns
        stored = (zt.view(torch.int16).numpy() if dt == "bf16" else z)
        cases.append(dict(logits=stored, dtype=dt, block_ids=x,
                          acc=int(ns["acceptance_length"]),
                          ids=torch.cat(ns["accept_ids"]).numpy().astype(np.int64),
                          branch=int(ns["valid_block"]),
                          output_ids=ns["state"].output_ids.numpy()[0]))
    return cases


def gen_dflash_cases(sample, rng: np.random.Generator):
    block = ref_block("generation/dflash_generator.py", "posterior, _ = sample(output.logits",
                      "state.output_ids[:, start + acceptance_length + 1] = posterior")
    cases = []
    for T in (1, 2, 8, 16):
        for V in (50, 700):
            for p in (0.0, 0.7, 1.0):
                z = rng.standard_normal((1, T, V)).astype(np.float32)
                zt = torch.from_numpy(z)
                amax = zt.argmax(-1).numpy()
                x = rng.integers(0, V, (1, T)).astype(np.int64)
                for t in range(1, T):
                    if rng.random() < p:
                        x[0, t] = amax[0, t - 1]
                start = 2
                ns = dict(torch=torch, sample=sample, temperature=0.0,
                          output=SimpleNamespace(logits=zt), block_output_ids=torch.from_numpy(x),
                          state=SimpleNamespace(output_ids=torch.full((1, start + T + 2), -7,
                                                                      dtype=torch.long)),
                          start=start)
                if T == 1:
                    continue  # the reference indexes posterior[:, acceptance_length] with T >= 2
                exec(block, ns)
                cases.append(dict(logits=z, block_ids=x, acc=int(ns["acceptance_length"]) + 1,
                                  output_ids=ns["state"].output_ids.numpy()[0]))
    return cases


# --------------------------------------------------------------------------
# commit
# --------------------------------------------------------------------------
def gen_commit_cases(rng: np.random.Generator):
    from transformers import DynamicCache
    # the first "if use_cascade:" in the file is the verify dispatch (line 187);
    # take the one that follows the acceptance walk
    lines = (REF / "generation/d3_generator.py").read_text().splitlines()
    i = next(k for k, l in enumerate(lines) if "if use_cascade:" in l and k > 220)
    j = next(k for k in range(i, len(lines)) if "layer.values = torch.cat" in lines[k])
    block = textwrap.dedent("\n".join(lines[i:j + 1]))
    cases = []
    for (L, B, Hk, P, T, D) in ((2, 3, 2, 5, 8, 16), (3, 8, 4, 17, 32, 8), (1, 1, 1, 0, 4, 8)):
        for acc in sorted({1, T // 2, T}):
            branch = int(rng.integers(0, B))
            cache = DynamicCache()
            ks = [rng.standard_normal((1, Hk, P, D)).astype(np.float32) for _ in range(L)]
            vs = [rng.standard_normal((1, Hk, P, D)).astype(np.float32) for _ in range(L)]
            for l in range(L):
                cache.update(torch.from_numpy(ks[l]), torch.from_numpy(vs[l]), l)
            new = [(rng.standard_normal((B, Hk, T, D)).astype(np.float32),
                    rng.standard_normal((B, Hk, T, D)).astype(np.float32)) for _ in range(L)]
            ns = dict(torch=torch, use_cascade=True, valid_block=torch.tensor(branch),
                      acceptance_length=acc,
                      state=SimpleNamespace(past_key_values_target=cache),
                      new_kv_list=[(torch.from_numpy(a), torch.from_numpy(b)) for a, b in new])
            exec(block, ns)
            outk = [layer.keys.numpy() for layer in cache.layers]
            outv = [layer.values.numpy() for layer in cache.layers]
            cases.append(dict(L=L, branch=branch, acc=acc, cache_k=np.stack(ks),
                              cache_v=np.stack(vs), new_k=np.stack([a for a, _ in new]),
                              new_v=np.stack([b for _, b in new]), out_k=np.stack(outk),
                              out_v=np.stack(outv)))
    return cases


def gen_hidden_cases(rng: np.random.Generator):
    from model.utils import extract_context_feature
    line = next(l for l in (REF / "generation/d3_generator.py").read_text().splitlines()
                if "state.target_hidden = extract_context_feature" in l and "valid_block" in l)
    block = textwrap.dedent(line)
    cases = []
    for (L, B, T, H, ids) in ((6, 3, 8, 32, (1, 3, 4)), (4, 8, 32, 16, (0, 2)),
                              (3, 1, 16, 16, (1,)), (8, 4, 16, 8, (0, 3, 5, 6))):
        for acc in sorted({1, T // 2, T}):
            branch = int(rng.integers(0, B))
            hs = [rng.standard_normal((B, T, H)).astype(np.float32) for _ in range(L + 2)]
            ns = dict(extract_context_feature=extract_context_feature,
                      output=SimpleNamespace(hidden_states=[torch.from_numpy(h) for h in hs]),
                      draft=SimpleNamespace(target_layer_ids=list(ids)),
                      valid_block=torch.tensor(branch), acceptance_length=acc,
                      state=SimpleNamespace())
            exec(block, ns)
            cases.append(dict(hidden=np.stack(hs), layer_ids=np.asarray(ids), branch=branch,
                              acc=acc, out=ns["state"].target_hidden.numpy()))
    return cases


def gen_rope_cases(ver, rng: np.random.Generator):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    cases = []
    for kind, B, T, Hq, Hk, D in (("qwen3", 3, 8, 8, 2, 128), ("qwen3", 2, 16, 4, 4, 64),
                                  ("gptoss", 3, 8, 8, 2, 64)):
        bf = lambda *shape: torch.from_numpy(  # noqa: E731
            rng.standard_normal(shape).astype(np.float32)).to(torch.bfloat16)
        q, k = bf(B, T, Hq, D) * 3, bf(B, T, Hk, D) * 3
        pos = np.arange(T) + int(rng.integers(0, 5000))
        inv = 1.0 / (1e6 ** (np.arange(0, D, 2) / D))
        ang = pos[:, None] * inv[None, :]
        half_c = torch.from_numpy(np.cos(ang).astype(np.float32)).to(torch.bfloat16)
        half_s = torch.from_numpy(np.sin(ang).astype(np.float32)).to(torch.bfloat16)
        entry = dict(kind=np.asarray(kind), q=q.view(torch.int16).numpy(),
                     k=k.view(torch.int16).numpy(), cos_half=half_c.view(torch.int16).numpy(),
                     sin_half=half_s.view(torch.int16).numpy())
        if kind == "qwen3":
            qn, kn = Qwen3RMSNorm(D, eps=1e-6), Qwen3RMSNorm(D, eps=1e-6)
            qn.weight.data = (1 + 0.1 * bf(D).float()).to(torch.bfloat16)
            kn.weight.data = (1 + 0.1 * bf(D).float()).to(torch.bfloat16)
            qn, kn = qn.to(torch.bfloat16), kn.to(torch.bfloat16)
            cos = torch.cat([half_c, half_c], -1)[None]
            sin = torch.cat([half_s, half_s], -1)[None]
            with torch.no_grad():
                qq, kk = ver._apply_rotary_pos_emb_qwen3(qn(q).transpose(1, 2),
                                                         kn(k).transpose(1, 2), cos, sin)
            entry.update(q_weight=qn.weight.data.view(torch.int16).numpy(),
                         k_weight=kn.weight.data.view(torch.int16).numpy())
        else:
            qq, kk = ver._apply_rotary_pos_emb_gpt_oss(q.transpose(1, 2), k.transpose(1, 2),
                                                       half_c[None], half_s[None])
        entry.update(q_out=qq.transpose(1, 2).contiguous().view(torch.int16).numpy(),
                     k_out=kk.transpose(1, 2).contiguous().view(torch.int16).numpy())
        cases.append(entry)
    return cases


# --------------------------------------------------------------------------
# attention through the reference's cascade_verify_forward
# --------------------------------------------------------------------------
class OracleFlashInfer:
    """Stands in for the flashinfer module inside generation.verification on the
    CPU: single_prefill_with_kv_cache / merge_state_in_place restated by the
    oracle, with every call recorded."""

    def __init__(self):
        from oracle import attention as A
        self.A = A
        self.calls = []

    def single_prefill_with_kv_cache(self, q, k, v, causal=False, return_lse=True, sm_scale=None):
        out, lse = self.A.single_prefill(q, k, v, causal=causal, sm_scale=sm_scale)
        self.calls.append(("prefill", causal, q.shape[0], k.shape[0]))
        return (torch.from_numpy(out).to(q.dtype), torch.from_numpy(lse).float())

    def merge_state_in_place(self, v, s, v_other, s_other):
        mv, ms = self.A.merge_state(v, s, v_other, s_other)
        v.copy_(torch.from_numpy(mv).to(v.dtype))
        s.copy_(torch.from_numpy(ms).to(s.dtype))
        self.calls.append(("merge",))


def tiny_model(kind: str):
    torch.manual_seed(0)
    if kind == "qwen3":
        from transformers import Qwen3Config, Qwen3ForCausalLM
        cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=256,
                          num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                          head_dim=64, rope_theta=1e6, max_position_embeddings=1024,
                          attn_implementation="sdpa")
        return Qwen3ForCausalLM(cfg).eval()
    from transformers import GptOssConfig, GptOssForCausalLM
    cfg = GptOssConfig(vocab_size=512, hidden_size=256, intermediate_size=256,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=64, num_local_experts=4, num_experts_per_tok=2,
                       sliding_window=128, layer_types=["sliding_attention", "full_attention"],
                       max_position_embeddings=1024, attn_implementation="eager")
    m = GptOssForCausalLM(cfg).eval()
    with torch.no_grad():
        for layer in m.model.layers:
            layer.self_attn.sinks.normal_()
    return m


def gen_attention_case(ver, kind: str, prefix: int, B: int, T: int):
    from transformers import DynamicCache
    model = tiny_model(kind)
    g = torch.Generator().manual_seed(1)
    V = model.config.vocab_size
    prompt = torch.randint(0, V, (1, prefix), generator=g)
    cache = DynamicCache()
    with torch.no_grad():
        model(prompt, past_key_values=cache, use_cache=True)
    block = torch.randint(0, V, (B, T), generator=g)
    block[:, 0] = block[0, 0]
    pos = torch.arange(prefix, prefix + T).unsqueeze(0)

    fi = OracleFlashInfer()
    ver.flashinfer = fi
    captured = []
    hooks = []
    for layer in model.model.layers:
        hooks.append(layer.self_attn.o_proj.register_forward_pre_hook(
            lambda mod, args: captured.append(args[0].detach().clone())))
    # q, k_new, v_new per layer: recorded from the level-1 call arguments
    qkv = []
    orig = fi.single_prefill_with_kv_cache

    def rec(q, k, v, causal=False, return_lse=True, sm_scale=None):
        if not causal and q.shape[0] == B * T:
            qkv.append((q.detach().clone(), k.detach().clone(), v.detach().clone()))
        return orig(q, k, v, causal=causal, return_lse=return_lse, sm_scale=sm_scale)

    fi.single_prefill_with_kv_cache = rec
    with torch.no_grad():
        logits, _, new_kv = ver.cascade_verify_forward(model, block, pos, copy.deepcopy(cache),
                                                       output_hidden_states=True,
                                                       cascade_graph_runner=None)
    for h in hooks:
        h.remove()
    summary = {}
    if kind == "qwen3":
        diffs = []
        for b in range(B):
            with torch.no_grad():
                out = ver.plain_verify_forward(model, block[b:b + 1], pos, copy.deepcopy(cache),
                                               output_hidden_states=False)
            diffs.append(float((out.logits[0] - logits[b]).abs().max()))
        summary["max_abs_logit_diff_cascade_vs_plain"] = max(diffs)
    layers = []
    for l, layer in enumerate(model.model.layers):
        attn = layer.self_attn
        q_all, k_pref_used, v_pref_used = qkv[l]
        k_full = cache.layers[l].keys[0].transpose(0, 1).numpy()  # [P, Hk, D]
        v_full = cache.layers[l].values[0].transpose(0, 1).numpy()
        k_new, v_new = new_kv[l]  # [B, Hk, T, D]
        sw = getattr(attn, "sliding_window", None)
        entry = dict(q=q_all.reshape(B, T, -1, q_all.shape[-1]).numpy(),
                     k_new=k_new.transpose(1, 2).numpy(), v_new=v_new.transpose(1, 2).numpy(),
                     k_prefix=k_full, v_prefix=v_full,
                     window=-1 if sw is None else int(sw),
                     out=captured[l].reshape(B, T, attn.config.num_attention_heads, -1).numpy())
        if kind == "gptoss":
            entry["sinks"] = attn.sinks.detach().float().numpy()
        layers.append(entry)
    return layers, summary


def save_cases(path: Path, cases, keys):
    flat = {}
    for i, c in enumerate(cases):
        for k in keys:
            if k in c:
                flat[f"c{i}_{k}"] = np.asarray(c[k])
    flat["n"] = np.asarray(len(cases))
    np.savez_compressed(path, **flat)


def main():
    ver, sample = import_reference()
    hd_cases = gen_hidden_cases(np.random.default_rng(20261202))
    save_cases(HERE / "hidden_cases.npz", hd_cases, ["hidden", "layer_ids", "branch", "acc", "out"])
    if "--only" in sys.argv and sys.argv[sys.argv.index("--only") + 1] == "hidden":
        print(json.dumps({"hidden_cases": len(hd_cases)}))
        return
    rp_cases = gen_rope_cases(ver, np.random.default_rng(20261203))
    save_cases(HERE / "rope_cases.npz", rp_cases,
               ["kind", "q", "k", "cos_half", "sin_half", "q_weight", "k_weight", "q_out", "k_out"])
    if "--only" in sys.argv and sys.argv[sys.argv.index("--only") + 1] == "rope":
        print(json.dumps({"rope_cases": len(rp_cases)}))
        return
    rng = np.random.default_rng(20260101)
    acc_cases = gen_accept_cases(sample, rng)
    save_cases(HERE / "accept_cases.npz", acc_cases,
               ["logits", "dtype", "block_ids", "acc", "ids", "branch", "output_ids"])
    df_cases = gen_dflash_cases(sample, rng)
    save_cases(HERE / "dflash_cases.npz", df_cases, ["logits", "block_ids", "acc", "output_ids"])
    cm_cases = gen_commit_cases(rng)
    save_cases(HERE / "commit_cases.npz", cm_cases,
               ["L", "branch", "acc", "cache_k", "cache_v", "new_k", "new_v", "out_k", "out_v"])
    summary = {"accept_cases": len(acc_cases), "dflash_cases": len(df_cases),
               "commit_cases": len(cm_cases), "hidden_cases": len(hd_cases)}
    for kind, P, B, T in (("qwen3", 300, 3, 8), ("gptoss", 300, 3, 8)):
        layers, s = gen_attention_case(ver, kind, P, B, T)
        save_cases(HERE / f"attention_{kind}.npz", layers,
                   ["q", "k_new", "v_new", "k_prefix", "v_prefix", "window", "out", "sinks"])
        summary[kind] = dict(prefix=P, branches=B, block=T, layers=len(layers), **s)
    (HERE / "reference_pin.json").write_text(json.dumps(summary, indent=1) + "\n")
    print(json.dumps(summary, indent=1))


if __name__ == "__main__":
    main()
