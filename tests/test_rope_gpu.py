"""QK-norm + RoPE of the block's q and k (generation/verification.py:113-124)
on the GPU against the reference-executed golden vectors and the CPU oracle.

Tolerance: the kernel makes every 16-bit rounding of the reference's eager
expressions in the same order; the differences are rsqrt and the mean's
summation order (the GPU's against the CPU's), which can move a normed value
across a bf16 rounding boundary, and the RoPE sum can cancel. So at least 99% of
the outputs must be bit-identical and all within the project's bf16 bound,
2e-2 absolute / 1e-2 relative."""
import numpy as np
import pytest
import torch

from conftest import load_cases
from oracle import rope as OR

pytestmark = pytest.mark.gpu


def _bf(a):
    return torch.from_numpy(a).view(torch.bfloat16)


def _check(got: torch.Tensor, ref: torch.Tensor):
    got, ref = got.float().cpu(), ref.float().cpu()
    same = (got == ref).float().mean().item()
    assert same >= 0.99, f"only {same:.4f} of the outputs are bit-identical"
    np.testing.assert_allclose(got.numpy(), ref.numpy(), rtol=1e-2, atol=2e-2)


def test_rope_golden(cuda_device):
    from d2sd_b200 import ops
    for c in load_cases("rope_cases.npz"):
        gpt = str(c["kind"]) == "gptoss"
        q, k = _bf(c["q"]), _bf(c["k"])
        B, T, Hq, D = q.shape
        qd = q.reshape(B * T, Hq, D).to(cuda_device)
        kd = k.reshape(B * T, k.shape[2], D).to(cuda_device)
        cos = _bf(c["cos_half"]).to(cuda_device)
        sin = _bf(c["sin_half"]).to(cuda_device)
        qw = None if gpt else _bf(c["q_weight"]).to(cuda_device)
        kw = None if gpt else _bf(c["k_weight"]).to(cuda_device)
        qo, ko = ops.qk_norm_rope(qd, kd, cos, sin, q_weight=qw, k_weight=kw, eps=1e-6,
                                  block_len=T)
        _check(qo.reshape(B, T, Hq, D), _bf(c["q_out"]))
        _check(ko.reshape(B, T, -1, D), _bf(c["k_out"]))


@pytest.mark.parametrize("B,T,Hq,Hk,D,full", [(8, 32, 32, 8, 128, True), (6, 16, 64, 8, 64, False)])
def test_rope_full_size_vs_oracle(cuda_device, B, T, Hq, Hk, D, full):
    """BASELINE config 3 (Qwen3-8B: full-width table, QK-norm) and config 5
    (GPT-OSS: half-width table, no norm) shapes; strided output views; a
    positions table, and the full-width table read through its first half."""
    from d2sd_b200 import ops
    g = torch.Generator().manual_seed(D + T)
    q = (torch.randn(B, T, Hq, D, generator=g) * 3).to(torch.bfloat16)
    k = (torch.randn(B, T, Hk, D, generator=g) * 3).to(torch.bfloat16)
    P = 64
    ang = torch.arange(P)[:, None].double() * (1.0 / (1e6 ** (torch.arange(0, D, 2) / D)))[None]
    ch, sh = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    pos = torch.randperm(P, generator=g)[:T].to(torch.int32)
    if full:
        qw = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
        kw = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
        cos_t, sin_t = torch.cat([ch, ch], -1), torch.cat([sh, sh], -1)
    else:
        qw = kw = None
        cos_t, sin_t = ch, sh
    rq, rk = OR.qk_norm_rope(q, k, (cos_t if full else ch)[pos.long()][None],
                             (sin_t if full else sh)[pos.long()][None], qw, kw, 1e-6,
                             gpt_oss=not full)
    dev = cuda_device
    q_out = torch.zeros(B * T, Hq, D + 8, dtype=torch.bfloat16, device=dev)[..., :D]
    k_out = torch.zeros(B * T, Hk, D + 8, dtype=torch.bfloat16, device=dev)[..., :D]
    ops.qk_norm_rope(q.reshape(B * T, Hq, D).to(dev), k.reshape(B * T, Hk, D).to(dev),
                     cos_t.to(dev), sin_t.to(dev),
                     q_weight=None if qw is None else qw.to(dev),
                     k_weight=None if kw is None else kw.to(dev), eps=1e-6, block_len=T,
                     positions=pos.to(dev), q_out=q_out, k_out=k_out)
    _check(q_out.reshape(B, T, Hq, D), rq)
    _check(k_out.reshape(B, T, Hk, D), rk)
