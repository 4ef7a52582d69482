"""The DTA drafter's cascade (model/dflash.py:99-136) composed from this
library's drop-ins, against the float64 oracle.

The reference's steps, restated with the d2sd functions in their place:
  k_shared = cat([k_cache[0], k[0, :, :ctx_len]], dim=1)          (:103-104)
  q_fi = q.transpose(1, 2); q_all = q_fi.reshape(bsz * q_len, ...)  (:109-111)
  out_shared, lse_shared = single_prefill_with_kv_cache(q_all, k_shared_fi,
      v_shared_fi, causal=False, return_lse=True)                   (:112-115)
  k_local_all = k[:, :, ctx_len:].transpose(1, 2).contiguous()     (:120-121)
  cascade_runner.run(q_fi, k_local_all, v_local_all, out_shared, lse_shared)
with the runner built non-causal, as benchmark.py:46-55 builds the DTA one.
q_fi is a transposed, non-contiguous view; kernel (b) reads it through its
block stride, so no copy of q is made. Tolerance: 2e-2 abs / 1e-2 rel (bf16).
"""
import numpy as np
import pytest
import torch

from oracle import attention as AT

pytestmark = pytest.mark.gpu


def f64(t):
    return t.detach().double().cpu().numpy()


@pytest.mark.parametrize("bsz,q_len,cached,ctx_len", [(5, 16, 300, 7), (2, 16, 129, 1),
                                                      (4, 32, 700, 16)])
def test_dta_cascade_composition(cuda_device, bsz, q_len, cached, ctx_len):
    import d2sd_b200 as d
    dev = cuda_device
    Hq, Hk, D = 32, 8, 128
    g = torch.Generator().manual_seed(bsz * 100 + q_len)
    bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).to(dev)  # noqa: E731
    q = bf(bsz, Hq, q_len, D)                  # after RoPE, [bsz, H, q_len, D]
    k = bf(bsz, Hk, ctx_len + q_len, D)        # context tokens, then the noise block
    v = bf(bsz, Hk, ctx_len + q_len, D)
    k_cache, v_cache = bf(1, Hk, cached, D), bf(1, Hk, cached, D)

    k_shared = torch.cat([k_cache[0], k[0, :, :ctx_len, :]], dim=1)
    v_shared = torch.cat([v_cache[0], v[0, :, :ctx_len, :]], dim=1)
    k_shared_fi = k_shared.transpose(0, 1).contiguous()
    v_shared_fi = v_shared.transpose(0, 1).contiguous()
    q_fi = q.transpose(1, 2)
    assert not q_fi.is_contiguous()
    q_all = q_fi.reshape(bsz * q_len, -1, D)
    out_shared, lse_shared = d.single_prefill_with_kv_cache(
        q_all, k_shared_fi, v_shared_fi, causal=False, return_lse=True, sm_scale=D ** -0.5)
    out_shared = out_shared.view(bsz, q_len, -1, D)
    lse_shared = lse_shared.view(bsz, q_len, -1)
    k_local_all = k[:, :, ctx_len:, :].transpose(1, 2).contiguous()
    v_local_all = v[:, :, ctx_len:, :].transpose(1, 2).contiguous()
    runner = d.CascadeGraphRunner(q_len, Hq, Hk, D, torch.bfloat16, dev, D ** -0.5, False)
    for b in range(2, 6):
        runner._capture(b)
    runner.run(q_fi, k_local_all, v_local_all, out_shared, lse_shared)
    attn_output = out_shared.reshape(bsz, q_len, -1)

    ro, rl = AT.cascade_attention(f64(q_fi), f64(k_local_all), f64(v_local_all),
                                  f64(k_shared_fi), f64(v_shared_fi), causal=False)
    np.testing.assert_allclose(f64(attn_output).reshape(ro.shape), ro, atol=2e-2, rtol=1e-2)
    np.testing.assert_allclose(f64(lse_shared), rl, atol=1e-2)
