"""The fp32 cascade (d2sd_cascade_attention_f32) against the float64 oracle at
BASELINE config 1 -- fp32, seed 0, prefix 512 with 8 kv heads, 32 query heads,
head_dim 128, 4 branches x 16 tokens, Q/K/V ~ N(0,1)/sqrt(128) -- within the
north star's fp32 tolerance of 1e-5, through each call surface that takes
fp32: cascade_attention, the CascadeGraphRunner drop-in and the
FlashInfer-signature single_prefill_with_kv_cache."""
import numpy as np
import pytest
import torch

from oracle import attention as AT

pytestmark = pytest.mark.gpu

TOL = 1e-5


def f64(t):
    return t.detach().double().cpu().numpy()


def cfg1(dev, seed=0, P=512, B=4, T=16, Hq=32, Hk=8, D=128):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: (torch.randn(*s, generator=g) / D ** 0.5).to(dev)  # noqa: E731
    return r(B, T, Hq, D), r(B, T, Hk, D), r(B, T, Hk, D), r(P, Hk, D), r(P, Hk, D)


@pytest.mark.parametrize("layout", ["nhd", "hnd"])
@pytest.mark.parametrize("window,sink_mode", [(None, None), (128, None), (None, "reference"),
                                              (128, "exact")])
def test_cascade_fp32_config1(cuda_device, layout, window, sink_mode):
    import d2sd_b200 as d
    q, kn, vn, kp, vp = cfg1(cuda_device)
    sinks = torch.randn(q.shape[2], generator=torch.Generator().manual_seed(1)).to(cuda_device) \
        if sink_mode else None
    kc, vc = (kp, vp) if layout == "nhd" else (kp.transpose(0, 1).contiguous(),
                                                vp.transpose(0, 1).contiguous())
    out, lse = d.cascade_attention(q, kn, vn, kc, vc, layout, kp.shape[0], sliding_window=window,
                                   sinks=sinks, sink_mode=sink_mode or "reference")
    assert out.dtype == torch.float32
    ro, rl = AT.cascade_attention(f64(q), f64(kn), f64(vn), f64(kp), f64(vp), causal=True,
                                  sliding_window=window,
                                  sinks=None if sinks is None else f64(sinks),
                                  sink_mode=sink_mode or "reference")
    np.testing.assert_allclose(f64(out), ro, atol=TOL, rtol=TOL)
    np.testing.assert_allclose(f64(lse), rl, atol=TOL, rtol=TOL)


@pytest.mark.parametrize("causal", [True, False])
def test_runner_and_single_prefill_fp32(cuda_device, causal):
    import d2sd_b200 as d
    q, kn, vn, kp, vp = cfg1(cuda_device, seed=3)
    B, T, Hq, D = q.shape
    Hk = kn.shape[2]
    out_s, lse_s = d.single_prefill_with_kv_cache(q.reshape(B * T, Hq, D), kp, vp, causal=False,
                                                  return_lse=True, sm_scale=D ** -0.5)
    ro, rl = AT.single_prefill(f64(q.reshape(B * T, Hq, D)), f64(kp), f64(vp), causal=False,
                               sm_scale=D ** -0.5)
    np.testing.assert_allclose(f64(out_s), ro, atol=TOL, rtol=TOL)
    np.testing.assert_allclose(f64(lse_s), rl, atol=TOL, rtol=TOL)
    r = d.CascadeGraphRunner(T, Hq, Hk, D, torch.float32, cuda_device, D ** -0.5, causal)
    out_s, lse_s = out_s.view(B, T, Hq, D), lse_s.view(B, T, Hq)
    r.run(q, kn, vn, out_s, lse_s)
    fo, fl = AT.cascade_attention(f64(q), f64(kn), f64(vn), f64(kp), f64(vp), causal=causal)
    np.testing.assert_allclose(f64(out_s), fo, atol=TOL, rtol=TOL)
    np.testing.assert_allclose(f64(lse_s), fl, atol=TOL, rtol=TOL)
    # the level-2 form of single_prefill: one block's causal attention to itself
    o2, l2 = d.single_prefill_with_kv_cache(q[0], kn[0], vn[0], causal=causal, return_lse=True)
    r2, rl2 = AT.single_prefill(f64(q[0]), f64(kn[0]), f64(vn[0]), causal=causal)
    np.testing.assert_allclose(f64(o2), r2, atol=TOL, rtol=TOL)
    np.testing.assert_allclose(f64(l2), rl2, atol=TOL, rtol=TOL)
