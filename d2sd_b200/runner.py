"""Drop-in ``CascadeGraphRunner`` (model/cascade_graph.py:5-112).

Same constructor, ``_capture(bsz)`` and ``run(q_local, k_local, v_local,
out_shared, lse_shared)``: after ``run`` returns, ``out_shared`` holds the
merged (shared + local) attention output and ``lse_shared`` the merged base-2
LSE, both updated in place.

The reference captures, per batch size, a CUDA graph of B single_prefill +
merge_state_in_place launches over static buffers, and pays 5 copies in and 2
copies out around every replay (cascade_graph.py:100-112). Kernel (b) does the
local attention of every branch and the merge in ONE launch that reads the
caller's (possibly non-contiguous) tensors and writes out_shared/lse_shared in
place, so there is nothing to copy and nothing left to capture: ``_capture``
only checks the shapes and warms the launch up, so that a later ``run`` inside
the caller's own stream capture is legal.
"""
from __future__ import annotations

import torch

from . import _lib, ops


class CascadeGraphRunner:
    def __init__(self, block_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device, sm_scale: float, causal: bool):
        if dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError("CascadeGraphRunner: dtype must be bf16, fp16 or fp32")
        if num_heads % num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.block_size = block_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.sm_scale = sm_scale
        self.causal = causal
        self._graphs: dict[int, None] = {}
        self._buffers: dict[int, dict[str, torch.Tensor]] = {}

    def _capture(self, bsz: int) -> None:
        """Prepare batch size ``bsz`` (the reference pre-captures 2..5,
        benchmark.py:68-70): one launch on scratch tensors."""
        T, H, Hk, D = self.block_size, self.num_heads, self.num_kv_heads, self.head_dim
        z = lambda *s: torch.zeros(*s, dtype=self.dtype, device=self.device)  # noqa: E731
        q, k, v, o = z(bsz, T, H, D), z(bsz, T, Hk, D), z(bsz, T, Hk, D), z(bsz, T, H, D)
        lse = torch.zeros(bsz, T, H, dtype=torch.float32, device=self.device)
        self._launch(q, k, v, o, lse)
        torch.cuda.synchronize(self.device)
        self._graphs[bsz] = None

    def _launch(self, q_local, k_local, v_local, out_shared, lse_shared) -> None:
        bsz, T = q_local.shape[0], q_local.shape[1]
        H, Hk, D = self.num_heads, self.num_kv_heads, self.head_dim

        def tok(t):  # [bsz, T, ...] -> [bsz*T, ...]; a view when the dims merge
            return t.flatten(0, 1) if _flat_ok(t) else t.reshape(bsz * T, *t.shape[2:])

        if self.dtype == torch.float32:  # fp32 end to end (d2sd_cascade_attention_f32)
            ops.cascade_attention_f32(
                tok(q_local), tok(out_shared), tok(lse_shared), num_blocks=bsz, block_len=T,
                num_kv_heads=Hk, sm_scale=self.sm_scale, k_local=tok(k_local),
                v_local=tok(v_local), mask_mode=_lib.MASK_CAUSAL if self.causal else _lib.MASK_NONE,
                prefix_out=tok(out_shared), prefix_lse=tok(lse_shared))
            return
        # q is read through its own block stride (a transposed per-block view,
        # model/dflash.py:109,124, needs no copy); k/v merge their token axes
        ops.suffix_merge(q_local, tok(k_local), tok(v_local), tok(out_shared),
                         tok(lse_shared), num_blocks=bsz, block_len=T, num_qo_heads=H,
                         num_kv_heads=Hk, sm_scale=self.sm_scale,
                         mask_mode=_lib.MASK_CAUSAL if self.causal else _lib.MASK_NONE,
                         prefix_out=tok(out_shared), prefix_lse=tok(lse_shared))

    def run(self, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
            out_shared: torch.Tensor, lse_shared: torch.Tensor) -> None:
        """q_local [bsz, T, H, D], k/v_local [bsz, T, Hk, D], out_shared [bsz, T, H, D]
        (updated in place), lse_shared [bsz, T, H] fp32 (updated in place)."""
        bsz, T = q_local.shape[0], q_local.shape[1]
        if T != self.block_size:
            raise ValueError(f"block length {T} != runner block_size {self.block_size}")
        if not (_flat_ok(out_shared) and _flat_ok(lse_shared)):
            raise ValueError("out_shared/lse_shared must allow a (bsz*T) token view")
        if bsz not in self._graphs:
            self._capture(bsz)
        self._launch(q_local, k_local, v_local, out_shared, lse_shared)


def _flat_ok(t: torch.Tensor) -> bool:
    """True if dims 0 and 1 can be merged into one token axis without a copy."""
    return t.shape[1] <= 1 or t.shape[0] <= 1 or t.stride(0) == t.stride(1) * t.shape[1]
