"""torch-tensor front end of the C ABI: argument checks, strides, streams.

Each function maps tensors onto one ``d2sd_*`` entry point of ``libd2sd.so`` and
launches on the current CUDA stream. Nothing here computes on the host; if the
library is missing the import of ``d2sd_b200._lib.load`` raises.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check, load

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
           torch.float16: _lib.DTYPE_F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("d2sd kernels take CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def num_sms(device: torch.device | None = None) -> int:
    return torch.cuda.get_device_properties(device or torch.cuda.current_device()).multi_processor_count


# ---------------------------------------------------------------------------
# KV views
# ---------------------------------------------------------------------------
@dataclass
class KVView:
    """How kernel (a) addresses a K or V tensor.

    layout "paged_umma": [pages, Hk, 16, D] holding each (page, head) block in
    the tensor core's core-matrix order (D2SD_KV_UMMA_PAGES, see
    kv_cache.PagedKVCache); "paged_hnd": [pages, Hk, page_size, D]; "paged_nhd": [pages,
    page_size, Hk, D]; "nhd": [tokens, Hk, D] (FlashInfer's NHD, the layout of
    generation/verification.py:139-140 after its transpose copy); "hnd":
    [Hk, tokens, D] (a DynamicCache layer [1, Hk, P, D] with the batch index
    dropped -- read in place, no transpose copy).
    """
    stride_page: int
    stride_slot: int
    stride_head: int
    page_size: int
    num_pages: int  # pages (paged) or tokens (contiguous)
    num_kv_heads: int
    head_dim: int
    paged: bool
    native: bool = False


def kv_view(t: torch.Tensor, layout: str) -> KVView:
    if t.stride(-1) != 1:
        raise ValueError("the head dimension of K/V must be contiguous")
    if layout == "paged_umma":
        P, H, S, D = t.shape
        if S != 16 or t.stride(2) != D or t.stride(1) != 16 * D:
            raise ValueError("paged_umma pools are contiguous [pages, Hk, 16, D] blocks")
        return KVView(t.stride(0), D, t.stride(1), S, P, H, D, True, True)
    if layout == "paged_hnd":
        P, H, S, D = t.shape
        return KVView(t.stride(0), t.stride(2), t.stride(1), S, P, H, D, True)
    if layout == "paged_nhd":
        P, S, H, D = t.shape
        return KVView(t.stride(0), t.stride(1), t.stride(2), S, P, H, D, True)
    if layout == "nhd":
        N, H, D = t.shape
        return KVView(0, t.stride(0), t.stride(1), 16, N, H, D, False)
    if layout == "hnd":
        H, N, D = t.shape
        return KVView(0, t.stride(1), t.stride(0), 16, N, H, D, False)
    raise ValueError(f"unknown kv layout {layout!r}")


# ---------------------------------------------------------------------------
# (a) shared-prefix attention
# ---------------------------------------------------------------------------
def prefix_plan(q_tokens, q_token_offset, kv_start, kv_end, num_qo_heads: int,
                num_kv_heads: int, num_ctas: int):
    """Host-side work plan (d2sd_prefix_plan). Returns (plan int32 numpy array,
    number of partial slots)."""
    lib = load()
    arrs = [np.ascontiguousarray(np.asarray(a, dtype=np.int32)) for a in
            (q_tokens, q_token_offset, kv_start, kv_end)]
    R = len(arrs[0])
    if any(len(a) != R for a in arrs):
        raise ValueError("per-request arrays must have equal length")
    total = int(max((int(o) + int(n) for o, n in zip(arrs[1], arrs[0])), default=0))
    cap = lib.d2sd_prefix_plan_capacity(R, num_qo_heads, num_kv_heads, num_ctas, total)
    if cap < 0:
        raise ValueError("invalid plan sizes")
    plan = np.zeros(cap, dtype=np.int32)
    nslots = np.zeros(1, dtype=np.int32)
    rc = lib.d2sd_prefix_plan(*(a.ctypes.data for a in arrs), R, num_qo_heads, num_kv_heads,
                              num_ctas, plan.ctypes.data, cap, nslots.ctypes.data)
    check(rc, "d2sd_prefix_plan")
    used = int(plan[11]) + int(plan[6])  # H_OFF_TOKENS + H_NUM_TOKENS
    return plan[:used].copy(), int(nslots[0])


def partial_slot_bytes(head_dim: int) -> int:
    return int(load().d2sd_partial_slot_bytes(head_dim))


def prefix_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_layout: str,
                     plan_dev: torch.Tensor, num_ctas: int, partial: torch.Tensor,
                     sm_scale: float, page_table: torch.Tensor | None = None,
                     page_table_offset: torch.Tensor | None = None,
                     status: torch.Tensor | None = None) -> None:
    """Launch kernel (a). q [tokens, Hq, D] bf16; k/v per ``kv_layout``."""
    dev = _require_cuda(q, k, v, plan_dev, partial, page_table, page_table_offset, status)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("prefix attention takes bf16 q/k/v")
    if q.dim() != 3 or q.stride(-1) != 1:
        raise ValueError("q must be [tokens, heads, head_dim] with a contiguous head_dim")
    kvw = kv_view(k, kv_layout)
    vvw = kv_view(v, kv_layout)
    if (kvw.stride_page, kvw.stride_slot, kvw.stride_head) != (vvw.stride_page, vvw.stride_slot,
                                                                 vvw.stride_head):
        raise ValueError("k and v must share a layout")
    if kvw.paged != (page_table is not None):
        raise ValueError("paged layouts need a page table, contiguous ones must not have one")
    N, Hq, D = q.shape
    if D != kvw.head_dim:
        raise ValueError("q and k head_dim differ")
    rc = load().d2sd_prefix_attention(
        q.data_ptr(), q.stride(0), q.stride(1), N, k.data_ptr(), v.data_ptr(), kvw.stride_page,
        kvw.stride_slot, kvw.stride_head, kvw.page_size,
        _lib.KV_UMMA_PAGES if kvw.native else _lib.KV_ROWS, kvw.num_pages, _ptr(page_table),
        _ptr(page_table_offset), Hq, kvw.num_kv_heads, D, float(sm_scale), plan_dev.data_ptr(),
        int(num_ctas), partial.data_ptr(), partial.numel() * partial.element_size(),
        _ptr(status), _stream(dev))
    check(rc, "d2sd_prefix_attention")


# ---------------------------------------------------------------------------
# (b) suffix attention + merge
# ---------------------------------------------------------------------------
def suffix_merge(q: torch.Tensor | None, k_local: torch.Tensor | None,
                 v_local: torch.Tensor | None, out: torch.Tensor, lse: torch.Tensor | None,
                 *, num_blocks: int, block_len: int, num_qo_heads: int, num_kv_heads: int,
                 sm_scale: float, mask_mode: int = _lib.MASK_CAUSAL,
                 custom_mask: torch.Tensor | None = None, partial: torch.Tensor | None = None,
                 plan_dev: torch.Tensor | None = None, prefix_token: torch.Tensor | None = None,
                 prefix_out: torch.Tensor | None = None, prefix_lse: torch.Tensor | None = None,
                 sinks: torch.Tensor | None = None, sink_mode: int = _lib.SINK_NONE,
                 status: torch.Tensor | None = None, exchange=None) -> None:
    """Launch kernel (b). Token-major 3-D views: q/out [tokens, Hq, D],
    k/v_local [tokens, Hk, D], lse/prefix_lse [tokens, Hq]; q may also be a 4-D
    [num_blocks, block_len, Hq, D] view with any block stride (read in place).

    exchange: a ``sharding.PeerExchange``; the merged rows then go into every
    rank's exchange buffer of this call's epoch parity at this rank's head
    offset (``out`` is not written; ``exchange.buffer`` is the result) and the
    launch completes once all ranks' rows are in this rank's buffer. Without a
    ``status`` tensor the exchange's own (``exchange.status``) receives the
    time-out code."""
    dev = _require_cuda(q, k_local, v_local, out, lse, custom_mask, partial, plan_dev,
                        prefix_token, prefix_out, prefix_lse, sinks, status)
    q_sb, q_st, q_sh = 0, 0, 0
    if q is not None and q.dim() == 4:  # [blocks, block_len, Hq, D] with its own block stride
        if q.shape[0] != num_blocks or q.shape[1] != block_len or q.stride(-1) != 1:
            raise ValueError("a 4-D q must be [num_blocks, block_len, heads, head_dim]")
        q_sb, q_st, q_sh = q.stride(0), q.stride(1), q.stride(2)
    elif q is not None:
        q_st, q_sh = q.stride(0), q.stride(1)
    for t in (k_local, v_local, out, prefix_out) + ((q,) if q is not None and q.dim() == 3 else ()):
        if t is not None and (t.dim() != 3 or t.stride(-1) != 1):
            raise ValueError("token tensors must be [tokens, heads, head_dim], head_dim contiguous")
    for t in (lse, prefix_lse):
        if t is not None and (t.dtype != torch.float32 or t.stride(-1) != 1):
            raise ValueError("lse tensors must be fp32 with a contiguous head axis")
    if k_local is not None and (k_local.stride() != v_local.stride()):
        raise ValueError("k_local and v_local must share strides")
    if sinks is not None and (sinks.dtype != torch.float32 or not sinks.is_contiguous()):
        raise ValueError("sinks must be a contiguous fp32 tensor")
    D = out.shape[-1]
    kst = k_local.stride(0) if k_local is not None else 0
    ksh = k_local.stride(1) if k_local is not None else 0
    args = (
        _ptr(q), q_st, q_sh, q_sb,
        _ptr(k_local), _ptr(v_local), kst, ksh, int(num_blocks), int(block_len), int(mask_mode),
        _ptr(custom_mask), _ptr(partial), _ptr(plan_dev), _ptr(prefix_token), _ptr(prefix_out),
        prefix_out.stride(0) if prefix_out is not None else 0,
        prefix_out.stride(1) if prefix_out is not None else 0, _ptr(prefix_lse),
        prefix_lse.stride(0) if prefix_lse is not None else 0, out.data_ptr(), out.stride(0),
        out.stride(1), _ptr(lse), lse.stride(0) if lse is not None else 0, _ptr(sinks),
        int(sink_mode), int(num_qo_heads), int(num_kv_heads), int(D), dtype_code(out),
        float(sm_scale))
    if exchange is None:
        check(load().d2sd_suffix_merge(*args, _ptr(status), _stream(dev)), "d2sd_suffix_merge")
        return
    if exchange.buffers.dtype != out.dtype or exchange.buffers.shape[-1] != D:
        raise ValueError("exchange buffer must match the output dtype and head_dim")
    if exchange.buffers.device != dev:
        raise ValueError("exchange buffers must be on the launch device")
    st = exchange.buffers[0].stride()
    epoch = exchange.epoch + 1
    check(load().d2sd_suffix_merge_gather(
        *args, exchange.out_ptrs.data_ptr(), exchange.counter_ptrs.data_ptr(), exchange.world,
        exchange.rank, int(exchange.head_offset), st[0], st[1], epoch,
        _ptr(status if status is not None else exchange.status), _stream(dev)),
        "d2sd_suffix_merge_gather")
    exchange.next_epoch()  # only a launched call advances the epoch


def cascade_attention_f32(q: torch.Tensor, out: torch.Tensor, lse: torch.Tensor | None, *,
                          num_blocks: int, block_len: int, num_kv_heads: int, sm_scale: float,
                          k_prefix: torch.Tensor | None = None,
                          v_prefix: torch.Tensor | None = None, kv_start: int = 0,
                          k_local: torch.Tensor | None = None, v_local: torch.Tensor | None = None,
                          mask_mode: int = _lib.MASK_CAUSAL,
                          custom_mask: torch.Tensor | None = None,
                          prefix_out: torch.Tensor | None = None,
                          prefix_lse: torch.Tensor | None = None,
                          sinks: torch.Tensor | None = None, sink_mode: int = _lib.SINK_NONE) -> None:
    """fp32 cascade attention (d2sd_cascade_attention_f32). Token-major views:
    q/out [tokens, Hq, D]; k/v_prefix [P, Hk, D] (any token/head strides);
    k/v_local [tokens, Hk, D]; prefix_out [tokens, Hq, D] and prefix_lse
    [tokens, Hq] (base 2) for a dense prefix state; lse [tokens, Hq]."""
    ts = (q, out, k_prefix, v_prefix, k_local, v_local, prefix_out)
    dev = _require_cuda(*ts, lse, custom_mask, prefix_lse, sinks)
    for t in ts + (lse, prefix_lse, sinks):
        if t is not None and (t.dtype != torch.float32 or t.stride(-1) != 1):
            raise ValueError("the fp32 cascade takes fp32 tensors with a contiguous last axis")
    if (k_prefix is None) != (v_prefix is None) or (k_local is None) != (v_local is None):
        raise ValueError("keys and values go together")
    if k_prefix is not None and k_prefix.stride() != v_prefix.stride():
        raise ValueError("k_prefix and v_prefix must share strides")
    if k_local is not None and k_local.stride() != v_local.stride():
        raise ValueError("k_local and v_local must share strides")
    N, Hq, D = q.shape
    P = 0 if k_prefix is None else k_prefix.shape[0]
    st = lambda t, i: t.stride(i) if t is not None else 0  # noqa: E731
    check(load().d2sd_cascade_attention_f32(
        q.data_ptr(), q.stride(0), q.stride(1), _ptr(k_prefix), _ptr(v_prefix), st(k_prefix, 0),
        st(k_prefix, 1), P, int(kv_start), _ptr(k_local), _ptr(v_local), st(k_local, 0),
        st(k_local, 1), int(num_blocks), int(block_len), int(mask_mode), _ptr(custom_mask),
        _ptr(prefix_out), st(prefix_out, 0), st(prefix_out, 1), _ptr(prefix_lse),
        st(prefix_lse, 0), _ptr(sinks), int(sink_mode), out.data_ptr(), out.stride(0),
        out.stride(1), _ptr(lse), st(lse, 0), Hq, int(num_kv_heads), D, float(sm_scale),
        _stream(dev)), "d2sd_cascade_attention_f32")


def merge_state(v: torch.Tensor, s: torch.Tensor, v_other: torch.Tensor,
                s_other: torch.Tensor) -> None:
    """In-place (v, s) <- merge((v, s), (v_other, s_other)); v [n, H, D], s [n, H]."""
    dev = _require_cuda(v, s, v_other, s_other)
    if v.dim() != 3 or v.shape != v_other.shape or s.shape != v.shape[:2] or s_other.shape != s.shape:
        raise ValueError("merge_state: v [n, H, D], s [n, H] with matching shapes")
    if v.stride(-1) != 1 or v_other.stride(-1) != 1 or s.stride(-1) != 1 or s_other.stride(-1) != 1:
        raise ValueError("merge_state: innermost dims must be contiguous")
    if s.dtype != torch.float32 or s_other.dtype != torch.float32 or v.dtype != v_other.dtype:
        raise ValueError("merge_state: fp32 lse and matching value dtypes")
    n, H, D = v.shape
    rc = load().d2sd_merge_state(v.data_ptr(), v.stride(0), v.stride(1), s.data_ptr(), s.stride(0),
                                 v_other.data_ptr(), v_other.stride(0), v_other.stride(1),
                                 s_other.data_ptr(), s_other.stride(0), n, H, D, dtype_code(v),
                                 _stream(dev))
    check(rc, "d2sd_merge_state")


# ---------------------------------------------------------------------------
# (c) acceptance
# ---------------------------------------------------------------------------
def accept_workspace_bytes(num_branches: int, block_len: int, vocab: int) -> int:
    return int(load().d2sd_verify_accept_workspace_size(num_branches, block_len, vocab))


def verify_accept(logits: torch.Tensor, block_ids: torch.Tensor, result: torch.Tensor,
                  accepted_ids: torch.Tensor, workspace: torch.Tensor,
                  argmax_out: torch.Tensor | None = None) -> None:
    """Launch kernel (c). logits [B, T, V] (vocab contiguous), block_ids int64 [B, T],
    result int32 [2], accepted_ids int64 [T], workspace zero-initialised bytes."""
    dev = _require_cuda(logits, block_ids, result, accepted_ids, workspace, argmax_out)
    if logits.dim() != 3 or logits.stride(-1) != 1:
        raise ValueError("logits must be [branches, block, vocab] with a contiguous vocab axis")
    B, T, V = logits.shape
    if block_ids.shape != (B, T) or block_ids.dtype != torch.int64:
        raise ValueError("block_ids must be int64 [branches, block]")
    if result.dtype != torch.int32 or result.numel() < 2:
        raise ValueError("result must be int32 with 2 entries")
    if accepted_ids.dtype != torch.int64 or accepted_ids.numel() < T:
        raise ValueError("accepted_ids must be int64 with block entries")
    rc = load().d2sd_verify_accept(
        logits.data_ptr(), dtype_code(logits), B, T, V, logits.stride(0), logits.stride(1),
        block_ids.data_ptr(), block_ids.stride(0), block_ids.stride(1), result.data_ptr(),
        accepted_ids.data_ptr(), _ptr(argmax_out), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _stream(dev))
    check(rc, "d2sd_verify_accept")


def accept_batch_workspace_bytes(num_requests: int, num_branches: int, block_len: int,
                                 vocab: int) -> int:
    return int(load().d2sd_verify_accept_batch_workspace_size(num_requests, num_branches,
                                                               block_len, vocab))


def _check_batch(logits, block_ids, result, accepted_ids):
    if logits.dim() != 4 or logits.stride(-1) != 1:
        raise ValueError("logits must be [requests, branches, block, vocab], vocab contiguous")
    R, B, T, _ = logits.shape
    if block_ids.shape != (R, B, T) or block_ids.dtype != torch.int64:
        raise ValueError("block_ids must be int64 [requests, branches, block]")
    if result.dtype != torch.int32 or not result.is_contiguous() or result.numel() < 2 * R:
        raise ValueError("result must be contiguous int32 [requests, 2]")
    if (accepted_ids.dtype != torch.int64 or not accepted_ids.is_contiguous()
            or accepted_ids.numel() < R * T):
        raise ValueError("accepted_ids must be contiguous int64 [requests, block]")
    return R, B, T


def verify_accept_batch(logits: torch.Tensor, block_ids: torch.Tensor, result: torch.Tensor,
                        accepted_ids: torch.Tensor, workspace: torch.Tensor,
                        argmax_out: torch.Tensor | None = None) -> None:
    """Kernel (c) over a batch of requests: logits [R, B, T, V], block_ids int64
    [R, B, T], result int32 [R, 2], accepted_ids int64 [R, T]."""
    dev = _require_cuda(logits, block_ids, result, accepted_ids, workspace, argmax_out)
    R, B, T = _check_batch(logits, block_ids, result, accepted_ids)
    V = logits.shape[-1]
    ls, ids = logits.stride(), block_ids.stride()
    check(load().d2sd_verify_accept_batch(
        logits.data_ptr(), dtype_code(logits), R, B, T, V, ls[0], ls[1], ls[2],
        block_ids.data_ptr(), ids[0], ids[1], ids[2], result.data_ptr(), accepted_ids.data_ptr(),
        _ptr(argmax_out), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
        _stream(dev)), "d2sd_verify_accept_batch")


def verify_accept_sharded(logits_slice: torch.Tensor, vocab_offset: int, block_ids: torch.Tensor,
                          result: torch.Tensor, accepted_ids: torch.Tensor,
                          workspace: torch.Tensor, exchange,
                          argmax_out: torch.Tensor | None = None) -> None:
    """Vocabulary-sharded kernel (c): logits_slice [R, B, T, V/world] holds
    columns [vocab_offset, vocab_offset + V/world) of the full vocabulary;
    ``exchange`` is a ``sharding.RecordExchange``. Results as
    verify_accept_batch, identical on every rank."""
    dev = _require_cuda(logits_slice, block_ids, result, accepted_ids, workspace, argmax_out)
    R, B, T = _check_batch(logits_slice, block_ids, result, accepted_ids)
    rows = R * B * T
    if rows > exchange.rows:
        raise ValueError(f"{rows} logits rows exceed the exchange's {exchange.rows}")
    ls, ids = logits_slice.stride(), block_ids.stride()
    epoch = exchange.epoch + 1
    check(load().d2sd_verify_accept_sharded(
        logits_slice.data_ptr(), dtype_code(logits_slice), R, B, T, logits_slice.shape[-1],
        int(vocab_offset), ls[0], ls[1], ls[2], block_ids.data_ptr(), ids[0], ids[1], ids[2],
        result.data_ptr(), accepted_ids.data_ptr(), _ptr(argmax_out), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), exchange.record_ptrs.data_ptr(),
        exchange.control_ptrs.data_ptr(), exchange.world, exchange.rank, epoch,
        exchange.status.data_ptr(), _stream(dev)), "d2sd_verify_accept_sharded")
    exchange.next_epoch()


# ---------------------------------------------------------------------------
# (d) KV commit
# ---------------------------------------------------------------------------
def commit_kv(layer_ptrs: torch.Tensor, *, num_layers: int, num_kv_heads: int, head_dim: int,
              elem_bytes: int, block_len: int, new_strides: tuple[int, int, int],
              cache_strides: tuple[int, int, int], page_size: int,
              page_table: torch.Tensor | None, accept_result: torch.Tensor,
              cache_len_dev: torch.Tensor | None = None, cache_len: int = 0,
              umma_pages: bool = False, hidden_src_ptrs: torch.Tensor | None = None,
              hidden_size: int = 0, hidden_elem_bytes: int = 2,
              hidden_strides: tuple[int, int] = (0, 0),
              hidden_dst: torch.Tensor | None = None) -> None:
    """Launch kernel (d). layer_ptrs: int64 device tensor [L*4] of
    {new_k, new_v, cache_k, cache_v} pointers; strides in elements:
    new (branch, head, token), cache (page, slot, head).

    With hidden_src_ptrs (int64 device tensor of the selected layers' hidden
    state pointers, each [branches, block, hidden_size] with element strides
    hidden_strides = (branch, token)), the same launch also writes
    hidden_dst[t] = cat_j(hidden_j[branch, t]) for t < acc (the draft's
    context feature)."""
    dev = _require_cuda(layer_ptrs, page_table, accept_result, cache_len_dev, hidden_src_ptrs,
                        hidden_dst)
    args = (layer_ptrs.data_ptr(), num_layers, num_kv_heads, head_dim, elem_bytes, block_len,
            *new_strides, *cache_strides, page_size,
            _lib.KV_UMMA_PAGES if umma_pages else _lib.KV_ROWS, _ptr(page_table),
            accept_result.data_ptr(), _ptr(cache_len_dev), int(cache_len))
    if hidden_src_ptrs is None:
        check(load().d2sd_commit_kv(*args, _stream(dev)), "d2sd_commit_kv")
        return
    if hidden_dst is None or hidden_dst.dim() != 2 or hidden_dst.stride(1) != 1:
        raise ValueError("hidden_dst must be [block, num_hidden * hidden_size], rows contiguous")
    check(load().d2sd_commit_kv_hidden(
        *args, hidden_src_ptrs.data_ptr(), int(hidden_src_ptrs.numel()), int(hidden_size),
        int(hidden_elem_bytes), int(hidden_strides[0]), int(hidden_strides[1]),
        hidden_dst.data_ptr(), hidden_dst.stride(0), _stream(dev)), "d2sd_commit_kv_hidden")


def commit_kv_batch(layer_ptrs: torch.Tensor, *, num_layers: int, num_requests: int,
                    num_kv_heads: int, head_dim: int, elem_bytes: int, block_len: int,
                    new_strides: tuple[int, int, int, int], cache_strides: tuple[int, int, int],
                    page_size: int, page_table: torch.Tensor, page_table_offset: torch.Tensor,
                    accept_results: torch.Tensor, cache_lens: torch.Tensor,
                    umma_pages: bool = False) -> None:
    """Kernel (d) for a batch of requests sharing one page pool per layer;
    new_strides = (request, branch, head, token) element strides of each layer's
    new K/V; accept_results int32 [R, 2]; cache_lens int32 [R] on the device."""
    dev = _require_cuda(layer_ptrs, page_table, page_table_offset, accept_results, cache_lens)
    for t, what in ((page_table_offset, "page_table_offset"), (accept_results, "accept_results"),
                    (cache_lens, "cache_lens"), (page_table, "page_table")):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{what} must be a contiguous int32 tensor")
    check(load().d2sd_commit_kv_batch(
        layer_ptrs.data_ptr(), num_layers, num_requests, num_kv_heads, head_dim, elem_bytes,
        block_len, *new_strides, *cache_strides, page_size,
        _lib.KV_UMMA_PAGES if umma_pages else _lib.KV_ROWS, page_table.data_ptr(),
        page_table_offset.data_ptr(), accept_results.data_ptr(), cache_lens.data_ptr(),
        _stream(dev)), "d2sd_commit_kv_batch")


# ---------------------------------------------------------------------------
# QK-norm + RoPE of the block's q and k (the step before (a)/(b))
# ---------------------------------------------------------------------------
def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *,
                 q_weight: torch.Tensor | None = None, k_weight: torch.Tensor | None = None,
                 eps: float = 1e-6, block_len: int | None = None,
                 positions: torch.Tensor | None = None, q_out: torch.Tensor | None = None,
                 k_out: torch.Tensor | None = None):
    """q [tokens, Hq, D], k [tokens, Hk, D] (token-major views, head_dim
    contiguous); cos/sin [positions, D or D/2] in the data dtype; q_weight /
    k_weight the per-head RMSNorm weights [D] (Qwen3) or None (GPT-OSS).
    Tokens are branch-major blocks of block_len tokens (default: all tokens one
    block); token t uses table row positions[t % block_len] (default t % block_len).
    Writes q_out/k_out (default: in place) and returns them."""
    dev = _require_cuda(q, k, cos, sin, q_weight, k_weight, positions, q_out, k_out)
    q_out = q if q_out is None else q_out
    k_out = k if k_out is None else k_out
    for t in (q, k, q_out, k_out):
        if t.dim() != 3 or t.stride(-1) != 1:
            raise ValueError("q/k must be [tokens, heads, head_dim] with head_dim contiguous")
    if q.dtype != k.dtype or cos.dtype != q.dtype or sin.dtype != q.dtype:
        raise ValueError("q, k, cos and sin must share a dtype")
    if cos.stride() != sin.stride() or cos.stride(-1) != 1:
        raise ValueError("cos and sin must share strides, columns contiguous")
    if positions is not None and positions.dtype != torch.int32:
        raise ValueError("positions must be int32")
    n, hq, D = q.shape
    bl = n if block_len is None else int(block_len)
    check(load().d2sd_qk_norm_rope(
        q.data_ptr(), q.stride(0), q.stride(1), q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
        k.data_ptr(), k.stride(0), k.stride(1), k_out.data_ptr(), k_out.stride(0),
        k_out.stride(1), n, hq, k.shape[1], D, dtype_code(q), _ptr(q_weight), _ptr(k_weight),
        float(eps), cos.data_ptr(), sin.data_ptr(), cos.stride(0), bl, _ptr(positions),
        _stream(dev)), "d2sd_qk_norm_rope")
    return q_out, k_out

