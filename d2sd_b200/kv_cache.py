"""Paged target KV cache and the accepted-branch commit (kernel (d)).

The reference keeps the target cache in a transformers DynamicCache and, after
every verify step, rebuilds every layer with torch.cat([layer.keys,
new_K[vb, :, :acc]], dim=2) (generation/d3_generator.py:227-232) -- a full
reallocation and copy of the cache, O(L * P) bytes per step. ``PagedKVCache``
holds fixed-capacity page pools instead; ``commit`` moves only the acc accepted
rows of every layer in one launch, reading acc and the winning branch from the
acceptance kernel's device result.

Pool layout per layer: [num_pages, Hk, 16, D], one contiguous 16 x D block per
(page, head). With layout="umma" (the default) each block is stored in the
tensor core's no-swizzle core-matrix order -- [2 groups of 8 rows][D/8 chunks of
8 elements][8 rows][8 elements] -- so kernel (a) moves a page with one bulk copy
and feeds it to tcgen05.mma as it lands, whatever the page table's order. With
layout="hnd" a block holds plain rows (fetched through TMA tensor boxes). Pools
are zero-initialised so every slot past a sequence's length holds finite values.
"""
from __future__ import annotations

import torch

from . import ops


class PagedKVCache:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_tokens: int,
                 page_size: int = 16, dtype: torch.dtype = torch.bfloat16, device="cuda",
                 page_order: torch.Tensor | None = None, layout: str = "umma"):
        if layout not in ("umma", "hnd"):
            raise ValueError("layout must be 'umma' or 'hnd'")
        if layout == "umma" and (page_size != 16 or head_dim % 8 or dtype.itemsize != 2):
            raise ValueError("umma pages hold 16 rows of 16-bit values")
        self.layout = layout
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.page_size = page_size
        self.dtype = dtype
        self.device = torch.device(device)
        self.num_pages = -(-max_tokens // page_size)
        shape = (num_layers, self.num_pages, num_kv_heads, page_size, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        # logical page i of the sequence -> physical page page_table[i]
        if page_order is None:
            page_order = torch.arange(self.num_pages)
        if page_order.numel() != self.num_pages:
            raise ValueError("page_order must list every page once")
        self.page_table = page_order.to(torch.int32).to(self.device)
        self.length = 0
        self._ptr_cache: dict = {}

    # -- views -------------------------------------------------------------
    def layer(self, l: int):
        """(k_pool, v_pool) of layer l, [num_pages, Hk, page_size, D]."""
        return self.k[l], self.v[l]

    @property
    def kv_layout(self) -> str:
        return "paged_umma" if self.layout == "umma" else "paged_hnd"

    def _block_view(self, pool: torch.Tensor) -> torch.Tensor:
        """[L, pages, Hk, 16, D] -> indexable (L, page, head, slot, d) in the
        core-matrix order: [L, pages, Hk, 2, D/8, 8, 8] permuted to
        [L, pages, Hk, 2, 8, D/8, 8] = (row group, row, chunk, element)."""
        L, P, H, S, D = pool.shape
        return pool.view(L, P, H, 2, D // 8, 8, 8).permute(0, 1, 2, 3, 5, 4, 6)

    def positions_to_slots(self, pos: torch.Tensor):
        pt = self.page_table.to(pos.device).long()
        return pt[pos // self.page_size], pos % self.page_size

    # -- host-side set-up (not on the hot path) ------------------------------
    def write(self, l: int, k: torch.Tensor, v: torch.Tensor, start: int = 0) -> None:
        """Write k, v [n, Hk, D] at positions start .. start+n-1 of layer l."""
        n = k.shape[0]
        pos = torch.arange(start, start + n, device=self.device)
        page, slot = self.positions_to_slots(pos)
        if self.layout == "hnd":
            self.k[l, page, :, slot] = k.to(self.dtype)
            self.v[l, page, :, slot] = v.to(self.dtype)
            return
        D = self.head_dim
        for pool, src in ((self.k, k), (self.v, v)):
            blk = self._block_view(pool)[l]  # [pages, Hk, 2, 8, D/8, 8]
            blk[page, :, slot // 8, slot % 8] = src.to(self.dtype).view(n, -1, D // 8, 8)

    def gather(self, l: int, length: int | None = None):
        """Layer l as contiguous [length, Hk, D] tensors (for checks)."""
        n = self.length if length is None else length
        pos = torch.arange(n, device=self.device)
        page, slot = self.positions_to_slots(pos)
        if self.layout == "hnd":
            return self.k[l, page, :, slot], self.v[l, page, :, slot]
        out = []
        for pool in (self.k, self.v):
            blk = self._block_view(pool)[l]
            out.append(blk[page, :, slot // 8, slot % 8].reshape(n, self.num_kv_heads,
                                                                   self.head_dim))
        return out[0], out[1]

    # -- kernel (d) ------------------------------------------------------------
    def _layer_ptrs(self, new_k, new_v):
        key = (tuple(t.data_ptr() for t in new_k), tuple(t.data_ptr() for t in new_v))
        ptrs = self._ptr_cache.get(key)
        if ptrs is None:
            vals = []
            for l in range(self.num_layers):
                vals += [new_k[l].data_ptr(), new_v[l].data_ptr(), self.k[l].data_ptr(),
                         self.v[l].data_ptr()]
            ptrs = torch.tensor(vals, dtype=torch.int64).to(self.device)
            if len(self._ptr_cache) > 16:
                self._ptr_cache.clear()
            self._ptr_cache[key] = ptrs
        return ptrs

    def commit(self, new_k, new_v, accept_result: torch.Tensor, advance_by: int | None = None,
               cache_len: int | None = None, target_hidden=None) -> None:
        """Append block positions 0..acc-1 of the winning branch to every layer.

        new_k/new_v: per-layer [B, Hk, T, D] tensors (a list, or a stacked
        [L, B, Hk, T, D] tensor) with identical strides; accept_result: the
        device int32 {acc, branch} of kernel (c). The rows land at positions
        cache_len (default: self.length) onward. ``advance_by`` (the host copy
        of acc, when the caller has read it) moves self.length forward.

        target_hidden: optional (hidden, out). hidden is the list of the draft's
        selected target layers' hidden states, each [B, T, H] with identical
        strides (generation/d3_generator.py:239 takes hidden_states[id + 1] for
        every id of draft.target_layer_ids); out is [T, len(hidden) * H]. The
        same launch writes out[t] = cat_j(hidden[j][branch, t]) for t < acc,
        the reference's extract_context_feature(...)[branch, :acc].
        """
        if isinstance(new_k, torch.Tensor):
            new_k = [new_k[l] for l in range(new_k.shape[0])]
            new_v = [new_v[l] for l in range(new_v.shape[0])]
        if len(new_k) != self.num_layers or len(new_v) != self.num_layers:
            raise ValueError("one new K/V tensor per layer is required")
        s = new_k[0].stride()
        for t in list(new_k) + list(new_v):
            if t.stride() != s or t.dtype != self.dtype or t.stride(-1) != 1:
                raise ValueError("new K/V tensors must share strides and the cache dtype")
        B, Hk, T, D = new_k[0].shape
        start = self.length if cache_len is None else cache_len
        if start + T > self.num_pages * self.page_size:
            raise ValueError("cache capacity exceeded")
        kl = self.k[0]
        hkw = {}
        if target_hidden is not None:
            hidden, out = target_hidden
            hs = hidden[0].stride()
            for h in hidden:
                if (h.dim() != 3 or h.shape[:2] != (B, T) or h.stride() != hs or h.stride(-1) != 1
                        or h.dtype != out.dtype):
                    raise ValueError("hidden states must be [B, T, H] with identical strides and "
                                     "the output's dtype")
            H = hidden[0].shape[-1]
            if out.shape[0] < T or out.shape[1] != len(hidden) * H:
                raise ValueError("target_hidden output must be [T, len(hidden) * H]")
            key = tuple(h.data_ptr() for h in hidden)
            ptrs = self._ptr_cache.get(("hidden", key))
            if ptrs is None:
                ptrs = torch.tensor(list(key), dtype=torch.int64).to(self.device)
                self._ptr_cache[("hidden", key)] = ptrs
            hkw = dict(hidden_src_ptrs=ptrs, hidden_size=H, hidden_elem_bytes=out.element_size(),
                       hidden_strides=(hs[0], hs[1]), hidden_dst=out)
        ops.commit_kv(self._layer_ptrs(new_k, new_v), num_layers=self.num_layers,
                      num_kv_heads=Hk, head_dim=D, elem_bytes=self.k.element_size(), block_len=T,
                      new_strides=(s[0], s[1], s[2]),
                      cache_strides=(kl.stride(0), kl.stride(2), kl.stride(1)),
                      page_size=self.page_size, page_table=self.page_table,
                      accept_result=accept_result, cache_len=start,
                      umma_pages=self.layout == "umma", **hkw)
        if advance_by is not None:
            self.length = start + int(advance_by)


class PagedKVPool(PagedKVCache):
    """Paged target caches of many sequences in one pool per layer (batched
    serving: each request of the batch is one sequence).

    Sequence s owns the pages page_table[page_offsets[s] : page_offsets[s] +
    pages_of(s)], so its position p lives in page page_table[page_offsets[s] +
    p // 16] -- the per-request page-table offset kernel (a) and the batched
    commit take. ``lengths_dev`` (int32, device) holds every sequence's cache
    length for the batched commit, which appends each request's accepted rows
    in one launch (``commit_batch``).
    """

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, capacities,
                 page_size: int = 16, dtype: torch.dtype = torch.bfloat16, device="cuda",
                 shuffle_seed: int | None = None, layout: str = "umma"):
        caps = [int(c) for c in capacities]
        pages = [-(-c // page_size) for c in caps]
        offsets, cur = [], 0
        for n in pages:
            offsets.append(cur)
            cur += n
        order = (torch.randperm(max(cur, 1), generator=torch.Generator().manual_seed(shuffle_seed))
                 if shuffle_seed is not None else torch.arange(max(cur, 1)))
        super().__init__(num_layers, num_kv_heads, head_dim, max(cur, 1) * page_size, page_size,
                         dtype, device, page_order=order, layout=layout)
        self.capacities = caps
        self.page_offsets_host = offsets
        self.page_offsets = torch.tensor(offsets, dtype=torch.int32, device=self.device)
        self.lengths = [0] * len(caps)
        self.lengths_dev = torch.zeros(len(caps), dtype=torch.int32, device=self.device)

    @property
    def num_seqs(self) -> int:
        return len(self.capacities)

    def set_lengths(self, lengths) -> None:
        self.lengths = [int(x) for x in lengths]
        self.lengths_dev.copy_(torch.tensor(self.lengths, dtype=torch.int32))

    def write_seq(self, l: int, s: int, k: torch.Tensor, v: torch.Tensor, start: int = 0) -> None:
        """Write k, v [n, Hk, D] at positions start.. of sequence s, layer l."""
        if start + k.shape[0] > self.capacities[s]:
            raise ValueError("sequence capacity exceeded")
        self.write(l, k, v, start=self.page_offsets_host[s] * self.page_size + start)

    def gather_seq(self, l: int, s: int, length: int):
        """Sequence s of layer l as contiguous [length, Hk, D] tensors (for checks)."""
        base = self.page_offsets_host[s] * self.page_size
        pos = torch.arange(base, base + length, device=self.device)
        page, slot = self.positions_to_slots(pos)
        if self.layout == "hnd":
            return self.k[l, page, :, slot], self.v[l, page, :, slot]
        out = []
        for pool in (self.k, self.v):
            blk = self._block_view(pool)[l]
            out.append(blk[page, :, slot // 8, slot % 8].reshape(length, self.num_kv_heads,
                                                                   self.head_dim))
        return out[0], out[1]

    def commit_batch(self, new_k, new_v, accept_results: torch.Tensor, num_branches: int) -> None:
        """Append every sequence's accepted rows (kernel (d), one launch).

        new_k/new_v: per-layer [S * num_branches, Hk, T, D] tensors (request s,
        branch b at row s * num_branches + b; a list or a stacked [L, ...]
        tensor) with identical strides; accept_results: int32 [S, 2] from
        ``BatchVerifier``. Rows land at each sequence's ``lengths_dev`` onward;
        the lengths are not advanced (the caller reads acc when it needs it)."""
        if isinstance(new_k, torch.Tensor):
            new_k = [new_k[l] for l in range(new_k.shape[0])]
            new_v = [new_v[l] for l in range(new_v.shape[0])]
        if len(new_k) != self.num_layers or len(new_v) != self.num_layers:
            raise ValueError("one new K/V tensor per layer is required")
        s = new_k[0].stride()
        for t in list(new_k) + list(new_v):
            if t.stride() != s or t.dtype != self.dtype or t.stride(-1) != 1:
                raise ValueError("new K/V tensors must share strides and the cache dtype")
        RB, Hk, T, D = new_k[0].shape
        if RB != self.num_seqs * num_branches:
            raise ValueError("new K/V rows must be sequences x branches")
        kl = self.k[0]
        ops.commit_kv_batch(self._layer_ptrs(new_k, new_v), num_layers=self.num_layers,
                            num_requests=self.num_seqs, num_kv_heads=Hk, head_dim=D,
                            elem_bytes=self.k.element_size(), block_len=T,
                            new_strides=(num_branches * s[0], s[0], s[1], s[2]),
                            cache_strides=(kl.stride(0), kl.stride(2), kl.stride(1)),
                            page_size=self.page_size, page_table=self.page_table,
                            page_table_offset=self.page_offsets, accept_results=accept_results,
                            cache_lens=self.lengths_dev, umma_pages=self.layout == "umma")
