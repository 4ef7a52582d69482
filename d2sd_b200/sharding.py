"""Work partitioning across the GPUs of one node.

The reference parallelises only over dataset samples (benchmark.py:162,
distributed.py:54-71: each rank a full replica, results gathered as Python
objects). The verify path adds two partitions:

* KV-head sharding (long single requests, BASELINE configs 3 and 5): rank r owns
  kv heads [r*Hk/N, (r+1)*Hk/N) of every layer, the G query heads of each, and
  those heads' pages of the prefix cache. Kernels (a), (b) and the commit (d)
  run on local data only; the one exchange is an all-gather of the attention
  output [tokens, Hq/N, D] per layer over NCCL (NVLink), after which every rank
  holds [tokens, Hq, D] for o_proj. Acceptance (c) runs on every rank over the
  replicated logits, so no rank waits for another to learn acc/branch.
* Request parallelism (batched serving, config 4): requests are independent;
  they are assigned to ranks by longest-processing-time-first on their cost
  (prefix length x query tokens) and never exchange data.
"""
from __future__ import annotations

import heapq
from typing import Callable, Sequence

import torch


def kv_head_range(num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """The kv heads [start, stop) rank `rank` owns."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not divide over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def qo_head_range(num_qo_heads: int, num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Query heads served by the rank's kv heads (head h reads kv head h // G)."""
    g = num_qo_heads // num_kv_heads
    s, e = kv_head_range(num_kv_heads, world, rank)
    return s * g, e * g


def lpt_partition(costs: Sequence[float], world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of items to `world` bins.
    Deterministic: ties broken by item index, then by bin index."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, b) for b in range(world)]
    bins: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, b = heapq.heappop(heap)
        bins[b].append(i)
        heapq.heappush(heap, (load + float(costs[i]), b))
    return [sorted(b) for b in bins]


def request_costs(prefix_lens: Sequence[int], q_tokens: Sequence[int]) -> list[float]:
    """Cost model of a request for kernel (a): prefix keys x query tokens, plus
    a per-request constant for the suffix/acceptance/commit work."""
    return [float(p) * q + 64.0 * q for p, q in zip(prefix_lens, q_tokens)]


def assemble_heads(gathered: torch.Tensor) -> torch.Tensor:
    """[world, tokens, H/world, D] from all_gather -> [tokens, H, D] with rank
    r's heads at [r*H/world, (r+1)*H/world)."""
    w, n, h, d = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(n, w * h, d)


class KVHeadShardedAttention:
    """Per-layer driver of KV-head-sharded cascade attention on one rank.

    ``compute(q_local, k_new_local, v_new_local, layer) -> out [tokens, hq, D]``
    runs the local attention (by default the d2sd kernels, see bench.py and
    cascade.py); ``forward`` all-gathers the local outputs into a preallocated
    [world * tokens, hq, D] buffer with NCCL's all_gather_into_tensor and returns
    the [tokens, Hq, D] assembled view. The buffers are allocated once, so the
    collective is CUDA-graph capturable.
    """

    def __init__(self, group, num_qo_heads: int, num_kv_heads: int, head_dim: int,
                 tokens: int, dtype: torch.dtype, device,
                 compute: Callable[..., torch.Tensor]):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.hk = kv_head_range(num_kv_heads, self.world, self.rank)
        self.hq = qo_head_range(num_qo_heads, num_kv_heads, self.world, self.rank)
        nq = self.hq[1] - self.hq[0]
        # [world * tokens, hq, D]: rank r's block at rows [r*tokens, (r+1)*tokens)
        self.gathered = torch.empty(self.world * tokens, nq, head_dim, dtype=dtype, device=device)
        self.tokens = tokens
        self.compute = compute

    def local_slices(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor):
        """Take this rank's heads of full-width tensors [tokens, H, D]."""
        return (q[:, self.hq[0]:self.hq[1]], k_new[:, self.hk[0]:self.hk[1]],
                v_new[:, self.hk[0]:self.hk[1]])

    def forward(self, q_local, k_local, v_local, layer: int) -> torch.Tensor:
        import torch.distributed as dist
        out = self.compute(q_local, k_local, v_local, layer)
        dist.all_gather_into_tensor(self.gathered, out.contiguous(), group=self.group)
        return assemble_heads(self.gathered.view(self.world, self.tokens, *self.gathered.shape[1:]))


class PeerExchange:
    """The all-gather of head-sharded attention outputs done by kernel (b)'s own
    stores over NVLink (``ops.suffix_merge(..., exchange=...)``), in place of
    ``all_gather_into_tensor`` after it.

    ``buffer`` [tokens, num_qo_heads, head_dim] is this rank's full-width
    output: rank r's heads land at [r*hq, (r+1)*hq). Each rank exports the
    buffer and a uint64 arrival counter with CUDA IPC (no multicast objects),
    opens its peers' and keeps device arrays of the world's pointers. Every
    rank must call ``suffix_merge`` with the same shapes in the same order, so
    that the epochs (calls) agree. ``close()`` unmaps the peers' buffers; call
    it before the process group is destroyed.
    """

    def __init__(self, tokens: int, num_qo_heads: int, num_kv_heads: int, head_dim: int, dtype,
                 device, group=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib
        lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        hq = qo_head_range(num_qo_heads, num_kv_heads, self.world, self.rank)
        self.head_offset = hq[0]
        self.buffer = torch.zeros(tokens, num_qo_heads, head_dim, dtype=dtype, device=device)
        self.counter = torch.zeros(1, dtype=torch.int64, device=device)
        mine = []
        for t in (self.buffer, self.counter):
            h = ctypes.create_string_buffer(64)
            off = ctypes.c_int64(0)
            _lib.check(lib.d2sd_ipc_handle(t.data_ptr(), h, ctypes.byref(off)), "d2sd_ipc_handle")
            mine.append((h.raw, off.value))
        allh: list = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        outs, ctrs = [], []
        for r, handles in enumerate(allh):
            if r == self.rank:
                outs.append(self.buffer.data_ptr())
                ctrs.append(self.counter.data_ptr())
                continue
            ptrs = []
            for raw, off in handles:
                base = ctypes.c_void_p()
                _lib.check(lib.d2sd_ipc_open(raw, ctypes.byref(base)), "d2sd_ipc_open")
                self._opened.append(base.value)
                ptrs.append(base.value + off)
            outs.append(ptrs[0])
            ctrs.append(ptrs[1])
        self.out_ptrs = torch.tensor(outs, dtype=torch.int64, device=device)
        self.counter_ptrs = torch.tensor(ctrs, dtype=torch.int64, device=device)
        self.epoch = 0

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def close(self) -> None:
        from . import _lib
        lib = _lib.load()
        for base in self._opened:
            _lib.check(lib.d2sd_ipc_close(base), "d2sd_ipc_close")
        self._opened = []

