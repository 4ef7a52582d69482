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

    ``buffers`` [2, tokens, num_qo_heads, head_dim] are this rank's full-width
    outputs, one per epoch parity: call e writes ``buffers[e % 2]`` on every
    rank, rank r's heads at [r*hq, (r+1)*hq); ``output()`` is the buffer of the
    last call. Each rank exports the buffers and an 8-word control block (the
    arrival counters of both parities, a CTA ticket and wait statistics) with
    CUDA IPC (no multicast objects), opens its peers' and keeps device arrays
    of the world's pointers. Every rank must call ``suffix_merge`` with the
    same shapes in the same order, so that the epochs (calls) agree.

    Consumption contract: the output of call e may be read by work enqueued on
    the same stream before call e + 1 (e.g. the layer's o_proj); the peers
    write call e + 2 into the same buffer only after this rank's call e + 1 has
    reached its epilogue. ``status`` (int32, device) receives 3 if a peer did
    not arrive within the kernel's bounded wait; the exchange is then broken.
    ``close()`` unmaps the peers' buffers; call it before the process group is
    destroyed.
    """

    CONTROL_WORDS = 8
    _WAIT_NS, _WAITS, _WAIT_MAX = 3, 4, 5

    def __init__(self, tokens: int, num_qo_heads: int, num_kv_heads: int, head_dim: int, dtype,
                 device, group=None):
        import torch.distributed as dist
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        hq = qo_head_range(num_qo_heads, num_kv_heads, self.world, self.rank)
        self.head_offset = hq[0]
        self.buffers = torch.zeros(2, tokens, num_qo_heads, head_dim, dtype=dtype, device=device)
        self.control = torch.zeros(self.CONTROL_WORDS, dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        handles = export_handles([self.buffers, self.control])
        allh: list = [None] * self.world
        dist.all_gather_object(allh, handles, group=group)
        self._opened: list[int] = []
        buf_ptrs, ctl_ptrs = [], []
        for r, hs in enumerate(allh):
            if r == self.rank:
                buf_ptrs.append(self.buffers.data_ptr())
                ctl_ptrs.append(self.control.data_ptr())
                continue
            ptrs = open_handles(hs, self._opened)
            buf_ptrs.append(ptrs[0])
            ctl_ptrs.append(ptrs[1])
        parity_bytes = self.buffers[0].numel() * self.buffers.element_size()
        outs = [p + par * parity_bytes for par in range(2) for p in buf_ptrs]
        self.out_ptrs = torch.tensor(outs, dtype=torch.int64, device=device)
        self.counter_ptrs = torch.tensor(ctl_ptrs, dtype=torch.int64, device=device)
        self.epoch = 0

    @property
    def buffer(self) -> torch.Tensor:
        """Output of the last call (``buffers[epoch % 2]``)."""
        return self.buffers[self.epoch % 2]

    def output(self, epoch: int | None = None) -> torch.Tensor:
        e = self.epoch if epoch is None else epoch
        return self.buffers[e % 2]

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def wait_stats(self) -> dict:
        """Time the signalling CTA of this rank's calls waited for its peers
        (reads the device; synchronises)."""
        c = self.control.tolist()
        n = max(1, c[self._WAITS])
        return {"waits": c[self._WAITS], "mean_wait_us": c[self._WAIT_NS] / n / 1e3,
                "max_wait_us": c[self._WAIT_MAX] / 1e3}

    def reset_stats(self) -> None:
        self.control[self._WAIT_NS:self._WAIT_MAX + 1].zero_()

    def close(self) -> None:
        from . import _lib
        lib = _lib.load()
        for base in self._opened:
            _lib.check(lib.d2sd_ipc_close(base), "d2sd_ipc_close")
        self._opened = []


def export_handles(tensors) -> list:
    """CUDA IPC handle and byte offset of each tensor's allocation."""
    import ctypes

    from . import _lib
    lib = _lib.load()
    out = []
    for t in tensors:
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_int64(0)
        _lib.check(lib.d2sd_ipc_handle(t.data_ptr(), h, ctypes.byref(off)), "d2sd_ipc_handle")
        out.append((h.raw, off.value))
    return out


def open_handles(handles, opened: list) -> list[int]:
    """Map a peer's exported handles; returns the device pointers and records
    the mapped bases in ``opened`` (to be closed later)."""
    import ctypes

    from . import _lib
    lib = _lib.load()
    ptrs = []
    for raw, off in handles:
        base = ctypes.c_void_p()
        _lib.check(lib.d2sd_ipc_open(raw, ctypes.byref(base)), "d2sd_ipc_open")
        opened.append(base.value)
        ptrs.append(base.value + off)
    return ptrs


class RecordExchange:
    """Peer buffers of the vocabulary-sharded acceptance
    (``ops.verify_accept_sharded``): every rank scans its slice of the
    vocabulary and kernel (c) trades each logits row's (max, first index)
    record with the other ranks over NVLink, so that every rank walks with
    the full-vocabulary argmax while reading only 1/world of the logits.

    ``records`` [2, world, rows, 16 bytes] (one buffer per epoch parity) and an
    8-word control block are exported with CUDA IPC; ``record_ptrs``
    ([parity][rank]) and ``control_ptrs`` are the device arrays the kernel
    takes. All ranks call with the same shapes in the same order. ``status``
    receives 3 if a rank did not arrive within the kernel's bounded wait.
    """

    def __init__(self, rows: int, device, group=None):
        import torch.distributed as dist
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows = int(rows)
        self.records = torch.zeros(2, self.world, self.rows, 4, dtype=torch.int32, device=device)
        self.control = torch.zeros(PeerExchange.CONTROL_WORDS, dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        handles = export_handles([self.records, self.control])
        allh: list = [None] * self.world
        dist.all_gather_object(allh, handles, group=group)
        self._opened: list[int] = []
        rec, ctl = [], []
        for r, hs in enumerate(allh):
            if r == self.rank:
                rec.append(self.records.data_ptr())
                ctl.append(self.control.data_ptr())
                continue
            ptrs = open_handles(hs, self._opened)
            rec.append(ptrs[0])
            ctl.append(ptrs[1])
        parity_bytes = self.records[0].numel() * self.records.element_size()
        self.record_ptrs = torch.tensor([p + par * parity_bytes for par in range(2) for p in rec],
                                        dtype=torch.int64, device=device)
        self.control_ptrs = torch.tensor(ctl, dtype=torch.int64, device=device)
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


def vocab_range(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [start, stop) of the vocabulary rank `rank` scans in the
    sharded acceptance: contiguous, ascending with the rank, the first
    vocab % world ranks one column longer."""
    base, extra = divmod(vocab, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)
