"""Greedy branch acceptance on the GPU (kernel (c)).

``verify(logits, block_ids)`` returns what the acceptance walk of
generation/d3_generator.py:204-225 produces -- (acceptance_length including
the bonus token, the accepted token ids with the bonus last, the winning
branch) -- from one kernel launch and a single device-to-host read, instead of
up to block_len iterations each with a full-vocab softmax and two host syncs.
``Verifier`` keeps the device buffers so a decode loop can launch without
allocating and read the result only when it needs it; the KV commit consumes
the device result directly.
"""
from __future__ import annotations

import torch

from . import ops


class Verifier:
    """Device buffers of kernel (c) for fixed (branches, block_len, vocab)."""

    def __init__(self, num_branches: int, block_len: int, vocab: int, device):
        self.shape = (num_branches, block_len, vocab)
        self.device = torch.device(device)
        nbytes = ops.accept_workspace_bytes(num_branches, block_len, vocab)
        # the kernel leaves the workspace zeroed; zero it once here
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self.result = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.accepted = torch.zeros(block_len, dtype=torch.int64, device=self.device)
        self.argmax = torch.zeros(num_branches * block_len, dtype=torch.int64, device=self.device)

    def launch(self, logits: torch.Tensor, block_ids: torch.Tensor) -> None:
        """Enqueue kernel (c); results stay on the device (self.result,
        self.accepted, self.argmax)."""
        if tuple(logits.shape) != self.shape:
            raise ValueError(f"logits shape {tuple(logits.shape)} != {self.shape}")
        if logits.stride(-1) != 1:
            logits = logits.contiguous()
        ops.verify_accept(logits, block_ids, self.result, self.accepted, self.workspace,
                          self.argmax)

    def read(self):
        """(acceptance_length, accepted ids [acc] on the device, branch); syncs."""
        acc, branch = (int(x) for x in self.result.tolist())
        return acc, self.accepted[:acc], branch


class BatchVerifier:
    """Device buffers of kernel (c) for a batch of R requests of fixed
    (branches, block_len, vocab): one launch verifies every request
    (batched serving); results stay on the device."""

    def __init__(self, num_requests: int, num_branches: int, block_len: int, vocab: int, device):
        self.shape = (num_requests, num_branches, block_len, vocab)
        self.device = torch.device(device)
        nbytes = ops.accept_batch_workspace_bytes(num_requests, num_branches, block_len, vocab)
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self.result = torch.zeros(num_requests, 2, dtype=torch.int32, device=self.device)
        self.accepted = torch.zeros(num_requests, block_len, dtype=torch.int64, device=self.device)

    def launch(self, logits: torch.Tensor, block_ids: torch.Tensor,
               argmax_out: torch.Tensor | None = None) -> None:
        if tuple(logits.shape) != self.shape:
            raise ValueError(f"logits shape {tuple(logits.shape)} != {self.shape}")
        ops.verify_accept_batch(logits, block_ids, self.result, self.accepted, self.workspace,
                                argmax_out)


class ShardedVerifier:
    """Vocabulary-sharded kernel (c) on one rank of a KV-head-sharded group:
    this rank holds columns ``vocab_range`` of the logits; the kernel trades
    the rows' bests with the other ranks over NVLink (``RecordExchange``) and
    every rank ends with the same acceptance results."""

    def __init__(self, num_requests: int, num_branches: int, block_len: int, vocab: int, device,
                 group=None):
        from .sharding import RecordExchange, vocab_range
        self.device = torch.device(device)
        self.exchange = RecordExchange(num_requests * num_branches * block_len, self.device, group)
        self.vocab = vocab
        self.columns = vocab_range(vocab, self.exchange.world, self.exchange.rank)
        width = self.columns[1] - self.columns[0]
        self.shape = (num_requests, num_branches, block_len, width)
        nbytes = ops.accept_batch_workspace_bytes(num_requests, num_branches, block_len, width)
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self.result = torch.zeros(num_requests, 2, dtype=torch.int32, device=self.device)
        self.accepted = torch.zeros(num_requests, block_len, dtype=torch.int64, device=self.device)

    @property
    def status(self) -> torch.Tensor:
        return self.exchange.status

    def launch(self, logits_slice: torch.Tensor, block_ids: torch.Tensor,
               argmax_out: torch.Tensor | None = None) -> None:
        """logits_slice [R, B, T, V/world]: this rank's columns of the logits."""
        if tuple(logits_slice.shape) != self.shape:
            raise ValueError(f"logits slice shape {tuple(logits_slice.shape)} != {self.shape}")
        ops.verify_accept_sharded(logits_slice, self.columns[0], block_ids, self.result,
                                  self.accepted, self.workspace, self.exchange, argmax_out)

    def close(self) -> None:
        self.exchange.close()


_verifiers: dict = {}


def verify(logits: torch.Tensor, block_ids: torch.Tensor, temperature: float = 0.0):
    """Greedy acceptance of `block_ids` [B, T] (int64, column 0 = anchor) under
    target `logits` [B, T, V] (fp32/bf16/fp16).

    Returns (acceptance_length, accepted_ids [acceptance_length] int64 on the
    device, branch). temperature >= 1e-5 is the reference's multinomial path
    (model/utils.py:33-35), which is RNG-dependent and not part of this kernel.
    """
    if temperature >= 1e-5:
        raise NotImplementedError("only greedy (temperature < 1e-5) acceptance is implemented")
    if logits.dim() == 2:  # [T, V] single branch
        logits = logits.unsqueeze(0)
    if block_ids.dim() == 1:
        block_ids = block_ids.unsqueeze(0)
    key = (tuple(logits.shape), str(logits.device))
    ver = _verifiers.get(key)
    if ver is None:
        ver = Verifier(*logits.shape, logits.device)
        _verifiers[key] = ver
    ver.launch(logits, block_ids.to(torch.int64))
    acc, ids, branch = ver.read()
    return acc, ids.clone(), branch
