"""CPU restatement of greedy acceptance (TEST INFRASTRUCTURE ONLY)."""
from __future__ import annotations

import numpy as np


def _as_np(x):
    if hasattr(x, "detach"):
        x = x.detach().cpu()
        if str(x.dtype) in ("torch.bfloat16", "torch.float16"):
            x = x.float()
        return x.numpy()
    return np.asarray(x)


def argmax_first(row) -> int:
    """torch.argmax over the vocab (model/utils.py:31-32 at temperature 0):
    the first maximal index, NaN counting as maximal (first NaN wins)."""
    return int(np.argmax(row))


def verify_accept(logits, block_ids):
    """Greedy multi-branch acceptance, generation/d3_generator.py:204-225.

    logits [B, T, V], block_ids [B, T] (column 0 is the anchor). The loop, line
    by line: valid_blocks = ones(B) (:205); acceptance_length = 0 (:206); repeat:
    valid_block = first index with valid_blocks > 0 (:209); sample the argmax of
    logits[valid_block, acceptance_length] (:210-211); acceptance_length += 1 and
    keep the token (:212-213); stop when it reaches the block length (:214-215);
    zero every branch whose block token at the new length differs (:216-218);
    stop when none is left (:219-220).
    Returns (acceptance_length, accepted token ids [acceptance_length] with the
    bonus token last, winning branch = valid_block of the last iteration).
    """
    z = _as_np(logits)
    x = _as_np(block_ids).astype(np.int64)
    B, T = x.shape
    valid = np.ones(B, dtype=bool)
    acc = 0
    ids = []
    while True:
        vb = int(np.flatnonzero(valid)[0])
        tok = argmax_first(z[vb, acc])
        acc += 1
        ids.append(tok)
        if acc == T:
            break
        valid &= x[:, acc] == tok
        if not valid.any():
            break
    return acc, np.asarray(ids, dtype=np.int64), vb


def dflash_accept(logits, block_ids):
    """Single-branch acceptance, generation/dflash_generator.py:110-125.

    posterior = argmax(logits) (:110); acceptance_length =
    cumprod(block_ids[:, 1:] == posterior[:, :-1]).sum() (:112-117); the block's
    first acceptance_length+1 tokens are kept and posterior[acceptance_length] is
    the bonus (:119-120); the recorded length is acceptance_length + 1 (:122).
    logits [1, T, V], block_ids [1, T]. Returns (acceptance_length + 1,
    accepted ids [a+1] = block_ids[0, 1:a+1] followed by the bonus, 0).
    """
    z = _as_np(logits)
    x = _as_np(block_ids).astype(np.int64)
    post = np.array([argmax_first(z[0, t]) for t in range(z.shape[1])], dtype=np.int64)
    a = int(np.cumprod(x[0, 1:] == post[:-1]).sum())
    ids = np.concatenate([x[0, 1:a + 1], post[a:a + 1]])
    return a + 1, ids.astype(np.int64), 0
