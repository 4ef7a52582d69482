"""CPU restatement of the accepted-branch KV commit (TEST INFRASTRUCTURE ONLY)."""
from __future__ import annotations

import numpy as np


def commit_contiguous(cache_k, cache_v, new_kv, branch: int, acc: int):
    """generation/d3_generator.py:227-232.

    For every layer: layer.keys = cat([layer.keys, new_K[branch:branch+1, :, :acc]],
    dim=2), the same for the values. cache_k/cache_v: lists of [1, Hk, P, D];
    new_kv: list of (K, V) with K, V [B, Hk, T, D]. Returns the new lists.
    """
    out_k, out_v = [], []
    for ck, cv, (nk, nv) in zip(cache_k, cache_v, new_kv):
        out_k.append(np.concatenate([ck, nk[branch:branch + 1, :, :acc]], axis=2))
        out_v.append(np.concatenate([cv, nv[branch:branch + 1, :, :acc]], axis=2))
    return out_k, out_v


def commit_paged(pool_k, pool_v, page_table, cache_len: int, new_k, new_v, branch: int,
                 acc: int, layout: str = "HND"):
    """The same commit into a paged pool, in place.

    Cache position p of head h lives in page page_table[p // page_size], slot
    p % page_size; layout "HND" pools are [pages, Hk, page_size, D], "NHD" pools
    [pages, page_size, Hk, D]. Block positions 0..acc-1 of `branch` go to cache
    positions cache_len .. cache_len+acc-1 (the same rows the contiguous form
    appends).
    """
    ps = pool_k.shape[2] if layout == "HND" else pool_k.shape[1]
    for t in range(acc):
        pos = cache_len + t
        page = int(page_table[pos // ps])
        slot = pos % ps
        if layout == "HND":
            pool_k[page, :, slot] = new_k[branch, :, t]
            pool_v[page, :, slot] = new_v[branch, :, t]
        else:
            pool_k[page, slot] = new_k[branch, :, t]
            pool_v[page, slot] = new_v[branch, :, t]
    return pool_k, pool_v


def context_feature(hidden_states, layer_ids, branch: int, acc: int):
    """generation/d3_generator.py:239 with model/utils.py:17-26.

    extract_context_feature concatenates hidden_states[id + 1] (the +1 skips
    the embedding output) of every selected layer id along the last axis; the
    generator keeps the winning branch's first acc rows:
    [acc, len(layer_ids) * H] (the reference adds a leading unit axis).
    """
    sel = [hidden_states[i + 1] for i in layer_ids]
    return np.concatenate(sel, axis=-1)[branch, :acc]
