"""Numpy restatement of the MoE dispatch bookkeeping (oracle; test infrastructure).

The reference dispatches with a Python loop (agillm41.py:4421-4428)::

    for rank in range(k):
        for e in range(E):
            rows = (idx[:, rank] == e).nonzero()    # ascending token order

so the rows an expert sees are the tokens that picked it, in ascending token
order within each rank. Because a token never picks the same expert twice
(``topk`` indices are distinct), the union over ranks of expert e's rows is a
set of distinct tokens; its canonical order is ascending token index. The
permuted layout that the CUDA path builds is exactly that canonical order,
with each expert's segment padded up to a multiple of the GEMM row tile:

* ``counts[e]``       = number of (token, rank) pairs routed to e
                        (= ``bincount(idx.flatten(), minlength=E)``)
* ``seg_start[e]``    = sum over e' < e of round_up(counts[e'], tile)
* ``row_of[t, r]``    = seg_start[idx[t,r]] + #{t' < t : idx[t', *] == idx[t,r]}
* ``token_of[row]``   = t for every filled row, -1 for padding rows
* ``tile_expert[m]``  = expert owning row tile m (tiles = seg rows / tile)

Only ``tests/`` use this module.
"""
from __future__ import annotations

import numpy as np


def round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def dispatch_layout(idx: np.ndarray, num_experts: int, tile: int = 128):
    """Return (counts, seg_start[E+1], row_of[N,k], token_of[rows], tile_expert)."""
    idx = np.asarray(idx, dtype=np.int64)
    n, k = idx.shape
    counts = np.bincount(idx.reshape(-1), minlength=num_experts).astype(np.int64)
    padded = np.array([round_up(int(c), tile) for c in counts], dtype=np.int64)
    seg_start = np.zeros(num_experts + 1, dtype=np.int64)
    seg_start[1:] = np.cumsum(padded)
    row_of = np.full((n, k), -1, dtype=np.int64)
    token_of = np.full(int(seg_start[-1]), -1, dtype=np.int64)
    fill = seg_start[:-1].copy()
    # Canonical order: ascending token; ranks of one token hit distinct experts.
    for t in range(n):
        for r in range(k):
            e = int(idx[t, r])
            row_of[t, r] = fill[e]
            token_of[fill[e]] = t
            fill[e] += 1
    tile_expert = np.repeat(np.arange(num_experts, dtype=np.int64), padded // tile)
    return counts, seg_start, row_of, token_of, tile_expert


def dispatch_layout_fast(idx: np.ndarray, num_experts: int, tile: int = 128):
    """Vectorised form of :func:`dispatch_layout` for large N (same results)."""
    idx = np.asarray(idx, dtype=np.int64)
    n, k = idx.shape
    counts = np.bincount(idx.reshape(-1), minlength=num_experts).astype(np.int64)
    padded = (counts + tile - 1) // tile * tile
    seg_start = np.zeros(num_experts + 1, dtype=np.int64)
    seg_start[1:] = np.cumsum(padded)
    flat_e = idx.reshape(-1)                       # order: token-major, rank-minor
    order = np.argsort(flat_e, kind="stable")      # stable => ascending (token, rank)
    sorted_e = flat_e[order]
    first = np.searchsorted(sorted_e, np.arange(num_experts), side="left")
    pos_in_seg = np.arange(n * k) - first[sorted_e]
    rows = seg_start[sorted_e] + pos_in_seg
    row_of = np.empty(n * k, dtype=np.int64)
    row_of[order] = rows
    token_of = np.full(int(seg_start[-1]), -1, dtype=np.int64)
    token_of[rows] = order // k
    tile_expert = np.repeat(np.arange(num_experts, dtype=np.int64), padded // tile)
    return counts, seg_start, row_of.reshape(n, k), token_of, tile_expert
