"""Host-side batch planning: the reference's planners, and the packed planner
the B200 path uses.

The reference pads every batch to its longest member, so its planners bound
``inputs x longest`` padded tokens. The library runs packed variable-length
batches (no padding), so ``plan_packed`` bounds the sum of real tokens; after
``longest_first`` this is length bucketing: each batch holds texts of similar
length and texts are never split across batches.
"""
from __future__ import annotations

import heapq
from typing import Sequence

import numpy as np


def longest_first(lengths: Sequence[int]) -> list[int]:
    """Input indices by token length, longest first; ties keep input order.

    crates/inl-sparse/src/native.rs:548-552 and crates/inl-late/src/native.rs:686-690.
    """
    return sorted(range(len(lengths)), key=lambda i: -int(lengths[i]))


def plan_batches(lengths: Sequence[int], batch_size: int, max_batch_tokens: int) -> list[range]:
    """Consecutive batches of at most ``batch_size`` inputs and
    ``max_batch_tokens`` padded tokens (inputs x longest); one input always
    forms a batch. crates/inl-sparse/src/native.rs:557-582 (same rule in
    crates/inl-late/src/native.rs:694-719)."""
    batches: list[range] = []
    start, padded = 0, 0
    for index, length in enumerate(lengths):
        cand_padded = max(padded, max(int(length), 1))
        cand_len = index - start + 1
        if index > start and (cand_len > batch_size or cand_len * cand_padded > max_batch_tokens):
            batches.append(range(start, index))
            start = index
            padded = max(int(length), 1)
        else:
            padded = cand_padded
    if start < len(lengths):
        batches.append(range(start, len(lengths)))
    return batches


def plan_dense_batches(byte_lengths: Sequence[int], batch_size: int, max_length: int, per_row_bytes: int,
                       budget_bytes: int, max_batch_tokens: int, score_rows=lambda padded: 0,
                       slack: int = 8) -> list[range]:
    """The dense planner: contiguous ranges in input order bounded by
    ``batch_size``, attention scratch bytes and padded tokens, where a text's
    token bound is ``min(bytes + slack, max_length)``.
    crates/inl-text/src/native.rs:698-735 (fused attention: score_rows = 0)."""
    def bound(n: int) -> int:
        return min(int(n) + slack, max(max_length, 1))

    batches: list[range] = []
    start, padded = 0, 0
    for index, n in enumerate(byte_lengths):
        cand_padded = max(padded, bound(n))
        cand_len = index - start + 1
        attn = cand_len * per_row_bytes * cand_padded * score_rows(cand_padded)
        tokens = cand_len * cand_padded
        if index > start and (cand_len > batch_size or attn > budget_bytes or tokens > max_batch_tokens):
            batches.append(range(start, index))
            start = index
            padded = bound(n)
        else:
            padded = cand_padded
    if start < len(byte_lengths):
        batches.append(range(start, len(byte_lengths)))
    return batches


def plan_packed(lengths: Sequence[int], max_batch_tokens: int, max_texts: int | None = None) -> list[range]:
    """Consecutive batches whose REAL token sum stays within
    ``max_batch_tokens`` (and at most ``max_texts`` texts); one text always
    forms a batch. Apply to lengths in ``longest_first`` order for length
    bucketing."""
    batches: list[range] = []
    start, tokens = 0, 0
    for index, length in enumerate(lengths):
        n = int(length)
        cand_len = index - start + 1
        if index > start and (tokens + n > max_batch_tokens or (max_texts and cand_len > max_texts)):
            batches.append(range(start, index))
            start, tokens = index, n
        else:
            tokens += n
    if start < len(lengths):
        batches.append(range(start, len(lengths)))
    return batches


def batch_cost(lengths: Sequence[int], causal: bool = True, attn_weight: float = 1.0 / 3000.0) -> float:
    """Relative forward cost of one packed batch: linear layers scale with
    tokens, attention with sum(L^2) (halved when causal)."""
    L = np.asarray(lengths, dtype=np.float64)
    quad = float((L * L).sum()) * (0.5 if causal else 1.0)
    return float(L.sum()) + attn_weight * quad


def assign_lpt(costs: Sequence[float], n_workers: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of batches to workers (GPUs):
    each batch, heaviest first, goes to the least loaded worker."""
    heap = [(0.0, w) for w in range(n_workers)]
    heapq.heapify(heap)
    out: list[list[int]] = [[] for _ in range(n_workers)]
    for b in sorted(range(len(costs)), key=lambda i: -costs[i]):
        load, w = heapq.heappop(heap)
        out[w].append(b)
        heapq.heappush(heap, (load + costs[b], w))
    return out


def pack(token_lists: Sequence[np.ndarray], order: Sequence[int]) -> tuple[np.ndarray, np.ndarray]:
    """Concatenate the texts ``order`` names into (ids uint32 [T], cu int32 [n+1])."""
    lens = np.array([len(token_lists[i]) for i in order], dtype=np.int64)
    cu = np.zeros(len(order) + 1, dtype=np.int32)
    np.cumsum(lens, out=cu[1:])
    ids = (np.concatenate([np.asarray(token_lists[i], dtype=np.uint32) for i in order])
           if len(order) else np.zeros(0, dtype=np.uint32))
    return np.ascontiguousarray(ids, dtype=np.uint32), cu
