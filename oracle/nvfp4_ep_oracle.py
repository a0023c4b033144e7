"""CPU oracle for the expert-parallel exchange -- TEST INFRASTRUCTURE ONLY.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may use
this module, and only as a checker.

The reference is single-GPU and has no expert-parallel path; these functions state the
placement rule the library's exchange kernels (nvfp4_ep_layout / nvfp4_ep_dispatch)
implement, and ``place_pairs`` restates it a second, independent way (pair by pair) so the
two can be checked against each other:

* rank p owns experts [p * E / P, (p + 1) * E / P);
* in an owner's receive slab its experts' segments follow expert order, each starting on a
  128-row boundary; inside expert e's segment come the pairs from rank 0, then rank 1, ...,
  each rank's pairs in its local dispatched (token) order;
* a segment that does not fit the slab is dropped on every rank.
"""
from __future__ import annotations

import numpy as np

from . import nvfp4_moe_oracle as M


def ep_layout(mat: np.ndarray, world: int, rank: int, capacity: int):
    """mat [world, E] pairs per (source rank, expert). Returns (seg_offsets [E/world],
    seg_counts [E/world]) of `rank` as owner, send_base [E] of `rank` as source (-1 when
    dropped), and whether any segment was dropped."""
    mat = np.asarray(mat, dtype=np.int64)
    E = mat.shape[1]
    epr = E // world
    total = mat.sum(axis=0)
    start = np.zeros(E, dtype=np.int64)
    for p in range(world):
        acc = 0
        for l in range(epr):
            e = p * epr + l
            start[e] = acc
            acc += (total[e] + 127) // 128 * 128
    fits = start + total <= capacity
    before = mat[:rank].sum(axis=0)
    send_base = np.where(fits, start + before, -1).astype(np.int32)
    own = slice(rank * epr, (rank + 1) * epr)
    seg_offsets = np.where(fits[own], start[own], 0).astype(np.int32)
    seg_counts = np.where(fits[own], total[own], 0).astype(np.int32)
    return seg_offsets, seg_counts, send_base, bool((~fits).any())


def place_pairs(ids_per_rank, num_experts: int, world: int, capacity: int):
    """Pair-by-pair placement: for every rank q, remote_rows [tokens_q * topk] (row in the
    owner's slab, -1 if dropped), and for every owner p a dict row -> (q, token)."""
    epr = num_experts // world
    routes = [M.route(np.asarray(ids), num_experts) for ids in ids_per_rank]
    counts = np.stack([r[0] for r in routes])  # [world, E]
    total = counts.sum(axis=0)
    next_row = {}
    for p in range(world):
        acc = 0
        for l in range(epr):
            e = p * epr + l
            seg_end = acc + total[e]
            next_row[e] = acc if seg_end <= capacity else None
            acc += (total[e] + 127) // 128 * 128
    remote = []
    received = [dict() for _ in range(world)]
    for q in range(world):
        ids = np.asarray(ids_per_rank[q], dtype=np.int64)
        _, offsets, dest, _ = routes[q]
        flat = ids.reshape(-1)
        rows = np.full(flat.shape, -1, dtype=np.int64)
        # Walk this rank's pairs in its dispatched order (expert, then token).
        order = np.argsort(np.where(dest >= 0, dest, np.iinfo(np.int64).max), kind="stable")
        for i in order:
            e, d = int(flat[i]), int(dest[i])
            if d < 0 or next_row[e] is None:
                continue
            rows[i] = next_row[e]
            received[e // epr][next_row[e]] = (q, int(i // ids.shape[1]))
            next_row[e] += 1
        remote.append(rows.astype(np.int32))
    return counts.astype(np.int32), remote, received


def presum_combine(y_pairs: np.ndarray, kept: np.ndarray, owner: np.ndarray,
                   weights: np.ndarray, world: int):
    """Owner-side sums followed by the per-owner combine (nvfp4_ep_return_sums +
    nvfp4_ep_combine_sums). y_pairs fp16 [tokens, topk, cols]: each pair's down-GEMM row;
    kept [tokens, topk]: pairs that reached their owner; owner [tokens, topk]: the rank owning
    the pair's expert; weights fp32 [tokens, topk].

    partial[t, p] = fp16(sum_j w[t, j] * y[t, j]) over t's kept pairs owned by p, slots in
    order, each product and each sum rounded to fp32 (the slot-order combine's arithmetic);
    out[t] = bf16(sum_p fp32(partial[t, p])) over the owners p (ascending) holding at least
    one kept pair of t. Returns (partial fp16 [tokens, world, cols], has [tokens, world],
    out bf16 bit patterns [tokens, cols])."""
    y32 = np.asarray(y_pairs, dtype=np.float16).astype(np.float32)
    tokens, topk, cols = y32.shape
    w = np.asarray(weights, dtype=np.float32)
    kept = np.asarray(kept, dtype=bool)
    owner = np.asarray(owner)
    partial = np.zeros((tokens, world, cols), dtype=np.float16)
    has = np.zeros((tokens, world), dtype=bool)
    for p in range(world):
        acc = np.zeros((tokens, cols), dtype=np.float32)
        for j in range(topk):
            ok = kept[:, j] & (owner[:, j] == p)
            prod = (w[:, j:j + 1] * y32[:, j]).astype(np.float32)
            acc = np.where(ok[:, None], (acc + prod).astype(np.float32), acc)
            has[:, p] |= ok
        partial[:, p] = acc.astype(np.float16)
    out = np.zeros((tokens, cols), dtype=np.float32)
    for p in range(world):
        out = np.where(has[:, p:p + 1], (out + partial[:, p].astype(np.float32)).astype(np.float32),
                       out)
    return partial, has, M.fp32_to_bf16_bits(out)
