"""CPU oracle for the MoE dispatch/combine steps -- TEST INFRASTRUCTURE ONLY.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
use this module, and only as a checker or as the timed CPU baseline.

The reference has no MoE layer (its groups arrive already formed); these functions state
the semantics the library's routing and combine kernels implement:

* ``route``: stable counting sort of the (token, slot) pairs by expert, token order inside
  each expert; every expert's rows start on a 128-row boundary.
* ``combine``: out[t] = bf16(sum_j fp32(w[t, j] * y[dest[t, j]])) with each product and each
  partial sum rounded to fp32, slots in order.
"""
from __future__ import annotations

import numpy as np


def route(ids: np.ndarray, num_experts: int):
    ids = np.asarray(ids, dtype=np.int64)
    tokens, topk = ids.shape
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < num_experts)
    counts = np.bincount(flat[valid], minlength=num_experts).astype(np.int32)
    padded = (counts + 127) // 128 * 128
    offsets = np.zeros(num_experts + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(padded)
    dest = np.full(flat.shape, -1, dtype=np.int32)
    src_rows = np.full(int(offsets[-1]), -1, dtype=np.int32)
    fill = offsets[:-1].copy()
    for p in np.flatnonzero(valid):          # token-major order: stable per expert
        e = flat[p]
        dest[p] = fill[e]
        src_rows[fill[e]] = p // topk
        fill[e] += 1
    return counts, offsets.astype(np.int32), dest, src_rows


def fp32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest, ties to even) and return the 16-bit patterns."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def combine(y: np.ndarray, dest: np.ndarray, weights: np.ndarray) -> np.ndarray:
    """bf16 bit patterns [tokens, cols] of the weighted combine (y fp16 [rows, cols])."""
    tokens, topk = weights.shape
    y32 = np.asarray(y, dtype=np.float16).astype(np.float32)
    w = np.asarray(weights, dtype=np.float32)
    d = np.asarray(dest).reshape(tokens, topk)
    acc = np.zeros((tokens, y.shape[1]), dtype=np.float32)
    for j in range(topk):
        ok = d[:, j] >= 0
        prod = (w[:, j:j + 1] * y32[np.where(ok, d[:, j], 0)]).astype(np.float32)
        acc = np.where(ok[:, None], (acc + prod).astype(np.float32), acc)
    return fp32_to_bf16_bits(acc)
