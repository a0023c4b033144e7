"""CPU checks of the owner-side sums oracle (``presum_combine``) that the expert-parallel
block's return_sums / combine_sums kernels are compared against on GPUs: a scalar restatement
of the same arithmetic on small random cases, the owner bookkeeping, and that with one owner
it is the slot-order combine with one extra fp16 rounding."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import nvfp4_ep_oracle as EPO
from oracle import nvfp4_moe_oracle as M


def _case(seed, tokens=7, topk=4, cols=24, world=3):
    rng = np.random.default_rng(seed)
    y = (rng.standard_normal((tokens, topk, cols)) * 4).astype(np.float16)
    w = rng.random((tokens, topk)).astype(np.float32)
    owner = rng.integers(0, world, size=(tokens, topk))
    kept = rng.random((tokens, topk)) > 0.2
    return y, w, owner, kept


def _scalar(y, w, owner, kept, world):
    tokens, topk, cols = y.shape
    out = np.zeros((tokens, cols), dtype=np.uint16)
    part = np.zeros((tokens, world, cols), dtype=np.float16)
    for t in range(tokens):
        for c in range(cols):
            total = np.float32(0)
            for p in range(world):
                acc = np.float32(0)
                hit = False
                for j in range(topk):
                    if kept[t, j] and owner[t, j] == p:
                        acc = np.float32(acc + np.float32(w[t, j] * np.float32(y[t, j, c])))
                        hit = True
                part[t, p, c] = np.float16(acc)
                if hit:
                    total = np.float32(total + np.float32(part[t, p, c]))
            out[t, c] = M.fp32_to_bf16_bits(np.array([total], dtype=np.float32))[0]
    return part, out


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_presum_matches_scalar_restatement(seed):
    y, w, owner, kept = _case(seed)
    part, has, out = EPO.presum_combine(y, kept, owner, w, 3)
    sp, so = _scalar(y, w, owner, kept, 3)
    assert np.array_equal(out, so)
    assert np.array_equal(part[has].view(np.uint16), sp[has].view(np.uint16))
    for t in range(y.shape[0]):
        assert set(np.flatnonzero(has[t])) == set(owner[t][kept[t]].tolist())


def test_one_owner_is_slot_order_combine_with_fp16_partial():
    y, w, _, kept = _case(5, world=1)
    owner = np.zeros(kept.shape, dtype=np.int64)
    _, has, out = EPO.presum_combine(y, kept, owner, w, 1)
    tokens, topk, cols = y.shape
    acc = np.zeros((tokens, cols), dtype=np.float32)
    for j in range(topk):
        prod = (w[:, j:j + 1] * y[:, j].astype(np.float32)).astype(np.float32)
        acc = np.where(kept[:, j:j + 1], (acc + prod).astype(np.float32), acc)
    expect = M.fp32_to_bf16_bits(acc.astype(np.float16).astype(np.float32))
    expect[~has[:, 0]] = 0
    assert np.array_equal(out, expect)
    # A token with no kept pair gets zeros.
    none = ~kept.any(axis=1)
    assert (out[none] == 0).all()
