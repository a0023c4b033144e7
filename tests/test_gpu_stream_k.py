"""Stream-K schedule of the weight-streaming kernel on a B200 (NVFP4_FLAG_STREAM_K, opt-in).

Launches of many small groups (non-empty groups averaging at most 64 rows, one K for all
groups, more tiles than SMs) end with the same amount of work on every CTA when the
workspace also holds the split scratch: all but the last full wave of tiles run whole, the
rest are shared out as equal k-iteration ranges, and a tile cut by a range boundary is
computed in two pieces whose fp32 rows are summed by the piece that finishes second. Each case
runs the same group table through the C ABI with the flag twice: with a workspace that has
the split scratch (stream-K) and with one that does not (the flag then falls back to
dynamic tile claims). Both must match the
oracle within the benchmark tolerance, the stream-K result must be bit-identical across
reruns, and at least one cut tile's partial rows must have been written to the scratch.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-2, atol=1e-2)


def _table(pkg, prob):
    t = np.zeros(prob.num_groups, dtype=pkg._native.GROUP_DTYPE)
    t["a"] = [x.data_ptr() for x in prob.a]
    t["b"] = [x.data_ptr() for x in prob.b]
    t["sfa"] = [x.data_ptr() for x in prob.sfa]
    t["sfb"] = [x.data_ptr() for x in prob.sfb]
    t["c"] = [x.data_ptr() for x in prob.c]
    t["m"] = prob.m
    t["n"] = prob.n
    t["k"] = prob.k
    t["alpha"] = prob.alpha
    t["alpha2"] = 1.0
    return t


def _run(pkg, prob, ws):
    for c in prob.c:
        c.fill_(float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    pkg._native.grouped_gemm_raw(_table(pkg, prob), pkg._native.FLAG_STREAM_K, ws.data_ptr(),
                                 ws.numel(), stream)
    assert pkg._native.workspace_check(ws.data_ptr(), stream) == 0
    return [c.clone() for c in prob.c]


def _check_oracle(prob, outs):
    for g in range(prob.num_groups):
        if prob.m[g] == 0:
            continue
        a, b = prob.a[g].cpu().numpy(), prob.b[g].cpu().numpy()
        ref32 = O.ref_gemm_fp32(a, b, prob.sfa_plain[g].cpu().numpy(),
                                prob.sfb_plain[g].cpu().numpy()) * np.float32(prob.alpha[g])
        with np.errstate(over="ignore"):
            exp = ref32.astype(np.float16)
        res = O.compare_fp16(outs[g].cpu().numpy(), exp, ref32, **TOL)
        assert res["ok"], f"{prob.name} group {g} (m={prob.m[g]}): {res}"


def _rows(seed, groups, total, cap):
    """Zipf-like rows per group: many small groups, a few large, some empty."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, groups + 1) ** 1.2
    p /= p.sum()
    rows = np.minimum(rng.multinomial(total, p), cap)
    rng.shuffle(rows)
    return [int(x) for x in rows]


CASES = [
    # name, rows per group, N, K
    ("zipf64_k1024", _rows(1, 64, 4096, 500), 1536, 1024),
    ("zipf64_ragged_n", _rows(2, 64, 3000, 300), 1544, 512),
    ("small_groups_k256", [((7 * g) % 23) for g in range(200)], 768, 256),
    ("tall_and_tiny", [1, 0, 257, 2, 33, 0, 9, 5, 3] * 12, 1280, 768),
]


@pytest.mark.parametrize("name,rows,n,k", CASES, ids=[c[0] for c in CASES])
def test_stream_k_matches_oracle_and_is_deterministic(pkg, name, rows, n, k):
    active = [m for m in rows if m > 0]
    assert sum(active) <= 64 * len(active)  # the weight-streaming kernel's shapes
    prob = pkg.workloads.make_problem(name, rows, n, k, seed=11, device="cuda",
                                      alpha_range=(0.5, 2.0))
    G = prob.num_groups
    plain_bytes = pkg._native.workspace_size(G)
    split_bytes = pkg._native.workspace_size_with_split(G)
    ws_plain = torch.zeros(plain_bytes, dtype=torch.uint8, device="cuda")
    ws_split = torch.zeros(split_bytes, dtype=torch.uint8, device="cuda")

    claims = _run(pkg, prob, ws_plain)
    _check_oracle(prob, claims)
    first = _run(pkg, prob, ws_split)
    _check_oracle(prob, first)
    for _ in range(2):
        again = _run(pkg, prob, ws_split)
        for g, (x, y) in enumerate(zip(first, again)):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16)), f"group {g} changed"
    # The two schedules differ only in how a cut tile's fp32 sum is associated.
    for g in range(G):
        if prob.m[g]:
            d = (first[g].float() - claims[g].float()).abs()
            ok = torch.isfinite(d) | (first[g] == claims[g])
            assert bool(ok.all()), f"group {g}: non-finite difference"
            assert float(d[torch.isfinite(d)].max()) <= 1e-2 * float(claims[g].float().abs().max()) + 1e-2

    # White box: the cut tiles' partial rows live after the split counters.
    partials = (plain_bytes + 255) // 256 * 256 + 4096
    counters = ws_split[(plain_bytes + 255) // 256 * 256:partials].view(torch.int32)
    assert int(counters.abs().sum()) == 0, "stream-K counters must be back at 0"
    # All but the last full wave of tiles are whole; the rest are shared out in ranges of
    # w k-iterations, and a range boundary inside a tile cuts it.
    kt = k // 256
    tiles = sum(math.ceil(m / 128) * math.ceil(n / 256) for m in active)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    full = tiles // sms
    if full >= 1 and tiles % sms:
        w = math.ceil((tiles - (full - 1) * sms) * kt / sms)
        if w % kt:
            assert int(ws_split[partials:].count_nonzero()) > 0, "no cut tile wrote partial rows"
