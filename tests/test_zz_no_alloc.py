"""The allocation-free entry point (nvfp4_grouped_gemm_noalloc) against the regular one.

Callers that cannot allocate device memory (pool-owning frameworks, plugins
handed only their buffers, latency-critical paths) use the variant whose scratch
lives in an array compiled into the library. This file is collected last so that
a failure here never hides the other tests; it passes both on its own in a fresh
process and after the rest of the suite.
"""
from __future__ import annotations


import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-2, atol=1e-2)


def _table(pkg, prob):
    N = pkg._native
    t = np.zeros(prob.num_groups, dtype=N.GROUP_DTYPE)
    t["a"] = [x.data_ptr() for x in prob.a]
    t["b"] = [x.data_ptr() for x in prob.b]
    t["sfa"] = [x.data_ptr() for x in prob.sfa]
    t["sfb"] = [x.data_ptr() for x in prob.sfb]
    t["c"] = [x.data_ptr() for x in prob.c]
    if prob.gated:
        t["b2"] = [x.data_ptr() for x in prob.b2]
        t["sfb2"] = [x.data_ptr() for x in prob.sfb2]
    t["m"] = prob.m
    t["n"] = prob.n
    t["k"] = prob.k
    t["alpha"] = prob.alpha
    t["alpha2"] = prob.alpha2 if prob.gated else 1.0
    return t


def _run_regular(pkg, prob):
    pkg.grouped_gemm(prob.a, prob.b, prob.sfa, prob.sfb, prob.c, prob.problem_sizes(),
                     alpha=prob.alpha, b2=prob.b2, sfb2=prob.sfb2, alpha2=prob.alpha2)
    torch.cuda.synchronize()
    return [c.clone() for c in prob.c]


def _run_noalloc(pkg, prob, flags=0):
    lib = pkg.load_library()
    t = _table(pkg, prob)
    for c in prob.c:
        c.fill_(float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.nvfp4_grouped_gemm_noalloc(t.ctypes.data, prob.num_groups,
                                        flags | (pkg._native.FLAG_GATED if prob.gated else 0),
                                        stream)
    pkg._native.check(st, lib)
    torch.cuda.synchronize()
    return [c.clone() for c in prob.c]


def _compare(regular, noalloc, prob):
    for g, (r, z) in enumerate(zip(regular, noalloc)):
        if prob.m[g] == 0:
            continue
        res = O.compare_fp16(z.cpu().numpy(), r.cpu().numpy(), None, **TOL)
        assert res["ok"], f"group {g}: {res}"


def test_noalloc_matches_regular_entry_point_two_calls(pkg):
    # Two consecutive calls with different group tables share the built-in scratch.
    first = pkg.workloads.make_problem("na1", [128, 0, 77, 300], 256, 512, seed=31,
                                       device="cuda", alpha_range=(0.5, 2.0))
    second = pkg.workloads.make_problem("na2", [64, 200], 384, 768, gated=True, seed=32,
                                        device="cuda", alpha_range=(0.5, 2.0))
    for prob in (first, second):
        regular = _run_regular(pkg, prob)
        noalloc = _run_noalloc(pkg, prob)
        _compare(regular, noalloc, prob)


def test_noalloc_rejects_more_groups_than_its_scratch_holds(pkg):
    lib = pkg.load_library()
    G = pkg._native.NOALLOC_MAX_GROUPS + 1
    t = np.zeros(G, dtype=pkg._native.GROUP_DTYPE)
    st = lib.nvfp4_grouped_gemm_noalloc(t.ctypes.data, G, 0, None)
    assert st == pkg._native.ERR_INVALID_ARGUMENT
    assert b"exceeds" in lib.nvfp4_last_error_detail()
