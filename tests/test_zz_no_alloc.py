"""The allocation-free entry point (nvfp4_grouped_gemm_noalloc) through the C ABI.

Some callers cannot allocate device memory where they run the GEMM: frameworks whose
device memory is all owned by their own pool allocator, plugins that a host
application hands only their input and output buffers, and latency-critical paths that
cannot pay for cudaMalloc's implicit synchronisation. They call the variant whose
scratch (group records, tensor maps, device error word) lives in an array compiled
into the library. These tests check, on two calls in a row with different group
tables, that its outputs equal the regular entry point's bit for bit and the CPU
oracle's within the benchmark tolerance, that its device error word reads zero
through nvfp4_noalloc_check, and that a repeated call with
NVFP4_FLAG_REUSE_DESCRIPTORS gives the same bits.

This file is collected last so that a failure here never hides the other tests; it
passes both on its own in a fresh process and after the rest of the suite.
"""
from __future__ import annotations

import ctypes

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


def _noalloc_error_bits(lib, stream) -> tuple:
    bits = ctypes.c_uint(0xFFFFFFFF)
    st = lib.nvfp4_noalloc_check(stream, ctypes.byref(bits))
    return st, int(bits.value)


def _run_noalloc(pkg, prob, table=None, flags=0):
    lib = pkg.load_library()
    t = _table(pkg, prob) if table is None else table
    for c in prob.c:
        c.fill_(float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.nvfp4_grouped_gemm_noalloc(t.ctypes.data, prob.num_groups,
                                        flags | (pkg._native.FLAG_GATED if prob.gated else 0),
                                        stream)
    pkg._native.check(st, lib)
    st, bits = _noalloc_error_bits(lib, stream)
    assert st == pkg._native.OK and bits == 0, f"status {st}, device error bits 0x{bits:x}"
    return [c.clone() for c in prob.c], t


def _oracle(prob, g):
    a, b = prob.a[g].cpu().numpy(), prob.b[g].cpu().numpy()
    sfa, sfb = prob.sfa_plain[g].cpu().numpy(), prob.sfb_plain[g].cpu().numpy()
    if prob.gated:
        return O.ref_gated(a, b, prob.b2[g].cpu().numpy(), sfa, sfb,
                           prob.sfb2_plain[g].cpu().numpy(), prob.alpha[g], prob.alpha2[g]), None
    ref32 = O.ref_gemm_fp32(a, b, sfa, sfb) * np.float32(prob.alpha[g])
    with np.errstate(over="ignore"):
        return ref32.astype(np.float16), ref32


def _check(regular, noalloc, prob):
    for g, (r, z) in enumerate(zip(regular, noalloc)):
        if prob.m[g] == 0:
            continue
        # Same table, same kernel choice: the two entry points agree bit for bit.
        assert torch.equal(z.view(torch.int16), r.view(torch.int16)), f"group {g} differs"
        exp, ref32 = _oracle(prob, g)
        res = O.compare_fp16(z.cpu().numpy(), exp, ref32, **TOL)
        assert res["ok"], f"group {g} against the oracle: {res}"


def test_noalloc_matches_regular_entry_point_and_oracle_two_calls(pkg):
    # Two consecutive calls with different group tables share the built-in scratch.
    first = pkg.workloads.make_problem("na1", [128, 0, 77, 300], 256, 512, seed=31,
                                       device="cuda", alpha_range=(0.5, 2.0))
    second = pkg.workloads.make_problem("na2", [64, 200], 384, 768, gated=True, seed=32,
                                        device="cuda", alpha_range=(0.5, 2.0))
    for prob in (first, second):
        regular = _run_regular(pkg, prob)
        noalloc, table = _run_noalloc(pkg, prob)
        _check(regular, noalloc, prob)
    # The scratch array now holds the second table: a repeat with descriptor reuse
    # skips the upload and must give the same bits.
    again, _ = _run_noalloc(pkg, second, table=table, flags=pkg._native.FLAG_REUSE_DESCRIPTORS)
    _check(regular, again, second)


def test_noalloc_rejects_more_groups_than_its_scratch_holds(pkg):
    lib = pkg.load_library()
    G = pkg._native.NOALLOC_MAX_GROUPS + 1
    t = np.zeros(G, dtype=pkg._native.GROUP_DTYPE)
    st = lib.nvfp4_grouped_gemm_noalloc(t.ctypes.data, G, 0, None)
    assert st == pkg._native.ERR_INVALID_ARGUMENT
    assert b"exceeds" in lib.nvfp4_last_error_detail()
