"""The C-ABI library loads and exports every declared symbol; host-side validation
returns the documented status codes without launching anything (CPU only)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT


def _declared_symbols() -> set:
    hdr = open(os.path.join(ROOT, "include", "nvfp4_group_gemm.h")).read()
    return set(re.findall(r"NVFP4_API\s+[\w\s\*]+?\b(nvfp4_\w+)\s*\(", hdr))


def test_header_declarations_match_binding(pkg):
    assert _declared_symbols() == set(pkg._native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.load_library()
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", pkg._native.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert _declared_symbols() <= exported
    # Nothing else with C linkage leaks out besides the declared API.
    assert {s for s in exported if s.startswith("nvfp4_")} == _declared_symbols()


def test_struct_layout_matches_header(pkg):
    N = pkg._native
    assert ctypes.sizeof(N.Nvfp4Group) == 80
    assert N.Nvfp4Group.m.offset == 56 and N.Nvfp4Group.alpha2.offset == 72
    assert N.GROUP_DTYPE.itemsize == 80


def test_version_and_strings(pkg):
    lib = pkg.load_library()
    assert lib.nvfp4_abi_version() == pkg._native.ABI_VERSION
    hdr = open(os.path.join(ROOT, "include", "nvfp4_group_gemm.h")).read()
    assert f"#define NVFP4_ABI_VERSION {pkg._native.ABI_VERSION}" in hdr
    assert lib.nvfp4_strerror(0) == b"success"
    assert b"timed out" in lib.nvfp4_strerror(7)
    assert lib.nvfp4_strerror(999) == b"unknown status"


def test_size_queries(pkg):
    N = pkg._native
    assert N.workspace_size(0) == 256
    # header + records + maps + segment row offsets (records and offsets padded to 128 B)
    assert N.workspace_size(8) == 256 + 8 * 64 + 8 * 8 * 128 + 128
    assert N.workspace_size(3) == 512 + 3 * 8 * 128 + 128
    assert N.workspace_size(40) == 256 + 40 * 64 + 40 * 8 * 128 + 256
    assert N.sf_blocked_size(80, 32) == 1 * 8 * 512
    assert N.sf_blocked_size(129, 5) == 2 * 2 * 512
    assert N.sf_blocked_size(0, 4) == 0


def _table(N, **kw):
    t = np.zeros(1, dtype=N.GROUP_DTYPE)
    base = dict(a=0x10000, b=0x20000, sfa=0x30000, sfb=0x40000, c=0x50000, m=128, n=256, k=512,
                alpha=1.0, alpha2=1.0)
    base.update(kw)
    for k, v in base.items():
        t[k] = v
    return t


@pytest.mark.parametrize("kw,flags,status", [
    (dict(k=100), 0, 2),            # K not a multiple of 256
    (dict(k=0), 0, 2),
    (dict(n=100), 0, 2),            # N % 8
    (dict(m=-1), 0, 2),
    (dict(a=0), 0, 4),              # NULL operand of a non-empty group
    (dict(c=0x50008), 0, 3),        # misaligned output
    (dict(b2=0), 1, 4),             # gated without up weights
    (dict(), 0x400, 1),             # unknown flag bit
    (dict(), 0x10 | 0x20, 1),       # exclusive CTA modes
    (dict(), 0x10 | 0x2, 1),        # pairs need 256-column tiles
    (dict(), 0x2 | 0x4, 1),         # exclusive tile flags
    (dict(), 0x80 | 0x1, 1),        # weight-stationary tiles are non-gated
    (dict(), 0x80 | 0x10, 1),       # ... and exclusive with the other tile shapes
    (dict(), 0x80 | 0x2, 1),
    (dict(k=100), 0x80, 2),         # shape checks apply to every kernel
])
def test_validation_errors_before_launch(pkg, kw, flags, status):
    N = pkg._native
    lib = pkg.load_library()
    t = _table(N, **kw)
    ws = ctypes.create_string_buffer(N.workspace_size(1) + 256)
    ws_ptr = (ctypes.addressof(ws) + 255) & ~255
    st = lib.nvfp4_grouped_gemm(t.ctypes.data, 1, flags, ws_ptr, N.workspace_size(1), None)
    assert st == status, lib.nvfp4_last_error_detail()
    assert lib.nvfp4_last_error_detail()


@pytest.mark.parametrize("case,flags,status", [
    ("null_offsets", 0, 4),
    ("misaligned_counts", 0, 3),
    ("m_differs", 0, 2),            # every group addresses the same slab
    ("weight_stationary", 0x80, 1),
    ("split_k", 0x100, 1),
    ("bad_k", 0, 2),                # the usual shape checks still apply
    ("no_workspace", 0, 5),
    ("nvfp4_out_not_gated", 0, 1),  # NVFP4 output is for gated launches
    ("nvfp4_out_bad_scale", 1, 1),
    ("nvfp4_out_misaligned", 1, 3),
    ("nvfp4_out_n", 1, 2),          # n must be a multiple of 64
    ("scatter_gated", 1, 1),        # scattered rows are for non-gated launches
    ("scatter_ld", 0, 3),           # dest_ld a multiple of 16
    ("scatter_short_ld", 0, 1),     # dest_ld >= 2 n
    ("scatter_base", 0, 3),         # bases 16-byte aligned
])
def test_segment_validation_errors_before_launch(pkg, case, flags, status):
    N = pkg._native
    lib = pkg.load_library()
    t = np.zeros(2, dtype=N.GROUP_DTYPE)  # (np.concatenate would drop the record padding)
    t[0] = _table(N)[0]
    t[1] = _table(N, m=128 if case != "m_differs" else 64)[0]
    if case == "bad_k":
        t["k"] = 100
    if case == "nvfp4_out_n":
        t["n"] = 200
    t["b2"], t["sfb2"] = 0x60000, 0x68000
    ws = ctypes.create_string_buffer(N.workspace_size(2) + 256)
    ws_ptr = (ctypes.addressof(ws) + 255) & ~255
    offs = 0 if case == "null_offsets" else 0x70000
    counts = 0x70102 if case == "misaligned_counts" else 0x70100
    out = None
    if case.startswith("nvfp4_out"):
        out = N.SegmentOutput.nvfp4(0x78008 if case == "nvfp4_out_misaligned" else 0x78000,
                                    0.0 if case == "nvfp4_out_bad_scale" else 0.5)
    elif case.startswith("scatter"):
        ld = {"scatter_ld": 520, "scatter_short_ld": 256}.get(case, 512)
        bases = [0x90008 if case == "scatter_base" else 0x90000, 0xA0000]
        out = N.SegmentOutput.scattered(0x88000, bases, ld)
    st = lib.nvfp4_grouped_gemm_segments(t.ctypes.data, 2, flags, offs, counts, 0,
                                         ctypes.byref(out) if out is not None else None,
                                         None if case == "no_workspace" else ws_ptr,
                                         N.workspace_size(2), None)
    assert st == status, lib.nvfp4_last_error_detail()
    assert lib.nvfp4_last_error_detail()


def test_workspace_errors(pkg):
    N = pkg._native
    lib = pkg.load_library()
    t = _table(N)
    assert lib.nvfp4_grouped_gemm(t.ctypes.data, 1, 0, None, 1 << 20, None) == 5
    assert lib.nvfp4_grouped_gemm(t.ctypes.data, 1, 0, 0x1000 + 8, 1 << 20, None) == 5
    assert lib.nvfp4_grouped_gemm(t.ctypes.data, 1, 0, 0x1000, 16, None) == 5
    assert lib.nvfp4_grouped_gemm(None, 1, 0, 0x1000, 1 << 20, None) == 1
    assert lib.nvfp4_grouped_gemm(t.ctypes.data, -1, 0, 0x1000, 1 << 20, None) == 1
    assert lib.nvfp4_grouped_gemm(None, 0, 0, None, 0, None) == 0   # empty launch is a no-op


def test_empty_groups_launch_nothing(pkg):
    """All groups empty -> success without touching the device (works on a CPU box)."""
    N = pkg._native
    lib = pkg.load_library()
    t = _table(N, m=0, a=0, b=0, c=0, sfa=0, sfb=0)
    assert lib.nvfp4_grouped_gemm(t.ctypes.data, 1, 0, 0x1000, N.workspace_size(1), None) == 0


def test_sf_converter_validation(pkg):
    lib = pkg.load_library()
    assert lib.nvfp4_sf_to_blocked(None, None, 0, 4, 4, None) == 0
    assert lib.nvfp4_sf_to_blocked(None, None, 4, 4, 4, None) == 4
    assert lib.nvfp4_sf_to_blocked(0x1000, 0x2000, -1, 4, 4, None) == 2
    assert lib.nvfp4_sf_to_blocked(0x1000, 0x2008, 4, 4, 4, None) == 3
    assert lib.nvfp4_sf_to_blocked(0x1000, 0x2000, 4, 8, 4, None) == 1


def test_quantize_validation_before_launch(pkg):
    lib = pkg.load_library()
    ok = dict(x=0x1000, rows=4, cols=64, ld=64, dtype=0, sg=1.0, packed=0x2000, pld=32, sf=0x3000)

    def call(**kw):
        a = dict(ok, **kw)
        return lib.nvfp4_quantize(a["x"], a["rows"], a["cols"], a["ld"], a["dtype"], a["sg"],
                                  a["packed"], a["pld"], a["sf"], None)

    assert call(dtype=2) == 1                # unknown dtype
    assert call(sg=0.0) == 1                 # scale must be > 0
    assert call(sg=float("inf")) == 1
    assert call(cols=96) == 2                # cols % 64
    assert call(rows=-1) == 2
    assert call(rows=0) == 0                 # nothing to do
    assert call(x=0) == 4                    # NULL input
    assert call(ld=32) == 1                  # ld < cols
    assert call(x=0x1008) == 3               # misaligned input
    assert call(pld=40) == 3                 # packed row stride not a multiple of 16
    assert lib.nvfp4_last_error_detail()


def test_split_scratch_constant_matches_header(pkg):
    hdr = open(os.path.join(ROOT, "include", "nvfp4_group_gemm.h")).read()
    m = re.search(r"#define NVFP4_SPLIT_SCRATCH_BYTES \((\d+)u \+ (\d+)u \* (\d+)u\)", hdr)
    assert m, "NVFP4_SPLIT_SCRATCH_BYTES not found"
    a, b, c = (int(x) for x in m.groups())
    assert a + b * c == pkg._native.SPLIT_SCRATCH_BYTES
    assert pkg._native.workspace_size_with_split(8) % 256 == 0


@pytest.mark.parametrize("case,flags,status", [
    ("reuse_flag", 0x8, 1),      # a plan uploads its own descriptors
    ("split_flag", 0x100, 1),
    ("no_groups", 0, 2),
    ("bad_k", 0, 2),
    ("misaligned_ws", 0, 5),
    ("null_out", 0, 1),
])
def test_plan_create_validation(pkg, case, flags, status):
    N = pkg._native
    lib = pkg.load_library()
    t = _table(N, k=100 if case == "bad_k" else 512)
    ws = ctypes.create_string_buffer(N.workspace_size(1) + 512)
    ws_ptr = (ctypes.addressof(ws) + 255) & ~255
    if case == "misaligned_ws":
        ws_ptr += 16
    out = ctypes.c_void_p()
    st = lib.nvfp4_plan_create(t.ctypes.data, 0 if case == "no_groups" else 1, flags, ws_ptr,
                               N.workspace_size(1), None,
                               None if case == "null_out" else ctypes.byref(out))
    assert st == status, lib.nvfp4_last_error_detail()
    assert out.value is None
    assert lib.nvfp4_plan_launch(None, None) == 1
    lib.nvfp4_plan_destroy(None)  # destroying nothing is allowed


def test_expert_parallel_validation_before_launch(pkg):
    """Every nvfp4_ep_* entry point rejects bad ranks, shapes, NULL and misaligned buffers
    with its status code before anything is launched."""
    from importlib import import_module

    N = import_module(pkg.__name__ + "._native")
    lib = pkg.load_library()
    peers2 = N.EpPeers.of([0x10000, 0x20000])
    nullpeer = N.EpPeers.of([0x10000, 0])
    A, B, C, D = 0x1000, 0x2000, 0x3000, 0x4000
    # publish counts / layout: world and expert checks
    assert lib.nvfp4_ep_publish_counts(A, 16, 0, 9, peers2, None) == 1
    assert lib.nvfp4_ep_publish_counts(A, 15, 0, 2, peers2, None) == 1
    assert lib.nvfp4_ep_publish_counts(None, 16, 0, 2, peers2, None) == 4
    assert lib.nvfp4_ep_layout(A, 16, 2, 2, 1024, B, C, D, A, None) == 1
    # token-once dispatch
    def dt(**kw):
        a = dict(ids=A, tokens=4, topk=2, E=16, rank=0, world=2, codes=0x5000, ld=256,
                 sf=0x6000, cols=512, tok=peers2, tsf=peers2)
        a.update(kw)
        return lib.nvfp4_ep_dispatch_tokens(a["ids"], a["tokens"], a["topk"], a["E"], a["rank"],
                                            a["world"], B, C, D, a["codes"], a["ld"], a["sf"],
                                            a["cols"], a["tok"], a["tsf"], 1 << 20, 0x7000, None)
    assert dt(world=9) == 1
    assert dt(cols=320) == 2
    assert dt(tokens=0) == 0
    assert dt(ids=0) == 4
    assert dt(codes=0x5008) == 3
    assert dt(ld=200) == 3
    assert dt(tok=nullpeer) == 4
    # expand
    assert lib.nvfp4_ep_expand(A, 4, 2, 0, B, C, 512, D, 0x5000, 1024, None) == 1
    assert lib.nvfp4_ep_expand(A, 4, 2, 2, B, C, 100, D, 0x5000, 1024, None) == 2
    assert lib.nvfp4_ep_expand(0, 4, 2, 2, B, C, 512, D, 0x5000, 1024, None) == 4
    assert lib.nvfp4_ep_expand(A, 4, 2, 2, B + 8, C, 512, D, 0x5000, 1024, None) == 3
    # pair tables
    assert lib.nvfp4_ep_publish_pairs(A, B, 0, 4, 2, 16, 0, 2, peers2, peers2, None) == 4
    assert lib.nvfp4_ep_publish_pairs(A, B, C, 4, 2, 16, 0, 2, peers2, nullpeer, None) == 4
    assert lib.nvfp4_ep_publish_pairs(A, B, C, 4, 0, 16, 0, 2, peers2, peers2, None) == 2
    # return sums
    assert lib.nvfp4_ep_return_sums(A, B, 4, 2, 2, 2, C, 512, 512, peers2, None) == 1
    assert lib.nvfp4_ep_return_sums(A, B, 4, 2, 0, 2, C, 512, 12, peers2, None) == 2
    assert lib.nvfp4_ep_return_sums(A, B, 4, 2, 0, 2, C + 8, 512, 512, peers2, None) == 3
    assert lib.nvfp4_ep_return_sums(A, B, 4, 2, 0, 2, C, 256, 512, peers2, None) == 3
    assert lib.nvfp4_ep_return_sums(A, B, 4, 2, 0, 2, C, 512, 512, nullpeer, None) == 4
    # combine of the sums
    assert lib.nvfp4_ep_combine_sums(A, B, 4, 2, 15, 2, C, 512, D, 512, None) == 1
    assert lib.nvfp4_ep_combine_sums(A, B, 4, 2, 16, 2, C, 512, D + 8, 512, None) == 3
    assert lib.nvfp4_ep_combine_sums(A, 0, 4, 2, 16, 2, C, 512, D, 512, None) == 4
    assert lib.nvfp4_last_error_detail()
