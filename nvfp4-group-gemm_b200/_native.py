"""ctypes binding of the C ABI declared in ``include/nvfp4_group_gemm.h``.

The shared library is the only compute path: if it is missing or cannot be
loaded, every entry point raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

from . import build as _build

LIB_PATH = _build.LIB_PATH

# Status codes (nvfp4_status).
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_BAD_SHAPE = 2
ERR_MISALIGNED = 3
ERR_NULL_POINTER = 4
ERR_WORKSPACE = 5
ERR_CUDA = 6
ERR_DEVICE_TIMEOUT = 7
ERR_UNSUPPORTED_DEVICE = 8
ERR_DRIVER = 9

# Flags (NVFP4_FLAG_*).
FLAG_GATED = 0x1
FLAG_TILE_N128 = 0x2
FLAG_TILE_N256 = 0x4
FLAG_REUSE_DESCRIPTORS = 0x8
FLAG_CTA_PAIR = 0x10
FLAG_SINGLE_CTA = 0x20
FLAG_DIAG_SKIP_MMA = 0x40
FLAG_WEIGHT_STATIONARY = 0x80
FLAG_SPLIT_K = 0x100
FLAG_STREAM_K = 0x200

# Device error bits (WorkspaceHeader::error_bits).
DEV_ERR_PRODUCER_TIMEOUT = 1 << 0
DEV_ERR_MMA_TIMEOUT = 1 << 1
DEV_ERR_ACC_TIMEOUT = 1 << 2
DEV_ERR_EPILOGUE_TIMEOUT = 1 << 3
DEV_ERR_DRAIN_TIMEOUT = 1 << 4
DEV_ERR_BAD_SEGMENT = 1 << 5  # a segment launch skipped an out-of-range row segment

# Every symbol the public header declares; the library must export all of them.
EXPORTED_SYMBOLS = (
    "nvfp4_abi_version",
    "nvfp4_strerror",
    "nvfp4_last_error_detail",
    "nvfp4_workspace_size",
    "nvfp4_grouped_gemm",
    "nvfp4_sf_blocked_size",
    "nvfp4_sf_to_blocked",
    "nvfp4_workspace_check",
    "nvfp4_grouped_gemm_noalloc",
    "nvfp4_noalloc_check",
    "nvfp4_grouped_gemm_segments",
    "nvfp4_grouped_gemm_replicated",
    "nvfp4_plan_create",
    "nvfp4_plan_launch",
    "nvfp4_plan_destroy",
    "nvfp4_quantize",
    "nvfp4_quantize_rows",
    "nvfp4_moe_route_workspace_size",
    "nvfp4_moe_route",
    "nvfp4_moe_combine",
    "nvfp4_moe_gather_quantized",
    "nvfp4_ep_publish_counts",
    "nvfp4_ep_layout",
    "nvfp4_ep_dispatch",
    "nvfp4_ep_combine",
    "nvfp4_ep_dispatch_tokens",
    "nvfp4_ep_expand",
    "nvfp4_ep_publish_pairs",
    "nvfp4_ep_return_sums",
    "nvfp4_ep_combine_sums",
)

ABI_VERSION = 2   # NVFP4_ABI_VERSION
EP_MAX_RANKS = 8  # NVFP4_EP_MAX_RANKS
MAX_REPLICAS = 7  # replicas nvfp4_grouped_gemm_replicated accepts
EP_ERR_CAPACITY = 1 << 0  # an expert segment did not fit the owner's receive slab


class SegmentOutput(ctypes.Structure):
    """nvfp4_segment_output: NVFP4 output (sf, scale) or scattered rows (row_dest,
    dest_base, dest_ld) of a segment launch."""

    _fields_ = [("sf", ctypes.c_void_p), ("scale", ctypes.c_float),
                ("row_dest", ctypes.c_void_p), ("dest_base", ctypes.c_void_p * EP_MAX_RANKS),
                ("dest_ld", ctypes.c_int64)]

    @classmethod
    def nvfp4(cls, sf_ptr: int, scale: float) -> "SegmentOutput":
        o = cls()
        o.sf, o.scale = int(sf_ptr), float(scale)
        return o

    @classmethod
    def scattered(cls, row_dest_ptr: int, bases, ld: int) -> "SegmentOutput":
        o = cls()
        o.row_dest, o.dest_ld = int(row_dest_ptr), int(ld)
        for i, b in enumerate(bases):
            o.dest_base[i] = int(b)
        return o


class EpPeers(ctypes.Structure):
    """nvfp4_ep_peers: one device address per rank (passed by value)."""

    _fields_ = [("ptr", ctypes.c_void_p * EP_MAX_RANKS)]

    @classmethod
    def of(cls, addresses) -> "EpPeers":
        if len(addresses) > EP_MAX_RANKS:
            raise ValueError(f"at most {EP_MAX_RANKS} ranks")
        p = cls()
        for i, a in enumerate(addresses):
            p.ptr[i] = int(a)
        return p

# Row-map modes of nvfp4_quantize_rows (NVFP4_ROWS_*).
ROWS_GATHER = 1
ROWS_MASK = 2

# Input dtypes of nvfp4_quantize (NVFP4_DTYPE_*).
DTYPE_BF16 = 0
DTYPE_FP16 = 1

# Largest group count nvfp4_grouped_gemm_noalloc accepts (NVFP4_NOALLOC_MAX_GROUPS).
NOALLOC_MAX_GROUPS = 512

# Extra workspace that enables split-K of a launch's last partial wave (NVFP4_SPLIT_SCRATCH_BYTES).
SPLIT_SCRATCH_BYTES = 4096 + 148 * 131072


class Nvfp4Group(ctypes.Structure):
    """Mirror of ``nvfp4_group`` (80 bytes)."""

    _fields_ = [
        ("a", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("b2", ctypes.c_void_p),
        ("sfa", ctypes.c_void_p),
        ("sfb", ctypes.c_void_p),
        ("sfb2", ctypes.c_void_p),
        ("c", ctypes.c_void_p),
        ("m", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("alpha", ctypes.c_float),
        ("alpha2", ctypes.c_float),
    ]


# The same record as a numpy structured dtype, so that a whole group table is
# filled with a few vectorised column assignments instead of per-field ctypes calls.
GROUP_DTYPE = np.dtype(
    {
        "names": [f[0] for f in Nvfp4Group._fields_],
        "formats": ["<u8"] * 7 + ["<i4"] * 3 + ["<f4"] * 2,
        "offsets": [getattr(Nvfp4Group, f[0]).offset for f in Nvfp4Group._fields_],
        "itemsize": ctypes.sizeof(Nvfp4Group),
    }
)
assert GROUP_DTYPE.itemsize == 80


class Nvfp4Error(RuntimeError):
    """A non-zero status returned by the native library."""

    def __init__(self, status: int, message: str, detail: str = ""):
        self.status = status
        self.detail = detail
        text = f"nvfp4 status {status}: {message}"
        if detail:
            text += f" ({detail})"
        super().__init__(text)


_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the native library, declaring argument types."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        # NVFP4_LIBRARY selects another build of the same library (same ABI), e.g. one
        # compiled with different tuning constants.
        p = path or os.environ.get("NVFP4_LIBRARY") or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"native library {p} is missing; build it with "
                "`python __graft_entry__.py build` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(p)
        vp, sz, i32, i64, u32 = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                 ctypes.c_int64, ctypes.c_uint)
        lib.nvfp4_abi_version.argtypes = []
        lib.nvfp4_abi_version.restype = i32
        found = int(lib.nvfp4_abi_version())
        if found != ABI_VERSION:
            raise ImportError(f"native library {p} has ABI version {found}, this package needs "
                              f"{ABI_VERSION}; rebuild it with `python __graft_entry__.py build`")
        lib.nvfp4_strerror.argtypes = [i32]
        lib.nvfp4_strerror.restype = ctypes.c_char_p
        lib.nvfp4_last_error_detail.argtypes = []
        lib.nvfp4_last_error_detail.restype = ctypes.c_char_p
        lib.nvfp4_workspace_size.argtypes = [i32]
        lib.nvfp4_workspace_size.restype = sz
        lib.nvfp4_grouped_gemm.argtypes = [vp, i32, u32, vp, sz, vp]
        lib.nvfp4_grouped_gemm.restype = i32
        lib.nvfp4_sf_blocked_size.argtypes = [i32, i32]
        lib.nvfp4_sf_blocked_size.restype = sz
        lib.nvfp4_sf_to_blocked.argtypes = [vp, vp, i32, i32, i64, vp]
        lib.nvfp4_sf_to_blocked.restype = i32
        lib.nvfp4_workspace_check.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint)]
        lib.nvfp4_workspace_check.restype = i32
        lib.nvfp4_grouped_gemm_noalloc.argtypes = [vp, i32, u32, vp]
        lib.nvfp4_grouped_gemm_noalloc.restype = i32
        lib.nvfp4_grouped_gemm_replicated.argtypes = [vp, i32, u32, vp, sz, vp, i32, vp]
        lib.nvfp4_grouped_gemm_replicated.restype = i32
        lib.nvfp4_noalloc_check.argtypes = [vp, ctypes.POINTER(ctypes.c_uint)]
        lib.nvfp4_noalloc_check.restype = i32
        lib.nvfp4_grouped_gemm_segments.argtypes = [vp, i32, u32, vp, vp, i64,
                                                    ctypes.POINTER(SegmentOutput), vp, sz, vp]
        lib.nvfp4_grouped_gemm_segments.restype = i32
        lib.nvfp4_plan_create.argtypes = [vp, i32, u32, vp, sz, vp, ctypes.POINTER(vp)]
        lib.nvfp4_plan_create.restype = i32
        lib.nvfp4_plan_launch.argtypes = [vp, vp]
        lib.nvfp4_plan_launch.restype = i32
        lib.nvfp4_plan_destroy.argtypes = [vp]
        lib.nvfp4_plan_destroy.restype = None
        lib.nvfp4_quantize.argtypes = [vp, i32, i32, i64, i32, ctypes.c_float, vp, i64, vp, vp]
        lib.nvfp4_quantize.restype = i32
        lib.nvfp4_quantize_rows.argtypes = [vp, i32, i32, i64, i32, ctypes.c_float, vp, i32, vp,
                                            i64, vp, vp]
        lib.nvfp4_quantize_rows.restype = i32
        lib.nvfp4_moe_route_workspace_size.argtypes = [i64, i32]
        lib.nvfp4_moe_route_workspace_size.restype = sz
        lib.nvfp4_moe_route.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp, i64, vp, sz, vp]
        lib.nvfp4_moe_route.restype = i32
        lib.nvfp4_moe_combine.argtypes = [vp, i64, vp, vp, i32, i32, i32, vp, i64, vp]
        lib.nvfp4_moe_combine.restype = i32
        lib.nvfp4_moe_gather_quantized.argtypes = [vp, i64, vp, vp, i32, i32, vp, i64, vp, vp]
        lib.nvfp4_moe_gather_quantized.restype = i32
        lib.nvfp4_ep_publish_counts.argtypes = [vp, i32, i32, i32, EpPeers, vp]
        lib.nvfp4_ep_publish_counts.restype = i32
        lib.nvfp4_ep_layout.argtypes = [vp, i32, i32, i32, i64, vp, vp, vp, vp, vp]
        lib.nvfp4_ep_layout.restype = i32
        lib.nvfp4_ep_dispatch.argtypes = [vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, i64, vp,
                                          i32, EpPeers, EpPeers, EpPeers, i64, vp, vp]
        lib.nvfp4_ep_dispatch.restype = i32
        lib.nvfp4_ep_combine.argtypes = [vp, vp, i32, i32, vp, i32, vp, i64, vp]
        lib.nvfp4_ep_combine.restype = i32
        lib.nvfp4_ep_dispatch_tokens.argtypes = [vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, i64,
                                                 vp, i32, EpPeers, EpPeers, i64, vp, vp]
        lib.nvfp4_ep_dispatch_tokens.restype = i32
        lib.nvfp4_ep_expand.argtypes = [vp, i32, i32, i32, vp, vp, i32, vp, vp, i64, vp]
        lib.nvfp4_ep_expand.restype = i32
        lib.nvfp4_ep_publish_pairs.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, EpPeers,
                                               EpPeers, vp]
        lib.nvfp4_ep_publish_pairs.restype = i32
        lib.nvfp4_ep_return_sums.argtypes = [vp, vp, i32, i32, i32, i32, vp, i64, i32, EpPeers, vp]
        lib.nvfp4_ep_return_sums.restype = i32
        lib.nvfp4_ep_combine_sums.argtypes = [vp, vp, i32, i32, i32, i32, vp, i32, vp, i64, vp]
        lib.nvfp4_ep_combine_sums.restype = i32
        if path is None:
            _lib = lib
        return lib


def check(status: int, lib: ctypes.CDLL | None = None) -> None:
    """Raise Nvfp4Error for a non-zero status (with the library's detail text)."""
    if status == OK:
        return
    lib = lib or load_library()
    msg = lib.nvfp4_strerror(status).decode()
    detail = lib.nvfp4_last_error_detail().decode()
    raise Nvfp4Error(status, msg, detail)


def workspace_size(num_groups: int) -> int:
    return int(load_library().nvfp4_workspace_size(num_groups))


def workspace_size_with_split(num_groups: int) -> int:
    """Workspace bytes that also enable split-K: the workspace rounded up to 256 bytes plus
    SPLIT_SCRATCH_BYTES."""
    return (workspace_size(num_groups) + 255) // 256 * 256 + SPLIT_SCRATCH_BYTES


def sf_blocked_size(rows: int, sf_cols: int) -> int:
    return int(load_library().nvfp4_sf_blocked_size(rows, sf_cols))


def grouped_gemm_raw(table: np.ndarray, flags: int, workspace_ptr: int, workspace_bytes: int,
                     stream_ptr: int) -> None:
    """Call nvfp4_grouped_gemm on a GROUP_DTYPE table (host memory)."""
    assert table.dtype == GROUP_DTYPE and table.flags["C_CONTIGUOUS"]
    lib = load_library()
    st = lib.nvfp4_grouped_gemm(table.ctypes.data, int(table.shape[0]), flags, workspace_ptr,
                                workspace_bytes, stream_ptr)
    check(st, lib)


def grouped_gemm_segments_raw(table: np.ndarray, flags: int, offsets_ptr: int, counts_ptr: int,
                              expected_rows: int, workspace_ptr: int, workspace_bytes: int,
                              stream_ptr: int, output: "SegmentOutput | None" = None) -> None:
    """Call nvfp4_grouped_gemm_segments on a GROUP_DTYPE table (host memory) whose rows are
    given by device int32 arrays of per-group first rows and row counts; ``output`` selects
    NVFP4 or scattered output (None: fp16 rows into c)."""
    assert table.dtype == GROUP_DTYPE and table.flags["C_CONTIGUOUS"]
    lib = load_library()
    st = lib.nvfp4_grouped_gemm_segments(table.ctypes.data, int(table.shape[0]), flags,
                                         offsets_ptr, counts_ptr, int(expected_rows),
                                         ctypes.byref(output) if output is not None else None,
                                         workspace_ptr, workspace_bytes, stream_ptr)
    check(st, lib)


def quantize_raw(x_ptr: int, rows: int, cols: int, ld: int, dtype: int, global_scale: float,
                 packed_ptr: int, packed_ld: int, sf_ptr: int, stream_ptr: int) -> None:
    """Call nvfp4_quantize (device pointers, row strides in elements / bytes)."""
    lib = load_library()
    check(lib.nvfp4_quantize(x_ptr, rows, cols, ld, dtype, global_scale, packed_ptr, packed_ld,
                             sf_ptr, stream_ptr), lib)


def sf_to_blocked_raw(plain_ptr: int, blocked_ptr: int, rows: int, sf_cols: int, ld: int,
                      stream_ptr: int) -> None:
    lib = load_library()
    check(lib.nvfp4_sf_to_blocked(plain_ptr, blocked_ptr, rows, sf_cols, ld, stream_ptr), lib)


def workspace_check(workspace_ptr: int, stream_ptr: int) -> int:
    """Synchronise and return the device error bits (raises on timeout bits)."""
    lib = load_library()
    bits = ctypes.c_uint(0)
    st = lib.nvfp4_workspace_check(workspace_ptr, stream_ptr, ctypes.byref(bits))
    check(st, lib)
    return int(bits.value)
