"""Harness-facing entry points: ``custom_kernel(data)`` / ``solve(data)``.

Mirrors the reference submission's interface (submission.py:788-891):

* 4-tuple grouped form ``(abc_tensors, sfasfb_tensors, sfasfb_reordered_tensors,
  problem_sizes)`` (REFERENCE_IMPL.md:52, submission.py:804-858): one grouped
  launch; element 1 (plain CPU scales) is ignored exactly as the reference does;
  each ``c`` is written in place and the list of ``c`` tensors is returned.
* 10-tuple dual GEMM ``(a, b1, b2, sfa, sfb1, sfb2, sfa_perm, sfb1_perm,
  sfb2_perm, c)`` (submission.py:860-886): ``c = silu(a@b1) * (a@b2)`` with the
  two products rounded to fp16 first; here it is one fused launch.

Extensions (no counterpart in the reference, which has no global scale and no
grouped gated form):

* an optional 5th element (or the ``global_scales`` keyword) holding one fp32
  scale per group, or a (gate, up) pair per group when gated;
* a grouped gated form: a 4-tuple whose ``abc_tensors`` entries are
  ``(a, b_gate, b_up, c)`` and whose reordered scale entries are
  ``(sfa, sfb_gate, sfb_up)``.

Errors: malformed input raises ValueError before anything is launched; a
failure reported by the native library raises ``Nvfp4Error`` (a RuntimeError).
There is no CPU or library fallback.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Sequence

import numpy as np
import torch

from . import _native
from .layout import blocked_sf_bytes, ceil_div

input_t = tuple
output_t = list

_FP4_DTYPES = tuple(
    d for d in (getattr(torch, "float4_e2m1fn_x2", None), torch.uint8, torch.int8) if d is not None
)


def _current_raw_stream(device_index: int) -> int:
    """Handle of the current stream of a device (torch's C accessor when it exists: it
    skips building a Stream object, which costs a few microseconds per call)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


# ----------------------------------------------------------------------------
# Workspace and descriptor-table cache (one per device and stream)
# ----------------------------------------------------------------------------
class _Workspace:
    __slots__ = ("buf", "nbytes", "last_table", "last_flags", "last_sig", "plan")

    def __init__(self):
        self.buf = None
        self.nbytes = 0
        self.last_table = None
        self.last_flags = None
        self.last_sig = None
        self.plan = None  # native prepared launch of last_table (nvfp4_plan_create)

    def drop_plan(self):
        """Forget the prepared launch (the workspace is about to hold other descriptors)."""
        if self.plan is not None:
            _native.load_library().nvfp4_plan_destroy(self.plan)
            self.plan = None


_ws_lock = threading.Lock()
_workspaces: dict = {}


def _workspace_for(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> _Workspace:
    key = (device.index, stream.cuda_stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None:
            ws = _workspaces[key] = _Workspace()
    if ws.nbytes < nbytes:
        size = max(nbytes, 2 * ws.nbytes, 1 << 16)
        # Zero-filled: the first 4 bytes are the device error word.
        ws.drop_plan()
        ws.buf = torch.zeros(size, dtype=torch.uint8, device=device)
        ws.nbytes = size
        ws.last_table = None
        ws.last_sig = None
    return ws


def check_device_errors(device: torch.device | int | None = None,
                        stream: torch.cuda.Stream | None = None) -> int:
    """Synchronise and return the device error bits of this stream's workspace."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    s = stream or torch.cuda.current_stream(dev)
    ws = _workspaces.get((dev.index, s.cuda_stream))
    if ws is None or ws.buf is None:
        return 0
    with torch.cuda.device(dev):
        return _native.workspace_check(ws.buf.data_ptr(), s.cuda_stream)


# ----------------------------------------------------------------------------
# Validation helpers
# ----------------------------------------------------------------------------
def _as_2d_kmajor(t: torch.Tensor, rows: int, cols_bytes: int, name: str) -> torch.Tensor:
    """Accept [rows, cols] or [rows, cols, 1] tensors with dense, row-major rows."""
    if t.dim() == 3:
        if t.shape[2] != 1:
            raise ValueError(f"{name}: only L=1 is supported, got shape {tuple(t.shape)}")
        t = t[:, :, 0]
    if t.dim() != 2:
        raise ValueError(f"{name}: expected [rows, cols(, 1)], got shape {tuple(t.shape)}")
    if tuple(t.shape) != (rows, cols_bytes):
        raise ValueError(f"{name}: expected shape ({rows}, {cols_bytes}), got {tuple(t.shape)}")
    if rows > 0 and cols_bytes > 0 and (t.stride(1) != 1 or (rows > 1 and t.stride(0) != cols_bytes)):
        raise ValueError(f"{name}: rows must be dense and K-major (strides {t.stride()})")
    return t


def _check_fp4(t: torch.Tensor, name: str) -> None:
    if t.dtype not in _FP4_DTYPES:
        raise ValueError(f"{name}: expected packed e2m1 (float4_e2m1fn_x2/uint8), got {t.dtype}")


def _check_sf(t: torch.Tensor, rows: int, k: int, name: str) -> None:
    if t.element_size() != 1:
        raise ValueError(f"{name}: scale factors must be 1-byte E4M3 values, got {t.dtype}")
    need = blocked_sf_bytes(rows, ceil_div(k, 16))
    if t.numel() < need:
        raise ValueError(f"{name}: holds {t.numel()} scale bytes, blocked layout needs {need}")


# ----------------------------------------------------------------------------
# Core grouped launch
# ----------------------------------------------------------------------------
def _prepare(a, b, sfa, sfb, c, problem_sizes, alpha, b2, sfb2, alpha2, tile_n, cta,
             split_k=False):
    """Validate one grouped launch and build its group table.

    Returns ``(table, flags, device)``, or None when there is nothing to launch (no
    groups, or every group empty). Raises ValueError on malformed input.
    """
    if cta not in (None, "pair", "single", "weights"):
        raise ValueError(f"cta must be None, 'pair', 'single' or 'weights', got {cta!r}")
    G = len(problem_sizes)
    if not (len(a) == len(b) == len(sfa) == len(sfb) == len(c) == G):
        raise ValueError("a, b, sfa, sfb, c and problem_sizes must have one entry per group")
    gated = b2 is not None
    if gated and (sfb2 is None or len(b2) != G or len(sfb2) != G):
        raise ValueError("gated launches need b2 and sfb2 for every group")
    if G == 0:
        return None
    device = None
    table = np.zeros(G, dtype=_native.GROUP_DTYPE)
    ms = np.empty(G, dtype=np.int64)
    ns = np.empty(G, dtype=np.int64)
    ks = np.empty(G, dtype=np.int64)
    for g, ps in enumerate(problem_sizes):
        if len(ps) == 4 and int(ps[3]) != 1:
            raise ValueError(f"group {g}: only L=1 is supported (problem size {tuple(ps)})")
        m, n, k = int(ps[0]), int(ps[1]), int(ps[2])
        ms[g], ns[g], ks[g] = m, n, k
        if m < 0 or n < 0 or k < 0:
            raise ValueError(f"group {g}: negative size {tuple(ps)}")
        if m == 0 or n == 0:
            continue
        if k <= 0 or k % 256 != 0:
            raise ValueError(f"group {g}: K={k} must be a positive multiple of 256")
        if n % 8 != 0:
            raise ValueError(f"group {g}: N={n} must be a multiple of 8")
        tensors = [a[g], b[g], sfa[g], sfb[g], c[g]] + ([b2[g], sfb2[g]] if gated else [])
        for t in tensors:
            if not isinstance(t, torch.Tensor) or not t.is_cuda:
                raise ValueError(f"group {g}: every tensor must be a CUDA tensor")
            if device is None:
                device = t.device
            elif t.device != device:
                raise ValueError(f"group {g}: tensors span devices {device} and {t.device}")
        _check_fp4(a[g], f"a[{g}]")
        _check_fp4(b[g], f"b[{g}]")
        _as_2d_kmajor(a[g], m, k // 2, f"a[{g}]")
        _as_2d_kmajor(b[g], n, k // 2, f"b[{g}]")
        if c[g].dtype != torch.float16:
            raise ValueError(f"c[{g}]: expected float16, got {c[g].dtype}")
        _as_2d_kmajor(c[g], m, n, f"c[{g}]")
        _check_sf(sfa[g], m, k, f"sfa[{g}]")
        _check_sf(sfb[g], n, k, f"sfb[{g}]")
        if gated:
            _check_fp4(b2[g], f"b2[{g}]")
            _as_2d_kmajor(b2[g], n, k // 2, f"b2[{g}]")
            _check_sf(sfb2[g], n, k, f"sfb2[{g}]")
    if device is None:  # every group empty
        return None
    table["a"] = [t.data_ptr() for t in a]
    table["b"] = [t.data_ptr() for t in b]
    table["sfa"] = [t.data_ptr() for t in sfa]
    table["sfb"] = [t.data_ptr() for t in sfb]
    table["c"] = [t.data_ptr() for t in c]
    if gated:
        table["b2"] = [t.data_ptr() for t in b2]
        table["sfb2"] = [t.data_ptr() for t in sfb2]
    table["m"], table["n"], table["k"] = ms, ns, ks
    table["alpha"] = 1.0 if alpha is None else np.asarray(alpha, dtype=np.float32)
    table["alpha2"] = 1.0 if alpha2 is None else np.asarray(alpha2, dtype=np.float32)

    flags = _native.FLAG_GATED if gated else 0
    if cta == "pair":
        flags |= _native.FLAG_CTA_PAIR
    elif cta == "single":
        flags |= _native.FLAG_SINGLE_CTA
    elif cta == "weights":
        if gated:
            raise ValueError("the weight-stationary kernel is non-gated")
        if tile_n is not None:
            raise ValueError("the weight-stationary kernel has its own tile shape")
        flags |= _native.FLAG_WEIGHT_STATIONARY
    if tile_n == 128 and cta == "pair":
        raise ValueError("CTA pairs use 256-column tiles")
    if tile_n is not None and not gated:
        if tile_n == 128:
            flags |= _native.FLAG_TILE_N128
        elif tile_n == 256:
            flags |= _native.FLAG_TILE_N256
        else:
            raise ValueError(f"tile_n must be 128 or 256, got {tile_n}")
    if split_k:
        flags |= _native.FLAG_SPLIT_K
    return table, flags, device


def grouped_gemm(a: Sequence[torch.Tensor], b: Sequence[torch.Tensor],
                 sfa: Sequence[torch.Tensor], sfb: Sequence[torch.Tensor],
                 c: Sequence[torch.Tensor], problem_sizes: Sequence[Sequence[int]],
                 alpha: Sequence[float] | None = None,
                 b2: Sequence[torch.Tensor] | None = None,
                 sfb2: Sequence[torch.Tensor] | None = None,
                 alpha2: Sequence[float] | None = None,
                 tile_n: int | None = None,
                 stream: torch.cuda.Stream | None = None,
                 reuse_descriptors: bool = True,
                 cta: str | None = None, split_k: bool = False) -> list:
    """One grouped NVFP4 launch. Scale tensors are in the blocked layout.

    ``problem_sizes`` holds (m, n, k[, l]) per group. When ``b2``/``sfb2`` are given
    the launch is gated: ``c = fp16(silu(fp16(alpha*A.B^T)) * fp16(alpha2*A.B2^T))``.
    ``cta`` forces 256-row tiles on CTA pairs (``"pair"``), 128-row tiles on single
    CTAs (``"single"``) or the weight-stationary kernel's 128-weight-row x 64-token
    tiles (``"weights"``, non-gated only); by default the library picks pairs when the
    groups average at least 192 rows (96 with K >= 4096) and single CTAs otherwise.
    ``tile_n`` (128 or 256) applies to single-CTA tiles. ``split_k`` lets a single-CTA
    launch split the K loop of the tiles of its last, partly idle wave (the stream's
    workspace then also holds the split scratch, about 19 MB); results stay bit-identical
    from run to run.
    """
    if cta not in (None, "pair", "single", "weights"):
        raise ValueError(f"cta must be None, 'pair', 'single' or 'weights', got {cta!r}")
    G = len(problem_sizes)
    if not (len(a) == len(b) == len(sfa) == len(sfb) == len(c) == G):
        raise ValueError("a, b, sfa, sfb, c and problem_sizes must have one entry per group")
    gated = b2 is not None
    # Fast path: the same tensor objects at the same addresses, sizes, scales and tile
    # choice as the previous call on this stream were validated then, and the workspace
    # still holds their descriptors -> launch directly.
    sig = None
    if reuse_descriptors and G > 0 and isinstance(c[0], torch.Tensor) and c[0].is_cuda:
        lists = (a, b, sfa, sfb, c) + ((b2, sfb2) if gated else ())
        try:
            sig = (tuple(id(t) for lst in lists for t in lst),
                   tuple(t.data_ptr() for lst in lists for t in lst),
                   tuple(tuple(ps) for ps in problem_sizes),
                   None if alpha is None else tuple(alpha),
                   None if alpha2 is None else tuple(alpha2), tile_n, gated, cta, split_k)
        except (AttributeError, TypeError):
            sig = None
        if sig is not None:
            device = c[0].device
            s = stream or torch.cuda.current_stream(device)
            ws = _workspaces.get((device.index, s.cuda_stream))
            if ws is not None and ws.last_sig == sig and ws.last_table is not None:
                with torch.cuda.device(device):
                    if ws.plan is not None:  # the launch itself only
                        _native.check(_native.load_library().nvfp4_plan_launch(ws.plan,
                                                                               s.cuda_stream))
                    else:
                        _native.grouped_gemm_raw(ws.last_table,
                                                 ws.last_flags | _native.FLAG_REUSE_DESCRIPTORS,
                                                 ws.buf.data_ptr(), ws.nbytes, s.cuda_stream)
                return list(c)
    prepared = _prepare(a, b, sfa, sfb, c, problem_sizes, alpha, b2, sfb2, alpha2, tile_n, cta,
                        split_k)
    if prepared is None:
        return list(c)
    table, flags, device = prepared
    s = stream or torch.cuda.current_stream(device)
    ws = _workspace_for(device, s, _native.workspace_size_with_split(G) if split_k
                        else _native.workspace_size(G))
    same = (reuse_descriptors and ws.last_flags == flags and ws.last_table is not None
            and ws.last_table.shape == table.shape and np.array_equal(ws.last_table, table))
    lib = _native.load_library()
    with torch.cuda.device(device):
        if same and ws.plan is not None:
            _native.check(lib.nvfp4_plan_launch(ws.plan, s.cuda_stream), lib)
        elif reuse_descriptors and not split_k:
            # Upload once into a native prepared launch; repeated calls on the same tensors
            # then replay only the kernel launch.
            ws.drop_plan()
            out = ctypes.c_void_p()
            _native.check(lib.nvfp4_plan_create(table.ctypes.data, int(table.shape[0]), flags,
                                                ws.buf.data_ptr(), ws.nbytes, s.cuda_stream,
                                                ctypes.byref(out)), lib)
            ws.plan = out.value
            _native.check(lib.nvfp4_plan_launch(ws.plan, s.cuda_stream), lib)
        else:
            ws.drop_plan()
            call_flags = flags | (_native.FLAG_REUSE_DESCRIPTORS if same else 0)
            _native.grouped_gemm_raw(table, call_flags, ws.buf.data_ptr(), ws.nbytes,
                                     s.cuda_stream)
    ws.last_table = table
    ws.last_flags = flags
    ws.last_sig = sig
    return list(c)



def grouped_gemm_table(table: np.ndarray, flags: int, device: torch.device,
                       stream: torch.cuda.Stream | None = None) -> None:
    """Launch a prebuilt ``GROUP_DTYPE`` table (device pointers, sizes, scales) through this
    stream's workspace. For callers that assemble the table themselves from buffers they
    have already validated (the MoE block builds it from dispatch offsets in a few vectorised
    column operations); the library still checks every record before launching."""
    s = stream or torch.cuda.current_stream(device)
    G = int(table.shape[0])
    ws = _workspace_for(device, s, _native.workspace_size_with_split(G)
                        if flags & (_native.FLAG_SPLIT_K | _native.FLAG_STREAM_K)
                        else _native.workspace_size(G))
    with torch.cuda.device(device):
        _native.grouped_gemm_raw(table, flags, ws.buf.data_ptr(), ws.nbytes, s.cuda_stream)
    ws.drop_plan()
    ws.last_table = None  # the next grouped_gemm call on this stream rebuilds its descriptors
    ws.last_sig = None

def grouped_gemm_segments(a: torch.Tensor, sfa: torch.Tensor, c: torch.Tensor,
                          b: Sequence[torch.Tensor], sfb: Sequence[torch.Tensor],
                          seg_offsets: torch.Tensor, seg_counts: torch.Tensor,
                          alpha: Sequence[float] | None = None,
                          b2: Sequence[torch.Tensor] | None = None,
                          sfb2: Sequence[torch.Tensor] | None = None,
                          alpha2: Sequence[float] | None = None, expected_rows: int = 0,
                          cta: str | None = None, out_sf: torch.Tensor | None = None,
                          out_scale: float | None = None, row_dest: torch.Tensor | None = None,
                          dest: Sequence[torch.Tensor] | None = None,
                          stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Grouped GEMM over row segments of one slab, with the segments read on the GPU.

    ``a`` (packed e2m1 [R, K/2]), ``sfa`` (blocked scales of R rows) and ``c`` (fp16
    [R, N]) are slabs shared by all groups; group g multiplies rows
    ``[seg_offsets[g], seg_offsets[g] + seg_counts[g])`` of ``a`` by its weights ``b[g]``
    (with ``b2[g]`` for the gated form) into the same rows of ``c``. ``seg_offsets`` and
    ``seg_counts`` are int32 CUDA tensors, e.g. a routing step's output: nothing is read back
    to the host, so the call can be captured in a CUDA graph. Offsets must be multiples of
    128 inside the slab (a group that breaks this is skipped and :func:`check_device_errors`
    raises); the rows from a segment's end up to the next multiple of 128 may be
    overwritten. ``expected_rows`` (the host's estimate of the rows, e.g. tokens x top-k)
    picks the tile shape like the rows of :func:`grouped_gemm`; ``cta`` forces it.

    NVFP4 output (gated only): with ``out_sf`` (blocked scales of R rows x N) and
    ``out_scale``, ``c`` is a uint8 [R, N/2] slab that receives the e2m1 codes of the
    output, bit-identical to ``quantize(fp16 output, out_scale)``; N % 64 == 0.

    Scattered output (non-gated only): with ``row_dest`` (int64 CUDA tensor, one entry per
    slab row) and ``dest`` (up to 8 fp16 [*, N] tensors with the same row stride, which may
    live on peer GPUs), slab row r is stored to row ``row_dest[r] & (2**40 - 1)`` of
    ``dest[row_dest[r] >> 40]`` instead of ``c`` (negative entries: not stored).
    """
    if cta not in (None, "pair", "single"):
        raise ValueError(f"cta must be None, 'pair' or 'single', got {cta!r}")
    G = len(b)
    if len(sfb) != G:
        raise ValueError("b and sfb must have one entry per group")
    gated = b2 is not None
    if gated and (sfb2 is None or len(b2) != G or len(sfb2) != G):
        raise ValueError("b2 and sfb2 must both be given, one per group")
    for name, t in (("seg_offsets", seg_offsets), ("seg_counts", seg_counts)):
        if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous() or t.numel() < G:
            raise ValueError(f"{name} must be a contiguous CUDA int32 tensor of >= {G} entries")
    quant_out = out_sf is not None
    if quant_out:
        if not gated:
            raise ValueError("NVFP4 output (out_sf) is for gated launches")
        if out_scale is None or not (out_scale > 0) or not np.isfinite(out_scale):
            raise ValueError("out_scale must be finite and > 0 with out_sf")
        if c.dtype != torch.uint8 or c.dim() != 2 or not c.is_cuda:
            raise ValueError("with out_sf, c must be a CUDA uint8 [rows, N/2] tensor of codes")
        rows, n = int(c.shape[0]), int(c.shape[1]) * 2
        if n % 64:
            raise ValueError(f"N={n} must be a multiple of 64 for NVFP4 output")
        _as_2d_kmajor(c, rows, n // 2, "c")
        _check_sf(out_sf, rows, n, "out_sf")
    else:
        if c.dtype != torch.float16 or c.dim() != 2 or not c.is_cuda:
            raise ValueError("c must be a CUDA fp16 [rows, N] tensor")
        rows, n = int(c.shape[0]), int(c.shape[1])
        _as_2d_kmajor(c, rows, n, "c")  # dense fp16 rows
    scatter = None
    if row_dest is not None:
        if gated:
            raise ValueError("scattered output (row_dest) is for non-gated launches")
        if row_dest.dtype != torch.int64 or not row_dest.is_cuda or not row_dest.is_contiguous() \
                or row_dest.numel() < rows:
            raise ValueError(f"row_dest must be a contiguous CUDA int64 tensor of >= {rows} entries")
        if not dest or len(dest) > _native.EP_MAX_RANKS:
            raise ValueError(f"dest must hold 1..{_native.EP_MAX_RANKS} tensors")
        ld = int(dest[0].stride(0)) * 2
        for i, t in enumerate(dest):
            if t.dtype != torch.float16 or t.dim() != 2 or int(t.shape[1]) < n or \
                    t.stride(1) != 1 or int(t.stride(0)) * 2 != ld:
                raise ValueError(f"dest[{i}] must be fp16 [*, >= {n}] with the row stride of dest[0]")
        scatter = _native.SegmentOutput.scattered(row_dest.data_ptr(),
                                                  [t.data_ptr() for t in dest], ld)
    k = int(a.shape[1]) * 2 if a.dim() >= 2 else 0
    _check_fp4(a, "a")
    a = _as_2d_kmajor(a, rows, k // 2, "a")
    _check_sf(sfa, rows, k, "sfa")
    for g in range(G):
        _check_fp4(b[g], f"b[{g}]")
        _as_2d_kmajor(b[g], n, k // 2, f"b[{g}]")
        _check_sf(sfb[g], n, k, f"sfb[{g}]")
        if gated:
            _check_fp4(b2[g], f"b2[{g}]")
            _as_2d_kmajor(b2[g], n, k // 2, f"b2[{g}]")
            _check_sf(sfb2[g], n, k, f"sfb2[{g}]")
    device = c.device
    table = np.zeros(G, dtype=_native.GROUP_DTYPE)
    table["a"], table["sfa"], table["c"] = a.data_ptr(), sfa.data_ptr(), c.data_ptr()
    table["b"] = [t.data_ptr() for t in b]
    table["sfb"] = [t.data_ptr() for t in sfb]
    if gated:
        table["b2"] = [t.data_ptr() for t in b2]
        table["sfb2"] = [t.data_ptr() for t in sfb2]
    table["m"], table["n"], table["k"] = rows, n, k
    table["alpha"] = 1.0 if alpha is None else np.asarray(alpha, dtype=np.float32)
    table["alpha2"] = 1.0 if alpha2 is None else np.asarray(alpha2, dtype=np.float32)
    flags = _native.FLAG_GATED if gated else 0
    if cta == "pair":
        flags |= _native.FLAG_CTA_PAIR
    elif cta == "single":
        flags |= _native.FLAG_SINGLE_CTA
    if G == 0 or rows == 0:
        return c
    s = stream or torch.cuda.current_stream(device)
    ws = _workspace_for(device, s, _native.workspace_size(G))
    call_flags = flags
    if (ws.last_flags == flags and ws.last_table is not None
            and ws.last_table.shape == table.shape and np.array_equal(ws.last_table, table)):
        call_flags |= _native.FLAG_REUSE_DESCRIPTORS
    with torch.cuda.device(device):
        _native.grouped_gemm_segments_raw(table, call_flags, seg_offsets.data_ptr(),
                                          seg_counts.data_ptr(), int(expected_rows),
                                          ws.buf.data_ptr(), ws.nbytes, s.cuda_stream,
                                          _native.SegmentOutput.nvfp4(out_sf.data_ptr(), out_scale)
                                          if quant_out else scatter)
    ws.drop_plan()
    ws.last_table = table
    ws.last_flags = flags
    ws.last_sig = None
    return c


class GroupedGemmPlan:
    """A grouped launch validated once and then run many times on the same tensors.

    For callers that issue the same grouped GEMM repeatedly over fixed buffers (an
    MoE layer's expert weights and its activation and output slabs): the group table
    is checked and built once, the first run uploads the tensor maps, and every
    later run is a single library call that reuses them
    (``NVFP4_FLAG_REUSE_DESCRIPTORS``), with no per-tensor Python work. Arguments
    are those of :func:`grouped_gemm`. The tensors must keep their storage (same
    addresses and shapes) while the plan is used; their contents may change between
    runs. Runs of one plan share its workspace, so they must be ordered on the GPU
    (one stream, or synchronised streams).
    """

    def __init__(self, a, b, sfa, sfb, c, problem_sizes, *, alpha=None, b2=None, sfb2=None,
                 alpha2=None, tile_n=None, cta=None, split_k=False):
        prepared = _prepare(a, b, sfa, sfb, c, problem_sizes, alpha, b2, sfb2, alpha2, tile_n,
                            cta, split_k)
        self.outputs = list(c)
        self._keep = (a, b, sfa, sfb, c, b2, sfb2)  # the table holds their addresses
        self._table = None
        if prepared is None:
            return
        self._table, self._flags, self.device = prepared
        G = len(problem_sizes)
        self._nbytes = (_native.workspace_size_with_split(G) if split_k
                        else _native.workspace_size(G))
        # Zero-filled: the first 4 bytes are the device error word.
        self._ws = torch.zeros(self._nbytes, dtype=torch.uint8, device=self.device)
        self._lib = _native.load_library()
        self._uploaded = False
        # The first run makes a native plan (validates, uploads the descriptors, keeps the
        # launch); later runs replay only the kernel launch. Split-K launches keep the plain
        # entry point.
        self._native_plan = None
        self._use_native_plan = not split_k
        self._launch = self._lib.nvfp4_plan_launch

    def __del__(self):
        plan = getattr(self, "_native_plan", None)
        if plan is not None:
            self._lib.nvfp4_plan_destroy(plan)
            self._native_plan = None

    def run(self, stream: torch.cuda.Stream | None = None) -> list:
        """Launch on ``stream`` (default: the current stream); returns the outputs."""
        if self._table is None:
            return self.outputs
        idx = self.device.index
        plan = self._native_plan
        if plan is not None and torch.cuda.current_device() == idx:
            # Fast path: one native call that only launches the kernel.
            s = stream.cuda_stream if stream is not None else _current_raw_stream(idx)
            st = self._launch(plan, s)
            if st:
                _native.check(st, self._lib)
            return self.outputs
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        if self._use_native_plan:
            if plan is None:
                out = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    _native.check(self._lib.nvfp4_plan_create(
                        self._table.ctypes.data, int(self._table.shape[0]), self._flags,
                        self._ws.data_ptr(), self._nbytes, s, ctypes.byref(out)), self._lib)
                self._native_plan = plan = out.value
            with torch.cuda.device(self.device):
                _native.check(self._launch(plan, s), self._lib)
            self._uploaded = True
            return self.outputs
        flags = self._flags | (_native.FLAG_REUSE_DESCRIPTORS if self._uploaded else 0)
        args = (self._table.ctypes.data, int(self._table.shape[0]), flags, self._ws.data_ptr(),
                self._nbytes, s)
        if torch.cuda.current_device() == self.device.index:
            st = self._lib.nvfp4_grouped_gemm(*args)
        else:
            with torch.cuda.device(self.device):
                st = self._lib.nvfp4_grouped_gemm(*args)
        _native.check(st, self._lib)
        self._uploaded = True
        return self.outputs

    def check_device_errors(self, stream: torch.cuda.Stream | None = None) -> int:
        """Synchronise and return the device error bits of this plan's runs (raises
        ``Nvfp4Error`` when a kernel gave up waiting)."""
        if self._table is None:
            return 0
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        with torch.cuda.device(self.device):
            return _native.workspace_check(self._ws.data_ptr(), s)


# ----------------------------------------------------------------------------
# Reference-shaped entry points
# ----------------------------------------------------------------------------
def _split_scales(global_scales, G: int, gated: bool):
    if global_scales is None:
        return None, None
    gs = global_scales.detach().cpu().tolist() if isinstance(global_scales, torch.Tensor) \
        else list(global_scales)
    if len(gs) != G:
        raise ValueError(f"global_scales has {len(gs)} entries for {G} groups")
    if gated:
        pairs = [(float(x), float(x)) if np.isscalar(x) else (float(x[0]), float(x[1])) for x in gs]
        return [p[0] for p in pairs], [p[1] for p in pairs]
    return [float(x) for x in gs], None


class _CallCache:
    """The last grouped custom_kernel call that left a prepared launch in its stream's
    workspace: the same input object with the same tensors (identities and addresses), sizes
    and options may replay that launch without rebuilding anything."""

    __slots__ = ("data", "scales", "scales_val", "opts", "ids", "ptrs", "sizes", "ws", "sig",
                 "out", "ws_stream")


def _scales_value(global_scales):
    """A comparable copy of the global scales argument (lists may be changed in place)."""
    if global_scales is None:
        return None
    return tuple(tuple(x) if isinstance(x, (tuple, list)) else float(x) for x in global_scales)


_last_call: _CallCache | None = None


def _grouped_tensors(data) -> list:
    return [t for grp in data[0] for t in grp] + [t for grp in data[2] for t in grp]


def custom_kernel(data: input_t, *, global_scales=None, tile_n: int | None = None,
                  stream: torch.cuda.Stream | None = None, cta: str | None = None,
                  split_k: bool = False) -> output_t:
    """Drop-in replacement of the reference's ``custom_kernel`` (submission.py:788).
    The keyword options are those of :func:`grouped_gemm`."""
    global _last_call
    last = _last_call
    if (last is not None and data is last.data and global_scales is last.scales
            and (global_scales is None or _scales_value(global_scales) == last.scales_val)
            and last.opts == (tile_n, cta, split_k,
                              stream.cuda_stream if stream is not None else None)
            and last.ws.plan is not None and last.ws.last_sig is last.sig):
        ts = _grouped_tensors(data)
        if ([id(t) for t in ts] == last.ids and [t.data_ptr() for t in ts] == last.ptrs
                and [tuple(ps) for ps in data[3]] == last.sizes):
            dev = last.out[0].device
            if torch.cuda.current_device() == dev.index:
                s = stream.cuda_stream if stream is not None else _current_raw_stream(dev.index)
                if s == last.ws_stream:
                    st = _native.load_library().nvfp4_plan_launch(last.ws.plan, s)
                    if st:
                        _native.check(st)
                    return list(last.out)
    if not isinstance(data, (tuple, list)):
        raise ValueError(f"unsupported input: expected a tuple, got {type(data).__name__}")
    if len(data) == 10:
        a, b1, b2, _sfa, _sfb1, _sfb2, sfa_p, sfb1_p, sfb2_p, c = data
        if c.dim() == 3 and c.shape[2] != 1:
            raise ValueError("only L=1 is supported")
        m, n = int(c.shape[0]), int(c.shape[1])
        k = int(a.shape[1]) * 2
        alpha, alpha2 = _split_scales(global_scales, 1, True)
        grouped_gemm([a], [b1], [sfa_p], [sfb1_p], [c], [(m, n, k, 1)], alpha=alpha,
                     b2=[b2], sfb2=[sfb2_p], alpha2=alpha2, stream=stream, cta=cta,
                     split_k=split_k)
        return c
    if len(data) not in (4, 5):
        raise ValueError(f"unsupported input format with {len(data)} elements "
                         "(expected the 4-tuple grouped form or the 10-tuple dual form)")
    abc_tensors, _plain_sf, sf_reordered, problem_sizes = data[:4]
    if len(data) == 5:
        if global_scales is not None:
            raise ValueError("global scales given twice")
        global_scales = data[4]
    G = len(problem_sizes)
    if len(abc_tensors) != G or len(sf_reordered) != G:
        raise ValueError("abc_tensors, sf tensors and problem_sizes differ in length")
    if G == 0:
        return []
    gated = len(abc_tensors[0]) == 4
    if gated:
        a = [t[0] for t in abc_tensors]
        b = [t[1] for t in abc_tensors]
        b2 = [t[2] for t in abc_tensors]
        c = [t[3] for t in abc_tensors]
        if any(len(s) != 3 for s in sf_reordered):
            raise ValueError("gated grouped form needs (sfa, sfb_gate, sfb_up) per group")
        sfa = [s[0] for s in sf_reordered]
        sfb = [s[1] for s in sf_reordered]
        sfb2 = [s[2] for s in sf_reordered]
    else:
        if any(len(t) != 3 for t in abc_tensors):
            raise ValueError("grouped form needs (a, b, c) per group")
        a = [t[0] for t in abc_tensors]
        b = [t[1] for t in abc_tensors]
        c = [t[2] for t in abc_tensors]
        sfa = [s[0] for s in sf_reordered]
        sfb = [s[1] for s in sf_reordered]
        b2 = sfb2 = None
    alpha, alpha2 = _split_scales(global_scales, G, gated)
    grouped_gemm(a, b, sfa, sfb, c, problem_sizes, alpha=alpha, b2=b2, sfb2=sfb2,
                 alpha2=alpha2, tile_n=tile_n, stream=stream, cta=cta, split_k=split_k)
    # Remember the call if it left a prepared launch (see _CallCache).
    _last_call = None
    if len(data) == 4 and G > 0 and isinstance(c[0], torch.Tensor) and c[0].is_cuda:
        dev = c[0].device
        s = (stream or torch.cuda.current_stream(dev)).cuda_stream
        ws = _workspaces.get((dev.index, s))
        if ws is not None and ws.plan is not None and ws.last_sig is not None:
            entry = _CallCache()
            ts = _grouped_tensors(data)
            entry.data, entry.scales = data, global_scales
            entry.scales_val = _scales_value(global_scales)
            entry.opts = (tile_n, cta, split_k, stream.cuda_stream if stream is not None else None)
            entry.ids = [id(t) for t in ts]
            entry.ptrs = [t.data_ptr() for t in ts]
            entry.sizes = [tuple(ps) for ps in problem_sizes]
            entry.ws, entry.sig, entry.out = ws, ws.last_sig, list(c)
            entry.ws_stream = s
            _last_call = entry
    return list(c)


def solve(data: input_t) -> output_t:
    """Alias of custom_kernel (submission.py:889-891)."""
    return custom_kernel(data)
