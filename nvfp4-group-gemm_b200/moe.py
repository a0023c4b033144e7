"""An NVFP4 mixture-of-experts feed-forward block built around the grouped GEMM.

    x (bf16 [tokens, H]) --route--> per-expert rows --quantize+gather--> A (NVFP4)
      --gated grouped GEMM (gate/up, fused SiLU)--> h (fp16 [rows, I])
      --quantize--> h (NVFP4) --grouped GEMM (down)--> y (fp16 [rows, H])
      --weighted combine--> out (bf16 [tokens, H])

Every step is a kernel of this library (nvfp4_moe_route, nvfp4_quantize_rows,
nvfp4_grouped_gemm, nvfp4_moe_combine). Dispatched buffers give every expert's rows a
128-row-aligned range, so one blocked scale buffer serves all experts and every per-expert
operand is a view.

Two forms: ``moe_ffn`` reads the per-expert row counts once per call (one device -> host
copy) and sizes its buffers and group tables to them; ``MoEBlock`` sizes every buffer once
for a token count, keeps the routing metadata on the GPU and runs both expert GEMMs through
nvfp4_grouped_gemm_segments, so a call is a fixed sequence of launches with no host read,
which ``MoEBlock.capture`` records in a CUDA graph. Its gate/up GEMM writes the SiLU output
directly as NVFP4 codes and scales (the separate quantise-h pass and the fp16 h are gone).

The reference has no counterpart: it runs a grouped GEMM whose groups arrive already formed
and quantised. This is the surrounding layer (token dispatch, activation quantisation,
down-projection and combine) that a model calls.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _native
from .interface import grouped_gemm_table
from .layout import blocked_sf_bytes
from .quantize import _DTYPES, global_scale_for, quantize


@dataclass
class Routing:
    """Dispatch metadata of one batch (see nvfp4_moe_route)."""

    tokens: int
    topk: int
    num_experts: int
    counts: list            # rows per expert (host)
    offsets: list           # first dispatched row per expert, 128-aligned (host, E + 1 entries)
    dest: torch.Tensor      # int32 [tokens * topk] dispatched row of each pair (-1: dropped)
    src_rows: torch.Tensor  # int32 [capacity] token of each dispatched row (-1: padding)

    @property
    def rows(self) -> int:
        """Dispatched rows including each expert's padding to a multiple of 128."""
        return self.offsets[-1]


def route(topk_ids: torch.Tensor, num_experts: int, stream: torch.cuda.Stream | None = None) -> Routing:
    """Route (token, slot) pairs to experts: ``topk_ids`` int32 [tokens, topk] on the GPU."""
    if topk_ids.dtype != torch.int32 or topk_ids.dim() != 2 or not topk_ids.is_cuda:
        raise ValueError("topk_ids must be a CUDA int32 tensor [tokens, topk]")
    ids = topk_ids.contiguous()
    tokens, topk = int(ids.shape[0]), int(ids.shape[1])
    dev = ids.device
    pairs = tokens * topk
    capacity = pairs + 127 * num_experts
    meta = torch.empty(2 * num_experts + 1, dtype=torch.int32, device=dev)
    counts, offsets = meta[:num_experts], meta[num_experts:]
    dest = torch.empty(max(pairs, 1), dtype=torch.int32, device=dev)
    src_rows = torch.empty(max(capacity, 1), dtype=torch.int32, device=dev)
    lib = _native.load_library()
    ws_bytes = int(lib.nvfp4_moe_route_workspace_size(pairs, num_experts))
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    s = stream or torch.cuda.current_stream(dev)
    with torch.cuda.device(dev):
        _native.check(lib.nvfp4_moe_route(ids.data_ptr(), tokens, topk, num_experts,
                                          counts.data_ptr(), offsets.data_ptr(), dest.data_ptr(),
                                          src_rows.data_ptr(), capacity, ws.data_ptr(), ws_bytes,
                                          s.cuda_stream), lib)
    host = meta.cpu().tolist()  # the one host read of the call
    return Routing(tokens, topk, num_experts, host[:num_experts], host[num_experts:],
                   dest[:pairs], src_rows)


def quantize_rows(x: torch.Tensor, rows: int, src_rows: torch.Tensor, mode: int,
                  global_scale: float, stream: torch.cuda.Stream | None = None) -> tuple:
    """nvfp4_quantize_rows: ``rows`` output rows through a row map (gather or mask)."""
    if x.dtype not in _DTYPES or x.dim() != 2 or x.stride(1) != 1 or not x.is_cuda:
        raise ValueError("x must be a CUDA bf16/fp16 2-D tensor with unit inner stride")
    cols = int(x.shape[1])
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
    sf = torch.empty(max(blocked_sf_bytes(rows, cols // 16), 16), dtype=torch.uint8, device=x.device)
    s = stream or torch.cuda.current_stream(x.device)
    lib = _native.load_library()
    with torch.cuda.device(x.device):
        _native.check(lib.nvfp4_quantize_rows(x.data_ptr(), rows, cols, x.stride(0), _DTYPES[x.dtype],
                                              float(global_scale), src_rows.data_ptr(), mode,
                                              packed.data_ptr(), packed.stride(0), sf.data_ptr(),
                                              s.cuda_stream), lib)
    return packed, sf


def gather_quantized(packed: torch.Tensor, sf: torch.Tensor, routing: Routing,
                     stream: torch.cuda.Stream | None = None) -> tuple:
    """Dispatch already-quantised token rows (``quantize(x)``'s packed codes and blocked
    scales) into the dispatched order: bit-identical to quantising the gathered rows, with a
    quarter of the bytes moved per dispatched row."""
    rows = routing.rows
    cols = int(packed.shape[1]) * 2
    out = torch.empty((rows, cols // 2), dtype=torch.uint8, device=packed.device)
    out_sf = torch.empty(max(blocked_sf_bytes(rows, cols // 16), 16), dtype=torch.uint8,
                         device=packed.device)
    s = stream or torch.cuda.current_stream(packed.device)
    lib = _native.load_library()
    with torch.cuda.device(packed.device):
        _native.check(lib.nvfp4_moe_gather_quantized(
            packed.data_ptr(), packed.stride(0), sf.data_ptr(), routing.src_rows.data_ptr(), rows,
            cols, out.data_ptr(), out.stride(0), out_sf.data_ptr(), s.cuda_stream), lib)
    return out, out_sf


def combine(y: torch.Tensor, routing: Routing, topk_weights: torch.Tensor,
            stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out[t] = sum_j w[t, j] * y[dest[t, j]] (fp32 accumulation, bf16 result)."""
    if y.dtype != torch.float16 or y.dim() != 2 or y.stride(1) != 1:
        raise ValueError("y must be fp16 [rows, cols] with unit inner stride")
    w = topk_weights.to(torch.float32).contiguous()
    if tuple(w.shape) != (routing.tokens, routing.topk):
        raise ValueError("topk_weights must be [tokens, topk]")
    cols = int(y.shape[1])
    out = torch.empty((routing.tokens, cols), dtype=torch.bfloat16, device=y.device)
    s = stream or torch.cuda.current_stream(y.device)
    lib = _native.load_library()
    with torch.cuda.device(y.device):
        _native.check(lib.nvfp4_moe_combine(y.data_ptr(), y.stride(0), routing.dest.data_ptr(),
                                            w.data_ptr(), routing.tokens, routing.topk, cols,
                                            out.data_ptr(), out.stride(0), s.cuda_stream), lib)
    return out


def expert_views(routing: Routing, packed: torch.Tensor, sf: torch.Tensor, out: torch.Tensor,
                 k: int) -> tuple:
    """Per-expert A, scale and output views into dispatched buffers (no copies)."""
    sf_block = (k // 64) * 512  # bytes of one 128-row block of scales
    a, sfa, c, m = [], [], [], []
    for e in range(routing.num_experts):
        r0, n_e = routing.offsets[e], routing.counts[e]
        a.append(packed[r0:r0 + n_e])
        b0 = (r0 // 128) * sf_block
        sfa.append(sf[b0:b0 + max(blocked_sf_bytes(n_e, k // 16), 0)])
        c.append(out[r0:r0 + n_e])
        m.append(n_e)
    return a, sfa, c, m


@dataclass
class ExpertWeights:
    """NVFP4 weights of the experts: gate/up [I, H] and down [H, I] per expert (packed codes,
    blocked scales) with their per-expert global scales."""

    w_gate: list
    sf_gate: list
    w_up: list
    sf_up: list
    w_down: list
    sf_down: list
    s_gate: list
    s_up: list
    s_down: list

    @property
    def num_experts(self) -> int:
        return len(self.w_gate)

    def pointers(self) -> dict:
        """Device addresses of every expert's weights and scales (computed once)."""
        if getattr(self, "_ptrs", None) is None:
            self._ptrs = {name: np.array([t.data_ptr() for t in getattr(self, name)], dtype=np.uint64)
                          for name in ("w_gate", "sf_gate", "w_up", "sf_up", "w_down", "sf_down")}
        return self._ptrs


def quantize_expert_weights(gate: list, up: list, down: list) -> ExpertWeights:
    """Quantise bf16 expert weights (gate/up [I, H], down [H, I]) with this library's kernel."""
    out = {k: [] for k in ("w_gate", "sf_gate", "w_up", "sf_up", "w_down", "sf_down",
                           "s_gate", "s_up", "s_down")}
    for g, u, d in zip(gate, up, down):
        for name, w in (("gate", g), ("up", u), ("down", d)):
            s = global_scale_for(w)
            q, sf = quantize(w, s)
            out[f"w_{name}"].append(q)
            out[f"sf_{name}"].append(sf)
            out[f"s_{name}"].append(s)
    return ExpertWeights(**out)


def dispatched_table(routing: Routing, a: torch.Tensor, sfa: torch.Tensor, c: torch.Tensor,
                     b_ptrs: np.ndarray, sfb_ptrs: np.ndarray, n: int, k: int, alpha: np.ndarray,
                     b2_ptrs: np.ndarray | None = None, sfb2_ptrs: np.ndarray | None = None,
                     alpha2: np.ndarray | None = None) -> np.ndarray:
    """Group table of a grouped GEMM over dispatched buffers: expert e's A rows, scale block
    and output rows start at routing.offsets[e]; built with vectorised column operations."""
    E = routing.num_experts
    off = np.asarray(routing.offsets[:E], dtype=np.uint64)
    t = np.zeros(E, dtype=_native.GROUP_DTYPE)
    t["a"] = a.data_ptr() + off * np.uint64(k // 2)
    t["sfa"] = sfa.data_ptr() + (off // np.uint64(128)) * np.uint64((k // 64) * 512)
    t["c"] = c.data_ptr() + off * np.uint64(n * c.element_size())
    t["b"], t["sfb"] = b_ptrs, sfb_ptrs
    if b2_ptrs is not None:
        t["b2"], t["sfb2"] = b2_ptrs, sfb2_ptrs
        t["alpha2"] = alpha2
    else:
        t["alpha2"] = 1.0
    t["m"] = np.asarray(routing.counts, dtype=np.int32)
    t["n"], t["k"] = n, k
    t["alpha"] = alpha
    return t


def moe_ffn(x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
            weights: ExpertWeights, act_scale: float | None = None,
            hidden_scale: float | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """One MoE feed-forward block: out[t] = sum_j w[t, j] * down_e(silu(gate_e(x_t)) * up_e(x_t))
    with e = topk_ids[t, j], all products in NVFP4 with fp32 accumulation.

    ``act_scale`` / ``hidden_scale`` are the per-tensor scales of x and of the SiLU output;
    when None they are computed from the data (one device reduction and host read each).
    """
    tokens, hdim = int(x.shape[0]), int(x.shape[1])
    E = weights.num_experts
    idim = int(weights.w_gate[0].shape[0])
    if hdim % 256 or idim % 256:
        raise ValueError(f"hidden ({hdim}) and intermediate ({idim}) sizes must be multiples of 256 "
                         "(the K of the two grouped GEMMs)")
    r = route(topk_ids, E, stream)
    s_x = global_scale_for(x) if act_scale is None else act_scale
    # Each token is quantised once and its codes and scales are gathered topk times.
    qx, sfx = quantize(x, s_x, stream=stream)
    a, sfa = gather_quantized(qx, sfx, r, stream)
    # Padding rows of h are never written by the GEMM; zero them when the SiLU output's
    # scale is computed from the data, so that they cannot enter its amax.
    alloc = torch.zeros if hidden_scale is None else torch.empty
    h = alloc((max(r.rows, 1), idim), dtype=torch.float16, device=x.device)
    P = weights.pointers()
    t1 = dispatched_table(r, a, sfa, h, P["w_gate"], P["sf_gate"], idim, hdim,
                          s_x * np.asarray(weights.s_gate, dtype=np.float32),
                          P["w_up"], P["sf_up"], s_x * np.asarray(weights.s_up, dtype=np.float32))
    grouped_gemm_table(t1, _native.FLAG_GATED, x.device, stream)
    s_h = global_scale_for(h) if hidden_scale is None else hidden_scale
    a2, sfa2 = quantize_rows(h, r.rows, r.src_rows, _native.ROWS_MASK, s_h, stream)
    y = torch.empty((max(r.rows, 1), hdim), dtype=torch.float16, device=x.device)
    t2 = dispatched_table(r, a2, sfa2, y, P["w_down"], P["sf_down"], hdim, idim,
                          s_h * np.asarray(weights.s_down, dtype=np.float32))
    grouped_gemm_table(t2, 0, x.device, stream)
    return combine(y, r, topk_weights, stream)


class MoEBlock:
    """The MoE feed-forward block over buffers sized once for ``tokens`` x ``topk``, with no
    device -> host read in :meth:`run`.

    Routing metadata (per-expert counts and 128-aligned offsets, each pair's dispatched row,
    each dispatched row's token) stays on the GPU; the gate/up and down GEMMs run over the
    whole dispatched slabs and take every expert's rows from the device
    (nvfp4_grouped_gemm_segments), the gate/up GEMM writing NVFP4 codes and scales of the
    SiLU output for the down GEMM (bit-identical to quantising its fp16 output). The
    per-tensor scales of x and of the SiLU output are
    fixed at construction (calibrated scales). Dispatched slabs hold ``tokens * topk +
    127 * experts`` rows, the most any routing can need.

    :meth:`run` returns ``self.out`` (bf16 [tokens, H]), overwritten by the next run.
    :meth:`capture` records one run into a CUDA graph over the given input tensors; each
    replay recomputes the block from whatever those tensors hold at that time.
    """

    def __init__(self, weights: ExpertWeights, tokens: int, topk: int, act_scale: float,
                 hidden_scale: float, device: torch.device | None = None,
                 cta: str | None = None):
        if cta not in (None, "pair", "single"):
            raise ValueError(f"cta must be None, 'pair' or 'single', got {cta!r}")
        self._cta_flags = {None: 0, "pair": _native.FLAG_CTA_PAIR,
                           "single": _native.FLAG_SINGLE_CTA}[cta]
        if not (act_scale > 0 and hidden_scale > 0):
            raise ValueError("act_scale and hidden_scale must be positive")
        dev = torch.device(device) if device is not None else weights.w_gate[0].device
        E = weights.num_experts
        idim = int(weights.w_gate[0].shape[0])
        hdim = int(weights.w_gate[0].shape[1]) * 2
        if hdim % 256 or idim % 256:
            raise ValueError(f"hidden ({hdim}) and intermediate ({idim}) sizes must be multiples "
                             "of 256 (the K of the two grouped GEMMs)")
        if tokens <= 0 or topk <= 0:
            raise ValueError("tokens and topk must be positive")
        self.tokens, self.topk, self.num_experts = tokens, topk, E
        self.hidden, self.intermediate = hdim, idim
        self.act_scale, self.hidden_scale = float(act_scale), float(hidden_scale)
        self.device = dev
        pairs = tokens * topk
        cap = pairs + 127 * E
        self.capacity = cap
        i32 = dict(dtype=torch.int32, device=dev)
        u8 = dict(dtype=torch.uint8, device=dev)
        self._meta = torch.zeros(2 * E + 1, **i32)
        self.counts, self.offsets = self._meta[:E], self._meta[E:]
        self.dest = torch.empty(pairs, **i32)
        self.src_rows = torch.empty(cap, **i32)
        lib = _native.load_library()
        self._lib = lib
        self._route_ws_bytes = int(lib.nvfp4_moe_route_workspace_size(pairs, E))
        self._route_ws = torch.empty(max(self._route_ws_bytes, 16), **u8)
        self._qx = torch.empty((tokens, hdim // 2), **u8)
        self._sfx = torch.empty(blocked_sf_bytes(tokens, hdim // 16), **u8)
        self._a = torch.empty((cap, hdim // 2), **u8)
        self._sfa = torch.empty(blocked_sf_bytes(cap, hdim // 16), **u8)
        # Codes and scales of the SiLU output (padding rows keep these zeros or earlier data).
        self._a2 = torch.zeros((cap, idim // 2), **u8)
        self._sfa2 = torch.zeros(blocked_sf_bytes(cap, idim // 16), **u8)
        self._y = torch.empty((cap, hdim), dtype=torch.float16, device=dev)
        self._w = torch.empty((tokens, topk), dtype=torch.float32, device=dev)
        self.out = torch.empty((tokens, hdim), dtype=torch.bfloat16, device=dev)
        P = weights.pointers()
        self._weights = weights  # the tables hold its addresses

        def slab_table(a, sfa, c, b, sfb, n, k, alpha, b2=None, sfb2=None, alpha2=None):
            t = np.zeros(E, dtype=_native.GROUP_DTYPE)
            t["a"], t["sfa"], t["c"] = a.data_ptr(), sfa.data_ptr(), c.data_ptr()
            t["b"], t["sfb"] = b, sfb
            if b2 is not None:
                t["b2"], t["sfb2"], t["alpha2"] = b2, sfb2, alpha2
            else:
                t["alpha2"] = 1.0
            t["m"], t["n"], t["k"], t["alpha"] = cap, n, k, alpha
            return t

        s_x, s_h = self.act_scale, self.hidden_scale
        self._t1 = slab_table(self._a, self._sfa, self._a2, P["w_gate"], P["sf_gate"], idim, hdim,
                              s_x * np.asarray(weights.s_gate, dtype=np.float32),
                              P["w_up"], P["sf_up"],
                              s_x * np.asarray(weights.s_up, dtype=np.float32))
        self._t2 = slab_table(self._a2, self._sfa2, self._y, P["w_down"], P["sf_down"], hdim,
                              idim, s_h * np.asarray(weights.s_down, dtype=np.float32))
        self._nvfp4_out = _native.SegmentOutput.nvfp4(self._sfa2.data_ptr(), self.hidden_scale)
        ws_bytes = _native.workspace_size(E)
        # Zero-filled: the first 4 bytes are the device error word.
        self._ws1 = torch.zeros(ws_bytes, **u8)
        self._ws2 = torch.zeros(ws_bytes, **u8)
        self._ws_bytes = ws_bytes
        self._uploaded = False

    def _check_inputs(self, x, topk_ids, topk_weights):
        if x.dtype not in _DTYPES or tuple(x.shape) != (self.tokens, self.hidden) or \
                x.stride(1) != 1 or x.device != self.device:
            raise ValueError(f"x must be bf16/fp16 [{self.tokens}, {self.hidden}] on {self.device}")
        if topk_ids.dtype != torch.int32 or tuple(topk_ids.shape) != (self.tokens, self.topk) or \
                not topk_ids.is_contiguous() or topk_ids.device != self.device:
            raise ValueError(f"topk_ids must be contiguous int32 [{self.tokens}, {self.topk}]")
        if tuple(topk_weights.shape) != (self.tokens, self.topk) or \
                topk_weights.device != self.device:
            raise ValueError(f"topk_weights must be [{self.tokens}, {self.topk}]")

    def run(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
            stream: torch.cuda.Stream | None = None, stage_events: list | None = None) -> torch.Tensor:
        """One block on ``stream``: route, quantise x once per token, dispatch codes and
        scales, gated GEMM (segments, NVFP4 output), down GEMM (segments), combine. With
        ``stage_events`` (a list, eager runs only), (stage name, CUDA event recorded after
        it) pairs are appended for timing."""
        self._check_inputs(x, topk_ids, topk_weights)
        lib = self._lib
        st = stream or torch.cuda.current_stream(self.device)
        s = st.cuda_stream

        def mark(name):
            if stage_events is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(st)
                stage_events.append((name, ev))

        mark("start")
        E, T, K, H, cap = self.num_experts, self.tokens, self.topk, self.hidden, self.capacity
        chk = _native.check
        with torch.cuda.device(self.device):
            chk(lib.nvfp4_moe_route(topk_ids.data_ptr(), T, K, E, self.counts.data_ptr(),
                                    self.offsets.data_ptr(), self.dest.data_ptr(),
                                    self.src_rows.data_ptr(), cap, self._route_ws.data_ptr(),
                                    self._route_ws_bytes, s), lib)
            mark("route")
            chk(lib.nvfp4_quantize(x.data_ptr(), T, H, x.stride(0), _DTYPES[x.dtype],
                                   self.act_scale, self._qx.data_ptr(), self._qx.stride(0),
                                   self._sfx.data_ptr(), s), lib)
            mark("quantise x")
            chk(lib.nvfp4_moe_gather_quantized(self._qx.data_ptr(), self._qx.stride(0),
                                               self._sfx.data_ptr(), self.src_rows.data_ptr(), cap,
                                               H, self._a.data_ptr(), self._a.stride(0),
                                               self._sfa.data_ptr(), s), lib)
            mark("dispatch (gather codes + scales)")
            flags = (_native.FLAG_REUSE_DESCRIPTORS if self._uploaded else 0) | self._cta_flags
            _native.grouped_gemm_segments_raw(self._t1, _native.FLAG_GATED | flags,
                                              self.offsets.data_ptr(), self.counts.data_ptr(),
                                              T * K, self._ws1.data_ptr(), self._ws_bytes, s,
                                              self._nvfp4_out)
            mark("gate/up GEMM + SiLU (NVFP4 output)")
            _native.grouped_gemm_segments_raw(self._t2, flags, self.offsets.data_ptr(),
                                              self.counts.data_ptr(), T * K,
                                              self._ws2.data_ptr(), self._ws_bytes, s)
            mark("down GEMM")
            self._uploaded = True
            w = topk_weights
            if w.dtype != torch.float32 or not w.is_contiguous():
                with torch.cuda.stream(st):
                    self._w.copy_(w)
                w = self._w
            chk(lib.nvfp4_moe_combine(self._y.data_ptr(), self._y.stride(0), self.dest.data_ptr(),
                                      w.data_ptr(), T, K, H, self.out.data_ptr(),
                                      self.out.stride(0), s), lib)
            mark("combine")
        return self.out

    def check_device_errors(self) -> int:
        """Synchronise and return the device error bits of both GEMM workspaces (raises
        Nvfp4Error when a segment was out of range or a wait timed out)."""
        s = torch.cuda.current_stream(self.device).cuda_stream
        with torch.cuda.device(self.device):
            return (_native.workspace_check(self._ws1.data_ptr(), s) |
                    _native.workspace_check(self._ws2.data_ptr(), s))

    def capture(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                warmup: int = 1) -> torch.cuda.CUDAGraph:
        """Record one run over these input tensors into a CUDA graph (after ``warmup`` eager
        runs, which upload the GEMMs' descriptors so the graph holds only their launches).
        ``graph.replay()`` then recomputes ``self.out`` from the tensors' current contents."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(max(warmup, 1)):
                self.run(x, topk_ids, topk_weights, side)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self.run(x, topk_ids, topk_weights, side)
        return graph
