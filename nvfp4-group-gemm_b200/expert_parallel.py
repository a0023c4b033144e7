"""Expert-parallel sharding of a grouped NVFP4 GEMM across the GPUs of one node.

Groups (experts) are independent work units, so each rank owns a contiguous
slice of experts and runs the grouped kernel on it with no collective on the
data path. An optional all-gather makes every expert's fp16 output available on
every rank (NCCL over NVLink on GPUs; any torch.distributed backend works since
the exchange moves raw bytes).

The reference is single-GPU; this module has no counterpart there.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def expert_shard(num_experts: int, world_size: int, rank: int) -> range:
    """Contiguous, balanced slice of experts owned by `rank` (first ranks take the remainder)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of size {world_size}")
    if num_experts < 0:
        raise ValueError("num_experts must be >= 0")
    base, extra = divmod(num_experts, world_size)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def slab_layout(rows_per_expert: Sequence[int], n: int, world_size: int) -> list:
    """Per rank: (first expert, expert count, slab elements) of its fp16 output slab."""
    out = []
    G = len(rows_per_expert)
    for r in range(world_size):
        sh = expert_shard(G, world_size, r)
        out.append((sh.start, len(sh), int(sum(rows_per_expert[sh.start:sh.stop])) * n))
    return out


def all_gather_expert_outputs(local_outputs: Sequence[torch.Tensor],
                              rows_per_expert: Sequence[int], n: int,
                              group: dist.ProcessGroup | None = None) -> list:
    """All-gather every rank's per-expert outputs ([M_g, n] fp16) onto every rank.

    Each rank packs its experts' outputs into one slab, slabs are padded to the
    largest slab and exchanged with one all_gather of bytes, then split back into
    one tensor per expert in global expert order.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    layout = slab_layout(rows_per_expert, n, world)
    first, count, elems = layout[rank]
    if len(local_outputs) != count:
        raise ValueError(f"rank {rank} owns {count} experts, got {len(local_outputs)} outputs")
    device = local_outputs[0].device if local_outputs else (
        torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl"
        else torch.device("cpu"))
    max_elems = max(e for _, _, e in layout)
    send = torch.zeros(max_elems, dtype=torch.float16, device=device)
    off = 0
    for t, m in zip(local_outputs, rows_per_expert[first:first + count]):
        if tuple(t.shape[:2]) != (m, n):
            raise ValueError(f"expert output shape {tuple(t.shape)} != ({m}, {n})")
        send[off:off + m * n] = t.reshape(-1)
        off += m * n
    recv = torch.empty(world * max_elems, dtype=torch.float16, device=device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(recv.view(torch.uint8), send.view(torch.uint8), group=group)
    else:
        dist.all_gather(list(recv.view(torch.uint8).chunk(world)), send.view(torch.uint8),
                        group=group)
    outs = []
    for r, (f, cnt, _) in enumerate(layout):
        base = r * max_elems
        o = 0
        for g in range(f, f + cnt):
            m = rows_per_expert[g]
            outs.append(recv[base + o: base + o + m * n].view(m, n))
            o += m * n
    return outs


class ExpertOutputGather:
    """Preallocated all-gather of every rank's per-expert fp16 outputs.

    The same exchange as :func:`all_gather_expert_outputs` without its packing copy and
    per-call allocations: ``local_outputs`` are [M_g, n] views into this rank's part of
    the send slab, so the grouped GEMM writes its outputs where NCCL reads them, and
    :meth:`run` is one ``all_gather_into_tensor``. ``outputs`` are views of the receive
    slab in global expert order (rank r's experts expert_shard(G, P, r)); their contents
    are those of the last :meth:`run`.
    """

    def __init__(self, rows_per_expert: Sequence[int], n: int, device: torch.device,
                 group: dist.ProcessGroup | None = None):
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.rows = [int(m) for m in rows_per_expert]
        self.n = int(n)
        layout = slab_layout(self.rows, self.n, world)
        self.max_elems = max(e for _, _, e in layout)
        self.send = torch.zeros(self.max_elems, dtype=torch.float16, device=device)
        self.recv = torch.empty(world * self.max_elems, dtype=torch.float16, device=device)
        first, count, _ = layout[rank]
        self.local_outputs = self._views(self.send, 0, first, count)
        self.outputs = []
        for r, (f, cnt, _) in enumerate(layout):
            self.outputs += self._views(self.recv, r * self.max_elems, f, cnt)
        self.bytes_received = int((world - 1) * self.max_elems * 2)

    def _views(self, buf: torch.Tensor, base: int, first: int, count: int) -> list:
        out, off = [], base
        for g in range(first, first + count):
            m = self.rows[g]
            out.append(buf[off:off + m * self.n].view(m, self.n))
            off += m * self.n
        return out

    def run(self) -> list:
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self.recv.view(torch.uint8), self.send.view(torch.uint8),
                                        group=self.group)
        else:
            world = dist.get_world_size(self.group)
            dist.all_gather(list(self.recv.view(torch.uint8).chunk(world)),
                            self.send.view(torch.uint8), group=self.group)
        return self.outputs


class ProcessGroupFabric:
    """How the ranks of an expert-parallel group reach each other: one process per GPU in a
    torch.distributed group (NCCL). Buffers come from torch symmetric memory, so every rank
    maps every peer's copy over NVLink; the barrier is a one-element NCCL all-reduce on the
    caller's stream (capturable in a CUDA graph); :meth:`meet` is a host-side barrier.

    A fabric exposes ``world``, ``rank``, ``allocate(nbytes, device) -> (tensor, bases)``
    (a zeroed uint8 tensor and, per rank, the device address of that rank's copy of its
    first byte), ``barrier(device)`` and ``meet()``; :class:`FusedOutputGather` and
    :class:`EPMoEBlock` take one as ``fabric=``."""

    def __init__(self, group: dist.ProcessGroup | None = None):
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self._handles = []  # rendezvous handles keep the peers' mappings alive
        self._bar = None

    def allocate(self, nbytes: int, device: torch.device):
        from torch.distributed import _symmetric_memory as symm

        buf = symm.empty(nbytes, dtype=torch.uint8, device=device)
        buf.zero_()
        try:
            handle = symm.rendezvous(buf, self.group)
        except RuntimeError:  # older releases want the group registered first
            symm.enable_symm_mem_for_group(self.group.group_name)
            handle = symm.rendezvous(buf, self.group)
        self._handles.append(handle)
        if self._bar is None:  # made here, not in the first barrier (which may be captured)
            self._bar = torch.zeros(1, dtype=torch.int32, device=device)
        bases = [int(b) for b in handle.buffer_ptrs]
        # The tensor sits at the same offset inside every rank's copy of the allocation.
        delta = buf.data_ptr() - bases[self.rank]
        return buf, [b + delta for b in bases]

    def barrier(self, device: torch.device) -> None:
        if self._bar is None or self._bar.device != device:
            self._bar = torch.zeros(1, dtype=torch.int32, device=device)
        dist.all_reduce(self._bar, group=self.group)

    def meet(self) -> None:
        dist.barrier(group=self.group)


class SingleDeviceFabric:
    """Every rank of an expert-parallel group emulated on one GPU.

    Rank r's buffers are plain allocations on ``device``, so a "peer" address is an address
    of the same GPU and the exchange kernels, the replicated GEMM epilogue and the return
    paths run exactly as across GPUs, minus NVLink. The ranks' calls run one after another
    on one stream (:func:`run_lockstep`), and stream order stands in for the barriers: no
    kernel of this library waits on another rank, so the emulation cannot deadlock, and
    it replays one of the interleavings the real ranks may take. Used to test world sizes
    up to 8 on a one-GPU machine and to check a deployment's layouts before it gets GPUs.

    ``fabric.rank_view(r)`` is the object to pass as ``fabric=`` to rank r's block; every
    rank must allocate the same sizes in the same order (as every rank's constructor does).
    """

    def __init__(self, world: int, device: torch.device):
        if world < 1:
            raise ValueError("world must be >= 1")
        self.world = int(world)
        self.device = torch.device(device)
        self._allocs = []             # per allocation: one tensor per rank
        self._next = [0] * self.world  # allocations made so far, per rank

    def rank_view(self, rank: int) -> "_EmulatedRank":
        if not 0 <= rank < self.world:
            raise ValueError(f"rank {rank} outside world of size {self.world}")
        return _EmulatedRank(self, rank)


class _EmulatedRank:
    """One rank of a :class:`SingleDeviceFabric` (the ``fabric=`` argument of its blocks)."""

    def __init__(self, fabric: SingleDeviceFabric, rank: int):
        self.fabric, self.world, self.rank = fabric, fabric.world, rank

    def allocate(self, nbytes: int, device: torch.device):
        f = self.fabric
        if torch.device(device) != f.device:
            raise ValueError(f"emulated ranks live on {f.device}, not {device}")
        i = f._next[self.rank]
        f._next[self.rank] += 1
        if i == len(f._allocs):
            f._allocs.append([torch.zeros(nbytes, dtype=torch.uint8, device=f.device)
                              for _ in range(f.world)])
        bufs = f._allocs[i]
        if bufs[self.rank].numel() != nbytes:
            raise ValueError(f"rank {self.rank} asks for {nbytes} bytes in allocation {i}, "
                             f"another rank for {bufs[self.rank].numel()}")
        return bufs[self.rank], [b.data_ptr() for b in bufs]

    def barrier(self, device: torch.device) -> None:
        pass  # one stream: stream order is the barrier

    def meet(self) -> None:
        pass


def run_lockstep(blocks: Sequence, inputs: Sequence) -> list:
    """One call of every emulated rank's :class:`EPMoEBlock` (blocks built on the rank views
    of one :class:`SingleDeviceFabric`, ``inputs[r] = (x, topk_ids, topk_weights)``): the
    ranks' phases run in rank order on the current stream, each barrier point reached by
    every rank before any rank passes it. Returns every rank's ``out``."""
    if len(blocks) != len(inputs):
        raise ValueError("one input triple per block")
    pending = [blk.phases(*inp) for blk, inp in zip(blocks, inputs)]
    while pending:
        alive = []
        for g in pending:
            try:
                next(g)
                alive.append(g)
            except StopIteration:
                pass
        if alive and len(alive) != len(pending):
            raise RuntimeError("the ranks' calls reached different numbers of barriers")
        pending = alive
    return [blk.out for blk in blocks]


class FusedOutputGather:
    """The output all-gather of an expert-parallel grouped GEMM, fused into the GEMM.

    One allocation of the fabric (``fabric=``; by default torch symmetric memory over the
    process group, :class:`ProcessGroupFabric`) holds, on every rank, the fp16 output slab
    of every rank (rank r's experts ``expert_shard(G, P, r)`` in slab r, the layout of
    :class:`ExpertOutputGather`'s receive buffer). :meth:`gemm` runs this rank's experts with
    ``nvfp4_grouped_gemm_replicated``: the kernel stores each output tile into this rank's
    slab locally and, from its epilogue, into the same slab of every other rank's copy over
    NVLink, so the exchange overlaps the math tile by tile. After :meth:`barrier` (a
    one-element NCCL all-reduce on the stream) every rank holds every expert's output in
    ``outputs`` (global expert order). The caller orders reuse: a rank's next :meth:`gemm`
    writes into its peers' copies, so they must be done reading the previous results.
    """

    def __init__(self, rows_per_expert: Sequence[int], n: int, device: torch.device,
                 group: dist.ProcessGroup | None = None, fabric=None):
        from . import _native

        self.fabric = fabric if fabric is not None else ProcessGroupFabric(group)
        world, rank = self.fabric.world, self.fabric.rank
        if world - 1 > _native.MAX_REPLICAS:
            raise ValueError(f"at most {_native.MAX_REPLICAS + 1} ranks")
        self.world, self.rank = world, rank
        self.rows = [int(m) for m in rows_per_expert]
        self.n = int(n)
        layout = slab_layout(self.rows, self.n, world)
        self.max_elems = max(e for _, _, e in layout)
        nbytes = world * self.max_elems * 2
        self._symm, bases = self.fabric.allocate(max(nbytes, 256), torch.device(device))
        # Every rank's copy has the same layout: a peer's copy of a byte is at
        # (its base - this base) from this rank's copy of it.
        self.replica_offsets = [bases[p] - bases[rank] for p in range(world) if p != rank]
        self.slabs = self._symm[:nbytes].view(torch.float16)
        first, count, _ = layout[rank]
        self.local_outputs = self._views(rank * self.max_elems, first, count)
        self.outputs = []
        for r, (f, cnt, _) in enumerate(layout):
            self.outputs += self._views(r * self.max_elems, f, cnt)
        self.bytes_sent = int((world - 1) * layout[rank][2] * 2)
        self._table = None
        self._ws = None
        self._sig = None

    def _views(self, base: int, first: int, count: int) -> list:
        out, off = [], base
        for g in range(first, first + count):
            m = self.rows[g]
            out.append(self.slabs[off:off + m * self.n].view(m, self.n))
            off += m * self.n
        return out

    def gemm(self, a, b, sfa, sfb, problem_sizes, *, alpha=None, b2=None, sfb2=None,
             alpha2=None, cta: str | None = None,
             stream: torch.cuda.Stream | None = None) -> list:
        """This rank's experts (operands as for :func:`interface.grouped_gemm`, outputs into
        ``local_outputs``) with every output row also stored into the peers' copies."""
        import ctypes

        import numpy as np

        from . import _native
        from .interface import _prepare

        sig = (tuple(t.data_ptr() for t in list(a) + list(b) + list(sfa) + list(sfb)),
               tuple(tuple(ps) for ps in problem_sizes), None if alpha is None else tuple(alpha),
               None if b2 is None else tuple(t.data_ptr() for t in list(b2) + list(sfb2)),
               None if alpha2 is None else tuple(alpha2), cta)
        reuse = sig == self._sig and self._table is not None
        if not reuse:
            prepared = _prepare(a, b, sfa, sfb, self.local_outputs, problem_sizes, alpha, b2,
                                sfb2, alpha2, None, cta)
            if prepared is None:
                return self.local_outputs
            self._table, self._flags, dev = prepared
            G = int(self._table.shape[0])
            if self._ws is None or self._ws.numel() < _native.workspace_size(G):
                self._ws = torch.zeros(_native.workspace_size(G), dtype=torch.uint8, device=dev)
            self._sig = sig
        s = (stream or torch.cuda.current_stream(self._symm.device)).cuda_stream
        lib = _native.load_library()
        flags = self._flags | (_native.FLAG_REUSE_DESCRIPTORS if reuse else 0)
        t = self._table
        if self.world == 1:
            st = lib.nvfp4_grouped_gemm(t.ctypes.data, int(t.shape[0]), flags,
                                        self._ws.data_ptr(), self._ws.numel(), s)
        else:
            offs = np.asarray(self.replica_offsets, dtype=np.int64)
            st = lib.nvfp4_grouped_gemm_replicated(
                t.ctypes.data, int(t.shape[0]), flags, self._ws.data_ptr(), self._ws.numel(),
                offs.ctypes.data_as(ctypes.c_void_p), len(self.replica_offsets), s)
        _native.check(st, lib)
        return self.local_outputs

    def barrier(self) -> None:
        """Cross-rank barrier on the current stream: after it every rank's kernel (and so
        every replica store) has completed."""
        self.fabric.barrier(self._symm.device)

    def check_device_errors(self, stream: torch.cuda.Stream | None = None) -> int:
        from . import _native

        s = (stream or torch.cuda.current_stream(self._symm.device)).cuda_stream
        return 0 if self._ws is None else _native.workspace_check(self._ws.data_ptr(), s)


class ExpertParallelGroupedGemm:
    """Run this rank's shard of a grouped problem and optionally gather all outputs.

    `local_gemm(problem)` computes the local experts' outputs in place (the
    grouped kernel on GPUs); it is a parameter so that the bookkeeping can be
    exercised on CPU ranks with a host implementation.
    """

    def __init__(self, num_experts: int, group: dist.ProcessGroup | None = None,
                 local_gemm: Callable | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.num_experts = num_experts
        self.shard = expert_shard(num_experts, self.world, self.rank)
        self.local_gemm = local_gemm

    def run(self, local_problem, rows_per_expert: Sequence[int], gather: bool = False) -> list:
        if self.local_gemm is None:
            from .interface import grouped_gemm

            p = local_problem
            grouped_gemm(p.a, p.b, p.sfa, p.sfb, p.c, p.problem_sizes(), alpha=p.alpha,
                         b2=p.b2, sfb2=p.sfb2, alpha2=p.alpha2)
            outs = list(p.c)
        else:
            outs = list(self.local_gemm(local_problem))
        if not gather or self.world == 1:
            return outs
        return all_gather_expert_outputs(outs, rows_per_expert, local_problem.n, self.group)


class EPMoEBlock:
    """Expert-parallel MoE feed-forward block: one process per GPU, every rank holding
    ``tokens`` tokens and the weights of its own experts (rank p: experts [p*E/P,
    (p+1)*E/P)), exchanging NVFP4 token rows and fp16 expert outputs over NVLink peer
    memory (nvfp4_ep_* kernels) with no device-to-host read.

    Per call (one stream; barriers are one-element NCCL all-reduces):
    route + quantise the local tokens; publish per-expert counts into every rank's count
    matrix | layout (all ranks derive the same placement); dispatch codes + scale rows (and
    each row's return address) into the owners' receive slabs | owner: scales to the blocked
    layout, gated GEMM over its expert segments with NVFP4 output, then the down GEMM and
    the return, in one of two forms (``return_mode``):

    * ``"sums"`` (default): dispatch sends each token once to every owner of its pairs (not
      once per pair) and publishes each pair's slab row and routing weight into its owner's
      pair tables | the owner copies the token rows into its receive slab
      (nvfp4_ep_expand); the down GEMM writes its rows locally, and nvfp4_ep_return_sums
      adds each source token's rows of this owner (weighted, slot order, fp32) and stores
      one fp16 row per (token, owner) into the token's rank | combine: fp32 sum of each
      token's per-owner rows in owner order, bf16. A token's slots that meet on one owner
      cross NVLink as one row each way.
    * ``"rows"``: the down GEMM's epilogue stores every output row into its token's rank
      (NVLink stores overlapping the GEMM) | combine: weighted fp32 sum of each token's
      returned rows in slot order, bf16 -- bit-identical to the single-GPU MoEBlock.

    The receive slabs hold ``world * tokens * topk + 127 * E/P`` rows (every pair of every
    rank routed here, plus segment padding), so the exchange never drops a pair. Count
    matrix, receive slabs, return addresses, pair tables and the return buffer ([tokens,
    world, H] fp16 for sums, [tokens * topk, H] for rows) live in one allocation of the
    fabric (``fabric=``): torch symmetric memory over the process group by default
    (:class:`ProcessGroupFabric`), or one GPU holding every rank (:class:`SingleDeviceFabric`,
    calls driven by :func:`run_lockstep`).
    """

    def __init__(self, local_weights, num_experts: int, tokens: int, topk: int,
                 act_scale: float, hidden_scale: float, group=None, cta: str | None = None,
                 return_mode: str = "sums", fabric=None):
        import numpy as np

        from . import _native
        from .layout import blocked_sf_bytes

        if cta not in (None, "pair", "single"):
            raise ValueError(f"cta must be None, 'pair' or 'single', got {cta!r}")
        if return_mode not in ("sums", "rows"):
            raise ValueError(f"return_mode must be 'sums' or 'rows', got {return_mode!r}")
        self.return_mode = return_mode
        self.fabric = fabric if fabric is not None else ProcessGroupFabric(group)
        world, rank = self.fabric.world, self.fabric.rank
        if world > _native.EP_MAX_RANKS:
            raise ValueError(f"at most {_native.EP_MAX_RANKS} ranks")
        if num_experts % world:
            raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
        epr = num_experts // world
        if local_weights.num_experts != epr:
            raise ValueError(f"rank {rank} must hold {epr} experts, got {local_weights.num_experts}")
        if not (act_scale > 0 and hidden_scale > 0):
            raise ValueError("act_scale and hidden_scale must be positive")
        dev = local_weights.w_gate[0].device
        idim = int(local_weights.w_gate[0].shape[0])
        hdim = int(local_weights.w_gate[0].shape[1]) * 2
        if hdim % 256 or idim % 256:
            raise ValueError("hidden and intermediate sizes must be multiples of 256")
        self.world, self.rank, self.num_experts, self.experts_per_rank = world, rank, num_experts, epr
        self.tokens, self.topk, self.hidden, self.intermediate = tokens, topk, hdim, idim
        self.act_scale, self.hidden_scale = float(act_scale), float(hidden_scale)
        self.device = dev
        self._cta_flags = {None: 0, "pair": _native.FLAG_CTA_PAIR,
                           "single": _native.FLAG_SINGLE_CTA}[cta]
        self._lib = lib = _native.load_library()
        pairs = tokens * topk
        cap = world * pairs + 127 * epr
        self.capacity = cap

        # One symmetric allocation: count matrix | received codes | received plain scales |
        # return address of each received row | returned rows (sums: one per token and owner;
        # rows: one per pair) | pair tables of the sums (slab row and weight of each source
        # rank's pairs here) | token slabs of the sums (codes, plain scales of each source
        # rank's tokens with pairs here).
        sums = return_mode == "sums"

        def up(n):
            return (n + 255) // 256 * 256
        sizes = [world * num_experts * 4, cap * hdim // 2, cap * hdim // 16, cap * 8,
                 (tokens * world if sums else pairs) * hdim * 2,
                 world * pairs * 4 if sums else 0, world * pairs * 4 if sums else 0,
                 world * tokens * hdim // 2 if sums else 0,
                 world * tokens * hdim // 16 if sums else 0]
        offs = [0]
        for n in sizes[:-1]:
            offs.append(offs[-1] + up(n))
        total = offs[-1] + max(up(sizes[-1]), 256)
        self._symm, bases = self.fabric.allocate(total, dev)
        self._peers = [_native.EpPeers.of([b + o for b in bases]) for o in offs]
        sl = [self._symm[o:o + n] for o, n in zip(offs, sizes)]
        self._mat = sl[0].view(torch.int32).view(world, num_experts)
        self._recv_codes = sl[1].view(cap, hdim // 2)
        self._recv_sf = sl[2].view(cap, hdim // 16)
        self._recv_meta = sl[3].view(torch.int64)
        if sums:
            self._ret = sl[4].view(torch.float16).view(tokens, world, hdim)
            self._pair_rows = sl[5].view(torch.int32).view(world, pairs)
            self._pair_w = sl[6].view(torch.float32).view(world, pairs)
            self._tok_codes = sl[7].view(world * tokens, hdim // 2)
            self._tok_sf = sl[8].view(world * tokens, hdim // 16)
            # The down GEMM's rows stay here (slab order); return_sums reads them.
            self._y = torch.empty((cap, hdim), dtype=torch.float16, device=dev)
            self._scatter = None
        else:
            self._ret = sl[4].view(torch.float16).view(pairs, hdim)
            # The down GEMM's output rows go to the token's rank: row r of this rank's slab to
            # return buffer (recv_meta[r] >> 40) at pair (recv_meta[r] & (2^40 - 1)).
            self._scatter = _native.SegmentOutput.scattered(
                self._recv_meta.data_ptr(), [b + offs[4] for b in bases], hdim * 2)

        i32 = dict(dtype=torch.int32, device=dev)
        u8 = dict(dtype=torch.uint8, device=dev)
        self._meta = torch.zeros(2 * num_experts + 1, **i32)
        self._counts, self._offsets = self._meta[:num_experts], self._meta[num_experts:]
        self._dest = torch.empty(pairs, **i32)
        self._src_rows = torch.empty(pairs + 127 * num_experts, **i32)
        self._route_ws_bytes = int(lib.nvfp4_moe_route_workspace_size(pairs, num_experts))
        self._route_ws = torch.empty(max(self._route_ws_bytes, 16), **u8)
        self._qx = torch.empty((tokens, hdim // 2), **u8)
        self._sfx = torch.empty(blocked_sf_bytes(tokens, hdim // 16), **u8)
        self.seg_offsets = torch.zeros(epr, **i32)
        self.seg_counts = torch.zeros(epr, **i32)
        self.send_base = torch.zeros(num_experts, **i32)
        self.remote_rows = torch.empty(pairs, **i32)
        self._err = torch.zeros(1, **i32)
        self._recv_sfa = torch.zeros(blocked_sf_bytes(cap, hdim // 16), **u8)
        self._a2 = torch.zeros((cap, idim // 2), **u8)
        self._sfa2 = torch.zeros(blocked_sf_bytes(cap, idim // 16), **u8)
        self._w = torch.empty((tokens, topk), dtype=torch.float32, device=dev)
        self.out = torch.empty((tokens, hdim), dtype=torch.bfloat16, device=dev)

        W = local_weights
        P = W.pointers()
        s_x, s_h = self.act_scale, self.hidden_scale

        def slab_table(a, sfa, c, b, sfb, n, k, alpha, b2=None, sfb2=None, alpha2=None):
            t = np.zeros(epr, dtype=_native.GROUP_DTYPE)
            t["a"], t["sfa"], t["c"] = a.data_ptr(), sfa.data_ptr(), c.data_ptr()
            t["b"], t["sfb"] = b, sfb
            if b2 is not None:
                t["b2"], t["sfb2"], t["alpha2"] = b2, sfb2, alpha2
            else:
                t["alpha2"] = 1.0
            t["m"], t["n"], t["k"], t["alpha"] = cap, n, k, alpha
            return t

        self._weights = W  # the tables hold its addresses
        self._t1 = slab_table(self._recv_codes, self._recv_sfa, self._a2, P["w_gate"], P["sf_gate"],
                              idim, hdim, s_x * np.asarray(W.s_gate, dtype=np.float32),
                              P["w_up"], P["sf_up"], s_x * np.asarray(W.s_up, dtype=np.float32))
        # c of the down GEMM: the local slab (sums), or never written (rows: scattered output;
        # any valid aligned address).
        self._t2 = slab_table(self._a2, self._sfa2, self._y if sums else self._ret, P["w_down"],
                              P["sf_down"], hdim, idim,
                              s_h * np.asarray(W.s_down, dtype=np.float32))
        self._nvfp4_out = _native.SegmentOutput.nvfp4(self._sfa2.data_ptr(), self.hidden_scale)
        ws_bytes = _native.workspace_size(epr)
        self._ws1 = torch.zeros(ws_bytes, **u8)
        self._ws2 = torch.zeros(ws_bytes, **u8)
        self._ws_bytes = ws_bytes
        self._uploaded = False
        self.fabric.meet()

    def run(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
            stage_events: list | None = None) -> torch.Tensor:
        """One expert-parallel block on the current stream; returns ``self.out`` (bf16
        [tokens, H]) for this rank's tokens. Every rank of the group must call it. With
        ``stage_events`` (a list), (stage name, CUDA event recorded after it) pairs are
        appended for timing."""
        for _ in self.phases(x, topk_ids, topk_weights, stage_events):
            self.fabric.barrier(self.device)
        return self.out

    def phases(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
               stage_events: list | None = None):
        """The call of :meth:`run` as a generator that yields at each of its three
        cross-rank barriers (which the caller takes: :meth:`run` through the fabric,
        :func:`run_lockstep` by running every emulated rank up to the same point)."""
        from . import _native
        from .quantize import _DTYPES

        T, K, H, E, world, rank = (self.tokens, self.topk, self.hidden, self.num_experts,
                                   self.world, self.rank)
        if x.dtype not in _DTYPES or tuple(x.shape) != (T, H) or x.stride(1) != 1:
            raise ValueError(f"x must be bf16/fp16 [{T}, {H}]")
        if topk_ids.dtype != torch.int32 or tuple(topk_ids.shape) != (T, K) or \
                not topk_ids.is_contiguous():
            raise ValueError(f"topk_ids must be contiguous int32 [{T}, {K}]")
        lib, chk = self._lib, _native.check
        st = torch.cuda.current_stream(self.device)
        s = st.cuda_stream
        cap = self.capacity

        def mark(name):
            if stage_events is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(st)
                stage_events.append((name, ev))

        mark("start")
        chk(lib.nvfp4_moe_route(topk_ids.data_ptr(), T, K, E, self._counts.data_ptr(),
                                self._offsets.data_ptr(), self._dest.data_ptr(),
                                self._src_rows.data_ptr(), self._src_rows.numel(),
                                self._route_ws.data_ptr(), self._route_ws_bytes, s), lib)
        chk(lib.nvfp4_quantize(x.data_ptr(), T, H, x.stride(0), _DTYPES[x.dtype], self.act_scale,
                               self._qx.data_ptr(), self._qx.stride(0), self._sfx.data_ptr(), s), lib)
        mark("route + quantise")
        chk(lib.nvfp4_ep_publish_counts(self._counts.data_ptr(), E, rank, world, self._peers[0], s),
            lib)
        yield
        mark("publish counts + barrier")
        chk(lib.nvfp4_ep_layout(self._mat.data_ptr(), E, rank, world, cap,
                                self.seg_offsets.data_ptr(), self.seg_counts.data_ptr(),
                                self.send_base.data_ptr(), self._err.data_ptr(), s), lib)
        if self._scatter is None:
            chk(lib.nvfp4_ep_dispatch_tokens(topk_ids.data_ptr(), T, K, E, rank, world,
                                             self._dest.data_ptr(), self._offsets.data_ptr(),
                                             self.send_base.data_ptr(), self._qx.data_ptr(),
                                             self._qx.stride(0), self._sfx.data_ptr(), H,
                                             self._peers[7], self._peers[8], cap,
                                             self.remote_rows.data_ptr(), s), lib)
        else:
            chk(lib.nvfp4_ep_dispatch(topk_ids.data_ptr(), T, K, E, rank, world,
                                      self._dest.data_ptr(), self._offsets.data_ptr(),
                                      self.send_base.data_ptr(), self._qx.data_ptr(),
                                      self._qx.stride(0), self._sfx.data_ptr(), H, self._peers[1],
                                      self._peers[2], self._peers[3], cap,
                                      self.remote_rows.data_ptr(), s), lib)
        w = topk_weights
        if w.dtype != torch.float32 or not w.is_contiguous():
            self._w.copy_(w)
            w = self._w
        if self._scatter is None:
            chk(lib.nvfp4_ep_publish_pairs(topk_ids.data_ptr(), self.remote_rows.data_ptr(),
                                           w.data_ptr(), T, K, E, rank, world, self._peers[5],
                                           self._peers[6], s), lib)
        mark("layout + dispatch")
        yield
        mark("barrier")
        if self._scatter is None:
            chk(lib.nvfp4_ep_expand(self._pair_rows.data_ptr(), T, K, world,
                                    self._tok_codes.data_ptr(), self._tok_sf.data_ptr(), H,
                                    self._recv_codes.data_ptr(), self._recv_sf.data_ptr(), cap, s),
                lib)
            mark("expand")
        _native.sf_to_blocked_raw(self._recv_sf.data_ptr(), self._recv_sfa.data_ptr(), cap,
                                  H // 16, H // 16, s)
        flags = (_native.FLAG_REUSE_DESCRIPTORS if self._uploaded else 0) | self._cta_flags
        _native.grouped_gemm_segments_raw(self._t1, _native.FLAG_GATED | flags,
                                          self.seg_offsets.data_ptr(), self.seg_counts.data_ptr(),
                                          T * K, self._ws1.data_ptr(), self._ws_bytes, s,
                                          self._nvfp4_out)
        mark("scale layout + gate/up GEMM")
        _native.grouped_gemm_segments_raw(self._t2, flags, self.seg_offsets.data_ptr(),
                                          self.seg_counts.data_ptr(), T * K,
                                          self._ws2.data_ptr(), self._ws_bytes, s, self._scatter)
        self._uploaded = True
        if self._scatter is None:
            mark("down GEMM")
            chk(lib.nvfp4_ep_return_sums(self._pair_rows.data_ptr(), self._pair_w.data_ptr(), T,
                                         K, rank, world, self._y.data_ptr(), self._y.stride(0), H,
                                         self._peers[4], s), lib)
            mark("return sums")
        else:
            mark("down GEMM + return rows")
        yield
        mark("barrier 2")
        if self._scatter is None:
            chk(lib.nvfp4_ep_combine_sums(topk_ids.data_ptr(), self.remote_rows.data_ptr(), T, K,
                                          E, world, self._ret.data_ptr(), H,
                                          self.out.data_ptr(), self.out.stride(0), s), lib)
        else:
            chk(lib.nvfp4_ep_combine(self.remote_rows.data_ptr(), w.data_ptr(), T, K,
                                     self._ret.data_ptr(), H, self.out.data_ptr(),
                                     self.out.stride(0), s), lib)
        mark("combine")

    def capture(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                warmup: int = 1) -> torch.cuda.CUDAGraph:
        """Record one call over these input tensors into a CUDA graph, NCCL barriers
        included (after ``warmup`` eager calls, which upload the GEMMs' descriptors). Every
        rank of the group must capture, and replay in the same order; ``graph.replay()``
        recomputes ``self.out`` from the tensors' current contents."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(max(warmup, 1)):
                self.run(x, topk_ids, topk_weights)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self.run(x, topk_ids, topk_weights)
        return graph

    def check_errors(self) -> int:
        """Synchronise; returns the exchange's error bits (EP_ERR_CAPACITY) and raises if a
        GEMM reported a device error."""
        from . import _native

        s = torch.cuda.current_stream(self.device).cuda_stream
        _native.workspace_check(self._ws1.data_ptr(), s)
        _native.workspace_check(self._ws2.data_ptr(), s)
        return int(self._err.item())
