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
