"""Expert parallelism on 2 GPUs: each rank runs its contiguous expert shard through the CUDA
kernel and the outputs are all-gathered over NCCL (skipped when fewer than 2 GPUs exist).

Each rank checks its own experts against the oracle; the parent then checks that every
rank's gathered list equals, byte for byte, the concatenation of all ranks' local outputs.
Three exchanges are covered: all_gather_expert_outputs (packs the outputs per call),
ExpertOutputGather (the GEMM writes its outputs into the preallocated send slab of one NCCL
all-gather) and FusedOutputGather (the GEMM's epilogue stores every output tile into each
peer's copy of the slab over NVLink; two calls, the second after A changed in place, so the
descriptor-reuse path is covered too).
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROWS = [5, 0, 130, 64, 1, 300, 17, 0, 256, 9, 40, 128]  # 12 experts, some empty
N, K = 256, 512


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, gated, mode, q):
    try:
        import sys

        import torch.distributed as dist

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import submission
        from oracle import nvfp4_oracle as O

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        pkg = submission.load_package()
        EP = pkg.expert_parallel
        ep = EP.ExpertParallelGroupedGemm(len(ROWS))
        sh = ep.shard
        prob = pkg.workloads.make_problem(f"ep{rank}", ROWS[sh.start:sh.stop], N, K, gated=gated,
                                          seed=100 + rank, device=dev, alpha_range=(0.5, 2.0))
        calls = 1
        if mode == "slab":
            gat = EP.ExpertOutputGather(ROWS, N, dev)
            for c, v in zip(prob.c, gat.local_outputs):
                v.copy_(c)  # the harness's randn prefill, now in the slab
            prob.c = list(gat.local_outputs)
            pkg.grouped_gemm(prob.a, prob.b, prob.sfa, prob.sfb, prob.c, prob.problem_sizes(),
                             alpha=prob.alpha, b2=prob.b2, sfb2=prob.sfb2, alpha2=prob.alpha2)
            outs = gat.run()
        elif mode == "fused":
            gat = EP.FusedOutputGather(ROWS, N, dev)
            prob.c = list(gat.local_outputs)
            calls = 2
        else:
            outs = ep.run(prob, ROWS, gather=True)
        for call in range(calls):
            if mode == "fused":
                if call:
                    for t in prob.a:
                        t ^= 0x11  # new operand values behind the same pointers
                    dist.barrier(device_ids=[rank])  # peers are done reading the last call
                gat.gemm(prob.a, prob.b, prob.sfa, prob.sfb, prob.problem_sizes(),
                         alpha=prob.alpha, b2=prob.b2, sfb2=prob.sfb2, alpha2=prob.alpha2)
                gat.barrier()
                outs = gat.outputs
            torch.cuda.synchronize()
            _check_local(prob, gated, rank, O)
        if mode == "fused":
            assert gat.check_device_errors() == 0
        local = [c.cpu().numpy() for c in prob.c]
        gathered = [o.cpu().numpy() for o in outs]
        q.put((rank, local, gathered, (sh.start, sh.stop)))
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
    except BaseException as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None, None))


def _check_local(prob, gated, rank, O):
    """This rank's experts against the oracle."""
    for i in range(prob.num_groups):
        if prob.m[i] == 0:
            continue
        a, b = prob.a[i].cpu().numpy(), prob.b[i].cpu().numpy()
        sfa, sfb = prob.sfa_plain[i].cpu().numpy(), prob.sfb_plain[i].cpu().numpy()
        got = prob.c[i].cpu().numpy()
        if gated:
            exp = O.ref_gated(a, b, prob.b2[i].cpu().numpy(), sfa, sfb,
                              prob.sfb2_plain[i].cpu().numpy(), prob.alpha[i], prob.alpha2[i])
            ref32 = None
        else:
            ref32 = O.ref_gemm_fp32(a, b, sfa, sfb) * np.float32(prob.alpha[i])
            exp = ref32.astype(np.float16)
        res = O.compare_fp16(got, exp, ref32, rtol=1e-2, atol=1e-2)
        assert res["ok"], (rank, i, res)


MODES = [(g, m) for m in ("list", "slab", "fused") for g in (False, True)]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("gated,mode", MODES, ids=[f"{m}-{'gated' if g else 'plain'}"
                                                   for g, m in MODES])
def test_two_gpu_shards_and_nccl_gather(gated, mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, gated, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, local, gathered, shard = q.get(timeout=300)
        assert shard is not None, local
        results[rank] = (local, gathered, shard)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    everything = []
    covered = []
    for r in range(world):
        local, _, shard = results[r]
        everything.extend(local)
        covered.extend(range(*shard))
    assert covered == list(range(len(ROWS)))
    for r in range(world):
        gathered = results[r][1]
        assert len(gathered) == len(ROWS)
        for g, (x, y) in enumerate(zip(gathered, everything)):
            assert x.shape == (ROWS[g], N)
            assert np.array_equal(x.view(np.uint16), y.view(np.uint16)), (r, g)
