"""Expert-parallel sharding and output all-gather on CPU ranks (gloo, world size 2 and 3).

Each rank computes its experts with the CPU oracle standing in for the kernel;
the gathered outputs must equal the single-process oracle outputs for every
expert, in global order.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expected(pkg, rows, n, k, seed):
    from oracle import nvfp4_oracle as O

    prob = pkg.workloads.make_problem("ep", rows, n, k, seed=seed, device="cpu")
    return [O.ref_gemm(prob.a[g].numpy(), prob.b[g].numpy(), prob.sfa_plain[g].numpy(),
                       prob.sfb_plain[g].numpy()) for g in range(len(rows))]


def _worker(rank, world, port, rows, n, k, seed, q):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import submission
        from oracle import nvfp4_oracle as O

        pkg = submission.load_package()
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        full = pkg.workloads.make_problem("ep", rows, n, k, seed=seed, device="cpu")
        ep = pkg.expert_parallel.ExpertParallelGroupedGemm(
            len(rows), local_gemm=lambda p: [
                torch.from_numpy(O.ref_gemm(p["a"][i].numpy(), p["b"][i].numpy(),
                                            p["sfa"][i].numpy(), p["sfb"][i].numpy()))
                for i in range(len(p["a"]))])
        sh = ep.shard
        local = {"a": full.a[sh.start:sh.stop], "b": full.b[sh.start:sh.stop],
                 "sfa": full.sfa_plain[sh.start:sh.stop], "sfb": full.sfb_plain[sh.start:sh.stop]}

        class _P(dict):
            n = full.n

        outs = ep.run(_P(local), rows, gather=True)
        q.put((rank, [o.numpy() for o in outs], (sh.start, sh.stop)))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


@pytest.mark.parametrize("world,rows", [(2, [5, 0, 17, 3, 64]), (3, [1, 2, 3, 0, 0, 7, 9])])
def test_gather_matches_single_process(pkg, world, rows):
    n, k, seed = 128, 256, 42
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, n, k, seed, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, outs, shard = q.get(timeout=180)
        assert shard is not None, outs
        results[rank] = (outs, shard)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expected = _expected(pkg, rows, n, k, seed)
    covered = []
    for rank in range(world):
        outs, shard = results[rank]
        covered.extend(range(*shard))
        assert len(outs) == len(rows)
        for g in range(len(rows)):
            assert np.array_equal(outs[g], expected[g]), (rank, g)
    assert sorted(covered) == list(range(len(rows)))


def test_shard_bookkeeping(pkg):
    EP = pkg.expert_parallel
    for G in (0, 1, 7, 256):
        for P in (1, 2, 3, 8):
            shards = [EP.expert_shard(G, P, r) for r in range(P)]
            assert sum(len(s) for s in shards) == G
            assert [x for s in shards for x in s] == list(range(G))
            assert max(len(s) for s in shards) - min(len(s) for s in shards) <= 1
    lay = EP.slab_layout([4, 0, 2, 6], 8, 2)
    assert lay == [(0, 2, 32), (2, 2, 64)]
    with pytest.raises(ValueError):
        EP.expert_shard(4, 2, 2)
