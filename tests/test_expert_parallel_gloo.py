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


def _slab_worker(rank, world, port, rows, n, q):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import submission

        pkg = submission.load_package()
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        EP = pkg.expert_parallel
        gat = EP.ExpertOutputGather(rows, n, torch.device("cpu"))
        sh = EP.expert_shard(len(rows), world, rank)
        assert len(gat.local_outputs) == len(sh)
        results = []
        for call in range(2):  # the slabs are reused: the second call overwrites the first
            for g, t in zip(sh, gat.local_outputs):
                t.copy_(_slab_rows(rows[g], n, g, call))
            results.append([o.clone().numpy() for o in gat.run()])
        q.put((rank, results))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


def _slab_rows(m, n, expert, call):
    return (torch.arange(m * n, dtype=torch.float32).view(m, n) * 0.25
            + 1000 * expert + 7 * call).to(torch.float16)


@pytest.mark.parametrize("world,rows", [(2, [5, 0, 17, 3, 64]), (3, [1, 2, 3, 0, 0, 7, 9])])
def test_preallocated_gather_slabs(world, rows):
    """ExpertOutputGather: each rank writes its experts' rows into its send-slab views;
    after run() every rank holds every expert's rows in global order, on two calls."""
    n = 24
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_slab_worker, args=(r, world, port, rows, n, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        assert isinstance(res[rank], list), res[rank]
        for call, outs in enumerate(res[rank]):
            assert len(outs) == len(rows)
            for g, o in enumerate(outs):
                assert np.array_equal(o, _slab_rows(rows[g], n, g, call).numpy()), (rank, call, g)


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


# ----------------------------------------------------------------------------
# The expert-parallel MoE exchange: placement rule of nvfp4_ep_layout / nvfp4_ep_dispatch
# ----------------------------------------------------------------------------
def _ids(tokens, topk, experts, seed):
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, experts + 1) ** 1.2
    p /= p.sum()
    ids = np.stack([rng.choice(experts, size=topk, replace=False, p=p) for _ in range(tokens)])
    ids[rng.random(ids.shape) < 0.03] = -1
    return ids.astype(np.int32)


@pytest.mark.parametrize("world,experts,tokens,topk", [(2, 16, 300, 4), (4, 64, 129, 8),
                                                       (8, 256, 64, 8), (3, 12, 1, 2)])
def test_ep_layout_matches_pairwise_placement(world, experts, tokens, topk):
    """The closed-form layout (segment starts + earlier ranks' counts) puts every pair where a
    pair-by-pair walk puts it; segments are 128-aligned, disjoint and exactly filled."""
    from oracle import nvfp4_ep_oracle as EPO

    ids = [_ids(tokens, topk, experts, seed=world * 100 + q) for q in range(world)]
    cap = world * tokens * topk + 127 * (experts // world)
    counts, remote, received = EPO.place_pairs(ids, experts, world, cap)
    from oracle import nvfp4_moe_oracle as M

    for q in range(world):
        seg_off, seg_cnt, send_base, dropped = EPO.ep_layout(counts, world, q, cap)
        assert not dropped
        assert np.all(seg_off % 128 == 0)
        _, offsets, dest, _ = M.route(ids[q], experts)
        flat = ids[q].reshape(-1)
        for i, e in enumerate(flat):
            if dest[i] < 0:
                assert remote[q][i] == -1
                continue
            assert remote[q][i] == send_base[e] + dest[i] - offsets[e]
        # As owner: the received rows are exactly the segments' first seg_cnt rows.
        rows = sorted(received[q])
        want = sorted(r for o, c in zip(seg_off, seg_cnt) for r in range(o, o + c))
        assert rows == want


def test_ep_layout_drops_segments_that_do_not_fit():
    from oracle import nvfp4_ep_oracle as EPO

    world, experts = 2, 8
    mat = np.array([[100, 0, 50, 200, 0, 1, 3, 7], [30, 5, 0, 100, 9, 0, 0, 1]])
    seg_off, seg_cnt, send_base, dropped = EPO.ep_layout(mat, world, 0, capacity=400)
    # owner 0: experts 0..3 with totals 130, 5, 50, 300 -> starts 0, 256, 384, 512
    assert dropped
    assert list(seg_off[:3]) == [0, 256, 0] and list(seg_cnt) == [130, 5, 0, 0]
    assert send_base[0] == 0 and send_base[1] == 256 and send_base[2] == -1 and send_base[3] == -1


def _ep_gloo_worker(rank, world, port, experts, tokens, topk, q):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import nvfp4_ep_oracle as EPO
        from oracle import nvfp4_moe_oracle as M

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        ids = _ids(tokens, topk, experts, seed=rank + 7)
        counts = torch.from_numpy(M.route(ids, experts)[0].astype(np.int32))
        # The count matrix every rank assembles (the device path writes it with peer stores).
        mat = [torch.zeros_like(counts) for _ in range(world)]
        dist.all_gather(mat, counts)
        mat = torch.stack(mat).numpy()
        cap = world * tokens * topk + 127 * (experts // world)
        seg_off, seg_cnt, send_base, _ = EPO.ep_layout(mat, world, rank, cap)
        _, offsets, dest, _ = M.route(ids, experts)
        flat = ids.reshape(-1)
        rows = [(int(e) // (experts // world), int(send_base[e] + dest[i] - offsets[e]))
                for i, e in enumerate(flat) if dest[i] >= 0]
        everything = [None] * world
        dist.all_gather_object(everything, (rows, seg_off.tolist(), seg_cnt.tolist()))
        q.put((rank, everything))
        dist.destroy_process_group()
    except BaseException as e:
        q.put((rank, repr(e)))


def test_ep_placement_over_gloo_ranks():
    """Two CPU ranks exchange their routing counts over gloo and place their pairs: the
    rows written into each owner's slab are distinct and fill its segments exactly."""
    world, experts, tokens, topk = 2, 16, 200, 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_gloo_worker, args=(r, world, port, experts, tokens, topk, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    everything = res[0]
    assert isinstance(everything, list), everything
    for owner in range(world):
        written = [r for rows, _, _ in everything for (o, r) in rows if o == owner]
        assert len(written) == len(set(written))
        _, seg_off, seg_cnt = everything[owner]
        want = sorted(r for o, c in zip(seg_off, seg_cnt) for r in range(o, o + c))
        assert sorted(written) == want


def _pair_rows(rank, tokens, topk, cols):
    """The down GEMM's fp16 row of every pair of source `rank` (a stand-in any rank can
    rebuild: seeded by the source rank)."""
    rng = np.random.default_rng(1000 + rank)
    return (rng.standard_normal((tokens, topk, cols)) * 3).astype(np.float16)


def _presum_gloo_worker(rank, world, port, experts, tokens, topk, cols, q):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import nvfp4_ep_oracle as EPO

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        epr = experts // world
        routing = []  # every source's (ids, weights, kept), rebuilt from seeds on every rank
        for src in range(world):
            ids = _ids(tokens, topk, experts, seed=src + 7)
            w = np.random.default_rng(50 + src).random((tokens, topk)).astype(np.float32)
            routing.append((ids, w, ids >= 0))
        # As owner: one partial row per (source, token) with pairs here (return_sums), sent to
        # the source rank (the device path stores them into its return buffer over NVLink).
        outgoing = []
        for src in range(world):
            ids, w, kept = routing[src]
            y = _pair_rows(src, tokens, topk, cols)
            mine = kept & (ids // epr == rank)
            part, has, _ = EPO.presum_combine(y, mine, np.where(mine, rank, -1), w, world)
            outgoing.append((part[:, rank], has[:, rank]))
        received = [None] * world
        for src in range(world):  # rank src collects every owner's rows for its tokens
            gathered = [None] * world
            dist.all_gather_object(gathered, outgoing[src])
            if src == rank:
                received = gathered
        # combine_sums: owner order, fp32, over the owners that hold a kept pair.
        ids, w, kept = routing[rank]
        owner = np.where(kept, ids // epr, -1)
        acc = np.zeros((tokens, cols), dtype=np.float32)
        for p in range(world):
            part_p, has_p = received[p]
            has_expect = (kept & (owner == p)).any(axis=1)
            assert np.array_equal(has_p, has_expect)
            acc = np.where(has_p[:, None], (acc + part_p.astype(np.float32)).astype(np.float32),
                           acc)
        from oracle import nvfp4_moe_oracle as M
        got = M.fp32_to_bf16_bits(acc)
        _, _, want = EPO.presum_combine(_pair_rows(rank, tokens, topk, cols), kept, owner, w,
                                        world)
        q.put((rank, bool(np.array_equal(got, want))))
        dist.destroy_process_group()
    except BaseException as e:
        q.put((rank, repr(e)))


def test_ep_owner_sums_over_gloo_ranks():
    """Two CPU ranks play owners and sources of the owner-side sums: each owner sums the
    rows of every source token it holds pairs of and sends one row per (token, owner) back
    over gloo; each source's owner-order combine of what it received equals the one-process
    oracle over its own tokens bit for bit."""
    world, experts, tokens, topk, cols = 2, 16, 120, 4, 32
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_presum_gloo_worker,
                         args=(r, world, port, experts, tokens, topk, cols, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}, res
