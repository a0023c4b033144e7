"""Expert-parallel MoE block on 2 GPUs (EPMoEBlock: routed NVFP4 rows pushed into the owners'
receive slabs over NVLink, expert GEMMs over device-side segments, each result row stored
back into its token's rank by the down GEMM's epilogue, then combined). Skipped with fewer
than 2 GPUs.

Each rank checks, for its own tokens: the placement (count matrix, segments, every pair's
row in its owner's slab) against the CPU oracle of the exchange, and the block's output
against the single-GPU MoEBlock run over the same tokens with all experts, whose down-GEMM
rows are the same rows (tiles forced to single CTAs so both pick the same kernels):

* return_mode "rows": bit for bit equal to MoEBlock's output (same rows, same weights, same
  slot-order arithmetic);
* return_mode "sums": the per-(token, owner) rows in the return buffer and the output bit
  for bit equal to the oracle's owner-side sums (``presum_combine``) over MoEBlock's rows.

Two calls with different tokens and routings check the buffers' reuse; a CUDA graph of a
whole call (NCCL barriers included), replayed on new inputs, must equal an eager call.
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

E, H, I, T, TOPK = 16, 512, 256, 300, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    scores = torch.rand((T, E), generator=g) ** 3
    top = torch.topk(scores, TOPK, dim=1)
    ids = top.indices.to(torch.int32)
    ids[::37, 1] = -1  # a few dropped pairs
    wts = torch.softmax(top.values, dim=1)
    return x.to(dev), ids.to(dev), wts.to(dev)


def _worker(rank, world, port, cta, mode, q):
    try:
        import sys

        import torch.distributed as dist

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import submission
        from oracle import nvfp4_ep_oracle as EPO

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        pkg = submission.load_package()
        g = torch.Generator().manual_seed(5)
        gate = [(torch.randn((I, H), generator=g) * 0.05).to(torch.bfloat16).to(dev) for _ in range(E)]
        up = [(torch.randn((I, H), generator=g) * 0.05).to(torch.bfloat16).to(dev) for _ in range(E)]
        down = [(torch.randn((H, I), generator=g) * 0.05).to(torch.bfloat16).to(dev) for _ in range(E)]
        W = pkg.moe.quantize_expert_weights(gate, up, down)
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        local = pkg.moe.ExpertWeights(**{f: getattr(W, f)[sl] for f in (
            "w_gate", "sf_gate", "w_up", "sf_up", "w_down", "sf_down", "s_gate", "s_up", "s_down")})
        s_x, s_h = 0.004, 0.002
        ep = pkg.expert_parallel.EPMoEBlock(local, E, T, TOPK, s_x, s_h, cta=cta, return_mode=mode)
        ref_blk = pkg.moe.MoEBlock(W, T, TOPK, s_x, s_h, cta=cta)
        checks = []
        for call in range(2):
            x, ids, wts = _inputs(1000 * call + rank, dev)
            out = ep.run(x, ids, wts).clone()
            torch.cuda.synchronize()
            err = ep.check_errors()
            ref = ref_blk.run(x, ids, wts)
            torch.cuda.synchronize()
            # Placement against the oracle (every rank's routing is rebuilt here from seeds).
            all_ids = [_inputs(1000 * call + r, "cpu")[1].numpy() for r in range(world)]
            counts, remote, _ = EPO.place_pairs(all_ids, E, world, ep.capacity)
            seg_off, seg_cnt, send_base, dropped = EPO.ep_layout(counts, world, rank, ep.capacity)
            sums = {}
            if mode == "sums":
                # MoEBlock's down-GEMM row of every pair, then the owner-side sums over them.
                dest = ref_blk.dest.cpu().numpy().reshape(T, TOPK)
                y = ref_blk._y.cpu().numpy()[np.maximum(dest, 0)]
                kept = ep.remote_rows.cpu().numpy().reshape(T, TOPK) >= 0
                owner = ids.cpu().numpy() // epr
                part, has, bits = EPO.presum_combine(y, kept, owner, wts.cpu().numpy(), world)
                ret = ep._ret.cpu().numpy()
                sums = dict(
                    kept_is_dest=bool(np.array_equal(kept, dest >= 0)),
                    partials=bool(np.array_equal(ret[has].view(np.uint16),
                                                 part[has].view(np.uint16))),
                    out_oracle=bool(np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16),
                                                   bits)))
            checks.append(dict(sums,
                err=err, dropped=dropped,
                mat=np.array_equal(ep._mat.cpu().numpy(), counts),
                seg=np.array_equal(ep.seg_offsets.cpu().numpy(), seg_off) and
                np.array_equal(ep.seg_counts.cpu().numpy(), seg_cnt),
                send=np.array_equal(ep.send_base.cpu().numpy(), send_base),
                rows=np.array_equal(ep.remote_rows.cpu().numpy(), remote[rank]),
                out_equal=bool(torch.equal(out.view(torch.int16), ref.view(torch.int16))),
                rel=float((out.float() - ref.float()).norm() / ref.float().norm()),
                finite=bool(torch.isfinite(out.float()).all())))
            # The peer's next call starts by publishing its counts into this rank's matrix:
            # read this call's exchange state before either rank moves on.
            dist.barrier(device_ids=[rank])
        # CUDA graph of the whole exchange (NCCL barriers included), replayed on new inputs
        # written into the captured tensors: identical to an eager call.
        x, ids, wts = _inputs(77 + rank, dev)
        graph = ep.capture(x, ids, wts)
        x2, ids2, wts2 = _inputs(5000 + rank, dev)
        x.copy_(x2)
        ids.copy_(ids2)
        wts.copy_(wts2)
        graph.replay()
        torch.cuda.synchronize()
        replayed = ep.out.clone()
        eager = ep.run(x, ids, wts)
        torch.cuda.synchronize()
        checks.append(dict(graph_equal=bool(torch.equal(replayed.view(torch.int16),
                                                        eager.view(torch.int16))),
                           err=ep.check_errors()))
        del graph
        q.put((rank, checks))
        dist.barrier(device_ids=[rank])
        del ep
        dist.destroy_process_group()
    except BaseException as e:  # report instead of hanging the parent
        import traceback

        q.put((rank, traceback.format_exc()[-2000:] + repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("cta,mode", [("single", "sums"), ("single", "rows"), (None, "sums")])
def test_ep_moe_block_two_gpus(cta, mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cta, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, res = q.get(timeout=600)
        results[rank] = res
    for p in procs:
        p.join(timeout=60)
    for rank in range(world):
        res = results[rank]
        assert isinstance(res, list), res
        *calls, graph = res
        assert graph["graph_equal"] and graph["err"] == 0, (rank, graph)
        for call, c in enumerate(calls):
            assert c["err"] == 0 and not c["dropped"], (rank, call, c)
            assert c["mat"] and c["seg"] and c["send"] and c["rows"], (rank, call, c)
            assert c["finite"], (rank, call, c)
            if cta == "single" and mode == "rows":
                assert c["out_equal"], (rank, call, c)
            elif cta == "single":
                assert c["kept_is_dest"] and c["partials"] and c["out_oracle"], (rank, call, c)
            else:
                assert c["rel"] < 1e-2, (rank, call, c)
    for p in procs:
        assert p.exitcode == 0
