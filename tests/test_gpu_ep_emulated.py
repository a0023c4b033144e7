"""Expert parallelism with every rank emulated on ONE GPU (``SingleDeviceFabric``).

The exchange kernels (count publication, layout, dispatch, expand, pair tables, owner-side
sums, scattered-row return, combine) and the replicated GEMM epilogue of the fused output
gather take their peers' buffers as plain device addresses. With every rank's buffers on
one GPU and the ranks' calls run one after another on one stream (stream order standing in
for the barriers; no kernel here waits on another rank), they run exactly as across GPUs,
minus NVLink. This covers world sizes 2, 4 and 8 on a one-GPU machine; the 2-GPU process
tests (test_gpu_ep.py, test_gpu_multigpu.py) cover the NCCL barriers and the NVLink stores.

Checks, per emulated rank:

* placement against the CPU oracle of the exchange (``oracle/nvfp4_ep_oracle.py``): the
  count matrix, the owner's segments, the send bases, every pair's row in its owner's slab,
  and the NVFP4 codes that arrived in every owner's receive slab (byte for byte);
* ``return_mode="rows"`` with single-CTA tiles: the block's output bit for bit equal to the
  single-GPU ``MoEBlock`` over the same tokens with all experts;
* ``return_mode="sums"`` with single-CTA tiles: the per-(token, owner) rows and the output
  bit for bit equal to the oracle's owner-side sums (``presum_combine``) over MoEBlock's
  down-GEMM rows; with the default tiles, within 1e-2 relative of MoEBlock;
* fused output gather: each rank's experts against the GEMM oracle (rtol = atol = 1e-2),
  and every rank's copy of every expert's output byte-equal to the owning rank's, on two
  calls (the second after A changed in place: descriptor reuse).

Two calls with different tokens check the buffers' reuse.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4_ep_oracle as EPO
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

E, H, I, T, TOPK = 16, 512, 256, 300, 4
S_X, S_H = 0.004, 0.002


def _inputs(seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    scores = torch.rand((T, E), generator=g) ** 3
    top = torch.topk(scores, TOPK, dim=1)
    ids = top.indices.to(torch.int32)
    ids[::37, 1] = -1  # a few dropped pairs
    wts = torch.softmax(top.values, dim=1)
    return x.to(dev), ids.to(dev), wts.to(dev)


@pytest.fixture(scope="module")
def weights(pkg):
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(5)
    gate = [(torch.randn((I, H), generator=g) * 0.05).to(torch.bfloat16).to(dev) for _ in range(E)]
    up = [(torch.randn((I, H), generator=g) * 0.05).to(torch.bfloat16).to(dev) for _ in range(E)]
    down = [(torch.randn((H, I), generator=g) * 0.05).to(torch.bfloat16).to(dev) for _ in range(E)]
    return pkg.moe.quantize_expert_weights(gate, up, down)


def _local(pkg, W, world, rank):
    epr = E // world
    sl = slice(rank * epr, (rank + 1) * epr)
    return pkg.moe.ExpertWeights(**{f: getattr(W, f)[sl] for f in (
        "w_gate", "sf_gate", "w_up", "sf_up", "w_down", "sf_down", "s_gate", "s_up", "s_down")})


CASES = [(2, "single", "sums"), (2, "single", "rows"), (4, "single", "sums"),
         (4, "single", "rows"), (8, "single", "sums"), (8, "single", "rows"), (4, None, "sums")]


@pytest.mark.parametrize("world,cta,mode", CASES,
                         ids=[f"w{w}-{c or 'auto'}-{m}" for w, c, m in CASES])
def test_ep_block_emulated(pkg, weights, world, cta, mode):
    EP = pkg.expert_parallel
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fab = EP.SingleDeviceFabric(world, dev)
    blocks = [EP.EPMoEBlock(_local(pkg, weights, world, r), E, T, TOPK, S_X, S_H, cta=cta,
                            return_mode=mode, fabric=fab.rank_view(r)) for r in range(world)]
    ref_blk = pkg.moe.MoEBlock(weights, T, TOPK, S_X, S_H, cta=cta)
    epr = E // world
    for call in range(2):
        inputs = [_inputs(1000 * call + r, dev) for r in range(world)]
        outs = [o.clone() for o in EP.run_lockstep(blocks, inputs)]
        torch.cuda.synchronize()
        for r, blk in enumerate(blocks):
            assert blk.check_errors() == 0, (world, r, call)
        all_ids = [inp[1].cpu().numpy() for inp in inputs]
        counts, remote, received = EPO.place_pairs(all_ids, E, world, blocks[0].capacity)
        for r, blk in enumerate(blocks):
            seg_off, seg_cnt, send_base, dropped = EPO.ep_layout(counts, world, r, blk.capacity)
            assert not dropped
            assert np.array_equal(blk._mat.cpu().numpy(), counts), (r, call)
            assert np.array_equal(blk.seg_offsets.cpu().numpy(), seg_off), (r, call)
            assert np.array_equal(blk.seg_counts.cpu().numpy(), seg_cnt), (r, call)
            assert np.array_equal(blk.send_base.cpu().numpy(), send_base), (r, call)
            assert np.array_equal(blk.remote_rows.cpu().numpy(), remote[r]), (r, call)
            # The codes that arrived in this owner's slab are the sources' quantised tokens.
            recv = blk._recv_codes.cpu().numpy()
            qx = [b._qx.cpu().numpy() for b in blocks]
            rows = np.array(sorted(received[r]), dtype=np.int64)
            src = np.array([received[r][int(i)] for i in rows], dtype=np.int64).reshape(-1, 2)
            if rows.size:
                expect = np.stack([qx[q][t] for q, t in src])
                assert np.array_equal(recv[rows], expect), (r, call)
        for r, blk in enumerate(blocks):
            x, ids, wts = inputs[r]
            ref = ref_blk.run(x, ids, wts)
            torch.cuda.synchronize()
            out = outs[r]
            assert bool(torch.isfinite(out.float()).all()), (r, call)
            if cta == "single" and mode == "rows":
                assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (world, r, call)
            elif cta == "single":
                dest = ref_blk.dest.cpu().numpy().reshape(T, TOPK)
                y = ref_blk._y.cpu().numpy()[np.maximum(dest, 0)]
                kept = blk.remote_rows.cpu().numpy().reshape(T, TOPK) >= 0
                assert np.array_equal(kept, dest >= 0), (r, call)
                owner = ids.cpu().numpy() // epr
                part, has, bits = EPO.presum_combine(y, kept, owner, wts.cpu().numpy(), world)
                ret = blk._ret.cpu().numpy()
                assert np.array_equal(ret[has].view(np.uint16), part[has].view(np.uint16)), (r, call)
                assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), bits), \
                    (world, r, call)
            else:
                rel = float((out.float() - ref.float()).norm() / ref.float().norm())
                assert rel < 1e-2, (world, r, call, rel)


ROWS = [5, 0, 130, 64, 1, 300, 17, 0, 256, 9, 40, 128, 77, 3, 0, 200]  # 16 experts, some empty
N, K = 256, 512


def _check_gemm(prob, gated):
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
        assert res["ok"], (i, res)


@pytest.mark.parametrize("gated", [False, True], ids=["plain", "gated"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_gather_emulated(pkg, world, gated):
    EP = pkg.expert_parallel
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fab = EP.SingleDeviceFabric(world, dev)
    gats, probs = [], []
    for r in range(world):
        sh = EP.expert_shard(len(ROWS), world, r)
        prob = pkg.workloads.make_problem(f"ep{r}", ROWS[sh.start:sh.stop], N, K, gated=gated,
                                          seed=100 + r, device=dev, alpha_range=(0.5, 2.0))
        gat = EP.FusedOutputGather(ROWS, N, dev, fabric=fab.rank_view(r))
        prob.c = list(gat.local_outputs)
        gats.append(gat)
        probs.append(prob)
    for call in range(2):
        if call:
            for prob in probs:
                for t in prob.a:
                    t ^= 0x11  # new operand values behind the same pointers
        for gat, prob in zip(gats, probs):
            gat.gemm(prob.a, prob.b, prob.sfa, prob.sfb, prob.problem_sizes(), alpha=prob.alpha,
                     b2=prob.b2, sfb2=prob.sfb2, alpha2=prob.alpha2)
        for gat in gats:
            gat.barrier()
        torch.cuda.synchronize()
        for gat, prob in zip(gats, probs):
            assert gat.check_device_errors() == 0
            _check_gemm(prob, gated)
        owners = [c.cpu().numpy() for prob in probs for c in prob.c]  # global expert order
        for r, gat in enumerate(gats):
            assert len(gat.outputs) == len(ROWS)
            for g, (x, y) in enumerate(zip(gat.outputs, owners)):
                assert x.shape == (ROWS[g], N)
                assert np.array_equal(x.cpu().numpy().view(np.uint16), y.view(np.uint16)), \
                    (world, r, g, call)
