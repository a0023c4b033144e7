"""MoE block on the GPU: routing, gather-quantise and combine bit-exact against their CPU
oracles; the whole feed-forward block checked stage by stage against the oracles and end
to end against a bf16 dense computation."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4_moe_oracle as M
from oracle import nvfp4_oracle as O
from oracle import nvfp4_quant_oracle as Q

pytestmark = pytest.mark.gpu


def _ids(tokens, topk, experts, seed, drop=0.0, invalid=0.0):
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    ids = np.stack([rng.choice(experts, size=topk, replace=False, p=p) for _ in range(tokens)])
    mask = rng.random(ids.shape)
    ids[mask < drop] = -1
    ids[(mask >= drop) & (mask < drop + invalid)] = experts + 3
    return ids.astype(np.int32)


@pytest.mark.parametrize("tokens,topk,experts,drop", [(1, 1, 1, 0.0), (37, 2, 8, 0.1),
                                                     (4096, 8, 64, 0.02), (32768, 8, 256, 0.0)])
def test_route_bit_exact(pkg, tokens, topk, experts, drop):
    ids = _ids(tokens, topk, experts, seed=tokens + experts, drop=drop, invalid=drop / 2)
    r = pkg.moe.route(torch.from_numpy(ids).cuda(), experts)
    counts, offsets, dest, src = M.route(ids, experts)
    assert r.counts == counts.tolist()
    assert r.offsets == offsets.tolist()
    assert np.array_equal(r.dest.cpu().numpy(), dest)
    assert np.array_equal(r.src_rows[:r.rows].cpu().numpy(), src)


def test_gather_quantize_and_combine_bit_exact(pkg):
    tokens, topk, experts, hdim = 300, 4, 16, 512
    ids = _ids(tokens, topk, experts, seed=5, drop=0.05)
    x = (torch.randn((tokens, hdim), generator=torch.Generator().manual_seed(2)) * 2).to(torch.bfloat16)
    r = pkg.moe.route(torch.from_numpy(ids).cuda(), experts)
    sg = float(x.abs().amax().float()) / (6 * 448)
    a, sf = pkg.moe.quantize_rows(x.cuda(), r.rows, r.src_rows, pkg._native.ROWS_GATHER, sg)
    torch.cuda.synchronize()
    src = r.src_rows[:r.rows].cpu().numpy()
    xg = np.where(src[:, None] >= 0, x.float().numpy()[np.maximum(src, 0)], 0.0).astype(np.float32)
    exp_packed, exp_sf = Q.quantize_nvfp4_blocked(xg, sg)
    assert np.array_equal(a.cpu().numpy(), exp_packed)
    assert np.array_equal(sf.cpu().numpy()[:exp_sf.size], exp_sf)
    # Quantise once, then gather: the same bytes.
    qx, sfx = pkg.quantize(x.cuda(), sg)
    a2, sf2 = pkg.moe.gather_quantized(qx, sfx, r)
    torch.cuda.synchronize()
    assert torch.equal(a2, a)
    assert torch.equal(sf2[:exp_sf.size], sf[:exp_sf.size])
    # combine of an arbitrary fp16 dispatched buffer
    y = (torch.randn((r.rows, hdim), generator=torch.Generator().manual_seed(3))).to(torch.float16)
    w = torch.rand((tokens, topk), generator=torch.Generator().manual_seed(4))
    out = pkg.moe.combine(y.cuda(), r, w.cuda())
    torch.cuda.synchronize()
    exp = M.combine(y.numpy(), r.dest.cpu().numpy(), w.numpy())
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), exp)


def test_moe_ffn_stage_by_stage_and_end_to_end(pkg):
    tokens, topk, experts, hdim, idim = 256, 2, 8, 512, 256
    g = torch.Generator().manual_seed(11)
    x = (torch.randn((tokens, hdim), generator=g)).to(torch.bfloat16).cuda()
    gate = [(torch.randn((idim, hdim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    up = [(torch.randn((idim, hdim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    down = [(torch.randn((hdim, idim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    ids = torch.from_numpy(_ids(tokens, topk, experts, seed=7)).cuda()
    wts = torch.softmax(torch.randn((tokens, topk), generator=g), dim=1).cuda()
    W = pkg.moe.quantize_expert_weights(gate, up, down)
    out = pkg.moe.moe_ffn(x, ids, wts, W)
    torch.cuda.synchronize()
    assert out.shape == (tokens, hdim) and out.dtype == torch.bfloat16
    assert torch.isfinite(out.float()).all()
    # End to end against the dense bf16 computation (NVFP4 error of two chained GEMMs).
    ref = torch.zeros((tokens, hdim), dtype=torch.float32, device="cuda")
    xf = x.float()
    for t_slot in range(topk):
        e_col = ids[:, t_slot].long()
        for e in range(experts):
            sel = (e_col == e).nonzero().flatten()
            if sel.numel() == 0:
                continue
            h = torch.nn.functional.silu(xf[sel] @ gate[e].float().t()) * (xf[sel] @ up[e].float().t())
            ref[sel] += wts[sel, t_slot:t_slot + 1] * (h @ down[e].float().t())
    rel = (torch.linalg.norm(out.float() - ref) / torch.linalg.norm(ref)).item()
    assert rel < 0.3, rel
    # Stage by stage: the gate/up GEMM of the dispatched, quantised rows against the oracle.
    r = pkg.moe.route(ids, experts)
    s_x = pkg.global_scale_for(x)
    a, sfa = pkg.moe.quantize_rows(x, r.rows, r.src_rows, pkg._native.ROWS_GATHER, s_x)
    h = torch.zeros((r.rows, idim), dtype=torch.float16, device="cuda")
    av, sfav, hv, m = pkg.moe.expert_views(r, a, sfa, h, hdim)
    pkg.grouped_gemm(av, W.w_gate, sfav, W.sf_gate, hv, [(mi, idim, hdim) for mi in m],
                     alpha=[s_x * s for s in W.s_gate], b2=W.w_up, sfb2=W.sf_up,
                     alpha2=[s_x * s for s in W.s_up])
    torch.cuda.synchronize()
    for e in range(experts):
        if m[e] == 0:
            continue
        ae = av[e].cpu().numpy()
        sfa_e = O.from_blocked(sfav[e].cpu().numpy(), m[e], hdim // 16)
        bg, bu = W.w_gate[e].cpu().numpy(), W.w_up[e].cpu().numpy()
        sfg = O.from_blocked(W.sf_gate[e].cpu().numpy(), idim, hdim // 16)
        sfu = O.from_blocked(W.sf_up[e].cpu().numpy(), idim, hdim // 16)
        exp = O.ref_gated(ae, bg, bu, sfa_e, sfg, sfu, s_x * W.s_gate[e], s_x * W.s_up[e])
        res = O.compare_fp16(hv[e].cpu().numpy(), exp, None, rtol=1e-2, atol=1e-2)
        assert res["ok"], (e, res)


@pytest.mark.parametrize("tokens,topk,experts", [(1, 1, 4), (3, 2, 64), (0, 2, 4)])
def test_moe_ffn_edge_cases(pkg, tokens, topk, experts):
    """A single token, most experts unused, and an empty batch."""
    hdim, idim = 256, 256
    g = torch.Generator().manual_seed(tokens + experts)
    x = torch.randn((tokens, hdim), generator=g).to(torch.bfloat16).cuda()
    gate = [(torch.randn((idim, hdim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    up = [(torch.randn((idim, hdim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    down = [(torch.randn((hdim, idim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    W = pkg.moe.quantize_expert_weights(gate, up, down)
    ids = torch.from_numpy(_ids(tokens, topk, experts, seed=3) if tokens else
                           np.zeros((0, topk), dtype=np.int32)).cuda()
    wts = torch.full((tokens, topk), 1.0 / topk, device="cuda")
    out = pkg.moe.moe_ffn(x, ids, wts, W, act_scale=0.01, hidden_scale=0.001)
    torch.cuda.synchronize()
    assert out.shape == (tokens, hdim)
    if tokens:
        assert torch.isfinite(out.float()).all()
        r = pkg.moe.route(ids, experts)
        assert sum(r.counts) == tokens * topk and r.rows % 128 == 0
