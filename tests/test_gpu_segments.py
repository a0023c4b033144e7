"""Segment launches (nvfp4_grouped_gemm_segments): every group's rows are read on the GPU
from device offsets/counts over one slab. Checked bit-identical to the host-sized launch of
the same rows, rows outside every segment left untouched, out-of-range segments skipped
with a device error, descriptor reuse across different segments; and the MoE block built on
them (MoEBlock: no host read) equal to moe_ffn and replayable as a CUDA graph."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

SENTINEL = -7.0


def _codes(g, rows, cols):
    # e2m1 codes of the reference generator's value set {0, +-0.5, +-1, +-1.5}.
    return (torch.randint(0, 256, (rows, cols // 2), generator=g, dtype=torch.int32)
            .to(torch.uint8) & 0xBB).cuda()


def _scales(pkg, g, rows, cols):
    plain = torch.where(torch.rand((rows, cols // 16), generator=g) < 0.5,
                        torch.tensor(0x38, dtype=torch.uint8), torch.tensor(0x40, dtype=torch.uint8))
    return pkg.plain_to_blocked(plain.cuda())


def _segments(counts, gaps=None, tail=0):
    """128-aligned offsets of the given counts (plus `gaps[e]` 128-row blocks before
    segment e) and the slab rows needed (plus `tail` rows)."""
    offs, r = [], 0
    for e, c in enumerate(counts):
        r += 128 * (gaps[e] if gaps else 0)
        offs.append(r)
        r += (c + 127) // 128 * 128
    return offs, r + tail


def _slab_problem(pkg, counts, n, k, gated, seed, gaps=None, tail=40):
    g = torch.Generator().manual_seed(seed)
    offs, cap = _segments(counts, gaps, tail)
    G = len(counts)
    a = _codes(g, cap, k)
    sfa = _scales(pkg, g, cap, k)
    b = [_codes(g, n, k) for _ in range(G)]
    sfb = [_scales(pkg, g, n, k) for _ in range(G)]
    b2 = [_codes(g, n, k) for _ in range(G)] if gated else None
    sfb2 = [_scales(pkg, g, n, k) for _ in range(G)] if gated else None
    alpha = [float(v) for v in torch.rand(G, generator=g) * 0.02 + 0.01]
    alpha2 = [float(v) for v in torch.rand(G, generator=g) * 0.02 + 0.01] if gated else None
    return dict(offs=offs, cap=cap, a=a, sfa=sfa, b=b, sfb=sfb, b2=b2, sfb2=sfb2, alpha=alpha,
                alpha2=alpha2, n=n, k=k)


def _host_sized(pkg, P, counts, cta):
    """The same rows through the host-sized entry point (per-group views of the slabs)."""
    k, n = P["k"], P["n"]
    c = torch.full((P["cap"], n), SENTINEL, dtype=torch.float16, device="cuda")
    sf_block = (k // 64) * 512
    av, sfav, cv = [], [], []
    for off, cnt in zip(P["offs"], counts):
        av.append(P["a"][off:off + cnt])
        b0 = (off // 128) * sf_block
        sfav.append(P["sfa"][b0:b0 + max(pkg.blocked_sf_bytes(cnt, k // 16), 0)])
        cv.append(c[off:off + cnt])
    pkg.grouped_gemm(av, P["b"], sfav, P["sfb"], cv, [(cnt, n, k) for cnt in counts],
                     alpha=P["alpha"], b2=P["b2"], sfb2=P["sfb2"], alpha2=P["alpha2"], cta=cta)
    return c


def _segment_launch(pkg, P, offs, counts, cta, expected_rows=0):
    c = torch.full((P["cap"], P["n"]), SENTINEL, dtype=torch.float16, device="cuda")
    so = torch.tensor(offs, dtype=torch.int32, device="cuda")
    sc = torch.tensor(counts, dtype=torch.int32, device="cuda")
    pkg.grouped_gemm_segments(P["a"], P["sfa"], c, P["b"], P["sfb"], so, sc, alpha=P["alpha"],
                              b2=P["b2"], sfb2=P["sfb2"], alpha2=P["alpha2"],
                              expected_rows=expected_rows, cta=cta)
    return c


def _assert_segments_equal(got, ref, offs, counts, cap):
    covered = np.zeros(cap, dtype=bool)
    for e, (off, cnt) in enumerate(zip(offs, counts)):
        assert torch.equal(got[off:off + cnt].view(torch.int16), ref[off:off + cnt].view(torch.int16)), \
            f"segment {e} (rows {off}..{off + cnt}) differs"
        covered[off:off + (cnt + 127) // 128 * 128] = True
    # Rows outside every segment's 128-row-padded range are never written.
    outside = torch.from_numpy(np.nonzero(~covered)[0]).cuda()
    if outside.numel():
        assert bool((got[outside] == SENTINEL).all()), "a row outside every segment was written"


SEG_CASES = [
    # (name, counts, n, k, gated, gaps)
    ("ragged", [0, 1, 127, 128, 129, 300, 0, 64], 512, 512, False, None),
    ("gaps", [5, 200, 33], 264, 1024, False, [1, 0, 2]),
    ("gated", [0, 64, 300, 129, 1], 256, 512, True, None),
    ("tall", [700, 512, 256], 512, 2048, False, None),
]


@pytest.mark.parametrize("cta", [None, "single", "pair"])
@pytest.mark.parametrize("case", SEG_CASES, ids=[c[0] for c in SEG_CASES])
def test_segments_match_host_sized_launch(pkg, case, cta):
    name, counts, n, k, gated, gaps = case
    P = _slab_problem(pkg, counts, n, k, gated, seed=len(counts) * 7 + n, gaps=gaps)
    ref = _host_sized(pkg, P, counts, cta)
    for expected in (0, sum(counts)):
        got = _segment_launch(pkg, P, P["offs"], counts, cta, expected_rows=expected)
        torch.cuda.synchronize()
        _assert_segments_equal(got, ref, P["offs"], counts, P["cap"])
    assert pkg.check_device_errors() == 0


def test_segments_against_oracle(pkg):
    counts, n, k = [3, 130, 0, 77], 256, 512
    P = _slab_problem(pkg, counts, n, k, False, seed=99)
    got = _segment_launch(pkg, P, P["offs"], counts, None)
    torch.cuda.synchronize()
    sfa_plain = O.from_blocked(P["sfa"].cpu().numpy(), P["cap"], k // 16)
    a_np = P["a"].cpu().numpy()
    for e, (off, cnt) in enumerate(zip(P["offs"], counts)):
        if cnt == 0:
            continue
        sfb = O.from_blocked(P["sfb"][e].cpu().numpy(), n, k // 16)
        ref32 = O.ref_gemm_fp32(a_np[off:off + cnt], P["b"][e].cpu().numpy(),
                                sfa_plain[off:off + cnt], sfb) * np.float32(P["alpha"][e])
        res = O.compare_fp16(got[off:off + cnt].cpu().numpy(), ref32.astype(np.float16), ref32,
                             rtol=1e-2, atol=1e-2)
        assert res["ok"], (e, res)


def test_segments_reuse_descriptors_with_new_segments(pkg):
    """Same slabs and weights (descriptors reused), different segments each call."""
    n, k = 256, 512
    P = _slab_problem(pkg, [300, 300, 300], n, k, False, seed=5, tail=0)
    for counts in ([300, 0, 17], [1, 256, 299], [0, 0, 0], [128, 129, 2]):
        ref = _host_sized(pkg, P, counts, None)
        got = _segment_launch(pkg, P, P["offs"], counts, None, expected_rows=sum(counts))
        torch.cuda.synchronize()
        _assert_segments_equal(got, ref, P["offs"], counts, P["cap"])


def test_segments_out_of_range_are_skipped(pkg):
    """A misaligned offset and a segment past the slab's end: both groups are skipped (their
    rows untouched), the others computed, and the device error bit reported."""
    counts, n, k = [100, 50, 60, 10], 256, 512
    P = _slab_problem(pkg, counts, n, k, False, seed=8, tail=0)
    ref = _host_sized(pkg, P, counts, None)
    offs = list(P["offs"])
    offs[1] += 64                    # not a multiple of 128
    bad_counts = list(counts)
    bad_counts[3] = P["cap"]         # runs past the slab
    got = _segment_launch(pkg, P, offs, bad_counts, None)
    with pytest.raises(pkg.Nvfp4Error) as ei:
        pkg.check_device_errors()
    assert "segment" in str(ei.value)
    for e in (0, 2):
        off, cnt = P["offs"][e], counts[e]
        assert torch.equal(got[off:off + cnt], ref[off:off + cnt])
    for e in (1, 3):
        off = P["offs"][e]
        assert bool((got[off:off + 128] == SENTINEL).all())
    assert pkg.check_device_errors() == 0  # the error word was cleared


def test_segments_validation(pkg):
    P = _slab_problem(pkg, [10, 20], 256, 512, False, seed=1)
    so = torch.tensor(P["offs"], dtype=torch.int32, device="cuda")
    sc = torch.tensor([10, 20], dtype=torch.int32, device="cuda")
    c = torch.empty((P["cap"], 256), dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        pkg.grouped_gemm_segments(P["a"], P["sfa"], c, P["b"], P["sfb"], so.long(), sc)
    with pytest.raises(ValueError):
        pkg.grouped_gemm_segments(P["a"], P["sfa"], c, P["b"], P["sfb"], so, sc, cta="weights")
    with pytest.raises(ValueError):  # weights of the wrong width
        pkg.grouped_gemm_segments(P["a"], P["sfa"], c[:, :128], P["b"], P["sfb"], so, sc)


# ----------------------------------------------------------------------------
# The MoE block without host reads
# ----------------------------------------------------------------------------
def _moe_setup(pkg, tokens, topk, experts, hdim, idim, seed):
    g = torch.Generator().manual_seed(seed)
    gate = [(torch.randn((idim, hdim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    up = [(torch.randn((idim, hdim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    down = [(torch.randn((hdim, idim), generator=g) * 0.05).to(torch.bfloat16).cuda() for _ in range(experts)]
    W = pkg.moe.quantize_expert_weights(gate, up, down)
    return W, g


def _moe_inputs(g, tokens, topk, experts, hdim):
    x = torch.randn((tokens, hdim), generator=g).to(torch.bfloat16).cuda()
    scores = torch.rand((tokens, experts), generator=g) ** 3  # skewed
    top = torch.topk(scores, topk, dim=1)
    ids = top.indices.to(torch.int32).cuda()
    wts = torch.softmax(top.values, dim=1).cuda()
    return x, ids, wts


@pytest.mark.parametrize("tokens,topk,experts,hdim,idim", [
    (256, 2, 8, 512, 256), (1, 1, 4, 256, 256), (600, 4, 16, 256, 512), (64, 8, 64, 512, 256)])
def test_moe_block_matches_moe_ffn(pkg, tokens, topk, experts, hdim, idim):
    W, g = _moe_setup(pkg, tokens, topk, experts, hdim, idim, seed=tokens + experts)
    x, ids, wts = _moe_inputs(g, tokens, topk, experts, hdim)
    s_x, s_h = pkg.global_scale_for(x), 0.002
    ref = pkg.moe.moe_ffn(x, ids, wts, W, act_scale=s_x, hidden_scale=s_h)
    blk = pkg.moe.MoEBlock(W, tokens, topk, act_scale=s_x, hidden_scale=s_h)
    out = blk.run(x, ids, wts)
    torch.cuda.synchronize()
    assert blk.check_device_errors() == 0
    assert torch.isfinite(out.float()).all()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_moe_block_graph_replay(pkg):
    """Capture once, then replay on new tokens and a new routing written into the captured
    input buffers: identical to an eager run on the same inputs and to moe_ffn."""
    tokens, topk, experts, hdim, idim = 512, 4, 32, 512, 256
    W, g = _moe_setup(pkg, tokens, topk, experts, hdim, idim, seed=77)
    x, ids, wts = _moe_inputs(g, tokens, topk, experts, hdim)
    s_x, s_h = 0.004, 0.002
    blk = pkg.moe.MoEBlock(W, tokens, topk, act_scale=s_x, hidden_scale=s_h)
    graph = blk.capture(x, ids, wts)
    for rep in range(3):
        x2, ids2, wts2 = _moe_inputs(g, tokens, topk, experts, hdim)
        x.copy_(x2)
        ids.copy_(ids2)
        wts.copy_(wts2)
        graph.replay()
        torch.cuda.synchronize()
        got = blk.out.clone()
        ref = pkg.moe.moe_ffn(x, ids, wts, W, act_scale=s_x, hidden_scale=s_h)
        eager = blk.run(x, ids, wts)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), eager.view(torch.int16)), rep
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), rep
    assert blk.check_device_errors() == 0
    del graph


@pytest.mark.parametrize("cta", [None, "single", "pair"])
def test_gated_nvfp4_output_equals_quantised_fp16_output(pkg, cta):
    """The gated segment launch writing NVFP4 codes and blocked scales is bit-identical to
    the fp16 launch followed by the activation quantiser (over the real rows)."""
    counts, n, k = [0, 1, 127, 300, 129, 64], 256, 1024
    P = _slab_problem(pkg, counts, n, k, True, seed=31, tail=0)
    cap = P["cap"]
    so = torch.tensor(P["offs"], dtype=torch.int32, device="cuda")
    sc = torch.tensor(counts, dtype=torch.int32, device="cuda")
    h = torch.zeros((cap, n), dtype=torch.float16, device="cuda")
    kw = dict(alpha=P["alpha"], b2=P["b2"], sfb2=P["sfb2"], alpha2=P["alpha2"], cta=cta)
    pkg.grouped_gemm_segments(P["a"], P["sfa"], h, P["b"], P["sfb"], so, sc, **kw)
    s_h = pkg.global_scale_for(h)
    ref_codes, ref_sf = pkg.quantize(h, s_h)
    codes = torch.full((cap, n // 2), 0x5A, dtype=torch.uint8, device="cuda")
    sf = torch.full((pkg.blocked_sf_bytes(cap, n // 16),), 0x5A, dtype=torch.uint8, device="cuda")
    pkg.grouped_gemm_segments(P["a"], P["sfa"], codes, P["b"], P["sfb"], so, sc, out_sf=sf,
                              out_scale=s_h, **kw)
    torch.cuda.synchronize()
    assert pkg.check_device_errors() == 0
    plain = pkg.blocked_to_plain(sf, cap, n // 16)
    ref_plain = pkg.blocked_to_plain(ref_sf, cap, n // 16)
    for e, (off, cnt) in enumerate(zip(P["offs"], counts)):
        assert torch.equal(codes[off:off + cnt], ref_codes[off:off + cnt]), f"codes of segment {e}"
        assert torch.equal(plain[off:off + cnt], ref_plain[off:off + cnt]), f"scales of segment {e}"
    with pytest.raises(ValueError):  # non-gated launches have no NVFP4 output
        pkg.grouped_gemm_segments(P["a"], P["sfa"], codes, P["b"], P["sfb"], so, sc, out_sf=sf,
                                  out_scale=s_h)


@pytest.mark.parametrize("cta", [None, "single", "pair"])
def test_scattered_output_rows(pkg, cta):
    """Non-gated segment launch with scattered output: every slab row lands, bit for bit as
    the fp16 launch computes it, at the (buffer, row) its row_dest entry names; rows marked
    -1 and rows outside the segments are stored nowhere."""
    counts, n, k = [0, 1, 127, 300, 129, 64], 256, 1024
    P = _slab_problem(pkg, counts, n, k, False, seed=47, tail=0)
    cap = P["cap"]
    ref = _segment_launch(pkg, P, P["offs"], counts, cta)
    rng = np.random.default_rng(3)
    rows = [r for off, cnt in zip(P["offs"], counts) for r in range(off, off + cnt)]
    perm = rng.permutation(2 * cap)[:len(rows)]  # target slots over two buffers of cap rows
    code = np.full(cap, -1, dtype=np.int64)
    for r, slot in zip(rows, perm):
        if rng.random() < 0.1:
            continue  # not stored
        code[r] = (int(slot // cap) << 40) | int(slot % cap)
    dest = [torch.full((cap, n + 8), SENTINEL, dtype=torch.float16, device="cuda") for _ in range(2)]
    c = torch.full((cap, n), SENTINEL, dtype=torch.float16, device="cuda")
    so = torch.tensor(P["offs"], dtype=torch.int32, device="cuda")
    sc = torch.tensor(counts, dtype=torch.int32, device="cuda")
    pkg.grouped_gemm_segments(P["a"], P["sfa"], c, P["b"], P["sfb"], so, sc, alpha=P["alpha"],
                              cta=cta, row_dest=torch.from_numpy(code).cuda(), dest=dest)
    torch.cuda.synchronize()
    assert pkg.check_device_errors() == 0
    assert bool((c == SENTINEL).all()), "c must not be written"
    want = [torch.full((cap, n + 8), SENTINEL, dtype=torch.float16) for _ in range(2)]
    ref_cpu = ref.cpu()
    for r in range(cap):
        if code[r] >= 0:
            want[code[r] >> 40][code[r] & ((1 << 40) - 1), :n] = ref_cpu[r]
    for b in range(2):
        assert torch.equal(dest[b].cpu().view(torch.int16), want[b].view(torch.int16)), b
