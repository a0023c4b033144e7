"""NVFP4 activation quantiser on the GPU: bit-exact against the CPU oracle, and its output
used as the GEMM's A operand (the GEMM result checked against the oracle GEMM of the same
quantised data, and against the unquantised bf16 product within the format's error)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from oracle import nvfp4_quant_oracle as Q

pytestmark = pytest.mark.gpu


def _inputs(rows, cols, dtype, seed, ld=None):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn((rows, cols), generator=g) * 4.0
    # Special values: exact ties of the scaled grid, zero blocks, one large outlier per
    # tensor, tiny values whose block scale is subnormal in E4M3.
    if rows > 2 and cols >= 64:
        x[0, :16] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2)
        x[1, 16:32] = 0.0
        x[2, 32:48] = 1e-6 * torch.arange(16)
        x[rows // 2, cols // 2] = 900.0
    x = x.to(dtype)
    if ld is not None:
        wide = torch.zeros((rows, ld), dtype=dtype)
        wide[:, :cols] = x
        return wide.cuda()[:, :cols], x.float().numpy()
    return x.cuda(), x.float().numpy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols,ld", [(1, 64, None), (128, 256, None), (200, 448, None),
                                          (300, 1024, 1088), (1024, 7168, None)])
def test_quantize_bit_exact_against_oracle(pkg, dtype, rows, cols, ld):
    x, xf = _inputs(rows, cols, dtype, seed=rows + cols, ld=ld)
    for sg in (1.0, float(np.abs(xf).max()) / (6 * 448), 0.37):
        packed, sf = pkg.quantize(x, sg)
        torch.cuda.synchronize()
        exp_packed, exp_sf = Q.quantize_nvfp4(xf, sg)
        got_packed = packed.cpu().numpy()
        assert np.array_equal(got_packed, exp_packed), (
            f"packed mismatch at {np.argwhere(got_packed != exp_packed)[:5].tolist()}")
        got_sf = sf.cpu().numpy()
        assert np.array_equal(got_sf, O.to_blocked(exp_sf)), "scale mismatch"


def test_quantize_padding_rows_are_zero_and_outputs_in_place(pkg):
    rows, cols = 130, 128
    x, xf = _inputs(rows, cols, torch.bfloat16, seed=9)
    sf = torch.full((pkg.blocked_sf_bytes(rows, cols // 16),), 0xAB, dtype=torch.uint8,
                    device="cuda")
    packed = torch.full((rows, cols // 2), 0xCD, dtype=torch.uint8, device="cuda")
    p2, s2 = pkg.quantize(x, 0.5, packed=packed, sf=sf)
    assert p2.data_ptr() == packed.data_ptr() and s2.data_ptr() == sf.data_ptr()
    plain = O.from_blocked(sf.cpu().numpy(), 256, cols // 16)
    assert np.all(plain[rows:] == 0)
    exp_packed, exp_sf = Q.quantize_nvfp4(xf, 0.5)
    assert np.array_equal(plain[:rows], exp_sf)
    assert np.array_equal(packed.cpu().numpy(), exp_packed)


def test_quantize_validation(pkg):
    x = torch.zeros((4, 96), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        pkg.quantize(x, 1.0)          # cols % 64
    x = torch.zeros((4, 64), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        pkg.quantize(x, 1.0)          # dtype
    x = torch.zeros((4, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        pkg.quantize(x, 0.0)          # scale
    packed, sf = pkg.quantize(torch.zeros((0, 64), dtype=torch.bfloat16, device="cuda"), 1.0)
    assert packed.shape == (0, 32) and sf.numel() == 0


@pytest.mark.parametrize("m,n,k", [(256, 512, 1024), (100, 256, 512)])
def test_quantized_activations_through_the_gemm(pkg, m, n, k):
    """Activations and weights quantised on the GPU feed the grouped GEMM; alpha carries
    both global scales. Exact against the oracle GEMM of the same codes, and close to the
    bf16 product of the unquantised inputs."""
    g = torch.Generator(device="cpu").manual_seed(m + n + k)
    xa = (torch.randn((m, k), generator=g)).to(torch.bfloat16).cuda()
    xb = (torch.randn((n, k), generator=g) * 0.05).to(torch.bfloat16).cuda()
    sa, sb = pkg.global_scale_for(xa), pkg.global_scale_for(xb)
    a, sfa = pkg.quantize(xa, sa)
    b, sfb = pkg.quantize(xb, sb)
    c = torch.empty((m, n), dtype=torch.float16, device="cuda")
    pkg.grouped_gemm([a], [b], [sfa], [sfb], [c], [(m, n, k)], alpha=[sa * sb])
    torch.cuda.synchronize()
    got = c.cpu().numpy()
    sfa_plain = O.from_blocked(sfa.cpu().numpy(), m, k // 16)
    sfb_plain = O.from_blocked(sfb.cpu().numpy(), n, k // 16)
    ref32 = O.ref_gemm_fp32(a.cpu().numpy(), b.cpu().numpy(), sfa_plain, sfb_plain) * np.float32(sa * sb)
    res = O.compare_fp16(got, ref32.astype(np.float16), ref32, rtol=1e-2, atol=1e-2)
    assert res["ok"], res
    exact = (xa.float() @ xb.float().t()).cpu().numpy()
    rel = np.linalg.norm(got.astype(np.float32) - exact) / np.linalg.norm(exact)
    assert rel < 0.15, rel
