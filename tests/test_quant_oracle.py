"""The NVFP4 quantiser oracle on hand-computed cases (CPU only).

The reference has no quantiser, so these cases pin the oracle to the format definitions:
E4M3 and E2M1 rounding to nearest with ties to the even code, saturation, subnormal scales,
zero blocks, and the two-level scale recipe.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import nvfp4_oracle as O
from oracle import nvfp4_quant_oracle as Q


@pytest.mark.parametrize("v,code", [
    (0.0, 0), (0.25, 0), (0.26, 1), (0.5, 1), (0.75, 2), (1.25, 2), (1.5, 3), (1.75, 4),
    (2.5, 4), (3.0, 5), (3.5, 6), (5.0, 6), (5.01, 7), (6.0, 7), (7.0, 7), (1e9, 7),
    (-0.75, 0xA), (-6.5, 0xF), (-0.1, 0x8),
])
def test_e2m1_rounding(v, code):
    assert int(Q.e2m1_rne_satfinite(np.float32(v))) == code


@pytest.mark.parametrize("v,code", [
    (0.0, 0x00), (1.0, 0x38), (2.0, 0x40), (448.0, 0x7E), (500.0, 0x7E), (1e30, 0x7E),
    (2.0 ** -9, 0x01), (2.0 ** -10, 0x00), (1.5 * 2.0 ** -10, 0x01), (7 * 2.0 ** -9, 0x07),
    (2.0 ** -6, 0x08), (1.0625, 0x38), (1.1875, 0x3A), (1.125, 0x39),
])
def test_e4m3_rounding(v, code):
    assert int(Q.e4m3_rne_satfinite(np.float32(v))) == code
    assert O.E4M3_VALUES[code] == pytest.approx(min(v, 448.0), rel=0.07, abs=2.0 ** -10)


def test_quantize_hand_cases():
    x = np.zeros((2, 32), dtype=np.float32)
    x[0, :16] = 6.0                      # amax 6, s_g 1 -> scale 1.0, codes 7
    x[0, 16:] = np.linspace(-3, 3, 16)   # amax 3 -> scale 0.5 (0x30); x / 0.5 on the e2m1 grid?
    x[1, :16] = 0.0                      # zero block -> scale 0, codes 0
    x[1, 16] = 1000.0                    # saturating block: scale 1000/6 -> E4M3 160 (0x6A? rounded)
    packed, sf = Q.quantize_nvfp4(x, 1.0)
    assert sf[0, 0] == 0x38 and np.all(packed[0, :8] == 0x77)
    assert sf[0, 1] == Q.e4m3_rne_satfinite(np.float32(0.5)) == 0x30
    assert np.all(packed[1, :8] == 0) and sf[1, 0] == 0
    s = O.E4M3_VALUES[sf[1, 1]]
    assert s == O.E4M3_VALUES[Q.e4m3_rne_satfinite(np.float32(1000.0 / 6.0))]
    deq = Q.dequantize_nvfp4(packed, sf, 1.0)
    assert deq[0, 0] == 6.0
    assert deq[1, 16] == pytest.approx(1000.0, rel=0.1)


def test_global_scale_keeps_scales_finite_and_round_trip_error_small():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((64, 256)) * 3.0).astype(np.float32)
    x[3, 7] = 80.0
    sg = float(np.abs(x).max()) / (6 * 448)
    packed, sf = Q.quantize_nvfp4(x, sg)
    assert sf.max() <= 0x7E
    deq = Q.dequantize_nvfp4(packed, sf, sg)
    rel = np.linalg.norm(deq - x) / np.linalg.norm(x)
    assert rel < 0.12, rel
    # every element is within half an e2m1 step of its block scale, or saturated
    assert np.abs(deq[3, 7] - 80.0) <= 80.0 * 0.2


def test_blocked_variant_is_to_blocked():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((200, 128)).astype(np.float32)
    packed, blocked = Q.quantize_nvfp4_blocked(x, 0.01)
    p2, sf = Q.quantize_nvfp4(x, 0.01)
    assert np.array_equal(packed, p2)
    assert np.array_equal(blocked, O.to_blocked(sf))
    assert np.array_equal(O.from_blocked(blocked, 200, 8), sf)
