"""CPU oracle for the NVFP4 activation quantiser -- TEST INFRASTRUCTURE ONLY.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
use this module, and only as a checker or as the timed CPU baseline.

The reference has no quantiser: its inputs arrive already as e2m1 codes and E4M3 scales
(REFERENCE_IMPL.md:143-205 generates them directly). This file restates the published
two-level NVFP4 scaling recipe (NVIDIA's NVFP4 format description: 16-element blocks,
one E4M3 scale per block, one fp32 scale per tensor) with every fp32 operation spelled
out, so that the CUDA kernel can be required to match it bit for bit:

  d6      = fp32(6 * s_g)                       s_g: per-tensor fp32 scale (> 0)
  sf_f32  = fp32(amax_block / d6)                amax over the 16 elements of the block
  sf      = E4M3(sf_f32)                         round to nearest even, saturate to 448
  enc     = fp32(1 / fp32(value(sf) * s_g))      0 when value(sf) == 0
  q_i     = E2M1(fp32(x_i * enc))                round to nearest even, saturate to +-6

so that x_i ~= value(q_i) * value(sf) * s_g. Choosing s_g = amax_tensor / (6 * 448) keeps
every block scale in E4M3's range. Parity against the reference is unpinned (the reference
has no such function); the oracle itself is checked on hand-computed cases (ties, zeros,
saturation, subnormal scales) in tests/test_quant_oracle.py.
"""
from __future__ import annotations

import numpy as np

from .nvfp4_oracle import E2M1_VALUES, E4M3_VALUES, to_blocked

_E4M3_POS = E4M3_VALUES[:0x7F].astype(np.float64)   # codes 0x00..0x7E: 0 .. 448, increasing
_E2M1_POS = E2M1_VALUES[:8].astype(np.float64)      # codes 0..7: 0 .. 6, increasing


def _round_to_table(v: np.ndarray, table: np.ndarray, sign_bit: int) -> np.ndarray:
    """Nearest entry of a non-negative increasing code table, ties to the even code,
    saturating above the last entry; the sign goes to `sign_bit`."""
    v = np.asarray(v, dtype=np.float32)
    mag = np.minimum(np.abs(v).astype(np.float64), table[-1])
    hi = np.clip(np.searchsorted(table, mag, side="left"), 0, len(table) - 1)
    lo = np.maximum(hi - 1, 0)
    d_lo = mag - table[lo]
    d_hi = table[hi] - mag
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    neg = np.signbit(v)
    return np.where(neg, code | sign_bit, code).astype(np.uint8)


def e4m3_rne_satfinite(v: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn code, round to nearest even, saturating to +-448."""
    return _round_to_table(v, _E4M3_POS, 0x80)


def e2m1_rne_satfinite(v: np.ndarray) -> np.ndarray:
    """fp32 -> e2m1 code (4 bits), round to nearest even, saturating to +-6."""
    return _round_to_table(v, _E2M1_POS, 0x8)


def quantize_nvfp4(x: np.ndarray, global_scale: float):
    """x [rows, cols] (float32 holding bf16/fp16 values), cols % 16 == 0.

    Returns (packed uint8 [rows, cols/2] with the even element in the low nibble,
    plain scales uint8 [rows, cols/16]).
    """
    x = np.asarray(x, dtype=np.float32)
    rows, cols = x.shape
    assert cols % 16 == 0
    sg = np.float32(global_scale)
    blocks = x.reshape(rows, cols // 16, 16)
    amax = np.max(np.abs(blocks), axis=2)
    d6 = np.float32(np.float32(6.0) * sg)
    sf_f32 = (amax / d6).astype(np.float32)
    sf = e4m3_rne_satfinite(sf_f32)
    sval = E4M3_VALUES[sf].astype(np.float32)
    denom = (sval * sg).astype(np.float32)
    with np.errstate(divide="ignore"):
        enc = np.where(sval > 0, (np.float32(1.0) / np.where(denom > 0, denom, 1)).astype(np.float32),
                       np.float32(0.0)).astype(np.float32)
    scaled = (blocks * enc[:, :, None]).astype(np.float32)
    q = e2m1_rne_satfinite(scaled).reshape(rows, cols)
    packed = (q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)
    return packed.astype(np.uint8), sf


def quantize_nvfp4_blocked(x: np.ndarray, global_scale: float):
    """As quantize_nvfp4, with the scales in the GEMM's 128x4-blocked layout."""
    packed, sf = quantize_nvfp4(x, global_scale)
    return packed, to_blocked(sf)


def dequantize_nvfp4(packed: np.ndarray, sf: np.ndarray, global_scale: float) -> np.ndarray:
    rows = packed.shape[0]
    q = np.empty((rows, packed.shape[1] * 2), dtype=np.float32)
    q[:, 0::2] = E2M1_VALUES[packed & 0xF]
    q[:, 1::2] = E2M1_VALUES[packed >> 4]
    return q * np.repeat(E4M3_VALUES[sf], 16, axis=1) * np.float32(global_scale)
