"""CPU oracle for the NVFP4 block-scaled grouped GEMM -- TEST INFRASTRUCTURE ONLY.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may use this module, and only as a checker or as the timed CPU
baseline. The product path (the CUDA library behind ``custom_kernel``) never
calls it.

A numpy restatement of the reference harness (REFERENCE_IMPL.md), which itself
runs on the GPU through ``torch._scaled_mm`` (cuBLASLt) and so cannot run on a
CPU (``_scaled_mm`` rejects block-scaled FP4 on CPU):

* ``to_blocked``           REFERENCE_IMPL.md:19-42
* ``reorder_scales``       REFERENCE_IMPL.md:89-137 (create_reordered_scale_factor_tensor)
* ``ref_grouped_gemm``     REFERENCE_IMPL.md:48-81 (ref_kernel: dequantise, fp32 matmul, fp16)
* ``ref_gated``            submission.py:877-884 and :707-710 (two fp16 GEMMs, silu(g)*u)
* ``generate_input``       REFERENCE_IMPL.md:143-205 (distribution only; numpy RNG)

Pinning: ``tests/golden/`` holds inputs made by the reference's own generator
and ``to_blocked`` (run on CPU in the build container) and outputs of the
reference's arithmetic (``torch._scaled_mm`` on a B200); the oracle is checked
against both in ``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import numpy as np

SF_VEC = 16

# e2m1: sign | 2-bit exponent (bias 1) | 1-bit mantissa; code 0b0xyz -> value, 8+ negative.
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def _e4m3_table() -> np.ndarray:
    """float8_e4m3fn decoding: bias 7, no infinities, 0x7F/0xFF = NaN, subnormals at e=0."""
    t = np.empty(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_VALUES = _e4m3_table()


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


# ---------------------------------------------------------------------------
# Scale-factor layouts
# ---------------------------------------------------------------------------
def to_blocked(plain: np.ndarray) -> np.ndarray:
    """Restatement of to_blocked (REFERENCE_IMPL.md:19-42) on uint8 codes.

    Pads [rows, cols] to multiples of (128, 4) with zeros, splits it into 128x4
    blocks in row-block-major order and, inside a block, interleaves the four
    32-row bands: output[(blk*32 + r)*16 + band*4 + j] = block[band*32 + r, j].
    """
    rows, cols = plain.shape
    nrb, ncb = ceil_div(rows, 128), ceil_div(cols, 4)
    padded = np.zeros((nrb * 128, ncb * 4), dtype=np.uint8)
    padded[:rows, :cols] = plain
    blocks = padded.reshape(nrb, 128, ncb, 4).transpose(0, 2, 1, 3)     # [rb, cb, 128, 4]
    rearranged = blocks.reshape(-1, 4, 32, 4).transpose(0, 2, 1, 3)      # [blk, 32, band, 4]
    return rearranged.reshape(-1).copy()


def from_blocked(blocked: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Inverse of to_blocked (drops the zero padding)."""
    nrb, ncb = ceil_div(rows, 128), ceil_div(cols, 4)
    b = np.asarray(blocked, dtype=np.uint8).reshape(-1)[: nrb * ncb * 512]
    blocks = b.reshape(nrb * ncb, 32, 4, 4).transpose(0, 2, 1, 3).reshape(nrb, ncb, 128, 4)
    plain = blocks.transpose(0, 2, 1, 3).reshape(nrb * 128, ncb * 4)
    return plain[:rows, :cols].copy()


def reorder_scales(plain: np.ndarray, k: int, pad_value: np.ndarray | None = None) -> np.ndarray:
    """Restatement of create_reordered_scale_factor_tensor (REFERENCE_IMPL.md:89-137).

    Returns the (32, 4, rest_m, 4, rest_k, 1) array with
    out[i%32, (i%128)//32, i//128, j%4, j//4, 0] = plain[i, j]; positions no
    (i, j) maps to keep `pad_value` (the harness leaves random {1, 2} codes there).
    """
    mn, sf_k = plain.shape
    rest_m, rest_k = ceil_div(mn, 128), ceil_div(ceil_div(k, SF_VEC), 4)
    out = np.zeros((32, 4, rest_m, 4, rest_k, 1), dtype=np.uint8)
    if pad_value is not None:
        out[...] = pad_value
    i = np.arange(mn)[:, None]
    j = np.arange(sf_k)[None, :]
    out[i % 32, (i % 128) // 32, i // 128, j % 4, j // 4, 0] = plain
    return out


def reordered_storage(reordered: np.ndarray) -> np.ndarray:
    """Storage order of the reordered tensor: the (l, rest_m, rest_k, 32, 4, 4) allocation."""
    return np.ascontiguousarray(reordered.transpose(5, 2, 4, 0, 1, 3)).reshape(-1)


# ---------------------------------------------------------------------------
# Decoding and GEMM
# ---------------------------------------------------------------------------
def unpack_e2m1(packed: np.ndarray) -> np.ndarray:
    """[rows, K/2] packed bytes -> [rows, K] float32; the low nibble is the even element."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.float32)
    out[..., 0::2] = E2M1_VALUES[p & 0xF]
    out[..., 1::2] = E2M1_VALUES[p >> 4]
    return out


def dequantize(packed: np.ndarray, sf_plain: np.ndarray) -> np.ndarray:
    """Dequantised fp32 operand [rows, K] = e2m1 value * E4M3 scale of its 16-block."""
    vals = unpack_e2m1(packed)
    rows, k = vals.shape
    sf = E4M3_VALUES[np.asarray(sf_plain, dtype=np.uint8)[:rows, : k // SF_VEC]]
    return (vals.reshape(rows, k // SF_VEC, SF_VEC) * sf[:, :, None]).reshape(rows, k)


def ref_gemm_fp32(a: np.ndarray, b: np.ndarray, sfa: np.ndarray, sfb: np.ndarray) -> np.ndarray:
    """fp32 A_deq @ B_deq^T for one group (the product inside ref_kernel)."""
    if a.shape[0] == 0 or b.shape[0] == 0:
        return np.zeros((a.shape[0], b.shape[0]), dtype=np.float32)
    return dequantize(a, sfa) @ dequantize(b, sfb).T


def ref_gemm(a, b, sfa, sfb, alpha: float = 1.0) -> np.ndarray:
    """One group of ref_kernel: fp16(alpha * A_deq @ B_deq^T) (REFERENCE_IMPL.md:71-79)."""
    acc = ref_gemm_fp32(a, b, sfa, sfb)
    if alpha != 1.0:
        acc = acc * np.float32(alpha)
    with np.errstate(over="ignore"):
        return acc.astype(np.float16)


def silu_f32(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def ref_gated(a, b_gate, b_up, sfa, sfb_gate, sfb_up, alpha: float = 1.0,
              alpha2: float = 1.0) -> np.ndarray:
    """fp16(silu(fp16(gate).f32) * fp16(up).f32), the reference's dual-GEMM rounding."""
    g16 = ref_gemm(a, b_gate, sfa, sfb_gate, alpha)
    u16 = ref_gemm(a, b_up, sfa, sfb_up, alpha2)
    with np.errstate(over="ignore", invalid="ignore"):
        out = silu_f32(g16.astype(np.float32)) * u16.astype(np.float32)
        return out.astype(np.float16)


def ref_grouped_gemm(groups) -> list:
    """ref_kernel over a list of dicts with a, b, sfa, sfb (plain), optional alpha / gated keys."""
    outs = []
    for g in groups:
        if "b2" in g and g["b2"] is not None:
            outs.append(ref_gated(g["a"], g["b"], g["b2"], g["sfa"], g["sfb"], g["sfb2"],
                                  g.get("alpha", 1.0), g.get("alpha2", 1.0)))
        else:
            outs.append(ref_gemm(g["a"], g["b"], g["sfa"], g["sfb"], g.get("alpha", 1.0)))
    return outs


# ---------------------------------------------------------------------------
# Input generation (the harness's distribution, numpy RNG)
# ---------------------------------------------------------------------------
def generate_input(m, n, k, g: int, seed: int) -> dict:
    """Distributional restatement of generate_input (REFERENCE_IMPL.md:154-205).

    e2m1 bytes masked with 0b1011_1011 (REFERENCE_IMPL.md:143-151), scales
    randint(1, 3) as E4M3 (1.0 = 0x38, 2.0 = 0x40), L = 1.
    """
    rng = np.random.default_rng(seed)
    out = {"a": [], "b": [], "sfa": [], "sfb": [], "problem_sizes": []}
    for i in range(g):
        mi, ni, ki = int(m[i]), int(n[i]), int(k[i])
        out["a"].append(rng.integers(0, 255, (mi, ki // 2), dtype=np.uint8) & 0b1011_1011)
        out["b"].append(rng.integers(0, 255, (ni, ki // 2), dtype=np.uint8) & 0b1011_1011)
        out["sfa"].append(np.where(rng.integers(1, 3, (mi, ki // 16)) == 1, 0x38, 0x40).astype(np.uint8))
        out["sfb"].append(np.where(rng.integers(1, 3, (ni, ki // 16)) == 1, 0x38, 0x40).astype(np.uint8))
        out["problem_sizes"].append((mi, ni, ki, 1))
    return out


# ---------------------------------------------------------------------------
# Comparison with the harness tolerance semantics
# ---------------------------------------------------------------------------
def compare_fp16(actual: np.ndarray, expected: np.ndarray, ref_fp32: np.ndarray | None = None,
                 rtol: float = 1e-2, atol: float = 1e-2) -> dict:
    """torch.allclose-style check on fp16 outputs with overflow handled explicitly.

    An element matches when |actual - expected| <= atol + rtol*|expected|, or when
    both are infinite with the same sign, or when the fp32 reference magnitude
    exceeds the fp16 range and `actual` is +-inf or +-65504 with the right sign.
    """
    a = np.asarray(actual, dtype=np.float32)
    e = np.asarray(expected, dtype=np.float32)
    finite = np.isfinite(a) & np.isfinite(e)
    with np.errstate(invalid="ignore"):
        close = np.zeros(a.shape, dtype=bool)
        close[finite] = np.abs(a[finite] - e[finite]) <= atol + rtol * np.abs(e[finite])
        both_inf = np.isinf(a) & np.isinf(e) & (np.sign(a) == np.sign(e))
        overflow = np.zeros(a.shape, dtype=bool)
        if ref_fp32 is not None:
            r = np.asarray(ref_fp32, dtype=np.float32)
            big = np.abs(r) > 65504.0
            sat = (np.isinf(a) | (np.abs(a) == 65504.0)) & (np.sign(a) == np.sign(r))
            overflow = big & sat
    ok = close | both_inf | overflow
    return {
        "ok": bool(ok.all()),
        "mismatches": int((~ok).sum()),
        "overflow_elems": int((both_inf | overflow).sum()),
        "max_abs_err": float(np.max(np.abs(a[finite] - e[finite]))) if finite.any() else 0.0,
        "count": int(a.size),
    }
