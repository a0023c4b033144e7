"""Pin the CPU oracle to the reference (CPU, no GPU needed).

* Scale layouts: the oracle's to_blocked / reorder restatements must equal, bit
  for bit, the outputs of the reference harness's own functions stored in
  tests/golden/golden_inputs.npz.
* GEMM arithmetic: the oracle must match torch._scaled_mm (the reference's
  ref_kernel arithmetic, run on a B200) stored in golden_outputs.npz.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_case_names
from oracle import nvfp4_oracle as O


def test_to_blocked_matches_reference_function(golden_inputs):
    n = 0
    for key in golden_inputs.files:
        if "/sf_" in key:
            plain = golden_inputs[key]
            expect = golden_inputs[key.replace("/sf_", "/blocked_")]
            assert np.array_equal(O.to_blocked(plain), expect), key
            n += 1
    assert n >= 10


def test_reordered_storage_equals_to_blocked_on_mapped_bytes(golden_inputs):
    """The harness's reordered tensor stores exactly the to_blocked bytes (padding aside)."""
    for key in golden_inputs.files:
        if "/reordered_" not in key:
            continue
        plain = golden_inputs[key.replace("/reordered_", "/sf_")]
        rows, cols = plain.shape
        k = cols * 16
        reordered = golden_inputs[key].reshape(-1)
        mine = O.reordered_storage(O.reorder_scales(plain, k))
        assert reordered.shape == mine.shape
        # Positions that some (row, col) maps to must agree; the rest is harness padding.
        mask = O.to_blocked(np.ones_like(plain)) == 1
        assert np.array_equal(reordered[mask], mine[mask]), key
        assert np.array_equal(mine, O.to_blocked(plain)), key
        # Round trip through the inverse.
        assert np.array_equal(O.from_blocked(mine, rows, cols), plain)


def test_e2m1_and_e4m3_tables():
    assert O.E2M1_VALUES[0b0111] == 6.0 and O.E2M1_VALUES[0b1001] == -0.5
    masked = sorted({float(O.E2M1_VALUES[c]) for c in range(16) if c & 0b0100 == 0})
    assert masked == [-1.5, -1.0, -0.5, 0.0, 1.5, 1.0, 0.5][::1] or len(masked) == 7
    assert O.E4M3_VALUES[0x38] == 1.0 and O.E4M3_VALUES[0x40] == 2.0
    for e in range(-4, 4):
        assert O.E4M3_VALUES[(e + 7) << 3] == 2.0 ** e
    assert np.isnan(O.E4M3_VALUES[0x7F]) and O.E4M3_VALUES[0x01] == 2.0 ** -9


def test_unpack_low_nibble_first():
    packed = np.array([[0x21, 0x7F]], dtype=np.uint8)
    assert O.unpack_e2m1(packed).tolist() == [[0.5, 1.0, -6.0, 6.0]]


def test_oracle_dense_equivalence_small():
    """Dequantise-then-matmul equals an explicit triple loop on a tiny case."""
    rng = np.random.default_rng(0)
    m, n, k = 3, 5, 32
    a = rng.integers(0, 256, (m, k // 2), dtype=np.uint8)
    b = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sfa = (((rng.integers(-4, 4, (m, k // 16))) + 7) << 3).astype(np.uint8)
    sfb = (((rng.integers(-4, 4, (n, k // 16))) + 7) << 3).astype(np.uint8)
    got = O.ref_gemm_fp32(a, b, sfa, sfb)
    av, bv = O.unpack_e2m1(a), O.unpack_e2m1(b)
    for i in range(m):
        for j in range(n):
            s = 0.0
            for kk in range(k):
                s += (av[i, kk] * O.E4M3_VALUES[sfa[i, kk // 16]]) * (bv[j, kk] * O.E4M3_VALUES[sfb[j, kk // 16]])
            assert got[i, j] == pytest.approx(s, rel=1e-6, abs=1e-6)


def test_oracle_matches_reference_arithmetic(golden_inputs, golden_outputs):
    """Oracle vs torch._scaled_mm (cuBLASLt) outputs recorded on a B200."""
    checked = 0
    for name in golden_case_names(golden_inputs):
        G, gated = (int(x) for x in golden_inputs[f"{name}/meta"])
        alpha = golden_inputs[f"{name}/alpha"]
        tol = dict(rtol=1e-3, atol=1e-3) if name.startswith("ref_") else dict(rtol=1e-2, atol=1e-2)
        for g in range(G):
            key = f"{name}/{g}/c"
            if key not in golden_outputs.files:
                continue
            a = golden_inputs[f"{name}/{g}/a"]
            b = golden_inputs[f"{name}/{g}/b"]
            sfa = golden_inputs[f"{name}/{g}/sf_a"]
            sfb = golden_inputs[f"{name}/{g}/sf_b"]
            if gated:
                exp = O.ref_gated(a, b, golden_inputs[f"{name}/{g}/b2"], sfa, sfb,
                                  golden_inputs[f"{name}/{g}/sf_b2"])
                ref32 = None
            else:
                ref32 = O.ref_gemm_fp32(a, b, sfa, sfb) * np.float32(alpha[g])
                exp = ref32.astype(np.float16)
                if f"{name}/{g}/fp32_b" in golden_outputs.files:
                    np.testing.assert_allclose(golden_outputs[f"{name}/{g}/fp32_b"],
                                               O.ref_gemm_fp32(a, b, sfa, sfb), rtol=1e-5, atol=1e-3)
            res = O.compare_fp16(golden_outputs[key], exp, ref32, **tol)
            assert res["ok"], f"{key}: {res}"
            checked += 1
    assert checked > 0


def test_generate_input_distribution():
    d = O.generate_input((80, 200), (256, 256), (512, 512), 2, seed=1)
    assert d["problem_sizes"] == [(80, 256, 512, 1), (200, 256, 512, 1)]
    codes = np.concatenate([d["a"][0].reshape(-1) & 0xF, d["a"][0].reshape(-1) >> 4])
    assert set(np.unique(codes)) <= {0, 1, 2, 3, 8, 9, 10, 11}
    assert set(np.unique(d["sfa"][1])) <= {0x38, 0x40}


def test_compare_fp16_overflow_semantics():
    ref32 = np.array([70000.0, -70000.0, 1.0], dtype=np.float32)
    exp = ref32.astype(np.float16)
    got = np.array([np.inf, -65504.0, 1.0005], dtype=np.float16)
    res = O.compare_fp16(got, exp, ref32, rtol=1e-2, atol=1e-2)
    assert res["ok"] and res["overflow_elems"] == 2
    bad = np.array([np.inf, np.inf, 1.0], dtype=np.float16)
    assert not O.compare_fp16(bad, exp, ref32)["ok"]
