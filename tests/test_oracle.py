"""The oracle pinned against the reference: the C restatement (oracle/q4_oracle.c) must
reproduce the golden vectors the reference's own CPU C produced (tests/golden/make_golden.py),
bit for bit where the reference's arithmetic order is restated, and agree with the live
reference library when it is built here."""
import numpy as np
import pytest


def _peak_tol(want, got, tol):
    peak = max(1.0, float(np.abs(want).max()))
    return float(np.abs(want.astype(np.float64) - got).max()) <= tol * peak


def test_fp4km_cases_bit_exact(oracle_mod, golden):
    O, g = oracle_mod, golden["ref_tile_cases"]
    fp4, _ = O.reference_test_cases()
    for i, (M, K, N, x, packed, table) in enumerate(fp4):
        # the generator reproduces the reference test's inputs
        assert np.array_equal(x, g[f"fp4_{i}_x"]) and np.array_equal(packed, g[f"fp4_{i}_packed"])
        port = O.tile_gemm_fp4km(x, packed, table, M, K, N)
        assert np.array_equal(port, g[f"fp4_{i}_dyn"]), f"case {i}"
        assert np.array_equal(port, g[f"fp4_{i}_fixed"]), f"case {i}"
        if f"fp4_{i}_legacy" in g:
            assert np.array_equal(port, g[f"fp4_{i}_legacy"]), f"case {i} legacy"
        # tileGemmReference order differs; the reference test's own tolerance (1e-4 peak)
        assert _peak_tol(g[f"fp4_{i}_dyn"], O.tile_gemm_reference(x, packed, table, M, K, N), 1e-4)


def test_f16_cases_bit_exact(oracle_mod, golden):
    O, g = oracle_mod, golden["ref_tile_cases"]
    _, f16 = O.reference_test_cases()
    for i, (M, K, N, x, w, halves) in enumerate(f16):
        assert np.array_equal(halves, g[f"f16_{i}_halves"])
        port = O.tile_gemm_f16(x, halves, M, K, N)
        assert np.array_equal(port, g[f"f16_{i}_dyn"]), f"case {i}"
        assert _peak_tol(g[f"f16_{i}_f64"], port, 1e-4)


def test_gate_cases_exact(oracle_mod, golden):
    O, g = oracle_mod, golden["ref_gate"]
    x, packed, table = O.gate_fp4()
    port = O.tile_gemm_fp4km(x, packed, table, 37, 128, 80)
    assert np.array_equal(port, g["fp4_vm"])
    # exact data: every path agrees exactly
    assert np.array_equal(O.tile_gemm_reference(x, packed, table, 37, 128, 80), g["fp4_vm"])
    xh, w, halves = O.gate_f16()
    assert np.array_equal(O.tile_gemm_f16(xh, halves, 37, 128, 80), g["f16_vm"])
    assert np.array_equal(g["f16_vm"], g["f16_f64"])


def test_q4b32_three_routes_agree(oracle_mod, golden):
    """Format 2 pinned two ways: through the reference VM's FP4-KM op with a scale palette
    (bit-exact) and through nimf_cpu_matmul_q4 on the asymmetric repack."""
    O, g = oracle_mod, golden["ref_q4b32"]
    i = 0
    while f"q4_{i}_shape" in g:
        M, K, N = (int(v) for v in g[f"q4_{i}_shape"])
        p, s, xb = g[f"q4_{i}_packed"], g[f"q4_{i}_scales"], g[f"q4_{i}_x_bf16"]
        x = O.bf16_to_f32(xb)
        port = O.tile_gemm_q4b32(x, p, s, M, K, N)
        assert np.array_equal(port, g[f"q4_{i}_vm"]), f"case {i}"
        wq, sc, zp = O.q4b32_to_asym(p, s, N, K)
        asym = O.matmul_q4_asym(x, wq, sc, zp, M, K, N)
        assert np.array_equal(asym, g[f"q4_{i}_matmul_q4"]), f"case {i} matmul_q4"
        assert _peak_tol(g[f"q4_{i}_vm"], g[f"q4_{i}_q4gemv"], 1e-4)
        i += 1
    assert i == 8


def test_q4b32_dequant_formats_identical(oracle_mod):
    O = oracle_mod
    N, K = 48, 256
    p, s = O.gen_q4b32(N, K)
    pal = s.ravel()[:256].copy()
    s = pal[(np.arange(N * K // 32) * 7919) % 256].reshape(N, K // 32)
    blob, table = O.q4b32_to_fp4km(p, s, N, K)
    w1 = O.dequant_q4b32(p, s, N, K)
    assert np.array_equal(w1, O.dequant_fp4km(blob, table, N, K))
    # (float)q * (float)scale, q from the two's-complement nibble
    from bybylang_b200.formats import unpack_q4b32
    q = unpack_q4b32(p).astype(np.float32)
    assert np.array_equal(w1, q * O.f16_to_f32(np.repeat(s, 32, axis=1)))


def test_generators_distributions(oracle_mod):
    O = oracle_mod
    p, s = O.gen_q4b32(64, 4096)
    from bybylang_b200.formats import unpack_q4b32
    q = unpack_q4b32(p)
    assert q.min() == -8 and q.max() == 7
    counts = np.bincount((q.astype(np.int16) + 8).ravel(), minlength=16)
    assert counts.min() > 0.9 * counts.mean()
    sf = O.f16_to_f32(s)
    assert (sf > 0).all() and abs(np.mean(sf) - 0.02 * np.sqrt(2 / np.pi)) < 1e-3
    x = O.bf16_to_f32(O.gen_x_bf16(4, 4096))
    assert abs(x.mean()) < 0.05 and abs(x.std() - 1.0) < 0.05


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).ref_available()")
def test_live_reference_matches_port(oracle_mod):
    O = oracle_mod
    rng = np.random.default_rng(7)
    for (M, K, N) in [(3, 96, 40), (9, 320, 77), (1, 4096, 33)]:
        x = rng.standard_normal((M, K)).astype(np.float32)
        packed = rng.integers(0, 256, N * (K // 2) + N * (K // 32), dtype=np.uint8)
        table = np.concatenate([rng.standard_normal(16), np.abs(rng.standard_normal(256))]).astype(np.float32)
        ref = O.ref_tile_gemm(x, packed, table, M, K, N)
        assert np.array_equal(ref, O.tile_gemm_fp4km(x, packed, table, M, K, N))
        assert np.array_equal(ref, O.ref_tile_gemm(x, packed, table, M, K, N, threads=3))
