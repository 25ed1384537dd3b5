"""GPU parity of the tensor-core (tcgen05) prefill route against the reference's CPU arithmetic.

Route TC keeps every dequantised weight exact: w = q * s enters the MMAs as the two fp16 terms
q * s_hi + q * s_lo (s_hi: the fp16 scale with its 3 lowest mantissa bits cleared; both
products are exact), and bf16 activations are exact in fp16, so the only rounding is the fp32
accumulation.  Its outputs are held to the reference gate's per-element metric,
|got - want| / max(1, |want|) <= 1e-3 (backends/vulkan/vulkan_driver.nim:2752-2754), and to the
reference test's max|diff| <= tol * max(1, max|ref|) (tests/t_fp4_tile_gemm.nim:54-67).

fp32 activations enter this route as two fp16 rows each, x_hi = RNE16(x) and the remainder
x_lo = RNE16(x - x_hi) (about 22 of fp32's 24 significant bits), whose two products the
epilogue adds: per-element 1e-3 as well (test_tc_fp32_activations_per_element).  Route
TC_FP16W rounds each weight once to fp16, as the reference's cooperative lowering does
(micro_kernel/tile_gemm.nim:322-325, 414): the reference test's peak-normalised 1e-3.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from bybylang_b200 import _lib  # noqa: E402
from bybylang_b200 import gpubackend as gb  # noqa: E402

from gpu_helpers import assert_close, dev, elem_err, peak_err, q4_slot, run  # noqa: E402

TC_TOL = 1e-3
ELEM_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _init():
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    yield
    assert _lib.device_error() == 0


def _case(O, M, K, N, seed=0):
    p, s = O.gen_q4b32(N, K, seed=O.Xorshift32.SEED + seed)
    xb = O.gen_x_bf16(M, K, seed=O.Xorshift32.SEED + 2 + seed)
    slot, sb = q4_slot(p, s)
    return p, s, xb, slot, sb


def test_tc_golden_cases(golden, oracle_mod):
    """The reference VM's outputs (tests/golden/ref_q4b32.npz) for every case the route tiles."""
    g = golden["ref_q4b32"]
    ran = 0
    for i in range(8):
        M, K, N = (int(v) for v in g[f"q4_{i}_shape"])
        if K % 256:
            continue
        slot, sb = q4_slot(g[f"q4_{i}_packed"], g[f"q4_{i}_scales"])
        xb = dev(g[f"q4_{i}_x_bf16"]).view(torch.bfloat16)
        out = run(2, M, K, N, xb, slot, scale_base=sb, route=_lib.ROUTE_TC)
        assert_close(g[f"q4_{i}_vm"], out.cpu().numpy(), TC_TOL, ELEM_TOL, what=f"case {i} bf16")
        xf = dev(oracle_mod.bf16_to_f32(g[f"q4_{i}_x_bf16"]))
        out = run(2, M, K, N, xf, slot, scale_base=sb, route=_lib.ROUTE_TC)
        assert_close(g[f"q4_{i}_vm"], out.cpu().numpy(), TC_TOL, ELEM_TOL, what=f"case {i} f32")
        ran += 1
    assert ran == 3


@pytest.mark.parametrize("M,K,N", [(1, 256, 1), (17, 256, 130), (256, 512, 128), (300, 768, 200),
                                   (513, 1024, 384), (1000, 2048, 77)])
def test_tc_ragged_shapes_against_oracle(M, K, N, oracle_mod):
    """Partial token tiles and partial weight-row tiles.  With fewer tiles than half the CTA
    pairs the GEMM cuts its last wave's tiles into 2 to 8 K-parts of at least two weight
    stages, whose partial sums the last part adds: the cases with K >= 1024 take that path
    (2 and 4 parts; uneven parts at K = 11008 in test_gpu_configs.py)."""
    O = oracle_mod
    p, s, xb, slot, sb = _case(O, M, K, N, seed=M + N)
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N, threads=8)
    out = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb, route=_lib.ROUTE_TC)
    assert_close(want, out.cpu().numpy(), TC_TOL, ELEM_TOL, what=f"M={M} K={K} N={N}")


def test_tc_prefill_c3_full_size(parity_log):
    """Config C3 (M=2048, K=N=4096), every output: against the SIMT route, which is
    bit-identical to the reference CPU VM (checked in test_gpu_parity.py)."""
    from bybylang_b200.formats import synthetic_q4b32, synthetic_x
    M, K, N = 2048, 4096, 4096
    nib, sc = synthetic_q4b32(N, K, seed=11, device="cuda:0")
    w = gb.Q4B32Weights(nib, sc, device="cuda:0")
    x = synthetic_x(M, K, seed=12, device="cuda:0")
    tc = w.matmul(x, route=_lib.ROUTE_TC)
    fast = w.matmul(x, route=_lib.ROUTE_TC_FP16W)
    ref = w.matmul(x, route=_lib.ROUTE_SIMT)
    torch.cuda.synchronize()
    ref, tc, fast = ref.cpu().numpy(), tc.cpu().numpy(), fast.cpu().numpy()
    err = peak_err(ref, tc)
    worst = elem_err(ref, tc)
    parity_log.append(("C3 2048x4096x4096 route TC (exact weights), every output", worst, ELEM_TOL))
    assert err <= 5e-5, f"peak-normalised error {err:.3e}"   # only the fp32 accumulation differs
    assert worst <= ELEM_TOL, f"worst per-element error {worst:.3e}"
    # the fp16-rounded weights: inside the peak-normalised tolerance, not the per-element one
    err16, worst16 = peak_err(ref, fast), elem_err(ref, fast)
    parity_log.append(("C3 2048x4096x4096 route TC_FP16W (weights rounded to fp16), every output", worst16, 0))
    assert err16 <= TC_TOL and err16 > err, f"fp16-weight route: {err16:.3e}"


def test_tc_prefill_rows_against_oracle(oracle_mod):
    """C3 shape, sampled token rows through the CPU oracle directly."""
    O = oracle_mod
    M, K, N = 2048, 4096, 4096
    p, s, xb, slot, sb = _case(O, M, K, N, seed=5)
    out = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb, route=_lib.ROUTE_TC).cpu().numpy()
    rows = np.r_[0:8, 255:259, 1023:1027, 2040:2048]
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb[rows]), p, s, len(rows), K, N, threads=8)
    assert_close(want, out[rows], TC_TOL, ELEM_TOL, what="C3 sampled rows")


@pytest.mark.parametrize("M,K,N", [(32, 4096, 4096), (300, 1024, 384), (1000, 2048, 77)])
def test_tc_fp32_activations_per_element(M, K, N, oracle_mod, parity_log):
    """fp32 activations with their full mantissa (not bf16 values) on route TC, against the
    oracle's fp32 arithmetic, per element; the first shape is config C1."""
    O = oracle_mod
    p, s = O.gen_q4b32(N, K, seed=O.Xorshift32.SEED + M)
    xf = O.gen_x_f32(M, K, seed=O.Xorshift32.SEED + 7 + M)
    slot, sb = q4_slot(p, s)
    want = O.tile_gemm_q4b32(xf, p, s, M, K, N, threads=8)
    got = run(2, M, K, N, dev(xf), slot, scale_base=sb, route=_lib.ROUTE_TC).cpu().numpy()
    parity_log.append((f"{M}x{K}x{N} fp32 x, route TC (two fp16 terms per activation)", elem_err(want, got), ELEM_TOL))
    assert_close(want, got, TC_TOL, ELEM_TOL, what=f"fp32 x M={M} K={K} N={N}")
    b16 = run(2, M, K, N, dev(xf), slot, scale_base=sb, route=_lib.ROUTE_TC, out_dtype=torch.bfloat16)
    assert torch.equal(torch.from_numpy(got).to(torch.bfloat16), b16.cpu())


@pytest.mark.parametrize("M,N", [(8, 300), (13, 96), (16, 520)])
def test_auto_fp32_rows_long_k_per_element(M, N, oracle_mod, parity_log):
    """8 to 16 fp32 rows with K >= 8192: AUTO takes the tensor cores, whose split rows (16 to
    32 fp16 rows) run the 16- and 32-token tiles; per element against the oracle."""
    O = oracle_mod
    K = 8192
    p, s = O.gen_q4b32(N, K, seed=O.Xorshift32.SEED + 3 * M)
    xf = O.gen_x_f32(M, K, seed=O.Xorshift32.SEED + 11 + M)
    slot, sb = q4_slot(p, s)
    assert gb.route_for(2, M, K, N, _lib.DT_F32) == _lib.ROUTE_TC
    want = O.tile_gemm_q4b32(xf, p, s, M, K, N, threads=8)
    got = run(2, M, K, N, dev(xf), slot, scale_base=sb).cpu().numpy()
    parity_log.append((f"{M}x{K}x{N} fp32 x, AUTO (TC, two fp16 terms per activation)", elem_err(want, got), ELEM_TOL))
    assert_close(want, got, TC_TOL, ELEM_TOL, what=f"fp32 x M={M} K={K} N={N}")
    assert _lib.device_error() == 0


def test_tc_bf16_output_is_rounded_f32_output(oracle_mod):
    O = oracle_mod
    M, K, N = 300, 1024, 256
    p, s, xb, slot, sb = _case(O, M, K, N, seed=3)
    x = dev(xb).view(torch.bfloat16)
    f32 = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_TC)
    b16 = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_TC, out_dtype=torch.bfloat16)
    assert torch.equal(f32.to(torch.bfloat16), b16)


def test_tc_deterministic_across_calls(oracle_mod):
    O = oracle_mod
    M, K, N = 512, 2048, 640
    p, s, xb, slot, sb = _case(O, M, K, N, seed=4)
    x = dev(xb).view(torch.bfloat16)
    a = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_TC)
    b = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_TC)
    assert torch.equal(a, b)


def test_auto_route_prefill_is_tc(oracle_mod):
    assert gb.route_for(2, 2048, 4096, 4096) == _lib.ROUTE_TC
    assert gb.route_for(2, 64, 4096, 128256) == _lib.ROUTE_TC
    assert gb.route_for(2, 16, 4096, 4096) == _lib.ROUTE_GEMV
    assert gb.route_for(2, 7, 11008, 4096) == _lib.ROUTE_GEMV                 # few rows
    assert gb.route_for(2, 8, 11008, 4096) == _lib.ROUTE_TC                   # long rows
    assert gb.route_for(2, 11, 4096, 128256) == _lib.ROUTE_GEMV
    assert gb.route_for(2, 12, 4096, 128256) == _lib.ROUTE_TC                 # very wide output
    assert gb.route_for(2, 7, 11008, 4096, _lib.DT_F32) == _lib.ROUTE_GEMV
    assert gb.route_for(2, 8, 11008, 4096, _lib.DT_F32) == _lib.ROUTE_TC     # long fp32 rows too
    assert gb.route_for(2, 12, 4096, 128256, _lib.DT_F32) == _lib.ROUTE_TC
    assert gb.route_for(2, 32, 4096, 4096) == _lib.ROUTE_TC                  # bf16 rows
    assert gb.route_for(2, 32, 4096, 4096, _lib.DT_F32) == _lib.ROUTE_TC     # two fp16 terms per fp32 value
    assert gb.route_for(2, 33, 4096, 4096, _lib.DT_F32) == _lib.ROUTE_TC
    assert gb.route_for(2, 64, 4128, 4096) != _lib.ROUTE_TC    # K % 256 != 0
    O = oracle_mod
    M, K, N = 40, 512, 96
    p, s, xb, slot, sb = _case(O, M, K, N, seed=6)
    out = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb)
    assert_close(O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N), out.cpu().numpy(), TC_TOL)


def test_tc_fp16_weight_route(oracle_mod, parity_log):
    """Route TC_FP16W: one rounding per weight, the reference's cooperative lowering; the
    peak-normalised tolerance holds, and on exact data (scales with <= 8 significant bits) it
    equals route TC bit for bit."""
    O = oracle_mod
    M, K, N = 300, 1024, 384
    p, s, xb, slot, sb = _case(O, M, K, N, seed=9)
    x = dev(xb).view(torch.bfloat16)
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N, threads=8)
    fast = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_TC_FP16W).cpu().numpy()
    assert_close(want, fast, TC_TOL, what="TC_FP16W")
    parity_log.append((f"{M}x{K}x{N} route TC_FP16W", elem_err(want, fast), 0))
    # q * s exact in fp16 (8 significant bits), and s / 16 still a normal fp16 number (s >= 2^-9),
    # which the one-rounding form's high-nibble product goes through
    s8 = (np.maximum(np.asarray(s, np.uint16), 0x1800) & 0xFFF8).astype(np.uint16)
    slot8, sb8 = q4_slot(p, s8)
    a = run(2, M, K, N, x, slot8, scale_base=sb8, route=_lib.ROUTE_TC_FP16W)
    b = run(2, M, K, N, x, slot8, scale_base=sb8, route=_lib.ROUTE_TC)
    assert torch.allclose(a, b, rtol=0, atol=1e-6 * float(b.abs().max()))


def test_tc_rejects_untileable_shapes(oracle_mod):
    O = oracle_mod
    M, K, N = 32, 288, 64
    p, s, xb, slot, sb = _case(O, M, K, N)
    with pytest.raises(_lib.BybyCudaError, match="tensor-core route"):
        run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb, route=_lib.ROUTE_TC)


def test_tc_activation_outside_fp16_range_is_reported(oracle_mod):
    """|x| >= 65520 cannot be staged as fp16: the pre-pass records device error 7 (no fault)."""
    O = oracle_mod
    M, K, N = 20, 256, 128
    p, s, xb, slot, sb = _case(O, M, K, N)
    x = dev(xb).view(torch.bfloat16).clone()
    x[3, 17] = 1.0e6
    run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_TC)
    assert _lib.device_error() == 7
    assert _lib.device_error() == 0   # read-and-clear


# ----------------------------------------------------------------------------------------
# Format 1 (fp16 weights) on the tensor cores: both operands straight from shared memory
# ----------------------------------------------------------------------------------------

@pytest.mark.parametrize("M,K,N,xdt", [(64, 1024, 512, "f32"), (200, 2048, 300, "bf16"), (9, 128, 40, "f32"),
                                       (512, 1024, 1024, "bf16"), (129, 4096, 257, "f32")])
def test_f16_tensor_core_against_oracle(M, K, N, xdt):
    from oracle import oracle as O
    rng = np.random.default_rng(M + K + N)
    halves = rng.normal(0, 0.05, size=(N, K)).astype(np.float16)
    packed = dev(halves.view(np.uint8).reshape(-1).copy())
    if xdt == "bf16":
        xb = O.gen_x_bf16(M, K, seed=M)
        x, xf = dev(xb).view(torch.bfloat16), O.bf16_to_f32(xb)
    else:
        xf = O.gen_x_f32(M, K, seed=M)
        x = dev(xf)
    want = O.tile_gemm_f16(xf, halves.view(np.uint16), M, K, N)
    out = run(1, M, K, N, x, packed, route=_lib.ROUTE_TC)
    assert_close(want, out.cpu().numpy(), TC_TOL, what=f"M={M} K={K} N={N} {xdt}")
    if M > 8:   # AUTO takes the same route above the decode route's 8 rows
        assert torch.equal(out, run(1, M, K, N, x, packed))
    assert _lib.device_error() == 0


def test_f16_tensor_core_bf16_out_and_range():
    from oracle import oracle as O
    M, K, N = 32, 256, 64
    halves = np.random.default_rng(1).normal(0, 0.05, size=(N, K)).astype(np.float16)
    packed = dev(halves.view(np.uint8).reshape(-1).copy())
    xf = O.gen_x_f32(M, K)
    want = O.tile_gemm_f16(xf, halves.view(np.uint16), M, K, N)
    out = run(1, M, K, N, dev(xf), packed, route=_lib.ROUTE_TC, out_dtype=torch.bfloat16)
    assert_close(want, out.float().cpu().numpy(), 1e-2, what="bf16 out")
    big = xf.copy()
    big[3, 7] = 1e6   # no fp16 image: device error 7, no fault
    run(1, M, K, N, dev(big), packed, route=_lib.ROUTE_TC)
    assert _lib.device_error() == 7
    assert _lib.device_error() == 0
