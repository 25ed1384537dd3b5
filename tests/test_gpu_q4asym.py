"""Asymmetric Q4 (matmul_q4) on the GPU against the reference's own CPU kernel.

The reference: nimf_cpu_matmul_q4 (backends/cpu/cpu_kernels_impl.inc:293-319), built unchanged
into oracle/_ref, and its restatement in the oracle port.  Data: interleaved nibbles
[N, (K+1)/2] (even k in the low nibble), fp32 scales and zero points [N, groups].

Tolerances (written here):
* decode kernel (route AUTO at M = 1, group 32): the reference test's max|diff| <= 1e-4 *
  max(1, max|ref|), the north star's 1e-3 per element (|diff| / max(1, |ref|)), and per
  element its fixed-point bound against float64,
  |diff| <= 2^-29 * sum_b max|x_b| * sum_{k in b} |w[n, k]| plus fp32 slack, on inputs of any
  dynamic range (fp32 activations travel as two fixed-point images per 32-block).
* exact kernel (route SIMT, and AUTO for every other shape): the same bounds against the
  reference (its k-order fmaf differs from nimf_cpu_matmul_q4's evaluation order only by
  fp32 rounding).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from bybylang_b200 import _lib  # noqa: E402
from bybylang_b200 import gpubackend as gb  # noqa: E402

from gpu_helpers import DEV, assert_close, elem_err  # noqa: E402

PEAK_TOL, ELEM_TOL = 1e-4, 1e-3


@pytest.fixture(scope="module", autouse=True)
def _init():
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    yield
    assert _lib.device_error() == 0


def gen_q4(M, K, N, group=32, seed=0, integer_zeros=False):
    rng = np.random.default_rng(seed)
    groups = (K + group - 1) // group
    wq = rng.integers(0, 256, size=(N, (K + 1) // 2), dtype=np.uint8)
    scales = np.abs(rng.normal(0, 0.02, size=(N, groups))).astype(np.float32) + np.float32(1e-4)
    zeros = (np.full((N, groups), 8.0, np.float32) if integer_zeros
             else rng.uniform(0, 15, size=(N, groups)).astype(np.float32))
    a = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    return a, wq, scales, zeros


def run_q4(a, wq, scales, zeros, M, K, N, group, route=_lib.ROUTE_AUTO, n_groups=None):
    n_groups = n_groups if n_groups is not None else scales.shape[1]
    t = [torch.from_numpy(np.ascontiguousarray(v)).to(DEV) for v in (a, wq, scales, zeros)]
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device=DEV)
    _lib.check(_lib.load().bybycu_matmul_q4(*[C.c_void_p(v.data_ptr()) for v in t], C.c_void_p(out.data_ptr()),
                                            M, K, N, group, n_groups, route, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def dequant_np(wq, scales, zeros, K, group):
    """(u - z) * s per element, in float64."""
    N = wq.shape[0]
    u = np.empty((N, (K + 1) // 2 * 2), np.float64)
    u[:, 0::2] = wq & 15
    u[:, 1::2] = wq >> 4
    u = u[:, :K]
    g = np.arange(K) // group
    return (u - zeros[:, g].astype(np.float64)) * scales[:, g].astype(np.float64)


def assert_fixed_point_bound(x, wq, scales, zeros, K, got):
    """Per element against float64: |diff| <= 2^-29 sum_b max|x_b| sum_{k in b} |w| + slack."""
    N = wq.shape[0]
    w = dequant_np(wq, scales, zeros, K, 32)
    xd = x.astype(np.float64)
    want = w @ xd
    blk_max = np.abs(xd).reshape(-1, 32).max(axis=1)
    quant = 2.0 ** -29 * (np.abs(w).reshape(N, -1, 32).sum(axis=2) * blk_max).sum(axis=1)
    slack = 1e-5 * (np.abs(w) * np.abs(xd)).sum(axis=1) + 1e-30
    err = np.abs(np.asarray(got, np.float64) - want)
    assert np.isfinite(got).all()
    assert (err <= quant + slack).all(), f"worst excess {(err - quant - slack).max():.3e}"


@pytest.mark.parametrize("K,N", [(4096, 11008), (4096, 4096), (11008, 4096), (128, 1), (1152, 17), (2048, 300)])
def test_decode_kernel_against_reference(K, N, oracle_mod, parity_log):
    O = oracle_mod
    a, wq, scales, zeros = gen_q4(1, K, N, seed=K + N)
    want = O.ref_matmul_q4(a, wq, scales, zeros, 1, K, N, 32, threads=8)
    got = run_q4(a, wq, scales, zeros, 1, K, N, 32, route=_lib.ROUTE_GEMV)
    assert_close(want, got, PEAK_TOL, ELEM_TOL, f"K={K} N={N}")
    if N >= 1024:
        parity_log.append((f"asym Q4 1x{K}x{N} fp32 x, decode kernel (two images)", elem_err(want, got), ELEM_TOL))
    assert_close(O.matmul_q4_asym(a, wq, scales, zeros, 1, K, N, 32), got, PEAK_TOL, ELEM_TOL, "port")
    assert_fixed_point_bound(a[0], wq, scales, zeros, K, got[0])


def test_decode_kernel_integer_zero_points(oracle_mod):
    O = oracle_mod
    K, N = 4096, 2048
    a, wq, scales, zeros = gen_q4(1, K, N, seed=3, integer_zeros=True)
    got = run_q4(a, wq, scales, zeros, 1, K, N, 32)
    assert_close(O.ref_matmul_q4(a, wq, scales, zeros, 1, K, N, 32, threads=8), got, PEAK_TOL, ELEM_TOL)
    assert_fixed_point_bound(a[0], wq, scales, zeros, K, got[0])


def test_decode_kernel_dynamic_range():
    """fp32 activations over 48 binades, zeros, a lone outlier, tiny blocks: inside the
    fixed-point bound against float64."""
    K, N = 4096, 1024
    a, wq, scales, zeros = gen_q4(1, K, N, seed=11)
    rng = np.random.default_rng(12)
    x = (rng.choice([-1.0, 1.0], K) * np.exp2(rng.uniform(-30, 18, K))).astype(np.float32)
    x[rng.random(K) < 0.1] = 0.0
    x[64:96] = 0.0
    x[160:192] = 1e-7
    x[170] = 5e4
    x[224:256] = 1e-35
    a[0] = x
    assert_fixed_point_bound(x, wq, scales, zeros, K, run_q4(a, wq, scales, zeros, 1, K, N, 32)[0])
    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,K,N,group,route", [(3, 512, 300, 32, _lib.ROUTE_SIMT), (1, 512, 100, 64, _lib.ROUTE_AUTO),
                                                (16, 256, 40, 32, _lib.ROUTE_SIMT), (1, 96, 7, 32, _lib.ROUTE_AUTO),
                                                (5, 384, 50, 32, _lib.ROUTE_AUTO), (4, 512, 64, 64, _lib.ROUTE_AUTO)])
def test_exact_kernel_shapes(M, K, N, group, route, oracle_mod):
    """The exact kernel: route SIMT, and AUTO for the shapes neither fast route takes (group
    64, K % 128 != 0 at M = 1, K % 256 != 0 above)."""
    O = oracle_mod
    a, wq, scales, zeros = gen_q4(M, K, N, group=group, seed=M * K + N)
    got = run_q4(a, wq, scales, zeros, M, K, N, group, route=route)
    assert_close(O.ref_matmul_q4(a, wq, scales, zeros, M, K, N, group), got, PEAK_TOL, ELEM_TOL)


TC_TOL = 1e-3   # the tensor-core route: weights and activations rounded once to fp16


@pytest.mark.parametrize("M,K,N", [(64, 4096, 2048), (200, 1024, 300), (2, 256, 40), (129, 2048, 513)])
def test_tensor_core_prefill_against_reference(M, K, N, oracle_mod, parity_log):
    """M > 1, group 32, K % 256 == 0: AUTO takes the tcgen05 GEMM (the same kernel as the
    Q4B32 prefill, dequantising w = RNE16(u s - z s)); checked with the reference test's metric
    at the tensor-core tolerance (the reference's own gate for its matrix-unit Q4 plans is
    3e-3 of the peak, backends/vulkan/q4_autotune.nim:506), and explicit route TC gives the
    same bits.  The per-element error is logged, not bounded: fp16 rounding of s, z s and x."""
    O = oracle_mod
    a, wq, scales, zeros = gen_q4(M, K, N, seed=M + K + N)
    want = O.ref_matmul_q4(a, wq, scales, zeros, M, K, N, 32, threads=8)
    got = run_q4(a, wq, scales, zeros, M, K, N, 32)
    assert_close(want, got, TC_TOL, None, f"M={M} K={K} N={N}")
    parity_log.append((f"asym Q4 {M}x{K}x{N} fp32 x, route TC (one fp16 rounding)", elem_err(want, got), 0.0))
    assert np.array_equal(got, run_q4(a, wq, scales, zeros, M, K, N, 32, route=_lib.ROUTE_TC))
    assert _lib.device_error() == 0


def test_tensor_core_route_rules():
    K, N = 512, 64
    a, wq, scales, zeros = gen_q4(4, K, N, seed=3)
    with pytest.raises(_lib.BybyCudaError):   # M = 1 is the decode kernel's
        run_q4(a[:1], wq, scales, zeros, 1, K, N, 32, route=_lib.ROUTE_TC)
    a2, wq2, s2, z2 = gen_q4(4, 384, N, seed=4)
    with pytest.raises(_lib.BybyCudaError):   # K % 256 != 0
        run_q4(a2, wq2, s2, z2, 4, 384, N, 32, route=_lib.ROUTE_TC)
    big = a.copy()
    big[2, 5] = 1e6                           # no fp16 image: device error 7, no fault
    run_q4(big, wq, scales, zeros, 4, K, N, 32, route=_lib.ROUTE_TC)
    assert _lib.device_error() == 7
    assert _lib.device_error() == 0


def test_exact_kernel_odd_k_and_one_group():
    """K odd (the last byte's high nibble unused) and group_size <= 0 (one group per row)."""
    M, K, N = 2, 33, 9
    a, wq, scales, zeros = gen_q4(M, K, N, group=32, seed=5)
    want = a.astype(np.float64) @ dequant_np(wq, scales, zeros, K, 32).T
    assert_close(want, run_q4(a, wq, scales, zeros, M, K, N, 32), PEAK_TOL, ELEM_TOL, "odd K")
    s1, z1 = scales[:, :1].copy(), zeros[:, :1].copy()
    want = a.astype(np.float64) @ dequant_np(wq, s1, z1, K, K + 1).T
    assert_close(want, run_q4(a, wq, s1, z1, M, K, N, 0, n_groups=1), PEAK_TOL, ELEM_TOL, "group 0")


def test_routes_and_errors(oracle_mod):
    K, N = 1024, 64
    a, wq, scales, zeros = gen_q4(1, K, N, seed=9)
    fast = run_q4(a, wq, scales, zeros, 1, K, N, 32, route=_lib.ROUTE_GEMV)
    exact = run_q4(a, wq, scales, zeros, 1, K, N, 32, route=_lib.ROUTE_SIMT)
    assert_close(oracle_mod.ref_matmul_q4(a, wq, scales, zeros, 1, K, N, 32), exact, PEAK_TOL, ELEM_TOL, "exact")
    assert_close(exact, fast, PEAK_TOL, None)
    assert_fixed_point_bound(a[0], wq, scales, zeros, K, fast[0])
    with pytest.raises(_lib.BybyCudaError):   # the decode route refuses M > 1
        run_q4(np.vstack([a, a]), wq, scales, zeros, 2, K, N, 32, route=_lib.ROUTE_GEMV)
    with pytest.raises(_lib.BybyCudaError):   # too few groups per row
        run_q4(a, wq, scales, zeros, 1, K, N, 32, n_groups=8)


def test_nonfinite_activation_is_reported():
    K, N = 1024, 128
    a, wq, scales, zeros = gen_q4(1, K, N, seed=13)
    a[0, 77] = np.inf
    run_q4(a, wq, scales, zeros, 1, K, N, 32)
    assert _lib.device_error() == 7
    assert _lib.device_error() == 0


def test_session_resident_api_like_reference(oracle_mod):
    """residentUploadQ4 + sessionMatmulQ4 inside a session, and gpuMatmulQ4 (immediate)."""
    O = oracle_mod
    be = gb.GpuBackend.gbCuda
    M, K, N = 1, 2048, 512
    a, wq, scales, zeros = gen_q4(M, K, N, seed=21)
    want = O.ref_matmul_q4(a, wq, scales, zeros, M, K, N, 32)
    w = gb.residentUploadQ4(be, wq, scales, zeros, K, N, 32, K // 32)
    assert gb.residentPrepareQ4(w, M)
    assert gb.sessionBegin(be)
    ha = gb.sessionUpload(be, a)
    hc = gb.SessionHandle()
    assert gb.sessionMatmulQ4(be, ha, w, hc, M)
    assert gb.sessionEnd(be)
    assert_close(want, gb.sessionRead(be, hc, M * N).reshape(M, N), PEAK_TOL, None)
    for h in (ha, hc):
        gb.sessionFree(be, h)
    gb.residentFreeQ4(be, w)
    got = gb.gpuMatmulQ4(be, a, wq, scales, zeros, M, K, N, 32, K // 32)
    assert_close(want, got, PEAK_TOL, None)
    assert_fixed_point_bound(a[0], wq, scales, zeros, K, got[0])
    W = gb.Q4AsymWeights(wq, scales, zeros, K)
    out = W.matmul(torch.from_numpy(a).to(DEV))
    torch.cuda.synchronize()
    assert_close(want, out.cpu().numpy(), PEAK_TOL, None)


# ----------------------------------------------------------------------------------------
# The fused decode GEMV (sessionMatmulQ4Fused, gpubackend.nim:3185-3231): one launch
# ----------------------------------------------------------------------------------------

def _bound(w, x):
    """The decode kernel's per-element fixed-point bound for W . x (float64 arrays)."""
    N = w.shape[0]
    blk_max = np.abs(x).reshape(-1, 32).max(axis=1)
    quant = 2.0 ** -29 * (np.abs(w).reshape(N, -1, 32).sum(axis=2) * blk_max).sum(axis=1)
    return quant + 1e-5 * (np.abs(w) * np.abs(x)).sum(axis=1) + 1e-30


def _fused_case(Ns, K, seed, norm, res):
    rng = np.random.default_rng(seed)
    mats = [gen_q4(1, K, N, seed=seed + 17 * i)[1:] for i, N in enumerate(Ns)]
    x = rng.normal(0, 1, size=(1, K)).astype(np.float32)
    gamma = (rng.uniform(0.5, 1.5, K).astype(np.float32) if norm else None)
    r = rng.normal(0, 1, size=max(Ns)).astype(np.float32) if res else None
    xe = (x[0] * gamma).astype(np.float32) if norm else x[0]          # x * gamma in fp32, as the kernel
    inv = 1.0 / np.sqrt(np.mean(x[0].astype(np.float64) ** 2) + 1e-5) if norm else 1.0
    return mats, x, gamma, r, xe.astype(np.float64), inv


def _run_fused(mode, mats, x, gamma, r, K, eps=1e-5):
    Ws = [gb.Q4AsymWeights(wq, sc, zp, K) for wq, sc, zp in mats]
    outs = [torch.full((1, W.N), float("nan"), device=DEV) for W in Ws]
    dev_t = lambda v: None if v is None else torch.from_numpy(v).to(DEV)  # noqa: E731
    gb.matmul_q4_fused(mode, torch.from_numpy(x).to(DEV), Ws, outs, res=dev_t(r), gamma=dev_t(gamma), eps=eps)
    torch.cuda.synchronize()
    return [o.cpu().numpy()[0].astype(np.float64) for o in outs]


@pytest.mark.parametrize("norm,res", [(False, False), (True, True), (True, False), (False, True)])
def test_fused_mode0_shared_activations(norm, res):
    """Three matrices (q, k, v shapes) from one x: each output within its bound."""
    K, Ns = 4096, (4096, 1024, 1024)
    mats, x, gamma, r, xe, inv = _fused_case(Ns, K, 31, norm, res)
    got = _run_fused(0, mats, x, gamma, r, K)
    for (wq, sc, zp), N, o in zip(mats, Ns, got):
        w = dequant_np(wq, sc, zp, K, 32)
        want = inv * (w @ xe) + (r[:N].astype(np.float64) if res else 0.0)
        err = np.abs(o - want)
        assert (err <= inv * _bound(w, xe) + 1e-5 * np.abs(want)).all(), f"N={N}: {err.max():.3e}"
    assert _lib.device_error() == 0


@pytest.mark.parametrize("N,norm,res", [(11008, True, True), (32000, False, False), (300, True, False)])
def test_fused_mode1_silu_gate_up(N, norm, res):
    """silu(gate) * up (+ residual), gate and up rows in the same CTA; N = 32000 takes several
    gate / up pass pairs per CTA."""
    K = 4096
    mats, x, gamma, r, xe, inv = _fused_case((N, N), K, 41, norm, res)
    got = _run_fused(1, mats, x, gamma, r, K)[0]
    wg, wu = (dequant_np(*m, K, 32) for m in mats)
    g, u = inv * (wg @ xe), inv * (wu @ xe)
    sig = 1.0 / (1.0 + np.exp(-g))
    want = g * sig * u + (r[:N].astype(np.float64) if res else 0.0)
    dg, du = inv * _bound(wg, xe), inv * _bound(wu, xe)
    dsilu = np.abs(sig * (1.0 + g * (1.0 - sig)))                    # |silu'(g)| <= 1.1
    bound = (dsilu + 1e-3) * np.abs(u) * dg + np.abs(g * sig) * du + dg * du + 1e-5 * np.abs(want) + 1e-6
    err = np.abs(got - want)
    assert np.isfinite(got).all()
    assert (err <= bound).all(), f"worst excess {(err - bound).max():.3e}"


def test_fused_gate_up_pinned_to_reference_kernel(oracle_mod):
    """The fused decode GEMV (mode 1 with RMSNorm and the residual) against the reference's own
    nimf_cpu_matmul_q4 (oracle/_ref) for both products, then the fused shader's order on top
    (backends/vulkan/q4_autotune.nim:194-325): x * gamma feeds the products, the RMS of the raw
    x gives inv = 1 / sqrt(mean(x^2) + eps), gate and up are scaled by inv, silu(gate) * up,
    then + residual.  Bound: the decode kernel's fixed-point bound on each product."""
    O = oracle_mod
    if not O.ref_available():
        pytest.skip("oracle/_ref (the reference's CPU C) is not built")
    K, N, eps = 4096, 11008, 1e-5
    mats, x, gamma, r, xe, _ = _fused_case((N, N), K, 61, True, True)
    got = _run_fused(1, mats, x, gamma, r, K, eps=eps)[0]
    xg = (x[0] * gamma).astype(np.float32)[None, :]       # the shader's x[t] = raw * gamma[k + t]
    g_raw, u_raw = (O.ref_matmul_q4(xg, wq, sc, zp, 1, K, N, 32, threads=8)[0].astype(np.float64)
                    for wq, sc, zp in mats)
    inv = 1.0 / np.sqrt(np.float32(np.sum(x[0].astype(np.float32) ** 2)) / np.float32(K) + np.float32(eps))
    g, u = g_raw * inv, u_raw * inv
    sig = 1.0 / (1.0 + np.exp(-g))
    want = g * sig * u + r[:N].astype(np.float64)
    wg, wu = (dequant_np(*m, K, 32) for m in mats)
    dg, du = inv * _bound(wg, xe), inv * _bound(wu, xe)
    dsilu = np.abs(sig * (1.0 + g * (1.0 - sig)))
    bound = (dsilu + 1e-3) * np.abs(u) * dg + np.abs(g * sig) * du + dg * du + 1e-5 * np.abs(want) + 1e-6
    err = np.abs(got - want)
    assert np.isfinite(got).all()
    assert (err <= bound).all(), f"worst excess {(err - bound).max():.3e}"
    assert np.abs(got - want).max() <= 1e-3 * max(1.0, np.abs(want).max())


def test_fused_session_api_and_unsupported():
    be = gb.GpuBackend.gbCuda
    K, N = 2048, 512
    mats, x, gamma, r, xe, inv = _fused_case((N, N), K, 51, True, True)
    ws = [gb.residentUploadQ4(be, wq, sc, zp, K, N, 32, K // 32) for wq, sc, zp in mats]
    assert gb.sessionBegin(be)
    ha, hg, hr = gb.sessionUpload(be, x), gb.sessionUpload(be, gamma), gb.sessionUpload(be, r)
    outs = [gb.sessionAllocScratch(be, N), gb.sessionAllocScratch(be, N)]
    assert gb.sessionMatmulQ4Fused(be, 1, ha, ws, outs, hr, True, hg, 1e-5, True)
    # unsupported forms return False and leave the session usable
    assert not gb.sessionMatmulQ4Fused(be, 1, ha, ws[:1], outs, hr, True, hg, 1e-5, True)   # mode 1 needs 2
    assert not gb.sessionMatmulQ4Fused(be, 0, ha, ws, [outs[0]], hr, False)                 # too few outputs
    assert gb.sessionEnd(be)
    got = gb.sessionRead(be, outs[0], N).astype(np.float64)
    wg, wu = (dequant_np(*m, K, 32) for m in mats)
    g, u = inv * (wg @ xe), inv * (wu @ xe)
    want = g / (1.0 + np.exp(-g)) * u + r.astype(np.float64)
    assert np.abs(got - want).max() <= 1e-3 * max(1.0, np.abs(want).max())
    for h in (ha, hg, hr, *outs):
        gb.sessionFree(be, h)
    for w in ws:
        gb.residentFreeQ4(be, w)
    # a K the fused kernel cannot tile: BYBYCU_ERR_SHAPE for the caller's unfused fallback
    Ws = [gb.Q4AsymWeights(*gen_q4(1, 96, 16, seed=3)[1:], 96)]
    with pytest.raises(_lib.BybyCudaError) as ei:
        gb.matmul_q4_fused(0, torch.zeros(1, 96, device=DEV), Ws, [torch.empty(1, 16, device=DEV)])
    assert ei.value.code == _lib.ERR_SHAPE
