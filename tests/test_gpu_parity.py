"""GPU parity of libbybycuda.so against the reference's CPU arithmetic, through the C ABI.

Tolerances (written here, per route):
* SIMT route: bit-identical to the reference CPU VM (same fmaf order).
* GEMV route: the reference test's own check, max|diff| <= 1e-4 * max(1, max|ref|)
  (tests/t_fp4_tile_gemm.nim:54-67), and per element |diff| <= 1e-3 * max(1, |ref|) (the
  1e-3 relative bound of the path's parity gate, vulkan_driver.nim:2754).
* GEMV route at M = 1 (the decode kernel's integer mode): the activations of each 32-block
  become 15-bit fixed point on the block's largest exponent, so besides the bounds above,
  on inputs of any dynamic range |diff| <= 2^-14 * sum_b max|x_b| * sum_{k in b} |w[n, k]|
  plus fp32 slack (test_gemv_m1_activation_dynamic_range).
* dequantisation: bit-exact for every format.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from bybylang_b200 import _lib  # noqa: E402
from bybylang_b200 import gpubackend as gb  # noqa: E402

from gpu_helpers import DEV, dev, q4_slot, run  # noqa: E402
from gpu_helpers import assert_close as _assert_close  # noqa: E402

PEAK_TOL = 1e-4
ELEM_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _init():
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    yield
    assert _lib.device_error() == 0


def lib():
    return _lib.load()


def assert_close(want, got, peak_tol=PEAK_TOL, elem_tol=ELEM_TOL, what=""):
    _assert_close(want, got, peak_tol, elem_tol, what)


# ----------------------------------------------------------------------------------------
# SIMT route: bit-identical to the reference CPU VM
# ----------------------------------------------------------------------------------------

def test_simt_fp4km_reference_cases_bit_exact(golden):
    g = golden["ref_tile_cases"]
    for i in range(5):
        M, K, N = (int(v) for v in g[f"fp4_{i}_shape"])
        out = run(0, M, K, N, dev(g[f"fp4_{i}_x"]), dev(g[f"fp4_{i}_packed"]), scale_base=N * K // 2,
                  lut=dev(g[f"fp4_{i}_table"]), route=_lib.ROUTE_SIMT)
        assert np.array_equal(out.cpu().numpy(), g[f"fp4_{i}_dyn"]), f"case {i}"


def test_simt_f16_reference_cases_bit_exact(golden):
    g = golden["ref_tile_cases"]
    for i in range(5):
        M, K, N = (int(v) for v in g[f"f16_{i}_shape"])
        out = run(1, M, K, N, dev(g[f"f16_{i}_x"]), dev(g[f"f16_{i}_halves"].view(np.uint8)), route=_lib.ROUTE_SIMT)
        assert np.array_equal(out.cpu().numpy(), g[f"f16_{i}_dyn"]), f"case {i}"


def test_simt_q4b32_bit_exact(golden, oracle_mod):
    g = golden["ref_q4b32"]
    for i in range(8):
        M, K, N = (int(v) for v in g[f"q4_{i}_shape"])
        slot, sb = q4_slot(g[f"q4_{i}_packed"], g[f"q4_{i}_scales"])
        x = dev(oracle_mod.bf16_to_f32(g[f"q4_{i}_x_bf16"]))
        out = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_SIMT)
        assert np.array_equal(out.cpu().numpy(), g[f"q4_{i}_vm"]), f"case {i}"
        xb = dev(g[f"q4_{i}_x_bf16"]).view(torch.bfloat16)
        out = run(2, M, K, N, xb, slot, scale_base=sb, route=_lib.ROUTE_SIMT)
        assert np.array_equal(out.cpu().numpy(), g[f"q4_{i}_vm"]), f"case {i} bf16 input"


# ----------------------------------------------------------------------------------------
# GEMV route (format 2, M <= 16)
# ----------------------------------------------------------------------------------------

def test_gemv_q4b32_golden_cases(golden, oracle_mod):
    g = golden["ref_q4b32"]
    ran = 0
    for i in range(8):
        M, K, N = (int(v) for v in g[f"q4_{i}_shape"])
        if M > 16:
            continue
        slot, sb = q4_slot(g[f"q4_{i}_packed"], g[f"q4_{i}_scales"])
        xb = dev(g[f"q4_{i}_x_bf16"]).view(torch.bfloat16)
        out = run(2, M, K, N, xb, slot, scale_base=sb, route=_lib.ROUTE_GEMV)
        assert_close(g[f"q4_{i}_vm"], out.cpu().numpy(), what=f"case {i} bf16")
        xf = dev(oracle_mod.bf16_to_f32(g[f"q4_{i}_x_bf16"]))
        out = run(2, M, K, N, xf, slot, scale_base=sb, route=_lib.ROUTE_GEMV)
        assert_close(g[f"q4_{i}_vm"], out.cpu().numpy(), what=f"case {i} f32")
        ran += 1
    assert ran == 5


@pytest.mark.parametrize("M,K,N", [(1, 4096, 11008), (16, 4096, 11008), (1, 11008, 4096), (16, 11008, 4096),
                                   (4, 4096, 4096), (9, 4096, 12288)])
def test_gemv_benchmark_shapes_against_oracle(M, K, N, oracle_mod):
    O = oracle_mod
    p, s = O.gen_q4b32(N, K)
    xb = O.gen_x_bf16(M, K)
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N, threads=8)
    slot, sb = q4_slot(p, s)
    out = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb, route=_lib.ROUTE_GEMV)
    assert_close(want, out.cpu().numpy(), what=f"M={M} K={K} N={N}")


def test_gemv_lm_head_columns_against_oracle(oracle_mod):
    """C5 (N = 128256): the whole GEMM on the GPU, a column sample through the oracle."""
    O = oracle_mod
    M, K, N = 1, 4096, 128256
    p, s = O.gen_q4b32(N, K)
    xb = O.gen_x_bf16(M, K)
    slot, sb = q4_slot(p, s)
    out = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb, route=_lib.ROUTE_GEMV).cpu().numpy()
    cols = np.r_[0:512, 60000:60512, N - 512:N]
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p[cols], s[cols], M, K, len(cols), threads=8)
    assert_close(want, out[:, cols], what="lm head")


@pytest.mark.parametrize("M,N", [(9, 11008), (16, 11008)])
def test_gemv_fp32_rows_beside_wide_tiles(M, N, oracle_mod):
    """fp32 rows of 9-16 activations beside 80-row weight tiles: four ring stages do not fit in
    shared memory, so the GEMV plans two or three."""
    O = oracle_mod
    K = 4096
    p, s = O.gen_q4b32(N, K, seed=77 + M)
    xf = O.gen_x_f32(M, K, seed=78 + M)
    want = O.tile_gemm_q4b32(xf, p, s, M, K, N, threads=8)
    slot, sb = q4_slot(p, s)
    out = run(2, M, K, N, dev(xf), slot, scale_base=sb, route=_lib.ROUTE_GEMV)
    assert_close(want, out.cpu().numpy(), 1e-4, 1e-3, what=f"fp32 M={M} N={N}")


@pytest.mark.parametrize("M,K,N", [(1, 32, 1), (2, 96, 15), (3, 288, 17), (7, 4128, 130), (8, 256, 16),
                                   (12, 800, 33), (16, 64, 1000), (5, 4096, 1)])
def test_gemv_ragged_shapes(M, K, N, oracle_mod):
    O = oracle_mod
    p, s = O.gen_q4b32(N, K, seed=1234 + M)
    xb = O.gen_x_bf16(M, K, seed=99 + K)
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N)
    slot, sb = q4_slot(p, s)
    out = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb, route=_lib.ROUTE_GEMV)
    assert_close(want, out.cpu().numpy(), what=f"M={M} K={K} N={N}")
    # an unaligned scale block (scale_base not a multiple of 16) takes the non-TMA scale loads
    blob = np.zeros(p.size + 2 + s.size * 2, np.uint8)
    blob[:p.size] = p.ravel()
    blob[p.size + 2:] = s.view(np.uint8).ravel()
    out = run(2, M, K, N, dev(xb).view(torch.bfloat16), dev(blob), scale_base=p.size + 2, route=_lib.ROUTE_GEMV)
    assert_close(want, out.cpu().numpy(), what=f"M={M} K={K} N={N} unaligned scales")


def _bf16_bits(f):
    """float32 -> bf16 bits, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(f, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("xdt", ["bf16", "f32"])
@pytest.mark.parametrize("K,N", [(4096, 2048), (800, 300)])
def test_gemv_m1_activation_dynamic_range(K, N, xdt, oracle_mod):
    """Activations over 36 binades, zeros, a lone outlier over tiny values, all-tiny blocks:
    the decode kernel stays inside its fixed-point error bound against the f64 reference:
    2^-14 of each block's largest value for bf16 rows (one image), 2^-29 for full-precision
    fp32 rows (two images)."""
    O = oracle_mod
    rng = np.random.default_rng(K + N)
    p, s = O.gen_q4b32(N, K, seed=77)
    xf = (rng.choice([-1.0, 1.0], K) * np.exp2(rng.uniform(-24, 12, K))).astype(np.float32)
    xf[rng.random(K) < 0.1] = 0.0
    xf[3 * 32:4 * 32] = 0.0                         # an all-zero block
    xf[5 * 32:6 * 32] = 1e-6
    xf[5 * 32 + 7] = -3e4                           # one outlier over tiny values
    xf[7 * 32:8 * 32] = 1e-30                       # a block of tiny values
    xf[9 * 32:10 * 32] = -2.0                       # equal values
    xb = _bf16_bits(xf).reshape(1, K)
    x = O.bf16_to_f32(xb) if xdt == "bf16" else xf.reshape(1, K)
    want = O.tile_gemm_q4b32_f64(x, p, s, 1, K, N)[0]
    slot, sb = q4_slot(p, s)
    xd = dev(xb).view(torch.bfloat16) if xdt == "bf16" else dev(x)
    got = run(2, 1, K, N, xd, slot, scale_base=sb, route=_lib.ROUTE_GEMV).cpu().numpy()[0].astype(np.float64)
    w = np.abs(O.dequant_q4b32(p, s, N, K).astype(np.float64))   # |q| * |s|
    xa = np.abs(x[0].astype(np.float64))
    blk_max = xa.reshape(-1, 32).max(axis=1)
    quant = 2.0 ** (-14 if xdt == "bf16" else -29) * (w.reshape(N, -1, 32).sum(axis=2) * blk_max).sum(axis=1)
    slack = 1e-5 * (w * xa).sum(axis=1) + 1e-30
    err = np.abs(got - want)
    assert np.isfinite(got).all()
    assert (err <= quant + slack).all(), f"worst excess {(err - quant - slack).max():.3e}"
    assert _lib.device_error() == 0


@pytest.mark.parametrize("K,N", [(4096, 11008), (11008, 4096), (4192, 300), (1024, 64)])
def test_gemv_m1_f32_rows_per_element(K, N, oracle_mod, parity_log):
    """fp32 decode rows with their full mantissa (the integer mode's two fixed-point images):
    per element within 1e-3 of the oracle's fp32 arithmetic, and within 2e-5 of the f64
    result (the reference's own fp32 chain is about that far from it)."""
    from gpu_helpers import elem_err
    O = oracle_mod
    p, s = O.gen_q4b32(N, K, seed=K + 3)
    xf = O.gen_x_f32(1, K, seed=N)
    slot, sb = q4_slot(p, s)
    got = run(2, 1, K, N, dev(xf), slot, scale_base=sb, route=_lib.ROUTE_GEMV).cpu().numpy()
    want = O.tile_gemm_q4b32(xf, p, s, 1, K, N, threads=8)
    assert_close(want, got, what=f"K={K} N={N}")
    worst = elem_err(want, got)
    parity_log.append((f"1x{K}x{N} fp32 x, route GEMV (integer mode, two images)", worst, 1e-3))
    exact = elem_err(O.tile_gemm_q4b32_f64(xf, p, s, 1, K, N), got)
    assert exact <= 2e-5, f"against f64: {exact:.3e}"
    assert _lib.device_error() == 0


def test_gemv_m1_nonfinite_f32_activation_is_reported(oracle_mod):
    """An fp32 inf or NaN activation has no fixed-point image either: device error 7, no
    fault; the next call is clean."""
    O = oracle_mod
    K, N = 2048, 256
    p, s = O.gen_q4b32(N, K)
    xf = O.gen_x_f32(1, K)
    slot, sb = q4_slot(p, s)
    for bad in (float("nan"), float("-inf")):
        x = dev(xf).clone()
        x[0, 1500] = bad
        run(2, 1, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_GEMV)
        assert _lib.device_error() == 7
        assert _lib.device_error() == 0   # read-and-clear
    out = run(2, 1, K, N, dev(xf), slot, scale_base=sb, route=_lib.ROUTE_GEMV)
    assert_close(O.tile_gemm_q4b32(xf, p, s, 1, K, N), out.cpu().numpy())


def test_gemv_m1_nonfinite_activation_is_reported(oracle_mod):
    """An inf activation has no fixed-point image: device error 7, no fault, and the
    context stays usable."""
    O = oracle_mod
    K, N = 1024, 256
    p, s = O.gen_q4b32(N, K)
    xb = O.gen_x_bf16(1, K)
    slot, sb = q4_slot(p, s)
    x = dev(xb).view(torch.bfloat16).clone()
    x[0, 100] = float("inf")
    run(2, 1, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_GEMV)
    assert _lib.device_error() == 7
    assert _lib.device_error() == 0   # read-and-clear
    out = run(2, 1, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb, route=_lib.ROUTE_GEMV)
    assert_close(O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, 1, K, N), out.cpu().numpy())


def test_gemv_bf16_output(oracle_mod):
    O = oracle_mod
    M, K, N = 3, 4096, 2048
    p, s = O.gen_q4b32(N, K)
    xb = O.gen_x_bf16(M, K)
    slot, sb = q4_slot(p, s)
    x = dev(xb).view(torch.bfloat16)
    f32 = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_GEMV)
    b16 = run(2, M, K, N, x, slot, scale_base=sb, route=_lib.ROUTE_GEMV, out_dtype=torch.bfloat16)
    assert torch.equal(f32.to(torch.bfloat16), b16)


def test_auto_route_small_m_is_gemv(oracle_mod):
    assert gb.route_for(2, 1, 4096, 11008) == _lib.ROUTE_GEMV
    O = oracle_mod
    p, s = O.gen_q4b32(96, 256)
    xb = O.gen_x_bf16(2, 256)
    slot, sb = q4_slot(p, s)
    out = run(2, 2, 256, 96, dev(xb).view(torch.bfloat16), slot, scale_base=sb)
    assert_close(O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, 2, 256, 96), out.cpu().numpy())


# ----------------------------------------------------------------------------------------
# Format 1 (fp16 weights) on the decode route (M <= 8): the GEMV tolerances
# ----------------------------------------------------------------------------------------

def test_f16_gemv_reference_cases(golden):
    g = golden["ref_tile_cases"]
    ran = 0
    for i in range(5):
        M, K, N = (int(v) for v in g[f"f16_{i}_shape"])
        if M > 8:
            continue
        out = run(1, M, K, N, dev(g[f"f16_{i}_x"]), dev(g[f"f16_{i}_halves"].view(np.uint8)), route=_lib.ROUTE_GEMV)
        assert_close(g[f"f16_{i}_dyn"], out.cpu().numpy(), what=f"case {i}")
        ran += 1
    assert ran >= 1


@pytest.mark.parametrize("M,K,N,xbf16", [(1, 4096, 11008, True), (1, 4096, 11008, False), (3, 512, 300, True),
                                         (8, 1024, 77, False), (1, 32, 1, True), (5, 2048, 1000, True)])
def test_f16_gemv_against_oracle(M, K, N, xbf16, oracle_mod):
    O = oracle_mod
    rng = np.random.default_rng(M * K + N)
    halves = (rng.normal(0, 0.05, size=(N, K))).astype(np.float16)
    if xbf16:
        xb = O.gen_x_bf16(M, K, seed=N)
        x = dev(xb).view(torch.bfloat16)
        xf = O.bf16_to_f32(xb)
    else:
        xf = rng.normal(0, 1, size=(M, K)).astype(np.float32)
        x = dev(xf)
    want = O.tile_gemm_f16(xf, halves.view(np.uint16), M, K, N)
    out = run(1, M, K, N, x, dev(halves.view(np.uint8)), route=_lib.ROUTE_GEMV)
    assert_close(want, out.cpu().numpy(), what=f"M={M} K={K} N={N}")
    b16 = run(1, M, K, N, x, dev(halves.view(np.uint8)), route=_lib.ROUTE_GEMV, out_dtype=torch.bfloat16)
    assert torch.equal(out.to(torch.bfloat16), b16)


def test_auto_route_f16_decode_is_gemv():
    assert gb.route_for(1, 1, 4096, 4096) == _lib.ROUTE_GEMV
    assert gb.route_for(1, 8, 4096, 4096) == _lib.ROUTE_GEMV
    assert gb.route_for(1, 9, 4096, 4096) == _lib.ROUTE_TC        # format 1 prefill: tcgen05
    assert gb.route_for(1, 9, 4096 + 32, 4096) == _lib.ROUTE_SIMT  # K % 128 != 0


# ----------------------------------------------------------------------------------------
# Dequantisation: bit-exact
# ----------------------------------------------------------------------------------------

def test_dequant_bit_exact_all_formats(golden, oracle_mod):
    O = oracle_mod
    N, K = 80, 4096
    p, s = O.gen_q4b32(N, K)
    slot, sb = q4_slot(p, s)
    w = torch.empty(N, K, dtype=torch.float32, device=DEV)
    gb.dequant(2, slot, w, K=K, N=N, scale_base=sb)
    torch.cuda.synchronize()
    assert np.array_equal(w.cpu().numpy(), O.dequant_q4b32(p, s, N, K))
    g = golden["ref_tile_cases"]
    M, K, N = (int(v) for v in g["fp4_3_shape"])
    w = torch.empty(N, K, dtype=torch.float32, device=DEV)
    gb.dequant(0, dev(g["fp4_3_packed"]), w, K=K, N=N, scale_base=N * K // 2, lut=dev(g["fp4_3_table"]))
    torch.cuda.synchronize()
    assert np.array_equal(w.cpu().numpy(), O.dequant_fp4km(g["fp4_3_packed"], g["fp4_3_table"], N, K))
    M, K, N = (int(v) for v in g["f16_4_shape"])
    w = torch.empty(N, K, dtype=torch.float32, device=DEV)
    gb.dequant(1, dev(g["f16_4_halves"].view(np.uint8)), w, K=K, N=N)
    torch.cuda.synchronize()
    assert np.array_equal(w.cpu().numpy(), O.f16_to_f32(g["f16_4_halves"]))


# ----------------------------------------------------------------------------------------
# The micro-VM twin and the session API
# ----------------------------------------------------------------------------------------

def _vm(code, mem_len, packed, lut, x):
    mem = torch.zeros(mem_len, dtype=torch.float32, device=DEV)
    err = C.create_string_buffer(256)
    words = np.ascontiguousarray(code, np.uint32)
    rc = lib().bybycu_vm_run_slots(words.ctypes.data_as(C.POINTER(C.c_uint32)), len(words),
                                   C.c_void_p(mem.data_ptr()), mem_len, C.c_void_p(packed.data_ptr()),
                                   packed.numel(), C.c_void_p(lut.data_ptr()), lut.numel(),
                                   C.c_void_p(x.data_ptr()), x.numel(), 128, 64, 128, err, 256, None)
    torch.cuda.synchronize()
    assert rc == 0, err.value
    return mem.cpu().numpy()


def test_vm_programs_match_reference(golden, oracle_mod):
    O = oracle_mod
    g = golden["ref_tile_cases"]
    for i in range(5):
        M, K, N = (int(v) for v in g[f"fp4_{i}_shape"])
        x, packed, table = dev(g[f"fp4_{i}_x"]), dev(g[f"fp4_{i}_packed"]), dev(g[f"fp4_{i}_table"])
        for rows in (0, M):
            got = _vm(O.fp4_tile_program(rows, K, N, N * K // 2), M * N, packed, table, x)
            assert np.array_equal(got, g[f"fp4_{i}_dyn"].ravel()), f"case {i} rows {rows}"
        if f"fp4_{i}_legacy" in g:
            lut_word = (N * (K // 2) + N * (K // 32) + 3) // 4
            blob = np.zeros(lut_word * 4 + 272 * 4, np.uint8)
            blob[:g[f"fp4_{i}_packed"].size] = g[f"fp4_{i}_packed"]
            blob[lut_word * 4:] = g[f"fp4_{i}_table"].view(np.uint8)
            code = np.array([0xAC, M, K, N, 32, K // 32, 1], np.uint32)
            db = dev(blob)
            got = _vm(code, M * N, db, db.view(torch.float32), x)
            assert np.array_equal(got, g[f"fp4_{i}_legacy"].ravel()), f"case {i} legacy"
    q = golden["ref_q4b32"]
    for i in range(8):
        M, K, N = (int(v) for v in q[f"q4_{i}_shape"])
        p, s = q[f"q4_{i}_packed"], q[f"q4_{i}_scales"]
        xf = dev(O.bf16_to_f32(q[f"q4_{i}_x_bf16"]))
        wq, sc, zp = O.q4b32_to_asym(p, s, N, K)
        sbw = (N * (K // 2) + 3) // 4
        blob = np.zeros((sbw + 2 * sc.size) * 4, np.uint8)
        blob[:wq.size] = wq
        f = blob.view(np.float32)
        f[sbw:sbw + sc.size], f[sbw + sc.size:] = sc, zp
        db = dev(blob)
        got = _vm(np.array([0xAB, M, K, N, 32, K // 32, 1], np.uint32), M * N, db, db.view(torch.float32), xf)
        assert np.array_equal(got, q[f"q4_{i}_q4gemv"].ravel()), f"q4 gemv case {i}"
        slot, sb = q4_slot(p, s)
        prog = np.array([0xB0 | (2 << 8), 0, K, N, sb, 0, 0xB1, 0xB2, 0xB4, 0xB5, 0x50, 0xB6, 0x50, 0xB3, 0xB7, 1],
                        np.uint32)
        got = _vm(prog, M * N, slot, torch.zeros(1, device=DEV), xf)
        assert_close(q[f"q4_{i}_vm"].ravel(), got, what=f"format 2 program case {i}")


def test_session_api_like_reference_test(golden):
    """The reference test's gpuRun (t_fp4_tile_gemm.nim:104-117) on the cuda backend."""
    be = gb.parseBackend("cuda")
    g = golden["ref_tile_cases"]
    for i in range(5):
        M, K, N = (int(v) for v in g[f"fp4_{i}_shape"])
        for tc in (True, False):
            assert gb.sessionBegin(be)
            hx = gb.sessionUpload(be, g[f"fp4_{i}_x"])
            hw = gb.sessionUpload(be, g[f"fp4_{i}_packed"])
            hl = gb.sessionUpload(be, g[f"fp4_{i}_table"])
            o = gb.sessionAllocScratch(be, M * N)
            enc = gb.sessionFp4GemmTensorCore if tc else gb.sessionFp4GemmTiledEnc
            assert enc(be, hx, hw, hl, o, M, K, N)
            assert gb.sessionEnd(be)
            got = gb.sessionRead(be, o, M * N)
            for h in (hx, hw, hl, o):
                gb.sessionFree(be, h)
            np.testing.assert_allclose(got, g[f"fp4_{i}_dyn"].ravel(), rtol=0,
                                       atol=1e-4 * max(1.0, float(np.abs(g[f"fp4_{i}_dyn"]).max())))
    assert gb.gForbidCpuFallback


def test_session_errors_raise_not_fall_back():
    be = gb.GpuBackend.gbCuda
    assert gb.sessionBegin(be)
    hx = gb.sessionUpload(be, np.zeros(64, np.float32))
    o = gb.sessionAllocScratch(be, 16)
    with pytest.raises(_lib.BybyCudaError, match="fallback is forbidden"):
        gb.sessionQ4B32Gemm(be, hx, hx, o, 1, 64, 16)   # weight slot too small
    with pytest.raises(_lib.BybyCudaError):
        gb.sessionEnd(be)   # reports the session's first failure
    gb.sessionFree(be, hx)
    gb.sessionFree(be, o)


def test_parity_gates():
    be = gb.GpuBackend.gbCuda
    for f16 in (False, True):
        assert gb.sessionTileGemmReady(be, f16, False)
    assert gb.sessionTileGemmReady(be, False, True, fmt=2)


@pytest.mark.parametrize("M,K,N,x_pinned,out_pinned", [
    (1, 4096, 11008, True, True),     # decode: x fetched by the upload kernel, result stored to host
    (1, 4096, 11008, False, True),    # pageable x: the copy engine
    (1, 8192, 1000, True, False),     # pageable output: out_dev and a copy back
    (3, 512, 300, True, True),        # M > 1 through the upload kernel
    (16, 4096, 256, True, True),      # 128 KB of x: the copy engine
])
def test_host_io_entry_point(M, K, N, x_pinned, out_pinned, oracle_mod):
    """bybycu_tile_gemm_host: host activations in, host output back (the e2e form)."""
    O = oracle_mod
    p, s = O.gen_q4b32(N, K, seed=M + K)
    xb = O.gen_x_bf16(M, K, seed=N)
    slot, sb = q4_slot(p, s)
    xh = torch.from_numpy(xb).pin_memory() if x_pinned else torch.from_numpy(xb.copy())
    oh = torch.zeros(M, N, dtype=torch.float32)
    if out_pinned:
        oh = oh.pin_memory()
    xd = torch.full((M, K), 7.0, dtype=torch.bfloat16, device=DEV)   # a sentinel
    od = torch.empty(M, N, dtype=torch.float32, device=DEV)
    rc = lib().bybycu_tile_gemm_host(2, M, K, N, C.c_void_p(xh.data_ptr()), _lib.DT_BF16, C.c_void_p(slot.data_ptr()),
                                     slot.numel(), sb, None, 0, 0, C.c_void_p(oh.data_ptr()), _lib.DT_F32,
                                     C.c_void_p(xd.data_ptr()), C.c_void_p(od.data_ptr()), _lib.ROUTE_AUTO, None)
    assert rc == 0, _lib.last_error()
    assert_close(O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N, threads=8), oh.numpy())
    assert torch.equal(xd.cpu(), xh.view(torch.bfloat16))   # x_dev holds the row either way


# ----------------------------------------------------------------------------------------
# Failure detection without a GPU fault: a peer that never signals
# ----------------------------------------------------------------------------------------

def test_allgather_wait_for_a_silent_peer_times_out_and_reports():
    """world = 2 with rank 1 absent: its output and signal arrays are local buffers that no
    kernel ever signals.  The GEMV's bounded wait gives up after ~2 s, records device error 5
    (peer wait) and returns; the context stays usable for the next call."""
    import time
    from bybylang_b200.formats import synthetic_q4b32, synthetic_x
    M, K, N = 1, 1024, 256
    n0, n1 = 0, 128
    nib, sc = synthetic_q4b32(N, K, seed=3, device=DEV)
    shard = gb.Q4B32Weights(nib[n0:n1], sc[n0:n1], device=DEV)
    x = synthetic_x(M, K, seed=4, device=DEV)
    out = torch.zeros(M, N, dtype=torch.float32, device=DEV)
    absent_out = torch.zeros(M, N, dtype=torch.float32, device=DEV)
    sig = [torch.zeros(16, dtype=torch.int32, device=DEV) for _ in range(2)]
    peer_out = (C.c_void_p * 2)(out.data_ptr(), absent_out.data_ptr())
    peer_sig = (C.POINTER(C.c_uint32) * 2)(*[C.cast(C.c_void_p(t.data_ptr()), C.POINTER(C.c_uint32)) for t in sig])
    assert _lib.device_error() == 0
    t0 = time.time()
    rc = lib().bybycu_tile_gemm_allgather(2, M, K, N, n0, n1, C.c_void_p(x.data_ptr()), _lib.DT_BF16,
                                          C.c_void_p(shard.packed.data_ptr()), shard.packed.numel(), shard.scale_base,
                                          None, 0, 0, C.c_void_p(out.data_ptr()), peer_out, peer_sig, 2, 0, 1, None)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert _lib.device_error() == 5          # the peer wait ran out
    assert 1.5 < waited < 30.0
    # this rank's slice was computed and "sent" before the wait
    ref = shard.matmul(x)
    assert torch.equal(out[:, n0:n1], ref)
    assert torch.equal(absent_out[:, n0:n1], ref)
    # the context is healthy: an ordinary call still works
    again = shard.matmul(x)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)
    assert _lib.device_error() == 0
