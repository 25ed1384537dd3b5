"""GPU parity at BASELINE's own configurations, through the automatic route, against the CPU
oracle (the C restatement pinned bit-exactly to the reference's CPU VM in test_oracle.py).

Every case is held to the reference gate's per-element metric,
|got - want| / max(1, |want|) <= 1e-3 (backends/vulkan/vulkan_driver.nim:2752-2754), on
seeded random data with BASELINE's distributions (q uniform in [-8, 7], fp16 scales
|N(0, 0.02)|, activations N(0, 1)), and to the reference test's peak-normalised metric
(tests/t_fp4_tile_gemm.nim:54-67): 1e-4 on the GEMV route, 1e-3 on the tensor-core route.
The measured worst per-element error of every case is printed in the run's summary.

* C1: M=32, K=N=4096, x fp32 (the reference CPU backend's own configuration).
* C4: the Llama-7B projections [4096x4096], [11008x4096], [4096x11008] at M = 1, 16 and 128.
* C5: the LM head [128256x4096] at M = 1 and 64, on a column sample.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from bybylang_b200 import _lib  # noqa: E402
from bybylang_b200 import gpubackend as gb  # noqa: E402

from gpu_helpers import assert_close, dev, elem_err, q4_slot, run  # noqa: E402

ELEM_TOL = 1e-3
THREADS = os.cpu_count() or 8


@pytest.fixture(scope="module", autouse=True)
def _init():
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    yield
    assert _lib.device_error() == 0


def _weights(O, N, K, seed):
    p, s = O.gen_q4b32(N, K, seed=O.Xorshift32.SEED + seed)
    slot, sb = q4_slot(p, s)
    return p, s, slot, sb


def _peak_tol(route):
    return 1e-4 if route == _lib.ROUTE_GEMV else 1e-3


def test_c1_fp32_rows_per_element(oracle_mod, parity_log):
    """C1 through AUTO: 32 fp32 rows take the tensor-core route, each activation as two fp16
    terms (x_hi and the remainder x_lo)."""
    O = oracle_mod
    M, K, N = 32, 4096, 4096
    p, s, slot, sb = _weights(O, N, K, 1)
    xf = O.gen_x_f32(M, K, seed=O.Xorshift32.SEED + 3)
    route = gb.route_for(2, M, K, N, _lib.DT_F32)
    assert route == _lib.ROUTE_TC
    want = O.tile_gemm_q4b32(xf, p, s, M, K, N, threads=THREADS)
    got = run(2, M, K, N, dev(xf), slot, scale_base=sb).cpu().numpy()
    worst = elem_err(want, got)
    parity_log.append(("C1 32x4096x4096 fp32 x, AUTO (TC, two fp16 terms per activation)", worst, ELEM_TOL))
    assert_close(want, got, _peak_tol(route), ELEM_TOL, what="C1")


@pytest.mark.parametrize("M", [1, 16, 128])
@pytest.mark.parametrize("N,K", [(4096, 4096), (11008, 4096), (4096, 11008)])
def test_c4_projection_per_element(M, N, K, oracle_mod, parity_log):
    """C4: one Llama-7B projection at decode (M = 1), small batch (16) and prefill (128), bf16
    activations, every output through AUTO."""
    O = oracle_mod
    p, s, slot, sb = _weights(O, N, K, 2 + M)
    xb = O.gen_x_bf16(M, K, seed=O.Xorshift32.SEED + 5 + M)
    route = gb.route_for(2, M, K, N)
    # the tensor cores from 4 bf16 rows on when K >= 8192 (the down projection)
    assert route == (_lib.ROUTE_GEMV if M == 1 or (M <= 16 and K < 8192) else _lib.ROUTE_TC)
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N, threads=THREADS)
    got = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb).cpu().numpy()
    worst = elem_err(want, got)
    parity_log.append((f"C4 {M}x{K}x{N} bf16 x, AUTO ({_lib.ROUTE_NAMES[route]})", worst, ELEM_TOL))
    assert_close(want, got, _peak_tol(route), ELEM_TOL, what=f"C4 M={M} N={N} K={K}")


@pytest.mark.parametrize("M", [1, 64])
def test_c5_lm_head_per_element(M, oracle_mod, parity_log):
    """C5: the whole [M, 128256] product on the GPU, 1536 columns (start, middle, end of the
    vocabulary) through the oracle."""
    O = oracle_mod
    K, N = 4096, 128256
    p, s, slot, sb = _weights(O, N, K, 9)
    xb = O.gen_x_bf16(M, K, seed=O.Xorshift32.SEED + 11)
    route = gb.route_for(2, M, K, N)
    assert route == (_lib.ROUTE_GEMV if M == 1 else _lib.ROUTE_TC)
    got = run(2, M, K, N, dev(xb).view(torch.bfloat16), slot, scale_base=sb).cpu().numpy()
    cols = np.r_[0:512, 64000:64512, N - 512:N]
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p[cols], s[cols], M, K, len(cols), threads=THREADS)
    worst = elem_err(want, got[:, cols])
    parity_log.append((f"C5 {M}x{K}x{N} bf16 x, AUTO ({_lib.ROUTE_NAMES[route]}), 1536 columns", worst, ELEM_TOL))
    assert_close(want, got[:, cols], _peak_tol(route), ELEM_TOL, what=f"C5 M={M}")
    assert np.isfinite(got).all()
