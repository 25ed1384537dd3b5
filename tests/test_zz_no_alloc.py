"""bybycu_tile_gemm_noalloc: the tensor-core GEMM with its activation staging in a fixed
module array instead of call-time allocations.  Compared through the C ABI with the pool
route of bybycu_tile_gemm (route TC) on back-to-back calls; the file is collected last so the
check also runs after every other test has used the library on the device."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from bybylang_b200 import _lib  # noqa: E402
from bybylang_b200 import gpubackend as gb  # noqa: E402

STATIC_SCRATCH_BYTES = 32 << 20


def _q4_case(M, K, N, seed):
    from bybylang_b200.formats import synthetic_q4b32, synthetic_x
    nib, sc = synthetic_q4b32(N, K, seed=seed, device="cuda:0")
    w = gb.Q4B32Weights(nib, sc, device="cuda:0")
    x = synthetic_x(M, K, seed=seed + 1, device="cuda:0")
    return w, x


def _noalloc(w, x, out):
    M, K = x.shape
    rc = _lib.load().bybycu_tile_gemm_noalloc(
        M, K, w.N, C.c_void_p(x.data_ptr()), _lib.DT_BF16, x.numel(), C.c_void_p(w.packed.data_ptr()),
        w.packed.numel(), w.scale_base, C.c_void_p(out.data_ptr()),
        _lib.DT_BF16 if out.dtype == torch.bfloat16 else _lib.DT_F32, out.numel(), None)
    assert rc == 0, _lib.last_error()[1]


def _pool(w, x, out):
    M, K = x.shape
    rc = _lib.load().bybycu_tile_gemm(
        2, M, K, w.N, C.c_void_p(x.data_ptr()), _lib.DT_BF16, x.numel(), C.c_void_p(w.packed.data_ptr()),
        w.packed.numel(), w.scale_base, None, 0, 0, C.c_void_p(out.data_ptr()),
        _lib.DT_BF16 if out.dtype == torch.bfloat16 else _lib.DT_F32, out.numel(), _lib.ROUTE_TC, None)
    assert rc == 0, _lib.last_error()[1]


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,dtype", [(300, 1024, 384, torch.float32), (2048, 4096, 4096, torch.bfloat16),
                                         (4096, 4096, 1024, torch.float32)])
def test_noalloc_matches_pool_route_on_two_calls_in_a_row(M, K, N, dtype):
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    cases = [_q4_case(M, K, N, seed=21), _q4_case(M, K, N, seed=57)]
    got = [torch.full((M, N), float("nan"), dtype=dtype, device="cuda:0") for _ in cases]
    for (w, x), o in zip(cases, got):      # back to back on one stream, no sync in between
        _noalloc(w, x, o)
    want = [torch.empty((M, N), dtype=dtype, device="cuda:0") for _ in cases]
    for (w, x), o in zip(cases, want):
        _pool(w, x, o)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    for g, r in zip(got, want):
        assert torch.equal(g, r)
    assert not torch.equal(got[0], got[1])


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch():
    """4097 x 4096 fp16 activations exceed the 32 MiB array: a range error before any launch."""
    M, K, N = 4097, 4096, 256
    assert M * K * 2 > STATIC_SCRATCH_BYTES
    buf = C.create_string_buffer(16)
    rc = _lib.load().bybycu_tile_gemm_noalloc(M, K, N, buf, _lib.DT_BF16, M * K, buf, N * K, N * K // 2, buf,
                                              _lib.DT_F32, M * N, None)
    assert rc == _lib.ERR_RANGE
    assert "32 MiB" in _lib.last_error()[1]


@pytest.mark.gpu
def test_noalloc_first_call_after_init_leaves_device_memory_unchanged():
    """bybycu_init loads the route's module (array and kernels) on the device, so the first
    no-alloc call after it must not change the device's free memory (cudaMemGetInfo)."""
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    M, K, N = 256, 1024, 512
    w, x = _q4_case(M, K, N, seed=5)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda:0")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(0)
    _noalloc(w, x, out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(0)
    assert _lib.device_error() == 0
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    assert torch.isfinite(out).all()
