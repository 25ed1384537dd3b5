"""The C-ABI boundary without a GPU: libbybycuda.so loads, exports every entry point that
include/bybycuda.h declares, the ctypes table matches, and the host-side checks (shapes,
ranges, formats, routes, shard ranges) answer with the reference's errors before any device
work."""
import ctypes as C
import os
import re

import pytest

from bybylang_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "bybycuda.h")).read()
    return sorted(set(re.findall(r"BYBYCU_API\s+int\s+(bybycu_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header disagree"
    # the exported dynamic symbols are exactly the ABI (everything else is hidden)
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l and "bybycu_" in l}
    assert exported == set(names)


def test_version_and_device_count():
    lib = _lib.load()
    assert lib.bybycu_version() == 1
    n = C.c_int(-1)
    assert lib.bybycu_device_count(C.byref(n)) == 0
    assert n.value >= 0


def _gemm(fmt=2, M=1, K=64, N=16, x_len=None, packed_len=None, scale_base=None, lut_len=0, out_len=None,
          x=1 << 20, packed=1 << 20, lut=None, out=1 << 20, x_dtype=1, out_dtype=0, route=0):
    lib = _lib.load()
    if x_len is None:
        x_len = M * K
    if out_len is None:
        out_len = M * N
    if scale_base is None:
        scale_base = N * K // 2
    if packed_len is None:
        packed_len = N * K // 2 + (N * K // 32) * (2 if fmt == 2 else 1) + (N * K * 2 if fmt == 1 else 0)
    return lib.bybycu_tile_gemm(fmt, M, K, N, C.c_void_p(x), x_dtype, x_len, C.c_void_p(packed), packed_len,
                                scale_base, C.c_void_p(lut), lut_len, 0, C.c_void_p(out), out_dtype, out_len,
                                route, None)


@pytest.mark.parametrize("kw,code,msg", [
    (dict(fmt=3), _lib.ERR_SHAPE, "weight format 3 is not supported"),
    (dict(K=48), _lib.ERR_SHAPE, "unsupported tile GEMM shape K=48"),
    (dict(N=0), _lib.ERR_SHAPE, "unsupported tile GEMM shape"),
    (dict(M=0), _lib.ERR_SHAPE, "row count"),
    (dict(x_len=10), _lib.ERR_RANGE, "input out of range"),
    (dict(out_len=3), _lib.ERR_RANGE, "input out of range"),
    (dict(packed_len=100), _lib.ERR_RANGE, "input out of range"),
    (dict(scale_base=513), _lib.ERR_SHAPE, "even byte"),
    (dict(fmt=0, lut=1 << 20, lut_len=271), _lib.ERR_RANGE, "input out of range"),
    (dict(fmt=0), _lib.ERR_ARGS, "slot is missing"),
    (dict(x=0), _lib.ERR_ARGS, "slot is missing"),
    (dict(x_dtype=7), _lib.ERR_ARGS, "F32 or BF16"),
    (dict(route=9), _lib.ERR_ARGS, "unknown route"),
    (dict(fmt=0, lut=1 << 20, lut_len=272, route=1), _lib.ERR_SHAPE, "GEMV route needs format 2"),
])
def test_tile_gemm_rejects_before_device_work(kw, code, msg):
    rc = _gemm(**kw)
    assert rc == code
    got_code, got_msg = _lib.last_error()
    assert got_code == code and msg in got_msg, got_msg


def test_route_table():
    from bybylang_b200.gpubackend import route_for
    assert route_for(2, 1, 4096, 11008) == _lib.ROUTE_GEMV
    assert route_for(2, 16, 4096, 11008) == _lib.ROUTE_GEMV
    assert route_for(1, 1, 4096, 4096) == _lib.ROUTE_SIMT
    assert route_for(0, 1, 4096, 4096) == _lib.ROUTE_SIMT


def test_init_without_device_fails_loudly():
    lib = _lib.load()
    n = C.c_int(0)
    lib.bybycu_device_count(C.byref(n))
    if n.value:
        pytest.skip("a device is present")
    assert lib.bybycu_init(0) == _lib.ERR_NODEV
    from bybylang_b200 import gpubackend as gb
    with pytest.raises(_lib.BybyCudaError):
        gb.detectBackend()


def test_vm_rejects_foreign_programs():
    lib = _lib.load()
    err = C.create_string_buffer(128)
    code = (C.c_uint32 * 3)(0x13, 0, 0x01)   # OP_LOAD_CONST ... HALT: not this path's program
    rc = lib.bybycu_vm_run_slots(code, 3, C.c_void_p(1 << 20), 16, None, 0, None, 0, None, 0, 128, 64, 128,
                                 err, 128, None)
    assert rc == _lib.ERR_PROGRAM and b"tile GEMM" in err.value
    bad = (C.c_uint32 * 16)(0xB0, 0, 64, 16, 512, 0, 0xB1, 0xB4, 0xB2, 0xB5, 0x50, 0xB6, 0x50, 0xB3, 0xB7, 0x01)
    rc = lib.bybycu_vm_run_slots(bad, 16, C.c_void_p(1 << 20), 16, C.c_void_p(1 << 20), 1024,
                                 C.c_void_p(1 << 20), 272, None, 0, 128, 64, 128, err, 128, None)
    assert rc == _lib.ERR_PROGRAM and b"K loop" in err.value
    rc = lib.bybycu_vm_run_slots(bad, 16, C.c_void_p(1 << 20), 16, None, 0, None, 0, None, 0, 0, 64, 128, err, 128,
                                 None)
    assert rc == _lib.ERR_ARGS and err.value == b"invalid CUDA VM arguments"


def test_session_order_errors():
    lib = _lib.load()
    assert lib.bybycu_session_end() == _lib.ERR_SESSION
    assert lib.bybycu_session_q4b32_gemm(None, None, None, 1, 64, 16, 1) == _lib.ERR_SESSION


def test_tuned_plan_table_host_checks(monkeypatch):
    """The plan table and the tuner's argument checks answer before any device call."""
    lib = _lib.load()
    assert lib.bybycu_plan_clear() == 0
    n, d = C.c_int(-1), C.c_int64(-1)
    assert lib.bybycu_tuning_stats(C.byref(n), C.byref(d)) == 0 and (n.value, d.value) == (0, 0)
    good = _lib.Plan(route=_lib.ROUTE_GEMV, variant=-1, stages=0, ms=0.0, name=b"x")
    assert lib.bybycu_plan_set(7, 2, 0, 1, 64, 16, 0, 0, good) == _lib.ERR_ARGS
    assert lib.bybycu_plan_set(_lib.OP_TILE_GEMM, 2, 0, 0, 64, 16, 0, 0, good) == _lib.ERR_SHAPE
    for bad in (dict(route=_lib.ROUTE_AUTO), dict(variant=-2), dict(stages=9)):
        p = _lib.Plan(route=bad.get("route", _lib.ROUTE_GEMV), variant=bad.get("variant", -1),
                      stages=bad.get("stages", 0), ms=0.0, name=b"bad")
        assert lib.bybycu_plan_set(_lib.OP_TILE_GEMM, 2, 0, 1, 64, 16, 0, 0, p) == _lib.ERR_ARGS, bad
    prepared = C.c_int(-1)
    vp = C.c_void_p(1 << 20)
    assert lib.bybycu_prepare_q4_tuned(vp, vp, vp, 1, 64, 16, 32, 2, None) == _lib.ERR_ARGS
    assert lib.bybycu_prepare_q4_tuned(vp, vp, vp, 1, 64, 16, 32, 1, C.byref(prepared)) == _lib.ERR_SHAPE
    assert prepared.value == 0
    assert lib.bybycu_prepare_tile_gemm_tuned(5, 0, 1, 64, 16, vp, 1 << 20, 512, C.byref(prepared)) == _lib.ERR_ARGS
    assert lib.bybycu_prepare_tile_gemm_tuned(2, 7, 1, 64, 16, vp, 1 << 20, 512, C.byref(prepared)) == _lib.ERR_ARGS
    assert lib.bybycu_prepare_tile_gemm_tuned(2, 0, 1, 64, 16, vp, 100, 512, C.byref(prepared)) == _lib.ERR_RANGE
    # switched off: answered without a device
    monkeypatch.setenv("BYBY_Q4_TUNED", "0")
    prepared.value = -1
    assert lib.bybycu_prepare_q4_tuned(vp, vp, vp, 1, 64, 16, 32, 2, C.byref(prepared)) == 0
    assert prepared.value == 0
    assert lib.bybycu_prepare_tile_gemm_tuned(2, 1, 1, 64, 16, vp, 1 << 20, 512, C.byref(prepared)) == 0
    assert prepared.value == 0
