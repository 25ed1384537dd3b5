"""ctypes binding of libbybycuda.so (include/bybycuda.h).

The library is built in-tree (``bybylang_b200/libbybycuda.so``, see ``build.py``).  There is
no CPU fallback anywhere in this package: if the library is missing, cannot be loaded, or a
call fails, a ``BybyCudaError`` is raised.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbybycuda.so")

# status codes
OK = 0
ERR_ARGS = -1
ERR_SHAPE = -2
ERR_RANGE = -3
ERR_CUDA = -4
ERR_NODEV = -5
ERR_PROGRAM = -6
ERR_DEVICE = -7
ERR_SESSION = -8
ERR_PARITY = -9

FMT_FP4KM = 0
FMT_F16 = 1
FMT_Q4B32 = 2
DT_F32 = 0
DT_BF16 = 1
ROUTE_AUTO = 0
ROUTE_GEMV = 1
ROUTE_TC = 2
ROUTE_SIMT = 3
ROUTE_TC_FP16W = 4
ROUTE_NAMES = {ROUTE_AUTO: "auto", ROUTE_GEMV: "gemv", ROUTE_TC: "tc", ROUTE_SIMT: "simt",
               ROUTE_TC_FP16W: "tc-fp16w"}


OP_TILE_GEMM = 0
OP_MATMUL_Q4 = 1


class Plan(C.Structure):
    """bybycu_plan: a tuned route and its launch knobs."""
    _fields_ = [("route", C.c_int32), ("variant", C.c_int32), ("stages", C.c_int32), ("ms", C.c_float),
                ("name", C.c_char * 32)]

    def __repr__(self) -> str:
        return (f"Plan({self.name.decode()!r}, route={ROUTE_NAMES.get(self.route, self.route)}, "
                f"variant={self.variant}, stages={self.stages}, ms={self.ms:.4f})")


class TensorInfo(C.Structure):
    """bybycu_tensor_info: one tensor of a checkpoint index."""
    _fields_ = [("name", C.c_char * 256), ("name_len", C.c_int32), ("kind", C.c_int32), ("rank", C.c_int32),
                ("scales", C.c_int32), ("shape", C.c_int64 * 8), ("offset", C.c_int64), ("bytes", C.c_int64),
                ("scale_offset", C.c_int64), ("group_size", C.c_int32), ("eb", C.c_int32), ("mb", C.c_int32),
                ("dtype", C.c_char * 16)]


class BybyCudaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[cuda] {message} (status {code})")
        self.code = code


_vp, _i32, _i64, _u32 = C.c_void_p, C.c_int, C.c_int64, C.c_uint32

# name -> argument types (every function returns int)
SIGNATURES = {
    "bybycu_version": [],
    "bybycu_last_error": [C.c_char_p, _i32],
    "bybycu_device_count": [C.POINTER(_i32)],
    "bybycu_init": [_i32],
    "bybycu_malloc": [C.POINTER(_vp), _i64],
    "bybycu_free": [_vp],
    "bybycu_upload": [_vp, _vp, _i64, _vp],
    "bybycu_download": [_vp, _vp, _i64, _vp],
    "bybycu_memset": [_vp, _i32, _i64, _vp],
    "bybycu_stream_create": [C.POINTER(_vp)],
    "bybycu_stream_destroy": [_vp],
    "bybycu_synchronize": [_vp],
    "bybycu_device_error": [C.POINTER(_i32)],
    "bybycu_tile_gemm": [_i32, _i32, _i32, _i32, _vp, _i32, _i64, _vp, _i64, _i64, _vp, _i64, _i64,
                         _vp, _i32, _i64, _i32, _vp],
    "bybycu_tile_gemm_host": [_i32, _i32, _i32, _i32, _vp, _i32, _vp, _i64, _i64, _vp, _i64, _i64,
                              _vp, _i32, _vp, _vp, _i32, _vp],
    "bybycu_tile_gemm_noalloc": [_i32, _i32, _i32, _vp, _i32, _i64, _vp, _i64, _i64, _vp, _i32, _i64, _vp],
    "bybycu_dequant": [_i32, _i32, _i32, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp],
    "bybycu_route_for": [_i32, _i32, _i32, _i32, _i32, C.POINTER(_i32)],
    "bybycu_vm_run_slots": [C.POINTER(_u32), _i32, _vp, _i32, _vp, _i32, _vp, _i32, _vp, _i32,
                            _i32, _i32, _i32, C.c_char_p, _i32, _vp],
    "bybycu_matmul_q4": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp],
    "bybycu_session_matmul_q4": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32],
    "bybycu_matmul_q4_fused": [_i32, _vp, _i32, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_i32),
                               C.POINTER(_vp), _vp, _vp, C.c_float, _i32, _i32, _i32, _vp],
    "bybycu_session_matmul_q4_fused": [_i32, _vp, _i32, C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp),
                                       C.POINTER(_i32), C.POINTER(_vp), _vp, _vp, C.c_float, _i32, _i32, _i32],
    "bybycu_session_begin": [],
    "bybycu_session_end": [],
    "bybycu_session_upload": [_vp, _i64, C.POINTER(_vp)],
    "bybycu_session_alloc_scratch": [_i64, C.POINTER(_vp)],
    "bybycu_session_read": [_vp, _vp, _i64],
    "bybycu_session_free": [_vp],
    "bybycu_session_fp4_gemm": [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32],
    "bybycu_session_f16_gemm": [_vp, _vp, _vp, _i32, _i32, _i32, _i32],
    "bybycu_session_q4b32_gemm": [_vp, _vp, _vp, _i32, _i32, _i32, _i32],
    "bybycu_tile_gemm_ready": [_i32, _i32, C.POINTER(_i32)],
    "bybycu_ipc_handle": [_vp, C.c_char_p, C.POINTER(_i64)],
    "bybycu_ipc_open": [C.c_char_p, _i64, C.POINTER(_vp)],
    "bybycu_ipc_close": [_vp],
    "bybycu_shard_range": [_i32, _i32, _i32, _i32, C.POINTER(_i32), C.POINTER(_i32)],
    "bybycu_tile_gemm_allgather": [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _i32, _vp, _i64, _i64,
                                   _vp, _i64, _i64, _vp, C.POINTER(_vp), C.POINTER(C.POINTER(_u32)),
                                   _i32, _i32, _u32, _vp],
    "bybycu_tile_gemm_allgather_split": [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _i32, _vp, _i64, _i64,
                                         _vp, _i64, _i64, _vp, C.POINTER(_vp), C.POINTER(C.POINTER(_u32)),
                                         _i32, _i32, _u32, _vp],
    "bybycu_allgather_wait": [C.POINTER(C.POINTER(_u32)), _i32, _i32, _u32, _vp],
    "bybycu_prepare_q4_tuned": [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, C.POINTER(_i32)],
    "bybycu_prepare_tile_gemm_tuned": [_i32, _i32, _i32, _i32, _i32, _vp, _i64, _i64, C.POINTER(_i32)],
    "bybycu_plan_get": [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, C.POINTER(Plan), C.POINTER(_i32)],
    "bybycu_plan_set": [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, C.POINTER(Plan)],
    "bybycu_plan_clear": [],
    "bybycu_tuning_stats": [C.POINTER(_i32), C.POINTER(_i64)],
    "bybycu_tune_cache_path": [C.c_char_p, _i32],
    "bybycu_map_file": [C.c_char_p, C.POINTER(_vp), C.POINTER(_i64), C.POINTER(_vp)],
    "bybycu_unmap_file": [_vp],
    "bybycu_upload_host_range": [_vp, _vp, _i64],
    "bybycu_session_upload_ptr": [_vp, _i64, C.POINTER(_vp)],
    "bybycu_fingerprint": [_vp, _i64, C.c_char_p, _i32],
    "bybycu_checkpoint_index": [C.c_char_p, C.POINTER(TensorInfo), _i32, C.POINTER(_i32)],
}

_lib = None


def load():
    """The loaded library; raises BybyCudaError when it is absent or broken."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise BybyCudaError(ERR_NODEV, f"{LIB_PATH} is missing: run `python -m bybylang_b200.build` "
                                           "(nvcc, sm_100a); there is no CPU fallback")
        lib = C.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = C.c_int
        if lib.bybycu_version() != 1:
            raise BybyCudaError(ERR_ARGS, "libbybycuda.so ABI version mismatch")
        _lib = lib
    return _lib


def last_error() -> tuple[int, str]:
    buf = C.create_string_buffer(512)
    code = load().bybycu_last_error(buf, 512)
    return code, buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        code, msg = last_error()
        raise BybyCudaError(rc, msg or f"status {rc}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def device_error() -> int:
    v = C.c_int(0)
    call("bybycu_device_error", C.byref(v))
    return v.value
