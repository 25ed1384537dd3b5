"""TEST INFRASTRUCTURE ONLY: numpy bindings of the CPU oracle.

Two libraries are wrapped here:

* ``libq4_oracle.so`` - the C restatement (``q4_oracle.c``) of the tile-GEMM arithmetic,
  the reference tests' seeded generators and the format converters;
* ``_ref/libref_oracle.so`` - the reference's own CPU C (``backends/cpu/cpu_vm.c`` and
  ``cpu_kernels.c``, compiled unchanged) behind the exporting shim ``ref_shim.c``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module, and only to check or time the reference arithmetic; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libq4_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_oracle.so")

OP_TILE_GEMM = 0xB0
OP_FP4_COOP_GEMM = 0xAC
OP_Q4_COOP_GEMM = 0xAA
OP_Q4_GEMV = 0xAB
OP_HALT = 0x01

_port = None
_ref = None


def reference_tree():
    """The reference project's source tree: BYBY_REFERENCE_TREE, else the `reference_path` that
    BASELINE.json at the repository root records; None when neither names an existing tree."""
    tree = os.environ.get("BYBY_REFERENCE_TREE")
    if not tree:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                tree = json.load(f).get("reference_path")
        except (OSError, ValueError):
            tree = None
    return tree if tree and os.path.isdir(tree) else None


def build() -> None:
    """Compile the restatement and, when the reference tree is present, the reference C."""
    tree = reference_tree()
    subprocess.run(["make", "-s", "-C", HERE] + ([f"REF={tree}"] if tree else []), check=True)


def _ptr(a: np.ndarray, ct=C.c_void_p):
    return a.ctypes.data_as(ct)


def port():
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build()
        lib = C.CDLL(PORT_SO)
        lib.q4o_xorshift32.restype = C.c_uint32
        lib.q4o_f32_to_f16.restype = C.c_uint16
        lib.q4o_f32_to_f16.argtypes = [C.c_float]
        lib.q4o_f16_to_f32.restype = C.c_float
        lib.q4o_f16_to_f32.argtypes = [C.c_uint16]
        lib.q4o_f32_to_bf16.restype = C.c_uint16
        lib.q4o_f32_to_bf16.argtypes = [C.c_float]
        lib.q4o_q4b32_to_fp4km.restype = C.c_int
        _port = lib
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own C; raises when oracle/_ref was never built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} is missing: build it where the reference tree exists")
        lib = C.CDLL(REF_SO)
        lib.refo_vm_run_slots.restype = C.c_int
        lib.refo_tile_gemm_mt.restype = C.c_int
        lib.refo_tile_gemm_mt.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                          C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                          C.c_int, C.c_char_p, C.c_int]
        _ref = lib
    return _ref


# --------------------------------------------------------------------------------------
# Generators (the reference tests' own, restated)
# --------------------------------------------------------------------------------------

class Xorshift32:
    """The reference test's global generator state (tests/t_fp4_tile_gemm.nim:30-33)."""

    SEED = 2463534242

    def __init__(self, seed: int = SEED):
        self.state = C.c_uint32(seed)

    def make_fp4_case(self, M: int, K: int, N: int):
        x = np.zeros(M * K, np.float32)
        packed = np.zeros(N * (K // 2) + N * (K // 32), np.uint8)
        table = np.zeros(272, np.float32)
        port().q4o_make_fp4_case(C.byref(self.state), M, K, N, _ptr(x), _ptr(packed), _ptr(table))
        return x.reshape(M, K), packed, table

    def make_f16_case(self, M: int, K: int, N: int):
        x = np.zeros(M * K, np.float32)
        w = np.zeros(N * K, np.float32)
        halves = np.zeros(N * K, np.uint16)
        port().q4o_make_f16_case(C.byref(self.state), M, K, N, _ptr(x), _ptr(w), _ptr(halves))
        return x.reshape(M, K), w.reshape(N, K), halves.reshape(N, K)


def reference_test_cases():
    """The five FP4-KM and five FP16 cases of tests/t_fp4_tile_gemm.nim:147-148,207-208,
    drawn in the reference test's order from one generator."""
    g = Xorshift32()
    fp4 = [(M, K, N) + g.make_fp4_case(M, K, N)
           for (M, K, N) in [(1, 64, 16), (5, 128, 96), (20, 64, 72), (37, 128, 130), (70, 96, 64)]]
    f16 = [(M, K, N) + g.make_f16_case(M, K, N)
           for (M, K, N) in [(1, 64, 16), (5, 128, 96), (20, 64, 72), (37, 128, 130), (70, 192, 64)]]
    return fp4, f16


def gate_fp4(M=37, K=128, N=80):
    x = np.zeros(M * K, np.float32)
    packed = np.zeros(N * (K // 2) + N * (K // 32), np.uint8)
    table = np.zeros(272, np.float32)
    port().q4o_make_gate_fp4(M, K, N, _ptr(x), _ptr(packed), _ptr(table))
    return x.reshape(M, K), packed, table


def gate_f16(M=37, K=128, N=80):
    x = np.zeros(M * K, np.float32)
    w = np.zeros(N * K, np.float32)
    halves = np.zeros(N * K, np.uint16)
    port().q4o_make_gate_f16(M, K, N, _ptr(x), _ptr(w), _ptr(halves))
    return x.reshape(M, K), w.reshape(N, K), halves.reshape(N, K)


def gen_q4b32(N: int, K: int, seed: int = Xorshift32.SEED):
    """Q4B32 weights of the benchmark configurations: packed nibbles [N, K/2] in the tile
    layout and fp16 scale bits [N, K/32]."""
    packed = np.zeros(N * (K // 2), np.uint8)
    scales = np.zeros(N * (K // 32), np.uint16)
    port().q4o_gen_q4b32(C.c_uint32(seed), N, K, _ptr(packed), _ptr(scales))
    return packed.reshape(N, K // 2), scales.reshape(N, K // 32)


def gen_x_bf16(M: int, K: int, seed: int = Xorshift32.SEED + 2):
    x = np.zeros(M * K, np.uint16)
    port().q4o_gen_x_bf16(C.c_uint32(seed), M, K, _ptr(x))
    return x.reshape(M, K)


def gen_x_f32(M: int, K: int, seed: int = Xorshift32.SEED + 2):
    x = np.zeros(M * K, np.float32)
    port().q4o_gen_x_f32(C.c_uint32(seed), M, K, _ptr(x))
    return x.reshape(M, K)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    return bits.astype(np.uint16).view(np.float16).astype(np.float32)


# --------------------------------------------------------------------------------------
# Port references
# --------------------------------------------------------------------------------------

def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def tile_gemm_fp4km(x, packed, table, M, K, N, scale_base=None):
    scale_base = N * (K // 2) if scale_base is None else scale_base
    out = np.zeros(M * N, np.float32)
    x = _f32(x)
    port().q4o_tile_gemm_fp4km(_ptr(x), _ptr(np.ascontiguousarray(packed)), C.c_int64(scale_base),
                               _ptr(_f32(table)), M, K, N, _ptr(out))
    return out.reshape(M, N)


def tile_gemm_reference(x, packed, table, M, K, N, scale_base=None):
    scale_base = N * (K // 2) if scale_base is None else scale_base
    out = np.zeros(M * N, np.float32)
    port().q4o_tile_gemm_reference(_ptr(_f32(x)), _ptr(np.ascontiguousarray(packed)),
                                   C.c_int64(scale_base), _ptr(_f32(table)), M, K, N, _ptr(out))
    return out.reshape(M, N)


def tile_gemm_f16(x, halves, M, K, N):
    out = np.zeros(M * N, np.float32)
    port().q4o_tile_gemm_f16(_ptr(_f32(x)), _ptr(np.ascontiguousarray(halves, np.uint16)), M, K, N,
                             _ptr(out))
    return out.reshape(M, N)


def tile_gemm_q4b32(x, packed, scales, M, K, N, threads: int = 1):
    out = np.zeros(M * N, np.float32)
    args = (_ptr(_f32(x)), _ptr(np.ascontiguousarray(packed, np.uint8)),
            _ptr(np.ascontiguousarray(scales, np.uint16)), M, K, N, _ptr(out))
    if threads > 1:
        port().q4o_tile_gemm_q4b32_mt(*args, threads)
    else:
        port().q4o_tile_gemm_q4b32(*args)
    return out.reshape(M, N)


def tile_gemm_q4b32_f64(x, packed, scales, M, K, N):
    out = np.zeros(M * N, np.float64)
    port().q4o_tile_gemm_q4b32_f64(_ptr(_f32(x)), _ptr(np.ascontiguousarray(packed, np.uint8)),
                                   _ptr(np.ascontiguousarray(scales, np.uint16)), M, K, N, _ptr(out))
    return out.reshape(M, N)


def matmul_q4_asym(a, wq, scales, zeros, M, K, N, group_size=32):
    out = np.zeros(M * N, np.float32)
    port().q4o_matmul_q4_asym(_ptr(_f32(a)), _ptr(np.ascontiguousarray(wq, np.uint8)),
                              _ptr(_f32(scales)), _ptr(_f32(zeros)), M, K, N, group_size,
                              K // group_size, _ptr(out))
    return out.reshape(M, N)


def dequant_q4b32(packed, scales, N, K):
    w = np.zeros(N * K, np.float32)
    port().q4o_dequant_q4b32(_ptr(np.ascontiguousarray(packed, np.uint8)),
                             _ptr(np.ascontiguousarray(scales, np.uint16)), N, K, _ptr(w))
    return w.reshape(N, K)


def dequant_fp4km(packed, table, N, K, scale_base=None):
    scale_base = N * (K // 2) if scale_base is None else scale_base
    w = np.zeros(N * K, np.float32)
    port().q4o_dequant_fp4km(_ptr(np.ascontiguousarray(packed, np.uint8)), C.c_int64(scale_base),
                             _ptr(_f32(table)), N, K, _ptr(w))
    return w.reshape(N, K)


def q4b32_to_asym(packed, scales, N, K):
    bpr = (K + 1) // 2
    wq = np.zeros(N * bpr, np.uint8)
    sc = np.zeros(N * (K // 32), np.float32)
    zp = np.zeros(N * (K // 32), np.float32)
    port().q4o_q4b32_to_asym(_ptr(np.ascontiguousarray(packed, np.uint8)),
                             _ptr(np.ascontiguousarray(scales, np.uint16)), N, K, _ptr(wq), _ptr(sc),
                             _ptr(zp))
    return wq, sc, zp


def q4b32_to_fp4km(packed, scales, N, K):
    """Returns (packed FP4-KM blob, 272-float table) or None with more than 256 scales."""
    out = np.zeros(N * (K // 2) + N * (K // 32), np.uint8)
    table = np.zeros(272, np.float32)
    n = port().q4o_q4b32_to_fp4km(_ptr(np.ascontiguousarray(packed, np.uint8)),
                                  _ptr(np.ascontiguousarray(scales, np.uint16)), N, K, _ptr(out),
                                  _ptr(table))
    return None if n < 0 else (out, table)


# --------------------------------------------------------------------------------------
# The reference's own C
# --------------------------------------------------------------------------------------

def fp4_tile_program(M, K, N, scale_base, lut_base=0, fmt=0):
    """buildFp4TileGemmProgram (micro_kernel/session_vm.nim:383-399) as raw words."""
    return np.array([OP_TILE_GEMM | (fmt << 8), M, K, N, scale_base, lut_base,
                     0xB1, 0xB2, 0xB4, 0xB5, 0x50, 0xB6, 0x50, 0xB3, 0xB7, OP_HALT], np.uint32)


def f16_tile_program(M, K, N):
    """buildF16TileGemmProgram (session_vm.nim:401-416)."""
    return np.array([OP_TILE_GEMM | (1 << 8), M, K, N, 0, 0,
                     0xB1, 0xB2, 0xB4, 0xB8, 0x50, 0xB6, 0x50, 0xB3, 0xB7, OP_HALT], np.uint32)


def ref_vm_run_slots(code, mem_len, packed, lut, x, n_threads=128, tg_floats=64, tg_size=128):
    """nimf_cpu_vm_run_slots on the given slots; returns (rc, mem, err)."""
    code = np.ascontiguousarray(code, np.uint32).copy()
    mem = np.zeros(max(mem_len, 1), np.float32)
    packed = np.ascontiguousarray(packed, np.uint8)
    lut = _f32(lut)
    x = _f32(x).ravel()
    err = C.create_string_buffer(256)
    rc = ref().refo_vm_run_slots(_ptr(code), len(code), _ptr(mem), mem_len, _ptr(packed),
                                 len(packed), _ptr(lut), len(lut), _ptr(x), len(x), n_threads,
                                 tg_floats, tg_size, err, 256)
    return rc, mem[:mem_len], err.value.decode()


def ref_tile_gemm(x, packed, table, M, K, N, scale_base=None, threads: int = 1):
    """OP_TILE_GEMM format 0 through the reference CPU VM (column-sharded when threads > 1)."""
    scale_base = N * (K // 2) if scale_base is None else scale_base
    out = np.zeros(M * N, np.float32)
    packed = np.ascontiguousarray(packed, np.uint8)
    err = C.create_string_buffer(160)
    rc = ref().refo_tile_gemm_mt(_ptr(_f32(x)), _ptr(packed), len(packed), scale_base,
                                 _ptr(_f32(table)), M, K, N, _ptr(out), threads, err, 160)
    if rc != 0:
        raise RuntimeError("reference CPU VM: " + err.value.decode())
    return out.reshape(M, N)


def ref_matmul_q4(a, wq, scales, zeros, M, K, N, group_size=32, threads: int = 1):
    """nimf_cpu_matmul_q4 (column-sharded when threads > 1)."""
    out = np.zeros(M * N, np.float32)
    a = _f32(a)
    wq = np.ascontiguousarray(wq, np.uint8)
    sc, zp = _f32(scales), _f32(zeros)
    if threads > 1:
        ref().refo_matmul_q4_mt(_ptr(a), _ptr(wq), _ptr(sc), _ptr(zp), _ptr(out), M, K, N,
                                group_size, K // group_size, threads)
    else:
        ref().refo_matmul_q4(_ptr(a), _ptr(wq), _ptr(sc), _ptr(zp), _ptr(out), M, K, N, group_size,
                             K // group_size)
    return out.reshape(M, N)
