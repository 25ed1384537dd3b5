"""The `cuda` GpuBackend of BybyLang's operator API for the tile-GEMM path (gpubackend.nim),
implemented over libbybycuda.so.

What changes against the reference: ``parseBackend("cuda")`` returns a real ``gbCuda`` (the
reference remaps it to Vulkan, gpubackend.nim:107-121), the cuda path forces
``gForbidCpuFallback`` on, and every session op of this path runs hand-written sm_100a
kernels.  There is no Vulkan, Metal or CPU dispatch here: a failure raises (the
``handleGpuFailure`` policy with fallback forbidden, gpubackend.nim:80-105).

Besides the session API, two tensor-level entry points serve Python callers:
``tile_gemm`` (device tensors in, device tensor out, asynchronous on the current stream)
and ``Q4B32Weights`` (weights resident on the device, the residentUploadQ4 role).
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import BybyCudaError, call, check, load
from .session_vm import (TileFormatF16, TileFormatFp4Km, TileFormatQ4B32, VmProgram,
                         tileWeightBytes)


class GpuBackend(enum.IntEnum):
    """gpubackend.nim:55-57."""
    gbAuto = 0
    gbCpu = 1
    gbCuda = 2
    gbMetal = 3
    gbVulkan = 4

    def __str__(self) -> str:
        return {0: "auto", 1: "cpu", 2: "cuda", 3: "metal", 4: "vulkan"}[int(self)]


gForbidCpuFallback = False


def setForbidCpuFallback(forbid: bool) -> None:
    """gpubackend.nim:75-76.  The cuda path turns it on by itself and keeps it on."""
    global gForbidCpuFallback
    gForbidCpuFallback = bool(forbid)


def parseBackend(s: str) -> GpuBackend:
    """gpubackend.nim:107-114, with `cuda` a real backend."""
    v = s.strip().lower()
    table = {"cuda": GpuBackend.gbCuda, "metal": GpuBackend.gbMetal, "cpu": GpuBackend.gbCpu,
             "vulkan": GpuBackend.gbVulkan, "auto": GpuBackend.gbAuto}
    if v not in table:
        raise ValueError(f"unknown BybyLang backend: {s}")
    return table[v]


def normalizeBackend(b: GpuBackend) -> GpuBackend:
    """gpubackend.nim:116-121 without the cuda -> vulkan remap."""
    return b


def detectBackend() -> GpuBackend:
    """gbCuda when an sm_100 device is present; this package provides no other backend."""
    n = C.c_int(0)
    call("bybycu_device_count", C.byref(n))
    if n.value == 0:
        raise BybyCudaError(_lib.ERR_NODEV, "no CUDA device: this package has no CPU, Vulkan or Metal path")
    return GpuBackend.gbCuda


def _chosen(backend: GpuBackend) -> GpuBackend:
    b = detectBackend() if backend == GpuBackend.gbAuto else backend
    if b != GpuBackend.gbCuda:
        raise BybyCudaError(_lib.ERR_ARGS, f"backend '{b}' is not provided by bybylang_b200 (only 'cuda')")
    return b


_initialised: set = set()


def ensureGpuInit(backend: GpuBackend = GpuBackend.gbCuda, device: int | None = None) -> bool:
    """Selects the device (BYBY_CUDA_DEVICE, default 0) and forbids CPU fallback."""
    _chosen(backend)
    dev = int(os.environ.get("BYBY_CUDA_DEVICE", "0")) if device is None else device
    call("bybycu_init", dev)
    _initialised.add(dev)
    setForbidCpuFallback(True)
    return True


def handleGpuFailure(backend: GpuBackend, opName: str, e: Exception):
    """gpubackend.nim:80-105 with fallback forbidden on this path: always raises."""
    msg = f"[GPU] backend '{backend}' failed during '{opName}' ({e})"
    raise BybyCudaError(getattr(e, "code", _lib.ERR_CUDA),
                        msg + ". CPU fallback is forbidden (gForbidCpuFallback=true).") from e


# --------------------------------------------------------------------------------------
# Session API (gpubackend.nim:1042-2722)
# --------------------------------------------------------------------------------------

@dataclass
class CudaResidentTensor:
    """gpubackend.nim:23-27: a device pointer and its size (here in bytes)."""
    dptr: int = 0
    n: int = 0


@dataclass
class SessionHandle:
    kind: GpuBackend = GpuBackend.gbCuda
    cudaHandle: CudaResidentTensor = field(default_factory=CudaResidentTensor)

    @property
    def ptr(self) -> int:
        return self.cudaHandle.dptr


def sessionBegin(backend: GpuBackend) -> bool:
    _chosen(backend)
    if not _initialised:
        ensureGpuInit(backend)
    try:
        call("bybycu_session_begin")
    except BybyCudaError as e:
        handleGpuFailure(backend, "sessionBegin", e)
    return True


def sessionEnd(backend: GpuBackend) -> bool:
    _chosen(backend)
    try:
        call("bybycu_session_end")
    except BybyCudaError as e:
        handleGpuFailure(backend, "sessionEnd", e)
    return True


def sessionUpload(backend: GpuBackend, data) -> SessionHandle:
    """gpubackend.nim:1133: the bytes of `data` (float32 words or any array) on the device."""
    _chosen(backend)
    a = np.ascontiguousarray(data)
    h = C.c_void_p()
    call("bybycu_session_upload", a.ctypes.data_as(C.c_void_p), a.nbytes, C.byref(h))
    return SessionHandle(GpuBackend.gbCuda, CudaResidentTensor(h.value, a.nbytes))


def sessionAllocScratch(backend: GpuBackend, n: int) -> SessionHandle:
    _chosen(backend)
    h = C.c_void_p()
    call("bybycu_session_alloc_scratch", int(n), C.byref(h))
    return SessionHandle(GpuBackend.gbCuda, CudaResidentTensor(h.value, int(n) * 4))


def sessionRead(backend: GpuBackend, h: SessionHandle, n: int) -> np.ndarray:
    _chosen(backend)
    out = np.zeros(int(n), np.float32)
    call("bybycu_session_read", C.c_void_p(h.ptr), out.ctypes.data_as(C.c_void_p), int(n))
    return out


def sessionFree(backend: GpuBackend, h: SessionHandle) -> None:
    _chosen(backend)
    if h.ptr:
        call("bybycu_session_free", C.c_void_p(h.ptr))
    h.cudaHandle = CudaResidentTensor()


def _gemm(name: str, backend: GpuBackend, args, c: SessionHandle, M: int, N: int) -> bool:
    _chosen(backend)
    if not c.ptr:
        c.cudaHandle = sessionAllocScratch(backend, M * N).cudaHandle
    try:
        call(name, *args)
    except BybyCudaError as e:
        handleGpuFailure(backend, name, e)
    return True


def sessionFp4GemmTensorCore(backend, a: SessionHandle, w: SessionHandle, lut: SessionHandle,
                             c: SessionHandle, M: int, K: int, N: int) -> bool:
    """gpubackend.nim:1442-1449: FP4-KM tile GEMM on the tensor-core routes."""
    if not c.ptr:
        c.cudaHandle = sessionAllocScratch(backend, M * N).cudaHandle
    return _gemm("bybycu_session_fp4_gemm", backend,
                 (C.c_void_p(a.ptr), C.c_void_p(w.ptr), C.c_void_p(lut.ptr), C.c_void_p(c.ptr), M, K, N, 1),
                 c, M, N)


def sessionFp4GemmTiledEnc(backend, a: SessionHandle, w: SessionHandle, lut: SessionHandle,
                           c: SessionHandle, M: int, K: int, N: int) -> bool:
    """gpubackend.nim:1465-1473: the FP32 register-tile route."""
    if not c.ptr:
        c.cudaHandle = sessionAllocScratch(backend, M * N).cudaHandle
    return _gemm("bybycu_session_fp4_gemm", backend,
                 (C.c_void_p(a.ptr), C.c_void_p(w.ptr), C.c_void_p(lut.ptr), C.c_void_p(c.ptr), M, K, N, 0),
                 c, M, N)


def sessionF16GemmTile(backend, a: SessionHandle, w: SessionHandle, c: SessionHandle, M: int, K: int,
                       N: int, tensorCore: bool) -> bool:
    """gpubackend.nim:1475-1482."""
    if not c.ptr:
        c.cudaHandle = sessionAllocScratch(backend, M * N).cudaHandle
    return _gemm("bybycu_session_f16_gemm", backend,
                 (C.c_void_p(a.ptr), C.c_void_p(w.ptr), C.c_void_p(c.ptr), M, K, N, int(bool(tensorCore))),
                 c, M, N)


def sessionQ4B32Gemm(backend, a: SessionHandle, w: SessionHandle, c: SessionHandle, M: int, K: int,
                     N: int, tensorCore: bool = True) -> bool:
    """Format 2 (Q4B32) through the same session encoder shape."""
    if not c.ptr:
        c.cudaHandle = sessionAllocScratch(backend, M * N).cudaHandle
    return _gemm("bybycu_session_q4b32_gemm", backend,
                 (C.c_void_p(a.ptr), C.c_void_p(w.ptr), C.c_void_p(c.ptr), M, K, N, int(bool(tensorCore))),
                 c, M, N)


def sessionTileGemmReady(backend, f16: bool, tensorCore: bool, fmt: int | None = None) -> bool:
    """gpubackend.nim:1484-1488: the exact-data parity gate, once per process."""
    _chosen(backend)
    if not _initialised:
        ensureGpuInit(backend)
    f = fmt if fmt is not None else (TileFormatF16 if f16 else TileFormatFp4Km)
    r = C.c_int(0)
    call("bybycu_tile_gemm_ready", f, int(bool(tensorCore)), C.byref(r))
    return bool(r.value)


def sessionMicroVmEnc(backend, code, mem: SessionHandle, nThreads: int, tgFloats: int, tgSize: int,
                      packed: SessionHandle | None = None, lut: SessionHandle | None = None,
                      inp: SessionHandle | None = None) -> bool:
    """gpubackend.nim:1065-1081 for tile-GEMM / shape-op programs.  With only `mem` the slots
    alias it as in nimf_cpu_vm_run (cpu_vm.c:822-828); the optional slots bind u8, lut and
    input separately as nimf_cpu_vm_run_slots does."""
    _chosen(backend)
    words = np.ascontiguousarray(code.words if isinstance(code, VmProgram) else code, np.uint32)
    pk = packed if packed is not None else mem
    lt = lut if lut is not None else mem
    err = C.create_string_buffer(256)
    rc = load().bybycu_vm_run_slots(
        words.ctypes.data_as(C.POINTER(C.c_uint32)), len(words), C.c_void_p(mem.ptr), mem.cudaHandle.n // 4,
        C.c_void_p(pk.ptr), pk.cudaHandle.n, C.c_void_p(lt.ptr), lt.cudaHandle.n // 4,
        C.c_void_p(inp.ptr if inp is not None else 0), (inp.cudaHandle.n // 4) if inp is not None else 0,
        nThreads, tgFloats, tgSize, err, 256, None)
    if rc != 0:
        handleGpuFailure(GpuBackend.gbCuda, "sessionMicroVmEnc", BybyCudaError(rc, err.value.decode()))
    return True


# --------------------------------------------------------------------------------------
# Tensor-level entry points (torch device tensors; plumbing only - the math is the library's)
# --------------------------------------------------------------------------------------

def _ptr(t) -> C.c_void_p:
    return C.c_void_p(0 if t is None else t.data_ptr())


def _dtype_code(t) -> int:
    import torch
    if t.dtype == torch.float32:
        return _lib.DT_F32
    if t.dtype == torch.bfloat16:
        return _lib.DT_BF16
    raise BybyCudaError(_lib.ERR_ARGS, f"unsupported element type {t.dtype} (float32 or bfloat16)")


def _stream_ptr(stream) -> C.c_void_p:
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return C.c_void_p(s.cuda_stream)


def tile_gemm(fmt: int, x, packed, out, *, M: int, K: int, N: int, scale_base: int = 0, lut=None,
              lut_base: int = 0, route: int = _lib.ROUTE_AUTO, stream=None):
    """out[M, N] = x[M, K] * dequant(W)^T for one OP_TILE_GEMM on device tensors.

    x: float32/bfloat16 [M, K]; packed: uint8 weight slot; out: float32/bfloat16 [M, N];
    lut: float32 table slot (format 0).  Asynchronous on `stream` (default: current).
    Every tensor must be contiguous: the library addresses the slots as dense arrays."""
    for name, t in (("x", x), ("packed", packed), ("out", out), ("lut", lut)):
        if t is not None and not t.is_contiguous():
            raise BybyCudaError(_lib.ERR_ARGS, f"tile GEMM slot {name} must be contiguous")
    check(load().bybycu_tile_gemm(
        fmt, M, K, N, _ptr(x), _dtype_code(x), x.numel(), _ptr(packed), packed.numel() * packed.element_size(),
        scale_base, _ptr(lut), 0 if lut is None else lut.numel(), lut_base, _ptr(out), _dtype_code(out),
        out.numel(), route, _stream_ptr(stream)))
    return out


def route_for(fmt: int, M: int, K: int, N: int, x_dtype: int = _lib.DT_BF16) -> int:
    r = C.c_int(0)
    call("bybycu_route_for", fmt, M, K, N, x_dtype, C.byref(r))
    return r.value


def dequant(fmt: int, packed, w_out, *, K: int, N: int, scale_base: int = 0, lut=None, lut_base: int = 0,
            stream=None):
    check(load().bybycu_dequant(fmt, K, N, _ptr(packed), packed.numel() * packed.element_size(), scale_base,
                                _ptr(lut), 0 if lut is None else lut.numel(), lut_base, _ptr(w_out),
                                _stream_ptr(stream)))
    return w_out


class Q4B32Weights:
    """Q4B32 weights resident on one device (the residentUploadQ4 role,
    gpubackend.nim:2883-2919): one uint8 slot holding the nibbles [N, K/2] in the tile layout
    followed by the fp16 scales [N, K/32] at byte ``scale_base`` (16-byte aligned)."""

    def __init__(self, nibbles, scales, device=None):
        import torch
        nib = torch.as_tensor(nibbles)
        sc = torch.as_tensor(scales)
        if nib.dtype != torch.uint8 or nib.dim() != 2:
            raise BybyCudaError(_lib.ERR_ARGS, "nibbles must be uint8 [N, K/2]")
        self.N, half = nib.shape
        self.K = half * 2
        if self.K % 32 or tuple(sc.shape) != (self.N, self.K // 32):
            raise BybyCudaError(_lib.ERR_SHAPE, f"unsupported tile GEMM shape K={self.K} N={self.N}")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        nb = self.N * half
        self.scale_base = (nb + 15) // 16 * 16
        self.packed = torch.zeros(self.scale_base + sc.numel() * 2, dtype=torch.uint8, device=dev)
        self.packed[:nb].copy_(nib.reshape(-1).to(dev))
        s16 = sc.reshape(-1).view(torch.int16) if sc.dtype in (torch.float16, torch.int16) else \
            sc.reshape(-1).to(torch.float16).view(torch.int16)
        self.packed[self.scale_base:].copy_(s16.to(dev).view(torch.uint8))

    def matmul(self, x, out=None, *, route: int = _lib.ROUTE_AUTO, stream=None):
        """out[M, N] = x[M, K] * W^T (sessionMatmulQ4's role for this format)."""
        import torch
        M = x.shape[0]
        if out is None:
            out = torch.empty(M, self.N, dtype=torch.float32, device=x.device)
        return tile_gemm(TileFormatQ4B32, x, self.packed, out, M=M, K=self.K, N=self.N,
                         scale_base=self.scale_base, route=route, stream=stream)

    def prepare(self, M: int = 1, x_dtype: int = _lib.DT_BF16) -> bool:
        """Autotunes the automatic route for M rows of x_dtype activations (residentPrepareQ4's
        role)."""
        return prepareTileGemmTuned(TileFormatQ4B32, self.packed, M=M, K=self.K, N=self.N,
                                    scale_base=self.scale_base, x_dtype=x_dtype)


# --------------------------------------------------------------------------------------
# Asymmetric Q4 (matmul_q4: gpubackend.nim:806-843, 2871-3060; cpu_kernels_impl.inc:293-319)
# --------------------------------------------------------------------------------------

@dataclass
class ResidentWeightHandle:
    """gpubackend.nim's ResidentWeightHandle for the CUDA backend: the packed nibbles
    [N, (K+1)/2] (even k in the low nibble) and the fp32 scales and zero points
    [N, nGroupsPerRow], uploaded once as three session handles."""
    kind: GpuBackend = GpuBackend.gbCuda
    wq: SessionHandle = field(default_factory=SessionHandle)
    scales: SessionHandle = field(default_factory=SessionHandle)
    zeros: SessionHandle = field(default_factory=SessionHandle)
    k: int = 0
    n: int = 0
    groupSize: int = 0
    nGroupsPerRow: int = 0


def _q4_shape_check(n_wq: int, n_scales: int, n_zeros: int, k: int, n: int, groupSize: int,
                    nGroupsPerRow: int) -> None:
    need = (k + groupSize - 1) // groupSize if groupSize > 0 else 1
    if k <= 0 or n <= 0 or nGroupsPerRow < need:
        raise BybyCudaError(_lib.ERR_SHAPE, f"unsupported matmul_q4 shape K={k} N={n} groups={nGroupsPerRow}")
    if n_wq < n * ((k + 1) // 2) or n_scales < n * nGroupsPerRow or n_zeros < n * nGroupsPerRow:
        raise BybyCudaError(_lib.ERR_RANGE, "matmul_q4: a weight slot is smaller than the shape needs")


def _q4_check(wq, scales, zeros, k: int, n: int, groupSize: int, nGroupsPerRow: int):
    wq = np.ascontiguousarray(wq, np.uint8).reshape(-1)
    scales = np.ascontiguousarray(scales, np.float32).reshape(-1)
    zeros = np.ascontiguousarray(zeros, np.float32).reshape(-1)
    _q4_shape_check(wq.size, scales.size, zeros.size, k, n, groupSize, nGroupsPerRow)
    return wq, scales, zeros


def residentUploadQ4(backend: GpuBackend, wq, scales, zeros, k: int, n: int, groupSize: int,
                     nGroupsPerRow: int) -> ResidentWeightHandle:
    """gpubackend.nim:2883-2919: the weights on the device once, at model load."""
    _chosen(backend)
    if not _initialised:
        ensureGpuInit(backend)
    wq, scales, zeros = _q4_check(wq, scales, zeros, k, n, groupSize, nGroupsPerRow)
    return ResidentWeightHandle(GpuBackend.gbCuda, sessionUpload(backend, wq), sessionUpload(backend, scales),
                                sessionUpload(backend, zeros), k, n, groupSize, nGroupsPerRow)


def residentPrepareQ4(w: ResidentWeightHandle, M: int = 1) -> bool:
    """gpubackend.nim:2871-2881 -> vulkanPrepareQ4Tuned (q4_autotune.nim:387-543): autotunes
    the plan that sessionMatmulQ4 / gpuMatmulQ4 use for these weights at M rows (M = 1 the
    decode plan, M > 1 the plan of M's power-of-two class), through the library's
    parity-gated candidate timing and its JSON plan cache.  True when a plan is installed;
    False when there is nothing to choose, tuning is switched off (BYBY_Q4_TUNED=0 or
    BYBY_GPU_AUTOTUNE=0) or the handle is not a CUDA one."""
    if w.kind != GpuBackend.gbCuda or not w.wq.ptr or M <= 0:
        return False
    prepared = C.c_int(0)
    call("bybycu_prepare_q4_tuned", C.c_void_p(w.wq.ptr), C.c_void_p(w.scales.ptr), C.c_void_p(w.zeros.ptr),
         int(M), w.k, w.n, w.groupSize, w.nGroupsPerRow, C.byref(prepared))
    return bool(prepared.value)


def prepareTileGemmTuned(fmt: int, packed, *, M: int, K: int, N: int, scale_base: int = 0,
                         x_dtype: int = _lib.DT_BF16) -> bool:
    """The tuner for the tile GEMM on resident `packed` weights (a torch device tensor):
    installs the fastest parity-checked route and knobs for format `fmt` at M rows of
    activations of type x_dtype (plans are kept per type)."""
    prepared = C.c_int(0)
    call("bybycu_prepare_tile_gemm_tuned", int(fmt), int(x_dtype), int(M), int(K), int(N), _ptr(packed),
         packed.numel() * packed.element_size(), int(scale_base), C.byref(prepared))
    return bool(prepared.value)


def tunedPlan(op: int, *, M: int, K: int, N: int, fmt: int = 0, x_dtype: int = _lib.DT_BF16,
              groupSize: int = 0, nGroupsPerRow: int = 0) -> "_lib.Plan | None":
    """The plan installed for a shape on the current device, or None."""
    plan, found = _lib.Plan(), C.c_int(0)
    call("bybycu_plan_get", int(op), int(fmt), int(x_dtype), int(M), int(K), int(N), int(groupSize),
         int(nGroupsPerRow), C.byref(plan), C.byref(found))
    return plan if found.value else None


def q4TuningStats() -> tuple[int, int]:
    """vulkanQ4TuningStats (q4_autotune.nim:545-546): (installed plans, ROUTE_AUTO launches
    that followed one)."""
    n, d = C.c_int(0), C.c_int64(0)
    call("bybycu_tuning_stats", C.byref(n), C.byref(d))
    return n.value, d.value


def tuneCachePath() -> str:
    """The plan cache file of the current device ('' when caching is off)."""
    buf = C.create_string_buffer(1024)
    call("bybycu_tune_cache_path", buf, 1024)
    return buf.value.decode()


def sessionUploadPrivatePtr(backend: GpuBackend, data: int, nbytes: int) -> SessionHandle:
    """gpubackend.nim:2940-2959: a device copy of `nbytes` at host address `data` (a model
    mapping or any host range), straight from there through the library's staging engine."""
    _chosen(backend)
    h = C.c_void_p()
    call("bybycu_session_upload_ptr", C.c_void_p(data), int(nbytes), C.byref(h))
    return SessionHandle(GpuBackend.gbCuda, CudaResidentTensor(h.value, int(nbytes)))


def sessionWrapHostRange(backend: GpuBackend, data: int, nbytes: int) -> tuple[SessionHandle, int]:
    """gpubackend.nim:2920-2938.  Wrapping host pages as a device buffer is for GPUs that share
    system memory; a B200 reads HBM, so the handle is always empty (callers then copy with
    sessionUploadPrivatePtr)."""
    _chosen(backend)
    return SessionHandle(GpuBackend.gbCuda, CudaResidentTensor()), 0


def residentUploadQ4Mapped(backend: GpuBackend, wq: int, wqBytes: int, scales, zeros, k: int, n: int,
                           groupSize: int, nGroupsPerRow: int) -> tuple[ResidentWeightHandle, bool]:
    """gpubackend.nim:2961-2998: residentUploadQ4 for packed nibbles that live in a model
    mapping at host address `wq`.  On a B200 (a dGPU) the nibbles are copied straight from the
    mapping into HBM, never through an intermediate host buffer, so zeroCopy is False and the
    mapping may be closed after the call.  Scales and zeros are small and copied."""
    _chosen(backend)
    if not _initialised:
        ensureGpuInit(backend)
    scales = np.ascontiguousarray(scales, np.float32).reshape(-1)
    zeros = np.ascontiguousarray(zeros, np.float32).reshape(-1)
    _q4_shape_check(int(wqBytes), scales.size, zeros.size, k, n, groupSize, nGroupsPerRow)
    if not wq:
        raise BybyCudaError(_lib.ERR_ARGS, "residentUploadQ4Mapped: wq is NULL")
    w = ResidentWeightHandle(GpuBackend.gbCuda, sessionUploadPrivatePtr(backend, wq, wqBytes),
                             sessionUpload(backend, scales), sessionUpload(backend, zeros), k, n, groupSize,
                             nGroupsPerRow)
    return w, False


def residentFreeQ4(backend: GpuBackend, w: ResidentWeightHandle) -> None:
    for h in (w.wq, w.scales, w.zeros):
        if h.ptr:
            sessionFree(backend, h)


def sessionMatmulQ4(backend: GpuBackend, a: SessionHandle, w: ResidentWeightHandle, c: SessionHandle,
                    M: int) -> bool:
    """gpubackend.nim:3000-3060: C(M x N) = A(M x K) @ W into the open session; an empty c
    gets a scratch buffer first (the reference's own fix for an unallocated output)."""
    if not c.ptr:
        c.cudaHandle = sessionAllocScratch(backend, M * w.n).cudaHandle
    return _gemm("bybycu_session_matmul_q4", backend,
                 (C.c_void_p(a.ptr), C.c_void_p(w.wq.ptr), C.c_void_p(w.scales.ptr), C.c_void_p(w.zeros.ptr),
                  C.c_void_p(c.ptr), M, w.k, w.n, w.groupSize, w.nGroupsPerRow), c, M, w.n)


def gpuMatmulQ4(backend: GpuBackend, a, wq, scales, zeros, m: int, k: int, n: int, groupSize: int,
                nGroupsPerRow: int) -> np.ndarray:
    """gpubackend.nim:806-843, immediate mode: host arrays in, the [m, n] fp32 product back."""
    import torch
    _chosen(backend)
    if not _initialised:
        ensureGpuInit(backend)
    wq, scales, zeros = _q4_check(wq, scales, zeros, k, n, groupSize, nGroupsPerRow)
    a = np.ascontiguousarray(a, np.float32).reshape(-1)
    if m <= 0 or a.size < m * k:
        raise BybyCudaError(_lib.ERR_RANGE, "matmul_q4: a is smaller than m * k")
    dev = torch.device("cuda", torch.cuda.current_device())
    t = [torch.from_numpy(v).to(dev) for v in (a[:m * k], wq, scales, zeros)]
    out = torch.empty(m, n, dtype=torch.float32, device=dev)
    try:
        call("bybycu_matmul_q4", *[_ptr(v) for v in t], _ptr(out), m, k, n, groupSize, nGroupsPerRow,
             _lib.ROUTE_AUTO, _stream_ptr(None))
    except BybyCudaError as e:
        handleGpuFailure(backend, "matmul_q4", e)
    return out.cpu().numpy()


def sessionMatmulQ4Fused(backend: GpuBackend, mode: int, a: SessionHandle, ws, outs, res: SessionHandle,
                         hasRes: bool, gamma: SessionHandle | None = None, eps: float = 0.0,
                         hasNorm: bool = False) -> bool:
    """gpubackend.nim:3185-3231: the fused decode GEMV (M = 1) in one launch.  mode 0: 1-3
    matrices share `a`, each into its own outs[i]; mode 1: ws = [gate, up] and outs[0] =
    silu(gate) * up.  hasRes adds `res`; hasNorm RMS-normalises `a` with `gamma` and `eps`.
    False when unsupported (the caller runs the unfused sequence); outputs must be allocated."""
    _chosen(backend)
    ws, outs = list(ws), list(outs)
    if not 1 <= len(ws) <= 3 or len(outs) < len(ws) or (mode == 1 and len(ws) != 2):
        return False
    if (hasRes and not res.ptr) or (hasNorm and (gamma is None or not gamma.ptr)):
        return False
    w0 = ws[0]
    for i, w in enumerate(ws):
        if w.kind != GpuBackend.gbCuda or not outs[i].ptr:
            return False
        if w.k != w0.k or w.groupSize != w0.groupSize or w.nGroupsPerRow != w0.nGroupsPerRow:
            return False
    n = len(ws)
    vp3 = C.c_void_p * n
    rc = _lib.load().bybycu_session_matmul_q4_fused(
        int(mode), C.c_void_p(a.ptr), n, vp3(*[w.wq.ptr for w in ws]), vp3(*[w.scales.ptr for w in ws]),
        vp3(*[w.zeros.ptr for w in ws]), (C.c_int * n)(*[w.n for w in ws]), vp3(*[o.ptr for o in outs[:n]]),
        C.c_void_p(res.ptr if hasRes else 0), C.c_void_p(gamma.ptr if hasNorm else 0), C.c_float(eps), w0.k,
        w0.groupSize, w0.nGroupsPerRow)
    if rc == _lib.ERR_SHAPE:
        return False
    if rc != 0:
        handleGpuFailure(backend, "matmul_q4_fused", BybyCudaError(rc, _lib.last_error()[1]))
    return True


def matmul_q4_fused(mode: int, x, weights, outs, *, res=None, gamma=None, eps: float = 0.0, stream=None):
    """The fused decode GEMV on torch tensors: x fp32 [1, K] (raw when gamma is given),
    weights a list of Q4AsymWeights, outs fp32 [1, N] tensors; raises when unsupported."""
    n = len(weights)
    vp = C.c_void_p * n
    call("bybycu_matmul_q4_fused", int(mode), _ptr(x), n, vp(*[w.wq.data_ptr() for w in weights]),
         vp(*[w.scales.data_ptr() for w in weights]), vp(*[w.zeros.data_ptr() for w in weights]),
         (C.c_int * n)(*[w.N for w in weights]), vp(*[o.data_ptr() for o in outs[:n]]), _ptr(res), _ptr(gamma),
         C.c_float(eps), weights[0].K, weights[0].group_size, weights[0].n_groups, _stream_ptr(stream))
    return outs


class Q4AsymWeights:
    """Asymmetric Q4 weights resident on one device, for torch callers: nibbles [N, (K+1)/2]
    (even k low), fp32 scales and zero points [N, groups] of ``group_size`` values."""

    def __init__(self, wq, scales, zeros, K: int, group_size: int = 32, device=None):
        import torch
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.wq = torch.as_tensor(wq).to(dev, torch.uint8).contiguous()
        self.scales = torch.as_tensor(scales).to(dev, torch.float32).contiguous()
        self.zeros = torch.as_tensor(zeros).to(dev, torch.float32).contiguous()
        self.N = self.wq.shape[0]
        self.K = K
        self.group_size = group_size
        self.n_groups = self.scales.shape[-1] if self.scales.dim() == 2 else self.scales.numel() // self.N
        _q4_shape_check(self.wq.numel(), self.scales.numel(), self.zeros.numel(), K, self.N, group_size,
                        self.n_groups)

    def matmul(self, x, out=None, *, route: int = _lib.ROUTE_AUTO, stream=None):
        """out[M, N] = x[M, K] . W^T, x fp32 on the device."""
        import torch
        M = x.shape[0]
        if out is None:
            out = torch.empty(M, self.N, dtype=torch.float32, device=x.device)
        call("bybycu_matmul_q4", _ptr(x), _ptr(self.wq), _ptr(self.scales), _ptr(self.zeros), _ptr(out), M, self.K,
             self.N, self.group_size, self.n_groups, int(route), _stream_ptr(stream))
        return out

    def prepare(self, M: int = 1) -> bool:
        """Autotunes the automatic route for M rows (residentPrepareQ4's role)."""
        prepared = C.c_int(0)
        call("bybycu_prepare_q4_tuned", _ptr(self.wq), _ptr(self.scales), _ptr(self.zeros), int(M), self.K, self.N,
             self.group_size, self.n_groups, C.byref(prepared))
        return bool(prepared.value)


__all__ = [
    "GpuBackend", "parseBackend", "normalizeBackend", "detectBackend", "ensureGpuInit",
    "setForbidCpuFallback", "gForbidCpuFallback", "handleGpuFailure", "SessionHandle",
    "CudaResidentTensor", "sessionBegin", "sessionEnd", "sessionUpload", "sessionAllocScratch",
    "sessionRead", "sessionFree", "sessionFp4GemmTensorCore", "sessionFp4GemmTiledEnc",
    "sessionF16GemmTile", "sessionQ4B32Gemm", "sessionTileGemmReady", "sessionMicroVmEnc",
    "tile_gemm", "route_for", "dequant", "Q4B32Weights", "tileWeightBytes", "TileFormatQ4B32",
    "ResidentWeightHandle", "residentUploadQ4", "residentPrepareQ4", "residentFreeQ4", "sessionMatmulQ4",
    "gpuMatmulQ4", "Q4AsymWeights", "sessionMatmulQ4Fused", "matmul_q4_fused", "prepareTileGemmTuned",
    "tunedPlan", "q4TuningStats", "tuneCachePath", "sessionUploadPrivatePtr", "sessionWrapHostRange",
    "residentUploadQ4Mapped",
]
