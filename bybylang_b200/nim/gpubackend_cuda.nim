## gpubackend_cuda.nim - the `gbCuda` backend of BybyLang's gpubackend.nim on libbybycuda.so.
##
## This file is INCLUDED into gpubackend.nim (`include backends/cuda/gpubackend_cuda`) right
## after the `SessionHandle` and `ResidentWeightHandle` type sections, so it sees their fields
## (`cudaHandle: CudaResidentTensor`, `cudaWq/cudaScales/cudaZeros`), `GpuBackend`,
## `gForbidCpuFallback` and `handleGpuFailure`.  It defines `cuda*` procs only; each public
## session proc of gpubackend.nim gains a one-line branch that calls its twin here (cudaXxx for
## each public proc Xxx).  It holds no state of its own: device pointers live in the handles,
## and every failure raises through handleGpuFailure (the cuda path never falls back to the
## CPU; gForbidCpuFallback is forced on at init).
##
## Pointers: CudaResidentTensor.dptr is the device address as uint64 and `n` its size in
## BYTES (the reference's Vulkan handles also carry byte sizes).

import std/[os, strutils]
import ./bybycuda

proc cudaCheck(rc: cint; op: string) =
  ## A non-zero status is a hard failure on the cuda backend.
  if rc != BYBYCU_OK:
    handleGpuFailure(gbCuda, op, newException(CatchableError, bybycuLastError()))

template dptr(h: SessionHandle): pointer = cast[pointer](h.cudaHandle.dptr)
template dptr(t: CudaResidentTensor): pointer = cast[pointer](t.dptr)

proc cudaHandleOf(p: pointer; bytes: int): SessionHandle =
  result.kind = gbCuda
  result.cudaHandle = CudaResidentTensor(dptr: cast[uint64](p), n: bytes)

# ---------------------------------------------------------------------------------------
# Backend selection and lifecycle (gpubackend.nim:107-131, 1025-1042)
# ---------------------------------------------------------------------------------------

var cudaInitialised = false

proc cudaEnsureInit*(): bool =
  ## Selects BYBY_CUDA_DEVICE (default 0), checks it is an sm_100 part, loads the library's
  ## module on it, and forbids the CPU fallback for the rest of the process.
  if cudaInitialised: return true
  if bybycu_version() != BYBYCU_ABI_VERSION:
    handleGpuFailure(gbCuda, "ensureGpuInit",
                     newException(CatchableError, "libbybycuda ABI version mismatch"))
  let dev = parseInt(getEnv("BYBY_CUDA_DEVICE", "0"))
  cudaCheck(bybycu_init(dev.cint), "ensureGpuInit")
  gForbidCpuFallback = true
  cudaInitialised = true
  true

proc cudaAvailable*(): bool =
  ## detectBackend's probe: a usable device without raising.
  var n: cint
  bybycu_device_count(addr n) == BYBYCU_OK and n > 0

proc cudaSessionBegin*(): bool =
  discard cudaEnsureInit()
  cudaCheck(bybycu_session_begin(), "sessionBegin")
  true

proc cudaSessionEnd*(): bool =
  cudaCheck(bybycu_session_end(), "sessionEnd")
  true

proc cudaSessionUpload*(data: seq[float32]): SessionHandle =
  var h: pointer
  let bytes = int64(data.len * sizeof(float32))
  cudaCheck(bybycu_session_upload(if data.len > 0: data[0].unsafeAddr else: nil, bytes, addr h),
            "sessionUpload")
  cudaHandleOf(h, bytes.int)

proc cudaSessionUploadBytes*(data: openArray[uint8]): SessionHandle =
  var h: pointer
  cudaCheck(bybycu_session_upload(if data.len > 0: data[0].unsafeAddr else: nil, data.len.int64, addr h),
            "sessionUpload")
  cudaHandleOf(h, data.len)

proc cudaSessionAllocScratch*(n: int): SessionHandle =
  var h: pointer
  cudaCheck(bybycu_session_alloc_scratch(n.int64, addr h), "sessionAllocScratch")
  cudaHandleOf(h, n * sizeof(float32))

proc cudaSessionRead*(h: SessionHandle; n: int): seq[float32] =
  result = newSeq[float32](n)
  if n > 0:
    cudaCheck(bybycu_session_read(h.dptr, result[0].addr, n.int64), "sessionRead")

proc cudaSessionFree*(h: var SessionHandle) =
  if h.cudaHandle.dptr != 0:
    cudaCheck(bybycu_session_free(h.dptr), "sessionFree")
  h.cudaHandle = CudaResidentTensor()

# ---------------------------------------------------------------------------------------
# The tile GEMM (gpubackend.nim:1442-1488): FP4-KM, FP16 and Q4B32 weights
# ---------------------------------------------------------------------------------------

proc cudaFp4Gemm*(a, w, lut: SessionHandle; c: var SessionHandle; M, K, N: int;
                  tensorCore: bool): bool =
  ## sessionFp4GemmTensorCore (tensorCore) and sessionFp4GemmTiledEnc (register tiles, the
  ## bit-exact SIMT loop).  False only for shapes the library reports it cannot run.
  if c.cudaHandle.dptr == 0: c = cudaSessionAllocScratch(M * N)
  let rc = bybycu_session_fp4_gemm(a.dptr, w.dptr, lut.dptr, c.dptr, M.cint, K.cint, N.cint,
                                   tensorCore.cint)
  if rc == BYBYCU_ERR_SHAPE: return false
  cudaCheck(rc, if tensorCore: "sessionFp4GemmTensorCore" else: "sessionFp4GemmTiledEnc")
  true

proc cudaF16GemmTile*(a, w: SessionHandle; c: var SessionHandle; M, K, N: int;
                      tensorCore: bool): bool =
  if c.cudaHandle.dptr == 0: c = cudaSessionAllocScratch(M * N)
  let rc = bybycu_session_f16_gemm(a.dptr, w.dptr, c.dptr, M.cint, K.cint, N.cint, tensorCore.cint)
  if rc == BYBYCU_ERR_SHAPE: return false
  cudaCheck(rc, "sessionF16GemmTile")
  true

proc cudaQ4B32Gemm*(a, w: SessionHandle; c: var SessionHandle; M, K, N: int;
                    tensorCore = true): bool =
  ## Format 2 (Q4B32): nibbles [N, K/2] in the tile layout, then fp16 scales [N, K/32] at a
  ## 16-byte aligned offset, in one uploaded slot.
  if c.cudaHandle.dptr == 0: c = cudaSessionAllocScratch(M * N)
  let rc = bybycu_session_q4b32_gemm(a.dptr, w.dptr, c.dptr, M.cint, K.cint, N.cint, tensorCore.cint)
  if rc == BYBYCU_ERR_SHAPE: return false
  cudaCheck(rc, "sessionQ4B32Gemm")
  true

proc cudaTileGemmReady*(f16, tensorCore: bool): bool =
  ## The exact-data parity gate (M=37, N=80, rel err <= 1e-3), once per process.
  discard cudaEnsureInit()
  var ready: cint
  let fmt = if f16: BYBYCU_FMT_F16 else: BYBYCU_FMT_FP4KM
  cudaCheck(bybycu_tile_gemm_ready(fmt, tensorCore.cint, addr ready), "sessionTileGemmReady")
  ready != 0

proc cudaMicroVmEnc*(code, mem: SessionHandle; nThreads, tgFloats, tgSize: int): bool =
  ## sessionMicroVmEnc on device slots.  The library takes the program words from host memory,
  ## so they are read back from `code` (a few dozen words).  Programs outside the tile-GEMM and
  ## Q4 GEMV families raise: there is no fallback on this backend.
  let nWords = code.cudaHandle.n div 4
  var words = newSeq[uint32](nWords)
  if nWords > 0:
    cudaCheck(bybycu_download(words[0].addr, code.dptr, int64(nWords * 4), nil), "sessionMicroVmEnc")
    cudaCheck(bybycu_synchronize(nil), "sessionMicroVmEnc")
  var err = newString(256)
  let memFloats = (mem.cudaHandle.n div 4).cint
  let rc = bybycu_vm_run_slots(if nWords > 0: words[0].addr else: nil, nWords.cint,
                               cast[ptr float32](mem.dptr), memFloats,
                               cast[ptr uint8](mem.dptr), mem.cudaHandle.n.cint,
                               cast[ptr float32](mem.dptr), memFloats, nil, 0,
                               nThreads.cint, tgFloats.cint, tgSize.cint, err.cstring, 256, nil)
  if rc != BYBYCU_OK:
    handleGpuFailure(gbCuda, "sessionMicroVmEnc", newException(CatchableError, $err.cstring))
  true

# ---------------------------------------------------------------------------------------
# Asymmetric Q4 (matmul_q4; gpubackend.nim:806-843, 2871-3060, 3185-3231)
# ---------------------------------------------------------------------------------------

proc cudaResidentUploadQ4*(wq: seq[uint8]; scales, zeros: seq[float32];
                           k, n, groupSize, nGroupsPerRow: int): ResidentWeightHandle =
  result.kind = gbCuda
  result.k = k; result.n = n; result.groupSize = groupSize; result.nGroupsPerRow = nGroupsPerRow
  result.cudaWq = cudaSessionUploadBytes(wq).cudaHandle
  result.cudaScales = cudaSessionUpload(scales).cudaHandle
  result.cudaZeros = cudaSessionUpload(zeros).cudaHandle
  result.cudaQ4Ready = true

proc cudaResidentUploadQ4Mapped*(wq: pointer; wqBytes: int; scales, zeros: openArray[float32];
                                 k, n, groupSize, nGroupsPerRow: int): tuple[w: ResidentWeightHandle,
                                                                             zeroCopy: bool] =
  ## A B200 reads HBM: the packed weights are copied once from the mapping by the library's
  ## staged engine (no Nim seq in between), never wrapped in place (zeroCopy = false).
  var w = ResidentWeightHandle(kind: gbCuda, k: k, n: n, groupSize: groupSize, nGroupsPerRow: nGroupsPerRow)
  var h: pointer
  cudaCheck(bybycu_session_upload_ptr(wq, wqBytes.int64, addr h), "residentUploadQ4Mapped")
  w.cudaWq = CudaResidentTensor(dptr: cast[uint64](h), n: wqBytes)
  w.cudaScales = cudaSessionUpload(@scales).cudaHandle
  w.cudaZeros = cudaSessionUpload(@zeros).cudaHandle
  w.cudaQ4Ready = true
  (w, false)

proc cudaResidentPrepareQ4*(w: ResidentWeightHandle; M = 1): bool =
  ## The autotuner for this shape and M class; the winning plan is cached on disk and used by
  ## later sessionMatmulQ4 calls.  BYBY_Q4_TUNED=0 / BYBY_GPU_AUTOTUNE=0 switch it off.
  var prepared: cint
  cudaCheck(bybycu_prepare_q4_tuned(w.cudaWq.dptr, w.cudaScales.dptr, w.cudaZeros.dptr, M.cint, w.k.cint,
                                    w.n.cint, w.groupSize.cint, w.nGroupsPerRow.cint, addr prepared),
            "residentPrepareQ4")
  prepared != 0

proc cudaSessionMatmulQ4*(a: SessionHandle; w: ResidentWeightHandle; c: var SessionHandle; M: int): bool =
  if c.cudaHandle.dptr == 0: c = cudaSessionAllocScratch(M * w.n)
  let rc = bybycu_session_matmul_q4(a.dptr, w.cudaWq.dptr, w.cudaScales.dptr, w.cudaZeros.dptr, c.dptr,
                                    M.cint, w.k.cint, w.n.cint, w.groupSize.cint, w.nGroupsPerRow.cint)
  if rc == BYBYCU_ERR_SHAPE: return false
  cudaCheck(rc, "sessionMatmulQ4")
  true

proc cudaSessionMatmulQ4Fused*(mode: int; a: SessionHandle; ws: openArray[ResidentWeightHandle];
                               outs: openArray[SessionHandle]; res: SessionHandle; hasRes: bool;
                               gamma: SessionHandle; eps: float32; hasNorm: bool): bool =
  ## One launch: 1-3 matrices sharing `a` (mode 0) or silu(gate) * up (mode 1), with RMSNorm
  ## and the residual when asked.  False (unsupported form) leaves the session usable; the
  ## caller runs the unfused sequence, as for the reference's encoder.
  if ws.len < 1 or ws.len > 3 or outs.len != (if mode == 1: 1 else: ws.len): return false
  var wq, sc, zp, op: array[3, pointer]
  var ns: array[3, cint]
  for i, w in ws:
    wq[i] = w.cudaWq.dptr; sc[i] = w.cudaScales.dptr; zp[i] = w.cudaZeros.dptr
    ns[i] = w.n.cint
  for i, o in outs: op[i] = o.dptr
  let rc = bybycu_session_matmul_q4_fused(mode.cint, a.dptr, ws.len.cint, wq[0].addr, sc[0].addr, zp[0].addr,
                                          ns[0].addr, op[0].addr, (if hasRes: res.dptr else: nil),
                                          (if hasNorm: gamma.dptr else: nil), eps, ws[0].k.cint,
                                          ws[0].groupSize.cint, ws[0].nGroupsPerRow.cint)
  if rc == BYBYCU_ERR_SHAPE: return false
  cudaCheck(rc, "sessionMatmulQ4Fused")
  true

proc cudaGpuMatmulQ4*(a: seq[float32]; wq: seq[uint8]; scales, zeros: seq[float32];
                      m, k, n, groupSize, nGroupsPerRow: int): seq[float32] =
  ## The one-shot form: upload, the automatic route, read back.
  discard cudaEnsureInit()
  var da, dw, ds, dz, dc: pointer
  template up(dst: var pointer; src: pointer; bytes: int) =
    cudaCheck(bybycu_malloc(addr dst, bytes.int64), "gpuMatmulQ4")
    cudaCheck(bybycu_upload(dst, src, bytes.int64, nil), "gpuMatmulQ4")
  up(da, a[0].unsafeAddr, a.len * 4)
  up(dw, wq[0].unsafeAddr, wq.len)
  up(ds, scales[0].unsafeAddr, scales.len * 4)
  up(dz, zeros[0].unsafeAddr, zeros.len * 4)
  cudaCheck(bybycu_malloc(addr dc, int64(m * n * 4)), "gpuMatmulQ4")
  try:
    cudaCheck(bybycu_matmul_q4(cast[ptr float32](da), cast[ptr uint8](dw), cast[ptr float32](ds),
                               cast[ptr float32](dz), cast[ptr float32](dc), m.cint, k.cint, n.cint,
                               groupSize.cint, nGroupsPerRow.cint, BYBYCU_ROUTE_AUTO, nil), "gpuMatmulQ4")
    result = newSeq[float32](m * n)
    cudaCheck(bybycu_download(result[0].addr, dc, int64(m * n * 4), nil), "gpuMatmulQ4")
    cudaCheck(bybycu_synchronize(nil), "gpuMatmulQ4")
  finally:
    for p in [da, dw, ds, dz, dc]: discard bybycu_free(p)

proc cudaQ4TuningStats*(): tuple[preparedPlans: int, tunedDispatches: int64] =
  ## vulkanQ4TuningStats' twin.
  var plans: cint
  var disp: int64
  cudaCheck(bybycu_tuning_stats(addr plans, addr disp), "q4TuningStats")
  (plans.int, disp)
