## bybycuda.nim - Nim binding of libbybycuda.so (include/bybycuda.h), the C ABI of the B200
## tile-GEMM / GEMV path.  Every proc returns 0 or a negative BYBYCU_ERR_* status; the message
## of the last failure on this thread comes from bybycu_last_error.
##
## This module is pure binding: it depends on nothing in BybyLang.  gpubackend_cuda.nim (included
## into gpubackend.nim) builds the `gbCuda` backend on it.
##
## Library location: the dynlib name below, resolved by the dynamic loader (put the directory of
## libbybycuda.so on LD_LIBRARY_PATH, or pass -d:bybycuLib=<path> to the compiler).

const bybycuLib* {.strdefine.} = "libbybycuda.so"

const
  BYBYCU_ABI_VERSION* = 1
  # status codes
  BYBYCU_OK* = 0.cint
  BYBYCU_ERR_ARGS* = -1.cint
  BYBYCU_ERR_SHAPE* = -2.cint
  BYBYCU_ERR_RANGE* = -3.cint
  BYBYCU_ERR_CUDA* = -4.cint
  BYBYCU_ERR_NODEV* = -5.cint
  BYBYCU_ERR_PROGRAM* = -6.cint
  BYBYCU_ERR_DEVICE* = -7.cint
  BYBYCU_ERR_SESSION* = -8.cint
  BYBYCU_ERR_PARITY* = -9.cint
  # tile formats (OP_TILE_GEMM's fmt field; 2 is the Q4B32 format of this path)
  BYBYCU_FMT_FP4KM* = 0.cint
  BYBYCU_FMT_F16* = 1.cint
  BYBYCU_FMT_Q4B32* = 2.cint
  # element types of x and out
  BYBYCU_DT_F32* = 0.cint
  BYBYCU_DT_BF16* = 1.cint
  # routes
  BYBYCU_ROUTE_AUTO* = 0.cint
  BYBYCU_ROUTE_GEMV* = 1.cint
  BYBYCU_ROUTE_TC* = 2.cint
  BYBYCU_ROUTE_SIMT* = 3.cint
  BYBYCU_ROUTE_TC_FP16W* = 4.cint
  # tuned-plan operations
  BYBYCU_OP_TILE_GEMM* = 0.cint
  BYBYCU_OP_MATMUL_Q4* = 1.cint

{.push importc, cdecl, dynlib: bybycuLib.}
proc bybycu_version*(): cint
proc bybycu_last_error*(buf: cstring, len: cint): cint
proc bybycu_device_count*(count: ptr cint): cint
proc bybycu_init*(device: cint): cint
proc bybycu_malloc*(dptr: ptr pointer, bytes: int64): cint
proc bybycu_free*(dptr: pointer): cint
proc bybycu_upload*(dst, src: pointer, bytes: int64, stream: pointer): cint
proc bybycu_download*(dst, src: pointer, bytes: int64, stream: pointer): cint
proc bybycu_memset*(dst: pointer; value: cint; bytes: int64; stream: pointer): cint
proc bybycu_stream_create*(stream: ptr pointer): cint
proc bybycu_stream_destroy*(stream: pointer): cint
proc bybycu_synchronize*(stream: pointer): cint
proc bybycu_device_error*(code: ptr cint): cint
# the op (OP_TILE_GEMM, session_vm.nim:106-122; slots out/packed/lut/x)
proc bybycu_tile_gemm*(fmt, M, K, N: cint; x: pointer; xDtype: cint; xLen: int64;
                      packed: pointer; packedLen, scaleBase: int64;
                      lut: ptr float32; lutLen, lutBase: int64;
                      outp: pointer; outDtype: cint; outLen: int64;
                      route: cint; stream: pointer): cint
proc bybycu_tile_gemm_host*(fmt, M, K, N: cint; xHost: pointer; xDtype: cint;
                           packed: pointer; packedLen, scaleBase: int64;
                           lut: ptr float32; lutLen, lutBase: int64;
                           outHost: pointer; outDtype: cint; xDev, outDev: pointer;
                           route: cint; stream: pointer): cint
proc bybycu_dequant*(fmt, K, N: cint; packed: pointer; packedLen, scaleBase: int64;
                    lut: ptr float32; lutLen, lutBase: int64; wOut: ptr float32;
                    stream: pointer): cint
proc bybycu_route_for*(fmt, M, K, N, xDtype: cint; route: ptr cint): cint
# nimf_cpu_vm_run_slots' device twin (cpu_kernels.h:118-121)
proc bybycu_vm_run_slots*(code: ptr uint32; nWords: cint; mem: ptr float32; memLen: cint;
                         packed: ptr uint8; packedLen: cint; lut: ptr float32; lutLen: cint;
                         inF32: ptr float32; inLen, nThreads, tgFloats, tgSize: cint;
                         err: cstring; errLen: cint; stream: pointer): cint
# session procs (gpubackend.nim:1042-1488)
proc bybycu_session_begin*(): cint
proc bybycu_session_end*(): cint
proc bybycu_session_upload*(host: pointer; bytes: int64; handle: ptr pointer): cint
proc bybycu_session_alloc_scratch*(nFloats: int64; handle: ptr pointer): cint
proc bybycu_session_read*(handle: pointer; host: ptr float32; nFloats: int64): cint
proc bybycu_session_free*(handle: pointer): cint
proc bybycu_session_fp4_gemm*(a, w, lut, c: pointer; M, K, N, tensorCore: cint): cint
proc bybycu_session_f16_gemm*(a, w, c: pointer; M, K, N, tensorCore: cint): cint
proc bybycu_session_q4b32_gemm*(a, w, c: pointer; M, K, N, tensorCore: cint): cint
proc bybycu_tile_gemm_ready*(fmt, tensorCore: cint; ready: ptr cint): cint
# asymmetric Q4, matmul_q4 (gpubackend.nim:806-843,2883-3060; cpu_kernels_impl.inc:293-319)
proc bybycu_matmul_q4*(a: ptr float32; wq: ptr uint8; scales, zeros: ptr float32; c: ptr float32;
                      M, K, N, groupSize, nGroupsPerRow, route: cint; stream: pointer): cint
proc bybycu_session_matmul_q4*(a, wq, scales, zeros, c: pointer;
                              M, K, N, groupSize, nGroupsPerRow: cint): cint
proc bybycu_matmul_q4_fused*(mode: cint; a: ptr float32; nMats: cint; wq, scales, zeros: ptr pointer;
                            N: ptr cint; outs: ptr pointer; res, gamma: ptr float32; eps: float32;
                            K, groupSize, nGroupsPerRow: cint; stream: pointer): cint
proc bybycu_session_matmul_q4_fused*(mode: cint; a: pointer; nMats: cint; wq, scales, zeros: ptr pointer;
                                    N: ptr cint; outs: ptr pointer; res, gamma: pointer; eps: float32;
                                    K, groupSize, nGroupsPerRow: cint): cint
# column shards and the device-side all-gather (distributed.nim:109-135, :304-375)
proc bybycu_shard_range*(N, world, rank, align: cint; n0, n1: ptr cint): cint
proc bybycu_ipc_handle*(dptr: pointer; handle: ptr array[64, uint8]; offset: ptr int64): cint
proc bybycu_ipc_open*(handle: ptr array[64, uint8]; offset: int64; dptr: ptr pointer): cint
proc bybycu_ipc_close*(dptr: pointer): cint
proc bybycu_tile_gemm_allgather*(fmt, M, K, N, n0, n1: cint; x: pointer; xDtype: cint;
                                packed: pointer; packedLen, scaleBase: int64;
                                lut: ptr float32; lutLen, lutBase: int64;
                                outp: pointer; peerOut: ptr pointer; peerSignal: ptr ptr uint32;
                                world, rank: cint; epoch: uint32; stream: pointer): cint
proc bybycu_tile_gemm_allgather_split*(fmt, M, K, N, n0, n1: cint; x: pointer; xDtype: cint;
                                       packed: pointer; packedLen, scaleBase: int64;
                                       lut: ptr float32; lutLen, lutBase: int64;
                                       outp: pointer; peerOut: ptr pointer; peerSignal: ptr ptr uint32;
                                       world, rank: cint; epoch: uint32; stream: pointer): cint
proc bybycu_allgather_wait*(peerSignal: ptr ptr uint32; world, rank: cint; epoch: uint32; stream: pointer): cint
proc bybycu_tile_gemm_noalloc*(M, K, N: cint; x: pointer; xDtype: cint; xLen: int64;
                              packed: pointer; packedLen, scaleBase: int64;
                              outp: pointer; outDtype: cint; outLen: int64; stream: pointer): cint
# tuned plans (q4_autotune.nim:2-117, 387-546)
type BybycuPlan* {.importc: "bybycu_plan", header: "bybycuda.h".} = object
  route*, variant*, stages*: int32
  ms*: float32
  name*: array[32, char]
proc bybycu_prepare_q4_tuned*(wq, scales, zeros: pointer; M, K, N, groupSize, nGroupsPerRow: cint;
                             prepared: ptr cint): cint
proc bybycu_prepare_tile_gemm_tuned*(fmt, xDtype, M, K, N: cint; packed: pointer;
                                    packedLen, scaleBase: int64; prepared: ptr cint): cint
proc bybycu_plan_get*(op, fmt, xDtype, M, K, N, groupSize, nGroupsPerRow: cint;
                     plan: ptr BybycuPlan; found: ptr cint): cint
proc bybycu_plan_set*(op, fmt, xDtype, M, K, N, groupSize, nGroupsPerRow: cint; plan: ptr BybycuPlan): cint
proc bybycu_plan_clear*(): cint
proc bybycu_tuning_stats*(preparedPlans: ptr cint; tunedDispatches: ptr int64): cint
proc bybycu_tune_cache_path*(buf: cstring; bufLen: cint): cint
# weight ingestion (mapped_file.nim, gpubackend.nim:2920-2998, probe_weights.nim, probe_data.nim)
type BybycuTensorInfo* {.importc: "bybycu_tensor_info", header: "bybycuda.h".} = object
  name*: array[256, char]
  nameLen*, kind*, rank*, scales*: int32
  shape*: array[8, int64]
  offset*, bytes*, scaleOffset*: int64
  groupSize*, eb*, mb*: int32
  dtype*: array[16, char]
proc bybycu_map_file*(path: cstring; data: ptr pointer; size: ptr int64; mapping: ptr pointer): cint
proc bybycu_unmap_file*(mapping: pointer): cint
proc bybycu_upload_host_range*(dst, src: pointer; bytes: int64): cint
proc bybycu_session_upload_ptr*(host: pointer; bytes: int64; handle: ptr pointer): cint
proc bybycu_fingerprint*(data: pointer; bytes: int64; outp: cstring; outLen: cint): cint
proc bybycu_checkpoint_index*(path: cstring; outp: ptr BybycuTensorInfo; cap: cint; count: ptr cint): cint
{.pop.}

proc bybycuLastError*(): string =
  ## The message of the last failed call on this thread.
  var buf = newString(512)
  discard bybycu_last_error(buf.cstring, 512)
  $buf.cstring
