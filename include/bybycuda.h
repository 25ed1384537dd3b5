/* bybycuda.h - C ABI of libbybycuda.so, the B200 (sm_100a) implementation of BybyLang's
 * 4-bit block-quantized tile-GEMM / GEMV path.
 *
 * Conventions (those of the reference's CPU C ABI, backends/cpu/cpu_kernels.h:39-121):
 *   - plain C types only: device buffers are `void*` device pointers (the value a
 *     CudaResidentTensor.dptr carries, gpubackend.nim:23-27), streams are `void*`
 *     (a cudaStream_t; NULL = the legacy default stream);
 *   - lengths are in elements of the slot's type, the packed-weight slot in bytes;
 *   - every `int` return is 0 on success or a negative BYBYCU_ERR_* code, and the message
 *     of the last failure on the calling host thread is copied by bybycu_last_error();
 *   - the caller owns every buffer and nothing is retained across calls (except the
 *     session handles of the session API, which the caller frees);
 *   - there is no CPU fallback: a call that cannot run on the GPU returns an error.
 *
 * Weight formats of OP_TILE_GEMM (micro_kernel/session_vm.nim:106-122) accepted here:
 *   0 FP4-KM  nibble bytes [N, K/2] from byte 0 of the packed slot (byte j of a 32-value group:
 *             low nibble = element j, high nibble = element j+16), scale bytes [N, K/32] at
 *             byte scale_base, weight = lut[lut_base + nibble] * lut[lut_base + 16 + scale byte]
 *   1 FP16    IEEE halves [N, K] from byte 0 of the packed slot; no table
 *   2 Q4B32   nibbles as format 0 holding signed int4 (two's complement, [-8, 7]); one IEEE
 *             half scale per 32-value block, [N, K/32] row-major at byte scale_base;
 *             weight = (float)q * (float)scale.  (New: no reference counterpart.)
 */
#ifndef BYBYCUDA_H
#define BYBYCUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BYBYCU_ABI_VERSION 1

#if defined(__GNUC__)
#define BYBYCU_API __attribute__((visibility("default")))
#else
#define BYBYCU_API
#endif

/* status codes */
#define BYBYCU_OK 0
#define BYBYCU_ERR_ARGS (-1)      /* null pointer, negative size, bad enum value */
#define BYBYCU_ERR_SHAPE (-2)     /* shape or format the op does not support */
#define BYBYCU_ERR_RANGE (-3)     /* a slot is too small for the shape */
#define BYBYCU_ERR_CUDA (-4)      /* CUDA runtime failure */
#define BYBYCU_ERR_NODEV (-5)     /* no usable sm_100 device */
#define BYBYCU_ERR_PROGRAM (-6)   /* VM program not accepted by the CUDA executor */
#define BYBYCU_ERR_DEVICE (-7)    /* a kernel reported a device-side error (bounded wait) */
#define BYBYCU_ERR_SESSION (-8)   /* session API used out of order */
#define BYBYCU_ERR_PARITY (-9)    /* a parity gate failed */

/* OP_TILE_GEMM weight formats */
#define BYBYCU_FMT_FP4KM 0
#define BYBYCU_FMT_F16 1
#define BYBYCU_FMT_Q4B32 2

/* element types of activations and outputs */
#define BYBYCU_DT_F32 0
#define BYBYCU_DT_BF16 1

/* kernel routes */
#define BYBYCU_ROUTE_AUTO 0   /* GEMV for M <= 16, tensor-core GEMM above;
                                 format 2: tensor cores from M = 8 when K >= 8192
                                 and from M = 12 when N >= 65536 */
#define BYBYCU_ROUTE_GEMV 1   /* decode GEMV: TMA-streamed weights, register dequant */
#define BYBYCU_ROUTE_TC 2     /* prefill GEMM: tcgen05 MMAs, fp32 accumulators in TMEM */
#define BYBYCU_ROUTE_SIMT 3   /* CUDA-core FP32 tile loop, every format and shape */
#define BYBYCU_ROUTE_TC_FP16W 4  /* format 2 on the tensor cores with each weight q*s rounded once
                                    to fp16 (the reference's cooperative-matrix lowering,
                                    micro_kernel/tile_gemm.nim:322-325): half the MMAs of route TC,
                                    which keeps every weight exact as two fp16 terms; only when
                                    asked for (AUTO never picks it) */

/* ---- library / device -------------------------------------------------------------- */

/* ABI version of the loaded library. */
BYBYCU_API int bybycu_version(void);

/* Copies the last error message of this host thread (NUL-terminated, truncated to
 * buf_len) and returns its status code.  Replaces the `err`/`err_len` pair of
 * nimf_cpu_vm_run_slots (backends/cpu/cpu_vm.c:168-175) and sessionGetLastError
 * (gpubackend.nim:2647-2667). */
BYBYCU_API int bybycu_last_error(char* buf, int buf_len);

/* Number of CUDA devices (detectBackend's probe, gpubackend.nim:131-142). */
BYBYCU_API int bybycu_device_count(int* count);

/* Makes `device` current on this host thread and checks it is an sm_100 part
 * (ensureGpuInit for the `cuda` backend; BYBY_CUDA_DEVICE chooses it in the host layer). */
BYBYCU_API int bybycu_init(int device);

/* Device memory (the CudaResidentTensor stubs cuUpload / cuFree, gpubackend.nim:23-31). */
BYBYCU_API int bybycu_malloc(void** dptr, int64_t bytes);
BYBYCU_API int bybycu_free(void* dptr);
BYBYCU_API int bybycu_upload(void* dst, const void* src, int64_t bytes, void* stream);
BYBYCU_API int bybycu_download(void* dst, const void* src, int64_t bytes, void* stream);
BYBYCU_API int bybycu_memset(void* dst, int value, int64_t bytes, void* stream);
BYBYCU_API int bybycu_stream_create(void** stream);
BYBYCU_API int bybycu_stream_destroy(void* stream);
BYBYCU_API int bybycu_synchronize(void* stream);

/* Reads and clears the device-side error word that kernels set when a bounded wait runs
 * out (synchronises the device first). *code = 0 when no kernel reported an error. */
BYBYCU_API int bybycu_device_error(int* code);

/* ---- the tile GEMM op -------------------------------------------------------------- */

/* out[M, N] = x[M, K] * dequant(W)[N, K]^T for one OP_TILE_GEMM (session_vm.nim:106-122,
 * :383-416), the slots of the micro-VM: out = slot 1, packed = slot 2, lut = slot 3,
 * x = slot 4 (micro_kernel/tile_gemm.nim:16-18).  Replaces the CPU VM arm
 * backends/cpu/cpu_vm.c:541-628 and the Vulkan dispatch tryTileGemm
 * (backends/vulkan/vulkan_driver.nim:2599-2646) with the same size checks.
 *   fmt        BYBYCU_FMT_*;  M > 0 rows, K > 0 a multiple of 32, N > 0 columns
 *   x          device, x_dtype (F32 or BF16), x_len >= M*K elements
 *   packed     device, packed_len bytes; scale_base = byte of the scale block (fmt 0, 2)
 *   lut        device float table, lut_len floats, lut_base = first of its 272 floats
 *              (fmt 0 only; may be NULL otherwise)
 *   out        device, out_dtype (F32 or BF16), out_len >= M*N elements
 *   route      BYBYCU_ROUTE_*; AUTO picks by M, an explicit route fails with
 *              BYBYCU_ERR_SHAPE if it cannot run the shape/format
 * Asynchronous on `stream`. */
BYBYCU_API int bybycu_tile_gemm(int fmt, int M, int K, int N,
                     const void* x, int x_dtype, int64_t x_len,
                     const void* packed, int64_t packed_len, int64_t scale_base,
                     const float* lut, int64_t lut_len, int64_t lut_base,
                     void* out, int out_dtype, int64_t out_len,
                     int route, void* stream);

/* The same op with HOST activations and output and DEVICE-resident weights: copies x in,
 * runs the op and copies out back, synchronising `stream` before it returns.  When out_host
 * is page-locked, mapped host memory (cudaHostAlloc / cudaHostRegister) the kernel stores the
 * result straight into it and out_dev is not used.  The immediate-mode form of the path
 * (gpuMatmulQ4, gpubackend.nim:806-843). */
BYBYCU_API int bybycu_tile_gemm_host(int fmt, int M, int K, int N,
                          const void* x_host, int x_dtype,
                          const void* packed, int64_t packed_len, int64_t scale_base,
                          const float* lut, int64_t lut_len, int64_t lut_base,
                          void* out_host, int out_dtype,
                          void* x_dev, void* out_dev, int route, void* stream);

/* The format-2 (Q4B32) tensor-core GEMM of bybycu_tile_gemm (route TC) for callers that
 * cannot allocate device memory at call time - e.g. a serving process that reserved
 * nearly all HBM for its own caches at start-up, where a call-time allocation can fail or
 * stall on the allocator.  This entry point has no reference counterpart: the reference
 * never stages activations, so it never needs scratch.
 *   Scratch: the fp16 staging copy of x (M*K*2 bytes) lives in one fixed 32 MiB array of
 *   the library's device memory.  CUDA loads a module lazily, so bybycu_init(device) loads
 *   this array and the route's kernels on that device; call it once per device before the
 *   first call here (and before any stream capture).  Each call then looks the array's
 *   address up (cudaGetSymbolAddress) in the current context; nothing is allocated or freed
 *   per call.  No part of it needs to start at zero: every byte the GEMM reads is written
 *   by the same call first.  When the route splits its last wave's tiles along K, the
 *   partial sums use the array's room past the staged activations; without room the tiles
 *   run whole (the same result within the route's tolerance, summed in another order).
 *   Limit: M*K <= 16,777,216 (e.g. M=4096 at K=4096); larger shapes fail with
 *   BYBYCU_ERR_RANGE before anything is launched.  Shapes the TC route cannot tile
 *   (K % 256 != 0, unaligned slots) fail with BYBYCU_ERR_SHAPE.
 *   Concurrency: there is one array per device.  Calls on the same stream are ordered and
 *   safe; calls that may run at the same time on one device (different streams, or
 *   different host threads) race on the array and corrupt each other's results.
 * Arguments as bybycu_tile_gemm (fmt = 2, no table); asynchronous on `stream`. */
BYBYCU_API int bybycu_tile_gemm_noalloc(int M, int K, int N,
                             const void* x, int x_dtype, int64_t x_len,
                             const void* packed, int64_t packed_len, int64_t scale_base,
                             void* out, int out_dtype, int64_t out_len, void* stream);

/* Dequantises W to fp32 w[N, K] (the bit-exact check of the format decode:
 * cpu_vm.c:612-617 for format 0). */
BYBYCU_API int bybycu_dequant(int fmt, int K, int N, const void* packed, int64_t packed_len,
                   int64_t scale_base, const float* lut, int64_t lut_len, int64_t lut_base,
                   float* w_out, void* stream);

/* The route AUTO takes for a shape, after the same checks as bybycu_tile_gemm. */
BYBYCU_API int bybycu_route_for(int fmt, int M, int K, int N, int x_dtype, int* route);

/* Asymmetric Q4, the reference's matmul_q4 (gpuMatmulQ4 / sessionMatmulQ4,
 * gpubackend.nim:806-843,3000-3060; nimf_cpu_matmul_q4, cpu_kernels_impl.inc:293-319):
 *     c[M, N] = a[M, K] . W^T,  W[n, k] = (u[n, k] - zeros[n, g]) * scales[n, g],
 * u the unsigned nibble k of wq[n, (K+1)/2] (even k in the low nibble), g = k / group_size
 * (one group when group_size <= 0).  Every slot is a DEVICE pointer: fp32 a, fp32 scales and
 * zeros [N, n_groups_per_row], fp32 c.
 *   route  AUTO: a tuned plan for the shape (bybycu_prepare_q4_tuned) where one is installed,
 *          else the decode kernel when it applies (M = 1, group 32, K % 128 == 0, 16-byte
 *          aligned slots: s8 tensor-core MMAs on the raw nibbles, activations in two-digit
 *          fixed point per 32-block), else the tensor-core GEMM when it applies (M > 1,
 *          group 32, K % 256 == 0, 16-byte aligned slots: tcgen05 MMAs on weights and
 *          activations rounded once to fp16), else SIMT; SIMT: one thread per output, fmaf in
 *          k order (the CPU VM's OP_Q4_GEMV arithmetic); GEMV / TC: that kernel, or
 *          BYBYCU_ERR_SHAPE when it does not apply.
 * Asynchronous on `stream`. */
BYBYCU_API int bybycu_matmul_q4(const float* a, const uint8_t* wq, const float* scales, const float* zeros,
                                float* c, int M, int K, int N, int group_size, int n_groups_per_row,
                                int route, void* stream);

/* sessionMatmulQ4 (gpubackend.nim:3000-3060): bybycu_matmul_q4 (route AUTO) into the open
 * session, on its stream.  a, wq, scales, zeros and c are session handles (sessionUpload /
 * sessionAllocScratch: residentUploadQ4 keeps the weights as three of them); each must hold
 * what the shape needs. */
BYBYCU_API int bybycu_session_matmul_q4(const void* a, const void* wq, const void* scales, const void* zeros,
                                        void* c, int M, int K, int N, int group_size, int n_groups_per_row);

/* The fused decode GEMV of asymmetric-Q4 weights (sessionMatmulQ4Fused, gpubackend.nim:3185-3231;
 * its shader q4_autotune.nim:194-325), one launch, M = 1:
 *   mode 0: n_mats (1..3) matrices share `a`; outs[m][0 .. N[m]) = a . W_m^T;
 *   mode 1: n_mats = 2 (gate, up; N[0] == N[1]); outs[0] = silu(a . Wg^T) * (a . Wu^T).
 * With gamma != NULL, a is the raw vector and the product uses RMSNorm(a) = a * gamma /
 * sqrt(mean(a^2) + eps); with res != NULL, res[0 .. N) is added to every output row.  wq, scales,
 * zeros, outs are HOST arrays of n_mats DEVICE pointers; a, res, gamma are device pointers.  The
 * decode kernel of bybycu_matmul_q4 (group 32, K % 128 == 0, 16-byte aligned slots); any other
 * shape returns BYBYCU_ERR_SHAPE, for the caller to run the unfused sequence. */
BYBYCU_API int bybycu_matmul_q4_fused(int mode, const float* a, int n_mats, const uint8_t* const* wq,
                                      const float* const* scales, const float* const* zeros, const int* N,
                                      float* const* outs, const float* res, const float* gamma, float eps,
                                      int K, int group_size, int n_groups_per_row, void* stream);

/* The same into the open session: every pointer is a session handle (wq / scales / zeros of
 * residentUploadQ4); BYBYCU_ERR_SHAPE means unsupported and does not fail the session. */
BYBYCU_API int bybycu_session_matmul_q4_fused(int mode, const void* a, int n_mats, const void* const* wq,
                                              const void* const* scales, const void* const* zeros, const int* N,
                                              void* const* outs, const void* res, const void* gamma, float eps,
                                              int K, int group_size, int n_groups_per_row);

/* ---- weight ingestion ---------------------------------------------------------------- */

/* Maps a checkpoint file read-only (openReadOnlyMapping, mapped_file.nim:10-13): *data and
 * *size describe the whole file, *mapping is the handle for bybycu_unmap_file
 * (unmapReadOnlyFile, mapped_file.nim:15-19).  The mapping outlives nothing it does not own:
 * device copies made from it stay valid after the unmap. */
BYBYCU_API int bybycu_map_file(const char* path, void** data, int64_t* size, void** mapping);
BYBYCU_API int bybycu_unmap_file(void* mapping);

/* Copies `bytes` of host memory - a file mapping or any pageable range - to device memory at
 * dst, and returns when they have landed.  Pageable ranges of 4 MiB and more go through the
 * library's pinned staging slots, several host threads at once (BYBY_CUDA_INGEST_THREADS,
 * default one per host thread, at most 16), so page faults, memcpy and DMA overlap; BYBY_CUDA_INGEST=register pins the
 * range in place instead where the OS allows.  The dGPU branch of residentUploadQ4Mapped
 * (gpubackend.nim:2961-2998): "copied straight from the mapping, never through an
 * intermediate" buffer of the caller's. */
BYBYCU_API int bybycu_upload_host_range(void* dst, const void* src, int64_t bytes);

/* sessionUploadPrivatePtr (gpubackend.nim:2940-2959): a new session handle holding a copy of
 * `bytes` of host memory, by the same engine. */
BYBYCU_API int bybycu_session_upload_ptr(const void* host, int64_t bytes, void** handle);

/* The sampled content identity of fingerprint (probe_data.nim:11-17): "sample1-" and 16 hex
 * digits of FNV-1a over the byte count and five 64-byte runs; out_len >= 25. */
BYBYCU_API int bybycu_fingerprint(const void* data, int64_t bytes, char* out, int out_len);

/* One tensor of a checkpoint index (ProbeTensor, probe_weights.nim:5-9). */
typedef struct bybycu_tensor_info {
    char name[256];          /* truncated when name_len >= 256 */
    int32_t name_len;
    int32_t kind;            /* NIMQ: the tensor's kind byte; NIMBIN: 0; safetensors: 0 for F32, else -1 */
    int32_t rank;            /* <= 8 */
    int32_t scales;          /* NIMQ: number of 8-byte scale entries at scale_offset */
    int64_t shape[8];
    int64_t offset, bytes;   /* the payload's byte range in the file */
    int64_t scale_offset;
    int32_t group_size, eb, mb;   /* NIMQ quantisation fields */
    char dtype[16];          /* safetensors dtype ("F32", "BF16", "U8", ...); "" otherwise */
} bybycu_tensor_info;

/* The tensor index of a NIMQ2, NIMQ3, NIMBIN or .safetensors checkpoint from its headers
 * alone (probeTensorIndex, probe_weights.nim:29-104, with its checks and messages; a
 * safetensors shape of more than 8 dimensions is rejected).  Fills up to cap entries and
 * sets *count to the number of tensors, so a caller may ask with cap = 0 first. */
BYBYCU_API int bybycu_checkpoint_index(const char* path, bybycu_tensor_info* out, int cap, int* count);

/* ---- tuned plans (the Q4 autotuner and its plan cache) ------------------------------ */

/* A launch plan: the route and its knobs.  variant: the operand form of the M = 1 Q4B32 GEMV
 * (0 bf16, 1 fp16, 2 s8 fixed point) or the CTAs per SM of the format-1 GEMV, -1 for the
 * route's default; stages: the ring depth of a GEMV's weight stream, 0 for the default.
 * Replaces VkQ4Plan (backends/vulkan/q4_autotune.nim:2-7). */
typedef struct bybycu_plan {
    int32_t route;     /* BYBYCU_ROUTE_SIMT, _GEMV or _TC */
    int32_t variant;
    int32_t stages;
    float ms;          /* the tuner's median time per launch (0 when set by hand) */
    char name[32];     /* the candidate's name, e.g. "gemv-s8-st2" */
} bybycu_plan;

#define BYBYCU_OP_TILE_GEMM 0   /* bybycu_tile_gemm, plans keyed by format, K, N and M class */
#define BYBYCU_OP_MATMUL_Q4 1   /* bybycu_matmul_q4, keyed by K, N, group, groups and M class */

/* Autotunes the asymmetric-Q4 matmul for these resident weights: every route and ring depth
 * the device supports runs on the weights and the input x[i] = ((17 i) mod 101 - 50) / 64;
 * candidates whose output differs from the exact kernel's by more than max(1e-5, 3e-3 of its
 * peak) are dropped, the rest are timed (three rounds, median; a candidate must be 3% faster
 * to win) and the winner becomes the plan of ROUTE_AUTO calls of this shape on this device.
 * M = 1 tunes the decode plan; M > 1 the plan of M's power-of-two class (2 .. 128, larger M
 * sharing the 128 plan).  Plans persist in <dir>/q4-plans-<hash of device, driver, library
 * build and route switches>.json, dir = BYBY_CUDA_TUNE_DIR (0: no file), else
 * $XDG_CACHE_HOME/bybylang_b200, else ~/.cache/bybylang_b200; a later process reads the plan
 * back instead of tuning.  *prepared = 1 when a plan is installed, 0 when there is nothing to
 * choose or BYBY_Q4_TUNED=0 / BYBY_GPU_AUTOTUNE=0.  Synchronous; allocates scratch (up to
 * ~256 MiB of weight copies that keep the timing out of L2).  Replaces vulkanPrepareQ4Tuned
 * (q4_autotune.nim:387-543), called by residentPrepareQ4 (gpubackend.nim:2871-2881). */
BYBYCU_API int bybycu_prepare_q4_tuned(const uint8_t* wq, const float* scales, const float* zeros,
                                       int M, int K, int N, int group_size, int n_groups_per_row,
                                       int* prepared);

/* The same for the tile GEMM of format `fmt` on device-resident `packed` weights, for
 * activations of type x_dtype (BYBYCU_DT_F32 or _BF16: plans are kept per type).  Format 2:
 * the routes SIMT, GEMV with each operand form and ring depth, TC; format 1: SIMT and the
 * fp16 GEMV with 1-3 CTAs per SM; format 0 has one route and is never prepared. */
BYBYCU_API int bybycu_prepare_tile_gemm_tuned(int fmt, int x_dtype, int M, int K, int N, const void* packed,
                                              int64_t packed_len, int64_t scale_base, int* prepared);

/* The installed plan of a shape on the current device (*found = 0 when none); group_size
 * and n_groups_per_row matter for BYBYCU_OP_MATMUL_Q4 only, fmt and x_dtype for
 * BYBYCU_OP_TILE_GEMM only. */
BYBYCU_API int bybycu_plan_get(int op, int fmt, int x_dtype, int M, int K, int N, int group_size,
                               int n_groups_per_row, bybycu_plan* plan, int* found);
/* Installs `plan` for a shape by hand (NULL removes it); ROUTE_AUTO calls then use it where
 * its route can run the call's arguments. */
BYBYCU_API int bybycu_plan_set(int op, int fmt, int x_dtype, int M, int K, int N, int group_size,
                               int n_groups_per_row, const bybycu_plan* plan);
/* Drops every installed plan (the cache file stays) and zeroes the dispatch count. */
BYBYCU_API int bybycu_plan_clear(void);
/* Installed plans and the ROUTE_AUTO launches that followed one (vulkanQ4TuningStats,
 * q4_autotune.nim:545-546). */
BYBYCU_API int bybycu_tuning_stats(int* prepared_plans, int64_t* tuned_dispatches);
/* The plan cache file of the current device ("" when caching is off). */
BYBYCU_API int bybycu_tune_cache_path(char* buf, int buf_len);

/* Device-pointer twin of nimf_cpu_vm_run_slots (backends/cpu/cpu_kernels.h:118-121,
 * cpu_vm.c:178-182): runs a micro-VM program whose first op is OP_TILE_GEMM (formats
 * 0/1/2, followed by the canonical tile ops), OP_FP4_COOP_GEMM, OP_Q4_GEMV or
 * OP_Q4_COOP_GEMM.  `code` is HOST memory; mem/packed/lut/in_f32 are device slots with the
 * reference's lengths (floats, bytes, floats, floats).  in_f32 = NULL reads x from mem.
 * Any other program returns BYBYCU_ERR_PROGRAM and -1-style message in err. */
BYBYCU_API int bybycu_vm_run_slots(const uint32_t* code, int n_words, float* mem, int mem_len,
                        const uint8_t* packed, int packed_len, const float* lut, int lut_len,
                        const float* in_f32, int in_len, int n_threads, int tg_floats,
                        int tg_size, char* err, int err_len, void* stream);

/* ---- session API (gpubackend.nim:1042-2722, the `cuda` branch) ------------------------ */

/* sessionBegin / sessionEnd (gpubackend.nim:1042, :2422): one open session per host
 * thread on the current device's session stream; End waits for every encoded op and
 * reports the first failure. */
BYBYCU_API int bybycu_session_begin(void);
BYBYCU_API int bybycu_session_end(void);
/* sessionUpload (gpubackend.nim:1133): a device copy of `bytes` host bytes. */
BYBYCU_API int bybycu_session_upload(const void* host, int64_t bytes, void** handle);
/* sessionAllocScratch (gpubackend.nim:1295): n_floats zeroed floats. */
BYBYCU_API int bybycu_session_alloc_scratch(int64_t n_floats, void** handle);
/* sessionRead (gpubackend.nim:2669): copies n_floats back (after sessionEnd). */
BYBYCU_API int bybycu_session_read(const void* handle, float* host, int64_t n_floats);
/* sessionFree (gpubackend.nim:2694). */
BYBYCU_API int bybycu_session_free(void* handle);
/* sessionFp4GemmTensorCore / sessionFp4GemmTiledEnc (gpubackend.nim:1442-1449, :1465-1473):
 * FP4-KM tile GEMM c[M, N] = a[M, K] * W^T with w = nibbles then scale bytes
 * (scaleBase = N*K/2) and the 272-float table at float 0 of lut; a is fp32.
 * tensor_core != 0 takes the tensor-core route, else the FP32 register-tile route. */
BYBYCU_API int bybycu_session_fp4_gemm(const void* a, const void* w, const void* lut, void* c,
                            int M, int K, int N, int tensor_core);
/* sessionF16GemmTile (gpubackend.nim:1475-1482): FP16 weights [N, K]. */
BYBYCU_API int bybycu_session_f16_gemm(const void* a, const void* w, void* c, int M, int K, int N,
                            int tensor_core);
/* Q4B32 weights (format 2; scales [N, K/32] halves right after the nibbles). */
BYBYCU_API int bybycu_session_q4b32_gemm(const void* a, const void* w, void* c, int M, int K, int N,
                              int tensor_core);
/* sessionTileGemmReady (gpubackend.nim:1484-1488 -> vulkanTileGemmReady,
 * vulkan_driver.nim:2681-2762): the exact-data parity gate (M=37, K=128, N=80; K=256 for
 * the tensor-core gate, the smallest K that route tiles; every route that can run it, max
 * rel err <= 1e-3), run once per process and format/route; *ready = 1 when it passed. */
BYBYCU_API int bybycu_tile_gemm_ready(int fmt, int tensor_core, int* ready);

/* ---- peer memory (the plumbing of the device-side all-gather) --------------------------- */

/* Exports the device allocation that holds `dptr` as a 64-byte CUDA IPC handle another
 * process can open, and *offset = the byte offset of dptr inside that allocation (a caching
 * allocator hands out pointers inside larger blocks; the handle always names the whole
 * block).  No reference counterpart: the reference's workers exchange text over pipes
 * (distributed.nim:224-276). */
BYBYCU_API int bybycu_ipc_handle(const void* dptr, uint8_t handle[64], int64_t* offset);
/* Maps a peer process's allocation into this process on the current device (peer access is
 * enabled by the mapping) and returns *dptr = its local base + offset.  Opening the same
 * handle again reuses the mapping; every successful open needs one bybycu_ipc_close. */
BYBYCU_API int bybycu_ipc_open(const uint8_t handle[64], int64_t offset, void** dptr);
BYBYCU_API int bybycu_ipc_close(void* dptr);

/* ---- column sharding (distributed.nim:109-135) ----------------------------------------- */

/* The column range [*n0, *n1) of `rank` among `world` shards of N columns: the
 * largest-remainder split of distributed.nim:109-135 with equal weights, taken over blocks
 * of `align` columns (the last block may be short). */
BYBYCU_API int bybycu_shard_range(int N, int world, int rank, int align, int* n0, int* n1);

/* One rank's share of a column-sharded tile GEMM whose output slices are exchanged in the
 * same kernel: the rank computes out[:, n0:n1) from its shard of W (rows n0..n1 of the
 * packed layout, `packed` pointing at the shard) and stores every element both into its own
 * out and, over NVLink peer pointers, into the `out` buffer of every other rank
 * (peer_out[r] = rank r's out as mapped on this device; peer_out[rank] = out).  It then
 * raises its counter in every rank's signal array (peer_signal[r]: 10 uint32 - one counter
 * per rank, the device-side epoch and a CTA completion counter - zero before first use) and
 * waits, bounded, until every rank's counter for this epoch is present in its own.  On the
 * decode (GEMV) route the GEMV kernel itself stores to the peers and waits, so one launch
 * does the whole step; on the tensor-core route the GEMM's epilogue does the same tile by
 * tile (after the staging pass); other routes add one copy kernel.  A rank may start writing the next call's slices into a peer's out
 * while that peer still reads the previous result: callers that read out while other ranks
 * may already run the next call alternate two sets of buffers.  epoch = 0 keeps the epoch on
 * the device (graph-capturable); epoch > 0 is the caller's count of calls, starting at 1.
 * out is [M, N] fp32 row-major on every rank.  Replaces the gather of text results
 * in runShards (distributed.nim:304-375) with a device-side all-gather. */
BYBYCU_API int bybycu_tile_gemm_allgather(int fmt, int M, int K, int N, int n0, int n1,
                               const void* x, int x_dtype,
                               const void* packed, int64_t packed_len, int64_t scale_base,
                               const float* lut, int64_t lut_len, int64_t lut_base,
                               void* out, void* const* peer_out, uint32_t* const* peer_signal,
                               int world, int rank, uint32_t epoch, void* stream);

/* The same step in split phase (the gather half of distributed.nim:304-375, overlapped with
 * the next step): the launch stores its slices and raises its counters, and does NOT wait
 * for the other ranks.  Instead, before it reads x or stores to a peer, it waits for every
 * rank's previous call, which makes the previous call's output complete on this rank. So
 * x may be the previous call's gathered output.  A step's output is complete after the next
 * split call on this stream has started, or after bybycu_allgather_wait.
 *   Buffers: consecutive calls alternate between two output buffers (and their peer_out
 *   arrays), with one signal array per rank shared by both.  A call writes into the buffers
 *   of two calls ago, whose readers were done when every rank signalled the previous call.
 *   Mixing this and bybycu_tile_gemm_allgather on one signal array is allowed; the counts
 *   stay in step. */
BYBYCU_API int bybycu_tile_gemm_allgather_split(int fmt, int M, int K, int N, int n0, int n1,
                               const void* x, int x_dtype,
                               const void* packed, int64_t packed_len, int64_t scale_base,
                               const float* lut, int64_t lut_len, int64_t lut_base,
                               void* out, void* const* peer_out, uint32_t* const* peer_signal,
                               int world, int rank, uint32_t epoch, void* stream);

/* Completes the last split-phase call on this rank (one small kernel on `stream`): waits,
 * bounded, until every rank's counter reached `epoch` (0: the epoch this rank signalled
 * last).  After it, stream-ordered readers see the whole gathered output. */
BYBYCU_API int bybycu_allgather_wait(uint32_t* const* peer_signal, int world, int rank, uint32_t epoch,
                                     void* stream);

#ifdef __cplusplus
}
#endif
#endif
