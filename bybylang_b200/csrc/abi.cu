// abi.cu - the extern "C" boundary of libbybycuda.so: status reporting, device memory,
// the tile-GEMM op with the reference's shape and range checks, route selection and the
// device-pointer twin of the CPU micro-VM entry point.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kernels.h"

namespace bybycu {

namespace {
struct ErrorState {
    int code = 0;
    char msg[512] = {0};
};
thread_local ErrorState t_err;
}  // namespace

int set_error(int code, const char* fmt, ...) {
    t_err.code = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err.msg, sizeof t_err.msg, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return set_error(BYBYCU_ERR_CUDA, "CUDA error %d (%s) in %s", static_cast<int>(e), cudaGetErrorString(e), what);
}

void clear_error() {
    t_err.code = 0;
    t_err.msg[0] = '\0';
}

int current_device_info(DeviceInfo* info) {
    int dev = -1;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    static DeviceInfo cache[64];
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && cache[dev].device == dev) {
        *info = cache[dev];
        return BYBYCU_OK;
    }
    DeviceInfo d;
    d.device = dev;
    BYBYCU_CUDA_TRY(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
    BYBYCU_CUDA_TRY(cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    BYBYCU_CUDA_TRY(cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    BYBYCU_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev));
    BYBYCU_CUDA_TRY(cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (dev >= 0 && dev < 64) cache[dev] = d;
    *info = d;
    return BYBYCU_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        BYBYCU_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p)
            return set_error(BYBYCU_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(BYBYCU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu box %u x %u",
                         static_cast<int>(r), static_cast<unsigned long long>(inner),
                         static_cast<unsigned long long>(outer), box_inner, box_outer);
    return BYBYCU_OK;
}

// ---------------------------------------------------------------------------------------
// Shape and slot checks of one tile-GEMM op.  The messages follow the reference's:
// tileGemmShape (micro_kernel/tile_gemm.nim:68-80) and the CPU VM's range checks
// (backends/cpu/cpu_vm.c:541-604).
// ---------------------------------------------------------------------------------------
int check_tile_gemm(int fmt, int M, int K, int N, int64_t x_len, int64_t packed_len, int64_t scale_base,
                    int64_t lut_len, int64_t lut_base, int64_t out_len) {
    if (fmt < 0 || fmt > 2)
        return set_error(BYBYCU_ERR_SHAPE,
                         "tile GEMM weight format %d is not supported (0 = FP4-KM, 1 = FP16, 2 = Q4B32)", fmt);
    if (K <= 0 || K % 32 != 0 || N <= 0)
        return set_error(BYBYCU_ERR_SHAPE, "unsupported tile GEMM shape K=%d N=%d", K, N);
    if (M <= 0) return set_error(BYBYCU_ERR_SHAPE, "unsupported tile GEMM row count M=%d", M);
    const int64_t G = K / 32;
    bool ok = static_cast<int64_t>(M) * K <= x_len && static_cast<int64_t>(M) * N <= out_len;
    if (fmt == BYBYCU_FMT_FP4KM) {
        ok = ok && scale_base >= 0 && lut_base >= 0 && static_cast<int64_t>(N) * (K / 2) <= packed_len &&
             scale_base + static_cast<int64_t>(N) * G <= packed_len && lut_base + 272 <= lut_len;
    } else if (fmt == BYBYCU_FMT_F16) {
        ok = ok && static_cast<int64_t>(N) * K * 2 <= packed_len;
    } else {
        if (scale_base & 1) return set_error(BYBYCU_ERR_SHAPE, "Q4B32 scale block must start on an even byte");
        ok = ok && scale_base >= 0 && static_cast<int64_t>(N) * (K / 2) <= packed_len &&
             scale_base + static_cast<int64_t>(N) * G * 2 <= packed_len;
    }
    if (!ok) return set_error(BYBYCU_ERR_RANGE, "tile GEMM input out of range");
    return BYBYCU_OK;
}

int choose_route(const GemmArgs& a, int requested, int* route) {
    if (requested == BYBYCU_ROUTE_SIMT) { *route = BYBYCU_ROUTE_SIMT; return BYBYCU_OK; }
    if (requested == BYBYCU_ROUTE_GEMV) {
        if (!gemv_supports(a))
            return set_error(BYBYCU_ERR_SHAPE, "GEMV route needs format 2 (M <= 32) or format 1 (M <= 8) and "
                                               "16-byte aligned slots");
        *route = BYBYCU_ROUTE_GEMV;
        return BYBYCU_OK;
    }
    if (requested == BYBYCU_ROUTE_TC || requested == BYBYCU_ROUTE_TC_FP16W) {
        if (!tc_supports(a) || (requested == BYBYCU_ROUTE_TC_FP16W && a.fmt != BYBYCU_FMT_Q4B32))
            return set_error(BYBYCU_ERR_SHAPE, "tensor-core route cannot run format %d M=%d K=%d N=%d", a.fmt, a.M,
                             a.K, a.N);
        *route = requested;
        return BYBYCU_OK;
    }
    if (requested != BYBYCU_ROUTE_AUTO) return set_error(BYBYCU_ERR_ARGS, "unknown route %d", requested);
    // GEMV up to 16 rows, the tensor cores above (fp32 rows enter them as two fp16 terms: C1,
    // 32 fp32 rows of 4096 x 4096, 19.3 us against 28.3 on the GEMV, measured on one B200).
    // Except where the GEMV's cost per row is highest: rows from 8 on with K >= 8192
    // (4096 x 11008 at M = 16: 21.9 us on the tensor cores against 31.9 for bf16 rows, 24.1
    // against 35.7 for fp32 rows; at M = 8 21.8 against 22.6 and 22.4 against 24.5; at M = 4
    // the GEMV wins), and from 12 on with N >= 65536 (128256 x 4096 at M = 16: 120 against
    // 158 us for bf16 rows, 129 against 182 for fp32 rows; fp32 rows at M = 8: 124 against 112).
    const bool tc_rows = a.fmt == BYBYCU_FMT_Q4B32 && a.M >= 8 && a.M <= 16 &&
                         (a.K >= 8192 || (a.M >= 12 && a.N >= 65536));
    const bool gemv_rows = !tc_rows && a.M <= 16;
    if (gemv_rows && gemv_supports(a)) *route = BYBYCU_ROUTE_GEMV;
    else if (tc_supports(a)) *route = BYBYCU_ROUTE_TC;
    else if (gemv_supports(a)) *route = BYBYCU_ROUTE_GEMV;
    else *route = BYBYCU_ROUTE_SIMT;
    return BYBYCU_OK;
}

int run_gemm(const GemmArgs& a, int route) {
    switch (route) {
        case BYBYCU_ROUTE_GEMV: return launch_gemv(a);
        case BYBYCU_ROUTE_TC: return launch_tc(a);
        case BYBYCU_ROUTE_TC_FP16W: return launch_tc(a, true);
        default: return launch_simt(a);
    }
}

int tile_gemm_impl(int fmt, int M, int K, int N, const void* x, int x_dtype, int64_t x_len, const void* packed,
                   int64_t packed_len, int64_t scale_base, const float* lut, int64_t lut_len, int64_t lut_base,
                   void* out, int out_dtype, int64_t out_len, int route, cudaStream_t stream) {
    if (!x || !packed || !out || (fmt == BYBYCU_FMT_FP4KM && !lut))
        return set_error(BYBYCU_ERR_ARGS, "tile GEMM slot is missing");
    if ((x_dtype != BYBYCU_DT_F32 && x_dtype != BYBYCU_DT_BF16) ||
        (out_dtype != BYBYCU_DT_F32 && out_dtype != BYBYCU_DT_BF16))
        return set_error(BYBYCU_ERR_ARGS, "tile GEMM element types must be F32 or BF16");
    if (int rc = check_tile_gemm(fmt, M, K, N, x_len, packed_len, scale_base, lut_len, lut_base, out_len)) return rc;
    GemmArgs a;
    a.fmt = fmt; a.M = M; a.K = K; a.N = N;
    a.x = x; a.x_dtype = x_dtype;
    a.packed = static_cast<const uint8_t*>(packed);
    a.packed_len = packed_len;
    a.scale_base = scale_base;
    a.lut = lut ? lut + lut_base : nullptr;
    a.out = out; a.out_dtype = out_dtype;
    a.out_ld = N; a.out_col0 = 0;
    a.stream = stream;
    if (route == BYBYCU_ROUTE_AUTO) apply_tile_gemm_plan(&a, &route);
    int r = 0;
    if (int rc = choose_route(a, route, &r)) return rc;
    return run_gemm(a, r);
}

}  // namespace bybycu

using namespace bybycu;

extern "C" {

int bybycu_version(void) { return BYBYCU_ABI_VERSION; }

int bybycu_last_error(char* buf, int buf_len) {
    if (buf && buf_len > 0) snprintf(buf, static_cast<size_t>(buf_len), "%s", t_err.msg);
    return t_err.code;
}

int bybycu_device_count(int* count) {
    if (!count) return set_error(BYBYCU_ERR_ARGS, "count is NULL");
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        *count = 0;
        return BYBYCU_OK;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    *count = n;
    return BYBYCU_OK;
}

int bybycu_init(int device) {
    int n = 0;
    if (int rc = bybycu_device_count(&n)) return rc;
    if (n == 0) return set_error(BYBYCU_ERR_NODEV, "no CUDA device");
    if (device < 0 || device >= n) return set_error(BYBYCU_ERR_ARGS, "device %d out of range (%d devices)", device, n);
    BYBYCU_CUDA_TRY(cudaSetDevice(device));
    DeviceInfo d;
    if (int rc = current_device_info(&d)) return rc;
    if (d.cc_major != 10)
        return set_error(BYBYCU_ERR_NODEV, "device %d is sm_%d%d; this library is built for sm_100a", device, d.cc_major,
                         d.cc_minor);
    // the static-scratch route allocates nothing after this: its module memory is loaded now;
    // the tensor-core routes' scratch pool and launch attributes are set up too, so that a
    // first call may be captured into a CUDA graph
    return tc_static_scratch_load();
}

int bybycu_malloc(void** dptr, int64_t bytes) {
    if (!dptr || bytes < 0) return set_error(BYBYCU_ERR_ARGS, "bybycu_malloc: bad arguments");
    *dptr = nullptr;
    if (bytes == 0) return BYBYCU_OK;
    BYBYCU_CUDA_TRY(cudaMalloc(dptr, static_cast<size_t>(bytes)));
    return BYBYCU_OK;
}

int bybycu_free(void* dptr) {
    if (dptr) BYBYCU_CUDA_TRY(cudaFree(dptr));
    return BYBYCU_OK;
}

int bybycu_upload(void* dst, const void* src, int64_t bytes, void* stream) {
    if (bytes < 0 || (bytes > 0 && (!dst || !src))) return set_error(BYBYCU_ERR_ARGS, "bybycu_upload: bad arguments");
    if (bytes) BYBYCU_CUDA_TRY(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyHostToDevice,
                                               static_cast<cudaStream_t>(stream)));
    return BYBYCU_OK;
}

int bybycu_download(void* dst, const void* src, int64_t bytes, void* stream) {
    if (bytes < 0 || (bytes > 0 && (!dst || !src))) return set_error(BYBYCU_ERR_ARGS, "bybycu_download: bad arguments");
    if (bytes) BYBYCU_CUDA_TRY(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToHost,
                                               static_cast<cudaStream_t>(stream)));
    return BYBYCU_OK;
}

int bybycu_memset(void* dst, int value, int64_t bytes, void* stream) {
    if (bytes < 0 || (bytes > 0 && !dst)) return set_error(BYBYCU_ERR_ARGS, "bybycu_memset: bad arguments");
    if (bytes) BYBYCU_CUDA_TRY(cudaMemsetAsync(dst, value, static_cast<size_t>(bytes), static_cast<cudaStream_t>(stream)));
    return BYBYCU_OK;
}

int bybycu_stream_create(void** stream) {
    if (!stream) return set_error(BYBYCU_ERR_ARGS, "stream is NULL");
    cudaStream_t s;
    BYBYCU_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = s;
    return BYBYCU_OK;
}

int bybycu_stream_destroy(void* stream) {
    if (stream) BYBYCU_CUDA_TRY(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
    return BYBYCU_OK;
}

int bybycu_synchronize(void* stream) {
    BYBYCU_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    return BYBYCU_OK;
}

int bybycu_device_error(int* code) {
    if (!code) return set_error(BYBYCU_ERR_ARGS, "code is NULL");
    BYBYCU_CUDA_TRY(cudaDeviceSynchronize());
    uint32_t v = 0;
    BYBYCU_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_error, sizeof v));
    const uint32_t zero = 0;
    BYBYCU_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero));
    *code = static_cast<int>(v);
    return BYBYCU_OK;
}

int bybycu_tile_gemm(int fmt, int M, int K, int N, const void* x, int x_dtype, int64_t x_len, const void* packed,
                     int64_t packed_len, int64_t scale_base, const float* lut, int64_t lut_len, int64_t lut_base,
                     void* out, int out_dtype, int64_t out_len, int route, void* stream) {
    return tile_gemm_impl(fmt, M, K, N, x, x_dtype, x_len, packed, packed_len, scale_base, lut, lut_len, lut_base, out,
                          out_dtype, out_len, route, static_cast<cudaStream_t>(stream));
}

int bybycu_tile_gemm_noalloc(int M, int K, int N, const void* x, int x_dtype, int64_t x_len, const void* packed,
                             int64_t packed_len, int64_t scale_base, void* out, int out_dtype, int64_t out_len,
                             void* stream) {
    if (!x || !packed || !out) return set_error(BYBYCU_ERR_ARGS, "tile GEMM slot is missing");
    if ((x_dtype != BYBYCU_DT_F32 && x_dtype != BYBYCU_DT_BF16) ||
        (out_dtype != BYBYCU_DT_F32 && out_dtype != BYBYCU_DT_BF16))
        return set_error(BYBYCU_ERR_ARGS, "tile GEMM element types must be F32 or BF16");
    if (int rc = check_tile_gemm(BYBYCU_FMT_Q4B32, M, K, N, x_len, packed_len, scale_base, 0, 0, out_len)) return rc;
    GemmArgs a;
    a.fmt = BYBYCU_FMT_Q4B32; a.M = M; a.K = K; a.N = N;
    a.x = x; a.x_dtype = x_dtype;
    a.packed = static_cast<const uint8_t*>(packed);
    a.packed_len = packed_len;
    a.scale_base = scale_base;
    a.out = out; a.out_dtype = out_dtype;
    a.out_ld = N; a.out_col0 = 0;
    a.stream = static_cast<cudaStream_t>(stream);
    return launch_tc_static_scratch(a);
}

int bybycu_tile_gemm_host(int fmt, int M, int K, int N, const void* x_host, int x_dtype, const void* packed,
                          int64_t packed_len, int64_t scale_base, const float* lut, int64_t lut_len, int64_t lut_base,
                          void* out_host, int out_dtype, void* x_dev, void* out_dev, int route, void* stream) {
    if (!x_host || !out_host || !x_dev || !out_dev) return set_error(BYBYCU_ERR_ARGS, "tile GEMM host slot is missing");
    if (M <= 0 || K <= 0 || N <= 0) return set_error(BYBYCU_ERR_SHAPE, "unsupported tile GEMM shape K=%d N=%d", K, N);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t xb = static_cast<int64_t>(M) * K * (x_dtype == BYBYCU_DT_BF16 ? 2 : 4);
    const int64_t ob = static_cast<int64_t>(M) * N * (out_dtype == BYBYCU_DT_BF16 ? 2 : 4);
    // Page-locked, mapped host output: the kernel stores the result straight into it over
    // PCIe (no device-to-host copy, no copy-engine latency); otherwise out_dev and a copy.
    void* out_target = out_dev;
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, out_host) == cudaSuccess && pa.type == cudaMemoryTypeHost && pa.devicePointer)
        out_target = pa.devicePointer;
    else
        cudaGetLastError();   // a pageable pointer is not an error here
    BYBYCU_CUDA_TRY(cudaMemcpyAsync(x_dev, x_host, static_cast<size_t>(xb), cudaMemcpyHostToDevice, s));
    if (int rc = tile_gemm_impl(fmt, M, K, N, x_dev, x_dtype, static_cast<int64_t>(M) * K, packed, packed_len,
                                scale_base, lut, lut_len, lut_base, out_target, out_dtype, static_cast<int64_t>(M) * N,
                                route, s))
        return rc;
    if (out_target == out_dev)
        BYBYCU_CUDA_TRY(cudaMemcpyAsync(out_host, out_dev, static_cast<size_t>(ob), cudaMemcpyDeviceToHost, s));
    // Poll rather than block: a blocking wait can add the host thread's wake-up latency to
    // every step of a latency-bound decode loop.
    cudaError_t q;
    while ((q = cudaStreamQuery(s)) == cudaErrorNotReady) {
    }
    BYBYCU_CUDA_TRY(q);
    return BYBYCU_OK;
}

int bybycu_dequant(int fmt, int K, int N, const void* packed, int64_t packed_len, int64_t scale_base, const float* lut,
                   int64_t lut_len, int64_t lut_base, float* w_out, void* stream) {
    if (!packed || !w_out || (fmt == BYBYCU_FMT_FP4KM && !lut)) return set_error(BYBYCU_ERR_ARGS, "dequant slot is missing");
    if (int rc = check_tile_gemm(fmt, 1, K, N, K, packed_len, scale_base, lut_len, lut_base, N)) return rc;
    return launch_dequant(fmt, K, N, static_cast<const uint8_t*>(packed), scale_base, lut ? lut + lut_base : nullptr,
                          w_out, static_cast<cudaStream_t>(stream));
}

int bybycu_route_for(int fmt, int M, int K, int N, int x_dtype, int* route) {
    if (!route) return set_error(BYBYCU_ERR_ARGS, "route is NULL");
    if (int rc = check_tile_gemm(fmt, M, K, N, INT64_MAX, INT64_MAX / 4, 0, INT64_MAX / 4, 0, INT64_MAX)) return rc;
    GemmArgs a;
    a.fmt = fmt; a.M = M; a.K = K; a.N = N; a.x_dtype = x_dtype;
    static const uint8_t* const aligned = reinterpret_cast<const uint8_t*>(uintptr_t(1) << 20);
    a.packed = aligned; a.x = aligned; a.out = const_cast<uint8_t*>(aligned);
    int requested = BYBYCU_ROUTE_AUTO;
    apply_tile_gemm_plan(&a, &requested);
    return choose_route(a, requested, route);
}

}  // extern "C"
