// session.cu - the `cuda` branch of BybyLang's session API (gpubackend.nim:1042-2722):
// begin / upload / alloc-scratch / tile-GEMM encoders / end / read / free, and the per-process
// parity gate of sessionTileGemmReady (backends/vulkan/vulkan_driver.nim:2681-2762).
//
// A session is per host thread and per device: its ops are enqueued on one stream, End
// waits for them and reports the first failure (kernel launch errors, CUDA errors and the
// device-side error word).  Handles are device pointers whose sizes are remembered so that
// the encoders can run the size checks of tryTileGemm (vulkan_driver.nim:2617-2619).
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "kernels.h"

namespace bybycu {

int tile_gemm_impl(int fmt, int M, int K, int N, const void* x, int x_dtype, int64_t x_len, const void* packed,
                   int64_t packed_len, int64_t scale_base, const float* lut, int64_t lut_len, int64_t lut_base,
                   void* out, int out_dtype, int64_t out_len, int route, cudaStream_t stream);

namespace {

struct Session {
    bool active = false;
    int device = -1;
    cudaStream_t streams[64] = {};
    int first_error = 0;
    char first_msg[512] = {0};
};
thread_local Session t_sess;

std::mutex g_handles_mu;
std::map<const void*, int64_t> g_handles;   // device pointer -> bytes

int64_t handle_bytes(const void* h) {
    std::lock_guard<std::mutex> lock(g_handles_mu);
    auto it = g_handles.find(h);
    return it == g_handles.end() ? -1 : it->second;
}

int session_note(int rc) {
    if (rc && !t_sess.first_error) {
        t_sess.first_error = rc;
        bybycu_last_error(t_sess.first_msg, sizeof t_sess.first_msg);
    }
    return rc;
}

int session_gemm(int fmt, const void* a, const void* w, const void* lut, void* c, int M, int K, int N,
                 int tensor_core) {
    if (!t_sess.active) return set_error(BYBYCU_ERR_SESSION, "no open session");
    const int64_t ab = handle_bytes(a), wb = handle_bytes(w), cb = handle_bytes(c);
    const int64_t lb = fmt == BYBYCU_FMT_FP4KM ? handle_bytes(lut) : 0;
    if (ab < 0 || wb < 0 || cb < 0 || lb < 0) return set_error(BYBYCU_ERR_ARGS, "unknown session handle");
    if (M <= 0 || N <= 0 || K <= 0) return set_error(BYBYCU_ERR_SHAPE, "unsupported tile GEMM shape K=%d N=%d", K, N);
    const int64_t G = K / 32;
    const int64_t scale_base = fmt == BYBYCU_FMT_F16 ? 0 : static_cast<int64_t>(N) * (K / 2);
    (void)G;
    const int route = tensor_core ? BYBYCU_ROUTE_AUTO : BYBYCU_ROUTE_SIMT;
    return session_note(tile_gemm_impl(fmt, M, K, N, a, BYBYCU_DT_F32, ab / 4, w, wb, scale_base,
                                       static_cast<const float*>(lut), lb / 4, 0, c, BYBYCU_DT_F32, cb / 4, route,
                                       t_sess.streams[t_sess.device]));
}

// ---- the parity gate ------------------------------------------------------------------
struct GateKey {
    int device, fmt, tc;
    bool operator<(const GateKey& o) const {
        return device != o.device ? device < o.device : fmt != o.fmt ? fmt < o.fmt : tc < o.tc;
    }
};
std::mutex g_gate_mu;
std::map<GateKey, int> g_gate;

uint16_t half_bits_exact(float v) {
    __half h = __float2half_rn(v);
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

// The exact-data case of vulkanTileGemmReady (M=37, K=128, N=80): every product and partial
// sum is exact in fp32 (and in fp16 inputs for the tensor-core routes).  The tensor-core gate
// uses K=256, the smallest K that route tiles.
int run_gate(int fmt, int tensor_core, int* ready) {
    constexpr int M = 37, N = 80;
    const int K = tensor_core ? 256 : 128, G = K / 32;
    std::vector<float> x(M * K), table(272, 0.0f), expected(M * N, 0.0f);
    for (int i = 0; i < M * K; ++i) x[i] = static_cast<float>((i * 7 + 3) % 33 - 16) / 64.0f;
    std::vector<uint8_t> w;
    static const float fp4[16] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f, -0.f, -.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};
    std::vector<double> wf(static_cast<size_t>(N) * K);
    if (fmt == BYBYCU_FMT_F16) {
        w.resize(static_cast<size_t>(N) * K * 2);
        for (int i = 0; i < N * K; ++i) {
            const float v = static_cast<float>((i * 5 + 1) % 29 - 14) / 16.0f;
            const uint16_t h = half_bits_exact(v);
            memcpy(&w[2 * i], &h, 2);
            wf[i] = v;
        }
    } else {
        const int nib = N * (K / 2);
        w.resize(static_cast<size_t>(nib) + (fmt == BYBYCU_FMT_FP4KM ? N * G : 2 * N * G));
        for (int i = 0; i < nib; ++i) w[i] = static_cast<uint8_t>((i * 37 + 11) % 256);
        for (int i = 0; i < 16; ++i) table[i] = fp4[i];
        for (int i = 0; i < 256; ++i) table[16 + i] = std::ldexp(1.0f, (i % 5) - 3);
        for (int i = 0; i < N * G; ++i) {
            if (fmt == BYBYCU_FMT_FP4KM) {
                w[nib + i] = static_cast<uint8_t>((i * 13 + 5) % 256);
            } else {
                const uint16_t h = half_bits_exact(std::ldexp(1.0f, (i % 5) - 3));
                memcpy(&w[nib + 2 * i], &h, 2);
            }
        }
        for (int n = 0; n < N; ++n)
            for (int k = 0; k < K; ++k) {
                const int g = k / 32, j = k % 32;
                const uint8_t b = w[n * (K / 2) + g * 16 + (j & 15)];
                const uint32_t nibv = j < 16 ? (b & 15u) : (b >> 4);
                double s, v;
                if (fmt == BYBYCU_FMT_FP4KM) {
                    s = table[16 + w[nib + n * G + g]];
                    v = fp4[nibv];
                } else {
                    s = std::ldexp(1.0, ((n * G + g) % 5) - 3);
                    v = static_cast<double>(static_cast<int>(nibv ^ 8u) - 8);
                }
                wf[static_cast<size_t>(n) * K + k] = v * s;
            }
    }
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            double s = 0.0;
            for (int k = 0; k < K; ++k) s += static_cast<double>(x[m * K + k]) * wf[static_cast<size_t>(n) * K + k];
            expected[m * N + n] = static_cast<float>(s);
        }

    void *dx = nullptr, *dw = nullptr, *dl = nullptr, *dout = nullptr;
    int rc = BYBYCU_OK;
    double worst = 0.0;
    bool ran_any = false;
    std::vector<int> routes;
    if (!tensor_core) routes.push_back(BYBYCU_ROUTE_SIMT);
    else { routes.push_back(BYBYCU_ROUTE_TC); routes.push_back(BYBYCU_ROUTE_GEMV); }
    std::vector<float> got(M * N);
    do {
        if ((rc = bybycu_malloc(&dx, static_cast<int64_t>(x.size()) * 4))) break;
        if ((rc = bybycu_malloc(&dw, static_cast<int64_t>(w.size())))) break;
        if ((rc = bybycu_malloc(&dl, 272 * 4))) break;
        if ((rc = bybycu_malloc(&dout, M * N * 4))) break;
        BYBYCU_CUDA_TRY(cudaMemcpy(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice));
        BYBYCU_CUDA_TRY(cudaMemcpy(dw, w.data(), w.size(), cudaMemcpyHostToDevice));
        BYBYCU_CUDA_TRY(cudaMemcpy(dl, table.data(), 272 * 4, cudaMemcpyHostToDevice));
        for (int route : routes) {
            const int rows = route == BYBYCU_ROUTE_GEMV ? 16 : M;
            const int64_t sb = fmt == BYBYCU_FMT_F16 ? 0 : static_cast<int64_t>(N) * (K / 2);
            BYBYCU_CUDA_TRY(cudaMemset(dout, 0xFF, M * N * 4));
            const int r = tile_gemm_impl(fmt, rows, K, N, dx, BYBYCU_DT_F32, M * K, dw, static_cast<int64_t>(w.size()),
                                         sb, static_cast<const float*>(dl), 272, 0, dout, BYBYCU_DT_F32, M * N, route,
                                         nullptr);
            if (r == BYBYCU_ERR_SHAPE) { clear_error(); continue; }   // the route cannot run this format
            if (r) { rc = r; break; }
            BYBYCU_CUDA_TRY(cudaMemcpy(got.data(), dout, M * N * 4, cudaMemcpyDeviceToHost));
            ran_any = true;
            for (int i = 0; i < rows * N; ++i) {
                const double e = std::fabs(static_cast<double>(got[i]) - expected[i]) /
                                 std::max(1.0, std::fabs(static_cast<double>(expected[i])));
                if (!(e <= worst)) worst = std::isnan(e) ? INFINITY : e;
            }
        }
    } while (false);
    bybycu_free(dx); bybycu_free(dw); bybycu_free(dl); bybycu_free(dout);
    if (rc) return rc;
    int dev_err = 0;
    if ((rc = bybycu_device_error(&dev_err))) return rc;
    *ready = ran_any && dev_err == 0 && worst <= 1e-3;
    fprintf(stderr, "[cuda] tile GEMM micro-kernel check format %d %s: %s (max rel err %.2e)\n", fmt,
            tensor_core ? "tensor core" : "register tiles", *ready ? "ok" : (ran_any ? "FAILED" : "no route"), worst);
    return BYBYCU_OK;
}

}  // namespace
}  // namespace bybycu

using namespace bybycu;

extern "C" {

int bybycu_session_begin(void) {
    if (t_sess.active) return set_error(BYBYCU_ERR_SESSION, "a session is already open on this thread");
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(BYBYCU_ERR_ARGS, "device %d out of range", dev);
    if (!t_sess.streams[dev]) BYBYCU_CUDA_TRY(cudaStreamCreateWithFlags(&t_sess.streams[dev], cudaStreamNonBlocking));
    t_sess.device = dev;
    t_sess.active = true;
    t_sess.first_error = 0;
    t_sess.first_msg[0] = '\0';
    return BYBYCU_OK;
}

int bybycu_session_end(void) {
    if (!t_sess.active) return set_error(BYBYCU_ERR_SESSION, "no open session");
    t_sess.active = false;
    const cudaError_t e = cudaStreamSynchronize(t_sess.streams[t_sess.device]);
    if (e != cudaSuccess) return cuda_fail(e, "sessionEnd");
    int dev_err = 0;
    if (int rc = bybycu_device_error(&dev_err)) return rc;
    if (dev_err) return set_error(BYBYCU_ERR_DEVICE, "a kernel of the session reported device error %d", dev_err);
    if (t_sess.first_error) return set_error(t_sess.first_error, "%s", t_sess.first_msg);
    return BYBYCU_OK;
}

int bybycu_session_upload(const void* host, int64_t bytes, void** handle) {
    if (!handle || bytes <= 0 || !host) return set_error(BYBYCU_ERR_ARGS, "sessionUpload: bad arguments");
    void* d = nullptr;
    BYBYCU_CUDA_TRY(cudaMalloc(&d, static_cast<size_t>(bytes)));
    if (int rc = upload_host_range(d, host, bytes)) {
        cudaFree(d);
        return rc;
    }
    {
        std::lock_guard<std::mutex> lock(g_handles_mu);
        g_handles[d] = bytes;
    }
    *handle = d;
    return BYBYCU_OK;
}

int bybycu_session_upload_ptr(const void* host, int64_t bytes, void** handle) {
    return bybycu_session_upload(host, bytes, handle);
}

int bybycu_session_alloc_scratch(int64_t n_floats, void** handle) {
    if (!handle || n_floats <= 0) return set_error(BYBYCU_ERR_ARGS, "sessionAllocScratch: bad arguments");
    void* d = nullptr;
    BYBYCU_CUDA_TRY(cudaMalloc(&d, static_cast<size_t>(n_floats) * 4));
    const cudaError_t e = cudaMemset(d, 0, static_cast<size_t>(n_floats) * 4);
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(e, "sessionAllocScratch");
    }
    {
        std::lock_guard<std::mutex> lock(g_handles_mu);
        g_handles[d] = n_floats * 4;
    }
    *handle = d;
    return BYBYCU_OK;
}

int bybycu_session_read(const void* handle, float* host, int64_t n_floats) {
    if (!handle || !host || n_floats < 0) return set_error(BYBYCU_ERR_ARGS, "sessionRead: bad arguments");
    const int64_t b = handle_bytes(handle);
    if (b < 0) return set_error(BYBYCU_ERR_ARGS, "sessionRead: unknown handle");
    if (n_floats * 4 > b) return set_error(BYBYCU_ERR_RANGE, "sessionRead: %lld floats from a %lld-byte buffer",
                                           static_cast<long long>(n_floats), static_cast<long long>(b));
    BYBYCU_CUDA_TRY(cudaMemcpy(host, handle, static_cast<size_t>(n_floats) * 4, cudaMemcpyDeviceToHost));
    return BYBYCU_OK;
}

int bybycu_session_free(void* handle) {
    if (!handle) return BYBYCU_OK;
    {
        std::lock_guard<std::mutex> lock(g_handles_mu);
        if (!g_handles.erase(handle)) return set_error(BYBYCU_ERR_ARGS, "sessionFree: unknown handle");
    }
    BYBYCU_CUDA_TRY(cudaFree(handle));
    return BYBYCU_OK;
}

int bybycu_session_fp4_gemm(const void* a, const void* w, const void* lut, void* c, int M, int K, int N,
                            int tensor_core) {
    return session_gemm(BYBYCU_FMT_FP4KM, a, w, lut, c, M, K, N, tensor_core);
}

int bybycu_session_f16_gemm(const void* a, const void* w, void* c, int M, int K, int N, int tensor_core) {
    return session_gemm(BYBYCU_FMT_F16, a, w, nullptr, c, M, K, N, tensor_core);
}

int bybycu_session_q4b32_gemm(const void* a, const void* w, void* c, int M, int K, int N, int tensor_core) {
    return session_gemm(BYBYCU_FMT_Q4B32, a, w, nullptr, c, M, K, N, tensor_core);
}

// sessionMatmulQ4 (gpubackend.nim:3000-3060): the asymmetric-Q4 matmul of resident weights
// (uploaded with sessionUpload, residentUploadQ4's form) into the open session.
int bybycu_session_matmul_q4(const void* a, const void* wq, const void* scales, const void* zeros, void* c, int M,
                             int K, int N, int group_size, int n_groups_per_row) {
    if (!t_sess.active) return set_error(BYBYCU_ERR_SESSION, "no open session");
    const int64_t ab = handle_bytes(a), wb = handle_bytes(wq), sb = handle_bytes(scales), zb = handle_bytes(zeros),
                  cb = handle_bytes(c);
    if (ab < 0 || wb < 0 || sb < 0 || zb < 0 || cb < 0) return set_error(BYBYCU_ERR_ARGS, "unknown session handle");
    if (M <= 0 || K <= 0 || N <= 0 || n_groups_per_row <= 0)
        return set_error(BYBYCU_ERR_SHAPE, "unsupported matmul_q4 shape M=%d K=%d N=%d", M, K, N);
    const int64_t params = static_cast<int64_t>(N) * n_groups_per_row * 4;
    if (ab < static_cast<int64_t>(M) * K * 4 || wb < static_cast<int64_t>(N) * ((K + 1) / 2) || sb < params ||
        zb < params || cb < static_cast<int64_t>(M) * N * 4)
        return session_note(set_error(BYBYCU_ERR_RANGE, "matmul_q4: a slot is smaller than M=%d K=%d N=%d needs", M, K, N));
    return session_note(bybycu_matmul_q4(static_cast<const float*>(a), static_cast<const uint8_t*>(wq),
                                         static_cast<const float*>(scales), static_cast<const float*>(zeros),
                                         static_cast<float*>(c), M, K, N, group_size, n_groups_per_row,
                                         BYBYCU_ROUTE_AUTO, t_sess.streams[t_sess.device]));
}

// sessionMatmulQ4Fused (gpubackend.nim:3185-3231): the fused decode GEMV of resident
// asymmetric-Q4 weights into the open session.  BYBYCU_ERR_SHAPE (not recorded as a session
// error) means "unsupported here": the caller runs the unfused sequence, as the reference does.
int bybycu_session_matmul_q4_fused(int mode, const void* a, int n_mats, const void* const* wq,
                                   const void* const* scales, const void* const* zeros, const int* N,
                                   void* const* outs, const void* res, const void* gamma, float eps, int K,
                                   int group_size, int n_groups_per_row) {
    if (!t_sess.active) return set_error(BYBYCU_ERR_SESSION, "no open session");
    if (!a || !wq || !scales || !zeros || !N || !outs || n_mats < 1 || n_mats > 3 || K <= 0 || n_groups_per_row <= 0)
        return set_error(BYBYCU_ERR_ARGS, "sessionMatmulQ4Fused: bad arguments");
    auto fits = [](const void* h, int64_t need) { const int64_t b = handle_bytes(h); return b >= need; };
    if (!fits(a, static_cast<int64_t>(K) * 4) || (res && !fits(res, static_cast<int64_t>(N[0]) * 4)) ||
        (gamma && !fits(gamma, static_cast<int64_t>(K) * 4)))
        return set_error(BYBYCU_ERR_RANGE, "sessionMatmulQ4Fused: a, res or gamma is not a large enough session handle");
    const uint8_t* w8[3] = {};
    const float* sc[3] = {};
    const float* zr[3] = {};
    float* out[3] = {};
    for (int m = 0; m < n_mats; ++m) {
        const int64_t params = static_cast<int64_t>(N[m]) * n_groups_per_row * 4;
        if (N[m] <= 0 || !fits(wq[m], static_cast<int64_t>(N[m]) * ((K + 1) / 2)) || !fits(scales[m], params) ||
            !fits(zeros[m], params) || !fits(outs[m], static_cast<int64_t>(N[m]) * 4))
            return set_error(BYBYCU_ERR_RANGE, "sessionMatmulQ4Fused: matrix %d's handles are too small", m);
        w8[m] = static_cast<const uint8_t*>(wq[m]);
        sc[m] = static_cast<const float*>(scales[m]);
        zr[m] = static_cast<const float*>(zeros[m]);
        out[m] = static_cast<float*>(outs[m]);
    }
    const int rc = bybycu_matmul_q4_fused(mode, static_cast<const float*>(a), n_mats, w8, sc, zr, N, out,
                                          static_cast<const float*>(res), static_cast<const float*>(gamma), eps, K,
                                          group_size, n_groups_per_row, t_sess.streams[t_sess.device]);
    return rc == BYBYCU_ERR_SHAPE ? rc : session_note(rc);
}

int bybycu_tile_gemm_ready(int fmt, int tensor_core, int* ready) {
    if (!ready) return set_error(BYBYCU_ERR_ARGS, "ready is NULL");
    if (fmt < 0 || fmt > 2) return set_error(BYBYCU_ERR_SHAPE, "tile GEMM weight format %d is not supported", fmt);
    if (t_sess.active) {
        // vulkanTileGemmReady: not checked yet and a session is open -> not ready
        std::lock_guard<std::mutex> lock(g_gate_mu);
        int dev = 0;
        cudaGetDevice(&dev);
        auto it = g_gate.find({dev, fmt, tensor_core ? 1 : 0});
        *ready = it == g_gate.end() ? 0 : it->second;
        return BYBYCU_OK;
    }
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    const GateKey key{dev, fmt, tensor_core ? 1 : 0};
    {
        std::lock_guard<std::mutex> lock(g_gate_mu);
        auto it = g_gate.find(key);
        if (it != g_gate.end()) {
            *ready = it->second;
            return BYBYCU_OK;
        }
    }
    int r = 0;
    if (int rc = run_gate(fmt, tensor_core, &r)) return rc;
    std::lock_guard<std::mutex> lock(g_gate_mu);
    g_gate[key] = r;
    *ready = r;
    return BYBYCU_OK;
}

}  // extern "C"
