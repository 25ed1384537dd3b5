// f16gemv.cu - the decode route (M <= 8) of the tile GEMM for format 1: fp16 weights W[N, K],
// row-major (buildF16TileGemmProgram, micro_kernel/session_vm.nim:400-416; the CPU VM's
// OP_TILE_LOAD_B_F16, backends/cpu/cpu_vm.c:550-581):  out[m, n] = sum_k x[m, k] * W[n, k].
//
// At 2 bytes per weight the job is the weight stream and nothing else: every warp owns four
// rows at a time and walks K with 16-byte loads (eight halves per lane, 512 contiguous bytes
// per row per warp step), all four rows' loads in flight together; the activations sit in
// shared memory as fp32 (one copy per CTA), and each lane's partial sums end in a warp
// reduction.  fp32 FMAs on the CUDA cores keep up with HBM (the stream needs ~11 weights per
// SM cycle against 128 FMA lanes), so no tensor-core path is needed.  The sums run in a
// different order from the reference's k-order fmaf: the route's tolerance applies, as for
// every fast route (the SIMT route stays the bit-exact one).
#include "kernels.h"

namespace bybycu {
namespace {

constexpr int kF16Rows = 4;        // rows per warp in flight
constexpr int kF16Warps = 16;      // warps per CTA
constexpr int kF16MaxM = 8;
constexpr int kF16Unroll = 2;    // K steps whose loads are in flight together

// MMAX activation rows at most; rows m >= M are skipped (warp-uniform).
template <int MMAX, bool XBF16, bool OUTBF16>
__global__ void __launch_bounds__(kF16Warps * 32) f16_gemv_kernel(const __half* __restrict__ w, const void* __restrict__ x,
                                                                  void* __restrict__ out, int M, int K, int N,
                                                                  int64_t out_ld, int64_t out_col0) {
    extern __shared__ __align__(16) float xs[];   // [M][K]
    pdl_launch_dependents();
    pdl_wait();   // the activations may come from the previous kernel
    for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
        float v;
        if constexpr (XBF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]);
        else v = static_cast<const float*>(x)[i];
        xs[i] = v;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int groups = (N + kF16Rows - 1) / kF16Rows;
    for (int grp = blockIdx.x * kF16Warps + warp; grp < groups; grp += gridDim.x * kF16Warps) {
        const int n0 = grp * kF16Rows;
        float acc[kF16Rows][MMAX];
#pragma unroll
        for (int r = 0; r < kF16Rows; ++r)
#pragma unroll
            for (int m = 0; m < MMAX; ++m) acc[r][m] = 0.0f;
        const uint4* rows[kF16Rows];
#pragma unroll
        for (int r = 0; r < kF16Rows; ++r)
            rows[r] = reinterpret_cast<const uint4*>(w + static_cast<int64_t>(min(n0 + r, N - 1)) * K);
        // two 16-byte loads per row in flight per lane (eight per lane in all): the stream is
        // bound by DRAM latency, so every load issued before the first FMA counts
        for (int k8 = lane; k8 < K / 8; k8 += 32 * kF16Unroll) {
            uint4 v[kF16Unroll][kF16Rows];
#pragma unroll
            for (int u = 0; u < kF16Unroll; ++u)
#pragma unroll
                for (int r = 0; r < kF16Rows; ++r)
                    v[u][r] = k8 + 32 * u < K / 8 ? __ldcs(rows[r] + k8 + 32 * u) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int u = 0; u < kF16Unroll; ++u) {
                const int kk = k8 + 32 * u;
                if (kk >= K / 8) break;
#pragma unroll
                for (int m = 0; m < MMAX; ++m) {
                    if (m >= M) break;
                    const float4 xa = *reinterpret_cast<const float4*>(xs + m * K + 8 * kk);
                    const float4 xb = *reinterpret_cast<const float4*>(xs + m * K + 8 * kk + 4);
#pragma unroll
                    for (int r = 0; r < kF16Rows; ++r) {
                        const uint32_t wv[4] = {v[u][r].x, v[u][r].y, v[u][r].z, v[u][r].w};
                        float2 f;
                        f = __half22float2(*reinterpret_cast<const __half2*>(&wv[0]));
                        acc[r][m] = fmaf(f.x, xa.x, acc[r][m]);
                        acc[r][m] = fmaf(f.y, xa.y, acc[r][m]);
                        f = __half22float2(*reinterpret_cast<const __half2*>(&wv[1]));
                        acc[r][m] = fmaf(f.x, xa.z, acc[r][m]);
                        acc[r][m] = fmaf(f.y, xa.w, acc[r][m]);
                        f = __half22float2(*reinterpret_cast<const __half2*>(&wv[2]));
                        acc[r][m] = fmaf(f.x, xb.x, acc[r][m]);
                        acc[r][m] = fmaf(f.y, xb.y, acc[r][m]);
                        f = __half22float2(*reinterpret_cast<const __half2*>(&wv[3]));
                        acc[r][m] = fmaf(f.x, xb.z, acc[r][m]);
                        acc[r][m] = fmaf(f.y, xb.w, acc[r][m]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kF16Rows; ++r)
#pragma unroll
            for (int m = 0; m < MMAX; ++m) {
                float v = acc[r][m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                acc[r][m] = v;
            }
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < kF16Rows; ++r) {
                if (n0 + r >= N) break;
#pragma unroll
                for (int m = 0; m < MMAX; ++m) {
                    if (m >= M) break;
                    const int64_t oi = m * out_ld + out_col0 + n0 + r;
                    if constexpr (OUTBF16) static_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(acc[r][m]);
                    else static_cast<float*>(out)[oi] = acc[r][m];
                }
            }
        }
    }
}

template <int MMAX>
int launch_f16_m(const GemmArgs& a, int grid, size_t smem) {
    const bool xb = a.x_dtype == BYBYCU_DT_BF16, ob = a.out_dtype == BYBYCU_DT_BF16;
    auto kern = xb ? (ob ? f16_gemv_kernel<MMAX, true, true> : f16_gemv_kernel<MMAX, true, false>)
                   : (ob ? f16_gemv_kernel<MMAX, false, true> : f16_gemv_kernel<MMAX, false, false>);
    if (smem > 48 * 1024) BYBYCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                               static_cast<int>(smem)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kF16Warps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    BYBYCU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const __half*>(a.packed), a.x, a.out, a.M, a.K,
                                       a.N, a.out_ld, a.out_col0));
    BYBYCU_LAUNCH_CHECK("f16_gemv_kernel");
    return BYBYCU_OK;
}

}  // namespace

bool f16_gemv_supports(const GemmArgs& a) {
    if (a.fmt != BYBYCU_FMT_F16 || a.M < 1 || a.M > kF16MaxM || a.K % 32 != 0 || a.N < 1) return false;
    if (reinterpret_cast<uintptr_t>(a.packed) & 15u) return false;   // 16-byte weight loads
    if (reinterpret_cast<uintptr_t>(a.x) & 3u) return false;
    DeviceInfo info;
    if (current_device_info(&info) != BYBYCU_OK) return false;
    return static_cast<int64_t>(a.M) * a.K * 4 <= info.max_smem_optin;   // the activations fit in shared memory
}

int launch_f16_gemv(const GemmArgs& a) {
    DeviceInfo dev;
    if (int rc = current_device_info(&dev)) return rc;
    const size_t smem = static_cast<size_t>(a.M) * a.K * 4;
    // CTAs per SM: as many as the activation copy and 48 warps allow (or a tuned plan's count,
    // a.variant, within that), and no more than the rows need
    int per_sm = std::max(1, std::min(3, static_cast<int>(dev.max_smem_optin / std::max<size_t>(smem, 1))));
    if (a.variant >= 1) per_sm = std::min(per_sm, a.variant);
    const int groups = static_cast<int>(ceil_div(a.N, kF16Rows));
    const int grid = std::max(1, std::min(dev.sm_count * per_sm, static_cast<int>(ceil_div(groups, kF16Warps))));
    if (a.M == 1) return launch_f16_m<1>(a, grid, smem);
    if (a.M == 2) return launch_f16_m<2>(a, grid, smem);
    if (a.M <= 4) return launch_f16_m<4>(a, grid, smem);
    return launch_f16_m<8>(a, grid, smem);
}

}  // namespace bybycu
