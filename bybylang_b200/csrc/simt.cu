// simt.cu - the CUDA-core FP32 route of the tile GEMM (the register-tile lowering's job,
// micro_kernel/tile_gemm.nim:444-541, for every format) and the dequantisation kernel.
//
// It is the route that runs every format and every K % 32 == 0 shape, and the one whose
// results are bit-identical to the reference CPU VM; it is not a fast route.
#include "kernels.h"

namespace bybycu {

namespace {

__device__ __forceinline__ float signed_nibble(uint32_t nib) {
    return static_cast<float>(static_cast<int>(nib ^ 8u) - 8);
}

// Decodes block c of weight row n into w[32] (w[j] is element k = 32c + j).
template <int FMT>
__device__ __forceinline__ void decode_block(const uint8_t* __restrict__ packed, int64_t scale_base,
                                             const float* __restrict__ lut, int K, int64_t n, int c,
                                             float* w) {
    const int G = K >> 5;
    if constexpr (FMT == BYBYCU_FMT_F16) {
        const __half* h = reinterpret_cast<const __half*>(packed) + n * K + 32 * c;
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = __half2float(h[j]);
    } else {
        const uint8_t* b = packed + n * (K >> 1) + 16 * c;
        uint8_t bytes[16];
        if ((reinterpret_cast<uintptr_t>(b) & 15u) == 0) {
            const uint4 v = *reinterpret_cast<const uint4*>(b);
            const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 16; ++i) bytes[i] = (words[i >> 2] >> (8 * (i & 3))) & 0xFFu;
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) bytes[i] = b[i];
        }
        float s;
        if constexpr (FMT == BYBYCU_FMT_FP4KM) {
            s = lut[16 + packed[scale_base + n * G + c]];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                w[j] = lut[bytes[j] & 15u] * s;
                w[16 + j] = lut[bytes[j] >> 4] * s;
            }
        } else {
            const __half* sc = reinterpret_cast<const __half*>(packed + scale_base);
            s = __half2float(sc[n * G + c]);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                w[j] = signed_nibble(bytes[j] & 15u) * s;
                w[16 + j] = signed_nibble(bytes[j] >> 4) * s;
            }
        }
    }
}

template <bool XBF16>
__device__ __forceinline__ float load_x(const void* x, int64_t i) {
    if constexpr (XBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
    else return reinterpret_cast<const float*>(x)[i];
}

// One thread per output element (m, n), summing in exactly the CPU VM's order: per block
// the 16 low nibbles then the 16 high nibbles, one fmaf each, the weight formed first as
// one fp32 product (backends/cpu/cpu_vm.c:605-626 for formats 0/2, :571-576 for format 1).
// The result is bit-identical to nimf_cpu_vm_run_slots on the same inputs.
template <int FMT, bool XBF16>
__global__ void __launch_bounds__(128)
simt_tile_gemm_kernel(GemmArgs a) {
    const int64_t n = static_cast<int64_t>(blockIdx.x) * 128 + threadIdx.x;
    const int64_t m = blockIdx.y;
    if (n >= a.N) return;
    const int K = a.K, G = K >> 5;
    const int64_t xo = m * K;
    float sum = 0.0f;
    for (int c = 0; c < G; ++c) {
        float w[32];
        decode_block<FMT>(a.packed, a.scale_base, a.lut, K, n, c, w);
#pragma unroll
        for (int j = 0; j < 32; ++j) sum = fmaf(load_x<XBF16>(a.x, xo + 32 * c + j), w[j], sum);
    }
    const int64_t oi = m * a.out_ld + a.out_col0 + n;
    if (a.out_dtype == BYBYCU_DT_BF16)
        reinterpret_cast<__nv_bfloat16*>(a.out)[oi] = __float2bfloat16_rn(sum);
    else
        reinterpret_cast<float*>(a.out)[oi] = sum;
}

template <int FMT>
__global__ void dequant_kernel(int K, int N, const uint8_t* __restrict__ packed, int64_t scale_base,
                               const float* __restrict__ lut, float* __restrict__ w) {
    const int G = K >> 5;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(N) * G) return;
    const int64_t n = i / G;
    const int c = static_cast<int>(i % G);
    float v[32];
    decode_block<FMT>(packed, scale_base, lut, K, n, c, v);
    float4* dst = reinterpret_cast<float4*>(w + n * K + 32 * c);
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

template <int FMT, bool XBF16>
int launch_simt_t(const GemmArgs& a) {
    const dim3 grid(static_cast<unsigned>(ceil_div(a.N, 128)), static_cast<unsigned>(a.M));
    simt_tile_gemm_kernel<FMT, XBF16><<<grid, 128, 0, a.stream>>>(a);
    BYBYCU_LAUNCH_CHECK("simt_tile_gemm_kernel");
    return BYBYCU_OK;
}

}  // namespace

int launch_simt(const GemmArgs& a) {
    const bool bf = a.x_dtype == BYBYCU_DT_BF16;
    switch (a.fmt) {
        case BYBYCU_FMT_FP4KM: return bf ? launch_simt_t<0, true>(a) : launch_simt_t<0, false>(a);
        case BYBYCU_FMT_F16: return bf ? launch_simt_t<1, true>(a) : launch_simt_t<1, false>(a);
        case BYBYCU_FMT_Q4B32: return bf ? launch_simt_t<2, true>(a) : launch_simt_t<2, false>(a);
        default: return set_error(BYBYCU_ERR_SHAPE, "SIMT route: unknown format %d", a.fmt);
    }
}

int launch_dequant(int fmt, int K, int N, const uint8_t* packed, int64_t scale_base,
                   const float* lut, float* w, cudaStream_t stream) {
    const int64_t items = static_cast<int64_t>(N) * (K / 32);
    if (items == 0) return BYBYCU_OK;
    const unsigned blocks = static_cast<unsigned>(ceil_div(items, 256));
    switch (fmt) {
        case 0: dequant_kernel<0><<<blocks, 256, 0, stream>>>(K, N, packed, scale_base, lut, w); break;
        case 1: dequant_kernel<1><<<blocks, 256, 0, stream>>>(K, N, packed, scale_base, lut, w); break;
        case 2: dequant_kernel<2><<<blocks, 256, 0, stream>>>(K, N, packed, scale_base, lut, w); break;
        default: return set_error(BYBYCU_ERR_SHAPE, "dequant: unknown format %d", fmt);
    }
    BYBYCU_LAUNCH_CHECK("dequant_kernel");
    return BYBYCU_OK;
}

}  // namespace bybycu
