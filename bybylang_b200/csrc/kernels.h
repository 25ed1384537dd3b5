// kernels.h - host-side launcher interface shared by the routes of libbybycuda.so.
#pragma once

#include "common.cuh"

namespace bybycu {

// One tile-GEMM launch after the ABI layer has validated it.  `lut` already points at the
// op's 272-float table (lut + lut_base) for format 0.  The output element (m, n) is stored at
// out[m * out_ld + out_col0 + n].
struct GemmArgs {
    int fmt = 0;
    int M = 0, K = 0, N = 0;
    const void* x = nullptr;
    int x_dtype = BYBYCU_DT_F32;
    const uint8_t* packed = nullptr;
    int64_t packed_len = 0;
    int64_t scale_base = 0;
    const float* lut = nullptr;
    void* out = nullptr;
    int out_dtype = BYBYCU_DT_F32;
    int64_t out_ld = 0;
    int64_t out_col0 = 0;
    cudaStream_t stream = nullptr;
};

// CUDA-core FP32 route: every format, every K % 32 == 0 shape.
int launch_simt(const GemmArgs& a);
// Decode GEMV route (format 2, M <= 16): TMA-streamed weights, bf16 mma.sync reductions with
// exact per-block fp32 scaling.
bool gemv_supports(const GemmArgs& a);
int launch_gemv(const GemmArgs& a);
// Prefill GEMM route: tcgen05 MMAs from shared-memory fp16 tiles, fp32 accumulators in TMEM.
bool tc_supports(const GemmArgs& a);
int launch_tc(const GemmArgs& a);
// The same route staging its activations in a fixed module array instead of pool memory.
int launch_tc_static_scratch(const GemmArgs& a);

int launch_dequant(int fmt, int K, int N, const uint8_t* packed, int64_t scale_base,
                   const float* lut, float* w, cudaStream_t stream);

}  // namespace bybycu
