// q4asym.cu - asymmetric Q4 (the reference's matmul_q4 data): C[M, N] = A[M, K] . W^T with
//     W[n, k] = (u[n, k] - zeros[n, k / group]) * scales[n, k / group],
// u the unsigned nibble k of row n in wq[n, K/2] (even k in the low nibble), fp32 scales and
// zero points [N, groups], fp32 A and C (backends/cpu/cpu_kernels_impl.inc:293-319, the CPU VM's
// OP_Q4_GEMV at backends/cpu/cpu_vm.c:420-482, the API of gpubackend.nim:806-843,2883-3060).
//
// Decode (M = 1, group 32, K % 128 == 0): q4a_m1_kernel streams the packed rows exactly like
// the Q4B32 decode kernel (the same producer, 128-byte TMA boxes, plus one fp32 zero-point box
// beside each fp32 scale box) and uses the same integer tensor-core form:
//   * one AND gives four s8 values u of a word's low nibbles (k = 8t, 8t+2, 8t+4, 8t+6 for
//     word t of a block) and a shift + AND its high nibbles (k = 8t+1, ...): the A fragment of
//     an m16n8k32 s8 MMA in the K order (slot s < 16 -> k = 2s, slot 16 + s -> k = 2s + 1);
//   * x becomes X = rint(x * 2^(140 - E)) per 32-block (E its largest fp32 exponent, |X| <=
//     2^14) in two signed byte digits laid out in the same K order, four blocks x two digits
//     filling the MMA's eight columns;
//   * per row and block the epilogue adds s * 2^(E-140) * (sum u X - z * sum X): the zero point
//     enters through the block's sum of X (the s (dot(a, u) - z sum(a)) factorisation of the
//     reference's GPU kernels).
// Everything else (any M, any group size, odd K, unaligned slots) runs q4a_exact_kernel: one
// thread per output, fmaf(x, (u - z) * s, sum) in k order (the CPU VM's OP_Q4_GEMV arithmetic).
#include "kernels.h"

namespace bybycu {
namespace {

// Tiles of 16 rows per pass, and the ring depth: one CTA per SM with three 64 KB stages.  Two
// co-resident CTAs (4-tile passes, two stages each) measured 30% slower at the C2 shape: CTAs
// with 5 tiles then need a second pass, while three stages keep enough of the 0.75 B/weight
// stream in flight for one CTA.
constexpr int kQ4aTP = 5;
constexpr int kQ4aStages = 3;

__global__ void __launch_bounds__(128) q4a_exact_kernel(int M, int K, int N, int group, int n_groups,
                                                        const uint8_t* __restrict__ wq,
                                                        const float* __restrict__ scales,
                                                        const float* __restrict__ zeros,
                                                        const float* __restrict__ x, float* __restrict__ out) {
    const int64_t n = static_cast<int64_t>(blockIdx.x) * 128 + threadIdx.x;
    const int64_t m = blockIdx.y;
    if (n >= N) return;
    const int64_t row_bytes = (K + 1) / 2;
    float sum = 0.0f;
    for (int k = 0; k < K; ++k) {
        const uint32_t byte = wq[n * row_bytes + (k >> 1)];
        const uint32_t nib = (byte >> ((k & 1) * 4)) & 15u;
        const int64_t gi = n * n_groups + (group > 0 ? k / group : 0);   // group <= 0: one group
        sum = fmaf(x[m * K + k], (static_cast<float>(nib) - zeros[gi]) * scales[gi], sum);
    }
    out[m * N + n] = sum;
}

template <int TP>
__global__ void __launch_bounds__(kM1Threads, 2)
q4a_m1_kernel(const __grid_constant__ GemvMaps maps, const GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(p.stages) * p.stage_bytes);
    uint64_t* empty_bar = full_bar + p.stages;
    volatile int* s_abort = reinterpret_cast<volatile int*>(empty_bar + p.stages);
    const uint32_t red = smem_u32(empty_bar + p.stages + 2);   // [kM1Warps][TP][16] floats

    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x;
    const int my_tiles = p.tiles_base + (b < p.tiles_extra ? 1 : 0);
    const int tile_begin = b * p.tiles_base + min(b, p.tiles_extra);
    const int passes = (my_tiles + p.tp - 1) / p.tp;
    const int total_it = passes * p.n_chunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kM1Warps);
        }
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == kM1Warps) {
        gemv_producer(maps, p, smem, full_bar, empty_bar, s_abort, lane, tile_begin, my_tiles, total_it);
        return;
    }
    if (warp > kM1Warps) return;   // the kernel shares the Q4B32 decode kernel's block shape

    const int g = lane >> 2, t = lane & 3;
    const int box = warp / kM1Parts, part = warp % kM1Parts;
    const int blk0 = part * kM1Blocks;   // this warp: blocks blk0 .. blk0 + 3 of its 256-value box
    const int q = g >> 1;                // lane (g, t) feeds B column g: digit g % 2 of block q
    float acc[TP][2];
#pragma unroll
    for (int i = 0; i < TP; ++i) acc[i][0] = acc[i][1] = 0.0f;
    uint32_t woff[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) woff[j] = g * 128 + (((blk0 + j) ^ g) << 4) + 4 * t;
    const float magic = (g & 1) ? 12583040.0f : 12582912.0f;   // 1.5 * 2^23 (+ 128: high digit)
    const uint32_t sel = (g & 1) ? 0x0051u : 0x0040u;          // byte 0 (low digit) / byte 1 (high)
    const int x_off_bits = (g & 1) ? 0x4B400080 : 0x4B400000;  // the sum's bits for X = 0
    bool waited = false;

    int s = 0, round = 0, chunk = 0, t0 = tile_begin;
    for (int it = 0; it < total_it; ++it) {
        const int nt = min(p.tp, tile_begin + my_tiles - t0);
        bool ok = !*s_abort;
        if (ok && !mbar_wait_bounded(&full_bar[s], round & 1, kDevErrFullWait)) {
            *s_abort = 1;
            ok = false;
        }
        const int c0 = chunk * (kM1KC / 32) + box * 8;   // this warp's box: blocks c0 .. c0 + 7 of K
        if (ok && c0 + blk0 < p.G) {
            const uint32_t st = static_cast<uint32_t>(s) * p.stage_bytes;
            // ---- activations: lane (g, t) takes x[8t .. 8t+7] of block q
            const bool live = c0 + blk0 + q < p.G;
            const uint32_t xr = st + p.x_off + ((box * 8 + blk0 + q) * 32 + 8 * t) * 4;
            uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
            if (live) {
                xa = lds_u128(base + xr);
                xb = lds_u128(base + xr + 16);
            }
            const uint32_t xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            uint32_t mx = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) mx = max(mx, xv[i] & 0x7FFFFFFFu);   // inf / NaN sort highest
            mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const int e = static_cast<int>(mx >> 23);
            if (live && e == 255 && t == 0 && !(g & 1)) record_device_error(kDevErrActRange);
            const int ec = max(e, 14);                               // normal factors 2^(ec - 140)
            const float up = __int_as_float((267 - ec) << 23);       // 2^(140 - ec)
            uint32_t r[8];
            int sx = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                r[i] = __float_as_uint(fmaf(__uint_as_float(xv[i]), up, magic));   // bits + X
                sx += static_cast<int>(r[i]) - x_off_bits;
            }
            const uint32_t b0 = prmt(prmt(r[0], r[2], sel), prmt(r[4], r[6], sel), 0x5410);   // k = 8t + 2i
            const uint32_t b1 = prmt(prmt(r[1], r[3], sel), prmt(r[5], r[7], sel), 0x5410);   // k = 8t + 2i + 1
            sx += __shfl_xor_sync(0xffffffffu, sx, 1);
            sx += __shfl_xor_sync(0xffffffffu, sx, 2);   // sum of X over block q
            uint32_t bq[4][2];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                bq[j][0] = q == j ? b0 : 0u;
                bq[j][1] = q == j ? b1 : 0u;
                asm volatile("" : "+r"(bq[j][0]), "+r"(bq[j][1]));   // keep them in registers
            }
            // lane (g, t) combines block t (built by lane 8t): its factor and its sum of X
            const int et = __shfl_sync(0xffffffffu, ec, 8 * t);
            const float ft = __int_as_float((et - 13) << 23);   // 2^(et - 140)
            const float sxt = static_cast<float>(__shfl_sync(0xffffffffu, sx, 8 * t));
            const uint32_t wbox = st + box * p.w_box_bytes;
            // ---- weights: four s8 MMAs per tile fill the eight columns
#pragma unroll
            for (int i = 0; i < TP; ++i) {
                int d[4] = {0, 0, 0, 0};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t wt = wbox + i * (kTileRows * 128) + woff[j];
                    const uint32_t w0 = sh_u32(smem, wt);
                    const uint32_t w8 = sh_u32(smem, wt + 1024);
                    const uint32_t a[4] = {w0 & 0x0F0F0F0Fu, w8 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu,
                                           (w8 >> 4) & 0x0F0F0F0Fu};
                    mma_s8(d, a, bq[j][0], bq[j][1]);
                }
                const float v0 = static_cast<float>(d[0] + d[1] * 256), v8 = static_cast<float>(d[2] + d[3] * 256);
                // scale and zero point of block t for rows g and g + 8 (128-byte swizzled boxes)
                const int cb = box * 8 + blk0 + t;   // block inside the chunk: 16-byte column cb / 4
                const uint32_t r0 = i * kTileRows + g, r8 = r0 + 8;
                const uint32_t o0 = r0 * 128 + ((((cb >> 2) ^ (r0 & 7)) << 4) | ((cb & 3) << 2));
                const uint32_t o8 = r8 * 128 + ((((cb >> 2) ^ (r8 & 7)) << 4) | ((cb & 3) << 2));
                const float s0 = *reinterpret_cast<const float*>(smem + st + p.s_off + o0);
                const float z0 = *reinterpret_cast<const float*>(smem + st + p.z_off + o0);
                const float s8 = *reinterpret_cast<const float*>(smem + st + p.s_off + o8);
                const float z8 = *reinterpret_cast<const float*>(smem + st + p.z_off + o8);
                acc[i][0] = fmaf(s0 * ft, fmaf(-z0, sxt, v0), acc[i][0]);
                acc[i][1] = fmaf(s8 * ft, fmaf(-z8, sxt, v8), acc[i][1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        if (++s == p.stages) { s = 0; ++round; }

        if (chunk == p.n_chunks - 1) {
            if (!waited) {   // the previous kernel may still read the outputs
                pdl_wait();
                waited = true;
            }
            // ---- end of pass: rows g and g+8 summed over the quad, then over the warps
#pragma unroll
            for (int i = 0; i < TP; ++i) {
                float v0 = acc[i][0], v8 = acc[i][1];
                v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
                v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
                v8 += __shfl_xor_sync(0xffffffffu, v8, 1);
                v8 += __shfl_xor_sync(0xffffffffu, v8, 2);
                if (t == 0) {
                    sts_f32(red + ((warp * TP + i) * 16 + g) * 4, v0);
                    sts_f32(red + ((warp * TP + i) * 16 + g + 8) * 4, v8);
                }
                acc[i][0] = acc[i][1] = 0.0f;
            }
            named_barrier(1, kM1Warps * 32);
            for (int e = threadIdx.x; e < nt * 16; e += kM1Warps * 32) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kM1Warps; ++w) sum += lds_f32(red + ((w * TP) * 16 + e) * 4);
                const int64_t n = static_cast<int64_t>(t0) * kTileRows + e;
                if (n < p.N) reinterpret_cast<float*>(p.out)[p.out_col0 + n] = sum;
            }
            named_barrier(1, kM1Warps * 32);
        }
        if (++chunk == p.n_chunks) { chunk = 0; t0 += p.tp; }
    }
}

}  // namespace

bool q4a_fast_supports(int M, int K, int N, int group, int n_groups, const void* x, const void* wq,
                       const void* scales, const void* zeros) {
    if (M != 1 || group != 32 || n_groups != K / 32 || K % 128 != 0 || K > (1 << 20) || N < 1) return false;
    auto al16 = [](const void* v) { return (reinterpret_cast<uintptr_t>(v) & 15u) == 0; };
    if (!al16(x) || !al16(wq) || !al16(scales) || !al16(zeros)) return false;
    DeviceInfo info;
    return current_device_info(&info) == BYBYCU_OK && info.cc_major == 10;
}

int launch_q4a(int M, int K, int N, int group, int n_groups, const float* x, const uint8_t* wq, const float* scales,
               const float* zeros, float* out, cudaStream_t stream) {
    DeviceInfo dev;
    if (int rc = current_device_info(&dev)) return rc;
    const int n_tiles = static_cast<int>(ceil_div(N, kTileRows));
    const int grid = std::min(n_tiles, dev.sm_count);
    const int tiles_max = static_cast<int>(ceil_div(n_tiles, grid));
    const int tp = std::min(tiles_max, kQ4aTP);
    const uint32_t rows = kTileRows * kQ4aTP;
    const uint32_t wb = rows * 128;                 // one 256-value nibble box
    const uint32_t s_off = 4 * wb;                  // four boxes per 1024-value chunk
    const uint32_t z_off = s_off + rows * 128;      // 32 fp32 scales per row, then 32 zero points
    const uint32_t x_off = z_off + rows * 128;
    const uint32_t stage_bytes = (x_off + kM1KC * 4 + 1023) / 1024 * 1024;
    const size_t red_bytes = static_cast<size_t>(kM1Warps) * kQ4aTP * 16 * sizeof(float);
    const size_t budget = static_cast<size_t>(dev.max_smem_optin) - 1024 - 64 - red_bytes;
    const int stages = std::min(kQ4aStages, static_cast<int>(budget / (stage_bytes + 16)));
    if (stages < 2) return set_error(BYBYCU_ERR_SHAPE, "matmul_q4 decode: shared memory too small");
    const size_t smem = 1024 + static_cast<size_t>(stages) * (stage_bytes + 16) + 16 + red_bytes;

    GemvParams p{};
    p.M = 1; p.K = K; p.N = N; p.G = K / 32;
    p.tiles_base = n_tiles / grid;
    p.tiles_extra = n_tiles % grid;
    p.kc = kM1KC;
    p.n_chunks = static_cast<int>(ceil_div(K, kM1KC));
    p.stages = stages;
    p.tp = tp;
    p.scale_tma = 1;
    p.zeros = 1;
    p.x_pitch = kM1KC * 4;
    p.stage_bytes = stage_bytes;
    p.w_box_bytes = wb;
    p.s_off = s_off;
    p.z_off = z_off;
    p.x_off = x_off;
    p.s_pitch = 128;
    p.x = reinterpret_cast<const uint8_t*>(x);
    p.x_elem = 4;
    p.out = out;
    p.out_ld = N;

    // tensor maps: nibbles as the Q4B32 decode kernel's, fp32 scales and zero points in
    // 32-value (128-byte) swizzled boxes of the same rows
    GemvMaps maps;
    const int box_rows[3] = {kTileRows * tp, kTileRows * std::max(1, tp - 1), kTileRows};
    for (int i = 0; i < 3; ++i) {
        if (int rc = encode_tensor_map_2d(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, K / 2, N, K / 2, 128,
                                          box_rows[i], CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return rc;
        if (int rc = encode_tensor_map_2d(&maps.s[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, scales, K / 32, N,
                                          static_cast<uint64_t>(K / 32) * 4, 32, box_rows[i],
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
            return rc;
        if (int rc = encode_tensor_map_2d(&maps.z[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, zeros, K / 32, N,
                                          static_cast<uint64_t>(K / 32) * 4, 32, box_rows[i],
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
            return rc;
    }
    static std::once_flag once[16];
    static cudaError_t attr_rc[16];
    const int di = dev.device & 15;
    std::call_once(once[di], [&] {
        attr_rc[di] = cudaFuncSetAttribute(q4a_m1_kernel<kQ4aTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           232448);
    });
    if (attr_rc[di] != cudaSuccess) return cuda_fail(attr_rc[di], "cudaFuncSetAttribute(q4a)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kM1Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    BYBYCU_CUDA_TRY(cudaLaunchKernelEx(&cfg, q4a_m1_kernel<kQ4aTP>, maps, p));
    BYBYCU_LAUNCH_CHECK("q4a_m1_kernel");
    return BYBYCU_OK;
}

}  // namespace bybycu

using namespace bybycu;

extern "C" int bybycu_matmul_q4(const float* a, const uint8_t* wq, const float* scales, const float* zeros, float* c,
                                int M, int K, int N, int group_size, int n_groups_per_row, int route, void* stream) {
    if (!a || !wq || !scales || !zeros || !c) return set_error(BYBYCU_ERR_ARGS, "matmul_q4 slot is missing");
    if (M <= 0 || K <= 0 || N <= 0) return set_error(BYBYCU_ERR_SHAPE, "unsupported matmul_q4 shape M=%d K=%d N=%d", M, K, N);
    const int64_t groups_needed = group_size > 0 ? (static_cast<int64_t>(K) + group_size - 1) / group_size : 1;
    if (n_groups_per_row < groups_needed)
        return set_error(BYBYCU_ERR_SHAPE, "matmul_q4: %d groups per row, K=%d with group %d needs %lld", n_groups_per_row,
                         K, group_size, static_cast<long long>(groups_needed));
    if (route != BYBYCU_ROUTE_AUTO && route != BYBYCU_ROUTE_SIMT && route != BYBYCU_ROUTE_GEMV)
        return set_error(BYBYCU_ERR_ARGS, "matmul_q4: route %d (AUTO, SIMT or GEMV)", route);
    const bool fast = q4a_fast_supports(M, K, N, group_size, n_groups_per_row, a, wq, scales, zeros);
    if (route == BYBYCU_ROUTE_GEMV && !fast)
        return set_error(BYBYCU_ERR_SHAPE, "matmul_q4: the decode route needs M=1, group 32, K %% 128 == 0 and "
                                           "16-byte aligned slots");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (route == BYBYCU_ROUTE_SIMT || !fast) {
        dim3 grid(static_cast<unsigned>(ceil_div(N, 128)), static_cast<unsigned>(M));
        q4a_exact_kernel<<<grid, 128, 0, s>>>(M, K, N, group_size, n_groups_per_row, wq, scales, zeros, a, c);
        BYBYCU_LAUNCH_CHECK("q4a_exact_kernel");
        return BYBYCU_OK;
    }
    return launch_q4a(M, K, N, group_size, n_groups_per_row, a, wq, scales, zeros, c, s);
}
