// gemv.cu - the decode GEMV route of the tile GEMM for Q4B32 weights (format 2), M <= 16.
//
// The arithmetic is the tile op's (backends/cpu/cpu_vm.c:605-626 with an fp16 block scale):
//     out[m, n] = sum_g s[n, g] * sum_{k in block g} x[m, k] * q[n, k]
// and the job is memory-bound: the packed weights (0.5625 B per weight with the scales) are
// read exactly once from HBM.
//
// Data movement (one persistent CTA per SM, warp-specialised):
//   * the CTA owns a contiguous run of 16-row weight tiles, processed in passes of up to TP
//     tiles; a pass walks K in chunks of 256 values (8 blocks of 32);
//   * a producer warp streams, per chunk, each tile's 16 rows x 128 B of nibbles, the tiles'
//     16 rows x 8 fp16 scales and the M x 256 activations with TMA (cp.async.bulk.tensor,
//     128-byte swizzle for the nibbles and activations) into a ring of stages guarded by
//     mbarriers ("full" completes on the transaction bytes, "empty" when all 8 consumer warps
//     released the stage);
//   * consumer warp w owns block w of every chunk for every tile of the pass.
//
// Math per (tile, block) in one warp: the nibbles of rows g and g+8 (lane = 4g + t holds
// bytes 4t..4t+3 of the block's 16) are turned into bf16 values 136 + q by one lop3 per pair
// (magic exponent 0x43 = 128, nibble ^ 8 = q + 8) and fed as the A operand of two
// mma.sync.m16n8k16 bf16 MMAs (low nibbles = k 0..15, high = k 16..31) whose B operand is
// the raw bf16 activations.  The fp32 block sums therefore hold sum(q x) + 136 sum(x); the
// offset is removed with the activation block sums, computed once per block by the same MMA
// with an all-ones A, and the block scale is applied in fp32: acc += s * (D - 136 Sx).
// q and x are exact in bf16, so the only rounding is the fp32 accumulation.  fp32
// activations are split into two bf16 terms (hi + lo) and both are multiplied.
//
// The 8 warps' partial sums of a tile meet in shared memory at the end of a pass.
#include "kernels.h"

namespace bybycu {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kKC = 256;           // K values per stage: one 32-value block per consumer warp
constexpr int kTileRows = 16;
constexpr int kTileBytes = kTileRows * (kKC / 2);   // 2048: 16 swizzled 128-byte rows
constexpr int kScaleTileBytes = kTileRows * 16;     // 16 rows x 8 halves
constexpr uint32_t kMagicA = 0x43084308u;           // bf16 128 | (nibble ^ 8) via lop3
constexpr uint32_t kOnesBf16x2 = 0x3F803F80u;

struct GemvParams {
    int M, K, N, G;
    int n_tiles;
    int tiles_base, tiles_extra;   // contiguous tile split over the grid
    int n_chunks;
    int stages;
    int tp;                        // tiles per pass (<= TP)
    int x_boxes;                   // activation boxes per stage
    int x_box_rows_bytes;          // bytes of one activation box in shared memory (1 KiB aligned)
    int scale_tma;                 // scales arrive by TMA (K % 256 == 0, aligned)
    uint32_t stage_bytes;          // W tiles + scale tiles + activations
    uint32_t w_off, s_off, x_off;  // offsets inside a stage
    const __half* scales;          // packed + scale_base
    void* out;
    int out_bf16;
    int64_t out_ld, out_col0;
};

__device__ __forceinline__ uint32_t lop3_magic(uint32_t a, uint32_t mask) {
    // (mask & (a ^ C)) | (~mask & C): nibble ^ 8 inside the mask, the bf16 exponent elsewhere.
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(mask), "r"(kMagicA));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The B fragment of one 16-k half block for activation row `m` (lane = 4g + t):
// k slots (2t, 2t+1) <-> elements (4t, 4t+2), slots (2t+8, 2t+9) <-> (4t+1, 4t+3), matching
// the A fragment built from the nibble bytes 4t..4t+3.  `e4` holds elements 4t..4t+3 as
// bf16 pairs (e01, e23).
__device__ __forceinline__ void b_frag(uint32_t e01, uint32_t e23, uint32_t& b0, uint32_t& b1) {
    b0 = prmt(e01, e23, 0x5410);
    b1 = prmt(e01, e23, 0x7632);
}

// Split 4 fp32 activations (elements 4t..4t+3) into bf16 hi/lo pairs in B-fragment order.
__device__ __forceinline__ void split_f32(const float4 v, uint32_t& h0, uint32_t& h1, uint32_t& l0,
                                          uint32_t& l1) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.z);   // slots 2t, 2t+1
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.y, v.w);   // slots 2t+8, 2t+9
    const float2 af = __bfloat1622float2(a), bf = __bfloat1622float2(b);
    const __nv_bfloat162 al = __floats2bfloat162_rn(v.x - af.x, v.z - af.y);
    const __nv_bfloat162 bl = __floats2bfloat162_rn(v.y - bf.x, v.w - bf.y);
    h0 = *reinterpret_cast<const uint32_t*>(&a);
    h1 = *reinterpret_cast<const uint32_t*>(&b);
    l0 = *reinterpret_cast<const uint32_t*>(&al);
    l1 = *reinterpret_cast<const uint32_t*>(&bl);
}

template <int TP, int NT, bool XF32>
__global__ void __launch_bounds__(kThreads, 1)
gemv_q4b32_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                  const __grid_constant__ CUtensorMap smap, const GemvParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* stages = smem;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(stages + static_cast<size_t>(p.stages) * p.stage_bytes);
    uint64_t* empty_bar = full_bar + p.stages;
    volatile int* s_abort = reinterpret_cast<volatile int*>(empty_bar + p.stages);
    float* red = reinterpret_cast<float*>(empty_bar + p.stages + 2);   // [8][TP][NT][32][4]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // contiguous tile run of this CTA
    const int b = blockIdx.x;
    const int my_tiles = p.tiles_base + (b < p.tiles_extra ? 1 : 0);
    const int tile_begin = b * p.tiles_base + min(b, p.tiles_extra);
    const int passes = (my_tiles + p.tp - 1) / p.tp;
    const int total_it = passes * p.n_chunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kConsumerWarps);
        }
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tensormap(&wmap);
            prefetch_tensormap(&xmap);
            if (p.scale_tma) prefetch_tensormap(&smap);
            const uint64_t policy = l2_policy_evict_first();
            int issued = 0;
            for (int it = 0; it < total_it; ++it) {
                const int s = it % p.stages;
                if (it >= p.stages) {
                    if (*s_abort) break;
                    if (!mbar_wait_bounded(&empty_bar[s], ((it / p.stages) - 1) & 1, kDevErrEmptyWait)) {
                        *s_abort = 1;
                        break;
                    }
                }
                const int pass = it / p.n_chunks, chunk = it % p.n_chunks;
                const int t0 = tile_begin + pass * p.tp;
                const int nt = min(p.tp, tile_begin + my_tiles - t0);
                const uint32_t bytes = nt * kTileBytes + (p.scale_tma ? nt * kScaleTileBytes : 0) +
                                       p.x_boxes * (p.M * 128);
                uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
                mbar_arrive_expect_tx(&full_bar[s], bytes);
                for (int i = 0; i < nt; ++i) {
                    tma_load_2d_hint(st + p.w_off + i * kTileBytes, &wmap, &full_bar[s], chunk * (kKC / 2),
                                     (t0 + i) * kTileRows, policy);
                    if (p.scale_tma)
                        tma_load_2d(st + p.s_off + i * kScaleTileBytes, &smap, &full_bar[s], chunk * 8,
                                    (t0 + i) * kTileRows);
                }
                const int box_elems = XF32 ? 32 : 64;
                for (int bx = 0; bx < p.x_boxes; ++bx)
                    tma_load_2d(st + p.x_off + bx * p.x_box_rows_bytes, &xmap, &full_bar[s],
                                chunk * kKC + bx * box_elems, 0);
                issued = it + 1;
            }
            // Before the CTA may exit, every copy it issued must have landed.
            for (int it = max(0, issued - p.stages); it < issued; ++it) {
                const int s = it % p.stages;
                if (!mbar_wait_bounded(&full_bar[s], (it / p.stages) & 1, kDevErrDrainWait)) break;
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    float acc[TP][NT][4];
#pragma unroll
    for (int i = 0; i < TP; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[i][j][v] = 0.0f;
    const uint32_t ones[4] = {kOnesBf16x2, kOnesBf16x2, kOnesBf16x2, kOnesBf16x2};

    for (int it = 0; it < total_it; ++it) {
        const int s = it % p.stages;
        const int pass = it / p.n_chunks, chunk = it % p.n_chunks;
        const int t0 = tile_begin + pass * p.tp;
        const int nt = min(p.tp, tile_begin + my_tiles - t0);
        bool ok = !*s_abort;
        if (ok && !mbar_wait_bounded(&full_bar[s], (it / p.stages) & 1, kDevErrFullWait)) {
            *s_abort = 1;
            ok = false;
        }
        const int c = chunk * 8 + warp;   // the 32-value block of this warp
        if (ok && c < p.G) {
            const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
            // ---- activation fragments of block c (B operands) and their block sums
            uint32_t blo[NT][XF32 ? 2 : 1][2], bhi[NT][XF32 ? 2 : 1][2];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int m = j * 8 + g;
                const bool live = m < p.M;
                if constexpr (!XF32) {
                    // bf16 box: 64 elements (128 B) per row; element e0 = 32*(w&1) + 4t
                    const uint8_t* box = st + p.x_off + (warp >> 1) * p.x_box_rows_bytes + m * 128;
                    const int jlo = 4 * (warp & 1) + (t >> 1), jhi = jlo + 2;
                    const int sub = 8 * (t & 1);
                    uint2 lo = make_uint2(0u, 0u), hi = make_uint2(0u, 0u);
                    if (live) {
                        lo = *reinterpret_cast<const uint2*>(box + ((jlo ^ (m & 7)) << 4) + sub);
                        hi = *reinterpret_cast<const uint2*>(box + ((jhi ^ (m & 7)) << 4) + sub);
                    }
                    b_frag(lo.x, lo.y, blo[j][0][0], blo[j][0][1]);
                    b_frag(hi.x, hi.y, bhi[j][0][0], bhi[j][0][1]);
                } else {
                    // fp32 box: 32 elements (128 B) per row, one box per block
                    const uint8_t* box = st + p.x_off + warp * p.x_box_rows_bytes + m * 128;
                    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
                    if (live) {
                        lo = *reinterpret_cast<const float4*>(box + ((t ^ (m & 7)) << 4));
                        hi = *reinterpret_cast<const float4*>(box + (((4 + t) ^ (m & 7)) << 4));
                    }
                    split_f32(lo, blo[j][0][0], blo[j][0][1], blo[j][1][0], blo[j][1][1]);
                    split_f32(hi, bhi[j][0][0], bhi[j][0][1], bhi[j][1][0], bhi[j][1][1]);
                }
            }
            float corr[NT][4];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                float sx[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int h = 0; h < (XF32 ? 2 : 1); ++h) {
                    mma_bf16(sx, ones, blo[j][h][0], blo[j][h][1]);
                    mma_bf16(sx, ones, bhi[j][h][0], bhi[j][h][1]);
                }
#pragma unroll
                for (int v = 0; v < 4; ++v) corr[j][v] = 136.0f * sx[v];
            }
            // ---- per tile: dequantise rows g and g+8 of block c, two MMAs, scale in fp32
#pragma unroll
            for (int i = 0; i < TP; ++i) {
                if (i < nt) {
                    const uint8_t* wt = st + p.w_off + i * kTileBytes;
                    const uint32_t off = g * 128 + ((warp ^ g) << 4) + 4 * t;
                    const uint32_t w0 = *reinterpret_cast<const uint32_t*>(wt + off);
                    const uint32_t w8 = *reinterpret_cast<const uint32_t*>(wt + off + 1024);
                    float s0, s8;
                    const int64_t row0 = static_cast<int64_t>(t0 + i) * kTileRows + g;
                    if (p.scale_tma) {
                        const __half* sc = reinterpret_cast<const __half*>(st + p.s_off + i * kScaleTileBytes);
                        s0 = __half2float(sc[g * 8 + warp]);
                        s8 = __half2float(sc[(g + 8) * 8 + warp]);
                    } else {
                        s0 = row0 < p.N ? __half2float(p.scales[row0 * p.G + c]) : 0.0f;
                        s8 = row0 + 8 < p.N ? __half2float(p.scales[(row0 + 8) * p.G + c]) : 0.0f;
                    }
                    uint32_t alo[4], ahi[4];
                    alo[0] = lop3_magic(w0, 0x000F000Fu);
                    alo[1] = lop3_magic(w8, 0x000F000Fu);
                    alo[2] = lop3_magic(w0 >> 8, 0x000F000Fu);
                    alo[3] = lop3_magic(w8 >> 8, 0x000F000Fu);
                    ahi[0] = lop3_magic(w0 >> 4, 0x000F000Fu);
                    ahi[1] = lop3_magic(w8 >> 4, 0x000F000Fu);
                    ahi[2] = lop3_magic(w0 >> 12, 0x000F000Fu);
                    ahi[3] = lop3_magic(w8 >> 12, 0x000F000Fu);
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int h = 0; h < (XF32 ? 2 : 1); ++h) {
                            mma_bf16(d, alo, blo[j][h][0], blo[j][h][1]);
                            mma_bf16(d, ahi, bhi[j][h][0], bhi[j][h][1]);
                        }
                        acc[i][j][0] = fmaf(s0, d[0] - corr[j][0], acc[i][j][0]);
                        acc[i][j][1] = fmaf(s0, d[1] - corr[j][1], acc[i][j][1]);
                        acc[i][j][2] = fmaf(s8, d[2] - corr[j][2], acc[i][j][2]);
                        acc[i][j][3] = fmaf(s8, d[3] - corr[j][3], acc[i][j][3]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);

        if (chunk == p.n_chunks - 1) {
            // ---- end of pass: the 8 warps' partial sums meet in shared memory
            float* mine = red + static_cast<size_t>(warp) * TP * NT * 128;
#pragma unroll
            for (int i = 0; i < TP; ++i)
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        mine[((i * NT + j) * 32 + lane) * 4 + v] = acc[i][j][v];
                        acc[i][j][v] = 0.0f;
                    }
            named_barrier(1, kConsumerWarps * 32);
            const int entries = nt * NT * 128;
            for (int e = threadIdx.x; e < entries; e += kConsumerWarps * 32) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) sum += red[static_cast<size_t>(w) * TP * NT * 128 + e];
                const int v = e & 3, ln = (e >> 2) & 31, ij = e >> 7;
                const int j = ij % NT, i = ij / NT;
                const int gg = ln >> 2, tt = ln & 3;
                const int64_t n = static_cast<int64_t>(t0 + i) * kTileRows + gg + (v >= 2 ? 8 : 0);
                const int m = j * 8 + 2 * tt + (v & 1);
                if (n < p.N && m < p.M) {
                    const int64_t oi = static_cast<int64_t>(m) * p.out_ld + p.out_col0 + n;
                    if (p.out_bf16) reinterpret_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(sum);
                    else reinterpret_cast<float*>(p.out)[oi] = sum;
                }
            }
            named_barrier(1, kConsumerWarps * 32);
        }
    }
}

struct GemvPlan {
    int tp, nt;
    bool xf32;
};

template <int TP, int NT, bool XF32>
int launch_t(const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& smap,
             const GemvParams& p, int grid, size_t smem, cudaStream_t stream) {
    auto kern = gemv_q4b32_kernel<TP, NT, XF32>;
    static bool configured = false;   // per instantiation; the limit is a device property
    if (!configured) {
        BYBYCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448));
        configured = true;
    }
    kern<<<grid, kThreads, smem, stream>>>(wmap, xmap, smap, p);
    BYBYCU_LAUNCH_CHECK("gemv_q4b32_kernel");
    return BYBYCU_OK;
}

template <int TP>
int dispatch_tp(int nt, bool xf32, const CUtensorMap& w, const CUtensorMap& x, const CUtensorMap& s,
                const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
    if (nt == 1) return xf32 ? launch_t<TP, 1, true>(w, x, s, p, grid, smem, st)
                             : launch_t<TP, 1, false>(w, x, s, p, grid, smem, st);
    return xf32 ? launch_t<TP, 2, true>(w, x, s, p, grid, smem, st)
                : launch_t<TP, 2, false>(w, x, s, p, grid, smem, st);
}

}  // namespace

bool gemv_supports(const GemmArgs& a) {
    if (a.fmt != BYBYCU_FMT_Q4B32) return false;
    if (a.M < 1 || a.M > 16 || a.K % 32 != 0 || a.N < 1) return false;
    if (a.x_dtype != BYBYCU_DT_BF16 && a.x_dtype != BYBYCU_DT_F32) return false;
    // TMA needs 16-byte aligned global bases; scales need 2-byte alignment.
    if ((reinterpret_cast<uintptr_t>(a.packed) & 15u) || (reinterpret_cast<uintptr_t>(a.x) & 15u)) return false;
    if (a.scale_base & 1) return false;
    return true;
}

int launch_gemv(const GemmArgs& a) {
    DeviceInfo dev;
    if (int rc = current_device_info(&dev)) return rc;
    const bool xf32 = a.x_dtype == BYBYCU_DT_F32;
    const int n_tiles = static_cast<int>(ceil_div(a.N, kTileRows));
    const int grid = std::min(n_tiles, dev.sm_count);
    const int tiles_max = static_cast<int>(ceil_div(n_tiles, grid));
    const int tp = tiles_max <= 1 ? 1 : tiles_max <= 2 ? 2 : tiles_max <= 4 ? 4 : tiles_max <= 5 ? 5 : 8;
    const int ntn = a.M > 8 ? 2 : 1;

    GemvParams p{};
    p.M = a.M; p.K = a.K; p.N = a.N; p.G = a.K / 32;
    p.n_tiles = n_tiles;
    p.tiles_base = n_tiles / grid;
    p.tiles_extra = n_tiles % grid;
    p.n_chunks = static_cast<int>(ceil_div(a.K, kKC));
    p.tp = std::min(tp, tiles_max);
    const uint8_t* scale_ptr = a.packed + a.scale_base;
    p.scale_tma = (a.K % kKC == 0) && ((reinterpret_cast<uintptr_t>(scale_ptr) & 15u) == 0);
    p.x_boxes = xf32 ? kKC / 32 : kKC / 64;
    p.x_box_rows_bytes = static_cast<int>(ceil_div(a.M * 128, 1024) * 1024);
    p.w_off = 0;
    p.s_off = tp * kTileBytes;
    p.x_off = p.s_off + static_cast<uint32_t>(ceil_div(tp * kScaleTileBytes, 1024) * 1024);
    p.stage_bytes = p.x_off + p.x_boxes * p.x_box_rows_bytes;
    p.scales = reinterpret_cast<const __half*>(scale_ptr);
    p.out = a.out;
    p.out_bf16 = a.out_dtype == BYBYCU_DT_BF16;
    p.out_ld = a.out_ld;
    p.out_col0 = a.out_col0;

    const size_t red_bytes = static_cast<size_t>(kConsumerWarps) * tp * ntn * 128 * sizeof(float);
    const size_t fixed = 1024 /*align slack*/ + red_bytes + 64;
    const size_t budget = static_cast<size_t>(dev.max_smem_optin);
    const int passes_max = static_cast<int>(ceil_div(tiles_max, p.tp));
    const int want = passes_max * p.n_chunks;
    int stages = static_cast<int>((budget - fixed) / (p.stage_bytes + 16));
    stages = std::max(1, std::min(stages, want));
    if (stages < 2 && want > 1)
        return set_error(BYBYCU_ERR_SHAPE, "GEMV: shared memory too small for M=%d", a.M);
    p.stages = stages;
    const size_t smem = fixed + static_cast<size_t>(stages) * (p.stage_bytes + 16);

    CUtensorMap wmap, xmap, smap;
    if (int rc = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.packed, a.K / 2, a.N, a.K / 2,
                                      kKC / 2, kTileRows, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
        return rc;
    if (xf32) {
        if (int rc = encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.x, a.K, a.M,
                                          static_cast<uint64_t>(a.K) * 4, 32, a.M, CU_TENSOR_MAP_SWIZZLE_128B,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
            return rc;
    } else {
        if (int rc = encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.x, a.K, a.M,
                                          static_cast<uint64_t>(a.K) * 2, 64, a.M, CU_TENSOR_MAP_SWIZZLE_128B,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
            return rc;
    }
    if (p.scale_tma) {
        if (int rc = encode_tensor_map_2d(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, scale_ptr, p.G, a.N,
                                          static_cast<uint64_t>(p.G) * 2, 8, kTileRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
            return rc;
    } else {
        smap = wmap;   // unused
    }
    switch (tp) {
        case 1: return dispatch_tp<1>(ntn, xf32, wmap, xmap, smap, p, grid, smem, a.stream);
        case 2: return dispatch_tp<2>(ntn, xf32, wmap, xmap, smap, p, grid, smem, a.stream);
        case 4: return dispatch_tp<4>(ntn, xf32, wmap, xmap, smap, p, grid, smem, a.stream);
        case 5: return dispatch_tp<5>(ntn, xf32, wmap, xmap, smap, p, grid, smem, a.stream);
        default: return dispatch_tp<8>(ntn, xf32, wmap, xmap, smap, p, grid, smem, a.stream);
    }
}

}  // namespace bybycu
