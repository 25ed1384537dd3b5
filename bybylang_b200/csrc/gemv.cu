// gemv.cu - the decode GEMV route of the tile GEMM for Q4B32 weights (format 2), M <= 16 per
// launch (17..32 rows run as one launch per 16 rows).
//
// The arithmetic is the tile op's (backends/cpu/cpu_vm.c:605-626 with an fp16 block scale):
//     out[m, n] = sum_g s[n, g] * sum_{k in block g} x[m, k] * q[n, k]
// and the job is memory-bound: the packed weights (0.5625 B per weight with the scales) are
// read exactly once from HBM.
//
// Data movement (one persistent CTA per SM, warp-specialised):
//   * the CTA owns a contiguous run of 16-row weight tiles, processed in passes of up to TP
//     tiles; a pass walks K in chunks of KC values (2048, or 1024 / 512 when shared memory
//     is short);
//   * a producer warp streams each chunk with few, large TMA operations - the TMA unit's
//     cost is per operation, so every weight box spans all rows of the pass:
//       - nibbles: KC/256 boxes of 128 bytes x (16 * tiles) rows, 128-byte swizzle;
//       - scales: one box of KC/32 halves x (16 * tiles) rows;
//       - activations: one 1D bulk copy per activation row into a padded smem row;
//     into a ring of stages guarded by mbarriers ("full" completes on the transaction bytes,
//     "empty" when all 16 consumer warps released the stage);
//   * consumer warp w owns blocks w, w+16, ... of every chunk, for every tile of the pass.
//   * programmatic dependent launch: the weights of every initially free stage are requested
//     before griddepcontrol.wait (they are not written by the previous kernel); activations and the
//     outputs are touched only after it.
//
// Math per (tile, block) in one warp: the nibbles of rows g and g+8 (lane = 4g + t holds
// bytes 4t..4t+3 of the block's 16) are turned into bf16 values 136 + q by one lop3 per pair
// (magic exponent 0x43 = 128, nibble ^ 8 = q + 8) and fed as the A operand of two
// mma.sync.m16n8k16 bf16 MMAs (low nibbles = k 0..15, high = k 16..31) whose B operand is
// the raw bf16 activations.  The fp32 block sums would hold sum(q x) + 136 sum(x); the
// offset is removed through the MMA's accumulator input, -136 Sx, where Sx (the activation
// block sums) comes once per block from the same MMA with an all-ones A.  The block scale is
// then applied in fp32: acc += s * D.  q and x are exact in bf16, so the only rounding is
// the fp32 accumulation.  fp32 activations are split into two bf16 terms (hi + lo).
//
// The 16 warps' partial sums of a tile meet in shared memory at the end of a pass, in a fixed
// order (the result does not depend on timing).  Shared memory is read by 32-bit shared
// addresses only.
#include <cstdlib>
#include <cstring>

#include "kernels.h"

#include <atomic>
#include <mutex>

namespace bybycu {

namespace {

// Consumer warps of the M >= 2 kernel: 16, one CTA per SM, where a CTA makes several passes
// over its rows; 8 where it makes one, so that two CTAs fit an SM (registers) and a launch's
// CTAs stream beside the previous launch's, as the M = 1 kernel's do (4096 x 4096 at M = 2:
// 7.0 against 9.3 us; the 128256-row head at M = 4, several passes: 93 against 105 us).
constexpr int kWarpsMany = 16, kWarpsOnePass = 8;
constexpr int kTileRows = 16;
constexpr int kRedSlots = 4;                        // partial-sum slots of the cross-warp reduction
constexpr uint32_t kMagicA = 0x43084308u;           // bf16 128 | (nibble ^ 8) via lop3
constexpr uint32_t kOnesBf16x2 = 0x3F803F80u;

struct GemvParams {
    int M, K, N, G;
    int tiles_base, tiles_extra;   // contiguous split over the grid: tiles, or rows with row_split
    int row_split;                 // M = 1: every CTA takes 74 or 75 rows (say), not 4 or 5 tiles
    int rem_rows;                  // row_split: rows of the short last pass of a base-size CTA
    int kc;                        // K values per chunk (512, 1024 or 2048)
    int n_chunks;
    int stages;
    int tp;                        // tiles per pass (<= TP)
    int scale_tma;                 // scales arrive by TMA (K % 256 == 0, 16-byte aligned)
    int x_pitch;                   // bytes between activation rows in shared memory
    uint32_t stage_bytes;          // W boxes + scale box + activations
    uint32_t w_box_bytes;          // one nibble box: 16 * TP rows x 128 B
    uint32_t s_off, x_off;         // offsets inside a stage
    uint32_t s_pitch;              // bytes per row of the scale box
    int x_whole;                   // M = 1 integer mode: the activation row arrives once per launch,
    uint32_t xbar_off;             // one 1024-value chunk per barrier (then one "digits ready"
    uint32_t x_all_off;            // barrier per chunk), at x_all_off; block factors after it
    int zeros;                     // asymmetric Q4: a zero-point box beside each scale box ...
    uint32_t z_off;                // ... at this offset inside the stage
    const __half* scales;          // packed + scale_base
    const uint8_t* x;              // activations [M, K] (global)
    int x_elem;                    // 2 (bf16) or 4 (fp32)
    void* out;
    int out_bf16;
    int64_t out_ld, out_col0;
    PeerGather pg;                 // world > 1: every output value also goes to every peer
};

// End of a GEMV launch that gathers: the barrier orders every consumer thread's stores before
// thread 0's release (cumulative), then the last CTA signals the ranks and waits for theirs.
// One release per CTA: a system fence per thread cost microseconds per step.
__device__ __forceinline__ void gemv_gather_end(const PeerGather& pg, uint32_t consumer_threads) {
    if (pg.world <= 1) return;
    named_barrier(2, consumer_threads);
    if (threadIdx.x == 0) peer_gather_finish(pg);
}

// Three nibble maps and three scale maps: boxes of 16 * TP rows (full pass), 16 * (TP - 1)
// rows (the short pass of a balanced split) and 16 rows (any other remainder).
struct GemvMaps {
    CUtensorMap w[3];
    CUtensorMap s[3];
    CUtensorMap z[3];   // asymmetric Q4 only: the fp32 zero points, boxed like the scales
};

// The nibbles in bits 0-3 and 16-19 of `a` as two bf16 values 128 + (nibble ^ 8) = 136 + q:
// (a & 0x000F000F) ^ 0x43084308 (the bf16 exponent of 128, and the xor with 8), one LOP3.
__device__ __forceinline__ uint32_t lop3_magic(uint32_t a) { return (a & 0x000F000Fu) ^ kMagicA; }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }

// d = a * b + c  (m16n8k16, bf16 inputs, fp32 accumulators)
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                         const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %11, %12, %13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// d = a * b + c  (m16n8k16, fp16 inputs, fp32 accumulators)
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                        const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %11, %12, %13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// d += a * b  (m16n8k32, s8 inputs, s32 accumulators)
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16 dequantisation: the low nibbles (bits 0-3 / 16-19) become 1024 + (nibble ^ 8) =
// 1032 + q, the high nibbles stay in place (bits 4-7 / 20-23, still mantissa in fp16) and
// become 1024 + 16 (nibble ^ 8) = 1152 + 16 q; one LOP3 each.
__device__ __forceinline__ uint32_t f16_lo(uint32_t a) { return (a & 0x000F000Fu) ^ 0x64086408u; }
__device__ __forceinline__ uint32_t f16_hi(uint32_t a) { return (a & 0x00F000F0u) ^ 0x64806480u; }

// bf16 pair -> fp16 pair (exact for |x| >= 2^-17), optionally scaled by 1/16 (exact).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v, float scale) {
    const float lo = __uint_as_float(v << 16) * scale, hi = __uint_as_float(v & 0xFFFF0000u) * scale;
    const __half2 h = __floats2half2_rn(lo, hi);
    uint32_t r;
    memcpy(&r, &h, sizeof r);
    return r;
}

// The B fragment of one 16-k half block for activation row `m` (lane = 4g + t):
// k slots (2t, 2t+1) <-> elements (4t, 4t+2), slots (2t+8, 2t+9) <-> (4t+1, 4t+3), matching
// the A fragment built from the nibble bytes 4t..4t+3.  (e01, e23) hold elements 4t..4t+3.
__device__ __forceinline__ void b_frag(uint32_t e01, uint32_t e23, uint32_t& b0, uint32_t& b1) {
    b0 = prmt(e01, e23, 0x5410);
    b1 = prmt(e01, e23, 0x7632);
}

// Plain C++ loads from the shared window: ordinary memory accesses, so the compiler may
// schedule them freely among the math but never above a barrier wait (a memory clobber).
__device__ __forceinline__ uint32_t sh_u32(const uint8_t* smem, uint32_t off) {
    return *reinterpret_cast<const uint32_t*>(smem + off);
}
__device__ __forceinline__ uint2 sh_u64(const uint8_t* smem, uint32_t off) {
    return *reinterpret_cast<const uint2*>(smem + off);
}
__device__ __forceinline__ uint4 sh_u128(const uint8_t* smem, uint32_t off) {
    return *reinterpret_cast<const uint4*>(smem + off);
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t v) {
    __half2 h;
    memcpy(&h, &v, sizeof h);
    return __half22float2(h);
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

// The producer: lane 0 of the last warp streams every (pass, chunk) iteration of this CTA into
// the stage ring (see the file comment).  Shared by the M = 1 and the general kernels.
__device__ __forceinline__ void gemv_producer(const GemvMaps& maps, const GemvParams& p, uint8_t* smem,
                                              uint64_t* full_bar, uint64_t* empty_bar, volatile int* s_abort,
                                              int lane, int tile_begin, int my_tiles, int total_it) {
    // units: tiles, or rows with row_split; a pass covers `upass` of them
    const int wboxes = p.kc / 256;
    const int upass = p.row_split ? p.tp * kTileRows : p.tp;
    if (lane == 0) {
        for (int i = 0; i < 3; ++i) {
            prefetch_tensormap(&maps.w[i]);
            if (p.scale_tma) prefetch_tensormap(&maps.s[i]);
            if (p.zeros) prefetch_tensormap(&maps.z[i]);
        }
        const uint64_t policy = l2_policy_evict_first();
        // Issues the weight part of iteration (chunk, t0) into stage s and arms its barrier.
        auto issue_weights = [&](int s, int chunk, int t0) {
            const int nu = min(upass, tile_begin + my_tiles - t0);
            const int nt = p.row_split ? (nu + kTileRows - 1) / kTileRows : nu;
            const int k0 = chunk * p.kc;
            const int kn = min(p.kc, p.K - k0);
            const uint32_t rows = p.row_split ? nu : nt * kTileRows;
            const uint32_t bytes = wboxes * rows * 128 + (p.scale_tma ? rows * p.s_pitch : 0) +
                                   (p.zeros ? rows * p.s_pitch : 0) +
                                   (p.x_whole ? 0u : p.M * static_cast<uint32_t>(kn) * p.x_elem);
            uint8_t* st = smem + static_cast<size_t>(s) * p.stage_bytes;
            mbar_arrive_expect_tx(&full_bar[s], bytes);
            if (p.row_split) {   // one box of exactly the pass's rows: full, or one of two short heights
                const int mi = nu == upass ? 0 : (nu == p.rem_rows ? 1 : 2);
                for (int bx = 0; bx < wboxes; ++bx)
                    tma_load_2d_hint(st + bx * p.w_box_bytes, &maps.w[mi], &full_bar[s], k0 / 2 + bx * 128, t0,
                                     policy);
                if (p.scale_tma) tma_load_2d(st + p.s_off, &maps.s[mi], &full_bar[s], k0 / 32, t0);
                return;
            }
            // one box per 16 * nt rows when nt is TP or TP - 1, else one per tile
            const int mi = nt == p.tp ? 0 : (nt == p.tp - 1 ? 1 : 2);
            const int pieces = mi == 2 ? nt : 1;
            for (int q = 0; q < pieces; ++q) {
                const int row = (t0 + q) * kTileRows;
                const uint32_t roff = q * kTileRows * 128;
                for (int bx = 0; bx < wboxes; ++bx)
                    tma_load_2d_hint(st + bx * p.w_box_bytes + roff, &maps.w[mi], &full_bar[s], k0 / 2 + bx * 128,
                                     row, policy);
                if (p.scale_tma)
                    tma_load_2d(st + p.s_off + q * kTileRows * p.s_pitch, &maps.s[mi], &full_bar[s], k0 / 32, row);
                if (p.zeros)
                    tma_load_2d(st + p.z_off + q * kTileRows * p.s_pitch, &maps.z[mi], &full_bar[s], k0 / 32, row);
            }
        };
        // Issues the activation rows of iteration `chunk` into stage s.
        auto issue_x = [&](int s, int chunk) {
            if (p.x_whole) return;
            const int k0 = chunk * p.kc;
            const uint32_t x_row_bytes = static_cast<uint32_t>(min(p.kc, p.K - k0)) * p.x_elem;
            uint8_t* st = smem + static_cast<size_t>(s) * p.stage_bytes;
            for (int m = 0; m < p.M; ++m)
                bulk_load_1d(st + p.x_off + m * p.x_pitch, p.x + (static_cast<size_t>(m) * p.K + k0) * p.x_elem,
                             x_row_bytes, &full_bar[s]);
        };
        // Prologue: the weights of every free stage before griddepcontrol.wait (the previous
        // kernel does not write them), the activations after it.
        const int first = min(p.stages, total_it);
        {
            int chunk = 0, t0 = tile_begin;
            for (int it = 0; it < first; ++it) {
                issue_weights(it, chunk, t0);
                if (++chunk == p.n_chunks) { chunk = 0; t0 += upass; }
            }
            pdl_wait();
            // split-phase gather: every rank finished the previous launch (x may be its output,
            // and this launch's stores overwrite what that launch's readers read); on a
            // timeout the error is recorded and the launch goes on
            peer_gather_wait_previous(p.pg);
            if (p.x_whole) {   // the whole row, chunk by chunk, each on its own barrier
                uint64_t* x_bar = reinterpret_cast<uint64_t*>(smem + p.xbar_off);
                for (int c = 0; c < p.n_chunks; ++c) {
                    const uint32_t bytes = static_cast<uint32_t>(min(p.kc, p.K - c * p.kc)) * p.x_elem;
                    mbar_arrive_expect_tx(&x_bar[c], bytes);
                    bulk_load_1d(smem + p.x_all_off + static_cast<uint32_t>(c * p.kc) * p.x_elem,
                                 p.x + static_cast<size_t>(c) * p.kc * p.x_elem, bytes, &x_bar[c]);
                }
            }
            chunk = 0;
            for (int it = 0; it < first; ++it) {
                issue_x(it, chunk);
                if (++chunk == p.n_chunks) chunk = 0;
            }
        }
        int issued = first;
        int s = first % p.stages, round = first / p.stages;
        int chunk = first % p.n_chunks, t0 = tile_begin + (first / p.n_chunks) * upass;
        for (int it = first; it < total_it; ++it) {
            if (*s_abort) break;
            if (!mbar_wait_bounded(&empty_bar[s], (round - 1) & 1, kDevErrEmptyWait)) {
                *s_abort = 1;
                break;
            }
            issue_weights(s, chunk, t0);
            issue_x(s, chunk);
            issued = it + 1;
            if (++s == p.stages) { s = 0; ++round; }
            if (++chunk == p.n_chunks) { chunk = 0; t0 += upass; }
        }
        // Before the CTA may exit, every copy it issued must have landed.
        for (int it = max(0, issued - p.stages); it < issued; ++it) {
            const int ds = it % p.stages;
            if (!mbar_wait_bounded(&full_bar[ds], (it / p.stages) & 1, kDevErrDrainWait)) break;
        }
        if (p.x_whole)
            for (int c = 0; c < p.n_chunks; ++c)
                if (!mbar_wait_bounded(reinterpret_cast<uint64_t*>(smem + p.xbar_off) + c, 0, kDevErrDrainWait)) break;
    }
}

template <int TP, int NT, bool XF32, bool STMA, int W>
__global__ void __launch_bounds__((W + 1) * 32, W <= 8 ? 2 : 1)
gemv_q4b32_kernel(const __grid_constant__ GemvMaps maps, const GemvParams p) {
    constexpr int H = XF32 ? 2 : 1;   // bf16 terms per activation
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1 KiB-aligned base, kept in the shared window (32-bit addresses, shared loads only)
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(p.stages) * p.stage_bytes);
    uint64_t* empty_bar = full_bar + p.stages;
    volatile int* s_abort = reinterpret_cast<volatile int*>(empty_bar + p.stages);
    const uint32_t red = smem_u32(empty_bar + p.stages + 2);   // [kRedSlots][TP * NT * 128] floats

    pdl_launch_dependents();
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
            mbar_init(&empty_bar[s], W);
        }
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == W) {
        gemv_producer(maps, p, smem, full_bar, empty_bar, s_abort, lane, tile_begin, my_tiles, total_it);
        return;
    }

    // ---------------------------------------------------------------------- consumers
    pdl_wait();   // outputs may be read by the previous kernel; activations come from it
    const int g = lane >> 2, t = lane & 3;
    float acc[TP][NT][4];
#pragma unroll
    for (int i = 0; i < TP; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[i][j][v] = 0.0f;
    const uint32_t ones[4] = {kOnesBf16x2, kOnesBf16x2, kOnesBf16x2, kOnesBf16x2};
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    const int qblocks = p.kc / (32 * W);   // blocks of this warp per chunk: warp, warp + W, ...

    int s = 0, round = 0, chunk = 0, t0 = tile_begin;
    for (int it = 0; it < total_it; ++it) {
        const int nt = min(p.tp, tile_begin + my_tiles - t0);
        bool ok = !*s_abort;
        if (ok && !mbar_wait_bounded(&full_bar[s], round & 1, kDevErrFullWait)) {
            *s_abort = 1;
            ok = false;
        }
        const uint32_t st = base + static_cast<uint32_t>(s) * p.stage_bytes;
        for (int qb = 0; qb < qblocks; ++qb) {
            const int cb = warp + W * qb;   // block within the chunk
            const int c = chunk * (p.kc / 32) + cb;  // block within the row
            if (!ok || c >= p.G) break;
            // ---- activation fragments of block c (B operands); the offset term 136 * sum(x)
            //      goes into the MMA accumulator input
            uint32_t blo[NT][H][2], bhi[NT][H][2];
            float negcorr[NT][4];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int m = j * 8 + g;
                const bool live = m < p.M;
                const uint32_t xr = st + p.x_off + m * p.x_pitch;
                if constexpr (!XF32) {
                    uint2 lo = make_uint2(0u, 0u), hi = make_uint2(0u, 0u);
                    if (live) {
                        lo = lds_u64(xr + (32 * cb + 4 * t) * 2);
                        hi = lds_u64(xr + (32 * cb + 16 + 4 * t) * 2);
                    }
                    b_frag(lo.x, lo.y, blo[j][0][0], blo[j][0][1]);
                    b_frag(hi.x, hi.y, bhi[j][0][0], bhi[j][0][1]);
                } else {
                    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
                    if (live) {
                        const uint4 a = lds_u128(xr + (32 * cb + 4 * t) * 4);
                        const uint4 bb = lds_u128(xr + (32 * cb + 16 + 4 * t) * 4);
                        lo = make_float4(__uint_as_float(a.x), __uint_as_float(a.y), __uint_as_float(a.z),
                                         __uint_as_float(a.w));
                        hi = make_float4(__uint_as_float(bb.x), __uint_as_float(bb.y), __uint_as_float(bb.z),
                                         __uint_as_float(bb.w));
                    }
                    split_f32(lo, blo[j][0][0], blo[j][0][1], blo[j][1][0], blo[j][1][1]);
                    split_f32(hi, bhi[j][0][0], bhi[j][0][1], bhi[j][1][0], bhi[j][1][1]);
                }
                float sx[4];
                mma_bf16(sx, ones, blo[j][0][0], blo[j][0][1], zero4);
                mma_bf16(sx, ones, bhi[j][0][0], bhi[j][0][1], sx);
                if constexpr (XF32) {
                    mma_bf16(sx, ones, blo[j][1][0], blo[j][1][1], sx);
                    mma_bf16(sx, ones, bhi[j][1][0], bhi[j][1][1], sx);
                }
#pragma unroll
                for (int v = 0; v < 4; ++v) negcorr[j][v] = -136.0f * sx[v];
            }
            // this lane's word of block cb in the nibble box (row g; row g + 8 is 1 KiB further)
            const uint32_t wl = st + (cb >> 3) * p.w_box_bytes + g * 128 + ((((cb & 7) ^ g)) << 4) + 4 * t;
            const uint32_t sl = st + p.s_off + g * p.s_pitch +
                                (p.s_pitch == 128 ? ((((cb >> 3) ^ g) << 4) + 2 * (cb & 7)) : 2 * cb);
            // ---- per tile: dequantise rows g and g+8 of block c, two MMAs, scale in fp32.
            //      Every tile slot runs (no branch, so the compiler interleaves the TP
            //      independent tiles); the partial sums of slots >= nt are never stored.
#pragma unroll
            for (int i = 0; i < TP; ++i) {
                const uint32_t wt = wl + i * (kTileRows * 128);
                const uint32_t w0 = lds_u32(wt);
                const uint32_t w8 = lds_u32(wt + 1024);
                float s0, s8;
                if constexpr (STMA) {
                    const uint32_t sc = sl + i * kTileRows * p.s_pitch;
                    s0 = __half2float(__ushort_as_half(lds_u16(sc)));
                    s8 = __half2float(__ushort_as_half(lds_u16(sc + 8 * p.s_pitch)));
                } else {
                    const int64_t row0 = static_cast<int64_t>(t0 + i) * kTileRows + g;
                    s0 = (i < nt && row0 < p.N) ? __half2float(p.scales[row0 * p.G + c]) : 0.0f;
                    s8 = (i < nt && row0 + 8 < p.N) ? __half2float(p.scales[(row0 + 8) * p.G + c]) : 0.0f;
                }
                uint32_t alo[4], ahi[4];
                alo[0] = lop3_magic(w0);
                alo[1] = lop3_magic(w8);
                alo[2] = lop3_magic(w0 >> 8);
                alo[3] = lop3_magic(w8 >> 8);
                ahi[0] = lop3_magic(w0 >> 4);
                ahi[1] = lop3_magic(w8 >> 4);
                ahi[2] = lop3_magic(w0 >> 12);
                ahi[3] = lop3_magic(w8 >> 12);
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    float d[4];
                    mma_bf16(d, alo, blo[j][0][0], blo[j][0][1], negcorr[j]);
                    mma_bf16(d, ahi, bhi[j][0][0], bhi[j][0][1], d);
                    if constexpr (XF32) {
                        mma_bf16(d, alo, blo[j][1][0], blo[j][1][1], d);
                        mma_bf16(d, ahi, bhi[j][1][0], bhi[j][1][1], d);
                    }
                    acc[i][j][0] = fmaf(s0, d[0], acc[i][j][0]);
                    acc[i][j][1] = fmaf(s0, d[1], acc[i][j][1]);
                    acc[i][j][2] = fmaf(s8, d[2], acc[i][j][2]);
                    acc[i][j][3] = fmaf(s8, d[3], acc[i][j][3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        if (++s == p.stages) { s = 0; ++round; }

        if (chunk == p.n_chunks - 1) {
            // ---- end of pass: the warps' partial sums meet in shared memory in a fixed order:
            //      the last four warps store, then each group of four below adds in turn
            constexpr int E = TP * NT * 128;
            const uint32_t slot = red + static_cast<uint32_t>((warp & 3) * E * 4);
#pragma unroll
            for (int phase = W / 4 - 1; phase >= 0; --phase) {
                if ((warp >> 2) == phase) {
#pragma unroll
                    for (int i = 0; i < TP; ++i)
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            const uint32_t a = slot + ((i * NT + j) * 32 + lane) * 16;
                            if (phase == W / 4 - 1) {
                                sts_v4(a, acc[i][j][0], acc[i][j][1], acc[i][j][2], acc[i][j][3]);
                            } else {
                                const float4 o = lds_v4f(a);
                                sts_v4(a, o.x + acc[i][j][0], o.y + acc[i][j][1], o.z + acc[i][j][2],
                                       o.w + acc[i][j][3]);
                            }
                        }
                }
                named_barrier(1, W * 32);
            }
#pragma unroll
            for (int i = 0; i < TP; ++i)
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int v = 0; v < 4; ++v) acc[i][j][v] = 0.0f;
            const int entries = nt * NT * 128;
            for (int e = threadIdx.x; e < entries; e += W * 32) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kRedSlots; ++w) sum += lds_f32(red + static_cast<uint32_t>((w * E + e) * 4));
                const int v = e & 3, ln = (e >> 2) & 31, ij = e >> 7;
                const int j = ij % NT, i = ij / NT;
                const int gg = ln >> 2, tt = ln & 3;
                const int64_t n = static_cast<int64_t>(t0 + i) * kTileRows + gg + (v >= 2 ? 8 : 0);
                const int m = j * 8 + 2 * tt + (v & 1);
                if (n < p.N && m < p.M) {
                    const int64_t oi = static_cast<int64_t>(m) * p.out_ld + p.out_col0 + n;
                    if (p.out_bf16) reinterpret_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(sum);
                    else reinterpret_cast<float*>(p.out)[oi] = sum;
                    if (p.pg.world > 1) store_to_peers(p.pg, oi, sum);
                }
            }
            named_barrier(1, W * 32);
        }
        if (++chunk == p.n_chunks) { chunk = 0; t0 += p.tp; }
    }
    gemv_gather_end(p.pg, W * 32);
}


// ----------------------------------------------------------------------------------------
// M = 1 (decode) kernel.  The MMA's N dimension carries 8 blocks instead of 8 activation
// rows: column j of B holds block j's activations on that block's k slots and zeros on the
// others (block-diagonal), so one chain of MMAs over a 256-value box of K accumulates
// D[row][j] = offset_j + sum_{k in block j} q[row][k] x[k] for the box's blocks at once; the
// offset (136 sum(x_j) for bf16 operands) comes from the same MMA with a constant A and is
// removed in the fp32 epilogue, which runs once per chain instead of once per block.
// kM1Warps consumer warps: kM1Warps / 4 per 256-value box of a 1024-value chunk, each owning
// 8 / (kM1Warps / 4) blocks of the box.  The nibble dequantisation (one LOP3 per two weights,
// after a shift) runs on the ALU pipe, the kernel's binding resource; the block-diagonal
// selects are computed once per chunk and pinned in registers.
//
// The integer mode (the default) skips the dequantisation instead: a packed word already
// holds eight signed nibbles, and one AND (after a 4-bit shift for the low nibbles) turns it
// into four s8 values 16 q in exactly the K order of an m16n8k32 A fragment.  The activations
// of each 32-block become a fixed-point image X = rint(x * 2^(140 - E)) (E = the block's
// largest bf16 exponent, so |X| <= 2^14: exact for every element within 7 binades of the
// block's largest, 2^-15 of it otherwise) split into two signed byte digits,
// X = 256 h + sext8(X); an fp32 row adds a second image of the remainder (fp32's 24 bits are
// more than one image holds).  The four blocks of a warp share one accumulator: block j's low and
// high digits occupy B columns 2j and 2j+1, so four s8 MMAs (K = 32 each) fill all eight
// columns and lane (g, t) ends with block t's two digit sums for rows g and g + 8, exact in
// int32.  The epilogue is one integer combine, one conversion and one FMA with
// scale * 2^(E - 144) per row and block.
// ----------------------------------------------------------------------------------------
#ifndef BYBYCU_GEMV_M1_WARPS
#define BYBYCU_GEMV_M1_WARPS 8
#endif
constexpr int kM1Warps = BYBYCU_GEMV_M1_WARPS;   // 8 or 16
constexpr int kM1Threads = (kM1Warps + 2) * 32;   // + the producer and the digit warp
constexpr int kM1KC = 1024;
constexpr int kM1Parts = kM1Warps / 4;            // warps per box
constexpr int kM1Blocks = 8 / kM1Parts;           // blocks per warp
// operand modes of the M = 1 kernel
constexpr int kM1Bf16 = 0;   // bf16 MMAs on 136 + q
constexpr int kM1F16 = 1;    // fp16 MMAs on 1032 + q / 1152 + 16 q
constexpr int kM1I8 = 2;     // s8 MMAs on 16 q and two-digit fixed-point activations

// One 1024-value stage of the integer mode for one warp: blocks blk0 .. blk0 + 3 of box
// `box` (c0 = the box's first block of K) for the pass's nt tiles.  Lane (g, t) builds digit
// g % 2 of block g / 2 (its elements 4t..4t+3 and 16+4t..16+4t+3, the B fragment's k slots)
// and accumulates block t of each tile into acc.
// The integer mode's activation side, done by the digit warp once per launch: the resident
// bf16 (or fp32) row is turned in place into B-fragment words.  Lane t of quad g converts blocks g,
// g + 8, g + 16 and g + 24 of a chunk: in each it reads elements 4t..4t+3 (bytes 8t..8t+7 of
// the block) and 16+4t..16+4t+3 (bytes 32+8t..) and writes back at exactly those bytes the
// low and the high digits of the same elements, so block b's 64 bytes become
// [digit][t][k 4t.. | k 16+4t..] in s8.  X = rint(x * 2^(140 - E)) comes from one FFMA with
// 1.5 * 2^23, which leaves X, rounded to nearest even, in the float's low bits: its low byte
// is the low digit, and the second byte of the same sum with 128 more is the high digit
// (X + 128) >> 8.  The factor 2^(E - 144) of each block (it undoes the scaling and the 16 of
// the 16 q operands) goes to the factor table.  All loads come before all stores, so the four
// blocks' dependency chains overlap.  An fp32 row keeps 128 bytes per block; its digits take
// the first 64 of them, and the last 64 hold a second image of what the first leaves out:
// R = x * 2^(140 - E) - X (exact, |R| <= 1/2) as X2 = rint(R * 2^15) in the same two-digit
// form, so the pair carries x to 2^-29 of the block's largest value (fp32 keeps 2^-24 of
// each value).  Lane t's loads at bytes 16t.. and 64+16t.. feed the block's exponent, which
// the quad shuffles before any lane stores, so no store lands on bytes still unread.
template <bool XF32>
__device__ __forceinline__ float m1_x_elem(const uint2& lo, const uint2& hi, const uint4& lo4, const uint4& hi4, int i) {
    if constexpr (XF32) {
        const uint32_t w[8] = {lo4.x, lo4.y, lo4.z, lo4.w, hi4.x, hi4.y, hi4.z, hi4.w};
        return __uint_as_float(w[i]);
    } else {
        const uint32_t w[4] = {lo.x, lo.y, hi.x, hi.y};
        return __uint_as_float((i & 1) ? (w[i >> 1] & 0xFFFF0000u) : (w[i >> 1] << 16));
    }
}

// The biased exponent of the largest magnitude among a lane's 8 raw activations:
// magnitude bit patterns order like the values, and inf / NaN sort above every finite value.
template <bool XF32>
__device__ __forceinline__ int m1_max_exp(const uint2& lo, const uint2& hi, const uint4& lo4, const uint4& hi4) {
    if constexpr (XF32) {
        const uint32_t m = max(max(max(lo4.x & 0x7FFFFFFFu, lo4.y & 0x7FFFFFFFu), max(lo4.z & 0x7FFFFFFFu, lo4.w & 0x7FFFFFFFu)),
                               max(max(hi4.x & 0x7FFFFFFFu, hi4.y & 0x7FFFFFFFu), max(hi4.z & 0x7FFFFFFFu, hi4.w & 0x7FFFFFFFu)));
        return static_cast<int>(m >> 23);
    } else {
        const uint32_t m2 = __vmaxu2(__vmaxu2(lo.x & 0x7FFF7FFFu, lo.y & 0x7FFF7FFFu),
                                     __vmaxu2(hi.x & 0x7FFF7FFFu, hi.y & 0x7FFF7FFFu));
        return static_cast<int>(max(m2 & 0xFFFFu, m2 >> 16) >> 7);
    }
}

template <bool XF32>
__device__ __forceinline__ void m1_digits_chunk(const GemvParams& p, uint8_t* smem, int chunk, int g, int t) {
    constexpr int J = 4;
    constexpr uint32_t kPitch = XF32 ? 128u : 64u;   // bytes of one block of the resident row
    constexpr uint32_t kElem = XF32 ? 4u : 2u;
    uint2 lo[J], hi[J];
    uint4 lo4[J], hi4[J];
    uint32_t xr[J];
    bool live[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int blk = chunk * (kM1KC / 32) + 8 * j + g;
        live[j] = blk < p.G;
        xr[j] = p.x_all_off + blk * kPitch;
        if constexpr (XF32) {
            lo4[j] = live[j] ? sh_u128(smem, xr[j] + 16 * t) : make_uint4(0u, 0u, 0u, 0u);
            hi4[j] = live[j] ? sh_u128(smem, xr[j] + 64 + 16 * t) : make_uint4(0u, 0u, 0u, 0u);
        } else {
            lo[j] = live[j] ? sh_u64(smem, xr[j] + 8 * t) : make_uint2(0u, 0u);
            hi[j] = live[j] ? sh_u64(smem, xr[j] + 32 + 8 * t) : make_uint2(0u, 0u);
        }
    }
    int e[J];
#pragma unroll
    for (int j = 0; j < J; ++j) e[j] = m1_max_exp<XF32>(lo[j], hi[j], lo4[j], hi4[j]);
#pragma unroll
    for (int j = 0; j < J; ++j) e[j] = max(e[j], __shfl_xor_sync(0xffffffffu, e[j], 1));
#pragma unroll
    for (int j = 0; j < J; ++j) e[j] = max(e[j], __shfl_xor_sync(0xffffffffu, e[j], 2));
    uint32_t out[J][4], out2[J][4];   // out2: fp32 rows' second image
#pragma unroll
    for (int j = 0; j < J; ++j) {
        if (live[j] && e[j] == 255 && t == 0) record_device_error(kDevErrActRange);   // inf or NaN
        e[j] = max(e[j], 18);                                  // blocks below 2^-109: normal factors
        const float up = __int_as_float((267 - e[j]) << 23);   // 2^(140 - E)
        uint32_t r[8], h[8], r2[8], h2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float f = m1_x_elem<XF32>(lo[j], hi[j], lo4[j], hi4[j], i);
            r[i] = __float_as_uint(fmaf(f, up, 12582912.0f));   // 0x4B400000 + X
            h[i] = __float_as_uint(fmaf(f, up, 12583040.0f));   // 0x4B400000 + X + 128
            if constexpr (XF32) {
                const float rem = fmaf(f, up, -(__uint_as_float(r[i]) - 12582912.0f));   // R, exact
                r2[i] = __float_as_uint(fmaf(rem, 32768.0f, 12582912.0f));
                h2[i] = __float_as_uint(fmaf(rem, 32768.0f, 12583040.0f));
            }
        }
        out[j][0] = prmt(prmt(r[0], r[1], 0x0040), prmt(r[2], r[3], 0x0040), 0x5410);
        out[j][1] = prmt(prmt(r[4], r[5], 0x0040), prmt(r[6], r[7], 0x0040), 0x5410);
        out[j][2] = prmt(prmt(h[0], h[1], 0x0051), prmt(h[2], h[3], 0x0051), 0x5410);
        out[j][3] = prmt(prmt(h[4], h[5], 0x0051), prmt(h[6], h[7], 0x0051), 0x5410);
        if constexpr (XF32) {
            out2[j][0] = prmt(prmt(r2[0], r2[1], 0x0040), prmt(r2[2], r2[3], 0x0040), 0x5410);
            out2[j][1] = prmt(prmt(r2[4], r2[5], 0x0040), prmt(r2[6], r2[7], 0x0040), 0x5410);
            out2[j][2] = prmt(prmt(h2[0], h2[1], 0x0051), prmt(h2[2], h2[3], 0x0051), 0x5410);
            out2[j][3] = prmt(prmt(h2[4], h2[5], 0x0051), prmt(h2[6], h2[7], 0x0051), 0x5410);
        }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
        if (!live[j]) continue;
        *reinterpret_cast<uint2*>(smem + xr[j] + 8 * t) = make_uint2(out[j][0], out[j][1]);
        *reinterpret_cast<uint2*>(smem + xr[j] + 32 + 8 * t) = make_uint2(out[j][2], out[j][3]);
        if constexpr (XF32) {
            *reinterpret_cast<uint2*>(smem + xr[j] + 64 + 8 * t) = make_uint2(out2[j][0], out2[j][1]);
            *reinterpret_cast<uint2*>(smem + xr[j] + 96 + 8 * t) = make_uint2(out2[j][2], out2[j][3]);
        }
        if (t == 0)
            *reinterpret_cast<float*>(smem + p.x_all_off + static_cast<uint32_t>(p.K) * kElem +
                                      (chunk * (kM1KC / 32) + 8 * j + g) * 4) = __int_as_float((e[j] - 17) << 23);
    }
}

// The digit warp: converts chunks 1, 2, ... as their activations land and marks each ready
// (the consumers build chunk 0's operands themselves from the raw row, so that the first
// MMAs wait for no conversion).  It always marks a chunk, after a timeout too, so that no
// consumer waits for it in vain.
template <bool XF32>
__device__ __forceinline__ void m1_digit_warp(const GemvParams& p, uint8_t* smem, volatile int* s_abort, int lane) {
    uint64_t* x_bar = reinterpret_cast<uint64_t*>(smem + p.xbar_off);
    uint64_t* ready = x_bar + p.n_chunks;
    for (int c = 1; c < p.n_chunks; ++c) {
        if (!*s_abort && !mbar_wait_bounded(&x_bar[c], 0, kDevErrFullWait)) *s_abort = 1;
        m1_digits_chunk<XF32>(p, smem, c, lane >> 2, lane & 3);
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[c]);   // release: the digits above before the arrival
    }
}

// Four raw bf16 activations (pairs e01, e23) -> one digit byte each, as in m1_digits_chunk:
// magic 1.5 * 2^23 and byte 0 for the low digit, magic + 128 and byte 1 for the high one.
__device__ __forceinline__ uint32_t digit4(uint32_t e01, uint32_t e23, float up, float magic, uint32_t sel) {
    const uint32_t r0 = __float_as_uint(fmaf(__uint_as_float(e01 << 16), up, magic));
    const uint32_t r1 = __float_as_uint(fmaf(__uint_as_float(e01 & 0xFFFF0000u), up, magic));
    const uint32_t r2 = __float_as_uint(fmaf(__uint_as_float(e23 << 16), up, magic));
    const uint32_t r3 = __float_as_uint(fmaf(__uint_as_float(e23 & 0xFFFF0000u), up, magic));
    return prmt(prmt(r0, r1, sel), prmt(r2, r3, sel), 0x5410);
}
// The same for four raw fp32 activations.
__device__ __forceinline__ uint32_t digit4f(uint4 v, float up, float magic, uint32_t sel) {
    const uint32_t r0 = __float_as_uint(fmaf(__uint_as_float(v.x), up, magic));
    const uint32_t r1 = __float_as_uint(fmaf(__uint_as_float(v.y), up, magic));
    const uint32_t r2 = __float_as_uint(fmaf(__uint_as_float(v.z), up, magic));
    const uint32_t r3 = __float_as_uint(fmaf(__uint_as_float(v.w), up, magic));
    return prmt(prmt(r0, r1, sel), prmt(r2, r3, sel), 0x5410);
}
// The second image's digit of one raw fp32 activation: R = x * 2^(140 - E) - X, exact, then
// rint(R * 2^15) through the same magic-number form.
__device__ __forceinline__ uint32_t residual_digit(uint32_t v, float up, float magic) {
    const float f = __uint_as_float(v);
    const float x1 = __uint_as_float(__float_as_uint(fmaf(f, up, 12582912.0f))) - 12582912.0f;   // X
    return __float_as_uint(fmaf(fmaf(f, up, -x1), 32768.0f, magic));
}
// The same, for four raw fp32 activations.
__device__ __forceinline__ uint32_t residual4f(uint4 v, float up, float magic, uint32_t sel) {
    const uint32_t r0 = residual_digit(v.x, up, magic), r1 = residual_digit(v.y, up, magic);
    const uint32_t r2 = residual_digit(v.z, up, magic), r3 = residual_digit(v.w, up, magic);
    return prmt(prmt(r0, r1, sel), prmt(r2, r3, sel), 0x5410);
}

// The weight side of one chunk in the integer mode for one warp: blocks blk0 .. blk0 + 3 of
// box `box` (c0 = the box's first block of K) for the pass's nt tiles, accumulated into acc.
// Lane (g, t) feeds B column g (digit g % 2 of block g / 2) and combines block t's two digit
// sums for rows g and g + 8.  fp32 rows run a second chain of the same A operands over the
// second image's digits and add its sums with weight 2^-15.
template <int TP, bool STMA, bool XF32>
__device__ __forceinline__ void m1_i8_stage(const GemvParams& p, const uint8_t* smem, uint32_t st, int box, int blk0,
                                            int c0, int g, int t, int64_t row0, int64_t row_end,
                                            const uint32_t (&woff)[4], bool raw, float (&acc)[TP][2]) {
    constexpr uint32_t kPitch = XF32 ? 128u : 64u;   // bytes of one block of the resident row
    constexpr uint32_t kElem = XF32 ? 4u : 2u;
    const int q = g >> 1;
    const int bb = c0 + blk0 + q, bt = c0 + blk0 + t;
    uint2 dw, dw2 = make_uint2(0u, 0u);
    float ft;
    if (raw) {   // chunk 0: the digits from the raw row, here (the same arithmetic as m1_digits_chunk)
        const uint32_t xr = p.x_all_off + bb * kPitch + 4 * t * kElem;
        uint2 lo = make_uint2(0u, 0u), hi = make_uint2(0u, 0u);
        uint4 lo4 = make_uint4(0u, 0u, 0u, 0u), hi4 = make_uint4(0u, 0u, 0u, 0u);
        if (bb < p.G) {
            if constexpr (XF32) {
                lo4 = sh_u128(smem, xr);
                hi4 = sh_u128(smem, xr + 64);
            } else {
                lo = sh_u64(smem, xr);
                hi = sh_u64(smem, xr + 32);
            }
        }
        int e = m1_max_exp<XF32>(lo, hi, lo4, hi4);
        e = max(e, __shfl_xor_sync(0xffffffffu, e, 1));
        e = max(e, __shfl_xor_sync(0xffffffffu, e, 2));
        if (bb < p.G && e == 255 && t == 0 && !(g & 1)) record_device_error(kDevErrActRange);   // inf or NaN
        e = max(e, 18);
        const float up = __int_as_float((267 - e) << 23);
        const float magic = (g & 1) ? 12583040.0f : 12582912.0f;
        const uint32_t sel = (g & 1) ? 0x0051u : 0x0040u;
        if constexpr (XF32) {
            dw = make_uint2(digit4f(lo4, up, magic, sel), digit4f(hi4, up, magic, sel));
            dw2 = make_uint2(residual4f(lo4, up, magic, sel), residual4f(hi4, up, magic, sel));
        } else {
            dw = make_uint2(digit4(lo.x, lo.y, up, magic, sel), digit4(hi.x, hi.y, up, magic, sel));
        }
        const int et = __shfl_sync(0xffffffffu, e, 8 * t);   // lane 8t built block t
        ft = bt < p.G ? __int_as_float((et - 17) << 23) : 0.0f;
    } else {
        dw = bb < p.G ? sh_u64(smem, p.x_all_off + bb * kPitch + (g & 1) * 32 + 8 * t) : make_uint2(0u, 0u);
        if constexpr (XF32)
            dw2 = bb < p.G ? sh_u64(smem, p.x_all_off + bb * kPitch + 64 + (g & 1) * 32 + 8 * t) : make_uint2(0u, 0u);
        ft = bt < p.G ? *reinterpret_cast<const float*>(smem + p.x_all_off + static_cast<uint32_t>(p.K) * kElem + bt * 4)
                      : 0.0f;
    }
    uint32_t bq[4][2], bq2[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        bq[j][0] = q == j ? dw.x : 0u;
        bq[j][1] = q == j ? dw.y : 0u;
        asm volatile("" : "+r"(bq[j][0]), "+r"(bq[j][1]));   // keep them in registers
        if constexpr (XF32) {
            bq2[j][0] = q == j ? dw2.x : 0u;
            bq2[j][1] = q == j ? dw2.y : 0u;
            asm volatile("" : "+r"(bq2[j][0]), "+r"(bq2[j][1]));
        }
    }
    const uint32_t wbox = st + box * p.w_box_bytes;
#pragma unroll
    for (int i = 0; i < TP; ++i) {
        int d[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t wt = wbox + i * (kTileRows * 128) + woff[j];
            const uint32_t w0 = sh_u32(smem, wt);
            const uint32_t w8 = sh_u32(smem, wt + 1024);
            const uint32_t a[4] = {(w0 << 4) & 0xF0F0F0F0u, (w8 << 4) & 0xF0F0F0F0u, w0 & 0xF0F0F0F0u,
                                   w8 & 0xF0F0F0F0u};
            mma_s8(d, a, bq[j][0], bq[j][1]);
            if constexpr (XF32) mma_s8(d2, a, bq2[j][0], bq2[j][1]);
        }
        float v0 = static_cast<float>(d[0] + d[1] * 256), v8 = static_cast<float>(d[2] + d[3] * 256);
        if constexpr (XF32) {   // the second image: |sum| <= 2^26, exact in int32
            v0 = fmaf(static_cast<float>(d2[0] + d2[1] * 256), 1.0f / 32768.0f, v0);
            v8 = fmaf(static_cast<float>(d2[2] + d2[3] * 256), 1.0f / 32768.0f, v8);
        }
        float sg, sg8;
        if constexpr (STMA) {
            const uint32_t sa = st + p.s_off + (i * kTileRows + g) * p.s_pitch + (box * 8 + blk0 + t) * 2;
            sg = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(smem + sa)));
            sg8 = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(smem + sa + 8 * p.s_pitch)));
        } else {
            const int64_t r0 = row0 + i * kTileRows + g;
            const int ca = c0 + blk0 + t;
            const bool ok0 = r0 < row_end && ca < p.G, ok8 = r0 + 8 < row_end && ca < p.G;
            sg = ok0 ? __half2float(p.scales[r0 * p.G + ca]) : 0.0f;
            sg8 = ok8 ? __half2float(p.scales[(r0 + 8) * p.G + ca]) : 0.0f;
        }
        acc[i][0] = fmaf(sg * ft, v0, acc[i][0]);
        acc[i][1] = fmaf(sg8 * ft, v8, acc[i][1]);
    }
}

// Two CTAs per SM: the register cap (96) lets the next launch's CTA sit beside the running
// one, so its producer streams weights while this one computes (programmatic dependent launch).
template <int TP, bool STMA, int MODE, bool XF32 = false>
__global__ void __launch_bounds__(kM1Threads, 2)
gemv_m1_kernel(const __grid_constant__ GemvMaps maps, const GemvParams p) {
    static_assert(!XF32 || MODE == kM1I8, "fp32 activations: the integer mode only");
    constexpr int S = 2 * kM1Blocks;   // MMA steps per warp per box (low / high half per block)
    constexpr bool F16A = MODE == kM1F16;
    static_assert(MODE != kM1I8 || kM1Blocks == 4, "the integer mode fills 8 columns with 4 blocks x 2 digits");
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
    const int my_tiles = p.tiles_base + (b < p.tiles_extra ? 1 : 0);            // units: rows when row_split
    const int tile_begin = b * p.tiles_base + min(b, p.tiles_extra);
    const int upass = p.row_split ? p.tp * kTileRows : p.tp;
    const int passes = (my_tiles + upass - 1) / upass;
    const int total_it = passes * p.n_chunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kM1Warps);
        }
        if (MODE == kM1I8)   // per chunk: activations landed, digits ready
            for (int c = 0; c < 2 * p.n_chunks; ++c) mbar_init(reinterpret_cast<uint64_t*>(smem + p.xbar_off) + c, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kM1Warps) {
        gemv_producer(maps, p, smem, full_bar, empty_bar, s_abort, lane, tile_begin, my_tiles, total_it);
        return;
    }
    if (warp == kM1Warps + 1) {
        if constexpr (MODE == kM1I8) m1_digit_warp<XF32>(p, smem, s_abort, lane);
        return;
    }

    const int g = lane >> 2, t = lane & 3;
    const int box = warp / kM1Parts, part = warp % kM1Parts;   // blocks part*kM1Blocks .. +kM1Blocks-1
    const int blk0 = part * kM1Blocks;
    float acc[TP][2];
#pragma unroll
    for (int i = 0; i < TP; ++i) acc[i][0] = acc[i][1] = 0.0f;
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    // per-block word offsets inside a tile (row g; row g+8 is 1 KiB further), swizzled
    uint32_t woff[kM1Blocks];
#pragma unroll
    for (int q = 0; q < kM1Blocks; ++q) woff[q] = g * 128 + (((blk0 + q) ^ g) << 4) + 4 * t;
    bool waited = false;

    int s = 0, round = 0, chunk = 0, t0 = tile_begin;
    for (int it = 0; it < total_it; ++it) {
        // this pass: tiles nt, rows [row0, row_end)
        const int nu = min(upass, tile_begin + my_tiles - t0);
        const int nt = p.row_split ? (nu + kTileRows - 1) / kTileRows : nu;
        const int64_t row0 = p.row_split ? t0 : static_cast<int64_t>(t0) * kTileRows;
        const int64_t row_end = min(static_cast<int64_t>(p.N), row0 + (p.row_split ? nu : nu * kTileRows));
        bool ok = !*s_abort;
        if (ok && !mbar_wait_bounded(&full_bar[s], round & 1, kDevErrFullWait)) {
            *s_abort = 1;
            ok = false;
        }
        const int c0 = chunk * (kM1KC / 32) + box * 8;   // first block of this warp's box
        if constexpr (MODE == kM1I8) {
            // chunk 0: its raw activations; later chunks: their digits (each completes once
            // per launch, so later passes find them ready)
            uint64_t* xb = reinterpret_cast<uint64_t*>(smem + p.xbar_off);
            if (ok && !mbar_wait_bounded(chunk == 0 ? xb : xb + p.n_chunks + chunk, 0, kDevErrFullWait)) {
                *s_abort = 1;
                ok = false;
            }
            if (ok && c0 + blk0 < p.G)
                m1_i8_stage<TP, STMA, XF32>(p, smem, static_cast<uint32_t>(s) * p.stage_bytes, box, blk0, c0, g, t,
                                            row0, row_end, woff, chunk == 0, acc);
        } else if (ok && c0 + blk0 < p.G) {
            const uint32_t st = static_cast<uint32_t>(s) * p.stage_bytes;   // offset of the stage in smem
            // ---- block g of the box: this lane's activation fragments (zero past K)
            const bool live = c0 + g < p.G;
            const uint32_t xr = st + p.x_off + (32 * (box * 8 + g) + 4 * t) * 2;
            uint2 lo = make_uint2(0u, 0u), hi = make_uint2(0u, 0u);
            if (live) {
                lo = sh_u64(smem, xr);
                hi = sh_u64(smem, xr + 32);
            }
            uint32_t xl0, xl1, xh0, xh1;
            b_frag(lo.x, lo.y, xl0, xl1);
            b_frag(hi.x, hi.y, xh0, xh1);
            if constexpr (F16A) {   // fp16 activations; the high half pre-scaled by 1/16
                xl0 = bf16x2_to_f16x2(xl0, 1.0f);
                xl1 = bf16x2_to_f16x2(xl1, 1.0f);
                xh0 = bf16x2_to_f16x2(xh0, 0.0625f);
                xh1 = bf16x2_to_f16x2(xh1, 0.0625f);
            }
            // block-diagonal B for this warp's S steps: step j (block blk0 + j/2, half j&1)
            // is nonzero only in that block's column, i.e. on lanes whose g is that block
            uint32_t bd[S][2];
#pragma unroll
            for (int j = 0; j < S; ++j) {
                const bool mine = g == blk0 + (j >> 1);
                bd[j][0] = mine ? ((j & 1) ? xh0 : xl0) : 0u;
                bd[j][1] = mine ? ((j & 1) ? xh1 : xl1) : 0u;
                asm volatile("" : "+r"(bd[j][0]), "+r"(bd[j][1]));   // keep them in registers
            }
            // the offsets of this warp's columns (runs beside the tile chains)
            float corr[4];
            if constexpr (F16A) {
                const uint32_t c_lo[4] = {0x64086408u, 0x64086408u, 0x64086408u, 0x64086408u};   // 1032
                const uint32_t c_hi[4] = {0x64806480u, 0x64806480u, 0x64806480u, 0x64806480u};   // 1152
                mma_f16(corr, c_lo, bd[0][0], bd[0][1], zero4);
                mma_f16(corr, c_hi, bd[1][0], bd[1][1], corr);
#pragma unroll
                for (int j = 2; j < S; j += 2) {
                    mma_f16(corr, c_lo, bd[j][0], bd[j][1], corr);
                    mma_f16(corr, c_hi, bd[j + 1][0], bd[j + 1][1], corr);
                }
            } else {
                const uint32_t c136[4] = {0x43084308u, 0x43084308u, 0x43084308u, 0x43084308u};   // 136
                mma_bf16(corr, c136, bd[0][0], bd[0][1], zero4);
#pragma unroll
                for (int j = 1; j < S; ++j) mma_bf16(corr, c136, bd[j][0], bd[j][1], corr);
            }
            const uint32_t wbox = st + box * p.w_box_bytes;
#pragma unroll
            for (int i = 0; i < TP; ++i) {
                float d[4];
#pragma unroll
                for (int q = 0; q < kM1Blocks; ++q) {
                    const uint32_t wt = wbox + i * (kTileRows * 128) + woff[q];
                    const uint32_t w0 = sh_u32(smem, wt);
                    const uint32_t w8 = sh_u32(smem, wt + 1024);
                    uint32_t alo[4], ahi[4];
                    if constexpr (F16A) {
                        const uint32_t v0 = w0 >> 8, v8 = w8 >> 8;
                        alo[0] = f16_lo(w0);
                        alo[1] = f16_lo(w8);
                        alo[2] = f16_lo(v0);
                        alo[3] = f16_lo(v8);
                        ahi[0] = f16_hi(w0);
                        ahi[1] = f16_hi(w8);
                        ahi[2] = f16_hi(v0);
                        ahi[3] = f16_hi(v8);
                        if (q == 0) mma_f16(d, alo, bd[0][0], bd[0][1], zero4);
                        else mma_f16(d, alo, bd[2 * q][0], bd[2 * q][1], d);
                        mma_f16(d, ahi, bd[2 * q + 1][0], bd[2 * q + 1][1], d);
                    } else {
                        alo[0] = lop3_magic(w0);
                        alo[1] = lop3_magic(w8);
                        alo[2] = lop3_magic(w0 >> 8);
                        alo[3] = lop3_magic(w8 >> 8);
                        ahi[0] = lop3_magic(w0 >> 4);
                        ahi[1] = lop3_magic(w8 >> 4);
                        ahi[2] = lop3_magic(w0 >> 12);
                        ahi[3] = lop3_magic(w8 >> 12);
                        if (q == 0) mma_bf16(d, alo, bd[0][0], bd[0][1], zero4);
                        else mma_bf16(d, alo, bd[2 * q][0], bd[2 * q][1], d);
                        mma_bf16(d, ahi, bd[2 * q + 1][0], bd[2 * q + 1][1], d);
                    }
                }
                // scales of blocks 2t and 2t+1 of the box for rows g and g+8 (the columns of
                // the box's other warps hold zeros on this warp)
                float2 sg, sg8;
                if constexpr (STMA) {
                    const uint32_t sa = st + p.s_off + (i * kTileRows + g) * p.s_pitch + (box * 8 + 2 * t) * 2;
                    sg = half2_bits_to_float2(sh_u32(smem, sa));
                    sg8 = half2_bits_to_float2(sh_u32(smem, sa + 8 * p.s_pitch));
                } else {
                    const int64_t r0 = row0 + i * kTileRows + g;
                    const int ca = c0 + 2 * t, cc = ca + 1;
                    const bool v0 = r0 < row_end, v8 = r0 + 8 < row_end;
                    sg.x = (v0 && ca < p.G) ? __half2float(p.scales[r0 * p.G + ca]) : 0.0f;
                    sg.y = (v0 && cc < p.G) ? __half2float(p.scales[r0 * p.G + cc]) : 0.0f;
                    sg8.x = (v8 && ca < p.G) ? __half2float(p.scales[(r0 + 8) * p.G + ca]) : 0.0f;
                    sg8.y = (v8 && cc < p.G) ? __half2float(p.scales[(r0 + 8) * p.G + cc]) : 0.0f;
                }
                acc[i][0] = fmaf(sg.x, d[0] - corr[0], acc[i][0]);
                acc[i][0] = fmaf(sg.y, d[1] - corr[1], acc[i][0]);
                acc[i][1] = fmaf(sg8.x, d[2] - corr[2], acc[i][1]);
                acc[i][1] = fmaf(sg8.y, d[3] - corr[3], acc[i][1]);
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
                const int64_t n = row0 + e;
                if (n < row_end) {
                    const int64_t oi = p.out_col0 + n;
                    if (p.out_bf16) reinterpret_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(sum);
                    else reinterpret_cast<float*>(p.out)[oi] = sum;
                    if (p.pg.world > 1) store_to_peers(p.pg, oi, sum);
                }
            }
            named_barrier(1, kM1Warps * 32);
        }
        if (++chunk == p.n_chunks) { chunk = 0; t0 += upass; }
    }
    gemv_gather_end(p.pg, kM1Warps * 32);
}

bool pdl_enabled() {
    static const int on = [] {
        const char* e = getenv("BYBY_CUDA_PDL");
        return (e && e[0] == '0') ? 0 : 1;
    }();
    return on != 0;
}

template <int TP, int NT, bool XF32, bool STMA, int W>
int launch_t(const GemvMaps& maps, const GemvParams& p, int grid, size_t smem, cudaStream_t stream) {
    auto kern = gemv_q4b32_kernel<TP, NT, XF32, STMA, W>;
    static std::atomic<uint64_t> configured{0};   // per device: the opt-in smem limit is a function attribute
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(BYBYCU_ERR_ARGS, "device %d out of range", dev);
    if (!(configured.load(std::memory_order_acquire) >> dev & 1)) {
        BYBYCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448));
        configured.fetch_or(uint64_t(1) << dev, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3((W + 1) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    BYBYCU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, maps, p));
    BYBYCU_LAUNCH_CHECK("gemv_q4b32_kernel");
    return BYBYCU_OK;
}

// The operand mode of the M = 1 kernel: s8 MMAs on the raw nibbles (default), or, through
// BYBY_CUDA_GEMV_M1=f16 / bf16, the dequantising fp16 / bf16 forms kept for comparison.
int m1_mode() {
    static const int mode = [] {
        const char* e = getenv("BYBY_CUDA_GEMV_M1");
        if (e && !strcmp(e, "f16")) return kM1F16;
        if (e && !strcmp(e, "bf16")) return kM1Bf16;
        return kM1I8;
    }();
    return mode;
}

template <int TP, bool STMA>
int launch_m1(int mode, bool xf32, const GemvMaps& maps, const GemvParams& p, int grid, size_t smem,
              cudaStream_t stream) {
    auto kern = mode == kM1I8 ? (xf32 ? gemv_m1_kernel<TP, STMA, kM1I8, true> : gemv_m1_kernel<TP, STMA, kM1I8>)
              : mode == kM1F16 ? gemv_m1_kernel<TP, STMA, kM1F16> : gemv_m1_kernel<TP, STMA, kM1Bf16>;
    static std::atomic<uint64_t> configured[4];   // per operand form, per device (zero-initialised)
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(BYBYCU_ERR_ARGS, "device %d out of range", dev);
    const int fi = xf32 ? 3 : mode;
    if (!(configured[fi].load(std::memory_order_acquire) >> dev & 1)) {
        BYBYCU_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448));
        configured[fi].fetch_or(uint64_t(1) << dev, std::memory_order_release);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kM1Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    BYBYCU_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, maps, p));
    BYBYCU_LAUNCH_CHECK("gemv_m1_kernel");
    return BYBYCU_OK;
}

template <int TP, int NT, int W>
int dispatch_xw(bool xf32, const GemvMaps& m, const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
    if (p.scale_tma)
        return xf32 ? launch_t<TP, NT, true, true, W>(m, p, grid, smem, st)
                    : launch_t<TP, NT, false, true, W>(m, p, grid, smem, st);
    return xf32 ? launch_t<TP, NT, true, false, W>(m, p, grid, smem, st)
                : launch_t<TP, NT, false, false, W>(m, p, grid, smem, st);
}
template <int TP, int NT>
int dispatch_x(bool xf32, bool one_pass, const GemvMaps& m, const GemvParams& p, int grid, size_t smem,
               cudaStream_t st) {
    return one_pass ? dispatch_xw<TP, NT, kWarpsOnePass>(xf32, m, p, grid, smem, st)
                    : dispatch_xw<TP, NT, kWarpsMany>(xf32, m, p, grid, smem, st);
}

size_t round1k(size_t v) { return (v + 1023) / 1024 * 1024; }

}  // namespace

bool gemv_supports(const GemmArgs& a) {
    if (a.fmt == BYBYCU_FMT_F16) return f16_gemv_supports(a);   // f16gemv.cu
    if (a.fmt != BYBYCU_FMT_Q4B32) return false;
    if (a.M < 1 || a.M > kGemvMaxRows || a.K % 32 != 0 || a.N < 1) return false;
    if (a.x_dtype != BYBYCU_DT_BF16 && a.x_dtype != BYBYCU_DT_F32) return false;
    // TMA needs 16-byte aligned global bases; scales need 2-byte alignment.
    if ((reinterpret_cast<uintptr_t>(a.packed) & 15u) || (reinterpret_cast<uintptr_t>(a.x) & 15u)) return false;
    if (a.scale_base & 1) return false;
    return true;
}

// The tensor maps of one weight slot and tiling.  Encoding six maps costs microseconds per
// call, a large share of a decode step's host time, so encoded sets are kept per device in a
// small direct-mapped cache keyed by everything the maps depend on (a map holds only the
// address, the shape and the box; the same key always encodes the same maps).
int gemv_maps(const GemmArgs& a, const int (&box_rows)[3], int kc, bool scale_tma, uint32_t s_pitch, GemvMaps* maps) {
    struct Entry {
        const void* packed = nullptr;
        int64_t scale_base = 0;
        int K = 0, N = 0, rows[3] = {0, 0, 0}, kc = 0, device = -1;
        bool scale_tma = false;
        GemvMaps maps;
    };
    const int tp = box_rows[0] * 131 + box_rows[1] * 7 + box_rows[2];   // the box heights, hashed
    constexpr int kEntries = 64;
    static Entry cache[kEntries];
    static std::mutex mu;
    int device = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&device));
    const uint64_t key = reinterpret_cast<uintptr_t>(a.packed) ^ (static_cast<uint64_t>(a.N) << 20) ^
                         (static_cast<uint64_t>(a.K) << 40) ^ static_cast<uint64_t>(tp * 131 + kc + device * 7919);
    const int slot = static_cast<int>((key ^ (key >> 17) ^ (key >> 33)) % kEntries);
    {
        std::lock_guard<std::mutex> lock(mu);
        const Entry& e = cache[slot];
        if (e.packed == a.packed && e.scale_base == a.scale_base && e.K == a.K && e.N == a.N &&
            e.rows[0] == box_rows[0] && e.rows[1] == box_rows[1] && e.rows[2] == box_rows[2] && e.kc == kc &&
            e.device == device && e.scale_tma == scale_tma) {
            *maps = e.maps;
            return BYBYCU_OK;
        }
    }
    const uint8_t* scale_ptr = a.packed + a.scale_base;
    const int G = a.K / 32;
    for (int i = 0; i < 3; ++i) {
        if (int rc = encode_tensor_map_2d(&maps->w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, a.packed, a.K / 2, a.N, a.K / 2,
                                          128, box_rows[i], CU_TENSOR_MAP_SWIZZLE_128B,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return rc;
        if (scale_tma) {
            if (int rc = encode_tensor_map_2d(&maps->s[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, scale_ptr, G, a.N,
                                              static_cast<uint64_t>(G) * 2, kc / 32, box_rows[i],
                                              s_pitch == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
                return rc;
        } else {
            maps->s[i] = maps->w[i];   // unused
        }
    }
    std::lock_guard<std::mutex> lock(mu);
    Entry& e = cache[slot];
    e.packed = a.packed;
    e.scale_base = a.scale_base;
    e.K = a.K;
    e.N = a.N;
    for (int i = 0; i < 3; ++i) e.rows[i] = box_rows[i];
    e.kc = kc;
    e.device = device;
    e.scale_tma = scale_tma;
    e.maps = *maps;
    return BYBYCU_OK;
}

int launch_gemv(const GemmArgs& a, const PeerGather* pg) {
    if (a.fmt == BYBYCU_FMT_F16) {
        if (pg) return set_error(BYBYCU_ERR_ARGS, "the format-1 GEMV does not store to peers");
        return launch_f16_gemv(a);
    }
    if (a.M > 16) {
        // 17..32 rows: one launch per 16 rows (each streams the weights once more); this keeps
        // fp32 activation rows exact in two bf16 terms where the tensor-core route would round
        // them to fp16
        if (pg) return set_error(BYBYCU_ERR_ARGS, "the GEMV stores to peers for at most 16 rows");
        const size_t xe = a.x_dtype == BYBYCU_DT_F32 ? 4 : 2, oe = a.out_dtype == BYBYCU_DT_BF16 ? 2 : 4;
        for (int m0 = 0; m0 < a.M; m0 += 16) {
            GemmArgs b = a;
            b.M = std::min(16, a.M - m0);
            b.x = static_cast<const uint8_t*>(a.x) + static_cast<size_t>(m0) * a.K * xe;
            b.out = static_cast<uint8_t*>(a.out) + static_cast<size_t>(m0) * a.out_ld * oe;
            if (int rc = launch_gemv(b, nullptr)) return rc;
        }
        return BYBYCU_OK;
    }
    DeviceInfo dev;
    if (int rc = current_device_info(&dev)) return rc;
    const bool xf32 = a.x_dtype == BYBYCU_DT_F32;
    const int ntn = a.M > 8 ? 2 : 1;
    const int xe = xf32 ? 4 : 2;
    const int n_tiles = static_cast<int>(ceil_div(a.N, kTileRows));
    const int grid = std::min(n_tiles, dev.sm_count);
    // The M = 1 kernel takes bf16 rows in every operand mode and fp32 rows in the integer mode
    // (two fixed-point images, 2^-29 of each block's largest value).  The fp16 / bf16 modes
    // have no fp32 form: there fp32 rows take the general kernel's two bf16 terms.
    const int want_mode = a.variant >= kM1Bf16 && a.variant <= kM1I8 ? a.variant : m1_mode();
    const int mode = want_mode == kM1I8 && a.K > 32768 ? kM1F16 : want_mode;
    const bool m1 = a.M == 1 && (!xf32 || mode == kM1I8);
    // M = 1 splits rows, not tiles: 11008 rows over 148 CTAs is 74 or 75 rows each instead of 4
    // or 5 tiles (64 or 80 rows), so no CTA streams 6% more than its share and all end together
    const int rows_base = a.N / grid, rows_extra = a.N % grid;
    const int tiles_max = m1 ? static_cast<int>(ceil_div(rows_base + (rows_extra ? 1 : 0), kTileRows))
                             : static_cast<int>(ceil_div(n_tiles, grid));
    const uint8_t* scale_ptr = a.packed + a.scale_base;
    const int G = a.K / 32;
    const bool scale_tma = (G % 8 == 0) && ((reinterpret_cast<uintptr_t>(scale_ptr) & 15u) == 0);
    const size_t budget = static_cast<size_t>(dev.max_smem_optin) - 1024 - 64;

    // The integer mode keeps the whole activation row resident (converted in place into
    // digits, plus a factor per block and two barriers per 1024-value chunk) instead of a
    // slice per stage; rows longer than 32768 values take the fp16 mode.
    const bool x_whole = m1 && mode == kM1I8;
    const int n_xchunks = static_cast<int>(ceil_div(a.K, kM1KC));
    const size_t x_all = x_whole ? static_cast<size_t>(n_xchunks) * 16 +
                                       (static_cast<size_t>(a.K) * xe + static_cast<size_t>(G) * 4 + 15) / 16 * 16
                                 : 0;
    // K chunk: 512 values (fine pipelining: compute starts after the first 1/(K/512) of the
    // data) with boxes spanning all rows of the pass; larger chunks only when M is large.
    int kc = 0, tp = 0, tpl = 0, stages = 0;
    size_t stage_bytes = 0, red_bytes = 0;
    uint32_t s_pitch = 0, w_box = 0, s_off = 0, x_off = 0;
    int x_pitch = 0;
    // at least four stages in flight where they fit (two for the M = 1 kernel), else two:
    // 16 fp32 rows beside 80-row tiles leave room for three (M = 16, N = 11008)
    for (int need_st : {m1 ? 2 : 4, 2}) {
        if (kc) break;
        for (int kc_try : {512, 1024, 2048}) {
            if (m1 && kc_try != kM1KC) continue;   // the M = 1 kernel: one 256-value box per warp
            // M = 1: passes of 5 or 7 tiles, whichever needs fewer passes over a CTA's rows (each
            // pass is a whole sweep of K and ends in a cross-warp reduction); 5 on a tie, whose
            // smaller stages let two CTAs share an SM when one pass does
            const int tp_m1 = ceil_div(tiles_max, 7) < ceil_div(tiles_max, 5) ? 7 : 5;
            const int tp_try = std::min(tiles_max, m1 ? tp_m1 : ntn == 2 ? 5 : 8);
            const int tpl_try = tp_try <= 2 ? 2 : tp_try <= 5 ? 5 : (m1 ? 7 : 8);
            const uint32_t rows = 16 * tpl_try;
            const uint32_t sp = static_cast<uint32_t>(kc_try / 32 * 2);
            const uint32_t wb = rows * 128;
            const uint32_t so = (kc_try / 256) * wb;
            const uint32_t xo = static_cast<uint32_t>(so + round1k(scale_tma ? rows * sp : 0));
            const int xp = kc_try * xe + 32;
            const size_t sb = round1k(xo + (x_whole ? 0 : static_cast<size_t>(a.M) * xp));
            const size_t rb = m1 ? static_cast<size_t>(kM1Warps) * tpl_try * 16 * sizeof(float)
                                 : static_cast<size_t>(kRedSlots) * tpl_try * ntn * 128 * sizeof(float);
            const int nch = static_cast<int>(ceil_div(a.K, kc_try));
            const int want = static_cast<int>(ceil_div(tiles_max, tp_try)) * nch;
            if (budget < rb + x_all + sb + 16) continue;
            const int st = static_cast<int>((budget - rb - x_all) / (sb + 16));
            if (st >= std::min(need_st, want) && st >= 1) {
                kc = kc_try; tp = tp_try; tpl = tpl_try; stages = std::min(st, want);
                stage_bytes = sb; red_bytes = rb; s_pitch = sp; w_box = wb; s_off = so; x_off = xo; x_pitch = xp;
                break;
            }
        }
    }
    if (!kc) return set_error(BYBYCU_ERR_SHAPE, "GEMV: shared memory too small for M=%d", a.M);
    // Ring depth of the M = 1 kernel.  One pass per CTA: as many stages as leave room for two
    // CTAs per SM (at least two), so that the next launch's CTA streams its first stages - all
    // of them when they fit - while this one computes (C2, 75 rows a CTA: two stages, 6.4 us
    // against 7.1 with three and one CTA per SM; 28 rows a CTA at N = 4096: four).  Several
    // passes: three stages and one CTA per SM, whose deeper ring keeps the long stream in
    // flight (1 x 32000 x 4096: 16.1 us against 17.9).
    // A tuned plan's depth (a.stages), then BYBY_CUDA_GEMV_STAGES, override.
    const int fit = stages;   // the most that fit in shared memory (and are useful)
    const size_t half_sm = static_cast<size_t>(dev.smem_per_sm) / 2 - 1024;   // per CTA, two per SM
    const size_t fixed = 1024 + 16 + red_bytes + x_all;
    const int two_cta = half_sm > fixed ? static_cast<int>((half_sm - fixed) / (stage_bytes + 16)) : 0;
    if (m1) stages = std::min(fit, tiles_max > tp ? 3 : std::max(2, two_cta));
    // M >= 2, one pass per CTA: the 8-warp kernel, two CTAs per SM (as many stages as fit)
    const bool one_pass = !m1 && tiles_max <= tp;
    if (one_pass) stages = std::min(fit, std::max(2, two_cta));
    if (a.stages >= 1) stages = std::min(fit, a.stages);
    if (const char* e = getenv("BYBY_CUDA_GEMV_STAGES")) {
        const int want_stages = atoi(e);
        if (want_stages >= 1) stages = std::min(fit, want_stages);
    }

    GemvParams p{};
    p.M = a.M; p.K = a.K; p.N = a.N; p.G = G;
    p.tiles_base = m1 ? rows_base : n_tiles / grid;
    p.tiles_extra = m1 ? rows_extra : n_tiles % grid;
    p.row_split = m1 ? 1 : 0;
    p.rem_rows = rows_base % (tp * kTileRows);
    p.kc = kc;
    p.n_chunks = static_cast<int>(ceil_div(a.K, kc));
    p.stages = stages;
    p.tp = tp;
    p.scale_tma = scale_tma;
    p.x_pitch = x_pitch;
    p.stage_bytes = static_cast<uint32_t>(stage_bytes);
    p.w_box_bytes = w_box;
    p.s_off = s_off;
    p.x_off = x_off;
    p.s_pitch = s_pitch;
    p.scales = reinterpret_cast<const __half*>(scale_ptr);
    p.x = static_cast<const uint8_t*>(a.x);
    p.x_elem = xe;
    p.out = a.out;
    p.out_bf16 = a.out_dtype == BYBYCU_DT_BF16;
    p.out_ld = a.out_ld;
    p.out_col0 = a.out_col0;
    if (pg) {
        if (p.out_bf16) return set_error(BYBYCU_ERR_ARGS, "GEMV all-gather: the gathered output is fp32");
        p.pg = *pg;
    }
    const size_t smem = 1024 + static_cast<size_t>(stages) * (stage_bytes + 16) + 16 + red_bytes + x_all;
    p.x_whole = x_whole ? 1 : 0;
    p.xbar_off = static_cast<uint32_t>(static_cast<size_t>(stages) * (stage_bytes + 16) + 16 + red_bytes);
    p.x_all_off = p.xbar_off + static_cast<uint32_t>(n_xchunks) * 16;

    GemvMaps maps;
    int box_rows[3] = {kTileRows * tp, kTileRows * std::max(1, tp - 1), kTileRows};
    if (m1) {   // a full pass, and the short last passes of the two CTA sizes (unused slots: full)
        const int full = kTileRows * tp;
        const int ra = rows_base % full, rb = (rows_base + 1) % full;
        box_rows[1] = ra ? ra : full;
        box_rows[2] = rb ? rb : full;
    }
    if (int rc = gemv_maps(a, box_rows, kc, scale_tma, s_pitch, &maps)) return rc;
    const cudaStream_t st = a.stream;
    if (m1) {
        if (scale_tma)
            return tpl == 2 ? launch_m1<2, true>(mode, xf32, maps, p, grid, smem, st)
                 : tpl == 5 ? launch_m1<5, true>(mode, xf32, maps, p, grid, smem, st)
                            : launch_m1<7, true>(mode, xf32, maps, p, grid, smem, st);
        return tpl == 2 ? launch_m1<2, false>(mode, xf32, maps, p, grid, smem, st)
             : tpl == 5 ? launch_m1<5, false>(mode, xf32, maps, p, grid, smem, st)
                        : launch_m1<7, false>(mode, xf32, maps, p, grid, smem, st);
    }
    if (ntn == 2) {
        return tpl == 2 ? dispatch_x<2, 2>(xf32, one_pass, maps, p, grid, smem, st)
                        : dispatch_x<5, 2>(xf32, one_pass, maps, p, grid, smem, st);
    }
    switch (tpl) {
        case 2: return dispatch_x<2, 1>(xf32, one_pass, maps, p, grid, smem, st);
        case 5: return dispatch_x<5, 1>(xf32, one_pass, maps, p, grid, smem, st);
        default: return dispatch_x<8, 1>(xf32, one_pass, maps, p, grid, smem, st);
    }
}

}  // namespace bybycu
