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
//     filling the MMA's eight columns; the remainder R = x * 2^(140 - E) - X (exact, |R| <= 1/2)
//     becomes a second image X2 = rint(R * 2^15) in the same form, fed to a second chain of
//     MMAs on the same A registers, so x is carried to 2^-29 of its block's largest value
//     (one image, 15 bits, left fp32 rows outside 1e-3 per element near zero outputs);
//   * per row and block the epilogue adds s * 2^(E-140) * ((sum u X - z * sum X) + 2^-15 *
//     (sum u X2 - z * sum X2)): the zero point enters through the block's sums of X and X2 (the
//     s (dot(a, u) - z sum(a)) factorisation of the reference's GPU kernels).
// Everything else (any M, any group size, odd K, unaligned slots) runs q4a_exact_kernel: one
// thread per output, fmaf(x, (u - z) * s, sum) in k order (the CPU VM's OP_Q4_GEMV arithmetic).
//
// The same decode kernel is the fused decode GEMV (sessionMatmulQ4Fused, gpubackend.nim:3185-3231,
// its shader q4_autotune.nim:194-325): in one launch, mode 0 lets 1-3 matrices share x (the SMs
// are split between them in proportion to their rows) and mode 1 computes silu(gate) * up (each
// CTA streams its gate rows in one pass and the same up rows in the next, keeping the gate sums
// in shared memory).  Optionally x is RMS-normalised first (x * gamma is what gets quantised;
// every CTA sums the raw squares during its first sweep over K and scales its results by
// 1 / sqrt(mean + eps)), and a residual is added to every output row.
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

constexpr int kQ4aMaxMats = 3;

// Per matrix: nibbles, fp32 scales, fp32 zero points; boxes of tp, tp - 1 and 1 tiles.  A launch
// carries room for MATS matrices only: one-matrix calls keep the kernel parameters at 1.1 KB.
template <int MATS>
struct Q4aMaps {
    CUtensorMap w[MATS][3], s[MATS][3], z[MATS][3];
};

struct Q4aParams {
    int K, G, n_chunks, stages, tp;
    uint32_t stage_bytes, w_box_bytes, s_off, z_off, x_off, g_off;   // the stage layout
    const float* x;
    const float* gamma;   // RMSNorm weight (has_norm)
    const float* res;     // residual added to every output row (has_res)
    float* out[kQ4aMaxMats];
    int N[kQ4aMaxMats];
    int mode;             // 0: each matrix its own output; 1: out[0] = silu(gate) * up
    int n_mats, has_norm, has_res;
    float eps;
    // work split: mode 0, CTAs [cta0[m], cta0[m+1]) take matrix m's row tiles; mode 1, every CTA
    // takes the same row tiles of both matrices, gate in even passes and up in odd ones
    int cta0[kQ4aMaxMats + 1];
    int tiles_base[kQ4aMaxMats], tiles_extra[kQ4aMaxMats];
};

// The work of one CTA: its matrix segment, its first tile and tile count, and per pass the
// matrix and first tile.
struct Q4aWork {
    int seg, tile_begin, my_tiles, groups, passes;
    __device__ Q4aWork(const Q4aParams& p, int b) {
        seg = 0;
        if (p.mode == 0)
            while (seg + 1 < p.n_mats && b >= p.cta0[seg + 1]) ++seg;
        const int l = b - p.cta0[seg];
        my_tiles = p.tiles_base[seg] + (l < p.tiles_extra[seg] ? 1 : 0);
        tile_begin = l * p.tiles_base[seg] + min(l, p.tiles_extra[seg]);
        groups = (my_tiles + p.tp - 1) / p.tp;
        passes = p.mode == 1 ? 2 * groups : groups;
    }
    __device__ int mat(const Q4aParams& p, int pass) const { return p.mode == 1 ? (pass & 1) : seg; }
    __device__ int t0(const Q4aParams& p, int pass) const {
        return tile_begin + (p.mode == 1 ? pass >> 1 : pass) * p.tp;
    }
    __device__ int nt(const Q4aParams& p, int pass) const { return min(p.tp, tile_begin + my_tiles - t0(p, pass)); }
};

// The producer (lane 0 of warp kM1Warps): every (pass, chunk) iteration's nibble, scale and
// zero-point boxes into the stage ring, the activations (and gamma) after griddepcontrol.wait.
template <int MATS>
__device__ __forceinline__ void q4a_producer(const Q4aMaps<MATS>& maps, const Q4aParams& p, const Q4aWork& w, uint8_t* smem,
                                             uint64_t* full_bar, uint64_t* empty_bar, volatile int* s_abort,
                                             int total_it) {
    for (int m = 0; m < MATS && m < p.n_mats; ++m)
        for (int i = 0; i < 3; ++i) {
            prefetch_tensormap(&maps.w[m][i]);
            prefetch_tensormap(&maps.s[m][i]);
            prefetch_tensormap(&maps.z[m][i]);
        }
    const uint64_t policy = l2_policy_evict_first();
    auto issue_weights = [&](int s, int it) {
        const int pass = it / p.n_chunks, chunk = it % p.n_chunks;
        const int m = min(w.mat(p, pass), MATS - 1), t0 = w.t0(p, pass), nt = w.nt(p, pass);
        const int k0 = chunk * kM1KC, kn = min(kM1KC, p.K - k0);
        const uint32_t rows = nt * kTileRows;
        const uint32_t bytes =
            4 * rows * 128 + 2 * rows * 128 + static_cast<uint32_t>(kn) * 4 * (p.has_norm ? 2 : 1);
        uint8_t* st = smem + static_cast<size_t>(s) * p.stage_bytes;
        mbar_arrive_expect_tx(&full_bar[s], bytes);
        const int mi = nt == p.tp ? 0 : (nt == p.tp - 1 ? 1 : 2);   // box of nt, nt - 1 or 1 tile(s)
        const int pieces = mi == 2 ? nt : 1;
        for (int q = 0; q < pieces; ++q) {
            const int row = (t0 + q) * kTileRows;
            const uint32_t roff = q * kTileRows * 128;
            for (int bx = 0; bx < 4; ++bx)
                tma_load_2d_hint(st + bx * p.w_box_bytes + roff, &maps.w[m][mi], &full_bar[s], k0 / 2 + bx * 128, row,
                                 policy);
            tma_load_2d(st + p.s_off + roff, &maps.s[m][mi], &full_bar[s], k0 / 32, row);
            tma_load_2d(st + p.z_off + roff, &maps.z[m][mi], &full_bar[s], k0 / 32, row);
        }
    };
    auto issue_x = [&](int s, int it) {
        const int chunk = it % p.n_chunks;
        const int k0 = chunk * kM1KC, kn = min(kM1KC, p.K - k0);
        uint8_t* st = smem + static_cast<size_t>(s) * p.stage_bytes;
        bulk_load_1d(st + p.x_off, p.x + k0, static_cast<uint32_t>(kn) * 4, &full_bar[s]);
        if (p.has_norm) bulk_load_1d(st + p.g_off, p.gamma + k0, static_cast<uint32_t>(kn) * 4, &full_bar[s]);
    };
    const int first = min(p.stages, total_it);
    for (int it = 0; it < first; ++it) issue_weights(it, it);   // the weights do not depend on the previous kernel
    pdl_wait();
    for (int it = 0; it < first; ++it) issue_x(it, it);
    int issued = first;
    int s = first % p.stages, round = first / p.stages;
    for (int it = first; it < total_it; ++it) {
        if (*s_abort) break;
        if (!mbar_wait_bounded(&empty_bar[s], (round - 1) & 1, kDevErrEmptyWait)) {
            *s_abort = 1;
            break;
        }
        issue_weights(s, it);
        issue_x(s, it);
        issued = it + 1;
        if (++s == p.stages) { s = 0; ++round; }
    }
    // every copy must land before the CTA may exit
    for (int it = max(0, issued - p.stages); it < issued; ++it)
        if (!mbar_wait_bounded(&full_bar[it % p.stages], (it / p.stages) & 1, kDevErrDrainWait)) break;
}

template <int TP, int MATS>
__global__ void __launch_bounds__(kM1Threads, 1) q4a_kernel(const __grid_constant__ Q4aMaps<MATS> maps,
                                                            const Q4aParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(p.stages) * p.stage_bytes);
    uint64_t* empty_bar = full_bar + p.stages;
    volatile int* s_abort = reinterpret_cast<volatile int*>(empty_bar + p.stages);
    const uint32_t red = smem_u32(empty_bar + p.stages + 2);   // [kM1Warps][TP][16] floats
    float* sq_part = reinterpret_cast<float*>(smem + (red - base) + kM1Warps * TP * 16 * 4);   // [kM1Warps]
    float* gate_buf = sq_part + kM1Warps;                                                      // [TP * 16]

    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Q4aWork work(p, blockIdx.x);
    const int total_it = work.passes * p.n_chunks;

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
        if (lane == 0) q4a_producer(maps, p, work, smem, full_bar, empty_bar, s_abort, total_it);
        return;
    }
    if (warp > kM1Warps) return;   // the block shape of the Q4B32 decode kernel

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
    float sq = 0.0f;      // sum of the raw activations' squares (RMSNorm), first sweep over K
    float inv = 1.0f;     // 1 / rms after the first pass (1 without RMSNorm)
    bool waited = false;

    int s = 0, round = 0;
    for (int it = 0; it < total_it; ++it) {
        const int pass = it / p.n_chunks, chunk = it % p.n_chunks;
        bool ok = !*s_abort;
        if (ok && !mbar_wait_bounded(&full_bar[s], round & 1, kDevErrFullWait)) {
            *s_abort = 1;
            ok = false;
        }
        const int c0 = chunk * (kM1KC / 32) + box * 8;   // this warp's box: blocks c0 .. c0 + 7 of K
        if (ok && c0 + blk0 < p.G) {
            const uint32_t st = static_cast<uint32_t>(s) * p.stage_bytes;
            // ---- activations: lane (g, t) takes x[8t .. 8t+7] of block q (times gamma)
            const bool live = c0 + blk0 + q < p.G;
            const uint32_t xo = ((box * 8 + blk0 + q) * 32 + 8 * t) * 4;
            uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
            if (live) {
                xa = lds_u128(base + st + p.x_off + xo);
                xb = lds_u128(base + st + p.x_off + xo + 16);
            }
            uint32_t xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            if (p.has_norm) {
                uint4 ga = make_uint4(0u, 0u, 0u, 0u), gb = ga;
                if (live) {
                    ga = lds_u128(base + st + p.g_off + xo);
                    gb = lds_u128(base + st + p.g_off + xo + 16);
                }
                const uint32_t gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float r = __uint_as_float(xv[i]);
                    if (pass == 0 && !(g & 1)) sq = fmaf(r, r, sq);   // each element once: even-g lanes
                    xv[i] = __float_as_uint(r * __uint_as_float(gv[i]));
                }
            }
            uint32_t mx = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) mx = max(mx, xv[i] & 0x7FFFFFFFu);   // inf / NaN sort highest
            mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const int e = static_cast<int>(mx >> 23);
            if (live && e == 255 && t == 0 && !(g & 1)) record_device_error(kDevErrActRange);
            const int ec = max(e, 14);                               // normal factors 2^(ec - 140)
            const float up = __int_as_float((267 - ec) << 23);       // 2^(140 - ec)
            uint32_t r[8], r2[8];
            int sx = 0, sx2 = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float f = __uint_as_float(xv[i]);
                r[i] = __float_as_uint(fmaf(f, up, magic));   // bits + X
                sx += static_cast<int>(r[i]) - x_off_bits;
                const float rem = fmaf(f, up, -(__uint_as_float(r[i]) - magic));   // R, exact
                r2[i] = __float_as_uint(fmaf(rem, 32768.0f, magic));              // bits + X2
                sx2 += static_cast<int>(r2[i]) - x_off_bits;
            }
            const uint32_t b0 = prmt(prmt(r[0], r[2], sel), prmt(r[4], r[6], sel), 0x5410);   // k = 8t + 2i
            const uint32_t b1 = prmt(prmt(r[1], r[3], sel), prmt(r[5], r[7], sel), 0x5410);   // k = 8t + 2i + 1
            const uint32_t c0r = prmt(prmt(r2[0], r2[2], sel), prmt(r2[4], r2[6], sel), 0x5410);
            const uint32_t c1r = prmt(prmt(r2[1], r2[3], sel), prmt(r2[5], r2[7], sel), 0x5410);
            sx += __shfl_xor_sync(0xffffffffu, sx, 1);
            sx += __shfl_xor_sync(0xffffffffu, sx, 2);   // sum of X over block q
            sx2 += __shfl_xor_sync(0xffffffffu, sx2, 1);
            sx2 += __shfl_xor_sync(0xffffffffu, sx2, 2);   // sum of X2 over block q
            uint32_t bq[4][2], bq2[4][2];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                bq[j][0] = q == j ? b0 : 0u;
                bq[j][1] = q == j ? b1 : 0u;
                bq2[j][0] = q == j ? c0r : 0u;
                bq2[j][1] = q == j ? c1r : 0u;
                asm volatile("" : "+r"(bq[j][0]), "+r"(bq[j][1]), "+r"(bq2[j][0]), "+r"(bq2[j][1]));   // keep them in registers
            }
            // lane (g, t) combines block t (built by lane 8t): its factor and its sums of X, X2
            const int et = __shfl_sync(0xffffffffu, ec, 8 * t);
            const float ft = __int_as_float((et - 13) << 23);   // 2^(et - 140)
            const float sxt = static_cast<float>(__shfl_sync(0xffffffffu, sx, 8 * t));
            const float sxt2 = static_cast<float>(__shfl_sync(0xffffffffu, sx2, 8 * t));
            const uint32_t wbox = st + box * p.w_box_bytes;
            // ---- weights: four s8 MMAs per tile and image fill the eight columns
#pragma unroll
            for (int i = 0; i < TP; ++i) {
                int d[4] = {0, 0, 0, 0}, d2[4] = {0, 0, 0, 0};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t wt = wbox + i * (kTileRows * 128) + woff[j];
                    const uint32_t w0 = sh_u32(smem, wt);
                    const uint32_t w8 = sh_u32(smem, wt + 1024);
                    const uint32_t a[4] = {w0 & 0x0F0F0F0Fu, w8 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu,
                                           (w8 >> 4) & 0x0F0F0F0Fu};
                    mma_s8(d, a, bq[j][0], bq[j][1]);
                    mma_s8(d2, a, bq2[j][0], bq2[j][1]);
                }
                // sum u X and sum u X2 are below 2^23 in magnitude: exact as floats
                const float v0 = static_cast<float>(d[0] + d[1] * 256), v8 = static_cast<float>(d[2] + d[3] * 256);
                const float u0 = static_cast<float>(d2[0] + d2[1] * 256), u8 = static_cast<float>(d2[2] + d2[3] * 256);
                // scale and zero point of block t for rows g and g + 8 (128-byte swizzled boxes)
                const int cb = box * 8 + blk0 + t;   // block inside the chunk: 16-byte column cb / 4
                const uint32_t r0 = i * kTileRows + g, r8 = r0 + 8;
                const uint32_t o0 = r0 * 128 + ((((cb >> 2) ^ (r0 & 7)) << 4) | ((cb & 3) << 2));
                const uint32_t o8 = r8 * 128 + ((((cb >> 2) ^ (r8 & 7)) << 4) | ((cb & 3) << 2));
                const float s0 = *reinterpret_cast<const float*>(smem + st + p.s_off + o0);
                const float z0 = *reinterpret_cast<const float*>(smem + st + p.z_off + o0);
                const float s8 = *reinterpret_cast<const float*>(smem + st + p.s_off + o8);
                const float z8 = *reinterpret_cast<const float*>(smem + st + p.z_off + o8);
                const float y0 = fmaf(fmaf(-z0, sxt2, u0), 1.0f / 32768.0f, fmaf(-z0, sxt, v0));
                const float y8 = fmaf(fmaf(-z8, sxt2, u8), 1.0f / 32768.0f, fmaf(-z8, sxt, v8));
                acc[i][0] = fmaf(s0 * ft, y0, acc[i][0]);
                acc[i][1] = fmaf(s8 * ft, y8, acc[i][1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        if (++s == p.stages) { s = 0; ++round; }

        if (chunk == p.n_chunks - 1) {
            if (!waited) {   // the previous kernel may still read the outputs or write the residual
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
            if (p.has_norm && pass == 0) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane == 0) sq_part[warp] = sq;
            }
            named_barrier(1, kM1Warps * 32);
            if (p.has_norm && pass == 0) {
                float tot = 0.0f;
#pragma unroll
                for (int w = 0; w < kM1Warps; ++w) tot += sq_part[w];
                inv = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
            }
            const int m = work.mat(p, pass), t0 = work.t0(p, pass), nt = work.nt(p, pass);
            for (int e = threadIdx.x; e < nt * 16; e += kM1Warps * 32) {
                float sum = 0.0f;
#pragma unroll
                for (int w = 0; w < kM1Warps; ++w) sum += lds_f32(red + ((w * TP) * 16 + e) * 4);
                const int64_t n = static_cast<int64_t>(t0) * kTileRows + e;
                const float v = sum * inv;
                if (p.mode == 1 && m == 0) {
                    gate_buf[e] = v;   // the up pass of the same tiles comes next
                } else if (n < p.N[m]) {
                    float o = v;
                    if (p.mode == 1) {
                        const float gv = gate_buf[e];
                        o = gv / (1.0f + expf(-gv)) * v;   // silu(gate) * up
                    }
                    if (p.has_res) o += p.res[n];
                    p.out[p.mode == 1 ? 0 : m][n] = o;
                }
            }
            named_barrier(1, kM1Warps * 32);
        }
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

// One fused decode launch (see the file comment): mode 0 with 1-3 matrices, or mode 1 with
// gate and up.  The caller has checked q4a_fast_supports for every matrix.
struct Q4aFused {
    int mode = 0, n_mats = 1, K = 0;
    const float* x = nullptr;
    const uint8_t* wq[kQ4aMaxMats] = {};
    const float* scales[kQ4aMaxMats] = {};
    const float* zeros[kQ4aMaxMats] = {};
    int N[kQ4aMaxMats] = {};
    float* out[kQ4aMaxMats] = {};
    const float* res = nullptr;
    const float* gamma = nullptr;
    float eps = 0.0f;
    int stages = 0;   // ring depth; 0 = the default (three, as many as fit)
};

int launch_q4a_fused(const Q4aFused& f, cudaStream_t stream) {
    DeviceInfo dev;
    if (int rc = current_device_info(&dev)) return rc;
    Q4aParams p{};
    p.K = f.K;
    p.G = f.K / 32;
    p.n_chunks = static_cast<int>(ceil_div(f.K, kM1KC));
    p.mode = f.mode;
    p.n_mats = f.n_mats;
    p.has_norm = f.gamma != nullptr;
    p.has_res = f.res != nullptr;
    p.eps = f.eps;
    p.x = f.x;
    p.gamma = f.gamma;
    p.res = f.res;
    // the work split
    int tiles[kQ4aMaxMats] = {}, total_tiles = 0;
    for (int m = 0; m < f.n_mats; ++m) {
        p.N[m] = f.N[m];
        p.out[m] = f.out[m];
        tiles[m] = static_cast<int>(ceil_div(f.N[m], kTileRows));
        total_tiles += tiles[m];
    }
    int grid = 0, tiles_max = 0;
    if (f.mode == 1) {   // both matrices' rows of the same tiles in every CTA
        grid = std::min(tiles[0], dev.sm_count);
        p.cta0[0] = 0;
        p.cta0[1] = grid;
        p.tiles_base[0] = tiles[0] / grid;
        p.tiles_extra[0] = tiles[0] % grid;
        tiles_max = static_cast<int>(ceil_div(tiles[0], grid));
    } else {             // the SMs shared by the matrices in proportion to their tiles
        int ctas[kQ4aMaxMats] = {}, used = 0;
        for (int m = 0; m < f.n_mats; ++m) {
            ctas[m] = std::max(1, std::min(tiles[m], tiles[m] * dev.sm_count / std::max(1, total_tiles)));
            used += ctas[m];
        }
        for (int m = 0; used < dev.sm_count; m = (m + 1) % f.n_mats) {   // the rest, where tiles remain
            bool any = false;
            for (int k = 0; k < f.n_mats; ++k) any |= ctas[k] < tiles[k];
            if (!any) break;
            if (ctas[m] < tiles[m]) { ++ctas[m]; ++used; }
        }
        for (int m = 0; m < f.n_mats; ++m) {
            p.cta0[m + 1] = p.cta0[m] + ctas[m];
            p.tiles_base[m] = tiles[m] / ctas[m];
            p.tiles_extra[m] = tiles[m] % ctas[m];
            tiles_max = std::max(tiles_max, static_cast<int>(ceil_div(tiles[m], ctas[m])));
        }
        grid = p.cta0[f.n_mats];
    }
    const int tp = std::min(tiles_max, kQ4aTP);
    p.tp = tp;
    const uint32_t rows = kTileRows * kQ4aTP;
    p.w_box_bytes = rows * 128;                 // one 256-value nibble box
    p.s_off = 4 * p.w_box_bytes;                // four boxes per 1024-value chunk
    p.z_off = p.s_off + rows * 128;             // 32 fp32 scales per row, then 32 zero points
    p.x_off = p.z_off + rows * 128;
    p.g_off = p.x_off + kM1KC * 4;
    p.stage_bytes = (p.g_off + (p.has_norm ? kM1KC * 4 : 0) + 1023) / 1024 * 1024;
    const size_t tail = static_cast<size_t>(kM1Warps) * kQ4aTP * 16 * 4 + kM1Warps * 4 + rows * 4;   // red, sq, gate
    const size_t budget = static_cast<size_t>(dev.max_smem_optin) - 1024 - 64 - tail;
    p.stages = std::min(f.stages >= 2 ? f.stages : kQ4aStages, static_cast<int>(budget / (p.stage_bytes + 16)));
    if (p.stages < 2) return set_error(BYBYCU_ERR_SHAPE, "matmul_q4 decode: shared memory too small");
    const size_t smem = 1024 + static_cast<size_t>(p.stages) * (p.stage_bytes + 16) + 16 + tail;

    // tensor maps: nibbles as the Q4B32 decode kernel's, fp32 scales and zero points in 32-value
    // (128-byte) swizzled boxes of the same rows
    Q4aMaps<kQ4aMaxMats> maps;
    const int box_rows[3] = {kTileRows * tp, kTileRows * std::max(1, tp - 1), kTileRows};
    for (int m = 0; m < f.n_mats; ++m)
        for (int i = 0; i < 3; ++i) {
            if (int rc = encode_tensor_map_2d(&maps.w[m][i], CU_TENSOR_MAP_DATA_TYPE_UINT8, f.wq[m], f.K / 2, f.N[m],
                                              f.K / 2, 128, box_rows[i], CU_TENSOR_MAP_SWIZZLE_128B,
                                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
                return rc;
            const uint64_t pitch = static_cast<uint64_t>(f.K / 32) * 4;
            if (int rc = encode_tensor_map_2d(&maps.s[m][i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, f.scales[m], f.K / 32,
                                              f.N[m], pitch, 32, box_rows[i], CU_TENSOR_MAP_SWIZZLE_128B,
                                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
                return rc;
            if (int rc = encode_tensor_map_2d(&maps.z[m][i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, f.zeros[m], f.K / 32,
                                              f.N[m], pitch, 32, box_rows[i], CU_TENSOR_MAP_SWIZZLE_128B,
                                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
                return rc;
        }
    static std::once_flag once[64];
    static cudaError_t attr_rc[64];
    const int di = dev.device;
    if (di < 0 || di >= 64) return set_error(BYBYCU_ERR_ARGS, "device %d out of range", di);
    std::call_once(once[di], [&] {
        attr_rc[di] = cudaFuncSetAttribute(q4a_kernel<kQ4aTP, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
        if (attr_rc[di] == cudaSuccess)
            attr_rc[di] = cudaFuncSetAttribute(q4a_kernel<kQ4aTP, kQ4aMaxMats>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
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
    if (f.n_mats == 1) {
        Q4aMaps<1> one;
        for (int i = 0; i < 3; ++i) {
            one.w[0][i] = maps.w[0][i];
            one.s[0][i] = maps.s[0][i];
            one.z[0][i] = maps.z[0][i];
        }
        BYBYCU_CUDA_TRY(cudaLaunchKernelEx(&cfg, q4a_kernel<kQ4aTP, 1>, one, p));
    } else {
        BYBYCU_CUDA_TRY(cudaLaunchKernelEx(&cfg, q4a_kernel<kQ4aTP, kQ4aMaxMats>, maps, p));
    }
    BYBYCU_LAUNCH_CHECK("q4a_kernel");
    return BYBYCU_OK;
}

int launch_q4a(int K, int N, const float* x, const uint8_t* wq, const float* scales, const float* zeros, float* out,
               cudaStream_t stream, int stages = 0) {
    Q4aFused f;
    f.stages = stages;
    f.K = K;
    f.x = x;
    f.wq[0] = wq;
    f.scales[0] = scales;
    f.zeros[0] = zeros;
    f.N[0] = N;
    f.out[0] = out;
    return launch_q4a_fused(f, stream);
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
    if (route != BYBYCU_ROUTE_AUTO && route != BYBYCU_ROUTE_SIMT && route != BYBYCU_ROUTE_GEMV &&
        route != BYBYCU_ROUTE_TC)
        return set_error(BYBYCU_ERR_ARGS, "matmul_q4: route %d (AUTO, SIMT, GEMV or TC)", route);
    const bool fast = q4a_fast_supports(M, K, N, group_size, n_groups_per_row, a, wq, scales, zeros);
    const bool tc = M > 1 && tc_asym_supports(M, K, N, group_size, n_groups_per_row, a, wq, scales, zeros, c);
    int stages = 0;
    if (route == BYBYCU_ROUTE_AUTO) {
        apply_q4_plan(M, K, N, group_size, n_groups_per_row, fast, tc, &route, &stages);
        // no plan: the decode kernel at M = 1, the tensor-core GEMM above, else the exact kernel
        if (route == BYBYCU_ROUTE_AUTO) route = fast ? BYBYCU_ROUTE_GEMV : tc ? BYBYCU_ROUTE_TC : BYBYCU_ROUTE_SIMT;
    }
    if (route == BYBYCU_ROUTE_GEMV && !fast)
        return set_error(BYBYCU_ERR_SHAPE, "matmul_q4: the decode route needs M=1, group 32, K %% 128 == 0 and "
                                           "16-byte aligned slots");
    if (route == BYBYCU_ROUTE_TC && !tc)
        return set_error(BYBYCU_ERR_SHAPE, "matmul_q4: the tensor-core route needs M > 1, group 32, K %% 256 == 0 "
                                           "and 16-byte aligned slots");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (route == BYBYCU_ROUTE_TC) return launch_tc_asym(M, K, N, a, wq, scales, zeros, c, s);
    if (route == BYBYCU_ROUTE_SIMT) {
        dim3 grid(static_cast<unsigned>(ceil_div(N, 128)), static_cast<unsigned>(M));
        q4a_exact_kernel<<<grid, 128, 0, s>>>(M, K, N, group_size, n_groups_per_row, wq, scales, zeros, a, c);
        BYBYCU_LAUNCH_CHECK("q4a_exact_kernel");
        return BYBYCU_OK;
    }
    return launch_q4a(K, N, a, wq, scales, zeros, c, s, stages);
}

extern "C" int bybycu_matmul_q4_fused(int mode, const float* a, int n_mats, const uint8_t* const* wq,
                                      const float* const* scales, const float* const* zeros, const int* N,
                                      float* const* outs, const float* res, const float* gamma, float eps, int K,
                                      int group_size, int n_groups_per_row, void* stream) {
    if (!a || !wq || !scales || !zeros || !N || !outs) return set_error(BYBYCU_ERR_ARGS, "fused matmul_q4 slot is missing");
    if (mode != 0 && mode != 1) return set_error(BYBYCU_ERR_ARGS, "fused matmul_q4: mode %d (0 or 1)", mode);
    if (n_mats < 1 || n_mats > kQ4aMaxMats || (mode == 1 && n_mats != 2))
        return set_error(BYBYCU_ERR_SHAPE, "fused matmul_q4: %d matrices in mode %d", n_mats, mode);
    if (mode == 1 && N[0] != N[1]) return set_error(BYBYCU_ERR_SHAPE, "fused matmul_q4: gate and up differ in rows");
    if (gamma && (reinterpret_cast<uintptr_t>(gamma) & 15u))
        return set_error(BYBYCU_ERR_SHAPE, "fused matmul_q4: gamma is not 16-byte aligned");
    Q4aFused f;
    f.mode = mode;
    f.n_mats = n_mats;
    f.K = K;
    f.x = a;
    f.res = res;
    f.gamma = gamma;
    f.eps = eps;
    for (int m = 0; m < n_mats; ++m) {
        if (!wq[m] || !scales[m] || !zeros[m] || !outs[m]) return set_error(BYBYCU_ERR_ARGS, "fused matmul_q4 slot is missing");
        if (!q4a_fast_supports(1, K, N[m], group_size, n_groups_per_row, a, wq[m], scales[m], zeros[m]))
            return set_error(BYBYCU_ERR_SHAPE, "fused matmul_q4 needs group 32, K %% 128 == 0 and 16-byte aligned slots");
        f.wq[m] = wq[m];
        f.scales[m] = scales[m];
        f.zeros[m] = zeros[m];
        f.N[m] = N[m];
        f.out[m] = outs[m];
    }
    return launch_q4a_fused(f, static_cast<cudaStream_t>(stream));
}
