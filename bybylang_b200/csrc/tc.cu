// tc.cu - the prefill GEMM route: Q4B32 weights x activations on the 5th-generation tensor
// cores (tcgen05), CTA pairs (cta_group::2) persistent over the output tiles.
//
// The reference computes the same product with OP_TILE_GEMM's "matmul" phase
// (micro_kernel/tile_gemm.nim:20-34, backends/cpu/cpu_vm.c:605-626): out[m][n] =
// sum_k x[m][k] * w[n][k] in fp32.  Here:
//
//   * a pre-pass converts the activations to fp16 (exact for bf16 inputs inside the fp16
//     range) and permutes K inside every 32-block into the order the dequantizer produces
//     weight pairs in (stage_x_kernel);
//   * a pair tile is 256 weight rows (output features) x 128 tokens.  Each CTA of the pair
//     dequantizes its 128 weight rows into fp16 w = RNE(q * s) - one rounding per weight -
//     straight into its own tensor memory, where they are the MMA's A operand (one row per
//     TMEM lane, two K elements per 32-bit column): no shared-memory traffic for A;
//   * each CTA TMA-loads 64 of the tile's 128 token rows (128-byte swizzle); the pair's MMA
//     (M=256, N=128, K=16) reads both halves, so every activation byte crosses a shared-memory
//     port once per 256 weight rows - half of what a single-CTA 128-row tile needs, which is
//     what bounds the tensor pipe here;
//   * one thread of the even CTA issues the MMAs into fp32 accumulators in both CTAs' TMEM;
//     the accumulators are double-buffered, so the epilogue warps read tile t back
//     (tcgen05.ld) and store out[token][feature] while the MMAs of tile t+1 run.
//
// The same kernel, instantiated with ASYM, is the prefill route of the asymmetric Q4 matmul
// (matmul_q4, backends/cpu/cpu_kernels_impl.inc:293-319, whose Vulkan prefill runs on the
// cooperative-matrix units): interleaved nibbles (byte j holds k = 2j low, 2j + 1 high),
// fp32 scales and zero points per 32-block, each weight dequantised as
// w = RNE16(u * RNE16(s) + RNE16(-z * s)) by one half-precision FMA.
//
// Every wait is bounded (%globaltimer): on a timeout the kernel records an error code in
// g_device_error, drains its copies and MMAs, frees its tensor memory and returns.
#include "kernels.h"

#include <mutex>

namespace bybycu {
namespace tc {

constexpr int kRowsCta = 128;       // weight rows per CTA (MMA M = 2 x 128 per pair)
constexpr int kRowsPair = 256;
constexpr int kBN = 128;            // tokens per pair tile = MMA N
constexpr int kTokCta = kBN / 2;    // token rows each CTA loads
constexpr int kXK = 128;            // K per activation stage: two 128-byte swizzle rows of fp16
constexpr int kXSub = 64;           // K per 128-byte swizzle row (one TMA box)
constexpr int kWK = 256;            // K per weight stage: 128 packed bytes per row
constexpr int kStages = 8;          // activation stages in shared memory
constexpr int kASlots = 4;          // dequantized weight (A) slots in tensor memory
constexpr int kWStages = 3;         // weight stages in shared memory
constexpr int kSubs = kWK / kXK;    // activation stages per weight stage
// 20 warps: 0 X TMA, 1 MMA (even CTA) + TMEM alloc, 2 W TMA, 3 X relay (odd CTA),
// 4-15 dequant (three groups of four: activation stages i with i % 3 = group), 16-19 epilogue.
// The dequantisers are the kernel's throughput limit: a group needs longer to fill a stage's A
// slot than the pair's MMAs need to consume it, so three groups work on three stages at once.
constexpr int kThreads = 640;
constexpr int kDequantWarp0 = 4;
constexpr int kDequantGroups = 3;   // activation stage i is dequantised by group i % 3
constexpr int kEpilogueWarp0 = kDequantWarp0 + 4 * kDequantGroups;

constexpr uint32_t kXStageBytes = kTokCta * kXK * 2;         // 16 KiB per CTA
constexpr uint32_t kXSubBytes = kTokCta * kXSub * 2;         // 8 KiB
constexpr uint32_t kWStageBytes = kRowsCta * kWK / 2;        // 16 KiB
constexpr uint32_t kSStageBytes = kRowsCta * (kWK / 32) * 2; // 2 KiB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCols = kBN;                 // one accumulator buffer: a column per token
constexpr uint32_t kAOff = 2 * kAccCols;           // A slots after the two accumulator buffers
constexpr uint32_t kACols = kXK / 2;               // A slot: two fp16 per column
static_assert(kAOff + kASlots * kACols <= kTmemCols, "tensor memory budget");
// Arrivals that complete a stage on rank 0: its own TMA (with the bytes), the odd CTA's relay
// and the eight dequant warps of the pair.  The MMA thread polls this one barrier per stage:
// every shared-memory access of that thread stalls it for ~140 cycles while the tensor core
// streams operands, so it makes one per eight MMAs.
constexpr uint32_t kFullArrivals = 1 + 1 + 8;
// A scale stage holds fp16 scales (Q4B32) or fp32 scales followed by fp32 zero points
// (asymmetric Q4) of 128 rows x 8 blocks; the rest of the layout is in Cfg below.

// Token tiles of BN tokens: the MMA's N, the token rows each CTA of the pair loads (BN / 2)
// and the instruction descriptor.  BN = 128 for prefill; 16, 32 or 64 for a few rows, so that
// no MMA cycle goes to token columns that do not exist.
template <int BN>
struct TokTile {
    static_assert(BN == 16 || BN == 32 || BN == 64 || BN == 128, "token tile");
    static constexpr int kTokCta = BN / 2;
    static constexpr uint32_t kXStageBytes = kTokCta * kXK * 2;
    static constexpr uint32_t kXSubBytes = kTokCta * kXSub * 2;
    // kind::f16, D fp32, A and B fp16, both K-major, M = 256 (the pair), N = BN
    static constexpr uint32_t kIdesc = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(kRowsPair >> 4) << 24);
};

// The layout of one instantiation of the Q4 GEMM kernel.
template <bool ASYM, bool EXACT, int BN>
struct Cfg {
    using T = TokTile<BN>;
    // Two accumulator buffers: the epilogue drains one while the MMAs fill the other.
    static constexpr int kAccBufs = 2;
    static constexpr uint32_t kAOff = kAccBufs * BN;
    static constexpr uint32_t kSlotCols = EXACT ? 2 * kACols : kACols;   // tensor memory of one stage's A
    static constexpr int kAStagesFit = static_cast<int>((kTmemCols - kAOff) / kSlotCols);
    static constexpr int kAStages = kAStagesFit > 8 ? 8 : kAStagesFit;   // A stages in flight
    // Dequantiser groups at work: at most one per A stage in flight, so that no group waits
    // for a slot phase two rounds ahead (a phase-parity wait cannot tell those apart).
    static constexpr int kGroups = kDequantGroups < kAStages ? kDequantGroups : kAStages;
    // few tokens make a stage's MMAs short: a deeper weight ring keeps the stream in flight
    // (five stages at 128 tokens measured 3-7% slower than three)
    static constexpr int kWStages = BN >= 128 ? 3 : 6;
    static constexpr uint32_t kSBytes = ASYM ? 2 * kRowsCta * (kWK / 32) * 4 : kSStageBytes;
    static constexpr uint32_t kZOff = kSBytes / 2;
    static constexpr uint32_t kOffX = 0;
    static constexpr uint32_t kOffW = kOffX + kStages * T::kXStageBytes;
    static constexpr uint32_t kOffS = kOffW + kWStages * kWStageBytes;
    // barriers: full, x_empty [kStages]; a_empty [kAStages]; w_full, w_empty [kWStages];
    // d_full, d_empty [2]; done
    static constexpr uint32_t kNumBars = 2 * kStages + kAStages + 2 * kWStages + 5;
    static constexpr uint32_t kOffBar = kOffS + kWStages * kSBytes;
    static constexpr uint32_t kOffTmemSlot = kOffBar + kNumBars * 8;
    static constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
    // the epilogue's output staging: one chunk (up to 32 tokens x 32 fp32 features) per
    // epilogue warp, written back to the output rows with 16-byte stores
    static constexpr uint32_t kEpiWarpBytes = (BN < 32 ? BN : 32) * 32 * 4;
    static constexpr uint32_t kOffEpi = (kOffAbort + 4 + 15) / 16 * 16;
    static constexpr uint32_t kUsed = kOffEpi + 4 * kEpiWarpBytes + 1024;   // + alignment slack
    // more than half an SM's shared memory: one CTA per SM, so that no second CTA waits for
    // the tensor memory this one allocates
    static constexpr uint32_t kSmemBytes = kUsed > 117 * 1024 ? kUsed : 117 * 1024;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kAStages >= 2, "tensor memory budget");
};
// the largest shared-memory request of any instantiation (asymmetric scales, 128 tokens)
constexpr uint32_t kSmemBytes = Cfg<true, false, 128>::kSmemBytes > Cfg<false, true, 128>::kSmemBytes
                                    ? Cfg<true, false, 128>::kSmemBytes : Cfg<false, true, 128>::kSmemBytes;

// Instruction descriptor of kind::f16: D fp32, A and B fp16, both K-major, M=256, N=128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (uint32_t(kBN >> 3) << 17) |
                            (uint32_t(kRowsPair >> 4) << 24);

struct Maps {
    CUtensorMap x;   // fp16 [M, K], box 64 (K) x 64 (tokens), 128-byte swizzle
    CUtensorMap w;   // u8 [N, K/2], box 128 x 128, 128-byte swizzle
    CUtensorMap s;   // u16 [N, K/32] (asymmetric: fp32), box 8 x 128
    CUtensorMap z;   // asymmetric only: fp32 zero points [N, K/32], box 8 x 128
};

struct Params {
    int M, K, N;
    int tiles_n;      // 256-row weight tiles (N / 256, rounded up)
    int tiles;        // tiles_n * token tiles
    void* out;
    int64_t out_ld, out_col0;
    int out_bf16;
    PeerGather pg;    // world > 1: the epilogue also stores every value to the other ranks (fp32)
    // x_split: token rows come in pairs (x_hi, x_lo of one fp32 activation row, M counting
    // both); the epilogue stores row pair r as output row r / 2, the sum of the two
    int x_split = 0;
    // Work units (the Q4 kernels): tiles [0, full_tiles) whole, every later tile as `split`
    // K-parts (one unit each, weight-stage aligned) so that the last wave fills the pairs.
    // Parts 0 .. split-2 leave fp32 partial sums in `partial` ([tail tile][part][CTA][warp]
    // blocks of BN tokens x 32 features) and count them in `flags` (one counter per tail tile,
    // CTA and epilogue warp, zeroed by the staging pass); the last part adds them, in part
    // order, to its own and stores the tile.
    int units = 0;    // full_tiles + (tiles - full_tiles) * split
    int full_tiles = 0;
    int split = 1;
    float* partial = nullptr;
    uint32_t* flags = nullptr;
};

// One work unit: its tile, its part and its weight stages [kw0, kw1).
struct WorkUnit {
    int tile, part, kw0, kw1;
};
__device__ __forceinline__ WorkUnit work_unit(const Params& p, int u, int n_kw) {
    WorkUnit w;
    if (p.split <= 1 || u < p.full_tiles) {
        w.tile = u;
        w.part = 0;
        w.kw0 = 0;
        w.kw1 = n_kw;
    } else {
        const int v = u - p.full_tiles;
        w.tile = p.full_tiles + v / p.split;
        w.part = v % p.split;
        w.kw0 = w.part * n_kw / p.split;
        w.kw1 = (w.part + 1) * n_kw / p.split;
    }
    return w;
}

// 16-byte global -> shared copies (L2 only) and their completion.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Bounded wait (a whole warp) until a split-K counter reached `target`.
__device__ __forceinline__ bool wait_flag(const uint32_t* f, uint32_t target) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (v >= target) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            record_device_error(kDevErrSplitWait);
            return false;
        }
    }
}

// Bounded wait by plain try_wait polling.  With a suspend-time hint the waits of this kernel
// slept through tcgen05.commit arrivals (the GEMM ran 8x slower), so it polls.  The polls
// keep the default CTA-scope acquire even where the arrivals come from the peer CTA: what
// they order is complete before the arrive is issued (TMA complete_tx, tcgen05.wait::st /
// wait::ld), and a cluster-scope acquire costs the polling thread a memory barrier each time,
// which starved the MMA issuer.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            record_device_error(err);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------
// Cluster (CTA pair) helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Shared::cluster address of the same object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Arrive on a barrier given by its shared::cluster address (this CTA's or the peer's), with
// the default release semantics (see wait_bar).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05 wrappers (every tcgen05 operation of the kernel is cta_group::2)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The MMA-issuing warp runs its loop converged (all 32 lanes) and one lane, chosen by
// elect.sync, issues each tcgen05 operation.  Issuing from a single diverged lane instead
// left the tensor pipe idle ~40% of the time between stages.

// Arrives on `bar` in both CTAs of the pair once every tcgen05 operation issued before by
// this warp's elected lane has completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
            smem_u32(bar)),
        "h"(static_cast<uint16_t>(0x3))
        : "memory");
}
// The same, arriving on this CTA's `bar` only.
__device__ __forceinline__ void tc_commit_local(uint64_t* bar) {
    asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T over the pair: 256 x 128 x 16, fp16 in, fp32 accumulate.
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

// One activation stage: eight 256 x 128 x 16 MMAs over K = 128 from one elected lane (the
// first accumulating only when `accumulate` is set).  When `release` is set the previous
// stage's two release commits (activation stage and A slot, both CTAs) follow the first MMA,
// so a stage is freed as soon as possible without a commit between two queued MMAs.
__device__ __forceinline__ void mma_pair_stage(uint32_t d_tmem, uint32_t a0, const uint64_t (&b)[8],
                                               uint32_t accumulate, uint32_t release, uint32_t x_bar,
                                               uint32_t a_bar, uint32_t idesc = kIdesc) {
    asm volatile(
        "{\n\t.reg .pred e, p, q, r;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %2, 0;\n\t"
        "setp.eq.b32 q, %2, %2;\n\t"
        "setp.ne.and.b32 r, %19, 0, e;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %4, %3, p;\n\t"
        "@r tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%20], %22;\n\t"
        "@r tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%21], %22;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%5], %6, %3, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%7], %8, %3, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%9], %10, %3, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%11], %12, %3, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%13], %14, %3, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%15], %16, %3, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%17], %18, %3, q;\n\t}" ::"r"(d_tmem),
        "r"(a0), "r"(accumulate), "r"(idesc), "l"(b[0]), "r"(a0 + 8), "l"(b[1]), "r"(a0 + 16), "l"(b[2]),
        "r"(a0 + 24), "l"(b[3]), "r"(a0 + 32), "l"(b[4]), "r"(a0 + 40), "l"(b[5]), "r"(a0 + 48), "l"(b[6]),
        "r"(a0 + 56), "l"(b[7]), "r"(release), "r"(x_bar), "r"(a_bar), "h"(static_cast<uint16_t>(0x3))
        : "memory");
}

// The low weight term of an exact-weight stage: eight more MMAs from A slot `a0`, with the same
// activation descriptors, accumulating into the same D (issued right after mma_pair_stage).
__device__ __forceinline__ void mma_pair_accumulate8(uint32_t d_tmem, uint32_t a0, const uint64_t (&b)[8],
                                                     uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred e, q;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 q, %2, 0;\n\t"   // the instruction descriptor is never 0: accumulate
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %3, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%4], %5, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%6], %7, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%8], %9, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%10], %11, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%12], %13, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%14], %15, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%16], %17, %2, q;\n\t}" ::"r"(d_tmem),
        "r"(a0), "r"(idesc), "l"(b[0]), "r"(a0 + 8), "l"(b[1]), "r"(a0 + 16), "l"(b[2]), "r"(a0 + 24), "l"(b[3]),
        "r"(a0 + 32), "l"(b[4]), "r"(a0 + 40), "l"(b[5]), "r"(a0 + 48), "l"(b[6]), "r"(a0 + 56), "l"(b[7])
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

#define TC_REG32(v) \
    "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), \
    "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), \
    "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), \
    "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
#define TC_OUT32(v) \
    "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), \
    "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), \
    "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), \
    "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])

// This warp's 32 lanes, 32 consecutive 32-bit columns from `taddr`.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        TC_REG32(v)
        : "memory");
}
// This warp's 32 lanes, 16 consecutive 32-bit columns from `taddr`.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : TC_OUT32(v)
        : "r"(taddr)
        : "memory");
}

// This warp's 32 lanes, 16 consecutive 32-bit columns from `taddr`.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// ---------------------------------------------------------------------------------------
// Dequantization into the MMA's K order
//
// A packed 32-block is 16 bytes; byte j holds k = j (low nibble) and k = 16 + j (high
// nibble).  Word w (bytes 4w..4w+3) yields four fp16 pairs without any per-pair shift:
//   col 4w+0: low nibbles of bytes 4w, 4w+2      -> k = 4w,      4w+2
//   col 4w+1: high nibbles of bytes 4w, 4w+2     -> k = 16+4w,   18+4w
//   col 4w+2: low nibbles of bytes 4w+1, 4w+3    -> k = 4w+1,    4w+3
//   col 4w+3: high nibbles of bytes 4w+1, 4w+3   -> k = 17+4w,   19+4w
// so MMA position kk = 2*col + half of a block reads activation k = kPerm[kk]; the pre-pass
// writes the activations in that order.
// ---------------------------------------------------------------------------------------
// Asymmetric nibbles (byte j holds k = 2j low, 2j + 1 high) through the same extraction:
//   col 4w+0: low nibbles of bytes 4w, 4w+2  -> k = 8w,   8w+4
//   col 4w+1: high nibbles of bytes 4w, 4w+2 -> k = 8w+1, 8w+5
//   col 4w+2: low nibbles of bytes 4w+1, 4w+3 -> k = 8w+2, 8w+6
//   col 4w+3: high nibbles of bytes 4w+1, 4w+3 -> k = 8w+3, 8w+7
__host__ __device__ constexpr int perm_src_asym(int kk) { return (kk & ~7) + ((kk & 7) >> 1) + 4 * (kk & 1); }

__host__ __device__ constexpr int perm_src(int kk) {
    // kk = 8w + p  ->  source k inside the 32-block
    return (kk & 7) == 0 ? 4 * (kk >> 3)
         : (kk & 7) == 1 ? 4 * (kk >> 3) + 2
         : (kk & 7) == 2 ? 16 + 4 * (kk >> 3)
         : (kk & 7) == 3 ? 18 + 4 * (kk >> 3)
         : (kk & 7) == 4 ? 4 * (kk >> 3) + 1
         : (kk & 7) == 5 ? 4 * (kk >> 3) + 3
         : (kk & 7) == 6 ? 17 + 4 * (kk >> 3)
                         : 19 + 4 * (kk >> 3);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// One packed word -> four fp16x2 columns of w = RNE(q * s).  The nibble u is placed in the
// mantissa of 1024 (low nibble, value 1032 + q after the sign flip) or at 16x (high nibble,
// value 1152 + 16 q); the subtraction is exact, the product rounds once.  s16 = s / 16.
__device__ __forceinline__ void dequant_word(uint32_t v, __half2 s, __half2 s16, uint32_t* col) {
    const __half2 m_lo = bits_h2(0x64086408u), m_hi = bits_h2(0x64806480u);
    const uint32_t vh = v >> 8;
    col[0] = h2_bits(__hmul2(__hsub2(bits_h2((v & 0x000F000Fu) ^ 0x64086408u), m_lo), s));
    col[1] = h2_bits(__hmul2(__hsub2(bits_h2((v & 0x00F000F0u) ^ 0x64806480u), m_hi), s16));
    col[2] = h2_bits(__hmul2(__hsub2(bits_h2((vh & 0x000F000Fu) ^ 0x64086408u), m_lo), s));
    col[3] = h2_bits(__hmul2(__hsub2(bits_h2((vh & 0x00F000F0u) ^ 0x64806480u), m_hi), s16));
}

// The exact form: one packed word -> four fp16x2 columns of each of two weight terms,
// w = q * s_hi + q * s_lo, where s_hi is the fp16 scale with its three lowest mantissa bits
// cleared (at most 8 significant bits) and s_lo = s - s_hi (at most 3).  q has at most 3
// significant bits, so both products are exact in fp16 (q * s_hi needs at most 11 bits,
// q * s_lo at most 6) and their sum is q * s exactly: the tensor core's fp32 accumulation is
// the only rounding left.  Every nibble goes through the low-nibble form (1032 + q, one exact
// subtraction), the high ones after a 4-bit shift.
__device__ __forceinline__ void dequant_word_exact(uint32_t v, __half2 s_hi, __half2 s_lo, uint32_t* hi,
                                                   uint32_t* lo) {
    const __half2 m_lo = bits_h2(0x64086408u);
    const uint32_t src[4] = {v, v >> 4, v >> 8, v >> 12};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const __half2 q = __hsub2(bits_h2((src[c] & 0x000F000Fu) ^ 0x64086408u), m_lo);
        hi[c] = h2_bits(__hmul2(q, s_hi));
        lo[c] = h2_bits(__hmul2(q, s_lo));
    }
}

// One packed word of asymmetric nibbles -> four fp16x2 columns of w = RNE16(u s16 + m16), with
// s16 = RNE16(s) and m16 = RNE16(-z s) per block: the nibble placed in the mantissa of 1024
// minus 1024 is u exactly, and the half-precision FMA rounds once.  Three operations per
// two weights, as the Q4B32 dequantiser; the form that rounded an fp32 FMA once (byte
// permutes, FADD, FFMA, then one conversion: seven per pair) kept the ALU pipe 51% busy
// and the tensor pipe at 34% (644-666 TFLOP/s at 2048 x 4096 x 4096).  Rounding s and z s
// to fp16 costs ~2^-11 of each block's contribution, inside the route's 1e-3 tolerance.
__device__ __forceinline__ void dequant_word_asym(uint32_t v, __half2 s, __half2 mzs, uint32_t* col) {
    const __half2 m = bits_h2(0x64006400u);   // 1024
    const uint32_t vh = v >> 8;
    col[0] = h2_bits(__hfma2(__hsub2(bits_h2((v & 0x000F000Fu) | 0x64006400u), m), s, mzs));
    col[1] = h2_bits(__hfma2(__hsub2(bits_h2(((v >> 4) & 0x000F000Fu) | 0x64006400u), m), s, mzs));
    col[2] = h2_bits(__hfma2(__hsub2(bits_h2((vh & 0x000F000Fu) | 0x64006400u), m), s, mzs));
    col[3] = h2_bits(__hfma2(__hsub2(bits_h2(((vh >> 4) & 0x000F000Fu) | 0x64006400u), m), s, mzs));
}

// ---------------------------------------------------------------------------------------
// Pre-pass: activations (bf16 or fp32) -> fp16 in the permuted K order of the weight format.
// One thread per 32-block.  Values outside the fp16 range are recorded as a device error.
// ---------------------------------------------------------------------------------------
// PERM: kPermQ4B32, kPermAsym (the dequantisers' K orders) or kPermNone (fp16 weights).
constexpr int kPermQ4B32 = 0, kPermAsym = 1, kPermNone = 2;
__host__ __device__ constexpr int perm_of(int mode, int kk) {
    return mode == kPermAsym ? perm_src_asym(kk) : mode == kPermNone ? kk : perm_src(kk);
}
// SPLIT (fp32 x): two fp16 rows per activation row, x_hi = RNE16(x) in row 2m and the exact
// remainder x_lo = RNE16(x - x_hi) in row 2m + 1 (g: 32-blocks per row); together they keep
// about 22 of fp32's 24 significant bits.
template <bool XF32, int PERM = kPermQ4B32, bool SPLIT = false>
__global__ void __launch_bounds__(256) stage_x_kernel(const void* __restrict__ x, uint4* __restrict__ xp,
                                                      int64_t nblocks, PeerGather pg, uint32_t* flags = nullptr,
                                                      int n_flags = 0, int64_t g = 0) {
    static_assert(!SPLIT || XF32, "the two-term form is for fp32 activations");
    pdl_launch_dependents();   // the GEMM may start its prologue; it waits before reading xp
    if (blockIdx.x == 0)       // the GEMM's split-K counters (its griddepcontrol.wait sees these)
        for (int f = threadIdx.x; f < n_flags; f += blockDim.x) flags[f] = 0u;
    if (pg.split && pg.world > 1) {   // split phase: x may be the previous launch's gathered output
        if (threadIdx.x == 0) peer_gather_wait_previous(pg);
        __syncthreads();
    }
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    float v[32];
    if (XF32) {
        const float4* src = reinterpret_cast<const float4*>(x) + i * 8;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 f = __ldg(src + q);
            v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
        }
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(x) + i * 4;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 u = __ldg(src + q);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                v[8 * q + 2 * e] = __uint_as_float(w[e] << 16);
                v[8 * q + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
            }
        }
    }
    bool range_ok = true;
    uint32_t o[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const float a = v[perm_of(PERM, 2 * c)], b = v[perm_of(PERM, 2 * c + 1)];
        range_ok &= fabsf(a) < 65520.0f && fabsf(b) < 65520.0f;
        o[c] = h2_bits(__floats2half2_rn(a, b));
    }
    if (!range_ok) record_device_error(kDevErrActRange);
    if constexpr (SPLIT) {
        const int64_t m = i / g, c = i % g;
        uint4* hi = xp + ((2 * m) * g + c) * 4;
        uint4* lo = xp + ((2 * m + 1) * g + c) * 4;
        uint32_t r[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const __half2 h = bits_h2(o[k]);
            const float a = v[perm_of(PERM, 2 * k)] - __low2float(h), b = v[perm_of(PERM, 2 * k + 1)] - __high2float(h);
            r[k] = h2_bits(__floats2half2_rn(a, b));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            hi[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
            lo[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
        }
    } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) xp[i * 4 + q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
    }
}


// The epilogue warps of the GEMM kernels: accumulator buffer t % ACCB of each of this CTA's
// tiles of BN tokens back from tensor memory (tcgen05.ld, 32 or 16 columns at a time) and out
// to out[token][feature]; each warp owns the TMEM lane quarter `quarter` (32 features) and
// frees the buffer on rank 0 when done.
template <int BN, int ACCB>
__device__ __forceinline__ void epilogue_tiles_t(const Params& p, uint32_t tmem, uint64_t* d_full,
                                                 uint64_t* d_empty, volatile int* s_abort, int my_tiles, int pair,
                                                 int pairs, uint32_t rank, int quarter, int lane,
                                                 uint32_t stage_smem = 0, int max_slots = 0,
                                                 uint8_t* stage_gen = nullptr, uint8_t* epi_gen = nullptr) {
    constexpr int kChunk = BN < 32 ? BN : 32;
    constexpr int kBlock = BN * 32;   // floats of one warp's partial sums (BN tokens x 32 features)
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t lead_d_empty = map_to_rank(d_empty, 0);
    // Output chunks go through this warp's staging block when every 16-byte store is aligned:
    // a store instruction then writes 4 (fp32) or 8 (bf16) output rows of 128 / 64 contiguous
    // bytes instead of one strided value per lane (the strided form took ~1.2 us per chunk of
    // 32 tokens at 4096 columns, 4x the same stores into a contiguous block).
    // With a gather the same 16-byte segments go to every peer's buffer (fp32 outputs).
    const int esz = p.out_bf16 ? 2 : 4;
    bool peers_aligned = !p.out_bf16;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
        if (r < p.pg.world && reinterpret_cast<uintptr_t>(p.pg.out[r]) % 16 != 0) peers_aligned = false;
    const bool staged = epi_gen != nullptr && !p.x_split && (p.pg.world <= 1 || peers_aligned) &&
                        reinterpret_cast<uintptr_t>(p.out) % 16 == 0 && (p.out_ld * esz) % 16 == 0 &&
                        (p.out_col0 * esz) % 16 == 0;
    uint8_t* const epi = staged ? epi_gen + quarter * (kChunk * 32 * 4) : nullptr;
    for (int t = 0; t < my_tiles; ++t) {
        const int b = t % ACCB, u = t / ACCB;
        const int unit = pair + t * pairs;
        const WorkUnit w = work_unit(p, unit, 1);
        const int tile = w.tile;
        const int feat = (tile % p.tiles_n) * kRowsPair + static_cast<int>(rank) * kRowsCta + quarter * 32 + lane;
        const int tok0 = (tile / p.tiles_n) * BN;
        // split-K tail tile: this warp's partial sums of part q at part_at(q)
        const bool tail = p.split > 1 && unit >= p.full_tiles;
        const bool last = !tail || w.part == p.split - 1;
        const int tix = tail ? (unit - p.full_tiles) / p.split : 0;
        auto part_at = [&](int q) {
            return p.partial + ((static_cast<int64_t>(tix * (p.split - 1) + q) * 2 + rank) * 4 + quarter) * kBlock;
        };
        uint32_t* flag = tail ? p.flags + (tix * 2 + rank) * 4 + quarter : nullptr;
        bool ok = __all_sync(0xffffffffu, wait_bar(&d_full[b], u & 1, kDevErrMmaWait));
        if (ok && tail && last)   // the other parts of this tile stored their sums
            ok = __all_sync(0xffffffffu, wait_flag(flag, static_cast<uint32_t>(p.split - 1)));
        if (!ok) {
            *s_abort = 1;
            break;
        }
        tc_fence_after();
        // The last part sums the others' blocks in shared memory: the stage buffers, free once
        // this unit's MMAs completed (a tail unit is its pair's last), `max_slots` blocks per
        // warp.  Every block of a batch is fetched at once (one round trip per batch; one batch
        // when the parts fit); a later batch first folds the slots into slot 0, in part order.
        // The sums read the slots with plain loads (stage_gen is stage_smem's generic address),
        // so the compiler keeps many in flight: asm loads with a memory clobber issued one
        // dependent chain per token and left a 4-part finisher ~9 us behind the other CTAs.
        const uint32_t slot_off = static_cast<uint32_t>(quarter * max_slots) * (kBlock * 4);
        const uint32_t slot0 = stage_smem + slot_off;
        float* const slots = reinterpret_cast<float*>(stage_gen + slot_off);   // [max_slots][kBlock]
        int active = 0;   // slots holding parts still to add, slot 0 first
        if (tail && last) {
            auto fetch = [&](int q, int slot) {
                const float* src = part_at(q);
                const uint32_t dst = slot0 + static_cast<uint32_t>(slot) * (kBlock * 4);
#pragma unroll
                for (int k = 0; k < kBlock / 4 / 32; ++k)
                    cp_async16(dst + (k * 32 + lane) * 16, src + (k * 32 + lane) * 4);
            };
            const int parts = p.split - 1;
            int done = min(parts, max_slots);
            for (int q = 0; q < done; ++q) fetch(q, q);
            cp_async_commit();
            active = done;
            while (done < parts) {
                cp_async_wait<0>();
                __syncwarp();
#pragma unroll 8
                for (int tk = 0; tk < BN; ++tk) {
                    const int o = tk * 32 + lane;
                    float sum = slots[o];
                    for (int k = 1; k < active; ++k) sum += slots[k * kBlock + o];
                    slots[o] = sum;
                }
                __syncwarp();
                const int nb = min(max_slots - 1, parts - done);
                for (int k = 0; k < nb; ++k) fetch(done + k, 1 + k);
                cp_async_commit();
                done += nb;
                active = 1 + nb;
            }
            cp_async_wait<0>();
            __syncwarp();
        }
        const bool feat_ok = feat < p.N;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += kChunk) {
            uint32_t v[32];
            if constexpr (kChunk == 32) tmem_ld32(tmem + lane_addr + b * BN + c0, v);
            else tmem_ld16(tmem + lane_addr + b * BN + c0, v);
            tc_wait_ld();
            if (!last) {   // an earlier part: its partial sums, [token][feature] (coalesced)
                float* q = part_at(w.part) + c0 * 32 + lane;
#pragma unroll
                for (int j = 0; j < kChunk; ++j) q[j * 32] = __uint_as_float(v[j]);
                continue;
            }
            if (tail)   // the other parts in part order, then this part's
#pragma unroll
                for (int j = 0; j < kChunk; ++j) {
                    const int o = (c0 + j) * 32 + lane;
                    float sum = slots[o];
                    for (int k = 1; k < active; ++k) sum += slots[k * kBlock + o];
                    v[j] = __float_as_uint(sum + __uint_as_float(v[j]));
                }
            const int f0 = feat - lane;   // this warp's first feature
            if (staged && f0 + 32 <= p.N) {
                const int nt = min(kChunk, p.M - (tok0 + c0));
                const int64_t row0 = static_cast<int64_t>(tok0 + c0) * p.out_ld + p.out_col0 + f0;
                if (p.out_bf16) {   // [kChunk][32] bf16, then 8 rows of 64 bytes per store
                    __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(epi);
#pragma unroll
                    for (int j = 0; j < kChunk; ++j) st[j * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[j]));
                    __syncwarp();
#pragma unroll
                    for (int r = 0; r < kChunk / 8; ++r) {
                        const int j = r * 8 + (lane >> 2), f = (lane & 3) * 8;
                        if (j < nt)
                            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + row0 + j * p.out_ld + f) =
                                *reinterpret_cast<const uint4*>(st + j * 32 + f);
                    }
                } else {            // [kChunk][32] fp32, then 4 rows of 128 bytes per store
                    float* st = reinterpret_cast<float*>(epi);
#pragma unroll
                    for (int j = 0; j < kChunk; ++j) st[j * 32 + lane] = __uint_as_float(v[j]);
                    __syncwarp();
#pragma unroll
                    for (int r = 0; r < kChunk / 4; ++r) {
                        const int j = r * 4 + (lane >> 3), f = (lane & 7) * 4;
                        if (j < nt) {
                            const float4 val = *reinterpret_cast<const float4*>(st + j * 32 + f);
                            const int64_t oi = row0 + j * p.out_ld + f;
                            *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + oi) = val;
                            if (p.pg.world > 1)   // the fused all-gather: every peer's buffer
#pragma unroll
                                for (int q = 0; q < kMaxRanks; ++q)
                                    if (q < p.pg.world && q != p.pg.rank)
                                        *reinterpret_cast<float4*>(p.pg.out[q] + oi) = val;
                        }
                    }
                }
                __syncwarp();   // the block is read before the next chunk overwrites it
            } else if (feat_ok && p.x_split) {   // row pairs (x_hi, x_lo): one output row each
                const int nt = min(kChunk, p.M - (tok0 + c0));
                const int64_t o0 = p.out_col0 + feat + static_cast<int64_t>((tok0 + c0) >> 1) * p.out_ld;
#pragma unroll
                for (int j = 0; j < kChunk; j += 2) {
                    if (j >= nt) continue;
                    const float val = __uint_as_float(v[j]) + __uint_as_float(v[j + 1]);
                    const int64_t oi = o0 + (j >> 1) * p.out_ld;
                    if (p.out_bf16) reinterpret_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(val);
                    else reinterpret_cast<float*>(p.out)[oi] = val;
                    if (p.pg.world > 1) store_to_peers(p.pg, oi, val);
                }
            } else if (feat_ok) {
                const int nt = min(kChunk, p.M - (tok0 + c0));
                if (p.out_bf16) {
                    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + p.out_col0 + feat +
                                       static_cast<int64_t>(tok0 + c0) * p.out_ld;
#pragma unroll
                    for (int j = 0; j < kChunk; ++j)
                        if (j < nt) o[j * p.out_ld] = __float2bfloat16_rn(__uint_as_float(v[j]));
                } else {
                    const int64_t o0 = p.out_col0 + feat + static_cast<int64_t>(tok0 + c0) * p.out_ld;
                    float* o = reinterpret_cast<float*>(p.out) + o0;
#pragma unroll
                    for (int j = 0; j < kChunk; ++j)
                        if (j < nt) o[j * p.out_ld] = __uint_as_float(v[j]);
                    if (p.pg.world > 1)   // the fused all-gather: the same values into every rank
#pragma unroll
                        for (int j = 0; j < kChunk; ++j)
                            if (j < nt) store_to_peers(p.pg, o0 + j * p.out_ld, __uint_as_float(v[j]));
                }
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            if (!last)   // release: the warp's partial stores (ordered by the warp barrier) first
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(flag) : "memory");
            mbar_arrive_cluster(lead_d_empty + 8u * b);
        }
    }
}

// The 128-token, two-buffer form (the format-1 kernel's).
__device__ __forceinline__ void epilogue_tiles(const Params& p, uint32_t tmem, uint64_t* d_full, uint64_t* d_empty,
                                               volatile int* s_abort, int my_tiles, int pair, int pairs,
                                               uint32_t rank, int quarter, int lane) {
    epilogue_tiles_t<kBN, 2>(p, tmem, d_full, d_empty, s_abort, my_tiles, pair, pairs, rank, quarter, lane);
}

// ---------------------------------------------------------------------------------------
// The GEMM kernel (launched as clusters of two CTAs; rank 0 issues the MMAs)
// ---------------------------------------------------------------------------------------
// EXACT (Q4B32 only): the weights enter as the two exact fp16 terms of dequant_word_exact, in
// a pair of A slots per stage, sixteen MMAs per stage.  BN: tokens per pair tile (Cfg).
template <bool ASYM, bool EXACT, int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ Maps maps, const Params p) {
    static_assert(!(ASYM && EXACT), "the exact weight split is for Q4B32");
    using L = Cfg<ASYM, EXACT, BN>;
    using T = TokTile<BN>;
    constexpr int kAStages = L::kAStages;   // A stages in flight (a slot, or a slot pair when EXACT)
    constexpr int kWSt = L::kWStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
    // full[s]: on rank 0 the whole stage is ready (both activation halves, both A slots);
    // on rank 1 its own activation half landed (its relay forwards that to rank 0)
    uint64_t* full = bars;
    uint64_t* x_empty = bars + kStages;          // the pair's MMAs finished with the activation stage
    uint64_t* a_empty = bars + 2 * kStages;      // ... and with the A slot
    uint64_t* w_full = a_empty + kAStages;
    uint64_t* w_empty = w_full + kWSt;
    uint64_t* d_full = w_empty + kWSt;           // [2] accumulator buffer complete
    uint64_t* d_empty = d_full + 2;              // [2] (rank 0) both epilogues read it
    uint64_t* done_bar = d_full + 4;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + L::kOffTmemSlot);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::kOffAbort);

    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], leader ? kFullArrivals : 1);
            mbar_init(&x_empty[i], 1);
        }
        for (int i = 0; i < kAStages; ++i) mbar_init(&a_empty[i], 1);
        for (int i = 0; i < kWSt; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 8);       // both dequant groups
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&d_full[b], 1);
            mbar_init(&d_empty[b], 8);       // four epilogue warps in each CTA
        }
        mbar_init(done_bar, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), kTmemCols);
    tc_fence_before();
    cluster_sync();   // both CTAs' barriers initialised and tensor memory allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int pair = static_cast<int>(blockIdx.x >> 1), pairs = static_cast<int>(gridDim.x >> 1);
    const int my_units = p.units > pair ? (p.units - 1 - pair) / pairs + 1 : 0;
    const int n_kw = p.K / kWK;            // weight stages of a whole tile

    if (warp == 0) {
        // ------------------------------------------------------------ activation producer
        if (lane == 0) {
            prefetch_tensormap(&maps.x);
            pdl_wait();   // the staging pass that writes xp has completed
            // split-phase gather: every rank finished the previous launch before any value of
            // this one reaches a peer (the staging pass waited for the same; this costs one
            // already-satisfied load per rank)
            peer_gather_wait_previous(p.pg);
            int issued = 0;
            for (int t = 0; t < my_units && !*s_abort; ++t) {
                const WorkUnit w = work_unit(p, pair + t * pairs, n_kw);
                const int tok = (w.tile / p.tiles_n) * BN + static_cast<int>(rank) * T::kTokCta;
                for (int ks = w.kw0 * kSubs; ks < w.kw1 * kSubs; ++ks) {
                    const int s = issued % kStages, r = issued / kStages;
                    if (r > 0 && !wait_bar(&x_empty[s], (r - 1) & 1, kDevErrEmptyWait)) {
                        *s_abort = 1;
                        break;
                    }
                    if (*s_abort) break;
                    mbar_arrive_expect_tx(&full[s], T::kXStageBytes);
                    uint8_t* dst = smem + L::kOffX + s * T::kXStageBytes;
                    tma_load_2d(dst, &maps.x, &full[s], ks * kXK, tok);
                    tma_load_2d(dst + T::kXSubBytes, &maps.x, &full[s], ks * kXK + kXSub, tok);
                    ++issued;
                }
            }
            // rank 1 waits for its copies to land; rank 0's own full barrier also counts the
            // other arrivals, so it waits for the pair's MMAs to release the stages instead
            for (int it = issued > kStages ? issued - kStages : 0; it < issued; ++it) {
                const bool landed = leader ? wait_bar(&x_empty[it % kStages], (it / kStages) & 1, kDevErrDrainWait)
                                           : wait_bar(&full[it % kStages], (it / kStages) & 1, kDevErrDrainWait);
                if (!landed) break;
            }
        }
    } else if (warp == 3) {
        // ------------------------------- (odd CTA) tells rank 0 that its half has landed
        if (!leader && lane == 0) {
            const uint32_t lead_full = map_to_rank(full, 0);
            int total = 0;
            for (int t = 0; t < my_units; ++t) {
                const WorkUnit w = work_unit(p, pair + t * pairs, n_kw);
                total += (w.kw1 - w.kw0) * kSubs;
            }
            for (int i = 0; i < total; ++i) {
                const int s = i % kStages;
                if (!wait_bar(&full[s], (i / kStages) & 1, kDevErrFullWait) || *s_abort) {
                    *s_abort = 1;
                    break;
                }
                mbar_arrive_cluster(lead_full + 8u * s);
            }
        }
    } else if (warp == 2) {
        // ---------------------------------------------------------------- weight producer
        if (lane == 0) {
            prefetch_tensormap(&maps.w);
            prefetch_tensormap(&maps.s);
            if constexpr (ASYM) prefetch_tensormap(&maps.z);
            const uint64_t policy = l2_policy_evict_last();
            int issued = 0;
            for (int t = 0; t < my_units && !*s_abort; ++t) {
                const WorkUnit w = work_unit(p, pair + t * pairs, n_kw);
                const int row0 = (w.tile % p.tiles_n) * kRowsPair + static_cast<int>(rank) * kRowsCta;
                for (int kw = w.kw0; kw < w.kw1; ++kw) {
                    const int s = issued % kWSt, r = issued / kWSt;
                    if (r > 0 && !wait_bar(&w_empty[s], (r - 1) & 1, kDevErrEmptyWait)) {
                        *s_abort = 1;
                        break;
                    }
                    if (*s_abort) break;
                    mbar_arrive_expect_tx(&w_full[s], kWStageBytes + L::kSBytes);
                    tma_load_2d_hint(smem + L::kOffW + s * kWStageBytes, &maps.w, &w_full[s], kw * (kWK / 2), row0, policy);
                    tma_load_2d_hint(smem + L::kOffS + s * L::kSBytes, &maps.s, &w_full[s], kw * (kWK / 32), row0, policy);
                    if constexpr (ASYM)
                        tma_load_2d_hint(smem + L::kOffS + s * L::kSBytes + L::kZOff, &maps.z, &w_full[s], kw * (kWK / 32),
                                         row0, policy);
                    ++issued;
                }
            }
            for (int it = issued > kWSt ? issued - kWSt : 0; it < issued; ++it)
                if (!wait_bar(&w_full[it % kWSt], (it / kWSt) & 1, kDevErrDrainWait)) break;
        }
    } else if (warp == 1) {
        // ------------------------------------------------- MMA issuer (rank 0, whole warp)
        // A stage's release (its commit) is issued after the next stage's first MMA, so the
        // commit never stands between two MMAs in the issue stream.
        if (leader) {
            // stage i frees its activation stage and its A slot once its MMAs completed
            auto release_stage = [&](int i) {
                tc_commit_pair(&x_empty[i % kStages]);
                tc_commit_pair(&a_empty[i % kAStages]);
            };
            int consumed = 0, pending = -1;
            for (int t = 0; t < my_units && !*s_abort; ++t) {
                const WorkUnit w = work_unit(p, pair + t * pairs, n_kw);
                const int n_ks = (w.kw1 - w.kw0) * kSubs;   // this unit's activation stages
                const int b = t % L::kAccBufs, u = t / L::kAccBufs;
                if (u > 0 && !__all_sync(0xffffffffu, wait_bar(&d_empty[b], (u - 1) & 1, kDevErrMmaWait))) {
                    *s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * BN;
                bool ok = true;
                for (int ks = 0; ks < n_ks; ++ks) {
                    const int s = consumed % kStages, r = consumed / kStages;
                    if (!__all_sync(0xffffffffu, wait_bar(&full[s], r & 1, kDevErrFullWait))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdesc = sw128_desc(base + L::kOffX + s * T::kXStageBytes);
                    const uint32_t a0 = tmem + L::kAOff + (EXACT ? 2 : 1) * (consumed % kAStages) * kACols;
                    // 16-K steps advance 32 bytes inside a 128-byte swizzle row, then jump to
                    // the next 64-K box
                    uint64_t bk[8];
#pragma unroll
                    for (int k16 = 0; k16 < kXK / 16; ++k16)
                        bk[k16] = bdesc + static_cast<uint64_t>((k16 >> 2) * (T::kXSubBytes >> 4) + (k16 & 3) * 2);
                    const int pv = pending >= 0 ? pending : 0;
                    mma_pair_stage(d_tmem, a0, bk, ks != 0, pending >= 0, smem_u32(&x_empty[pv % kStages]),
                                   smem_u32(&a_empty[pv % kAStages]), T::kIdesc);
                    if constexpr (EXACT) mma_pair_accumulate8(d_tmem, a0 + kACols, bk, T::kIdesc);
                    pending = consumed;
                    ++consumed;
                }
                if (!ok) {
                    *s_abort = 1;
                    break;
                }
                release_stage(pending);   // the tile's last stage
                pending = -1;
                tc_commit_pair(&d_full[b]);
            }
            if (pending >= 0) release_stage(pending);
            // every MMA issued above has completed before the tensor memory is freed
            tc_commit_local(done_bar);
            __all_sync(0xffffffffu, wait_bar(done_bar, 0, kDevErrMmaWait));
        }
    } else if (warp < kEpilogueWarp0) {
        // ------------------------------------------------------------------ dequantizers
        // A weight stage (K=256) holds two activation stages (sub = 0, 1); activation stage i
        // of this CTA's tiles is group (i % 3)'s.  Each warp owns the TMEM lane quarter
        // (warp % 4) = 32 rows.
        const int grp = (warp - kDequantWarp0) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t lead_full = map_to_rank(full, 0);
        bool ok = grp < L::kGroups;
        // i counts the CTA's activation stages over its units, wbase its weight stages
        int i = 0, wbase = 0;
        for (int t = 0; t < my_units && ok; ++t) {
            const WorkUnit w = work_unit(p, pair + t * pairs, n_kw);
            const int n_ks = (w.kw1 - w.kw0) * kSubs;
            for (int ks = 0; ks < n_ks && ok; ++ks, ++i) {
                if (i % L::kGroups != grp) continue;
                const int wsg = wbase + ks / kSubs;                     // weight stage, counted over units
                const int sub = ks % kSubs;                             // which half of it
                const int ws = wsg % kWSt;
                ok = wait_bar(&w_full[ws], (wsg / kWSt) & 1, kDevErrFullWait) && !*s_abort;
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                // this stage's four 32-blocks of the weight stage: c = 4 * sub + h
                const uint32_t wrow = base + L::kOffW + ws * kWStageBytes + row * 128;
                uint4 chunk[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) chunk[h] = lds_u128(wrow + (((4 * sub + h) ^ (row & 7)) << 4));
                uint4 sc;
                float4 sa, za;   // asymmetric: fp32 scales and zero points of blocks 4 sub .. 4 sub + 3
                if constexpr (ASYM) {
                    const uint32_t sb = base + L::kOffS + ws * L::kSBytes + row * 32 + sub * 16;
                    sa = lds_v4f(sb);
                    za = lds_v4f(sb + L::kZOff);
                } else {
                    sc = lds_u128(base + L::kOffS + ws * L::kSBytes + row * 16);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&w_empty[ws]);   // the two groups of its halves release it
                const int s = i % kStages;                          // its activation stage (full barrier)
                const int slot = i % kAStages, r = i / kAStages;    // its A slot (pair, when EXACT)
                if (r > 0) ok = wait_bar(&a_empty[slot], (r - 1) & 1, kDevErrEmptyWait);
                ok = __all_sync(0xffffffffu, ok && !*s_abort);
                if (!ok) break;
                tc_fence_after();
                if constexpr (ASYM) {
                    const __half2 sv[4] = {__float2half2_rn(sa.x), __float2half2_rn(sa.y), __float2half2_rn(sa.z),
                                           __float2half2_rn(sa.w)};
                    const __half2 mz[4] = {__float2half2_rn(-za.x * sa.x), __float2half2_rn(-za.y * sa.y),
                                           __float2half2_rn(-za.z * sa.z), __float2half2_rn(-za.w * sa.w)};
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        uint32_t col[32];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int blk = 2 * half + h;
                            const uint4 u = chunk[blk];
                            dequant_word_asym(u.x, sv[blk], mz[blk], &col[16 * h + 0]);
                            dequant_word_asym(u.y, sv[blk], mz[blk], &col[16 * h + 4]);
                            dequant_word_asym(u.z, sv[blk], mz[blk], &col[16 * h + 8]);
                            dequant_word_asym(u.w, sv[blk], mz[blk], &col[16 * h + 12]);
                        }
                        tmem_st32(tmem + lane_addr + L::kAOff + slot * kACols + half * 32, col);
                    }
                } else if constexpr (EXACT) {
                    const uint32_t sw0 = sub ? sc.z : sc.x, sw1 = sub ? sc.w : sc.y;
                    const uint32_t a_hi = tmem + lane_addr + L::kAOff + 2 * slot * kACols;
                    // one block (16 columns of each term) at a time: 32 live column registers
#pragma unroll
                    for (int blk = 0; blk < 4; ++blk) {
                        const uint32_t pr = (blk >> 1) ? sw1 : sw0;           // two blocks' fp16 scales
                        const uint32_t prh = pr & 0xFFF8FFF8u;                // s_hi of both
                        const __half2 lo2 = __hsub2(bits_h2(pr), bits_h2(prh));   // s_lo, exact
                        const __half2 shi = (blk & 1) ? __high2half2(bits_h2(prh)) : __low2half2(bits_h2(prh));
                        const __half2 slo = (blk & 1) ? __high2half2(lo2) : __low2half2(lo2);
                        uint32_t hcol[16], lcol[16];
                        const uint4 u = chunk[blk];
                        dequant_word_exact(u.x, shi, slo, &hcol[0], &lcol[0]);
                        dequant_word_exact(u.y, shi, slo, &hcol[4], &lcol[4]);
                        dequant_word_exact(u.z, shi, slo, &hcol[8], &lcol[8]);
                        dequant_word_exact(u.w, shi, slo, &hcol[12], &lcol[12]);
                        tmem_st16(a_hi + blk * 16, hcol);
                        tmem_st16(a_hi + kACols + blk * 16, lcol);
                    }
                } else {
                    // scales of blocks 4 sub .. 4 sub + 3: two 32-bit words of the row's eight
                    const uint32_t sw0 = sub ? sc.z : sc.x, sw1 = sub ? sc.w : sc.y;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const __half2 pr = bits_h2(half ? sw1 : sw0);
                        uint32_t col[32];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const __half2 sv = h ? __half2half2(pr.y) : __half2half2(pr.x);
                            const __half2 s16 = __hmul2(sv, bits_h2(0x2C002C00u));   // x 1/16
                            const uint4 u = chunk[2 * half + h];
                            dequant_word(u.x, sv, s16, &col[16 * h + 0]);
                            dequant_word(u.y, sv, s16, &col[16 * h + 4]);
                            dequant_word(u.z, sv, s16, &col[16 * h + 8]);
                            dequant_word(u.w, sv, s16, &col[16 * h + 12]);
                        }
                        tmem_st32(tmem + lane_addr + L::kAOff + slot * kACols + half * 32, col);
                    }
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(lead_full + 8u * s);
            }
            wbase += w.kw1 - w.kw0;
        }
        if (!ok && grp < L::kGroups) *s_abort = 1;
    } else {
        // ---------------------------------------------------------------------- epilogue
        // split-K sums: two blocks of BN tokens x 32 fp32 features per epilogue warp in the
        // stage buffers (offsets 0 .. kOffBar).  Fetching every part at once into more slots
        // measured slower (16 and 64 tokens: 16.5 against 14.9 us, 22.5 against 18.8 us at
        // 4096 x 4096) than two slots and a fold between batches.
        constexpr int kSlots = 2;
        static_assert(4 * kSlots * BN * 32 * 4 <= L::kOffBar, "split-K sums: two blocks per warp");
        epilogue_tiles_t<BN, L::kAccBufs>(p, tmem, d_full, d_empty, s_abort, my_units, pair, pairs, rank, warp & 3,
                                          lane, base, kSlots, smem, smem + L::kOffEpi);
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();   // neither CTA frees its tensor memory while the pair may still use it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    // the barriers above ordered every epilogue store of this CTA before thread 0's release
    if (threadIdx.x == 0 && p.pg.world > 1) peer_gather_finish(p.pg);
}

}  // namespace tc

bool tc_supports(const GemmArgs& a) {
    if (a.fmt == BYBYCU_FMT_F16) return tc_f16_supports(a);
    if (a.fmt != BYBYCU_FMT_Q4B32) return false;
    if (a.K < tc::kWK || a.K % tc::kWK != 0 || a.M < 1 || a.N < 1) return false;
    if (a.x_dtype != BYBYCU_DT_BF16 && a.x_dtype != BYBYCU_DT_F32) return false;
    if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(a.packed) % 16 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(a.packed) + static_cast<uintptr_t>(a.scale_base)) % 16 != 0) return false;
    const size_t esz = a.out_dtype == BYBYCU_DT_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(a.out) % esz != 0) return false;
    DeviceInfo info;
    if (current_device_info(&info) != BYBYCU_OK) return false;
    return info.cc_major == 10 && info.max_smem_optin >= static_cast<int>(tc::kSmemBytes);
}

// Stream-ordered scratch for the staged activations: one pool per device that keeps its
// memory between calls (the default pool returns it at every synchronization, and mapping
// it again costs more than the GEMM).
static int scratch_pool(int device, cudaMemPool_t* pool) {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    if (device < 0 || device >= 64) return set_error(BYBYCU_ERR_ARGS, "device %d out of range", device);
    std::lock_guard<std::mutex> lock(mu);
    if (!pools[device]) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        cudaMemPool_t p = nullptr;
        BYBYCU_CUDA_TRY(cudaMemPoolCreate(&p, &props));
        uint64_t keep = UINT64_MAX;
        cudaError_t e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
        if (e != cudaSuccess) {
            cudaMemPoolDestroy(p);
            return cuda_fail(e, "cudaMemPoolSetAttribute(release threshold)");
        }
        pools[device] = p;
    }
    *pool = pools[device];
    return BYBYCU_OK;
}


// Token tile of an M-row call: the smallest of 16, 32 and 64 tokens that holds every row, else
// 128 (then the rows take ceil(M / 128) tiles).
static int tc_token_tile(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

// Device info, the kernel attribute and the number of CTA pairs that fit at once, per kernel
// instantiation and device.
template <bool ASYM, bool EXACT, int BN>
static int tc_setup(DeviceInfo* info, int* max_pairs) {
    if (int rc = current_device_info(info)) return rc;
    static std::once_flag once[64];
    static cudaError_t prep_rc[64];
    static int pairs[64];
    const int dev = info->device;
    if (dev < 0 || dev >= 64) return set_error(BYBYCU_ERR_ARGS, "device %d out of range", dev);
    constexpr uint32_t smem = tc::Cfg<ASYM, EXACT, BN>::kSmemBytes;
    std::call_once(once[dev], [&] {
        prep_rc[dev] = cudaFuncSetAttribute(tc::gemm_kernel<ASYM, EXACT, BN>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (prep_rc[dev] != cudaSuccess) return;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * (info->sm_count / 2));
        cfg.blockDim = dim3(tc::kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        prep_rc[dev] = cudaOccupancyMaxActiveClusters(&pairs[dev], tc::gemm_kernel<ASYM, EXACT, BN>, &cfg);
    });
    if (prep_rc[dev] != cudaSuccess) return cuda_fail(prep_rc[dev], "tensor-core GEMM set-up");
    if (pairs[dev] < 1) return set_error(BYBYCU_ERR_DEVICE, "no CTA pair of the tensor-core GEMM fits on the device");
    *max_pairs = pairs[dev];
    return BYBYCU_OK;
}

static int tc_check(const GemmArgs& a) {
    if (!tc_supports(a))
        return set_error(BYBYCU_ERR_SHAPE,
                         "tensor-core route needs format 2, K %% 256 == 0, 16-byte aligned x, packed and scales "
                         "(M=%d K=%d N=%d)", a.M, a.K, a.N);
    return BYBYCU_OK;
}

// The weights of one tensor-core GEMM: Q4B32 (nibbles and fp16 scales in `packed`) or
// asymmetric Q4 (nibbles, fp32 scales, fp32 zero points).
struct TcWeights {
    const uint8_t* nibbles = nullptr;
    const void* scales = nullptr;
    const float* zeros = nullptr;
};

// The split-K plan of a GEMM of `tiles` pair tiles on `max_pairs` co-resident pairs: when the
// last wave leaves at least half of the pairs idle, its tiles are cut into `split` K-parts
// (at most 8, weight-stage aligned) so that it fills them.  Every tail unit then lands in
// the last round of the round-robin over the pairs (full_tiles is a multiple of the pairs,
// or there are no full tiles and one unit per pair), which the epilogue relies on: a tail
// unit is its pair's last, so its activation stages are free for summing the parts.
struct SplitPlan {
    int full_tiles, split, units;
    int64_t partial_floats, flags;
};
static SplitPlan tc_split_plan(int64_t tiles, int max_pairs, int n_kw, int bn) {
    SplitPlan sp{static_cast<int>(tiles), 1, static_cast<int>(tiles), 0, 0};
    const int64_t full = (tiles / max_pairs) * max_pairs, tail = tiles - full;
    if (tail == 0) return sp;
    // at most 8 parts (4 for tiles of 64 or 128 tokens, whose last part sums larger blocks:
    // 2048 x 4096 at M = 128, 8 tiles, took 23.2 us in 4 parts against 29.1 in 8) of at
    // least two weight stages each
    const int max_split = bn >= 64 ? 4 : 8;
    const int split = static_cast<int>(std::min<int64_t>(std::min<int64_t>(max_pairs / tail, max_split), n_kw / 2));
    if (split < 2) return sp;
    sp.full_tiles = static_cast<int>(full);
    sp.split = split;
    sp.units = static_cast<int>(full + tail * split);
    sp.partial_floats = tail * (split - 1) * 2 * bn * tc::kRowsCta;
    sp.flags = tail * 2 * 4;
    return sp;
}

// The staging pass and the GEMM with BN-token tiles over the work units of `sp`, with `xp`
// (M * K fp16) as the staging buffer and `partial` / `flags` as the split-K scratch.
template <bool ASYM, bool EXACT, int BN>
static int tc_launch(const GemmArgs& a, const TcWeights& wt, void* xp, const SplitPlan& sp, float* partial,
                     uint32_t* flags, int max_pairs, int tiles_n, int64_t tiles) {
    const int64_t G = static_cast<int64_t>(a.K / 32);
    const int64_t nblocks = static_cast<int64_t>(a.x_split ? a.M / 2 : a.M) * G;   // 32-blocks of x
    const unsigned grid_x = static_cast<unsigned>(ceil_div(nblocks, 256));
    constexpr int perm = ASYM ? tc::kPermAsym : tc::kPermQ4B32;
    const PeerGather pg = a.pg ? *a.pg : PeerGather();
    const int n_flags = static_cast<int>(sp.flags);
    if (a.x_split)
        tc::stage_x_kernel<true, perm, true><<<grid_x, 256, 0, a.stream>>>(a.x, static_cast<uint4*>(xp), nblocks, pg,
                                                                           flags, n_flags, G);
    else if (a.x_dtype == BYBYCU_DT_F32)
        tc::stage_x_kernel<true, perm><<<grid_x, 256, 0, a.stream>>>(a.x, static_cast<uint4*>(xp), nblocks, pg, flags,
                                                                     n_flags);
    else
        tc::stage_x_kernel<false, perm><<<grid_x, 256, 0, a.stream>>>(a.x, static_cast<uint4*>(xp), nblocks, pg,
                                                                      flags, n_flags);
    BYBYCU_LAUNCH_CHECK("stage_x_kernel");

    tc::Maps maps;
    memset(&maps, 0, sizeof maps);
    int rc = encode_tensor_map_2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xp, a.K, a.M,
                                  static_cast<uint64_t>(a.K) * 2, tc::kXSub, tc::TokTile<BN>::kTokCta,
                                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (!rc)
        rc = encode_tensor_map_2d(&maps.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, wt.nibbles, a.K / 2, a.N, a.K / 2,
                                  tc::kWK / 2, tc::kRowsCta, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (!rc)
        rc = encode_tensor_map_2d(&maps.s, ASYM ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                                  wt.scales, G, a.N, G * (ASYM ? 4 : 2), tc::kWK / 32, tc::kRowsCta,
                                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    if (!rc && ASYM)
        rc = encode_tensor_map_2d(&maps.z, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, wt.zeros, G, a.N, G * 4, tc::kWK / 32,
                                  tc::kRowsCta, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    if (rc) return rc;
    tc::Params p;
    p.M = a.M;
    p.K = a.K;
    p.N = a.N;
    p.tiles_n = tiles_n;
    p.tiles = static_cast<int>(tiles);
    p.out = a.out;
    p.out_ld = a.out_ld;
    p.out_col0 = a.out_col0;
    p.out_bf16 = a.out_dtype == BYBYCU_DT_BF16;
    p.x_split = a.x_split ? 1 : 0;
    if (a.pg) {
        if (p.out_bf16) return set_error(BYBYCU_ERR_ARGS, "tensor-core all-gather: the gathered output is fp32");
        p.pg = *a.pg;
    }
    p.units = sp.units;
    p.full_tiles = sp.full_tiles;
    p.split = sp.split;
    p.partial = partial;
    p.flags = flags;
    const int pairs = std::min(sp.units, max_pairs);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // the GEMM's prologue, weight loads and first dequantization overlap the staging pass;
    // only its activation producer waits for that pass (griddepcontrol.wait)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::Cfg<ASYM, EXACT, BN>::kSmemBytes;
    cfg.stream = a.stream;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    BYBYCU_CUDA_TRY(cudaLaunchKernelEx(&cfg, tc::gemm_kernel<ASYM, EXACT, BN>, maps, p));
    return BYBYCU_OK;
}

// Where a split-K tail keeps its partial sums and counters: the stream-ordered pool, or a
// fixed region (`bytes` at `ptr`; a plan that needs more runs whole tiles).
struct SplitScratch {
    bool pool = false;
    void* ptr = nullptr;
    size_t bytes = 0;
};

// tc_launch with a split-K plan: a tail that leaves pairs idle is split when `ss` offers
// room for its partial sums and counters.
template <bool ASYM, bool EXACT, int BN>
static int tc_run(const GemmArgs& a, const TcWeights& wt, void* xp, const SplitScratch& ss) {
    DeviceInfo info;
    int max_pairs = 0;
    if (int rc = tc_setup<ASYM, EXACT, BN>(&info, &max_pairs)) return rc;
    const int tiles_n = static_cast<int>(ceil_div(a.N, tc::kRowsPair));
    const int64_t tiles = static_cast<int64_t>(tiles_n) * ceil_div(a.M, BN);
    if (tiles > (1 << 30)) return set_error(BYBYCU_ERR_SHAPE, "tensor-core route: too many tiles (M=%d N=%d)", a.M, a.N);
    const SplitPlan whole{static_cast<int>(tiles), 1, static_cast<int>(tiles), 0, 0};
    SplitPlan sp = tc_split_plan(tiles, max_pairs, a.K / tc::kWK, BN);
    const size_t sp_bytes = static_cast<size_t>(sp.partial_floats + sp.flags) * 4;
    if (sp.split > 1 && !ss.pool && sp_bytes > ss.bytes) sp = whole;
    if (sp.split == 1) return tc_launch<ASYM, EXACT, BN>(a, wt, xp, sp, nullptr, nullptr, max_pairs, tiles_n, tiles);
    if (!ss.pool) {
        float* partial = static_cast<float*>(ss.ptr);
        return tc_launch<ASYM, EXACT, BN>(a, wt, xp, sp, partial, reinterpret_cast<uint32_t*>(partial + sp.partial_floats),
                                          max_pairs, tiles_n, tiles);
    }
    cudaMemPool_t pool = nullptr;
    if (int rc = scratch_pool(info.device, &pool)) return rc;
    void* part = nullptr;
    BYBYCU_CUDA_TRY(cudaMallocFromPoolAsync(&part, sp_bytes, pool, a.stream));
    float* partial = static_cast<float*>(part);
    const int rc = tc_launch<ASYM, EXACT, BN>(a, wt, xp, sp, partial,
                                              reinterpret_cast<uint32_t*>(partial + sp.partial_floats), max_pairs,
                                              tiles_n, tiles);
    const cudaError_t fe = cudaFreeAsync(part, a.stream);
    if (rc) return rc;
    if (fe != cudaSuccess) return cuda_fail(fe, "cudaFreeAsync(tc split-K scratch)");
    return BYBYCU_OK;
}

template <bool ASYM, bool EXACT>
static int tc_run_rows(const GemmArgs& a, const TcWeights& wt, void* xp, const SplitScratch& ss) {
    switch (tc_token_tile(a.M)) {
        case 16: return tc_run<ASYM, EXACT, 16>(a, wt, xp, ss);
        case 32: return tc_run<ASYM, EXACT, 32>(a, wt, xp, ss);
        case 64: return tc_run<ASYM, EXACT, 64>(a, wt, xp, ss);
        default: return tc_run<ASYM, EXACT, 128>(a, wt, xp, ss);
    }
}

// Stages through stream-ordered pool scratch and runs the GEMM.
template <bool ASYM, bool EXACT>
static int tc_pooled(const GemmArgs& a, const TcWeights& wt) {
    DeviceInfo info;
    if (int rc = current_device_info(&info)) return rc;
    const size_t xp_bytes = static_cast<size_t>(a.M) * a.K * 2;
    void* xp = nullptr;
    cudaMemPool_t pool = nullptr;
    if (int rc = scratch_pool(info.device, &pool)) return rc;
    BYBYCU_CUDA_TRY(cudaMallocFromPoolAsync(&xp, xp_bytes, pool, a.stream));
    SplitScratch ss;
    ss.pool = true;
    const int rc = tc_run_rows<ASYM, EXACT>(a, wt, xp, ss);
    const cudaError_t fe = cudaFreeAsync(xp, a.stream);
    if (rc) return rc;
    if (fe != cudaSuccess) return cuda_fail(fe, "cudaFreeAsync(tc scratch)");
    return BYBYCU_OK;
}

// Q4B32 on the tensor cores: exact weight terms (route TC), or each weight rounded once to
// fp16 (route TC_FP16W, the reference's cooperative-matrix lowering).
// fp32 activations enter the tensor cores as two fp16 rows each (x_split), so that they keep
// ~22 significant bits instead of fp16's 11.
static GemmArgs tc_split_rows(const GemmArgs& a) {
    GemmArgs b = a;
    if (a.x_dtype == BYBYCU_DT_F32 && a.M <= (1 << 29)) {
        b.M = 2 * a.M;
        b.x_split = true;
    }
    return b;
}

int launch_tc(const GemmArgs& a, bool fp16_weights) {
    if (a.fmt == BYBYCU_FMT_F16) return launch_tc_f16(a);
    if (int rc = tc_check(a)) return rc;
    TcWeights wt;
    wt.nibbles = a.packed;
    wt.scales = a.packed + a.scale_base;
    const GemmArgs b = tc_split_rows(a);
    return fp16_weights ? tc_pooled<false, false>(b, wt) : tc_pooled<false, true>(b, wt);
}

bool tc_asym_supports(int M, int K, int N, int group, int n_groups, const void* x, const void* wq, const void* scales,
                      const void* zeros, const void* out) {
    if (group != 32 || n_groups != K / 32 || K < tc::kWK || K % tc::kWK != 0 || M < 1 || N < 1) return false;
    for (const void* ptr : {x, wq, scales, zeros})
        if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(out) % 4 != 0) return false;
    DeviceInfo info;
    if (current_device_info(&info) != BYBYCU_OK) return false;
    return info.cc_major == 10 && info.max_smem_optin >= static_cast<int>(tc::kSmemBytes);
}

int launch_tc_asym(int M, int K, int N, const float* x, const uint8_t* wq, const float* scales, const float* zeros,
                   float* out, cudaStream_t stream) {
    if (!tc_asym_supports(M, K, N, 32, K / 32, x, wq, scales, zeros, out))
        return set_error(BYBYCU_ERR_SHAPE, "matmul_q4 tensor-core route needs group 32, K %% 256 == 0 and 16-byte "
                                           "aligned slots (M=%d K=%d N=%d)", M, K, N);
    GemmArgs a;
    a.M = M; a.K = K; a.N = N;
    a.x = x; a.x_dtype = BYBYCU_DT_F32;
    a.out = out; a.out_dtype = BYBYCU_DT_F32;
    a.out_ld = N; a.out_col0 = 0;
    a.stream = stream;
    TcWeights wt;
    wt.nibbles = wq;
    wt.scales = scales;
    wt.zeros = zeros;
    return tc_pooled<true, false>(a, wt);
}

// ---------------------------------------------------------------------------------------
// The same GEMM with staging scratch that is never allocated at call time: a fixed array in
// the module's device memory.  With lazy module loading (the CUDA 12 default) a module gets
// its device memory - code and this array - when it is first used on a device, so
// tc_static_scratch_load() below, called by bybycu_init, uses it there: after that no call
// of this route allocates anything.
// ---------------------------------------------------------------------------------------
constexpr size_t kStaticScratchBytes = size_t(32) << 20;   // M * K <= 16 Mi activations
__device__ __align__(256) uint8_t g_tc_static_scratch[kStaticScratchBytes];

// The array's address in the current device's context.  Looked up on every call (cheap once
// the module is loaded), so a context created again after a device reset gets its own
// address, never a stale one.
static int static_scratch(void** ptr) {
    void* p = nullptr;
    BYBYCU_CUDA_TRY(cudaGetSymbolAddress(&p, g_tc_static_scratch));
    *ptr = p;
    return BYBYCU_OK;
}

// Loads, on the current device, the module's array and every kernel the static-scratch route
// launches, and sets the GEMM's attributes: the allocations of lazy loading happen here.
// Whether the sharded call stores to the peers from the GEMM's own epilogue: when some CTA
// pair has a second tile, so that the peer stores of one tile overlap the MMAs of the next,
// or when tiles are small (at most 32 tokens: 32 KB per tile to each peer).  With one round
// of large tiles every peer store sits in the launch's tail on the few SMs that finish tiles
// (2048 x 4096 at M = 128 over two GPUs: 48.5 us fused, 32.9 us with the copy kernel, which
// spreads the stores over every SM); at M = 16 the fused form wins (2048 x 11008: 22.9
// against 26.2 us).
bool tc_fuse_gather(const GemmArgs& a) {
    if (a.M <= 32) return true;
    DeviceInfo info;
    int max_pairs = 0;
    int rc = 0;
    switch (tc_token_tile(a.M)) {
        case 16: rc = tc_setup<false, true, 16>(&info, &max_pairs); break;
        case 32: rc = tc_setup<false, true, 32>(&info, &max_pairs); break;
        case 64: rc = tc_setup<false, true, 64>(&info, &max_pairs); break;
        default: rc = tc_setup<false, true, 128>(&info, &max_pairs); break;
    }
    if (rc || max_pairs <= 0) return false;
    const int64_t tiles = ceil_div(a.N, tc::kRowsPair) * ceil_div(a.M, tc_token_tile(a.M));
    return tiles > max_pairs;
}

int tc_static_scratch_load() {
    DeviceInfo info;
    if (int rc = current_device_info(&info)) return rc;
    if (info.cc_major != 10 || info.max_smem_optin < static_cast<int>(tc::kSmemBytes)) return BYBYCU_OK;
    void* p = nullptr;
    if (int rc = static_scratch(&p)) return rc;
    int max_pairs = 0;
    DeviceInfo d;
    if (int rc = tc_setup<false, true, 16>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<false, true, 32>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<false, true, 64>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<false, true, 128>(&d, &max_pairs)) return rc;
    // the pooled routes too, so that a first call may come inside a stream capture: the
    // scratch pool and every instantiation's attributes exist before it
    cudaMemPool_t pool = nullptr;
    if (int rc = scratch_pool(info.device, &pool)) return rc;
    if (int rc = tc_setup<false, false, 16>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<false, false, 32>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<false, false, 64>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<false, false, 128>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<true, false, 16>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<true, false, 32>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<true, false, 64>(&d, &max_pairs)) return rc;
    if (int rc = tc_setup<true, false, 128>(&d, &max_pairs)) return rc;
    cudaFuncAttributes fa;
    BYBYCU_CUDA_TRY(cudaFuncGetAttributes(&fa, tc::stage_x_kernel<false, tc::kPermQ4B32>));
    BYBYCU_CUDA_TRY(cudaFuncGetAttributes(&fa, tc::stage_x_kernel<true, tc::kPermQ4B32>));
    return BYBYCU_OK;
}

int launch_tc_static_scratch(const GemmArgs& a_in) {
    const int terms = a_in.x_dtype == BYBYCU_DT_F32 ? 2 : 1;   // fp32 rows stage as two fp16 rows
    const size_t need = static_cast<size_t>(a_in.M) * a_in.K * 2 * terms;
    if (need > kStaticScratchBytes)
        return set_error(BYBYCU_ERR_RANGE,
                         "static-scratch tensor-core GEMM stages M*K fp16 activations (two terms each for fp32 x) "
                         "in a fixed %zu MiB array: M=%d K=%d needs %zu bytes (at most M*K = %zu)",
                         kStaticScratchBytes >> 20, a_in.M, a_in.K, need, kStaticScratchBytes / 2 / terms);
    if (int rc = tc_check(a_in)) return rc;
    const GemmArgs a = tc_split_rows(a_in);
    void* xp = nullptr;
    if (int rc = static_scratch(&xp)) return rc;
    TcWeights wt;
    wt.nibbles = a.packed;
    wt.scales = a.packed + a.scale_base;
    // a split-K tail keeps its sums in the array's room past the activations when they fit
    // (the same plan, so the same sums, as the pooled route); otherwise whole tiles
    SplitScratch ss;
    const size_t used = (need + 255) / 256 * 256;
    ss.ptr = static_cast<uint8_t*>(xp) + used;
    ss.bytes = kStaticScratchBytes - used;
    return tc_run_rows<false, true>(a, wt, xp, ss);
}

}  // namespace bybycu
