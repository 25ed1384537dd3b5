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
    // Launch knobs of a tuned plan (tune.cu); the defaults leave each route's own choice.
    // variant: the M = 1 Q4B32 GEMV's operand form (kM1*), or the format-1 GEMV's CTAs per SM.
    // stages: the ring depth of the streamed weights (GEMV routes).
    int variant = -1;
    int stages = 0;
    // Tensor-core route, fp32 x: each activation row is staged as two fp16 rows, x_hi =
    // RNE16(x) and x_lo = RNE16(x - x_hi), and the GEMM runs over 2 * M token rows (M here
    // counts those), adding each row pair in its epilogue.
    bool x_split = false;
    // Set by the sharded entry points: the kernel also stores its slice into every rank's
    // output (the tensor-core route; the GEMV takes it as launch_gemv's argument).
    const struct PeerGather* pg = nullptr;
};

// Ranks of a column-sharded GEMM whose output slices are gathered over NVLink peer
// pointers.  sig[r] is rank r's signal array: kMaxRanks counters (one per source rank), the
// device-side epoch, and this rank's CTA completion counter.
constexpr int kMaxRanks = 8;
struct PeerGather {
    int world = 1, rank = 0;
    float* out[kMaxRanks] = {};      // every rank's output buffer as mapped here (out[rank] = local)
    uint32_t* sig[kMaxRanks] = {};   // every rank's signal array as mapped here
    uint32_t epoch = 0;              // 0: the epoch lives on the device (graph-capturable)
    // 1 (split phase): a launch signals its epoch without waiting for the other ranks; the next
    // split launch waits for every rank's previous epoch before it reads its input or stores
    // to a peer, and bybycu_allgather_wait completes the last one
    int split = 0;
};

// The fused all-gather: one output value to every other rank's buffer (plain NVLink stores).
__device__ __forceinline__ void store_to_peers(const PeerGather& pg, int64_t oi, float v) {
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
        if (r < pg.world && r != pg.rank) pg.out[r][oi] = v;
}

// Bounded wait (one thread) until every rank's counter in this rank's signal array reached
// `target`.  Acquire loads at system scope: what the ranks stored before their signals is
// visible after it.  False (device error recorded) when the wait ran out.
__device__ __forceinline__ bool peer_wait_epoch(const PeerGather& pg, uint32_t target) {
    const uint32_t* mine = pg.sig[pg.rank];
    for (int r = 0; r < pg.world; ++r) {
        const uint64_t t0 = globaltimer_ns();
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + r) : "memory");
            if (static_cast<int32_t>(v - target) >= 0) break;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                record_device_error(kDevErrPeerWait);
                return false;
            }
        }
    }
    return true;
}

// The epoch the previous launch of this rank signalled (device-side epochs), or epoch - 1.
__device__ __forceinline__ uint32_t peer_previous_epoch(const PeerGather& pg) {
    return pg.epoch ? pg.epoch - 1 : *reinterpret_cast<volatile const uint32_t*>(pg.sig[pg.rank] + kMaxRanks);
}

// Split phase, by one thread before anything of this launch reads its input or stores to a
// peer: every rank has finished the previous launch (its stores into this rank's buffers
// landed, and whatever its stream ran before that launch - the readers of the buffer this
// launch overwrites - is done).  Called after griddepcontrol.wait.
__device__ __forceinline__ bool peer_gather_wait_previous(const PeerGather& pg) {
    if (pg.world <= 1 || !pg.split) return true;
    return peer_wait_epoch(pg, peer_previous_epoch(pg));
}

// Called by one thread of every CTA after all of the CTA's output stores (local and to the
// peers).  The last CTA of the grid raises this rank's counter in every rank's signal array
// and waits, bounded, until every rank's counter reached this epoch.  Returns false when the
// wait ran out (the error is recorded in the device error word).
__device__ __forceinline__ bool peer_gather_finish(const PeerGather& pg) {
    // The CTA's completion count is an acq_rel atomic at GPU scope: a release of every store
    // this CTA made (the caller's barrier makes the other threads' stores this thread's), and,
    // for the last CTA, an acquire of every other CTA's.  The last CTA's system-scope release
    // fence then carries all of those stores before its signals, to the peers' acquire loads.
    uint32_t* mine = pg.sig[pg.rank];
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(mine + kMaxRanks + 1) : "memory");
    if (prev != gridDim.x * gridDim.y * gridDim.z - 1) return true;
    mine[kMaxRanks + 1] = 0;   // every CTA of this launch has counted
    // one system-scope release fence covers the signals to every rank
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < pg.world; ++r)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(pg.sig[r] + pg.rank) : "memory");
    const uint32_t target = pg.epoch ? pg.epoch : mine[kMaxRanks] + 1;
    if (pg.split) {   // the next launch (or bybycu_allgather_wait) waits for the ranks
        if (!pg.epoch) mine[kMaxRanks] = target;
        return true;
    }
    const bool ok = peer_wait_epoch(pg, target);
    if (!pg.epoch) mine[kMaxRanks] = target;
    return ok;
}

// CUDA-core FP32 route: every format, every K % 32 == 0 shape.
int launch_simt(const GemmArgs& a);
// Decode GEMV route (format 2, M <= 32 - one launch per 16 rows): TMA-streamed weights, s8 or
// bf16 mma.sync reductions with exact per-block fp32 scaling.
constexpr int kGemvMaxRows = 32;
bool gemv_supports(const GemmArgs& a);
// Format 1 (fp16 weights) decode GEMV, M <= 8: 16-byte weight streams, fp32 FMAs.
bool f16_gemv_supports(const GemmArgs& a);
int launch_f16_gemv(const GemmArgs& a);
int launch_gemv(const GemmArgs& a, const PeerGather* pg = nullptr);
// Prefill GEMM route: tcgen05 MMAs from shared-memory fp16 tiles, fp32 accumulators in TMEM
// (format 2 dequantised into tensor memory; format 1 straight from shared memory).
bool tc_supports(const GemmArgs& a);
int launch_tc(const GemmArgs& a, bool fp16_weights = false);
bool tc_f16_supports(const GemmArgs& a);
int launch_tc_f16(const GemmArgs& a);
// The same route staging its activations in a fixed module array instead of pool memory.
int launch_tc_static_scratch(const GemmArgs& a);
// Loads that route's module array and kernels on the current device (bybycu_init).
int tc_static_scratch_load();
// Whether a sharded tensor-core call (route TC, Q4B32) stores to the peers from its epilogue.
bool tc_fuse_gather(const GemmArgs& a);
// The asymmetric-Q4 form of the tensor-core route (matmul_q4 prefill): fp32 x [M, K],
// interleaved nibbles [N, K/2], fp32 scales and zero points [N, K/32], fp32 out [M, N].
bool tc_asym_supports(int M, int K, int N, int group, int n_groups, const void* x, const void* wq, const void* scales,
                      const void* zeros, const void* out);
int launch_tc_asym(int M, int K, int N, const float* x, const uint8_t* wq, const float* scales, const float* zeros,
                   float* out, cudaStream_t stream);

int launch_dequant(int fmt, int K, int N, const uint8_t* packed, int64_t scale_base,
                   const float* lut, float* w, cudaStream_t stream);

// Host -> device copy of a pageable (e.g. file-mapped) range through the staging engine of
// ingest.cu; synchronous.
int upload_host_range(void* dst, const void* src, int64_t bytes);

// Tuned plans (tune.cu).  When the caller asked for the automatic route and a plan was
// prepared for the shape on this device, the plan's route and knobs replace the built-in
// choice - if that route can run these exact arguments; otherwise nothing changes.
void apply_tile_gemm_plan(GemmArgs* a, int* route);
void apply_q4_plan(int M, int K, int N, int group, int groups, bool fast, bool tc, int* route, int* stages);

}  // namespace bybycu
