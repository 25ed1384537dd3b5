// tcf16.cu - the prefill route of tile format 1 (fp16 weights W[N, K], row-major:
// buildF16TileGemmProgram, micro_kernel/session_vm.nim:400-416; the CPU VM's
// OP_TILE_LOAD_B_F16, backends/cpu/cpu_vm.c:550-581; on Vulkan, sessionF16GemmTile with
// tensorCore, gpubackend.nim:1475-1482) on the 5th-generation tensor cores.
//
// The weights need no dequantisation, so both MMA operands come straight from shared memory:
//   * CTA pairs (cta_group::2) persistent over 256-feature x 128-token tiles, as the Q4B32
//     prefill kernel of tc.cu; each CTA TMA-loads its own 128 weight rows (the pair's A is
//     M = 256 split across the two CTAs' shared memory) and 64 of the tile's 128 token rows;
//   * one stage is K = 128: A 128 rows x 256 B and x 64 rows x 256 B per CTA, two 128-byte
//     swizzled boxes each, four stages in flight;
//   * one thread of the even CTA issues eight 256 x 128 x 16 MMAs per stage into fp32
//     accumulators in both CTAs' tensor memory (two buffers), and the epilogue of tc.cu
//     drains them;
//   * the activations are staged to fp16 first (exact for bf16 inputs inside the fp16 range;
//     values outside it are reported as device error 7).
// Every wait is bounded; on a timeout the kernel records the error, drains and frees its
// tensor memory.
#include "kernels.h"

namespace bybycu {
namespace tc {

constexpr int kF16Stages = 4;
constexpr int kF16Threads = 256;   // 0 TMA, 1 MMA + TMEM, 2 relay (odd CTA), 3 idle, 4-7 epilogue
constexpr uint32_t kF16ABox = kRowsCta * kXSub * 2;            // 16 KiB: 128 rows x 64 K
constexpr uint32_t kF16AStage = 2 * kF16ABox;                  // 32 KiB
constexpr uint32_t kF16Stage = kF16AStage + kXStageBytes;      // + 16 KiB of activations
constexpr uint32_t kF16TmemCols = 2 * kAccCols;                // two accumulator buffers
// barriers: full, empty [stages]; d_full, d_empty [2]; done; then the TMEM slot and abort flag
constexpr uint32_t kF16OffBar = kF16Stages * kF16Stage;
constexpr uint32_t kF16NumBars = 2 * kF16Stages + 5;
constexpr uint32_t kF16OffTmemSlot = kF16OffBar + kF16NumBars * 8;
constexpr uint32_t kF16OffAbort = kF16OffTmemSlot + 4;
constexpr uint32_t kF16SmemBytes = kF16OffAbort + 4 + 1024;
static_assert(kF16SmemBytes > 116 * 1024 && kF16SmemBytes <= 227 * 1024, "one CTA per SM");

struct F16Maps {
    CUtensorMap x;   // fp16 [M, K], box 64 (K) x 64 (tokens), 128-byte swizzle
    CUtensorMap w;   // fp16 [N, K], box 64 (K) x 128 (rows), 128-byte swizzle
};

// One stage: eight 256 x 128 x 16 MMAs (A and B from shared memory) from one elected lane.
__device__ __forceinline__ void mma_pair_smem_stage(uint32_t d_tmem, const uint64_t (&a)[8], const uint64_t (&b)[8],
                                                    uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p, q;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %1, 0;\n\t"
        "setp.eq.b32 q, %1, %1;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %3, %4, %2, p;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %5, %6, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %7, %8, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %9, %10, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %11, %12, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %13, %14, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %15, %16, %2, q;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %17, %18, %2, q;\n\t}" ::"r"(d_tmem),
        "r"(accumulate), "r"(kIdesc), "l"(a[0]), "l"(b[0]), "l"(a[1]), "l"(b[1]), "l"(a[2]), "l"(b[2]), "l"(a[3]),
        "l"(b[3]), "l"(a[4]), "l"(b[4]), "l"(a[5]), "l"(b[5]), "l"(a[6]), "l"(b[6]), "l"(a[7]), "l"(b[7])
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_n(uint32_t slot_smem, uint32_t ncols) { tmem_alloc(slot_smem, ncols); }

__global__ void __launch_bounds__(kF16Threads, 1) gemm_f16_kernel(const __grid_constant__ F16Maps maps, const Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kF16OffBar);
    // full[s]: on rank 0 both CTAs' halves of stage s landed (its own TMA and the odd CTA's
    // relay); on rank 1 its own half landed.  empty[s]: the pair's MMAs finished with it.
    uint64_t* full = bars;
    uint64_t* empty = bars + kF16Stages;
    uint64_t* d_full = empty + kF16Stages;   // [2]
    uint64_t* d_empty = d_full + 2;          // [2] (rank 0) both epilogues read the buffer
    uint64_t* done_bar = d_full + 4;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + kF16OffTmemSlot);
    volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kF16OffAbort);

    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kF16Stages; ++i) {
            mbar_init(&full[i], leader ? 2 : 1);
            mbar_init(&empty[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&d_full[b], 1);
            mbar_init(&d_empty[b], 8);   // four epilogue warps in each CTA
        }
        mbar_init(done_bar, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc_n(smem_u32(const_cast<uint32_t*>(tmem_slot)), kF16TmemCols);
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int pair = static_cast<int>(blockIdx.x >> 1), pairs = static_cast<int>(gridDim.x >> 1);
    const int my_tiles = p.tiles > pair ? (p.tiles - 1 - pair) / pairs + 1 : 0;
    const int n_ks = p.K / kXK;

    if (warp == 0) {
        // ------------------------------------------------------------- TMA producer (both)
        if (lane == 0) {
            prefetch_tensormap(&maps.x);
            prefetch_tensormap(&maps.w);
            const uint64_t policy = l2_policy_evict_last();
            int issued = 0;
            for (int t = 0; t < my_tiles && !*s_abort; ++t) {
                const int tile = pair + t * pairs;
                const int row0 = (tile % p.tiles_n) * kRowsPair + static_cast<int>(rank) * kRowsCta;
                const int tok = (tile / p.tiles_n) * kBN + static_cast<int>(rank) * kTokCta;
                for (int ks = 0; ks < n_ks; ++ks) {
                    const int s = issued % kF16Stages, r = issued / kF16Stages;
                    if (r > 0 && !wait_bar(&empty[s], (r - 1) & 1, kDevErrEmptyWait)) {
                        *s_abort = 1;
                        break;
                    }
                    if (*s_abort) break;
                    uint8_t* st = smem + s * kF16Stage;
                    mbar_arrive_expect_tx(&full[s], kF16Stage);
                    tma_load_2d_hint(st, &maps.w, &full[s], ks * kXK, row0, policy);
                    tma_load_2d_hint(st + kF16ABox, &maps.w, &full[s], ks * kXK + kXSub, row0, policy);
                    if (issued == 0) pdl_wait();   // the staging pass that writes x has completed
                    tma_load_2d(st + kF16AStage, &maps.x, &full[s], ks * kXK, tok);
                    tma_load_2d(st + kF16AStage + kXSubBytes, &maps.x, &full[s], ks * kXK + kXSub, tok);
                    ++issued;
                }
            }
            // rank 1 waits for its own copies; rank 0 for the pair's MMAs to release the stages
            for (int it = issued > kF16Stages ? issued - kF16Stages : 0; it < issued; ++it) {
                const bool landed = leader ? wait_bar(&empty[it % kF16Stages], (it / kF16Stages) & 1, kDevErrDrainWait)
                                           : wait_bar(&full[it % kF16Stages], (it / kF16Stages) & 1, kDevErrDrainWait);
                if (!landed) break;
            }
        }
    } else if (warp == 2) {
        // --------------------------------- (odd CTA) tells rank 0 that its half has landed
        if (!leader && lane == 0) {
            const uint32_t lead_full = map_to_rank(full, 0);
            const int total = my_tiles * n_ks;
            for (int i = 0; i < total; ++i) {
                const int s = i % kF16Stages;
                if (!wait_bar(&full[s], (i / kF16Stages) & 1, kDevErrFullWait) || *s_abort) {
                    *s_abort = 1;
                    break;
                }
                mbar_arrive_cluster(lead_full + 8u * s);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------- MMA issuer (rank 0, whole warp)
        if (leader) {
            int consumed = 0;
            for (int t = 0; t < my_tiles && !*s_abort; ++t) {
                const int b = t & 1, u = t >> 1;
                if (u > 0 && !__all_sync(0xffffffffu, wait_bar(&d_empty[b], (u - 1) & 1, kDevErrMmaWait))) {
                    *s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + b * kAccCols;
                bool ok = true;
                for (int ks = 0; ks < n_ks; ++ks) {
                    const int s = consumed % kF16Stages, r = consumed / kF16Stages;
                    if (!__all_sync(0xffffffffu, wait_bar(&full[s], r & 1, kDevErrFullWait))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = base + s * kF16Stage;
                    const uint64_t adesc = sw128_desc(st), bdesc = sw128_desc(st + kF16AStage);
                    // 16-K steps advance 32 bytes inside a 128-byte swizzle row, then jump to
                    // the next 64-K box
                    uint64_t ak[8], bk[8];
#pragma unroll
                    for (int k16 = 0; k16 < kXK / 16; ++k16) {
                        ak[k16] = adesc + static_cast<uint64_t>((k16 >> 2) * (kF16ABox >> 4) + (k16 & 3) * 2);
                        bk[k16] = bdesc + static_cast<uint64_t>((k16 >> 2) * (kXSubBytes >> 4) + (k16 & 3) * 2);
                    }
                    mma_pair_smem_stage(d_tmem, ak, bk, ks != 0);
                    tc_commit_pair(&empty[s]);   // both CTAs may refill the stage once these MMAs are done
                    ++consumed;
                }
                if (!ok) {
                    *s_abort = 1;
                    break;
                }
                tc_commit_pair(&d_full[b]);
            }
            tc_commit_local(done_bar);
            __all_sync(0xffffffffu, wait_bar(done_bar, 0, kDevErrMmaWait));
        }
    } else if (warp >= 4) {
        epilogue_tiles(p, tmem, d_full, d_empty, s_abort, my_tiles, pair, pairs, rank, warp & 3, lane);
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();   // neither CTA frees its tensor memory while the pair may still use it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kF16TmemCols);
    }
}

}  // namespace tc

bool tc_f16_supports(const GemmArgs& a) {
    if (a.fmt != BYBYCU_FMT_F16 || a.K < tc::kXK || a.K % tc::kXK != 0 || a.M < 1 || a.N < 1) return false;
    if (a.x_dtype != BYBYCU_DT_BF16 && a.x_dtype != BYBYCU_DT_F32) return false;
    if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || reinterpret_cast<uintptr_t>(a.packed) % 16 != 0) return false;
    const size_t esz = a.out_dtype == BYBYCU_DT_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(a.out) % esz != 0) return false;
    DeviceInfo info;
    if (current_device_info(&info) != BYBYCU_OK) return false;
    return info.cc_major == 10 && info.max_smem_optin >= static_cast<int>(tc::kF16SmemBytes);
}

int launch_tc_f16(const GemmArgs& a) {
    if (!tc_f16_supports(a))
        return set_error(BYBYCU_ERR_SHAPE, "format-1 tensor-core route needs K %% 128 == 0 and 16-byte aligned x and "
                                           "weights (M=%d K=%d N=%d)", a.M, a.K, a.N);
    DeviceInfo info;
    if (int rc = current_device_info(&info)) return rc;
    static std::once_flag once[64];
    static cudaError_t prep_rc[64];
    static int max_pairs[64];
    const int dev = info.device;
    if (dev < 0 || dev >= 64) return set_error(BYBYCU_ERR_ARGS, "device %d out of range", dev);
    std::call_once(once[dev], [&] {
        prep_rc[dev] = cudaFuncSetAttribute(tc::gemm_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(tc::kF16SmemBytes));
        if (prep_rc[dev] != cudaSuccess) return;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * (info.sm_count / 2));
        cfg.blockDim = dim3(tc::kF16Threads);
        cfg.dynamicSmemBytes = tc::kF16SmemBytes;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        prep_rc[dev] = cudaOccupancyMaxActiveClusters(&max_pairs[dev], tc::gemm_f16_kernel, &cfg);
    });
    if (prep_rc[dev] != cudaSuccess) return cuda_fail(prep_rc[dev], "format-1 tensor-core GEMM set-up");
    if (max_pairs[dev] < 1) return set_error(BYBYCU_ERR_DEVICE, "no CTA pair of the format-1 GEMM fits on the device");

    // activations -> fp16 in stream-ordered scratch, in K order
    const size_t xp_bytes = static_cast<size_t>(a.M) * a.K * 2;
    void* xp = nullptr;
    cudaMemPool_t pool = nullptr;
    if (int rc = scratch_pool(info.device, &pool)) return rc;
    BYBYCU_CUDA_TRY(cudaMallocFromPoolAsync(&xp, xp_bytes, pool, a.stream));
    int rc = BYBYCU_OK;
    {
        const int64_t nblocks = static_cast<int64_t>(a.M) * (a.K / 32);
        const unsigned grid_x = static_cast<unsigned>(ceil_div(nblocks, 256));
        if (a.x_dtype == BYBYCU_DT_F32)
            tc::stage_x_kernel<true, tc::kPermNone><<<grid_x, 256, 0, a.stream>>>(a.x, static_cast<uint4*>(xp), nblocks, PeerGather());
        else
            tc::stage_x_kernel<false, tc::kPermNone><<<grid_x, 256, 0, a.stream>>>(a.x, static_cast<uint4*>(xp), nblocks, PeerGather());
        const cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) rc = cuda_fail(le, "stage_x_kernel");
    }
    tc::F16Maps maps;
    memset(&maps, 0, sizeof maps);
    if (!rc)
        rc = encode_tensor_map_2d(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xp, a.K, a.M, static_cast<uint64_t>(a.K) * 2,
                                  tc::kXSub, tc::kTokCta, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (!rc)
        rc = encode_tensor_map_2d(&maps.w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.packed, a.K, a.N,
                                  static_cast<uint64_t>(a.K) * 2, tc::kXSub, tc::kRowsCta, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    tc::Params p;
    p.M = a.M;
    p.K = a.K;
    p.N = a.N;
    p.tiles_n = static_cast<int>(ceil_div(a.N, tc::kRowsPair));
    const int64_t tiles = static_cast<int64_t>(p.tiles_n) * ceil_div(a.M, tc::kBN);
    if (!rc && tiles > (1 << 30)) rc = set_error(BYBYCU_ERR_SHAPE, "format-1 tensor-core route: too many tiles");
    p.tiles = static_cast<int>(tiles);
    p.out = a.out;
    p.out_ld = a.out_ld;
    p.out_col0 = a.out_col0;
    p.out_bf16 = a.out_dtype == BYBYCU_DT_BF16;
    if (!rc) {
        const int pairs = static_cast<int>(std::min<int64_t>(tiles, max_pairs[dev]));
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = dim3(2 * pairs);
        cfg.blockDim = dim3(tc::kF16Threads);
        cfg.dynamicSmemBytes = tc::kF16SmemBytes;
        cfg.stream = a.stream;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        const cudaError_t le = cudaLaunchKernelEx(&cfg, tc::gemm_f16_kernel, maps, p);
        if (le != cudaSuccess) rc = cuda_fail(le, "gemm_f16_kernel");
    }
    const cudaError_t fe = cudaFreeAsync(xp, a.stream);
    if (rc) return rc;
    if (fe != cudaSuccess) return cuda_fail(fe, "cudaFreeAsync(format-1 scratch)");
    return BYBYCU_OK;
}

}  // namespace bybycu
