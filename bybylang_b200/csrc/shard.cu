// shard.cu - column sharding of the tile GEMM over GPUs.
//
// The split is distributed.nim's partition (distributed.nim:109-135): largest remainder
// over equal weights, computed in float64 exactly as the reference does, taken over blocks
// of `align` columns.  The exchange is device-side: each rank computes its column slice and
// stores it straight into every peer's output over NVLink (peer pointers) - from the GEMV's
// own epilogue on the decode route, from a copy kernel after the other routes.  The last CTA
// of that kernel raises this rank's counter in every rank's signal array and waits, bounded,
// for every rank's counter of this epoch, so the launch completes only with the whole output
// gathered.  No collective library is on the data path and no load reads another GPU's
// memory.
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "kernels.h"

namespace bybycu {

int check_tile_gemm(int fmt, int M, int K, int N, int64_t x_len, int64_t packed_len, int64_t scale_base,
                    int64_t lut_len, int64_t lut_base, int64_t out_len);
int choose_route(const GemmArgs& a, int requested, int* route);
int run_gemm(const GemmArgs& a, int route);

namespace {

constexpr int kExchangeCtas = 148;   // one per SM: enough stores in flight to fill NVLink

// Largest-remainder partition of `length` items over `world` equal weights
// (distributed.nim:109-135): floor of length * (1 / world), then one more to the largest
// remainders, first index first on ties.
std::vector<int> partition_equal(int length, int world) {
    std::vector<int> out(world, 0);
    std::vector<double> rem(world, 0.0);
    const double total = static_cast<double>(world);
    int assigned = 0;
    for (int i = 0; i < world; ++i) {
        const double exact = static_cast<double>(length) * (1.0 / total);
        out[i] = static_cast<int>(std::floor(exact));
        rem[i] = exact - static_cast<double>(out[i]);
        assigned += out[i];
    }
    while (assigned < length) {
        int best = -1;
        for (int i = 0; i < world; ++i)
            if (best < 0 || rem[i] > rem[best]) best = i;
        if (best < 0) break;
        ++out[best];
        rem[best] = -1.0;
        ++assigned;
    }
    return out;
}

// Copies out[:, n0:n1) of this rank into every other rank's out; the last CTA then signals
// the ranks and waits for theirs (peer_gather_finish).  Used after the routes that do not
// store to the peers themselves.
__global__ void __launch_bounds__(256) exchange_kernel(const float* __restrict__ out, int M, int N, int n0, int n1,
                                                       const PeerGather pg) {
    if (pg.split) {   // every rank done with the previous launch before anything goes to a peer
        if (threadIdx.x == 0) peer_gather_wait_previous(pg);
        __syncthreads();
    }
    const int cols = n1 - n0;
    const int64_t total = static_cast<int64_t>(M) * cols;
    const bool vec = ((n0 | cols | N) & 3) == 0;
    if (vec) {
        const int cols4 = cols / 4;
        const int64_t total4 = static_cast<int64_t>(M) * cols4;
        for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total4;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            const int64_t m = i / cols4;
            const int64_t c = (i % cols4) * 4;
            const int64_t off = m * N + n0 + c;
            const float4 v = *reinterpret_cast<const float4*>(out + off);
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r)
                if (r < pg.world && r != pg.rank) *reinterpret_cast<float4*>(pg.out[r] + off) = v;
        }
    } else {
        for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            const int64_t m = i / cols;
            const int64_t off = m * N + n0 + (i % cols);
            const float v = out[off];
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r)
                if (r < pg.world && r != pg.rank) pg.out[r][off] = v;
        }
    }
    __syncthreads();   // every thread's stores before thread 0's release (peer_gather_finish)
    if (threadIdx.x == 0) peer_gather_finish(pg);
}

// One thread waits until every rank reached an epoch: the previous one (`previous`, before a
// split launch that reads its input through another route), or the last one this rank
// signalled (bybycu_allgather_wait).
__global__ void allgather_wait_kernel(const PeerGather pg, int previous) {
    if (threadIdx.x != 0) return;
    const uint32_t last = pg.epoch ? pg.epoch
                                   : *reinterpret_cast<volatile const uint32_t*>(pg.sig[pg.rank] + kMaxRanks);
    peer_wait_epoch(pg, previous ? peer_previous_epoch(pg) : last);
}

int make_peer_gather(void* const* peer_out, uint32_t* const* peer_signal, int world, int rank, uint32_t epoch,
                     int split, PeerGather* pg) {
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || !peer_signal)
        return set_error(BYBYCU_ERR_ARGS, "all-gather: bad arguments");
    pg->world = world;
    pg->rank = rank;
    pg->epoch = epoch;
    pg->split = split;
    for (int r = 0; r < world; ++r) {
        if ((peer_out && !peer_out[r]) || !peer_signal[r])
            return set_error(BYBYCU_ERR_ARGS, "all-gather: peer %d missing", r);
        pg->out[r] = peer_out ? static_cast<float*>(peer_out[r]) : nullptr;
        pg->sig[r] = peer_signal[r];
    }
    return BYBYCU_OK;
}

// Peer allocations mapped into this process, shared by every pointer inside them.
struct IpcMapping {
    uint8_t handle[64];
    void* base;
    int refs;
};
std::mutex g_ipc_mu;
std::vector<IpcMapping> g_ipc;

// The allocation that contains dptr (cuMemGetAddressRange through the runtime's driver
// entry point; no libcuda link).
int allocation_range(const void* dptr, void** base, size_t* size) {
    using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static RangeFn fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        BYBYCU_CUDA_TRY(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) return set_error(BYBYCU_ERR_CUDA, "cuMemGetAddressRange is not available");
        fn = reinterpret_cast<RangeFn>(p);
    }
    CUdeviceptr b = 0;
    const CUresult r = fn(&b, size, reinterpret_cast<CUdeviceptr>(dptr));
    if (r != CUDA_SUCCESS) return set_error(BYBYCU_ERR_ARGS, "ipc handle: %p is not device memory (%d)", dptr, static_cast<int>(r));
    *base = reinterpret_cast<void*>(b);
    return BYBYCU_OK;
}

}  // namespace
}  // namespace bybycu

using namespace bybycu;

extern "C" {

int bybycu_ipc_handle(const void* dptr, uint8_t handle[64], int64_t* offset) {
    if (!dptr || !handle || !offset) return set_error(BYBYCU_ERR_ARGS, "ipc handle: bad arguments");
    // The handle names the whole allocation; a caching allocator hands out pointers inside
    // larger blocks, so the pointer's offset in its allocation travels with the handle.
    void* base = nullptr;
    size_t size = 0;
    if (int rc = allocation_range(dptr, &base, &size)) return rc;
    cudaIpcMemHandle_t h;
    BYBYCU_CUDA_TRY(cudaIpcGetMemHandle(&h, base));
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(handle, &h, 64);
    *offset = static_cast<const char*>(dptr) - static_cast<const char*>(base);
    return BYBYCU_OK;
}

int bybycu_ipc_open(const uint8_t handle[64], int64_t offset, void** dptr) {
    if (!dptr || !handle || offset < 0) return set_error(BYBYCU_ERR_ARGS, "ipc open: bad arguments");
    std::lock_guard<std::mutex> lock(g_ipc_mu);
    for (IpcMapping& m : g_ipc) {
        if (memcmp(m.handle, handle, 64) == 0) {   // the allocation is mapped already
            ++m.refs;
            *dptr = static_cast<char*>(m.base) + offset;
            return BYBYCU_OK;
        }
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    IpcMapping m;
    BYBYCU_CUDA_TRY(cudaIpcOpenMemHandle(&m.base, h, cudaIpcMemLazyEnablePeerAccess));
    memcpy(m.handle, handle, 64);
    m.refs = 1;
    g_ipc.push_back(m);
    *dptr = static_cast<char*>(m.base) + offset;
    return BYBYCU_OK;
}

int bybycu_ipc_close(void* dptr) {
    if (!dptr) return BYBYCU_OK;
    std::lock_guard<std::mutex> lock(g_ipc_mu);
    // the mapping whose base is the highest one not above dptr
    int best = -1;
    for (size_t i = 0; i < g_ipc.size(); ++i)
        if (g_ipc[i].base <= dptr && (best < 0 || g_ipc[i].base > g_ipc[best].base)) best = static_cast<int>(i);
    if (best < 0) return set_error(BYBYCU_ERR_ARGS, "ipc close: %p is not an opened peer buffer", dptr);
    if (--g_ipc[best].refs == 0) {
        void* base = g_ipc[best].base;
        g_ipc.erase(g_ipc.begin() + best);
        BYBYCU_CUDA_TRY(cudaIpcCloseMemHandle(base));
    }
    return BYBYCU_OK;
}

int bybycu_shard_range(int N, int world, int rank, int align, int* n0, int* n1) {
    if (!n0 || !n1 || N < 0 || world < 1 || rank < 0 || rank >= world || align < 1)
        return set_error(BYBYCU_ERR_ARGS, "shard range: bad arguments");
    const int blocks = static_cast<int>(ceil_div(N, align));
    const std::vector<int> parts = partition_equal(blocks, world);
    int start = 0;
    for (int r = 0; r < rank; ++r) start += parts[r];
    *n0 = std::min(N, start * align);
    *n1 = std::min(N, (start + parts[rank]) * align);
    return BYBYCU_OK;
}

static int tile_gemm_allgather(int fmt, int M, int K, int N, int n0, int n1, const void* x, int x_dtype,
                               const void* packed, int64_t packed_len, int64_t scale_base, const float* lut,
                               int64_t lut_len, int64_t lut_base, void* out, void* const* peer_out,
                               uint32_t* const* peer_signal, int world, int rank, uint32_t epoch, int split,
                               void* stream) {
    if (!peer_out || !out || !x || !packed) return set_error(BYBYCU_ERR_ARGS, "tile GEMM all-gather: bad arguments");
    if (n0 < 0 || n1 > N || n0 > n1) return set_error(BYBYCU_ERR_ARGS, "tile GEMM all-gather: bad column range");
    PeerGather pg;
    if (int rc = make_peer_gather(peer_out, peer_signal, world, rank, epoch, split, &pg)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int cols = n1 - n0;
    bool fused = false;
    if (cols > 0) {
        if (int rc = check_tile_gemm(fmt, M, K, cols, static_cast<int64_t>(M) * K, packed_len, scale_base, lut_len,
                                     lut_base, static_cast<int64_t>(M) * cols))
            return rc;
        GemmArgs a;
        a.fmt = fmt; a.M = M; a.K = K; a.N = cols;
        a.x = x; a.x_dtype = x_dtype;
        a.packed = static_cast<const uint8_t*>(packed); a.packed_len = packed_len; a.scale_base = scale_base;
        a.lut = lut ? lut + lut_base : nullptr;
        a.out = out; a.out_dtype = BYBYCU_DT_F32; a.out_ld = N; a.out_col0 = n0;
        a.stream = s;
        int route = 0;
        if (int rc = choose_route(a, BYBYCU_ROUTE_AUTO, &route)) return rc;
        if (route == BYBYCU_ROUTE_GEMV && fmt == BYBYCU_FMT_Q4B32 && M <= 16) {
            // the Q4B32 GEMV stores every value to the peers itself and ends with the signals
            // (in split phase its producer first waits for the ranks' previous launch)
            if (int rc = launch_gemv(a, &pg)) return rc;
            fused = true;
        } else if (route == BYBYCU_ROUTE_TC && fmt == BYBYCU_FMT_Q4B32 && tc_fuse_gather(a)) {
            // the tensor-core GEMM's epilogue does the same, tile by tile, so the transfer
            // overlaps the MMAs of the pair's next tiles
            a.pg = &pg;
            if (int rc = run_gemm(a, route)) return rc;
            fused = true;
        } else {
            if (split) {   // x may be the previous launch's gathered output: wait for it first
                allgather_wait_kernel<<<1, 32, 0, s>>>(pg, 1);
                BYBYCU_LAUNCH_CHECK("allgather_wait_kernel");
            }
            if (int rc = run_gemm(a, route)) return rc;
        }
    }
    if (!fused) {
        exchange_kernel<<<kExchangeCtas, 256, 0, s>>>(static_cast<const float*>(out), M, N, n0, n1, pg);
        BYBYCU_LAUNCH_CHECK("exchange_kernel");
    }
    return BYBYCU_OK;
}

int bybycu_tile_gemm_allgather(int fmt, int M, int K, int N, int n0, int n1, const void* x, int x_dtype,
                               const void* packed, int64_t packed_len, int64_t scale_base, const float* lut,
                               int64_t lut_len, int64_t lut_base, void* out, void* const* peer_out,
                               uint32_t* const* peer_signal, int world, int rank, uint32_t epoch, void* stream) {
    return tile_gemm_allgather(fmt, M, K, N, n0, n1, x, x_dtype, packed, packed_len, scale_base, lut, lut_len,
                               lut_base, out, peer_out, peer_signal, world, rank, epoch, 0, stream);
}

int bybycu_tile_gemm_allgather_split(int fmt, int M, int K, int N, int n0, int n1, const void* x, int x_dtype,
                                     const void* packed, int64_t packed_len, int64_t scale_base, const float* lut,
                                     int64_t lut_len, int64_t lut_base, void* out, void* const* peer_out,
                                     uint32_t* const* peer_signal, int world, int rank, uint32_t epoch,
                                     void* stream) {
    return tile_gemm_allgather(fmt, M, K, N, n0, n1, x, x_dtype, packed, packed_len, scale_base, lut, lut_len,
                               lut_base, out, peer_out, peer_signal, world, rank, epoch, 1, stream);
}

int bybycu_allgather_wait(uint32_t* const* peer_signal, int world, int rank, uint32_t epoch, void* stream) {
    PeerGather pg;
    if (int rc = make_peer_gather(nullptr, peer_signal, world, rank, epoch, 1, &pg)) return rc;
    allgather_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(pg, 0);
    BYBYCU_LAUNCH_CHECK("allgather_wait_kernel");
    return BYBYCU_OK;
}

}  // extern "C"
