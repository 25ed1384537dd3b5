// vm.cu - bybycu_vm_run_slots, the device-pointer twin of nimf_cpu_vm_run_slots for the
// micro-VM programs of this path, and the asymmetric-Q4 shape ops' kernel.
//
// Accepted programs (the shape/tile ops of micro_kernel/session_vm.nim:98-122):
//   OP_TILE_GEMM fmt, M, K, N, scaleBase, lutBase  followed by the tile ops of
//       buildFp4TileGemmProgram / buildF16TileGemmProgram (session_vm.nim:383-416), in the
//       order lowerTileGemm accepts (micro_kernel/tile_gemm.nim:616-661), ending in HALT;
//   OP_FP4_COOP_GEMM M, K, N, 32, K/32; HALT  (the legacy one-blob form, tile_gemm.nim:55-66);
//   OP_Q4_GEMV / OP_Q4_COOP_GEMM M, K, N, group, nGroups; HALT (asymmetric Q4 blob,
//       backends/cpu/cpu_vm.c:420-482).
// The slot checks and their messages are the CPU VM's (cpu_vm.c:420-604).
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "kernels.h"

namespace bybycu {

int check_tile_gemm(int fmt, int M, int K, int N, int64_t x_len, int64_t packed_len, int64_t scale_base,
                    int64_t lut_len, int64_t lut_base, int64_t out_len);
int choose_route(const GemmArgs& a, int requested, int* route);
int run_gemm(const GemmArgs& a, int route);

namespace {

enum : uint32_t {
    OP_NOP = 0x00, OP_HALT = 0x01, OP_BARRIER_TG = 0x50,
    OP_Q4_COOP_GEMM = 0xAA, OP_Q4_GEMV = 0xAB, OP_FP4_COOP_GEMM = 0xAC,
    OP_TILE_GEMM = 0xB0, OP_TILE_ZERO = 0xB1, OP_TILE_K_BEGIN = 0xB2, OP_TILE_K_END = 0xB3,
    OP_TILE_LOAD_A = 0xB4, OP_TILE_DECODE_FP4 = 0xB5, OP_TILE_MMA = 0xB6, OP_TILE_STORE = 0xB7,
    OP_TILE_LOAD_B_F16 = 0xB8,
};

// The 8-bit register field `a` (pack1/pack3 of session_vm.nim:199-218).
inline uint32_t field_a(uint32_t w) { return ((w >> 8) & 0x1Fu) | (((w >> 23) & 0x7u) << 5); }

// Asymmetric Q4 (cpu_vm.c:420-482): nibbles [N, K/2] interleaved (even k low), fp32 scales
// at float (N*K/2+3)/4 of the table slot, zeros after them; fmaf(x, (q - z) * s, sum) over
// k in order.  One thread per output, bit-identical to the CPU VM.
__global__ void q4_asym_kernel(int M, int K, int N, int group, int n_groups, const uint8_t* __restrict__ q,
                               const float* __restrict__ params, const float* __restrict__ x, float* __restrict__ out) {
    const int64_t n = static_cast<int64_t>(blockIdx.x) * 128 + threadIdx.x;
    const int64_t m = blockIdx.y;
    if (n >= N) return;
    const int64_t row_bytes = K / 2;
    const int64_t scale_base = (static_cast<int64_t>(N) * row_bytes + 3) / 4;
    const int64_t zero_base = scale_base + static_cast<int64_t>(N) * n_groups;
    float sum = 0.0f;
    for (int k = 0; k < K; ++k) {
        const uint32_t byte = q[n * row_bytes + (k >> 1)];
        const uint32_t nib = (byte >> ((k & 1) * 4)) & 15u;
        const int64_t gi = n * n_groups + k / group;
        const float w = (static_cast<float>(nib) - params[zero_base + gi]) * params[scale_base + gi];
        sum = fmaf(x[m * K + k], w, sum);
    }
    out[m * N + n] = sum;
}

int vm_fail(int code, char* err, int err_len, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (err && err_len > 0) snprintf(err, static_cast<size_t>(err_len), "%s", buf);
    return set_error(code, "%s", buf);
}

// The op sequence after an OP_TILE_GEMM header must be one lowerTileGemm accepts.
bool valid_tile_ops(const uint32_t* code, int n, int fmt, const char** why) {
    bool in_loop = false, stored = false, halted = false, zeroed = false;
    for (int pc = 6; pc < n; ++pc) {
        const uint32_t op = code[pc] & 0xFFu;
        if (halted) { *why = "tile GEMM: ops after HALT"; return false; }
        switch (op) {
            case OP_TILE_ZERO: zeroed = true; break;
            case OP_TILE_K_BEGIN:
                if (in_loop) { *why = "tile GEMM: nested K loop"; return false; }
                in_loop = true;
                break;
            case OP_TILE_K_END:
                if (!in_loop) { *why = "tile GEMM: K_END without K_BEGIN"; return false; }
                in_loop = false;
                break;
            case OP_TILE_LOAD_A: case OP_TILE_MMA:
                if (!in_loop) { *why = "tile GEMM: staging ops belong inside the K loop"; return false; }
                break;
            case OP_TILE_DECODE_FP4:
                if (!in_loop || fmt == 1) { *why = "tile GEMM: DECODE_FP4 misplaced"; return false; }
                break;
            case OP_TILE_LOAD_B_F16:
                if (!in_loop || fmt != 1) { *why = "tile GEMM: LOAD_B_F16 misplaced"; return false; }
                break;
            case OP_BARRIER_TG:
                if (!in_loop) { *why = "tile GEMM: barriers belong inside the K loop"; return false; }
                break;
            case OP_TILE_STORE:
                if (in_loop || !zeroed) { *why = "tile GEMM: STORE outside the accumulator's life"; return false; }
                stored = true;
                break;
            case OP_NOP: break;
            case OP_HALT: halted = true; break;
            default: *why = "tile GEMM: op has no tile lowering"; return false;
        }
    }
    if (!(halted && stored)) { *why = "tile GEMM program must store its tile and end with HALT"; return false; }
    return true;
}

}  // namespace
}  // namespace bybycu

using namespace bybycu;

extern "C" int bybycu_vm_run_slots(const uint32_t* code, int n_words, float* mem, int mem_len, const uint8_t* packed,
                                   int packed_len, const float* lut, int lut_len, const float* in_f32, int in_len,
                                   int n_threads, int tg_floats, int tg_size, char* err, int err_len, void* stream) {
    if (err && err_len > 0) err[0] = '\0';
    if (!code || n_words <= 0 || !mem || mem_len <= 0 || n_threads <= 0 || tg_size <= 0 || tg_floats < 0)
        return vm_fail(BYBYCU_ERR_ARGS, err, err_len, "invalid CUDA VM arguments");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint32_t op = code[0] & 0xFFu;
    if (op != OP_TILE_GEMM && op != OP_FP4_COOP_GEMM && op != OP_Q4_GEMV && op != OP_Q4_COOP_GEMM)
        return vm_fail(BYBYCU_ERR_PROGRAM, err, err_len,
                       "CUDA VM runs tile GEMM and Q4/FP4 shape-op programs only (first op 0x%02X)", op);
    if (n_words < 6) return vm_fail(BYBYCU_ERR_PROGRAM, err, err_len, "CUDA VM truncated tile GEMM header");
    const float* x = in_f32 ? in_f32 : mem;
    const int64_t x_len = in_f32 ? in_len : mem_len;
    uint32_t M = code[1];
    const uint32_t K = code[2], N = code[3];

    if (op == OP_TILE_GEMM) {
        const int fmt = static_cast<int>(field_a(code[0]));
        const int64_t scale_base = code[4], lut_base = code[5];
        if (fmt > 2 || !K || K % 32u || !N)
            return vm_fail(BYBYCU_ERR_SHAPE, err, err_len, "CUDA VM unsupported tile GEMM (format %d K %u N %u)", fmt, K, N);
        const char* why = nullptr;
        if (!valid_tile_ops(code, n_words, fmt, &why)) return vm_fail(BYBYCU_ERR_PROGRAM, err, err_len, "%s", why);
        if (!packed || (fmt == 0 && !lut) || x_len < 0)
            return vm_fail(BYBYCU_ERR_ARGS, err, err_len, "CUDA VM tile GEMM slot is missing");
        if (M == 0) M = static_cast<uint32_t>(x_len / K);
        if (M == 0 || check_tile_gemm(fmt, static_cast<int>(M), static_cast<int>(K), static_cast<int>(N), x_len,
                                      packed_len, scale_base, lut_len, lut_base, mem_len))
            return vm_fail(BYBYCU_ERR_RANGE, err, err_len, "CUDA VM tile GEMM input out of range");
        GemmArgs a;
        a.fmt = fmt; a.M = static_cast<int>(M); a.K = static_cast<int>(K); a.N = static_cast<int>(N);
        a.x = x; a.x_dtype = BYBYCU_DT_F32;
        a.packed = packed; a.packed_len = packed_len; a.scale_base = scale_base;
        a.lut = lut ? lut + lut_base : nullptr;
        a.out = mem; a.out_dtype = BYBYCU_DT_F32; a.out_ld = N; a.out_col0 = 0;
        a.stream = s;
        int route = 0;
        if (int rc = choose_route(a, BYBYCU_ROUTE_AUTO, &route)) return vm_fail(rc, err, err_len, "%s", "route");
        if (int rc = run_gemm(a, route)) {
            char msg[256];
            bybycu_last_error(msg, sizeof msg);
            return vm_fail(rc, err, err_len, "%s", msg);
        }
        return BYBYCU_OK;
    }

    // the five-word shape ops: M, K, N, group, nGroups; the program is the op and HALT
    if (n_words != 7 || (code[6] & 0xFFu) != OP_HALT)
        return vm_fail(BYBYCU_ERR_PROGRAM, err, err_len, "CUDA VM shape-op program must be the op followed by HALT");
    const uint32_t group = code[4], n_groups = code[5];
    if (op == OP_FP4_COOP_GEMM) {
        if (!M || !K || K % 64u || N < 16u || group != 32u || n_groups != K / 32u)
            return vm_fail(BYBYCU_ERR_SHAPE, err, err_len, "CUDA VM unsupported FP4 cooperative shape");
        if (!packed || !lut) return vm_fail(BYBYCU_ERR_ARGS, err, err_len, "CUDA VM FP4 cooperative slot is missing");
        const int64_t scale_bytes = static_cast<int64_t>(N) * (K / 2);
        const int64_t lut_base = (scale_bytes + static_cast<int64_t>(N) * n_groups + 3) / 4;
        if (scale_bytes + static_cast<int64_t>(N) * n_groups > packed_len || lut_base + 272 > lut_len ||
            static_cast<int64_t>(M) * K > x_len || static_cast<int64_t>(M) * N > mem_len)
            return vm_fail(BYBYCU_ERR_RANGE, err, err_len, "CUDA VM FP4 cooperative input out of range");
        GemmArgs a;
        a.fmt = 0; a.M = static_cast<int>(M); a.K = static_cast<int>(K); a.N = static_cast<int>(N);
        a.x = x; a.x_dtype = BYBYCU_DT_F32;
        a.packed = packed; a.packed_len = packed_len; a.scale_base = scale_bytes;
        a.lut = lut + lut_base;
        a.out = mem; a.out_dtype = BYBYCU_DT_F32; a.out_ld = N; a.out_col0 = 0;
        a.stream = s;
        int route = 0;
        if (int rc = choose_route(a, BYBYCU_ROUTE_AUTO, &route)) return vm_fail(rc, err, err_len, "route");
        if (int rc = run_gemm(a, route)) {
            char msg[256];
            bybycu_last_error(msg, sizeof msg);
            return vm_fail(rc, err, err_len, "%s", msg);
        }
        return BYBYCU_OK;
    }
    const bool coop = op == OP_Q4_COOP_GEMM;
    if (!M || !N || !K || !group || K % group || n_groups != K / group || (coop && (N < 16 || K % 64 || group % 2)) ||
        (!coop && (K % 8 || group % 8)))
        return vm_fail(BYBYCU_ERR_SHAPE, err, err_len, "CUDA VM unsupported Q4 %s shape", coop ? "cooperative" : "GEMV");
    if (!packed || !lut) return vm_fail(BYBYCU_ERR_ARGS, err, err_len, "CUDA VM Q4 cooperative slot is missing");
    const int64_t row_bytes = K / 2;
    const int64_t scale_base = (static_cast<int64_t>(N) * row_bytes + 3) / 4;
    const int64_t zero_end = scale_base + 2 * static_cast<int64_t>(N) * n_groups;
    if (static_cast<int64_t>(N) * row_bytes > packed_len || zero_end > lut_len || static_cast<int64_t>(M) * K > x_len ||
        static_cast<int64_t>(M) * N > mem_len)
        return vm_fail(BYBYCU_ERR_RANGE, err, err_len, "CUDA VM Q4 cooperative input out of range");
    if (M > 65535u) return vm_fail(BYBYCU_ERR_SHAPE, err, err_len, "CUDA VM Q4 shape op: M above 65535");
    const dim3 grid(static_cast<unsigned>(ceil_div(N, 128)), M);
    q4_asym_kernel<<<grid, 128, 0, s>>>(static_cast<int>(M), static_cast<int>(K), static_cast<int>(N),
                                        static_cast<int>(group), static_cast<int>(n_groups), packed, lut, x, mem);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return vm_fail(BYBYCU_ERR_CUDA, err, err_len, "q4_asym_kernel: %s", cudaGetErrorString(e));
    return BYBYCU_OK;
}
