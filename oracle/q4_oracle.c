/* q4_oracle.c - TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C restatement of the BybyLang tile-GEMM arithmetic for the three weight formats
 * of OP_TILE_GEMM (format 0 FP4-KM, format 1 FP16, format 2 Q4B32 = signed int4 + one fp16
 * scale per 32-value block), of the asymmetric-Q4 CPU kernel, and of the seeded generators
 * the reference's own tests use.  Built with -ffp-contract=off so that every product and
 * fmaf happens exactly where the reference C performs it.
 */
#include "q4_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------------------------
 * Generators
 * ------------------------------------------------------------------------------------- */

/* xorshift32 with shifts 13/17/5: tests/t_fp4_tile_gemm.nim:30-33. */
uint32_t q4o_xorshift32(uint32_t* state) {
    uint32_t s = *state;
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    *state = s;
    return s;
}

static const float kFp4Values[16] = {0.0f,  0.5f,  1.0f,  1.5f,  2.0f,  3.0f,  4.0f,  6.0f,
                                     -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

/* makeCase: tests/t_fp4_tile_gemm.nim:35-44.  x in {-1.000 .. +1.000} step 1e-3, random
 * nibble and scale bytes, the E2M1 value table and scale table (1 + i mod 13) / 64. */
void q4o_make_fp4_case(uint32_t* seed, int M, int K, int N, float* x, uint8_t* packed,
                       float* table) {
    for (int64_t i = 0; i < (int64_t)M * K; ++i)
        x[i] = (float)((int)(q4o_xorshift32(seed) % 2001u) - 1000) / 1000.0f;
    const int64_t nbytes = (int64_t)N * (K / 2) + (int64_t)N * (K / 32);
    for (int64_t i = 0; i < nbytes; ++i) packed[i] = (uint8_t)(q4o_xorshift32(seed) & 255u);
    for (int i = 0; i < 16; ++i) table[i] = kFp4Values[i];
    for (int i = 0; i < 256; ++i) table[16 + i] = (float)(1 + (i % 13)) / 64.0f;
}

/* makeF16Case: tests/t_fp4_tile_gemm.nim:205-219.  Weights k/1024 are exact halves. */
void q4o_make_f16_case(uint32_t* seed, int M, int K, int N, float* x, float* w,
                       uint16_t* halves) {
    for (int64_t i = 0; i < (int64_t)M * K; ++i)
        x[i] = (float)((int)(q4o_xorshift32(seed) % 2001u) - 1000) / 1000.0f;
    for (int64_t i = 0; i < (int64_t)N * K; ++i) {
        w[i] = (float)((int)(q4o_xorshift32(seed) % 2001u) - 1000) / 1024.0f;
        halves[i] = q4o_f32_to_f16(w[i]);
    }
}

/* The exact-data parity gate: backends/vulkan/vulkan_driver.nim:2694-2733 (FP4-KM branch):
 * power-of-two scales make every product and partial sum exact. */
void q4o_make_gate_fp4(int M, int K, int N, float* x, uint8_t* packed, float* table) {
    for (int i = 0; i < M * K; ++i) x[i] = (float)((i * 7 + 3) % 33 - 16) / 64.0f;
    for (int i = 0; i < 16; ++i) table[i] = kFp4Values[i];
    for (int i = 0; i < 256; ++i) table[16 + i] = ldexpf(1.0f, (i % 5) - 3);
    const int nib = N * (K / 2), groups = K / 32;
    for (int i = 0; i < nib; ++i) packed[i] = (uint8_t)((i * 37 + 11) % 256);
    for (int i = 0; i < N * groups; ++i) packed[nib + i] = (uint8_t)((i * 13 + 5) % 256);
}

/* The FP16 branch of the same gate: vulkan_driver.nim:2706-2717. */
void q4o_make_gate_f16(int M, int K, int N, float* x, float* w, uint16_t* halves) {
    for (int i = 0; i < M * K; ++i) x[i] = (float)((i * 7 + 3) % 33 - 16) / 64.0f;
    for (int i = 0; i < N * K; ++i) {
        w[i] = (float)((i * 5 + 1) % 29 - 14) / 16.0f;
        halves[i] = q4o_f32_to_f16(w[i]);
    }
}

/* ---------------------------------------------------------------------------------------
 * Scalar conversions
 * ------------------------------------------------------------------------------------- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary16 -> binary32, the mapping of backends/cpu/cpu_vm.c:53-69. */
float q4o_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return u2f(sign);
        /* subnormal: m * 2^-24 */
        float v = (float)m * ldexpf(1.0f, -24);
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* binary32 -> binary16, round to nearest even (overflow -> inf). */
uint16_t q4o_f32_to_f16(float f) {
    const uint32_t u = f2u(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (a > 0x7F800000u ? 0x200u : 0u));
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds past 65504 */
    if (a < 0x38800000u) {                                    /* subnormal or zero in fp16 */
        /* value = a_float; fp16 subnormal unit is 2^-24 */
        const float v = u2f(a) * 16777216.0f;                 /* exact scaling by 2^24 */
        const float r = nearbyintf(v);                        /* RNE under default mode */
        return (uint16_t)(sign | (uint16_t)r);
    }
    uint32_t mant = a & 0x7FFFFFu;
    uint32_t e = (a >> 23) - 112u;
    uint32_t h = (e << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

uint16_t q4o_f32_to_bf16(float f) {
    const uint32_t u = f2u(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

float q4o_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* ---------------------------------------------------------------------------------------
 * Synthetic inputs of the benchmark configurations.  Seeds: weights `seed`, scales
 * `seed + 1`; activations are drawn by the caller with its own seed (`seed + 2`).
 * ------------------------------------------------------------------------------------- */

static double normal01(uint32_t* st) {
    const double u1 = ((double)q4o_xorshift32(st) + 0.5) / 4294967296.0;
    const double u2 = ((double)q4o_xorshift32(st) + 0.5) / 4294967296.0;
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

/* q uniform over [-8, 7] as the raw two's-complement nibble, packed in the tile layout of
 * micro_kernel/session_vm.nim:384-387 (byte n*K/2 + 16g + j: low nibble k = 32g + j, high
 * nibble k = 32g + 16 + j); scales |N(0, 0.02)| rounded to fp16, exact zero -> 2^-24. */
void q4o_gen_q4b32(uint32_t seed, int N, int K, uint8_t* packed, uint16_t* scales) {
    uint32_t st = seed;
    const int G = K / 32;
    memset(packed, 0, (size_t)N * (size_t)(K / 2));
    for (int64_t n = 0; n < N; ++n) {
        uint8_t* row = packed + n * (K / 2);
        for (int k = 0; k < K; ++k) {
            const uint8_t nib = (uint8_t)(q4o_xorshift32(&st) & 15u);
            const int g = k / 32, j = k % 32;
            if (j < 16) row[g * 16 + j] |= nib;
            else row[g * 16 + (j - 16)] |= (uint8_t)(nib << 4);
        }
    }
    uint32_t ss = seed + 1u;
    for (int64_t i = 0; i < (int64_t)N * G; ++i) {
        uint16_t h = q4o_f32_to_f16((float)(fabs(normal01(&ss)) * 0.02));
        if ((h & 0x7FFFu) == 0) h = 0x0001u;
        scales[i] = h;
    }
}

void q4o_gen_x_bf16(uint32_t seed, int M, int K, uint16_t* x) {
    uint32_t st = seed;
    for (int64_t i = 0; i < (int64_t)M * K; ++i) x[i] = q4o_f32_to_bf16((float)normal01(&st));
}

void q4o_gen_x_f32(uint32_t seed, int M, int K, float* x) {
    uint32_t st = seed;
    for (int64_t i = 0; i < (int64_t)M * K; ++i) x[i] = (float)normal01(&st);
}

/* ---------------------------------------------------------------------------------------
 * References
 * ------------------------------------------------------------------------------------- */

static inline float nib_signed(uint32_t nib) { return (float)((int)(nib ^ 8u) - 8); }

/* OP_TILE_GEMM format 0 exactly as the CPU VM computes it: backends/cpu/cpu_vm.c:605-626
 * (per group: the 16 low nibbles then the 16 high nibbles, fmaf(x, table[nib] * scale)). */
void q4o_tile_gemm_fp4km(const float* x, const uint8_t* packed, int64_t scale_base,
                         const float* table, int M, int K, int N, float* out) {
    const int64_t row_bytes = K / 2, G = K / 32;
    const float* scales = table + 16;
    for (int64_t r = 0; r < M; ++r)
        for (int64_t c = 0; c < N; ++c) {
            float sum = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                const float s = scales[packed[scale_base + c * G + g]];
                const uint8_t* b = packed + c * row_bytes + g * 16;
                const float* xg = x + r * K + g * 32;
                for (int j = 0; j < 16; ++j) sum = fmaf(xg[j], table[b[j] & 15u] * s, sum);
                for (int j = 0; j < 16; ++j) sum = fmaf(xg[16 + j], table[b[j] >> 4] * s, sum);
            }
            out[r * N + c] = sum;
        }
}

/* tileGemmReference: micro_kernel/tile_gemm.nim:663-677 (low and high nibble of byte j
 * alternate; plain multiply then add). */
void q4o_tile_gemm_reference(const float* x, const uint8_t* packed, int64_t scale_base,
                             const float* table, int M, int K, int N, float* out) {
    const int64_t G = K / 32;
    for (int64_t r = 0; r < M; ++r)
        for (int64_t c = 0; c < N; ++c) {
            float sum = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                const float s = table[16 + packed[scale_base + c * G + g]];
                for (int j = 0; j < 16; ++j) {
                    const uint8_t b = packed[c * (K / 2) + g * 16 + j];
                    const float w0 = table[b & 15u] * s;
                    const float p0 = x[r * K + g * 32 + j] * w0;
                    sum = sum + p0;
                    const float w1 = table[b >> 4] * s;
                    const float p1 = x[r * K + g * 32 + 16 + j] * w1;
                    sum = sum + p1;
                }
            }
            out[r * N + c] = sum;
        }
}

/* OP_TILE_GEMM format 1 (IEEE halves [N, K]): backends/cpu/cpu_vm.c:550-581. */
void q4o_tile_gemm_f16(const float* x, const uint16_t* halves, int M, int K, int N,
                       float* out) {
    for (int64_t r = 0; r < M; ++r)
        for (int64_t c = 0; c < N; ++c) {
            float sum = 0.0f;
            for (int64_t k = 0; k < K; ++k)
                sum = fmaf(x[r * K + k], q4o_f16_to_f32(halves[c * K + k]), sum);
            out[r * N + c] = sum;
        }
}

/* Format 2 (Q4B32): the FP4-KM loop of cpu_vm.c:605-626 with table[nib] replaced by the
 * signed nibble and table[16 + scale byte] by the block's fp16 scale.  This is bit-identical
 * to the reference VM run on the palette conversion (q4o_q4b32_to_fp4km). */
void q4o_tile_gemm_q4b32(const float* x, const uint8_t* packed, const uint16_t* scales,
                         int M, int K, int N, float* out) {
    const int64_t row_bytes = K / 2, G = K / 32;
    for (int64_t r = 0; r < M; ++r)
        for (int64_t c = 0; c < N; ++c) {
            float sum = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                const float s = q4o_f16_to_f32(scales[c * G + g]);
                const uint8_t* b = packed + c * row_bytes + g * 16;
                const float* xg = x + r * K + g * 32;
                for (int j = 0; j < 16; ++j) sum = fmaf(xg[j], nib_signed(b[j] & 15u) * s, sum);
                for (int j = 0; j < 16; ++j) sum = fmaf(xg[16 + j], nib_signed(b[j] >> 4) * s, sum);
            }
            out[r * N + c] = sum;
        }
}

/* The same product accumulated in double: the tolerance yardstick for fp16-rounding paths. */
void q4o_tile_gemm_q4b32_f64(const float* x, const uint8_t* packed, const uint16_t* scales,
                             int M, int K, int N, double* out) {
    const int64_t row_bytes = K / 2, G = K / 32;
    for (int64_t r = 0; r < M; ++r)
        for (int64_t c = 0; c < N; ++c) {
            double sum = 0.0;
            for (int64_t g = 0; g < G; ++g) {
                const double s = (double)q4o_f16_to_f32(scales[c * G + g]);
                const uint8_t* b = packed + c * row_bytes + g * 16;
                const float* xg = x + r * K + g * 32;
                double part = 0.0;
                for (int j = 0; j < 16; ++j) part += (double)xg[j] * nib_signed(b[j] & 15u);
                for (int j = 0; j < 16; ++j) part += (double)xg[16 + j] * nib_signed(b[j] >> 4);
                sum += part * s;
            }
            out[r * N + c] = sum;
        }
}

typedef struct {
    const float* x; const uint8_t* packed; const uint16_t* scales;
    int M, K, N, c0, c1; float* out;
} MtJob;

static void* mt_worker(void* arg) {
    MtJob* j = (MtJob*)arg;
    const int64_t row_bytes = j->K / 2, G = j->K / 32;
    for (int64_t r = 0; r < j->M; ++r)
        for (int64_t c = j->c0; c < j->c1; ++c) {
            float sum = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                const float s = q4o_f16_to_f32(j->scales[c * G + g]);
                const uint8_t* b = j->packed + c * row_bytes + g * 16;
                const float* xg = j->x + r * j->K + g * 32;
                for (int q = 0; q < 16; ++q) sum = fmaf(xg[q], nib_signed(b[q] & 15u) * s, sum);
                for (int q = 0; q < 16; ++q) sum = fmaf(xg[16 + q], nib_signed(b[q] >> 4) * s, sum);
            }
            j->out[r * j->N + c] = sum;
        }
    return NULL;
}

/* Column-sharded threads: contiguous column ranges, largest-remainder split with equal
 * weights (the rule of distributed.nim:109-135). */
void q4o_tile_gemm_q4b32_mt(const float* x, const uint8_t* packed, const uint16_t* scales,
                            int M, int K, int N, float* out, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    MtJob jobs[256];
    int c = 0;
    for (int t = 0; t < n_threads; ++t) {
        const int cnt = N / n_threads + (t < N % n_threads ? 1 : 0);
        jobs[t] = (MtJob){x, packed, scales, M, K, N, c, c + cnt, out};
        c += cnt;
        pthread_create(&th[t], NULL, mt_worker, &jobs[t]);
    }
    for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}

/* nimf_cpu_matmul_q4: backends/cpu/cpu_kernels_impl.inc:293-319 (interleaved nibbles: even
 * k in the low nibble; w = (nib - zero) * scale; evaluated as (a * (nib - zp)) * sc). */
void q4o_matmul_q4_asym(const float* a, const uint8_t* wq, const float* scales,
                        const float* zeros, int M, int K, int N, int group_size,
                        int groups_per_row, float* c) {
    const int bytes_per_row = (K + 1) / 2;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            const uint8_t* wrow = wq + n * bytes_per_row;
            const int64_t rg = n * groups_per_row;
            float sum = 0.0f;
            for (int k = 0; k < K; ++k) {
                const int g = group_size > 0 ? k / group_size : 0;
                const float sc = scales[rg + g], zp = zeros[rg + g];
                const uint8_t byte = wrow[k >> 1];
                const uint8_t nib = (k & 1) ? (uint8_t)(byte >> 4) : (uint8_t)(byte & 0x0F);
                const float t = a[m * K + k] * ((float)nib - zp);
                sum += t * sc;
            }
            c[m * N + n] = sum;
        }
}

/* ---------------------------------------------------------------------------------------
 * Dequantisation (the bit-exact check: every format's weight is one fp32 product)
 * ------------------------------------------------------------------------------------- */

void q4o_dequant_q4b32(const uint8_t* packed, const uint16_t* scales, int N, int K, float* w) {
    const int64_t G = K / 32;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            const int64_t g = k / 32, j = k % 32;
            const uint8_t b = packed[n * (K / 2) + g * 16 + (j & 15)];
            const uint32_t nib = j < 16 ? (b & 15u) : (uint32_t)(b >> 4);
            w[n * K + k] = nib_signed(nib) * q4o_f16_to_f32(scales[n * G + g]);
        }
}

void q4o_dequant_fp4km(const uint8_t* packed, int64_t scale_base, const float* table, int N,
                       int K, float* w) {
    const int64_t G = K / 32;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            const int64_t g = k / 32, j = k % 32;
            const uint8_t b = packed[n * (K / 2) + g * 16 + (j & 15)];
            const uint32_t nib = j < 16 ? (b & 15u) : (uint32_t)(b >> 4);
            w[n * K + k] = table[nib] * table[16 + packed[scale_base + n * G + g]];
        }
}

/* ---------------------------------------------------------------------------------------
 * Format converters
 * ------------------------------------------------------------------------------------- */

/* Q4B32 -> the asymmetric Q4 of gpubackend.nim:288-311 / cpu_kernels_impl.inc:293-319:
 * u = q + 8 (= nibble ^ 8) interleaved (even k low), zero 8.0, scale (float)fp16. */
void q4o_q4b32_to_asym(const uint8_t* packed, const uint16_t* scales, int N, int K,
                       uint8_t* wq, float* asym_scales, float* zeros) {
    const int64_t G = K / 32, bpr = (K + 1) / 2;
    memset(wq, 0, (size_t)(N * bpr));
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) {
            const int64_t g = k / 32, j = k % 32;
            const uint8_t b = packed[n * (K / 2) + g * 16 + (j & 15)];
            const uint32_t nib = j < 16 ? (b & 15u) : (uint32_t)(b >> 4);
            const uint8_t u = (uint8_t)(nib ^ 8u);
            wq[n * bpr + (k >> 1)] |= (uint8_t)((k & 1) ? (u << 4) : u);
        }
        for (int64_t g = 0; g < G; ++g) {
            asym_scales[n * G + g] = q4o_f16_to_f32(scales[n * G + g]);
            zeros[n * G + g] = 8.0f;
        }
    }
}

/* Q4B32 -> FP4-KM when the fp16 scales take at most 256 distinct values: value table
 * {0..7, -8..-1}, scale table = the palette, scale byte = palette index, the nibble bytes
 * unchanged (both formats share the tile layout).  Returns the palette size or -1. */
int q4o_q4b32_to_fp4km(const uint8_t* packed, const uint16_t* scales, int N, int K,
                       uint8_t* out_packed, float* table) {
    const int64_t G = K / 32, nib_bytes = (int64_t)N * (K / 2);
    int* index = (int*)malloc(65536 * sizeof(int));
    if (!index) return -1;
    for (int i = 0; i < 65536; ++i) index[i] = -1;
    uint16_t palette[256];
    int np = 0;
    for (int64_t i = 0; i < (int64_t)N * G; ++i) {
        const uint16_t h = scales[i];
        if (index[h] < 0) {
            if (np == 256) { free(index); return -1; }
            index[h] = np;
            palette[np++] = h;
        }
        out_packed[nib_bytes + i] = (uint8_t)index[h];
    }
    memcpy(out_packed, packed, (size_t)nib_bytes);
    for (int i = 0; i < 16; ++i) table[i] = nib_signed((uint32_t)i);
    for (int i = 0; i < 256; ++i) table[16 + i] = i < np ? q4o_f16_to_f32(palette[i]) : 0.0f;
    free(index);
    return np;
}
