/* q4_oracle.h - TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the BybyLang 4-bit tile-GEMM arithmetic, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker.  The product
 * (bybylang_b200, libbybycuda.so) never links, loads or calls anything in this directory.
 *
 * Every function cites the reference file:line whose arithmetic it restates.  The
 * restatement is pinned against the reference's own C (oracle/_ref/libref_oracle.so, built
 * from backends/cpu/cpu_vm.c + cpu_kernels.c unchanged) and against the golden vectors in
 * tests/golden/ that the reference produced.
 */
#ifndef Q4_ORACLE_H
#define Q4_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- generators ---------------------------------------------------------------------- */
uint32_t q4o_xorshift32(uint32_t* state);
void q4o_make_fp4_case(uint32_t* seed, int M, int K, int N, float* x, uint8_t* packed,
                       float* table);
void q4o_make_f16_case(uint32_t* seed, int M, int K, int N, float* x, float* w,
                       uint16_t* halves);
void q4o_make_gate_fp4(int M, int K, int N, float* x, uint8_t* packed, float* table);
void q4o_make_gate_f16(int M, int K, int N, float* x, float* w, uint16_t* halves);

/* ---- scalar conversions (IEEE round-to-nearest-even) --------------------------------- */
uint16_t q4o_f32_to_f16(float f);
float q4o_f16_to_f32(uint16_t h);
uint16_t q4o_f32_to_bf16(float f);
float q4o_bf16_to_f32(uint16_t b);

/* ---- synthetic inputs of the benchmark configurations -------------------------------- */
void q4o_gen_q4b32(uint32_t seed, int N, int K, uint8_t* packed, uint16_t* scales);
void q4o_gen_x_bf16(uint32_t seed, int M, int K, uint16_t* x);
void q4o_gen_x_f32(uint32_t seed, int M, int K, float* x);

/* ---- references ---------------------------------------------------------------------- */
void q4o_tile_gemm_fp4km(const float* x, const uint8_t* packed, int64_t scale_base,
                         const float* table, int M, int K, int N, float* out);
void q4o_tile_gemm_reference(const float* x, const uint8_t* packed, int64_t scale_base,
                             const float* table, int M, int K, int N, float* out);
void q4o_tile_gemm_f16(const float* x, const uint16_t* halves, int M, int K, int N,
                       float* out);
void q4o_tile_gemm_q4b32(const float* x, const uint8_t* packed, const uint16_t* scales,
                         int M, int K, int N, float* out);
void q4o_tile_gemm_q4b32_f64(const float* x, const uint8_t* packed, const uint16_t* scales,
                             int M, int K, int N, double* out);
void q4o_tile_gemm_q4b32_mt(const float* x, const uint8_t* packed, const uint16_t* scales,
                            int M, int K, int N, float* out, int n_threads);
void q4o_matmul_q4_asym(const float* a, const uint8_t* wq, const float* scales,
                        const float* zeros, int M, int K, int N, int group_size,
                        int groups_per_row, float* c);

/* ---- dequantisation ------------------------------------------------------------------ */
void q4o_dequant_q4b32(const uint8_t* packed, const uint16_t* scales, int N, int K, float* w);
void q4o_dequant_fp4km(const uint8_t* packed, int64_t scale_base, const float* table, int N,
                       int K, float* w);

/* ---- format converters --------------------------------------------------------------- */
void q4o_q4b32_to_asym(const uint8_t* packed, const uint16_t* scales, int N, int K,
                       uint8_t* wq, float* asym_scales, float* zeros);
int q4o_q4b32_to_fp4km(const uint8_t* packed, const uint16_t* scales, int N, int K,
                       uint8_t* out_packed, float* table);

#ifdef __cplusplus
}
#endif
#endif
