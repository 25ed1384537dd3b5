/* ref_shim.c - TEST INFRASTRUCTURE ONLY.
 *
 * Exports the reference's own CPU implementation of the tile-GEMM path.  The reference
 * declares its C entry points with hidden visibility (backends/cpu/cpu_kernels.h:14-18), so
 * they cannot be dlopen'ed from a library built from those files alone; this shim is linked
 * into the same shared object as the UNCHANGED reference sources (backends/cpu/cpu_vm.c,
 * backends/cpu/cpu_kernels.c) and forwards to them.  oracle/Makefile builds the result into
 * oracle/_ref/libref_oracle.so.  Nothing in the product links it.
 */
#include "cpu_kernels.h"

#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define REFO_API __attribute__((visibility("default")))

/* nimf_cpu_vm_run_slots: backends/cpu/cpu_vm.c:178-182. */
REFO_API int refo_vm_run_slots(uint32_t* code, int n_words, float* mem, int mem_len,
                               const uint8_t* packed, int packed_len, const float* lut,
                               int lut_len, const float* in_f32, int in_len, int n_threads,
                               int tg_floats, int tg_size, char* err, int err_len) {
    return nimf_cpu_vm_run_slots(code, n_words, mem, mem_len, packed, packed_len, lut, lut_len,
                                 in_f32, in_len, n_threads, tg_floats, tg_size, err, err_len);
}

/* nimf_cpu_matmul_q4: backends/cpu/cpu_kernels.c:423-429. */
REFO_API void refo_matmul_q4(float* a, uint8_t* wq, float* scales, float* zeros, float* c,
                             int M, int K, int N, int group_size, int groups_per_row) {
    nimf_cpu_matmul_q4(a, wq, scales, zeros, c, M, K, N, group_size, groups_per_row);
}

/* ---- column-sharded runs over host threads ------------------------------------------
 * The reference is single-threaded (cpu_vm.c:588, cpu_kernels_impl.inc:303); its own way of
 * using more cores is to split the output columns over workers (distributed.nim:109-135,
 * largest-remainder with equal weights).  These helpers do that with one pthread per shard,
 * each running the unchanged reference entry point on its column range. */

typedef struct {
    const float* x; const uint8_t* packed; int64_t packed_len; const float* table;
    int M, K, N, c0, c1; int64_t scale_base; float* out; int rc; char err[160];
} TileJob;

static void* tile_worker(void* arg) {
    TileJob* j = (TileJob*)arg;
    const int nc = j->c1 - j->c0;
    if (nc <= 0) { j->rc = 0; return NULL; }
    const int64_t row_bytes = j->K / 2, G = j->K / 32;
    const int64_t off = (int64_t)j->c0 * row_bytes;
    /* The u8 slot starts at this shard's first nibble row; its scale bytes keep their place
       in the caller's buffer, so the program's scaleBase is relative to the new slot start. */
    const int64_t scale_rel = j->scale_base + (int64_t)j->c0 * G - off;
    uint32_t code[16] = {0xB0u, (uint32_t)j->M, (uint32_t)j->K, (uint32_t)nc,
                         (uint32_t)scale_rel, 0u, 0xB1u, 0xB2u, 0xB4u, 0xB5u, 0x50u, 0xB6u,
                         0x50u, 0xB3u, 0xB7u, 0x01u};
    float* mem = (float*)malloc((size_t)j->M * (size_t)nc * sizeof(float));
    if (!mem) { j->rc = -1; snprintf(j->err, sizeof j->err, "alloc"); return NULL; }
    j->rc = nimf_cpu_vm_run_slots(code, 16, mem, j->M * nc, j->packed + off,
                                  (int)(j->packed_len - off), j->table, 272, j->x,
                                  j->M * j->K, 128, 64, 128, j->err, (int)sizeof j->err);
    if (j->rc == 0)
        for (int r = 0; r < j->M; ++r)
            memcpy(j->out + (size_t)r * j->N + j->c0, mem + (size_t)r * nc,
                   (size_t)nc * sizeof(float));
    free(mem);
    return NULL;
}

/* OP_TILE_GEMM format 0 over `n_threads` column shards; returns 0 or -1 (message in err). */
REFO_API int refo_tile_gemm_mt(const float* x, const uint8_t* packed, int64_t packed_len,
                               int64_t scale_base, const float* table, int M, int K, int N,
                               float* out, int n_threads, char* err, int err_len) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    TileJob* jobs = (TileJob*)calloc((size_t)n_threads, sizeof(TileJob));
    if (!jobs) return -1;
    int c = 0;
    for (int t = 0; t < n_threads; ++t) {
        const int cnt = N / n_threads + (t < N % n_threads ? 1 : 0);
        jobs[t] = (TileJob){x, packed, packed_len, table, M, K, N, c, c + cnt, scale_base, out,
                            0, {0}};
        c += cnt;
        pthread_create(&th[t], NULL, tile_worker, &jobs[t]);
    }
    int rc = 0;
    for (int t = 0; t < n_threads; ++t) {
        pthread_join(th[t], NULL);
        if (jobs[t].rc != 0 && rc == 0) {
            rc = -1;
            if (err && err_len > 0) snprintf(err, (size_t)err_len, "%s", jobs[t].err);
        }
    }
    free(jobs);
    return rc;
}

typedef struct {
    float* a; uint8_t* wq; float* scales; float* zeros; float* c;
    int M, K, N, c0, c1, group_size, groups_per_row;
} Q4Job;

static void* q4_worker(void* arg) {
    Q4Job* j = (Q4Job*)arg;
    const int nc = j->c1 - j->c0;
    if (nc <= 0) return NULL;
    const int64_t bpr = (j->K + 1) / 2;
    float* tmp = (float*)malloc((size_t)j->M * (size_t)nc * sizeof(float));
    if (!tmp) return NULL;
    nimf_cpu_matmul_q4(j->a, j->wq + (int64_t)j->c0 * bpr,
                       j->scales + (int64_t)j->c0 * j->groups_per_row,
                       j->zeros + (int64_t)j->c0 * j->groups_per_row, tmp, j->M, j->K, nc,
                       j->group_size, j->groups_per_row);
    for (int r = 0; r < j->M; ++r)
        memcpy(j->c + (size_t)r * j->N + j->c0, tmp + (size_t)r * nc, (size_t)nc * sizeof(float));
    free(tmp);
    return NULL;
}

/* nimf_cpu_matmul_q4 over `n_threads` column shards. */
REFO_API void refo_matmul_q4_mt(float* a, uint8_t* wq, float* scales, float* zeros, float* c,
                                int M, int K, int N, int group_size, int groups_per_row,
                                int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    /* The ISA tables are initialised on first use; do it once before the threads race. */
    nimf_cpu_matmul_q4(a, wq, scales, zeros, c, 0, K, N, group_size, groups_per_row);
    pthread_t th[256];
    Q4Job jobs[256];
    int col = 0;
    for (int t = 0; t < n_threads; ++t) {
        const int cnt = N / n_threads + (t < N % n_threads ? 1 : 0);
        jobs[t] = (Q4Job){a, wq, scales, zeros, c, M, K, N, col, col + cnt, group_size,
                          groups_per_row};
        col += cnt;
        pthread_create(&th[t], NULL, q4_worker, &jobs[t]);
    }
    for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}
