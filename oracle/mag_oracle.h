/*
 * mag_oracle.h - CPU restatement of the magnetron f32 forward-op kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * backend: tests, the smoke check and the CPU-baseline leg of the benchmark
 * call it to produce the expected results.  Nothing in the product links it.
 *
 * Each function restates one reference routine on raw buffers (element
 * strides, dim 0 fastest, 6 dims) and cites the reference file:line it
 * follows.  Arithmetic is plain IEEE single precision with separately rounded
 * multiply and add (the reference's x86-64 build uses SSE2..SSE4.2 only, so it
 * has no FMA); the file is compiled with -ffp-contract=off.
 *
 * Pinning: tests/test_oracle_golden.py checks every function against golden
 * vectors produced by the reference library itself (tests/golden/).
 */
#ifndef MAG_ORACLE_H
#define MAG_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* PCG / Box-Muller input generators (magnetron/magnetron.c:747-814, :1856-1876). */
typedef struct orc_pcg_t { uint64_t state, inc; } orc_pcg_t;
void orc_pcg_seed(orc_pcg_t* g, uint64_t seed);
void orc_fill_uniform(orc_pcg_t* g, float* out, int64_t n, float min, float max);
void orc_fill_normal(orc_pcg_t* g, float* out, int64_t n, float mean, float stddev);
/* The reference context's Mersenne-twister generator: its state struct's layout
 * (magnetron/magnetron_internal.h:398-402), seeding and draws (magnetron/magnetron.c:751-777, :797-803). */
typedef struct orc_mt_t { uint32_t remaining, next, state[624]; } orc_mt_t;
void orc_mt_seed(orc_mt_t* g, uint64_t seed);
void orc_fill_uniform_mt(orc_mt_t* g, float* out, int64_t n, float min, float max);
void orc_fill_normal_mt(orc_mt_t* g, float* out, int64_t n, float mean, float stddev);
void orc_mt_words(const orc_mt_t* g, uint32_t* out, int64_t n);

/* Scalar transcendental helpers, exposed for unit tests. */
float orc_sse_expf(float x);
float orc_sse_logf(float x);
void orc_sse_sincosf(float x, float* s, float* c);

/* Unary op over rows: r[ri*r_s1 + c] = f(x[ri*x_s1 + c]), c < cols.
 * op uses the reference op numbering; xi is the scalar for ADDS..DIVS.
 * Returns 0, or -1 for an op the reference panics on (SILU_DV, GELU_DV). */
int orc_unary(int op, float* r, const float* x, int64_t rows, int64_t cols,
              int64_t r_s1, int64_t x_s1, float xi);

/* Binary tiling-broadcast op (magnetron/magnetron_cpu.c:1616-1714). */
void orc_binary(int op, float* r, const float* x, const float* y,
                const int64_t* x_shape, const int64_t* x_strides,
                const int64_t* r_strides,
                const int64_t* y_shape, const int64_t* y_strides);

/* Full-tensor reduction SUM/MEAN/MIN/MAX (magnetron/magnetron_cpu.c:1034-1152). */
float orc_reduce(int op, const float* x, const int64_t* x_shape, const int64_t* x_strides);

/* MATMUL: R[M,N] (+)= X[M,K] Y[K,N], i-k-j order (magnetron/magnetron_cpu.c:2151-2185). */
void orc_matmul(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N, int64_t r_ld);

/* Extensions the reference API cannot express, restated with its arithmetic. */
void orc_binary_bcast2(int op, float* r, const float* x, const float* y,
                       const int64_t* r_shape, const int64_t* x_shape, const int64_t* y_shape,
                       const int64_t* sample_idx, int64_t n_sample);
void orc_reduce_rows(int op, float* r, const float* x, int64_t rows, int64_t cols);
void orc_softmax_rows(float* r, const float* x, int64_t rows, int64_t cols);
void orc_matmul_batched(float* r, const float* x, const float* y, int64_t batch,
                        int64_t M, int64_t K, int64_t N);
void orc_matmul_rows(float* r, const float* x, const float* y, int64_t row0, int64_t nrows,
                     int64_t K, int64_t N);

#ifdef __cplusplus
}
#endif
#endif
