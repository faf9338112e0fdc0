/*
 * mcu_kernels.h - C-callable launchers of the sm_100a kernels.
 *
 * Every launcher enqueues on the given stream and returns a cudaError_t value
 * (0 on success).  Tensors are f32, strides are in elements, dim 0 is the
 * fastest dimension, exactly as in the magnetron core.
 */
#ifndef MCU_KERNELS_H
#define MCU_KERNELS_H
#include <stdint.h>
#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* k_elementwise.cu */
int mcu_launch_unary(int op, float* r, const float* x, int64_t rows, int64_t cols, int64_t r_s1, int64_t x_s1,
                     float xi, cudaStream_t st);
int mcu_launch_binary(int op, float* r, const float* x, const float* y, const int64_t* x_dims,
                      const int64_t* x_strides, const int64_t* r_strides, const int64_t* y_dims,
                      const int64_t* y_strides, cudaStream_t st);
int mcu_launch_bcast2(int op, float* r, const float* x, const float* y, const int64_t* r_dims,
                      const int64_t* x_dims, const int64_t* y_dims, cudaStream_t st);

/* k_reduce.cu: scratch needs mcu_reduce_scratch_bytes() bytes of device memory. */
size_t mcu_reduce_scratch_bytes(void);
int mcu_launch_reduce(int op, float* r, const float* x, const int64_t* x_dims, const int64_t* x_strides,
                      void* scratch, cudaStream_t st);
/* One shard's full-reduction record (a sharded SUM/MEAN/MIN/MAX exchanges these). */
typedef struct McuReducePart {
    double sum;
    float min, max;
    uint64_t count;
} McuReducePart;
int mcu_launch_reduce_partial(McuReducePart* part, const float* x, const int64_t* x_dims, const int64_t* x_strides,
                              void* scratch, cudaStream_t st);
int mcu_launch_reduce_combine(int op, float* r, const McuReducePart* parts, int nparts, cudaStream_t st);
int mcu_launch_reduce_rows(int op, float* r, const float* x, int64_t rows, int64_t cols, cudaStream_t st);
/* Normalised row softmax; scratch needs mcu_softmax_rows_scratch_bytes(rows, cols) bytes
 * (nonzero only for rows wider than 65536, whose fallback, when their cluster shape cannot be
 * scheduled, takes two passes over slice statistics and a per-row combine). */
size_t mcu_softmax_rows_scratch_bytes(int64_t rows, int64_t cols);
int mcu_softmax_rows_kernels(int64_t rows, int64_t cols); /* kernel launches of one call */
int mcu_launch_softmax_rows(float* r, const float* x, int64_t rows, int64_t cols, void* scratch, cudaStream_t st);

/* k_fill.cu: PCG stream fills (normal != 0: Box-Muller pairs; p0, p1 = mean, stddev,
 * else p0, p1 = min, max - min) and constant fills. */
uint64_t mcu_pcg_advance(uint64_t state, uint64_t inc, uint64_t n);
int mcu_launch_fill_pcg(float* r, int64_t n, int normal, float p0, float p1, uint64_t state, uint64_t inc,
                        cudaStream_t st);
int mcu_launch_fill_const(float* r, int64_t n, float x, cudaStream_t st);
/* k_fill_mt.cu: fills from the Mersenne-twister stream of st = {remaining, next, state[624]},
 * which is left as the host generator leaves it (the call waits when it draws past the current
 * block).  *launches = kernels launched. */
size_t mcu_fill_mt_scratch_bytes(int64_t n, uint32_t remaining, uint32_t next);
int mcu_launch_fill_mt(float* r, int64_t n, int normal, float p0, float p1, uint32_t* st, void* scratch,
                       cudaStream_t stream, int* launches);
int mcu_mt19937_degree(void);
int mcu_mt19937_jump_host(const uint32_t* win, uint64_t d, uint32_t* out);

/* k_image.cu: planar f32 [c][h][w] <-> interleaved u8 [h][w][c] (resized to rw x rh when both
 * are nonzero, with ws = (w-1)/(rw-1), hs = (h-1)/(rh-1) rounded to f32), box and text drawing
 * on 3-channel images; glyphs holds (x, y, glyph index) triples. */
int mcu_launch_img_from_u8(float* dst, const uint8_t* src, uint32_t w, uint32_t h, uint32_t c, uint32_t rw,
                           uint32_t rh, float ws, float hs, cudaStream_t st);
int mcu_launch_img_to_u8(uint8_t* dst, const float* src, uint32_t w, uint32_t h, uint32_t c, cudaStream_t st);
int mcu_launch_img_draw_box(float* img, int32_t w, int32_t h, int32_t x1, int32_t y1, int32_t x2, int32_t y2,
                            int32_t wi, float r, float g, float b, cudaStream_t st);
int mcu_launch_img_draw_text(float* img, int32_t w, int32_t h, const int32_t* glyphs, int32_t n, float r, float g,
                             float b, cudaStream_t st);

/* k_matmul_exact.cu: R[b][i*r_ld + j] = (accumulate ? R : 0) + sum_k X[b][i*K+k]*Y[b][k*N+j],
 * summed k = 0..K-1 in order with separately rounded multiply and add. */
int mcu_launch_matmul_exact(float* r, const float* x, const float* y, int64_t batch, int64_t M, int64_t K,
                            int64_t N, int64_t r_ld, int accumulate, cudaStream_t st);
/* A single bit-exact product with a fused dense-layer epilogue: r = act(xy + bias), the bias
 * read at the flat result index (bias_mod = 0) or at that index mod bias_mod (a bias broadcast
 * along dim 0), act 0 none, 1 GELU, 2 SIGMOID (their vector-lane formulas).  At most 1048560
 * rows. */
int mcu_launch_matmul_exact_ep(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                               const float* bias, int64_t bias_mod, int act, cudaStream_t st);
/* Kernels one exact product launches: a single product of more than 1048560 rows runs in slices. */
int mcu_matmul_exact_kernels(int64_t batch, int64_t M);
/* Largest K the tensor-core product takes (its padded K indexes a grid dimension); beyond it the
 * CUDA-core paths, which have no K limit, run the product. */
#define MCU_TC_MAX_K (((int64_t)1 << 21) - 32)

size_t mcu_matmul_skinny_scratch_bytes(int64_t M, int64_t K, int64_t N);
int mcu_launch_matmul_skinny(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                             int64_t r_ld, void* scratch, cudaStream_t st);

/* Allocation-free skinny product: scratch is a fixed device array of this library. */
size_t mcu_skinny_noalloc_limit(void);
int mcu_skinny_noalloc_scratch(void** out);

/* k_matmul_tc.cu: tcgen05 GEMM with a three-product split, R[M,N] = X[M,K] Y[K,N] (row-major);
 * f16 = 0: tf32 hi/lo split (kind::tf32), f16 = 1: scaled f16 hi/lo split (kind::f16).
 * scratch needs mcu_matmul_tc_scratch_bytes(M, K, N) bytes (either split). */
size_t mcu_matmul_tc_scratch_bytes(int64_t M, int64_t K, int64_t N);
/* Kernels one single (unbatched) product launches: operand splits, the GEMM, and the part sum
 * when K is split (for few tiles, or for the tiles of a mostly empty last wave); flags bit 0:
 * X arrives split by the previous layer's epilogue (tf32), bit 1: fused dense-layer epilogue. */
int mcu_matmul_tc_kernels(int64_t M, int64_t K, int64_t N, int f16, int flags);
int mcu_launch_matmul_tc(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                         void* scratch, int* status, cudaStream_t st, int f16);
int mcu_matmul_tc_supported(void);

/* Fused dense-layer epilogue for the tensor-core GEMM: out = act(X Y + bias) with
 * bias at the result's row-major index (or NULL), act 0 = none, 1 = GELU; when
 * out_hi/out_lo are set the tf32 hi/lo split of out is also written in the
 * [M][kp_out] layout the next product reads (kp_out = N rounded up to 32, N % 32 == 0).
 * a_hi/a_lo, when set, are X already split in that layout (no split pass).  The split
 * fields apply to the tf32 split only; the f16 split always splits X itself. */
typedef struct mcu_tc_epilogue {
    const float* a_hi;
    const float* a_lo;
    const float* bias;
    float* out_hi;
    float* out_lo;
    int64_t kp_out;
    int act;
    int bias_zero; /* the bias is known to be zero: add +0.0f (which maps -0 to +0) and read nothing */
} mcu_tc_epilogue;
size_t mcu_matmul_tc_batched_scratch_bytes(int64_t B, int64_t M, int64_t K, int64_t N);
int mcu_matmul_tc_batched_kernels(int64_t B, int64_t M, int64_t K, int64_t N, int f16);
int mcu_launch_matmul_tc_batched(float* r, const float* x, const float* y, int64_t B, int64_t M, int64_t K,
                                 int64_t N, void* scratch, int* status, cudaStream_t st, int f16);
int mcu_launch_matmul_tc_ex(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                            void* scratch, int* status, cudaStream_t st, const mcu_tc_epilogue* ep, int f16);

#ifdef __cplusplus
}
#endif
#endif
