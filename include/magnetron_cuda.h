/*
 * magnetron_cuda.h - C ABI of the B200 (sm_100a) compute backend for magnetron.
 *
 * Drop-in entry points
 * --------------------
 * The unchanged magnetron core, compiled with MAG_ENABLE_CUDA, declares and
 * calls exactly these two functions (magnetron/magnetron.c:31-35, called from
 * mag_compute_device_init / mag_compute_device_destroy at :883-926).  They
 * replace the stub of the same name in magnetron/magnetron_cuda.cuh:14-15 /
 * magnetron/magnetron_cuda.cu:39-60, which returned a device whose function
 * pointers were never set.
 *
 * Extension entry points (mag_cuda_*)
 * -----------------------------------
 * Additive exports with plain pointers and sizes for what the core's API
 * cannot express (deferred-graph execution, row reductions, normalised
 * softmax, two-sided broadcast, batched matmul, fused dense layers, per-op
 * device timing).  Device pointers are f32 buffers in this device's memory;
 * work is enqueued on the device's stream (mag_cuda_stream).  Every function
 * returns 0 on success or a nonzero code (a cudaError_t value, or
 * MAG_CUDA_E_* below) and never aborts.
 */
#ifndef MAGNETRON_CUDA_H
#define MAGNETRON_CUDA_H

#include <stdint.h>
#include <stddef.h>
#include "mag_cuda_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MAG_CUDA_EXPORT __attribute__((visibility("default")))
#else
#define MAG_CUDA_EXPORT
#endif

/* Error codes beyond the cudaError_t range. */
#define MAG_CUDA_E_INVALID 10001     /* bad argument (shape, size, null) */
#define MAG_CUDA_E_DEVICE_WAIT 10002 /* a kernel's bounded wait expired (device status word) */
#define MAG_CUDA_E_UNSUPPORTED 10003 /* op not available (e.g. the reference panics with NYI) */
#define MAG_CUDA_E_SCRATCH_LIMIT 10004 /* the call needs more than the fixed scratch array holds */
#define MAG_CUDA_E_IO 10005            /* a file could not be opened, read or written */

/* ---- drop-in device interface (magnetron/magnetron_cuda.cuh:14-15) ---- */

/* Creates the CUDA compute device for a context.  The GPU is MAG_CUDA_DEVICE
 * if set, else LOCAL_RANK, else the current device.  Returns NULL when no
 * sm_100 GPU is usable, which makes the core fall back to the CPU device
 * (magnetron/magnetron.c:895-899). */
MAG_CUDA_EXPORT mag_compute_device_t* mag_init_device_cuda(mag_ctx_t* ctx);
/* Releases the device created above (all tensors must be gone). */
MAG_CUDA_EXPORT void mag_destroy_device_cuda(mag_compute_device_t* dvc);

/* ---- device handle ---- */
MAG_CUDA_EXPORT int mag_cuda_device_ordinal(mag_compute_device_t* dvc);
/* Operand split of the tensor-core matmul: f16 hi/lo with exact power-of-two row/column
 * scaling on kind::f16 (the default, twice the tensor rate), or tf32 hi/lo on kind::tf32
 * (MAG_CUDA_TC_SPLIT=tf32 at init).  Both keep 22 significant bits per operand. */
#define MAG_CUDA_TC_SPLIT_TF32 0
#define MAG_CUDA_TC_SPLIT_F16 1
MAG_CUDA_EXPORT int mag_cuda_set_tc_split(mag_compute_device_t* dvc, int split);
MAG_CUDA_EXPORT void* mag_cuda_stream(mag_compute_device_t* dvc);          /* cudaStream_t */
/* Waits for the device's stream and reports asynchronous errors: a CUDA error code, or
 * MAG_CUDA_E_DEVICE_WAIT when a kernel gave up a bounded wait since the last report (the
 * status word is then cleared). */
MAG_CUDA_EXPORT int mag_cuda_synchronize(mag_compute_device_t* dvc);
MAG_CUDA_EXPORT int mag_cuda_last_error(mag_compute_device_t* dvc);        /* sticky error of the eager path */
/* MATMUL algorithm: 0 = automatic (default, or MAG_CUDA_MATMUL=exact|tc), 1 = the
 * bit-exact CUDA-core kernel, 2 = the 3xTF32 tensor-core kernel where the shape allows. */
MAG_CUDA_EXPORT int mag_cuda_set_matmul_mode(mag_compute_device_t* dvc, int mode);
/* Bytes currently held by tensor storage of this device. */
MAG_CUDA_EXPORT size_t mag_cuda_memory_in_use(mag_compute_device_t* dvc);

/* ---- deferred graphs (no counterpart in the reference, which records
 * op_inputs in MAG_EXEC_MODE_DEFERRED but never executes them,
 * magnetron/magnetron.c:1785-1787) ---- */
/* Runs every node that root depends on, inputs first.  The first call for a
 * root captures the launch sequence into a CUDA graph; later calls with the
 * same node set replay it.  Returns after enqueueing (asynchronous). */
MAG_CUDA_EXPORT int mag_cuda_graph_exec(mag_compute_device_t* dvc, mag_tensor_t* root);
/* As mag_cuda_graph_exec, and fuses dense layers, MATMUL -> ADD(same-shape bias)
 * [-> GELU], into one tensor-core GEMM per layer (bias, GELU and the next
 * layer's operand split in its epilogue).  Products below the tensor-core
 * threshold fuse MATMUL -> ADD(same-shape bias, or one broadcast along dim 0)
 * [-> GELU or SIGMOID] into the bit-exact kernel's store, with the same bits as
 * the separate ops (activations only when dim 0 is a multiple of 4).  After the
 * call the root and every tensor outside such chains hold their values; the
 * MATMUL and ADD results inside a fused chain are not written. */
MAG_CUDA_EXPORT int mag_cuda_graph_exec_fused(mag_compute_device_t* dvc, mag_tensor_t* root);
/* Drops the cached graphs of root (call before freeing the graph's tensors). */
MAG_CUDA_EXPORT int mag_cuda_graph_release(mag_compute_device_t* dvc, mag_tensor_t* root);
/* Executes one node eagerly, exactly as eager_exec_fwd would. */
MAG_CUDA_EXPORT int mag_cuda_exec_node(mag_compute_device_t* dvc, mag_tensor_t* node);

/* ---- plain-pointer forms of the core's ops (same arithmetic as eager_exec_fwd) ---- */
/* Unary / scalar op (op = MAG_ABI_OP_*), rows x cols, row starts at ri*r_s1 / ri*x_s1. */
MAG_CUDA_EXPORT int mag_cuda_unary_f32(mag_compute_device_t* dvc, int op, float* r, const float* x, int64_t rows,
                                       int64_t cols, int64_t r_s1, int64_t x_s1, float xi);
/* Binary tiling-broadcast op, shapes and strides in elements, 6 entries each. */
MAG_CUDA_EXPORT int mag_cuda_binary_f32(mag_compute_device_t* dvc, int op, float* r, const float* x,
                                        const float* y, const int64_t* x_dims, const int64_t* x_strides,
                                        const int64_t* r_strides, const int64_t* y_dims, const int64_t* y_strides);
/* Full reduction (SUM/MEAN/MIN/MAX) of a 6-D tensor into r[0]. */
MAG_CUDA_EXPORT int mag_cuda_reduce_f32(mag_compute_device_t* dvc, int op, float* r, const float* x,
                                        const int64_t* x_dims, const int64_t* x_strides);
/* Sharded full reduction (no counterpart in the reference, whose reductions run on one host
 * thread: mag_blas_{sum,mean,min,max}_f32, magnetron/magnetron_cpu.c:1034-1152).  Each shard
 * writes one 24-byte record to device memory; the records of all shards (gathered in shard
 * order, e.g. by an all-gather) combine into r[0]: the double sums added in record order and
 * rounded to f32 once, MEAN = that sum / total count, MIN/MAX by fminf/fmaxf.  One record
 * equals mag_cuda_reduce_f32 on the same tensor bit for bit.  Records must be 8-byte aligned. */
typedef struct mag_cuda_reduce_part {
    double sum;
    float min, max;
    uint64_t count;
} mag_cuda_reduce_part;
MAG_CUDA_EXPORT int mag_cuda_reduce_partial_f32(mag_compute_device_t* dvc, mag_cuda_reduce_part* part_device,
                                                const float* x, const int64_t* x_dims, const int64_t* x_strides);
MAG_CUDA_EXPORT int mag_cuda_reduce_combine_f32(mag_compute_device_t* dvc, int op, float* r,
                                                const mag_cuda_reduce_part* parts_device, int nparts);
/* R[M,N] = X[M,K] Y[K,N], all row-major. */
MAG_CUDA_EXPORT int mag_cuda_matmul_f32(mag_compute_device_t* dvc, float* r, const float* x, const float* y,
                                        int64_t M, int64_t K, int64_t N);

/* ---- extensions beyond the core's API ---- */
/* r[i] = x[i mod x_d] (op) y[i mod y_d] per dim; r_dims[k] must be a multiple of both. */
MAG_CUDA_EXPORT int mag_cuda_broadcast2_f32(mag_compute_device_t* dvc, int op, float* r, const float* x,
                                            const float* y, const int64_t* r_dims, const int64_t* x_dims,
                                            const int64_t* y_dims);
/* Per-row SUM/MEAN/MIN/MAX of a rows x cols row-major matrix into r[rows]. */
MAG_CUDA_EXPORT int mag_cuda_reduce_rows_f32(mag_compute_device_t* dvc, int op, float* r, const float* x,
                                             int64_t rows, int64_t cols);
/* Normalised softmax of each row: exp(x - max) / sum, the sum accumulated in double, exp from
 * CUDA's expf (within 2 ulp; the reference has no row softmax, only the elementwise exp op). */
MAG_CUDA_EXPORT int mag_cuda_softmax_rows_f32(mag_compute_device_t* dvc, float* r, const float* x, int64_t rows,
                                              int64_t cols);
/* R[b] = X[b] Y[b] for b < batch, each M x K times K x N (tensor cores for large products,
 * the bit-exact CUDA-core kernel otherwise or under matmul mode 1).  Batches longer than 65535
 * products run as consecutive slices of 65535. */
MAG_CUDA_EXPORT int mag_cuda_matmul_batched_f32(mag_compute_device_t* dvc, float* r, const float* x,
                                                const float* y, int64_t batch, int64_t M, int64_t K, int64_t N);

/* ---- asynchronous host copies (no counterpart in the reference, whose storage copies are
 * synchronous: magnetron/magnetron.c:1820-1824) ----
 * Queue a copy between pinned host memory and a tensor's storage on the device's copy
 * stream, so it overlaps kernels queued on the compute stream.  The copy starts after all
 * work queued on the compute stream before the call (which still sees the old contents);
 * every later op, graph replay or storage callback that touches the tensor waits for it.
 * host must be pinned (cudaHostAlloc / cudaHostRegister) and must stay untouched until the
 * copy has finished: mag_cuda_copies_synchronize, or any host read of the tensor.  An upload
 * shorter than the buffer leaves the rest zero.  Returns MAG_CUDA_E_INVALID for pageable
 * memory, a foreign pointer, a size beyond the buffer, or during a graph capture. */
MAG_CUDA_EXPORT int mag_cuda_tensor_upload_async(mag_compute_device_t* dvc, mag_tensor_t* t, const void* src,
                                                 size_t bytes);
MAG_CUDA_EXPORT int mag_cuda_tensor_download_async(mag_compute_device_t* dvc, mag_tensor_t* t, void* dst,
                                                   size_t bytes);
/* Waits for every queued asynchronous host copy of the device. */
MAG_CUDA_EXPORT int mag_cuda_copies_synchronize(mag_compute_device_t* dvc);

/* ---- seeded fills on the device ----
 * The core fills tensors on the host only (magnetron/magnetron.c:1826-1876 assert a
 * CPU context).  These generate the same PCG stream on the device: *state and inc are
 * the context's PCG state (magnetron/magnetron.c:779-790, seeded as at :805-808), the
 * values equal what mag_prng_generate_n would write from *state, and on return *state
 * has advanced by n steps, as the host generator would leave it.
 * Uniform: min + (max - min) * u, bit-identical to the host stream
 * (mag_tensor_fill_random_uniform, magnetron/magnetron.c:1844-1854).
 * Normal: Box-Muller pairs over the uniform(0, 1) stream, n even
 * (mag_tensor_fill_random_normal, magnetron/magnetron.c:1856-1876); log, sin and cos
 * are rounded once from f64, so a value can differ from the host libm's by its
 * rounding (a few ulp of the pair's magnitude). */
MAG_CUDA_EXPORT int mag_cuda_fill_uniform_pcg_f32(mag_compute_device_t* dvc, float* r, int64_t n, float min,
                                                  float max, uint64_t* state, uint64_t inc);
MAG_CUDA_EXPORT int mag_cuda_fill_normal_pcg_f32(mag_compute_device_t* dvc, float* r, int64_t n, float mean,
                                                 float stddev, uint64_t* state, uint64_t inc);
/* The same fills from the context's Mersenne-twister stream, the reference's default algorithm
 * (magnetron/magnetron.c:751-777, seeded at :800-805; mag_ctx_create2 zeroes the algorithm
 * field, :951).  mt points at the context's {remaining, next, state[624]}
 * (magnetron/magnetron_internal.h:398-402; 626 uint32 words).  The values equal what
 * mag_prng_generate_n would write from that state, and on return it holds what the host
 * generator would leave: the block of the last word drawn, next and remaining.  A fill that
 * draws past the current block reads that block back, so it waits for the device's stream.
 * MAG_CUDA_E_INVALID for a state the host generator cannot be in (remaining outside 1..624, or
 * next + remaining - 1 past the block). */
MAG_CUDA_EXPORT int mag_cuda_fill_uniform_mt19937_f32(mag_compute_device_t* dvc, float* r, int64_t n, float min,
                                                      float max, uint32_t* mt);
MAG_CUDA_EXPORT int mag_cuda_fill_normal_mt19937_f32(mag_compute_device_t* dvc, float* r, int64_t n, float mean,
                                                     float stddev, uint32_t* mt);
/* Host arithmetic behind those fills, for checking without a device: out = the 624-word window
 * d words after win (win at least one block into a stream), by the jump polynomials the fills
 * use; and the degree of the stream's minimal polynomial (0 if it could not be found). */
MAG_CUDA_EXPORT int mag_cuda_mt19937_jump(const uint32_t* win, uint64_t d, uint32_t* out);
MAG_CUDA_EXPORT int mag_cuda_mt19937_degree(void);
/* r[0..n) = x (mag_tensor_fill, magnetron/magnetron.c:1826-1842, for any x). */
MAG_CUDA_EXPORT int mag_cuda_fill_f32(mag_compute_device_t* dvc, float* r, int64_t n, float x);

/* ---- .magnetron storage with device-resident data ----
 * The storage v1 format of magnetron/magnetron.c:2688-3011, byte for byte.  The reference
 * serialises only CPU tensors (:2878, :2912 assert a CPU context); these stream tensor data
 * between the file and device memory in pinned chunks on several host threads.
 * Paths must end in ".magnetron" (mag_sto_has_mag_ext, :2925-2929).  Where the reference
 * panics (I/O failure, truncated data) these return MAG_CUDA_E_IO / MAG_CUDA_E_INVALID. */
typedef struct mag_cuda_sto_entry {
    char name[64];   /* MAG_MAX_TENSOR_NAME_LEN bytes, NUL forced at [63] as the reader does */
    uint32_t flags;  /* tensor flags, 4 bits */
    uint32_t dtype;  /* 0 = f32 */
    int64_t rank;    /* 1..6 */
    int64_t shape[6];
    uint64_t offset; /* byte offset of the tensor's data in the file */
    uint64_t bytes;  /* bytes of data */
} mag_cuda_sto_entry;

/* The reader's header checks (mag_sto_read_buffered, :2891-2916) over the first `avail`
 * bytes of a file of `total` bytes; the first min(cap, count) entries are filled. */
MAG_CUDA_EXPORT int mag_cuda_sto_parse(const void* buf, size_t avail, size_t total, mag_cuda_sto_entry* entries,
                                       uint32_t cap, uint32_t* n_tensors, uint32_t* version);
/* The file header and tensor headers the writer emits for these tensors
 * (mag_sto_write_buffered, :2861-2876); *size receives the header bytes. */
MAG_CUDA_EXPORT int mag_cuda_sto_write_header(const mag_tensor_t* const* tensors, uint32_t n, void* buf, size_t cap,
                                              size_t* size);
/* mag_tensor_save (:2931-2950) for n >= 1 tensors whose storage is on this device. */
MAG_CUDA_EXPORT int mag_cuda_tensor_save(mag_compute_device_t* dvc, const char* path,
                                         const mag_tensor_t* const* tensors, uint32_t n);
/* The header phase of mag_tensor_load (:2952-2977): the file's tensor directory. */
MAG_CUDA_EXPORT int mag_cuda_sto_read_directory(const char* path, mag_cuda_sto_entry* entries, uint32_t cap,
                                                uint32_t* n_tensors, uint32_t* version);
/* The data phase: the first n stored tensors into device tensors of the stored dtype, rank
 * and shape, whose name and flags are then set from the file as the reader does (:2907-2908). */
MAG_CUDA_EXPORT int mag_cuda_tensor_load(mag_compute_device_t* dvc, const char* path, mag_tensor_t* const* tensors,
                                         uint32_t n);

/* ---- image tensors on the device ----
 * An image tensor is rank 3, shape (c, h, w), planar f32 (magnetron/magnetron.h:394-396).
 * Results are bit-identical with the reference's CPU code for the same pixels. */
/* The pixel work of mag_tensor_load_image (magnetron/magnetron.c:3013-3087): interleaved u8
 * [h][w][c] (host or device memory, as the image decoder returns it) -> dst / 255, resized
 * to rw x rh by the reference's two-pass bilinear scheme when both are nonzero.  dst has shape
 * (c, rh, rw) or (c, h, w). */
MAG_CUDA_EXPORT int mag_cuda_img_from_u8(mag_compute_device_t* dvc, mag_tensor_t* dst, const uint8_t* src, uint32_t w,
                                         uint32_t h, uint32_t c, uint32_t rw, uint32_t rh);
/* The pixel work of mag_tensor_save_image (:3089-3109): interleaved u8 [h][w][c] of
 * (uint8_t)(x * 255) with x86 conversion semantics, into host or device memory; c in {1, 3, 4}. */
MAG_CUDA_EXPORT int mag_cuda_img_to_u8(mag_compute_device_t* dvc, const mag_tensor_t* src, uint8_t* dst);
/* mag_tensor_img_draw_box (:2159-2214) on a 3-channel image. */
MAG_CUDA_EXPORT int mag_cuda_img_draw_box(mag_compute_device_t* dvc, mag_tensor_t* t, int32_t x1, int32_t y1,
                                          int32_t x2, int32_t y2, int32_t wi, uint32_t rgb);
/* mag_tensor_img_draw_text (:2243-2270) on a 3-channel image; size is ignored, as there. */
MAG_CUDA_EXPORT int mag_cuda_img_draw_text(mag_compute_device_t* dvc, mag_tensor_t* t, int32_t x, int32_t y,
                                           int32_t size, uint32_t rgb, const char* txt);

/* ---- allocation-free entry point (no counterpart in the reference) ----
 * R[M,N] = X[M,K] Y[K,N] for 1 <= M <= 16, the same split-K kernels as
 * mag_cuda_matmul_f32 uses for such shapes, but it never allocates: for callers
 * that cannot call cudaMalloc when they need the product, such as a
 * latency-critical host path that must not enter the CUDA allocator (which can
 * block or synchronise) or code under a memory budget fixed up front.  Its
 * partial sums go to one fixed 16 MiB array in this library's device image,
 * which every GPU that loads the library keeps until the process exits.  Calls
 * needing more (slices x M x N x 4 bytes) return MAG_CUDA_E_SCRATCH_LIMIT.  On a
 * 148-SM B200 an M x 4096 x 4096 product takes 128 slices, 2 MiB per row of M:
 * M = 1..8 fits (M = 8 fills the array exactly) and M = 9..16 is rejected at that
 * size.  The first call on a device looks up the array's device address, so make
 * it before any stream capture; the address is kept for the life of the process,
 * so the entry point does not survive cudaDeviceReset.  All calls on a device
 * share the array: calls whose kernels overlap on the GPU race. */
MAG_CUDA_EXPORT int mag_cuda_matmul_skinny_f32_noalloc(mag_compute_device_t* dvc, float* r, const float* x,
                                                       const float* y, int64_t M, int64_t K, int64_t N);
/* Bytes of the fixed scratch array above. */
MAG_CUDA_EXPORT size_t mag_cuda_matmul_skinny_noalloc_limit(void);

/* ---- per-op device timing (the core's profiler times only the enqueue) ---- */
MAG_CUDA_EXPORT int mag_cuda_profile_start(mag_compute_device_t* dvc);
/* Adds the device time of every op finished so far (eager ops and the op
 * event nodes of graphs captured while profiling) to the per-op totals. */
MAG_CUDA_EXPORT int mag_cuda_profile_collect(mag_compute_device_t* dvc);
/* Per-op totals: executions and device microseconds. */
MAG_CUDA_EXPORT int mag_cuda_profile_stats(mag_compute_device_t* dvc, int op, uint64_t* count, double* total_us);
/* Collects, then prints or writes (csv_path != NULL) per-op device time in the
 * core's table layout (magnetron/magnetron.c:1093-1111), and stops. */
MAG_CUDA_EXPORT int mag_cuda_profile_stop(mag_compute_device_t* dvc, const char* csv_path);

/* Number of kernels this library launched since load (launch accounting). */
MAG_CUDA_EXPORT uint64_t mag_cuda_kernel_launches(void);

#ifdef __cplusplus
}
#endif
#endif /* MAGNETRON_CUDA_H */
