/*
 * device.c - the CUDA compute device behind the magnetron core (host side, C).
 *
 * Implements mag_compute_device_t (magnetron/magnetron_internal.h:336-346) for
 * one sm_100 GPU:
 *   - storage: a stream-ordered arena (cudaMallocAsync from the device's
 *     default pool with an unbounded release threshold, so freed blocks are
 *     reused without returning to the driver); host<->device copies through a
 *     double-buffered pinned staging ring, or straight DMA when the host
 *     buffer is already pinned;
 *   - zero-on-allocation: the CPU backend memsets every new buffer
 *     (magnetron/magnetron_cpu.c:2336-2349) and MATMUL/reductions rely on it.
 *     Here a new buffer is marked "zero pending" and cleared only if it is
 *     read, partially written or read back before a full overwrite, which
 *     saves 4 B/elem of HBM writes on every elementwise result;
 *   - eager execution: eager_exec_fwd enqueues the op's kernels on the
 *     device's single stream and returns (is_async = true); every host-visible
 *     read synchronises;
 *   - deferred graphs: mag_cuda_graph_exec walks op_inputs post-order and
 *     captures the launches into a CUDA graph, replayed on later calls.
 * Errors panic like mag_panic (print, abort) on the core-facing callbacks,
 * which have no error return, and return codes on the mag_cuda_* exports.
 */
#include "mag_cuda_abi.h"
#include "magnetron_cuda.h"
#include "mcu_device.h"
#include "mcu_kernels.h"

#include <cuda_runtime_api.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <stdatomic.h>

#define MCU_STAGE_BYTES ((size_t)32 << 20)
#define MCU_STAGE_SLOTS 2

/* ------------------------------------------------------------ errors --- */

static void mcu_panic(const char* fmt, ...) __attribute__((noreturn, format(printf, 1, 2)));
static void mcu_panic(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "[magnetron-cuda] panic: ");
    vfprintf(stderr, fmt, ap);
    fputc('\n', stderr);
    va_end(ap);
    fflush(stderr);
    abort();
}

#define MCU_CHECK(expr)                                                                   \
    do {                                                                                  \
        cudaError_t e_ = (cudaError_t)(expr);                                             \
        if (e_ != cudaSuccess)                                                            \
            mcu_panic("%s:%d %s failed: %s", __FILE__, __LINE__, #expr, cudaGetErrorString(e_)); \
    } while (0)

_Atomic uint64_t mcu_launch_counter = 0;
void mcu_count_launches(int n) { atomic_fetch_add(&mcu_launch_counter, (uint64_t)n); }
uint64_t mag_cuda_kernel_launches(void) { return atomic_load(&mcu_launch_counter); }

/* ------------------------------------------------------- device state --- */

typedef struct mcu_block {
    uintptr_t base;
    size_t size;
    uint8_t zero_pending; /* contents are zero by contract, the memset is not issued yet */
    uint8_t known_zero;   /* nothing has written the buffer since it was zeroed */
    uint8_t state;        /* 0 empty, 1 live, 2 deleted */
    uint8_t io_pending;   /* an async copy on the copy stream touches the buffer: io_ev marks its end */
    cudaEvent_t io_ev;
} mcu_block;

typedef struct mcu_graph {
    mag_tensor_t* root;
    int fused;
    uint64_t sig;
    size_t n_nodes;
    cudaGraphExec_t exec;
    void* scratch;
    /* event-record nodes around each op, present when captured while profiling */
    size_t n_ev;
    int* ev_op;
    cudaEvent_t* ev_a;
    cudaEvent_t* ev_b;
    int ran;
    uint64_t n_kernels; /* kernels one replay launches */
    struct mcu_graph* next;
} mcu_graph;

typedef struct mcu_prof_rec {
    int op;
    cudaEvent_t a, b;
} mcu_prof_rec;

typedef struct mcu_device {
    mag_compute_device_t* iface;
    int ordinal;
    int sm_count;
    cudaStream_t stream;
    cudaStream_t copy_stream; /* async uploads/downloads, ordered after the compute stream's tail */
    cudaEvent_t tail_ev;
    int managed;      /* MAG_CUDA_MANAGED=1: unified memory, synchronous ops */
    int eager_zero;   /* MAG_CUDA_EAGER_ZERO=1: memset on allocation */
    int matmul_mode;  /* MAG_CUDA_MATMUL: 0 auto, 1 exact, 2 tensor cores */
    int tc_f16;       /* tensor-core split: 1 scaled f16 (kind::f16), 0 tf32 (MAG_CUDA_TC_SPLIT=tf32) */
    int sticky_error;
    int capturing;
    mcu_block* tab;
    size_t tab_cap, tab_live, tab_used;
    size_t bytes_live;
    void* stage[MCU_STAGE_SLOTS];
    cudaEvent_t stage_ev[MCU_STAGE_SLOTS];
    int stage_next;
    void* scratch;
    size_t scratch_bytes;
    int* d_status;
    mcu_graph* graphs;
    void* graph_scratch; /* scratch of the graph being captured */
    int profiling;
    mcu_prof_rec* prof;
    size_t prof_n, prof_cap;
    double prof_us[MAG_ABI_OP__COUNT];
    uint64_t prof_cnt[MAG_ABI_OP__COUNT];
} mcu_device;

static mcu_device* dev_of(mag_compute_device_t* dvc) { return (mcu_device*)dvc->impl; }
static float* fptr(const mag_tensor_t* t) { return (float*)t->storage.base; }

/* ---------------------------------------------- block table (by base) --- */

static size_t hash_ptr(uintptr_t p, size_t cap) {
    uint64_t h = (uint64_t)p * 0x9E3779B97F4A7C15ull;
    return (size_t)(h >> 17) & (cap - 1);
}

static void tab_insert(mcu_device* d, uintptr_t base, size_t size, int zero_pending, int known_zero);
static mcu_block* tab_find(mcu_device* d, uintptr_t base);

static void tab_grow(mcu_device* d) {
    size_t old_cap = d->tab_cap;
    mcu_block* old = d->tab;
    d->tab_cap = old_cap ? old_cap * 2 : 1024;
    d->tab = (mcu_block*)calloc(d->tab_cap, sizeof(mcu_block));
    if (!d->tab) mcu_panic("out of host memory");
    d->tab_live = d->tab_used = 0;
    for (size_t i = 0; i < old_cap; ++i) {
        if (old[i].state != 1) continue;
        tab_insert(d, old[i].base, old[i].size, old[i].zero_pending, old[i].known_zero);
        mcu_block* nb = tab_find(d, old[i].base);
        nb->io_pending = old[i].io_pending;
        nb->io_ev = old[i].io_ev;
    }
    free(old);
}

static void tab_insert(mcu_device* d, uintptr_t base, size_t size, int zero_pending, int known_zero) {
    if ((d->tab_used + 1) * 2 > d->tab_cap) tab_grow(d);
    size_t i = hash_ptr(base, d->tab_cap);
    while (d->tab[i].state == 1) i = (i + 1) & (d->tab_cap - 1);
    if (d->tab[i].state == 0) d->tab_used++;
    d->tab[i] = (mcu_block){base, size, (uint8_t)zero_pending, (uint8_t)known_zero, 1, 0, NULL};
    d->tab_live++;
}

static mcu_block* tab_find(mcu_device* d, uintptr_t base) {
    if (!d->tab_cap) return NULL;
    size_t i = hash_ptr(base, d->tab_cap);
    while (d->tab[i].state != 0) {
        if (d->tab[i].state == 1 && d->tab[i].base == base) return &d->tab[i];
        i = (i + 1) & (d->tab_cap - 1);
    }
    return NULL;
}

/* The compute stream waits for an async copy of the buffer still in flight on the copy
 * stream (mag_cuda_tensor_upload_async / _download_async) before touching it.  Graph
 * captures never contain such a wait: pending copies are waited for before a capture
 * and before each replay. */
static void io_wait(mcu_device* d, mcu_block* b) {
    if (!b || !b->io_pending || d->capturing) return;
    MCU_CHECK(cudaStreamWaitEvent(d->stream, b->io_ev, 0));
    b->io_pending = 0;
}

/* Clears a pending buffer before its first read or partial write. */
static void materialize(mcu_device* d, uintptr_t base) {
    mcu_block* b = tab_find(d, base);
    io_wait(d, b);
    if (b && b->zero_pending) {
        MCU_CHECK(cudaMemsetAsync((void*)b->base, 0, b->size, d->stream));
        b->zero_pending = 0;
    }
}

/* The op about to run overwrites every byte of the buffer: no clear needed. */
static void overwritten(mcu_device* d, uintptr_t base) {
    mcu_block* b = tab_find(d, base);
    io_wait(d, b);
    if (b) b->zero_pending = b->known_zero = 0;
}

/* The op about to run writes part of the buffer: the rest must read as zero. */
static void partly_written(mcu_device* d, uintptr_t base) {
    materialize(d, base);
    mcu_block* b = tab_find(d, base);
    if (b) b->known_zero = 0;
}

static void result_written(mcu_device* d, uintptr_t base, int full) {
    if (full) overwritten(d, base);
    else partly_written(d, base);
}

/* --------------------------------------------------------- storage ---- */

static mcu_device* dev_of_storage(mag_storage_buffer* sto) { return dev_of(sto->host); }

static int host_is_pinned(const void* p) {
    struct cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeManaged;
}

static void check_status(mcu_device* d) {
    int st = 0;
    MCU_CHECK(cudaMemcpy(&st, d->d_status, sizeof(int), cudaMemcpyDeviceToHost));
    if (st) mcu_panic("a kernel on device %d gave up a bounded wait (status %d)", d->ordinal, st);
}

static void sto_set(mag_storage_buffer* sto, size_t offs, uint8_t x) {
    mcu_device* d = dev_of_storage(sto);
    if (offs > sto->size) mcu_panic("set: offset %zu beyond buffer of %zu bytes", offs, sto->size);
    if (offs == 0 && x == 0 && !d->eager_zero && !d->managed && !d->capturing) {
        mcu_block* b = tab_find(d, sto->base);
        io_wait(d, b);
        if (b) {
            b->zero_pending = b->known_zero = 1;
            return;
        }
    }
    partly_written(d, sto->base);
    MCU_CHECK(cudaMemsetAsync((void*)(sto->base + offs), x, sto->size - offs, d->stream));
    if (d->managed) MCU_CHECK(cudaStreamSynchronize(d->stream));
}

static void sto_cpy_host_device(mag_storage_buffer* sto, size_t offs, const void* src, size_t n) {
    mcu_device* d = dev_of_storage(sto);
    if (offs + n > sto->size) mcu_panic("host->device copy of %zu bytes at %zu overflows %zu", n, offs, sto->size);
    if (!n) return;
    result_written(d, sto->base, offs == 0 && n == sto->size);
    char* dst = (char*)(sto->base + offs);
    if (host_is_pinned(src) || n <= 65536) {
        MCU_CHECK(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, d->stream));
        MCU_CHECK(cudaStreamSynchronize(d->stream)); /* the caller may reuse src on return */
        return;
    }
    /* pageable source: copy through the pinned ring; DMA overlaps the next memcpy */
    const char* s = (const char*)src;
    for (size_t off = 0; off < n; off += MCU_STAGE_BYTES) {
        size_t len = n - off < MCU_STAGE_BYTES ? n - off : MCU_STAGE_BYTES;
        int slot = d->stage_next;
        d->stage_next = (slot + 1) % MCU_STAGE_SLOTS;
        MCU_CHECK(cudaEventSynchronize(d->stage_ev[slot]));
        memcpy(d->stage[slot], s + off, len);
        MCU_CHECK(cudaMemcpyAsync(dst + off, d->stage[slot], len, cudaMemcpyHostToDevice, d->stream));
        MCU_CHECK(cudaEventRecord(d->stage_ev[slot], d->stream));
    }
}

static void sto_cpy_device_host(mag_storage_buffer* sto, size_t offs, void* dst, size_t n) {
    mcu_device* d = dev_of_storage(sto);
    if (offs + n > sto->size) mcu_panic("device->host copy of %zu bytes at %zu overflows %zu", n, offs, sto->size);
    if (!n) return;
    mcu_block* b = tab_find(d, sto->base);
    io_wait(d, b);
    if (b && b->zero_pending) { /* never written: the contents are zero by contract */
        memset(dst, 0, n);
        return;
    }
    const char* src = (const char*)(sto->base + offs);
    if (host_is_pinned(dst) || n <= 65536) {
        MCU_CHECK(cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, d->stream));
        MCU_CHECK(cudaStreamSynchronize(d->stream));
    } else {
        char* o = (char*)dst;
        for (size_t off = 0; off < n; off += MCU_STAGE_BYTES) {
            size_t len = n - off < MCU_STAGE_BYTES ? n - off : MCU_STAGE_BYTES;
            int slot = d->stage_next;
            d->stage_next = (slot + 1) % MCU_STAGE_SLOTS;
            MCU_CHECK(cudaMemcpyAsync(d->stage[slot], src + off, len, cudaMemcpyDeviceToHost, d->stream));
            MCU_CHECK(cudaEventRecord(d->stage_ev[slot], d->stream));
            MCU_CHECK(cudaEventSynchronize(d->stage_ev[slot]));
            memcpy(o + off, d->stage[slot], len);
        }
    }
    check_status(d);
}

static void dvc_alloc_storage(mag_compute_device_t* dvc, mag_storage_buffer* out, size_t size, size_t align) {
    mcu_device* d = dev_of(dvc);
    if (!size) mcu_panic("storage size must be nonzero");
    if (align > 256) mcu_panic("alignment %zu above 256 bytes is not supported", align);
    void* p = NULL;
    if (d->managed) {
        MCU_CHECK(cudaMallocManaged(&p, size, cudaMemAttachGlobal));
        MCU_CHECK(cudaMemset(p, 0, size));
        MCU_CHECK(cudaDeviceSynchronize());
    } else {
        cudaError_t e = cudaMallocAsync(&p, size, d->stream);
        if (e != cudaSuccess) mcu_panic("device allocation of %zu bytes failed: %s", size, cudaGetErrorString(e));
        if (d->eager_zero) MCU_CHECK(cudaMemsetAsync(p, 0, size, d->stream));
    }
    tab_insert(d, (uintptr_t)p, size, !(d->managed || d->eager_zero), 1);
    d->bytes_live += size;
    *out = (mag_storage_buffer){
        .base = (uintptr_t)p,
        .size = size,
        .alignment = align,
        .host = dvc,
        .set = &sto_set,
        .cpy_host_device = &sto_cpy_host_device,
        .cpy_device_host = &sto_cpy_device_host,
    };
}

static void dvc_free_storage(mag_compute_device_t* dvc, mag_storage_buffer* buf) {
    mcu_device* d = dev_of(dvc);
    mcu_block* b = tab_find(d, buf->base);
    io_wait(d, b); /* the stream-ordered free follows any copy still in flight */
    if (b && b->io_ev) {
        cudaEventDestroy(b->io_ev);
        b->io_ev = NULL;
    }
    if (b) {
        b->state = 2;
        d->tab_live--;
        d->bytes_live -= b->size;
    }
    if (buf->base) {
        if (d->managed) {
            MCU_CHECK(cudaDeviceSynchronize());
            MCU_CHECK(cudaFree((void*)buf->base));
        } else {
            MCU_CHECK(cudaFreeAsync((void*)buf->base, d->stream));
        }
    }
    memset(buf, 0, sizeof(*buf));
}

/* ------------------------------------------------------------ scratch --- */

static void* scratch_get(mcu_device* d, size_t bytes) {
    if (d->capturing) {
        if (!d->graph_scratch || bytes > d->scratch_bytes) mcu_panic("graph scratch undersized (%zu bytes)", bytes);
        return d->graph_scratch;
    }
    if (bytes <= d->scratch_bytes && d->scratch) return d->scratch;
    if (d->scratch) MCU_CHECK(cudaFreeAsync(d->scratch, d->stream));
    size_t sz = bytes < ((size_t)1 << 20) ? ((size_t)1 << 20) : bytes;
    MCU_CHECK(cudaMallocAsync(&d->scratch, sz, d->stream));
    d->scratch_bytes = sz;
    return d->scratch;
}

/* ------------------------------------------------------------- ops ---- */

static int64_t rows_of(const mag_tensor_t* t) {
    return t->shape[1] * t->shape[2] * t->shape[3] * t->shape[4] * t->shape[5];
}

static int is_canonical(const mag_tensor_t* t) {
    int64_t acc = 1;
    for (int k = 0; k < 6; ++k) {
        if (t->shape[k] != 1 && t->strides[k] != acc) return 0;
        acc *= t->shape[k];
    }
    return 1;
}

static int64_t data_bytes(const mag_tensor_t* t) { return t->numel * 4; }

enum { MM_EXACT, MM_SKINNY, MM_TC };

static int matmul_path(mcu_device* d, int64_t M, int64_t K, int64_t N) {
    if (d->matmul_mode == 1) return MM_EXACT;
    int tc_ok = mcu_matmul_tc_supported() && M >= 32 && N >= 64 && K >= 32 && K <= MCU_TC_MAX_K &&
                M < ((int64_t)1 << 31) && N < ((int64_t)1 << 31);
    if (d->matmul_mode == 2 && tc_ok) return MM_TC;
    if (M < 32 && K * N >= ((int64_t)1 << 20)) return MM_SKINNY; /* HBM-bound: Y is read once */
    if (tc_ok && (double)M * (double)N * (double)K >= 1.0e9) return MM_TC; /* split K fills the GPU */
    if (M <= 64 && K * N >= ((int64_t)1 << 20)) return MM_SKINNY;
    return MM_EXACT;
}

static size_t node_scratch_bytes(mcu_device* d, const mag_tensor_t* r) {
    switch (r->op) {
        case MAG_ABI_OP_MEAN: case MAG_ABI_OP_MIN: case MAG_ABI_OP_MAX: case MAG_ABI_OP_SUM:
            return mcu_reduce_scratch_bytes();
        case MAG_ABI_OP_MATMUL: {
            const mag_tensor_t* x = r->op_inputs[0];
            const mag_tensor_t* y = r->op_inputs[1];
            int64_t M = x->shape[0], K = x->shape[1], N = y->shape[1];
            size_t extra = 0;
            if (r->storage.base == x->storage.base) extra += (size_t)data_bytes(x);
            if (r->storage.base == y->storage.base) extra += (size_t)data_bytes(y);
            int path = matmul_path(d, M, K, N);
            if (path == MM_SKINNY) return extra + mcu_matmul_skinny_scratch_bytes(M, K, N);
            if (path == MM_TC) return extra + mcu_matmul_tc_scratch_bytes(M, K, N);
            return extra;
        }
        default:
            return 0;
    }
}

/* Enqueues one op node.  Returns 0 or an error code. */
static int exec_node(mcu_device* d, mag_tensor_t* r) {
    const int op = r->op;
    mag_tensor_t* x = r->op_inputs[0];
    mag_tensor_t* y = r->op_inputs[1];
    cudaStream_t st = d->stream;
    int rc = 0;
    switch (op) {
        case MAG_ABI_OP_NOP: case MAG_ABI_OP_VIEW: case MAG_ABI_OP_TRANSPOSE: case MAG_ABI_OP_PERMUTE:
            return 0; /* metadata only (magnetron/magnetron_cpu.c:2228-2232) */
        case MAG_ABI_OP_CLONE: { /* memcpy of the data size (magnetron/magnetron_cpu.c:1022-1032) */
            materialize(d, x->storage.base);
            size_t n = (size_t)data_bytes(r);
            result_written(d, r->storage.base, n == r->storage.size);
            if (r->storage.base != x->storage.base && n)
                rc = cudaMemcpyAsync((void*)r->storage.base, (const void*)x->storage.base, n,
                                     cudaMemcpyDeviceToDevice, st);
            return rc;
        }
        case MAG_ABI_OP_MEAN: case MAG_ABI_OP_MIN: case MAG_ABI_OP_MAX: case MAG_ABI_OP_SUM: {
            materialize(d, x->storage.base);
            if (d->capturing && !(r->numel == 1 && r->storage.size == 4))
                MCU_CHECK(cudaMemsetAsync((void*)r->storage.base, 0, r->storage.size, st));
            result_written(d, r->storage.base, r->numel == 1 && r->storage.size == 4);
            void* scratch = scratch_get(d, mcu_reduce_scratch_bytes());
            rc = mcu_launch_reduce(op, fptr(r), fptr(x), x->shape, x->strides, scratch, st);
            if (!rc) mcu_count_launches(2);
            return rc;
        }
        case MAG_ABI_OP_SILU_DV: case MAG_ABI_OP_GELU_DV:
            if (x->numel > 0) mcu_panic("NYI"); /* mag_vsilu_dv_f32 / mag_vgelu_dv_f32 panic (magnetron_cpu.c:873-881, :1002-1010) */
            return 0;
        case MAG_ABI_OP_ADD: case MAG_ABI_OP_SUB: case MAG_ABI_OP_MUL: case MAG_ABI_OP_DIV: {
            materialize(d, x->storage.base);
            materialize(d, y->storage.base);
            result_written(d, r->storage.base, is_canonical(r) && (size_t)data_bytes(r) == r->storage.size);
            rc = mcu_launch_binary(op, fptr(r), fptr(x), fptr(y), x->shape, x->strides, r->strides, y->shape,
                                   y->strides, st);
            if (!rc) mcu_count_launches(1);
            return rc;
        }
        case MAG_ABI_OP_MATMUL: {
            /* shapes as in mag_blas_matmul_f32 (magnetron/magnetron_cpu.c:2158-2170) */
            if (x->shape[2] != 1 || x->shape[3] != 1 || y->shape[2] != 1 || y->shape[3] != 1)
                mcu_panic("%s:%d Assertion failed: x_d2 == 1 && x_d3 == 1 && y_d2 == 1 && y_d3 == 1", __FILE__, __LINE__);
            const int64_t M = x->shape[0], K = x->shape[1], N = y->shape[1], r_ld = r->shape[1];
            materialize(d, x->storage.base);
            materialize(d, y->storage.base);
            const float* px = fptr(x);
            const float* py = fptr(y);
            int aliased = r->storage.base == x->storage.base || r->storage.base == y->storage.base;
            mcu_block* rb = tab_find(d, r->storage.base);
            int full = r_ld == N && (size_t)(M * N * 4) == r->storage.size;
            /* the reference accumulates into whatever R holds, which is zero for a
             * fresh result; a graph replay recomputes R from zero every time */
            int accumulate = aliased || (!d->capturing && !(rb && rb->known_zero));
            if (d->capturing && !full && !aliased)
                MCU_CHECK(cudaMemsetAsync((void*)r->storage.base, 0, r->storage.size, st));
            result_written(d, r->storage.base, full && !accumulate);
            int path = matmul_path(d, M, K, N);
            if (accumulate && path != MM_EXACT) path = MM_EXACT;
            size_t need = node_scratch_bytes(d, r);
            char* scratch = need ? (char*)scratch_get(d, need) : NULL;
            if (aliased) { /* read a snapshot of the inputs, not the progressively updated R */
                size_t off = 0;
                if (r->storage.base == x->storage.base) {
                    MCU_CHECK(cudaMemcpyAsync(scratch, px, (size_t)data_bytes(x), cudaMemcpyDeviceToDevice, st));
                    px = (const float*)scratch;
                    off += (size_t)data_bytes(x);
                }
                if (r->storage.base == y->storage.base) {
                    MCU_CHECK(cudaMemcpyAsync(scratch + off, py, (size_t)data_bytes(y), cudaMemcpyDeviceToDevice, st));
                    py = (const float*)(scratch + off);
                }
            }
            if (path == MM_SKINNY) {
                rc = mcu_launch_matmul_skinny(fptr(r), px, py, M, K, N, r_ld, scratch, st);
                if (!rc) mcu_count_launches(2);
            } else if (path == MM_TC) {
                rc = mcu_launch_matmul_tc(fptr(r), px, py, M, K, N, scratch, d->d_status, st, d->tc_f16);
                if (!rc) mcu_count_launches(mcu_matmul_tc_kernels(M, K, N, d->tc_f16, 0));
            } else {
                rc = mcu_launch_matmul_exact(fptr(r), px, py, 1, M, K, N, r_ld, accumulate, st);
                if (!rc) mcu_count_launches(mcu_matmul_exact_kernels(1, M));
            }
            return rc;
        }
        default:
            break;
    }
    if (op >= MAG_ABI_OP_ABS && op <= MAG_ABI_OP_DIVS) { /* unary and scalar ops */
        const int64_t rows = rows_of(x), cols = x->shape[0];
        materialize(d, x->storage.base);
        result_written(d, r->storage.base,
                       (r->strides[1] == cols || rows == 1) && (size_t)(rows * cols * 4) == r->storage.size);
        float xi = (op >= MAG_ABI_OP_ADDS) ? mag_abi_param_f32(r->op_params[0]) : 0.0f;
        rc = mcu_launch_unary(op, fptr(r), fptr(x), rows, cols, r->strides[1], x->strides[1], xi, st);
        if (!rc) mcu_count_launches(1);
        return rc;
    }
    mcu_panic("unsupported op %d", op);
}

static void prof_begin(mcu_device* d, int op, mcu_prof_rec** rec) {
    *rec = NULL;
    if (!d->profiling || d->capturing) return;
    if (d->prof_n == d->prof_cap) {
        d->prof_cap = d->prof_cap ? d->prof_cap * 2 : 256;
        d->prof = (mcu_prof_rec*)realloc(d->prof, d->prof_cap * sizeof(mcu_prof_rec));
        if (!d->prof) mcu_panic("out of host memory");
    }
    mcu_prof_rec* p = &d->prof[d->prof_n++];
    p->op = op;
    MCU_CHECK(cudaEventCreate(&p->a));
    MCU_CHECK(cudaEventCreate(&p->b));
    MCU_CHECK(cudaEventRecord(p->a, d->stream));
    *rec = p;
}

static void prof_end(mcu_device* d, mcu_prof_rec* p) {
    if (p) MCU_CHECK(cudaEventRecord(p->b, d->stream));
}

static void dvc_exec(mag_compute_device_t* dvc, mag_tensor_t* root) {
    mcu_device* d = dev_of(dvc);
    mcu_prof_rec* p;
    prof_begin(d, root->op, &p);
    int rc = exec_node(d, root);
    prof_end(d, p);
    if (rc) mcu_panic("op %d failed to launch: %s", root->op, cudaGetErrorString((cudaError_t)rc));
    if (d->managed) {
        MCU_CHECK(cudaStreamSynchronize(d->stream));
        check_status(d);
    }
}

/* ------------------------------------------------------ init/destroy --- */

static int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

mag_compute_device_t* mag_init_device_cuda(mag_ctx_t* ctx) {
    (void)ctx;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        cudaGetLastError();
        fprintf(stderr, "[magnetron-cuda] no CUDA devices available\n");
        return NULL;
    }
    int ordinal = -1;
    const char* sel = getenv("MAG_CUDA_DEVICE");
    if (sel && *sel) ordinal = atoi(sel);
    else if (getenv("LOCAL_RANK")) ordinal = env_int("LOCAL_RANK", 0);
    else if (cudaGetDevice(&ordinal) != cudaSuccess) ordinal = 0;
    if (ordinal < 0 || ordinal >= count) {
        fprintf(stderr, "[magnetron-cuda] invalid device %d, using device 0\n", ordinal);
        ordinal = 0;
    }
    struct cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, ordinal) != cudaSuccess) return NULL;
    if (prop.major != 10) {
        fprintf(stderr, "[magnetron-cuda] device %d (%s, sm_%d%d) is not sm_100; kernels are built for sm_100a only\n",
                ordinal, prop.name, prop.major, prop.minor);
        return NULL;
    }
    MCU_CHECK(cudaSetDevice(ordinal));
    mcu_device* d = (mcu_device*)calloc(1, sizeof(mcu_device));
    mag_compute_device_t* dvc = (mag_compute_device_t*)calloc(1, sizeof(mag_compute_device_t));
    if (!d || !dvc) mcu_panic("out of host memory");
    d->iface = dvc;
    d->ordinal = ordinal;
    d->sm_count = prop.multiProcessorCount;
    d->managed = env_int("MAG_CUDA_MANAGED", 0);
    d->eager_zero = env_int("MAG_CUDA_EAGER_ZERO", 0);
    const char* mm = getenv("MAG_CUDA_MATMUL");
    d->matmul_mode = !mm ? 0 : (!strcmp(mm, "exact") ? 1 : (!strcmp(mm, "tc") ? 2 : 0));
    const char* ts = getenv("MAG_CUDA_TC_SPLIT");
    d->tc_f16 = !(ts && !strcmp(ts, "tf32"));
    MCU_CHECK(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
    MCU_CHECK(cudaStreamCreateWithFlags(&d->copy_stream, cudaStreamNonBlocking));
    MCU_CHECK(cudaEventCreateWithFlags(&d->tail_ev, cudaEventDisableTiming));
    cudaMemPool_t pool;
    MCU_CHECK(cudaDeviceGetDefaultMemPool(&pool, ordinal));
    uint64_t thresh = UINT64_MAX;
    MCU_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thresh));
    for (int i = 0; i < MCU_STAGE_SLOTS; ++i) {
        MCU_CHECK(cudaHostAlloc(&d->stage[i], MCU_STAGE_BYTES, cudaHostAllocDefault));
        MCU_CHECK(cudaEventCreateWithFlags(&d->stage_ev[i], cudaEventDisableTiming));
        MCU_CHECK(cudaEventRecord(d->stage_ev[i], d->stream));
    }
    MCU_CHECK(cudaMalloc((void**)&d->d_status, sizeof(int)));
    MCU_CHECK(cudaMemset(d->d_status, 0, sizeof(int)));
    snprintf(dvc->name, sizeof(dvc->name), "%.96s (sm_%d%d, %d SMs)", prop.name, prop.major, prop.minor,
             prop.multiProcessorCount);
    dvc->impl = d;
    dvc->is_async = true;
    dvc->type = MAG_ABI_DEVICE_CUDA;
    dvc->eager_exec_fwd = &dvc_exec;
    dvc->eager_exec_bwd = &dvc_exec; /* the reference's backward table is a copy of forward (magnetron_cpu.c:2269-2309) */
    dvc->alloc_storage = &dvc_alloc_storage;
    dvc->free_storage = &dvc_free_storage;
    return dvc;
}

static void graph_free(mcu_graph* g) {
    cudaGraphExecDestroy(g->exec);
    if (g->scratch) cudaFree(g->scratch);
    for (size_t i = 0; i < g->n_ev; ++i) {
        cudaEventDestroy(g->ev_a[i]);
        cudaEventDestroy(g->ev_b[i]);
    }
    free(g->ev_op);
    free(g->ev_a);
    free(g->ev_b);
    free(g);
}

void mag_destroy_device_cuda(mag_compute_device_t* dvc) {
    if (!dvc) return;
    mcu_device* d = dev_of(dvc);
    cudaSetDevice(d->ordinal);
    cudaStreamSynchronize(d->stream);
    for (mcu_graph* g = d->graphs; g;) {
        mcu_graph* n = g->next;
        graph_free(g);
        g = n;
    }
    for (size_t i = 0; i < d->prof_n; ++i) {
        cudaEventDestroy(d->prof[i].a);
        cudaEventDestroy(d->prof[i].b);
    }
    free(d->prof);
    if (d->scratch) cudaFreeAsync(d->scratch, d->stream);
    for (int i = 0; i < MCU_STAGE_SLOTS; ++i) {
        cudaEventSynchronize(d->stage_ev[i]);
        cudaEventDestroy(d->stage_ev[i]);
        cudaFreeHost(d->stage[i]);
    }
    cudaStreamSynchronize(d->stream);
    cudaFree(d->d_status);
    cudaStreamSynchronize(d->copy_stream);
    for (size_t i = 0; i < d->tab_cap; ++i)
        if (d->tab[i].io_ev) cudaEventDestroy(d->tab[i].io_ev);
    cudaEventDestroy(d->tail_ev);
    cudaStreamDestroy(d->copy_stream);
    cudaStreamDestroy(d->stream);
    free(d->tab);
    free(d);
    free(dvc);
}

/* ------------------------------------------------------- extensions --- */

/* Plain-pointer entry points keep the zero bookkeeping of tensor storage they
 * touch: inputs are cleared if still pending, outputs are marked written. */
/* The block holding p: by base first, else (a pointer into a buffer) by range. */
static mcu_block* tab_find_containing(mcu_device* d, uintptr_t p) {
    mcu_block* b = tab_find(d, p);
    if (b) return b;
    for (size_t i = 0; i < d->tab_cap; ++i)
        if (d->tab[i].state == 1 && d->tab[i].base <= p && p - d->tab[i].base < d->tab[i].size) return &d->tab[i];
    return NULL;
}
static void ext_in(mcu_device* d, const void* p) {
    mcu_block* b = tab_find_containing(d, (uintptr_t)p);
    if (b) materialize(d, b->base);
}
static void ext_out(mcu_device* d, void* p, size_t bytes) {
    mcu_block* b = tab_find_containing(d, (uintptr_t)p);
    if (b) result_written(d, b->base, b->base == (uintptr_t)p && bytes >= b->size);
}

int mag_cuda_device_ordinal(mag_compute_device_t* dvc) { return dev_of(dvc)->ordinal; }

int mcu_dev_ordinal(mag_compute_device_t* dvc) { return dev_of(dvc)->ordinal; }
int mcu_dev_sync(mag_compute_device_t* dvc) { return mag_cuda_synchronize(dvc); }
void mcu_dev_in(mag_compute_device_t* dvc, const void* p) { ext_in(dev_of(dvc), p); }
void mcu_dev_out(mag_compute_device_t* dvc, void* p, size_t bytes) { ext_out(dev_of(dvc), p, bytes); }

int mag_cuda_set_matmul_mode(mag_compute_device_t* dvc, int mode) {
    if (mode < 0 || mode > 2) return MAG_CUDA_E_INVALID;
    if (mode == 2 && !mcu_matmul_tc_supported()) return MAG_CUDA_E_UNSUPPORTED;
    dev_of(dvc)->matmul_mode = mode;
    return 0;
}
int mag_cuda_set_tc_split(mag_compute_device_t* dvc, int split) {
    if (split != MAG_CUDA_TC_SPLIT_TF32 && split != MAG_CUDA_TC_SPLIT_F16) return MAG_CUDA_E_INVALID;
    dev_of(dvc)->tc_f16 = split == MAG_CUDA_TC_SPLIT_F16;
    return 0;
}
void* mag_cuda_stream(mag_compute_device_t* dvc) { return (void*)dev_of(dvc)->stream; }
size_t mag_cuda_memory_in_use(mag_compute_device_t* dvc) { return dev_of(dvc)->bytes_live; }
int mag_cuda_last_error(mag_compute_device_t* dvc) { return dev_of(dvc)->sticky_error; }

int mag_cuda_synchronize(mag_compute_device_t* dvc) {
    mcu_device* d = dev_of(dvc);
    cudaError_t e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return (int)e;
    int st = 0;
    e = cudaMemcpy(&st, d->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return (int)e;
    if (!st) return 0;
    /* reported once: the word is cleared, so later work on this device reports its own status */
    e = cudaMemset(d->d_status, 0, sizeof(int));
    return e != cudaSuccess ? (int)e : MAG_CUDA_E_DEVICE_WAIT;
}

int mag_cuda_exec_node(mag_compute_device_t* dvc, mag_tensor_t* node) {
    if (!dvc || !node) return MAG_CUDA_E_INVALID;
    return exec_node(dev_of(dvc), node);
}

int mag_cuda_unary_f32(mag_compute_device_t* dvc, int op, float* r, const float* x, int64_t rows, int64_t cols,
                       int64_t r_s1, int64_t x_s1, float xi) {
    if (op == MAG_ABI_OP_SILU_DV || op == MAG_ABI_OP_GELU_DV) return MAG_CUDA_E_UNSUPPORTED;
    if (op < MAG_ABI_OP_ABS || op > MAG_ABI_OP_DIVS || op == MAG_ABI_OP_ADD || op == MAG_ABI_OP_SUB ||
        op == MAG_ABI_OP_MUL || op == MAG_ABI_OP_DIV)
        return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_out(d, r, (size_t)(rows * cols * 4));
    int rc = mcu_launch_unary(op, r, x, rows, cols, r_s1, x_s1, xi, d->stream);
    if (!rc) mcu_count_launches(1);
    return rc;
}

int mag_cuda_binary_f32(mag_compute_device_t* dvc, int op, float* r, const float* x, const float* y,
                        const int64_t* xd, const int64_t* xs, const int64_t* rs, const int64_t* yd,
                        const int64_t* ys) {
    if (op < MAG_ABI_OP_ADD || op > MAG_ABI_OP_DIV) return MAG_CUDA_E_INVALID;
    for (int k = 0; k < 6; ++k)
        if (yd[k] <= 0 || xd[k] % yd[k]) return MAG_CUDA_E_INVALID; /* mag_tensor_can_broadcast */
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_in(d, y);
    ext_out(d, r, (size_t)(xd[0] * xd[1] * xd[2] * xd[3] * xd[4] * xd[5] * 4));
    int rc = mcu_launch_binary(op, r, x, y, xd, xs, rs, yd, ys, d->stream);
    if (!rc) mcu_count_launches(1);
    return rc;
}

int mag_cuda_reduce_f32(mag_compute_device_t* dvc, int op, float* r, const float* x, const int64_t* xd,
                        const int64_t* xs) {
    if (op < MAG_ABI_OP_MEAN || op > MAG_ABI_OP_SUM) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_out(d, r, 4);
    int rc = mcu_launch_reduce(op, r, x, xd, xs, scratch_get(d, mcu_reduce_scratch_bytes()), d->stream);
    if (!rc) mcu_count_launches(2);
    return rc;
}

_Static_assert(sizeof(mag_cuda_reduce_part) == sizeof(McuReducePart), "reduce record layout");

int mag_cuda_reduce_partial_f32(mag_compute_device_t* dvc, mag_cuda_reduce_part* part, const float* x,
                                const int64_t* xd, const int64_t* xs) {
    if (!part || ((uintptr_t)part & 7)) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_out(d, part, sizeof(*part));
    int rc = mcu_launch_reduce_partial((McuReducePart*)part, x, xd, xs, scratch_get(d, mcu_reduce_scratch_bytes()),
                                       d->stream);
    if (!rc) mcu_count_launches(2);
    return rc;
}

int mag_cuda_reduce_combine_f32(mag_compute_device_t* dvc, int op, float* r, const mag_cuda_reduce_part* parts,
                                int nparts) {
    if (op < MAG_ABI_OP_MEAN || op > MAG_ABI_OP_SUM || !parts || nparts < 1 || ((uintptr_t)parts & 7))
        return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, parts);
    ext_out(d, r, 4);
    int rc = mcu_launch_reduce_combine(op, r, (const McuReducePart*)parts, nparts, d->stream);
    if (!rc) mcu_count_launches(1);
    return rc;
}

int mag_cuda_matmul_f32(mag_compute_device_t* dvc, float* r, const float* x, const float* y, int64_t M, int64_t K,
                        int64_t N) {
    if (M < 0 || K < 0 || N < 0) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_in(d, y);
    ext_out(d, r, (size_t)(M * N * 4));
    int path = matmul_path(d, M, K, N);
    int rc;
    if (path == MM_SKINNY) {
        rc = mcu_launch_matmul_skinny(r, x, y, M, K, N, N, scratch_get(d, mcu_matmul_skinny_scratch_bytes(M, K, N)),
                                      d->stream);
        if (!rc) mcu_count_launches(2);
    } else if (path == MM_TC) {
        rc = mcu_launch_matmul_tc(r, x, y, M, K, N, scratch_get(d, mcu_matmul_tc_scratch_bytes(M, K, N)),
                                  d->d_status, d->stream, d->tc_f16);
        if (!rc) mcu_count_launches(mcu_matmul_tc_kernels(M, K, N, d->tc_f16, 0));
    } else {
        rc = mcu_launch_matmul_exact(r, x, y, 1, M, K, N, N, 0, d->stream);
        if (!rc) mcu_count_launches(mcu_matmul_exact_kernels(1, M));
    }
    return rc;
}

size_t mag_cuda_matmul_skinny_noalloc_limit(void) { return mcu_skinny_noalloc_limit(); }

int mag_cuda_matmul_skinny_f32_noalloc(mag_compute_device_t* dvc, float* r, const float* x, const float* y,
                                       int64_t M, int64_t K, int64_t N) {
    if (!dvc || !r || !x || !y || M < 1 || M > 16 || K < 0 || N < 1) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    size_t need = mcu_matmul_skinny_scratch_bytes(M, K, N);
    if (need > mcu_skinny_noalloc_limit()) {
        fprintf(stderr,
                "[magnetron-cuda] mag_cuda_matmul_skinny_f32_noalloc: M=%lld K=%lld N=%lld needs %zu bytes of "
                "scratch, above the fixed %zu-byte array; use mag_cuda_matmul_f32\n",
                (long long)M, (long long)K, (long long)N, need, mcu_skinny_noalloc_limit());
        return MAG_CUDA_E_SCRATCH_LIMIT;
    }
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return (int)e;
    if (prev != d->ordinal && (e = cudaSetDevice(d->ordinal)) != cudaSuccess) return (int)e;
    void* scratch = NULL;
    int rc = mcu_skinny_noalloc_scratch(&scratch);
    if (!rc) {
        ext_in(d, x);
        ext_in(d, y);
        ext_out(d, r, (size_t)(M * N * 4));
        rc = mcu_launch_matmul_skinny(r, x, y, M, K, N, N, scratch, d->stream);
        if (!rc) mcu_count_launches(2);
    }
    if (prev != d->ordinal) cudaSetDevice(prev);
    return rc;
}

int mag_cuda_broadcast2_f32(mag_compute_device_t* dvc, int op, float* r, const float* x, const float* y,
                            const int64_t* rd, const int64_t* xd, const int64_t* yd) {
    if (op < MAG_ABI_OP_ADD || op > MAG_ABI_OP_DIV) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_in(d, y);
    ext_out(d, r, (size_t)(rd[0] * rd[1] * rd[2] * rd[3] * rd[4] * rd[5] * 4));
    int rc = mcu_launch_bcast2(op, r, x, y, rd, xd, yd, d->stream);
    if (!rc) mcu_count_launches(1);
    return rc;
}

int mag_cuda_reduce_rows_f32(mag_compute_device_t* dvc, int op, float* r, const float* x, int64_t rows,
                             int64_t cols) {
    if (op < MAG_ABI_OP_MEAN || op > MAG_ABI_OP_SUM) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_out(d, r, (size_t)(rows * 4));
    int rc = mcu_launch_reduce_rows(op, r, x, rows, cols, d->stream);
    if (!rc) mcu_count_launches(1);
    return rc;
}

int mag_cuda_softmax_rows_f32(mag_compute_device_t* dvc, float* r, const float* x, int64_t rows, int64_t cols) {
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_out(d, r, (size_t)(rows * cols * 4));
    const size_t sb = mcu_softmax_rows_scratch_bytes(rows, cols);
    int rc = mcu_launch_softmax_rows(r, x, rows, cols, sb ? scratch_get(d, sb) : NULL, d->stream);
    if (!rc) mcu_count_launches(mcu_softmax_rows_kernels(rows, cols));
    return rc;
}

/* ------------------------------------------------ async host copies --- */

/* Queues a copy between pinned host memory and a tensor's storage on the copy stream, after
 * everything queued so far on the compute stream, and marks the buffer so the next
 * compute-stream access waits for it. */
static int io_async(mag_compute_device_t* dvc, mag_tensor_t* t, void* host, size_t bytes, int upload) {
    if (!dvc || !t || !host) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    mcu_block* b = tab_find(d, t->storage.base);
    if (!b || bytes > b->size || d->capturing || d->managed || !host_is_pinned(host)) return MAG_CUDA_E_INVALID;
    if (!bytes) return 0;
    if (upload) result_written(d, b->base, bytes >= b->size); /* the rest of a partial upload reads as zero */
    else materialize(d, b->base);
    b = tab_find(d, t->storage.base);
    if (!b->io_ev) MCU_CHECK(cudaEventCreateWithFlags(&b->io_ev, cudaEventDisableTiming));
    MCU_CHECK(cudaEventRecord(d->tail_ev, d->stream));
    MCU_CHECK(cudaStreamWaitEvent(d->copy_stream, d->tail_ev, 0));
    cudaError_t e = upload ? cudaMemcpyAsync((void*)b->base, host, bytes, cudaMemcpyHostToDevice, d->copy_stream)
                           : cudaMemcpyAsync(host, (const void*)b->base, bytes, cudaMemcpyDeviceToHost, d->copy_stream);
    if (e != cudaSuccess) return (int)e;
    MCU_CHECK(cudaEventRecord(b->io_ev, d->copy_stream));
    b->io_pending = 1;
    return 0;
}

int mag_cuda_tensor_upload_async(mag_compute_device_t* dvc, mag_tensor_t* t, const void* src, size_t bytes) {
    return io_async(dvc, t, (void*)src, bytes, 1);
}

int mag_cuda_tensor_download_async(mag_compute_device_t* dvc, mag_tensor_t* t, void* dst, size_t bytes) {
    return io_async(dvc, t, dst, bytes, 0);
}

int mag_cuda_copies_synchronize(mag_compute_device_t* dvc) {
    if (!dvc) return MAG_CUDA_E_INVALID;
    return (int)cudaStreamSynchronize(dev_of(dvc)->copy_stream);
}

int mag_cuda_fill_uniform_pcg_f32(mag_compute_device_t* dvc, float* r, int64_t n, float min, float max,
                                  uint64_t* state, uint64_t inc) {
    if (n < 0 || !state) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_out(d, r, (size_t)n * 4);
    const float span = max - min; /* rounded to f32 as the host generator does */
    int rc = mcu_launch_fill_pcg(r, n, 0, min, span, *state, inc, d->stream);
    if (rc) return rc;
    if (n) mcu_count_launches(1);
    *state = mcu_pcg_advance(*state, inc, (uint64_t)n);
    return 0;
}

int mag_cuda_fill_normal_pcg_f32(mag_compute_device_t* dvc, float* r, int64_t n, float mean, float stddev,
                                 uint64_t* state, uint64_t inc) {
    if (n < 0 || (n & 1) || !state) return MAG_CUDA_E_INVALID; /* pairs, as the core asserts */
    mcu_device* d = dev_of(dvc);
    ext_out(d, r, (size_t)n * 4);
    int rc = mcu_launch_fill_pcg(r, n, 1, mean, stddev, *state, inc, d->stream);
    if (rc) return rc;
    if (n) mcu_count_launches(1);
    *state = mcu_pcg_advance(*state, inc, (uint64_t)n);
    return 0;
}

static int fill_mt(mag_compute_device_t* dvc, float* r, int64_t n, int normal, float p0, float p1, uint32_t* mt) {
    mcu_device* d = dev_of(dvc);
    ext_out(d, r, (size_t)n * 4);
    if (!n) return 0;
    const size_t sb = mcu_fill_mt_scratch_bytes(n, mt[0], mt[1]);
    if (!sb) return MAG_CUDA_E_INVALID; /* not a state the host generator can be in */
    int k = 0;
    int rc = mcu_launch_fill_mt(r, n, normal, p0, p1, mt, scratch_get(d, sb), d->stream, &k);
    if (k) mcu_count_launches(k);
    return rc;
}

int mag_cuda_fill_uniform_mt19937_f32(mag_compute_device_t* dvc, float* r, int64_t n, float min, float max,
                                      uint32_t* mt) {
    if (n < 0 || !mt) return MAG_CUDA_E_INVALID;
    return fill_mt(dvc, r, n, 0, min, max - min, mt); /* max - min rounded to f32 as on the host */
}

int mag_cuda_fill_normal_mt19937_f32(mag_compute_device_t* dvc, float* r, int64_t n, float mean, float stddev,
                                     uint32_t* mt) {
    if (n < 0 || (n & 1) || !mt) return MAG_CUDA_E_INVALID; /* pairs, as the core asserts */
    return fill_mt(dvc, r, n, 1, mean, stddev, mt);
}

int mag_cuda_mt19937_jump(const uint32_t* win, uint64_t d, uint32_t* out) {
    if (!win || !out) return MAG_CUDA_E_INVALID;
    return mcu_mt19937_jump_host(win, d, out) ? MAG_CUDA_E_INVALID : 0;
}

int mag_cuda_mt19937_degree(void) { return mcu_mt19937_degree(); }

int mag_cuda_fill_f32(mag_compute_device_t* dvc, float* r, int64_t n, float x) {
    if (n < 0) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_out(d, r, (size_t)n * 4);
    int rc = mcu_launch_fill_const(r, n, x, d->stream);
    if (!rc && n) mcu_count_launches(1);
    return rc;
}

/* ------------------------------------------------------------ images --- */

/* (c, h, w) of a rank-3 image tensor (mag_tensor_image_* macros, magnetron/magnetron.h:394-396). */
static int img_dims(const mag_tensor_t* t, int32_t* w, int32_t* h, int32_t* c) {
    if (!t || t->rank != 3 || t->dtype != 0) return MAG_CUDA_E_INVALID;
    if (t->shape[0] < 1 || t->shape[1] < 1 || t->shape[2] < 1 || t->shape[1] > INT32_MAX || t->shape[2] > INT32_MAX ||
        t->shape[0] > 4)
        return MAG_CUDA_E_INVALID;
    *c = (int32_t)t->shape[0];
    *h = (int32_t)t->shape[1];
    *w = (int32_t)t->shape[2];
    return 0;
}

static int is_device_ptr(const void* p) {
    struct cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

static float img_channel(uint32_t rgb, int shift) { return (float)((rgb >> shift) & 0xff) / 255.0f; }

int mag_cuda_img_from_u8(mag_compute_device_t* dvc, mag_tensor_t* dst, const uint8_t* src, uint32_t w, uint32_t h,
                         uint32_t c, uint32_t rw, uint32_t rh) {
    int32_t tw, th, tc;
    if (!src || !w || !h || !c || c > 4 || img_dims(dst, &tw, &th, &tc)) return MAG_CUDA_E_INVALID;
    const int resize = rw && rh;
    if ((uint32_t)tc != c || (uint32_t)tw != (resize ? rw : w) || (uint32_t)th != (resize ? rh : h))
        return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    const size_t bytes = (size_t)w * h * c;
    const uint8_t* s = src;
    const int host = !is_device_ptr(src);
    if (host) { /* the decoded file is a quarter of the f32 image: move it as bytes, expand on the device */
        uint8_t* tmp = (uint8_t*)scratch_get(d, bytes);
        MCU_CHECK(cudaMemcpyAsync(tmp, src, bytes, cudaMemcpyHostToDevice, d->stream));
        s = tmp;
    }
    ext_out(d, fptr(dst), (size_t)dst->numel * 4);
    /* the reference's scale factors, rounded to f32 on the host as it rounds them
     * (magnetron/magnetron.c:3028-3029) */
    const float ws = resize ? (float)(w - 1) / (float)(rw - 1) : 0.0f;
    const float hs = resize ? (float)(h - 1) / (float)(rh - 1) : 0.0f;
    int rc = mcu_launch_img_from_u8(fptr(dst), s, w, h, c, resize ? rw : 0, resize ? rh : 0, ws, hs, d->stream);
    if (rc) return rc;
    mcu_count_launches(1);
    if (host && host_is_pinned(src)) { /* the caller may reuse src on return */
        cudaError_t e = cudaStreamSynchronize(d->stream);
        if (e != cudaSuccess) return (int)e;
    }
    return 0;
}

int mag_cuda_img_to_u8(mag_compute_device_t* dvc, const mag_tensor_t* src, uint8_t* dst) {
    int32_t w, h, c;
    if (!dst || img_dims(src, &w, &h, &c) || !(c == 1 || c == 3 || c == 4)) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, fptr(src));
    const size_t bytes = (size_t)w * h * c;
    const int dev_dst = is_device_ptr(dst);
    uint8_t* out = dev_dst ? dst : (uint8_t*)scratch_get(d, bytes);
    int rc = mcu_launch_img_to_u8(out, fptr(src), (uint32_t)w, (uint32_t)h, (uint32_t)c, d->stream);
    if (rc) return rc;
    mcu_count_launches(1);
    if (!dev_dst) {
        MCU_CHECK(cudaMemcpyAsync(dst, out, bytes, cudaMemcpyDeviceToHost, d->stream));
        cudaError_t e = cudaStreamSynchronize(d->stream);
        if (e != cudaSuccess) return (int)e;
    }
    return 0;
}

/* Ring i of a box draws something while its horizontal edge (xx1 <= xx2) or vertical edge
 * (yy1 <= yy2) is non-empty; both bounds move monotonically with i. */
static int box_ring_draws(int64_t i, int32_t w, int32_t h, int32_t x1, int32_t y1, int32_t x2, int32_t y2) {
    int64_t xx1 = x1 + i, yy1 = y1 + i, xx2 = x2 - i, yy2 = y2 - i;
    if (xx1 >= w) xx1 = w - 1;
    if (xx2 >= w) xx2 = w - 1;
    if (yy1 >= h) yy1 = h - 1;
    if (yy2 >= h) yy2 = h - 1;
    return xx1 <= xx2 || yy1 <= yy2;
}

int mag_cuda_img_draw_box(mag_compute_device_t* dvc, mag_tensor_t* t, int32_t x1, int32_t y1, int32_t x2, int32_t y2,
                          int32_t wi, uint32_t rgb) {
    int32_t w, h, c;
    if (img_dims(t, &w, &h, &c) || c != 3) return MAG_CUDA_E_INVALID;
    if (!(x2 > x1 && y2 > y1 && x1 > 0 && y1 > 0 && x2 > 0 && y2 > 0)) return MAG_CUDA_E_INVALID;
    if (wi < 1) wi = 1;
    int64_t lo = 0, hi = wi; /* first ring that draws nothing, by bisection */
    while (lo < hi) {
        const int64_t mid = lo + (hi - lo) / 2;
        if (box_ring_draws(mid, w, h, x1, y1, x2, y2)) lo = mid + 1;
        else hi = mid;
    }
    mcu_device* d = dev_of(dvc);
    ext_out(d, fptr(t), 4); /* a partial write: pending zeros are cleared first */
    int rc = mcu_launch_img_draw_box(fptr(t), w, h, x1, y1, x2, y2, (int32_t)lo, img_channel(rgb, 16),
                                     img_channel(rgb, 8), img_channel(rgb, 0), d->stream);
    if (!rc && lo) mcu_count_launches(1);
    return rc;
}

int mag_cuda_img_draw_text(mag_compute_device_t* dvc, mag_tensor_t* t, int32_t x, int32_t y, int32_t size,
                           uint32_t rgb, const char* txt) {
    int32_t w, h, c;
    if (img_dims(t, &w, &h, &c) || c != 3 || x < 0 || y < 0 || size < 8 || !txt || !*txt) return MAG_CUDA_E_INVALID;
    const size_t len = strlen(txt);
    int32_t* cells = (int32_t*)malloc(3 * len * sizeof(int32_t));
    if (!cells) return MAG_CUDA_E_INVALID;
    int32_t n = 0, lx = x, ly = y;
    for (const unsigned char* p = (const unsigned char*)txt; *p; ++p) {
        /* printable in the C locale; space has no pixels; '\n' returns to x one line down */
        if (*p > 32 && *p < 127) {
            cells[3 * n] = lx;
            cells[3 * n + 1] = ly;
            cells[3 * n + 2] = *p - 33;
            ++n;
        }
        if (*p == '\n') {
            lx = x;
            ly += 14;
        } else {
            lx += 8;
        }
    }
    mcu_device* d = dev_of(dvc);
    int rc = 0;
    if (n) {
        int32_t* dev_cells = (int32_t*)scratch_get(d, (size_t)n * 3 * sizeof(int32_t));
        /* a pageable source is staged before the call returns, so cells can be freed below */
        MCU_CHECK(cudaMemcpyAsync(dev_cells, cells, (size_t)n * 3 * sizeof(int32_t), cudaMemcpyHostToDevice,
                                  d->stream));
        ext_out(d, fptr(t), 4);
        rc = mcu_launch_img_draw_text(fptr(t), w, h, dev_cells, n, img_channel(rgb, 16), img_channel(rgb, 8),
                                      img_channel(rgb, 0), d->stream);
        if (!rc) mcu_count_launches(1);
    }
    free(cells);
    return rc;
}

/* The batched kernels index the batch with a grid dimension of at most 65535 blocks, so longer
 * batches run as consecutive slices of that many products. */
#define MCU_BATCH_SLICE 65535

static int matmul_batched_slice(mcu_device* d, float* r, const float* x, const float* y, int64_t batch, int64_t M,
                                int64_t K, int64_t N) {
    int rc;
    if (d->matmul_mode != 1 && mcu_matmul_tc_supported() && M >= 128 && N >= 64 && K >= 32 && K <= MCU_TC_MAX_K &&
        batch * M < ((int64_t)1 << 31) && batch * N < ((int64_t)1 << 31) && (double)batch * M * N * K >= 1.0e9) {
        void* scratch = scratch_get(d, mcu_matmul_tc_batched_scratch_bytes(batch, M, K, N));
        rc = mcu_launch_matmul_tc_batched(r, x, y, batch, M, K, N, scratch, d->d_status, d->stream, d->tc_f16);
        if (!rc) mcu_count_launches(mcu_matmul_tc_batched_kernels(batch, M, K, N, d->tc_f16));
    } else {
        rc = mcu_launch_matmul_exact(r, x, y, batch, M, K, N, N, 0, d->stream);
        if (!rc) mcu_count_launches(mcu_matmul_exact_kernels(batch, M));
    }
    return rc;
}

int mag_cuda_matmul_batched_f32(mag_compute_device_t* dvc, float* r, const float* x, const float* y, int64_t batch,
                                int64_t M, int64_t K, int64_t N) {
    if (batch < 0 || M < 0 || K < 0 || N < 0) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    ext_in(d, x);
    ext_in(d, y);
    ext_out(d, r, (size_t)(batch * M * N * 4));
    int rc = 0;
    for (int64_t b0 = 0; b0 < batch && !rc; b0 += MCU_BATCH_SLICE) {
        const int64_t nb = batch - b0 < MCU_BATCH_SLICE ? batch - b0 : MCU_BATCH_SLICE;
        rc = matmul_batched_slice(d, r + b0 * M * N, x + b0 * M * K, y + b0 * K * N, nb, M, K, N);
    }
    return rc;
}

/* ------------------------------------------------------------ graphs --- */

typedef struct ptrset {
    uintptr_t* v;
    size_t cap, n;
} ptrset;

static int ptrset_add(ptrset* s, uintptr_t p) { /* 1 if newly added */
    if ((s->n + 1) * 2 > s->cap) {
        size_t oc = s->cap;
        uintptr_t* ov = s->v;
        s->cap = oc ? oc * 2 : 64;
        s->v = (uintptr_t*)calloc(s->cap, sizeof(uintptr_t));
        s->n = 0;
        for (size_t i = 0; i < oc; ++i)
            if (ov[i]) ptrset_add(s, ov[i]);
        free(ov);
    }
    size_t i = hash_ptr(p, s->cap);
    while (s->v[i]) {
        if (s->v[i] == p) return 0;
        i = (i + 1) & (s->cap - 1);
    }
    s->v[i] = p;
    s->n++;
    return 1;
}

/* Post-order of the DAG below root (inputs before users). */
static mag_tensor_t** topo_order(mag_tensor_t* root, size_t* n_out) {
    ptrset seen = {0};
    size_t cap = 64, n = 0, sp = 0, scap = 64;
    mag_tensor_t** order = (mag_tensor_t**)malloc(cap * sizeof(*order));
    struct frame { mag_tensor_t* t; int next; }* stack = malloc(scap * sizeof(*stack));
    ptrset_add(&seen, (uintptr_t)root);
    stack[sp++] = (struct frame){root, 0};
    while (sp) {
        struct frame* f = &stack[sp - 1];
        if (f->next < MAG_ABI_MAX_INPUTS) {
            mag_tensor_t* in = f->t->op_inputs[f->next++];
            if (in && ptrset_add(&seen, (uintptr_t)in)) {
                if (sp == scap) {
                    scap *= 2;
                    stack = realloc(stack, scap * sizeof(*stack));
                }
                stack[sp++] = (struct frame){in, 0};
            }
        } else {
            if (n == cap) {
                cap *= 2;
                order = (mag_tensor_t**)realloc(order, cap * sizeof(*order));
            }
            order[n++] = f->t;
            --sp;
        }
    }
    free(stack);
    free(seen.v);
    *n_out = n;
    return order;
}

static uint64_t mix(uint64_t h, uint64_t v) {
    h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    return h;
}

static int is_compute(const mag_tensor_t* t) {
    return t->op != MAG_ABI_OP_NOP && t->op != MAG_ABI_OP_VIEW && t->op != MAG_ABI_OP_TRANSPOSE &&
           t->op != MAG_ABI_OP_PERMUTE;
}

/* A leaf whose whole buffer holds zeros that nothing has overwritten since (fresh storage, or
 * set to zero through the storage callback). */
static int leaf_is_zero(mcu_device* d, const mag_tensor_t* t) {
    mcu_block* b = tab_find(d, t->storage.base);
    return b && b->known_zero && (size_t)(t->numel * 4) <= b->size;
}

static uint64_t graph_signature(mcu_device* d, mag_tensor_t** nodes, size_t n) {
    uint64_t h = 0x1234567ull;
    for (size_t i = 0; i < n; ++i) {
        mag_tensor_t* t = nodes[i];
        if (!is_compute(t)) h = mix(h, (uint64_t)leaf_is_zero(d, t)); /* zero biases are planned as such */
        h = mix(h, (uintptr_t)t);
        h = mix(h, (uint64_t)t->op);
        h = mix(h, (uint64_t)t->storage.base);
        for (int k = 0; k < 6; ++k) h = mix(mix(h, (uint64_t)t->shape[k]), (uint64_t)t->strides[k]);
        h = mix(h, t->op_params[0]);
        h = mix(mix(h, (uintptr_t)t->op_inputs[0]), (uintptr_t)t->op_inputs[1]);
    }
    return h;
}


/* ---- fusion planner for deferred graphs ----
 * Recognises dense layers, MATMUL -> ADD(same-shape bias) [-> GELU], whose
 * intermediates have no other consumer inside the graph, and runs each as one
 * tensor-core GEMM whose epilogue adds the bias, applies GELU and, when the
 * next node is a MATMUL reading this layer's output, also writes that
 * MATMUL's tf32 hi/lo operand split (so it skips its split pass).  Only the
 * fused chain's final tensor is written; the MATMUL and ADD results inside a
 * chain are not materialised. */

enum { PLAN_NORMAL = 0, PLAN_FUSED = 1, PLAN_SKIP = 2 };

typedef struct mcu_plan_item {
    int kind;
    mag_tensor_t* out;      /* fused: tensor whose storage receives the layer output */
    mag_tensor_t* bias;     /* fused: same-shape bias tensor or NULL */
    int act;                /* fused: 0 none, 1 GELU */
    int a_split;            /* -1, or activation split buffer holding A's hi/lo */
    int out_split;          /* -1, or activation split buffer receiving out's hi/lo */
    int exact;              /* fused on the bit-exact CUDA-core product (else the tensor-core one) */
    int64_t bias_mod;       /* exact: 0 full-shape bias, else the length of a bias broadcast along dim 0 */
    int bias_zero;          /* tensor-core: the bias is a leaf known to hold zeros (no bias read) */
} mcu_plan_item;

static int same_shape_canonical(const mag_tensor_t* a, const mag_tensor_t* b) {
    for (int k = 0; k < 6; ++k)
        if (a->shape[k] != b->shape[k]) return 0;
    return is_canonical(a) && is_canonical(b);
}

static int matmul_on_path(mcu_device* d, const mag_tensor_t* m, int path) {
    if (m->op != MAG_ABI_OP_MATMUL) return 0;
    const mag_tensor_t* x = m->op_inputs[0];
    const mag_tensor_t* y = m->op_inputs[1];
    if (!x || !y || x->shape[2] != 1 || x->shape[3] != 1 || y->shape[2] != 1 || y->shape[3] != 1) return 0;
    const int64_t M = x->shape[0], K = x->shape[1], N = y->shape[1];
    if (m->storage.base == x->storage.base || m->storage.base == y->storage.base) return 0;
    if (m->shape[1] != N || (size_t)(M * N * 4) != m->storage.size) return 0;
    if (path == MM_EXACT && M > 1048560) return 0; /* the fused exact product runs unsliced */
    return matmul_path(d, M, K, N) == path;
}

static int tc_matmul_ok(mcu_device* d, const mag_tensor_t* m) { return matmul_on_path(d, m, MM_TC); }

/* A bias the elementwise ADD broadcasts along dim 0 of the product: a canonical tensor of
 * shape (shape[0] of the product, 1, 1, 1, 1, 1), read at the flat index mod its length. */
static int row_bias(const mag_tensor_t* b, const mag_tensor_t* m) {
    if (!is_canonical(b) || b->shape[0] != m->shape[0]) return 0;
    for (int k = 1; k < 6; ++k)
        if (b->shape[k] != 1) return 0;
    return 1;
}

static size_t find_index(mag_tensor_t** nodes, size_t n, const mag_tensor_t* t) {
    for (size_t i = 0; i < n; ++i)
        if (nodes[i] == t) return i;
    return n;
}

/* Fills plan[n]; returns the bytes of one activation split buffer (0: none needed). */
static size_t plan_fusion(mcu_device* d, mag_tensor_t** nodes, size_t n, mag_tensor_t* root, mcu_plan_item* plan) {
    int* users = (int*)calloc(n, sizeof(int));
    size_t* user_of = (size_t*)malloc(n * sizeof(size_t));
    for (size_t i = 0; i < n; ++i) {
        plan[i] = (mcu_plan_item){PLAN_NORMAL, NULL, NULL, 0, -1, -1, 0, 0, 0};
        user_of[i] = n;
    }
    for (size_t i = 0; i < n; ++i)
        for (int k = 0; k < MAG_ABI_MAX_INPUTS; ++k) {
            mag_tensor_t* in = nodes[i]->op_inputs[k];
            if (!in) continue;
            size_t j = find_index(nodes, n, in);
            if (j < n) {
                users[j]++;
                user_of[j] = i;
            }
        }
    size_t split_bytes = 0;
    for (size_t i = 0; i < n; ++i) {
        mag_tensor_t* m = nodes[i];
        if (plan[i].kind != PLAN_NORMAL || m == root || users[i] != 1) continue;
        const int tc = tc_matmul_ok(d, m);
        const int exact = !tc && matmul_on_path(d, m, MM_EXACT);
        if (!tc && !exact) continue;
        size_t ia = user_of[i];
        mag_tensor_t* a = nodes[ia];
        if (a->op != MAG_ABI_OP_ADD || a->op_inputs[0] != m || a->op_inputs[1] == m) continue;
        mag_tensor_t* b = a->op_inputs[1];
        if (!same_shape_canonical(a, m) || a->storage.size != m->storage.size) continue;
        const int full = same_shape_canonical(b, m);
        if (!full && !(exact && row_bias(b, m))) continue;
        plan[i].kind = PLAN_FUSED;
        plan[i].bias = b;
        plan[i].out = a;
        plan[i].exact = exact;
        plan[i].bias_mod = full ? 0 : b->shape[0];
        /* a leaf bias that nothing has written since it was zeroed (the core's fresh tensors):
         * the epilogue adds +0.0f instead of reading it; the graph's key holds that state */
        plan[i].bias_zero = tc && full && !is_compute(b) && leaf_is_zero(d, b);
        plan[ia].kind = PLAN_SKIP;
        size_t last = ia;
        if (a != root && users[ia] == 1) {
            size_t ig = user_of[ia];
            mag_tensor_t* g = nodes[ig];
            /* every element on the activation's vector-lane formula: dim 0 a multiple of 4 */
            const int act = g->op == MAG_ABI_OP_GELU ? 1 : (exact && g->op == MAG_ABI_OP_SIGMOID ? 2 : 0);
            if (act && g->op_inputs[0] == a && same_shape_canonical(g, m) && g->storage.size == m->storage.size &&
                m->shape[0] % 4 == 0) {
                plan[i].act = act;
                plan[i].out = g;
                plan[ig].kind = PLAN_SKIP;
                last = ig;
            }
        }
        /* the next MATMUL reads this layer's output: hand it the split operand */
        mag_tensor_t* out = plan[i].out;
        const int64_t N = m->shape[1];
        if (tc && !d->tc_f16 && out != root && users[last] == 1 && N % 32 == 0) { /* the f16 split scales whole rows itself */
            size_t in2 = user_of[last];
            mag_tensor_t* m2 = nodes[in2];
            if (m2->op_inputs[0] == out && m2->op_inputs[1] != out && tc_matmul_ok(d, m2)) {
                int buf = plan[i].a_split == 0 ? 1 : 0;
                plan[i].out_split = buf;
                plan[in2].a_split = buf;
                size_t bytes = (size_t)(m->shape[0] * ((N + 31) / 32 * 32)) * 4 * 2;
                if (bytes > split_bytes) split_bytes = bytes;
            }
        }
    }
    free(users);
    free(user_of);
    return split_bytes;
}

/* Runs one planned MATMUL (fused or with a pre-split operand). */
static int exec_planned_matmul(mcu_device* d, mag_tensor_t* m, const mcu_plan_item* it, char* scratch,
                               size_t split_off, size_t split_bytes) {
    mag_tensor_t* x = m->op_inputs[0];
    mag_tensor_t* y = m->op_inputs[1];
    const int64_t M = x->shape[0], K = x->shape[1], N = y->shape[1];
    mag_tensor_t* out = it->kind == PLAN_FUSED ? it->out : m;
    if (it->a_split < 0) materialize(d, x->storage.base);
    materialize(d, y->storage.base);
    if (it->bias) materialize(d, it->bias->storage.base);
    result_written(d, out->storage.base, (size_t)(M * N * 4) == out->storage.size);
    if (it->exact) {
        int rc = mcu_launch_matmul_exact_ep(fptr(out), fptr(x), fptr(y), M, K, N, it->bias ? fptr(it->bias) : NULL,
                                            it->bias_mod, it->act, d->stream);
        if (!rc) mcu_count_launches(1);
        return rc;
    }
    mcu_tc_epilogue ep;
    memset(&ep, 0, sizeof(ep));
    const size_t half = split_bytes / 2;
    if (it->a_split >= 0) {
        char* b = scratch + split_off + (size_t)it->a_split * split_bytes;
        ep.a_hi = (const float*)b;
        ep.a_lo = (const float*)(b + half);
    }
    if (it->kind == PLAN_FUSED) {
        ep.bias = it->bias && !it->bias_zero ? fptr(it->bias) : NULL;
        ep.bias_zero = it->bias_zero;
        ep.act = it->act;
        if (it->out_split >= 0) {
            char* b = scratch + split_off + (size_t)it->out_split * split_bytes;
            ep.out_hi = (float*)b;
            ep.out_lo = (float*)(b + half);
            ep.kp_out = (N + 31) / 32 * 32;
        }
    }
    int rc = mcu_launch_matmul_tc_ex(fptr(out), fptr(x), fptr(y), M, K, N, scratch, d->d_status, d->stream, &ep,
                                     d->tc_f16);
    if (!rc)
        mcu_count_launches(mcu_matmul_tc_kernels(M, K, N, d->tc_f16,
                                                 (it->a_split >= 0 ? 1 : 0) | (it->kind == PLAN_FUSED ? 2 : 0)));
    return rc;
}

static void harvest_graph_events(mcu_device* d, mcu_graph* g, int wait);

static int graph_exec_impl(mag_compute_device_t* dvc, mag_tensor_t* root, int fuse) {
    if (!dvc || !root) return MAG_CUDA_E_INVALID;
    mcu_device* d = dev_of(dvc);
    size_t n = 0;
    mag_tensor_t** nodes = topo_order(root, &n);
    /* the matmul path and split kind are baked into a captured graph: part of its key */
    uint64_t sig = graph_signature(d, nodes, n) ^ ((uint64_t)(1 + d->tc_f16 + 2 * d->matmul_mode) * 0x9E3779B97F4A7C15ull);
    mcu_graph* g = d->graphs;
    while (g && (g->root != root || g->fused != fuse)) g = g->next;
    for (size_t i = 0; i < n; ++i) io_wait(d, tab_find(d, nodes[i]->storage.base)); /* outside any capture */
    if (g && g->sig == sig) {
        free(nodes);
        /* profiling: the previous replay's op events are read before this replay records over them
         * (waiting for that replay alone, so work queued after it keeps running) */
        if (g->ran && d->profiling) harvest_graph_events(d, g, 1);
        g->ran = g->n_ev > 0;
        mcu_count_launches((int)g->n_kernels);
        return (int)cudaGraphLaunch(g->exec, d->stream);
    }
    if (g) {
        mcu_graph** pp = &d->graphs;
        while (*pp != g) pp = &(*pp)->next;
        *pp = g->next;
        cudaStreamSynchronize(d->stream);
        graph_free(g);
    }
    mcu_plan_item* plan = (mcu_plan_item*)calloc(n ? n : 1, sizeof(mcu_plan_item));
    for (size_t i = 0; i < n; ++i) plan[i] = (mcu_plan_item){PLAN_NORMAL, NULL, NULL, 0, -1, -1, 0, 0, 0};
    size_t split_bytes = fuse ? plan_fusion(d, nodes, n, root, plan) : 0;
    /* leaves are materialised outside the capture so replays never clear data the caller wrote later */
    size_t scratch = 0;
    for (size_t i = 0; i < n; ++i) {
        if (!is_compute(nodes[i])) materialize(d, nodes[i]->storage.base);
        else if (plan[i].kind != PLAN_SKIP) {
            size_t s = node_scratch_bytes(d, nodes[i]);
            if (s > scratch) scratch = s;
        }
    }
    const size_t split_off = (scratch + 1023) & ~(size_t)1023;
    const size_t total = split_bytes ? split_off + 2 * split_bytes : scratch;
    g = (mcu_graph*)calloc(1, sizeof(mcu_graph));
    g->root = root;
    g->fused = fuse;
    g->sig = sig;
    g->n_nodes = n;
    if (total) {
        cudaError_t e = cudaMalloc(&g->scratch, total);
        if (e != cudaSuccess) {
            free(g);
            free(plan);
            free(nodes);
            return (int)e;
        }
    }
    MCU_CHECK(cudaStreamSynchronize(d->stream));
    cudaGraph_t graph;
    d->capturing = 1;
    d->graph_scratch = g->scratch;
    size_t saved_bytes = d->scratch_bytes;
    d->scratch_bytes = total;
    if (d->profiling) {
        g->ev_op = (int*)calloc(n, sizeof(int));
        g->ev_a = (cudaEvent_t*)calloc(n, sizeof(cudaEvent_t));
        g->ev_b = (cudaEvent_t*)calloc(n, sizeof(cudaEvent_t));
    }
    uint64_t launches_before = atomic_load(&mcu_launch_counter);
    MCU_CHECK(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal));
    int rc = 0;
    for (size_t i = 0; i < n && !rc; ++i) {
        if (!is_compute(nodes[i]) || plan[i].kind == PLAN_SKIP) continue;
        if (d->profiling) {
            size_t k = g->n_ev++;
            g->ev_op[k] = nodes[i]->op;
            MCU_CHECK(cudaEventCreate(&g->ev_a[k]));
            MCU_CHECK(cudaEventCreate(&g->ev_b[k]));
            MCU_CHECK(cudaEventRecordWithFlags(g->ev_a[k], d->stream, cudaEventRecordExternal));
        }
        if (plan[i].kind == PLAN_FUSED || plan[i].a_split >= 0)
            rc = exec_planned_matmul(d, nodes[i], &plan[i], (char*)g->scratch, split_off, split_bytes);
        else
            rc = exec_node(d, nodes[i]);
        if (d->profiling) MCU_CHECK(cudaEventRecordWithFlags(g->ev_b[g->n_ev - 1], d->stream, cudaEventRecordExternal));
    }
    cudaError_t ce = cudaStreamEndCapture(d->stream, &graph);
    g->n_kernels = atomic_load(&mcu_launch_counter) - launches_before;
    atomic_fetch_sub(&mcu_launch_counter, g->n_kernels); /* captured, not yet run */
    d->capturing = 0;
    d->graph_scratch = NULL;
    d->scratch_bytes = saved_bytes;
    free(nodes);
    free(plan);
    if (rc || ce != cudaSuccess) {
        if (ce == cudaSuccess) cudaGraphDestroy(graph);
        g->exec = NULL;
        graph_free(g);
        return rc ? rc : (int)ce;
    }
    ce = cudaGraphInstantiate(&g->exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess) {
        g->exec = NULL;
        graph_free(g);
        return (int)ce;
    }
    g->next = d->graphs;
    d->graphs = g;
    g->ran = g->n_ev > 0;
    mcu_count_launches((int)g->n_kernels);
    return (int)cudaGraphLaunch(g->exec, d->stream);
}

int mag_cuda_graph_exec(mag_compute_device_t* dvc, mag_tensor_t* root) { return graph_exec_impl(dvc, root, 0); }

int mag_cuda_graph_exec_fused(mag_compute_device_t* dvc, mag_tensor_t* root) {
    return graph_exec_impl(dvc, root, 1);
}

int mag_cuda_graph_release(mag_compute_device_t* dvc, mag_tensor_t* root) {
    mcu_device* d = dev_of(dvc);
    int found = 0;
    cudaStreamSynchronize(d->stream);
    for (mcu_graph** pp = &d->graphs; *pp;) {
        if ((*pp)->root == root) {
            mcu_graph* g = *pp;
            *pp = g->next;
            graph_free(g);
            found = 1;
        } else {
            pp = &(*pp)->next;
        }
    }
    return found ? 0 : MAG_CUDA_E_INVALID;
}

/* --------------------------------------------------------- profiling --- */

static const char* const k_op_names[MAG_ABI_OP__COUNT] = {
    "NOP", "CLONE", "VIEW", "TRANSPOSE", "PERMUTE", "MEAN", "MIN", "MAX", "SUM", "ABS", "NEG", "LOG", "SQR",
    "SQRT", "SIN", "COS", "STEP", "SOFTMAX", "SOFTMAX_DV", "SIGMOID", "SIGMOID_DV", "HARD_SIGMOID", "SILU",
    "SILU_DV", "TANH", "TANH_DV", "RELU", "RELU_DV", "GELU", "GELU_DV", "ADD", "SUB", "MUL", "DIV", "ADDS",
    "SUBS", "MULS", "DIVS", "MATMUL"};

/* Adds the op event times of g's last replay to the per-op totals (wait: first wait for that
 * replay's last event; the stream need not be idle). */
static void harvest_graph_events(mcu_device* d, mcu_graph* g, int wait) {
    if (wait && g->n_ev) cudaEventSynchronize(g->ev_b[g->n_ev - 1]);
    for (size_t i = 0; i < g->n_ev; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, g->ev_a[i], g->ev_b[i]) == cudaSuccess) {
            d->prof_us[g->ev_op[i]] += ms * 1e3;
            d->prof_cnt[g->ev_op[i]]++;
        }
    }
    g->ran = 0;
}

int mag_cuda_profile_start(mag_compute_device_t* dvc) {
    mcu_device* d = dev_of(dvc);
    d->profiling = 1;
    memset(d->prof_us, 0, sizeof(d->prof_us));
    memset(d->prof_cnt, 0, sizeof(d->prof_cnt));
    return 0;
}

int mag_cuda_profile_collect(mag_compute_device_t* dvc) {
    mcu_device* d = dev_of(dvc);
    cudaError_t e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return (int)e;
    for (size_t i = 0; i < d->prof_n; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, d->prof[i].a, d->prof[i].b) == cudaSuccess) {
            d->prof_us[d->prof[i].op] += ms * 1e3;
            d->prof_cnt[d->prof[i].op]++;
        }
        cudaEventDestroy(d->prof[i].a);
        cudaEventDestroy(d->prof[i].b);
    }
    d->prof_n = 0;
    for (mcu_graph* g = d->graphs; g; g = g->next)
        if (g->ran) harvest_graph_events(d, g, 0);
    cudaGetLastError();
    return 0;
}

int mag_cuda_profile_stats(mag_compute_device_t* dvc, int op, uint64_t* count, double* total_us) {
    mcu_device* d = dev_of(dvc);
    if (op < 0 || op >= MAG_ABI_OP__COUNT) return MAG_CUDA_E_INVALID;
    if (count) *count = d->prof_cnt[op];
    if (total_us) *total_us = d->prof_us[op];
    return 0;
}

int mag_cuda_profile_stop(mag_compute_device_t* dvc, const char* csv_path) {
    mcu_device* d = dev_of(dvc);
    int rc = mag_cuda_profile_collect(dvc);
    if (rc) return rc;
    d->profiling = 0;
    uint64_t all = 0;
    for (int op = 0; op < MAG_ABI_OP__COUNT; ++op) all += d->prof_cnt[op];
    FILE* f = csv_path ? fopen(csv_path, "wt") : stdout;
    if (!f) return MAG_CUDA_E_INVALID;
    if (csv_path) fprintf(f, "Operation,Executions,Usage,AVG Time,Total Time\n");
    else printf("%16s %16s %16s %16s %16s\n", "Operation", "Executions", "Usage (%)", "AVG Time (us)", "Total Time (us)");
    /* rows by total time, longest first, ties in op order (the core's qsort by elapsed time,
     * magnetron/magnetron.c:1037-1043, :1085) */
    int order[MAG_ABI_OP__COUNT];
    for (int i = 0; i < MAG_ABI_OP__COUNT; ++i) order[i] = i;
    for (int i = 1; i < MAG_ABI_OP__COUNT; ++i) {
        const int v = order[i];
        int j = i;
        for (; j > 0 && d->prof_us[order[j - 1]] < d->prof_us[v]; --j) order[j] = order[j - 1];
        order[j] = v;
    }
    for (int k = 0; k < MAG_ABI_OP__COUNT; ++k) {
        const int op = order[k];
        if (!d->prof_cnt[op]) continue;
        double perc = (double)d->prof_cnt[op] / (double)all * 100.0;
        double avg = d->prof_us[op] / (double)d->prof_cnt[op];
        if (csv_path)
            fprintf(f, "%s,%llu,%.1f,%f,%f\n", k_op_names[op], (unsigned long long)d->prof_cnt[op], perc, avg,
                    d->prof_us[op]);
        else
            printf("%16s %16llu %16.1f%16f%16f\n", k_op_names[op], (unsigned long long)d->prof_cnt[op], perc, avg,
                   d->prof_us[op]);
    }
    if (csv_path) fclose(f);
    return 0;
}
