/*
 * mag_cuda_abi.h - binary layout of the magnetron core types that a compute
 * device backend reads and writes.
 *
 * A device backend is loaded by the unchanged magnetron core and receives raw
 * pointers to the core's tensor, storage and device structs.  This header
 * restates exactly the layout the core uses on LP64 targets (x86-64, aarch64)
 * with MAG_SANITIZE_RC=0, so the backend can be compiled without the core's
 * private header.  Field order, types and sizes must match the core, which is
 * why the struct bodies below follow it member for member; every struct has
 * offset checks at the bottom of this file.
 *
 *   mag_storage_buffer    <- magnetron/magnetron_internal.h:324-334
 *   mag_compute_device_t  <- magnetron/magnetron_internal.h:336-346
 *   mag_tensor_t          <- magnetron/magnetron_internal.h:427-455
 *   mag_op_t numbering    <- magnetron/magnetron.h:136-178 (mag_op_def order)
 *   op parameter packing  <- magnetron/magnetron.c:1120-1138
 */
#ifndef MAG_CUDA_ABI_H
#define MAG_CUDA_ABI_H

#include <stdint.h>
#include <stddef.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MAG_ABI_MAX_DIMS 6
#define MAG_ABI_MAX_INPUTS 2
#define MAG_ABI_MAX_PARAMS 6
#define MAG_ABI_MAX_NAME 64

/* Compute device kinds (magnetron/magnetron.h:58-61). */
typedef enum mag_abi_device_type_t {
    MAG_ABI_DEVICE_CPU = 0,
    MAG_ABI_DEVICE_CUDA = 1
} mag_abi_device_type_t;

/* Operator codes in the order of the core's op table (magnetron/magnetron.h:136-178). */
typedef enum mag_abi_op_t {
    MAG_ABI_OP_NOP = 0,
    MAG_ABI_OP_CLONE,
    MAG_ABI_OP_VIEW,
    MAG_ABI_OP_TRANSPOSE,
    MAG_ABI_OP_PERMUTE,
    MAG_ABI_OP_MEAN,
    MAG_ABI_OP_MIN,
    MAG_ABI_OP_MAX,
    MAG_ABI_OP_SUM,
    MAG_ABI_OP_ABS,
    MAG_ABI_OP_NEG,
    MAG_ABI_OP_LOG,
    MAG_ABI_OP_SQR,
    MAG_ABI_OP_SQRT,
    MAG_ABI_OP_SIN,
    MAG_ABI_OP_COS,
    MAG_ABI_OP_STEP,
    MAG_ABI_OP_SOFTMAX,
    MAG_ABI_OP_SOFTMAX_DV,
    MAG_ABI_OP_SIGMOID,
    MAG_ABI_OP_SIGMOID_DV,
    MAG_ABI_OP_HARD_SIGMOID,
    MAG_ABI_OP_SILU,
    MAG_ABI_OP_SILU_DV,
    MAG_ABI_OP_TANH,
    MAG_ABI_OP_TANH_DV,
    MAG_ABI_OP_RELU,
    MAG_ABI_OP_RELU_DV,
    MAG_ABI_OP_GELU,
    MAG_ABI_OP_GELU_DV,
    MAG_ABI_OP_ADD,
    MAG_ABI_OP_SUB,
    MAG_ABI_OP_MUL,
    MAG_ABI_OP_DIV,
    MAG_ABI_OP_ADDS,
    MAG_ABI_OP_SUBS,
    MAG_ABI_OP_MULS,
    MAG_ABI_OP_DIVS,
    MAG_ABI_OP_MATMUL,
    MAG_ABI_OP__COUNT
} mag_abi_op_t;

/* Tensor flags (magnetron/magnetron_internal.h:416-423). */
enum {
    MAG_ABI_TFLAG_OWNER = 1 << 0,
    MAG_ABI_TFLAG_VIEW = 1 << 1
};

typedef struct mag_compute_device_t mag_compute_device_t;
typedef struct mag_storage_buffer mag_storage_buffer;
typedef struct mag_tensor_t mag_tensor_t;
typedef struct mag_ctx_t mag_ctx_t; /* opaque: a backend never dereferences the context */

/* Device buffer handle, copied by value into every view of a tensor. */
struct mag_storage_buffer {
    uintptr_t base;                 /* device address of the first byte */
    size_t size;                    /* bytes */
    size_t alignment;               /* bytes */
    mag_compute_device_t* host;     /* owning device */
    void (*set)(mag_storage_buffer* sto, size_t offs, uint8_t x);                              /* fill [offs, size) with byte x */
    void (*cpy_host_device)(mag_storage_buffer* sto, size_t offs, const void* src, size_t n);  /* host -> device */
    void (*cpy_device_host)(mag_storage_buffer* sto, size_t offs, void* dst, size_t n);        /* device -> host */
};

/* Device vtable the core calls for every tensor allocation and every op. */
struct mag_compute_device_t {
    char name[128];
    void* impl;
    bool is_async;
    int32_t type;                   /* mag_abi_device_type_t, stored as the core's enum (4 bytes) */
    void (*eager_exec_fwd)(mag_compute_device_t* dvc, mag_tensor_t* root);
    void (*eager_exec_bwd)(mag_compute_device_t* dvc, mag_tensor_t* root);
    void (*alloc_storage)(mag_compute_device_t* dvc, mag_storage_buffer* out, size_t size, size_t align);
    void (*free_storage)(mag_compute_device_t* dvc, mag_storage_buffer* buf);
};

typedef struct mag_abi_perf_mon_t {
    uint64_t elapsed_ns;
    uint64_t elapsed_ns_acc;
    uint64_t n_execs;
} mag_abi_perf_mon_t;

/* Tensor node: shape and strides in elements, dim 0 fastest, plus its op record. */
struct mag_tensor_t {
    struct {
        uint32_t rc_strong;
        uint32_t rc_weak;
    } rcb;
    mag_ctx_t* ctx;
    int64_t rank;
    int64_t shape[MAG_ABI_MAX_DIMS];
    int64_t strides[MAG_ABI_MAX_DIMS];
    int32_t dtype;                  /* 0 = f32 (the only dtype the core defines) */
    mag_storage_buffer storage;
    int64_t numel;
    int32_t flags;
    int32_t op;                     /* mag_abi_op_t */
    mag_tensor_t* op_inputs[MAG_ABI_MAX_INPUTS];
    uint64_t op_params[MAG_ABI_MAX_PARAMS];
    mag_tensor_t* view_uplink;
    size_t view_offs;
    mag_tensor_t* grad;
    mag_abi_perf_mon_t pmon;
    char name[MAG_ABI_MAX_NAME];
    void* ud;
};

/* Op parameter: 2-bit tag in bits 62..63 (0 = float, 1 = int), value in the low bits. */
static inline float mag_abi_param_f32(uint64_t p) {
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)(p & ((1ull << 62) - 1));
    return v.f;
}
static inline uint64_t mag_abi_param_from_f32(float x) {
    union { uint32_t u; float f; } v;
    v.f = x;
    return (uint64_t)v.u; /* tag 0 = float */
}

#if defined(__cplusplus)
#define MAG_ABI_SASSERT(e, m) static_assert(e, m)
#else
#define MAG_ABI_SASSERT(e, m) _Static_assert(e, m)
#endif
MAG_ABI_SASSERT(sizeof(mag_storage_buffer) == 56, "storage layout");
MAG_ABI_SASSERT(offsetof(mag_compute_device_t, impl) == 128, "device layout");
MAG_ABI_SASSERT(offsetof(mag_compute_device_t, type) == 140, "device layout");
MAG_ABI_SASSERT(offsetof(mag_compute_device_t, eager_exec_fwd) == 144, "device layout");
MAG_ABI_SASSERT(sizeof(mag_compute_device_t) == 176, "device layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, shape) == 24, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, strides) == 72, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, storage) == 128, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, numel) == 184, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, op) == 196, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, op_inputs) == 200, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, op_params) == 216, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, view_uplink) == 264, "tensor layout");
MAG_ABI_SASSERT(offsetof(mag_tensor_t, name) == 312, "tensor layout");
MAG_ABI_SASSERT(sizeof(mag_tensor_t) == 384, "tensor layout");

#ifdef __cplusplus
}
#endif
#endif /* MAG_CUDA_ABI_H */
