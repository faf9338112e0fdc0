// k_elementwise.cu - unary, scalar and binary (tiling-broadcast) f32 kernels.
//
// Reference semantics:
//   unary / scalar  r[ri*r_s1 + c] = f(x[ri*x_s1 + c]), ri < rows, c < cols
//                   (mag_blas_abs_f32 and siblings, magnetron/magnetron_cpu.c:1154-1570,
//                   :2016-2106); columns below cols & ~3 take the vector-lane
//                   formula, the rest the scalar tail.
//   binary          r[c + sum_k i_k*r_sk] = x[c + sum_k i_k*x_sk] (op)
//                   y[(c % y_d0)*y_s0 + sum_k (i_k % y_dk)*y_sk]
//                   (mag_blas_add_f32 and siblings, magnetron/magnetron_cpu.c:1616-2014)
//   broadcast2      r[i] = x[i mod x_d] (op) y[i mod y_d] per dim (extension)
//
// Layout: all three share HBM-streaming kernels: a linear path with 128-bit
// loads/stores for contiguous operands, and a row-segment path where one warp
// owns a 512-column segment of a row (all of its loads issued before the
// stores) and lane 0's row decomposition is broadcast with a shuffle, so
// per-element index work is one modulo at most.
#include <cuda_runtime.h>
#include <cstdint>
#include "mcu_math.cuh"
#include "mcu_kernels.h"

using namespace mcu;

namespace {

constexpr int kThreads = 256;

int g_sm_count = 0;
int sm_count() {
    if (!g_sm_count) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (g_sm_count <= 0) g_sm_count = 148;
    }
    return g_sm_count;
}

unsigned grid_for(uint64_t work_items, unsigned per_block) {
    uint64_t g = (work_items + per_block - 1) / per_block;
    uint64_t cap = (uint64_t)sm_count() * 16;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (unsigned)g;
}

// Out of line so a runtime lane/tail choice is a branch, not both evaluated.
template <int OP>
__device__ __noinline__ float tail_call(float x) { return tail_op<OP>(x); }

template <int OP>
__device__ __forceinline__ float uapply(float x, float xi, bool lane) {
    if constexpr (is_lane_op(OP)) {
        if (lane) return lane_op<OP>(x);
        return tail_call<OP>(x);
    } else {
        return exact_op<OP>(x, xi);
    }
}

// ---------------------------------------------------------------- unary ---

// Contiguous rows whose length is a multiple of 4: every element is a lane.
template <int OP>
__global__ void __launch_bounds__(kThreads) unary_vec4(float4* __restrict__ r, const float4* __restrict__ x,
                                                       uint64_t n4, float xi) {
    uint64_t stride = (uint64_t)gridDim.x * kThreads;
    uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
    if constexpr (is_lane_op(OP)) {
        // polynomial lanes: the next four loads are issued before this group is computed
        if (i + 3 * stride < n4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldcs(x + i + u * stride);
            for (;;) {
                const uint64_t in = i + 4 * stride;
                const bool more = in + 3 * stride < n4;
                float4 w[4];
                if (more) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) w[u] = __ldcs(x + in + u * stride);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float4 o;
                    o.x = uapply<OP>(v[u].x, xi, true);
                    o.y = uapply<OP>(v[u].y, xi, true);
                    o.z = uapply<OP>(v[u].z, xi, true);
                    o.w = uapply<OP>(v[u].w, xi, true);
                    __stcs(r + i + u * stride, o);
                }
                i = in;
                if (!more) break;
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = w[u];
            }
        }
    } else {
        for (; i + 3 * stride < n4; i += 4 * stride) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldcs(x + i + u * stride);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float4 o;
                o.x = uapply<OP>(v[u].x, xi, true);
                o.y = uapply<OP>(v[u].y, xi, true);
                o.z = uapply<OP>(v[u].z, xi, true);
                o.w = uapply<OP>(v[u].w, xi, true);
                __stcs(r + i + u * stride, o);
            }
        }
    }
    for (; i < n4; i += stride) {
        float4 v = __ldcs(x + i), o;
        o.x = uapply<OP>(v.x, xi, true);
        o.y = uapply<OP>(v.y, xi, true);
        o.z = uapply<OP>(v.z, xi, true);
        o.w = uapply<OP>(v.w, xi, true);
        __stcs(r + i, o);
    }
}

// Contiguous rows of any length: column = i % cols decides lane or tail.
template <int OP>
__global__ void __launch_bounds__(kThreads) unary_flat(float* __restrict__ r, const float* __restrict__ x,
                                                       uint64_t n, uint32_t vec_end, FastDiv cols, float xi) {
    uint64_t stride = (uint64_t)gridDim.x * kThreads;
    for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) {
        bool lane = true;
        if constexpr (is_lane_op(OP)) {
            uint32_t ii = (uint32_t)i;
            uint32_t c = ii - fdiv(ii, cols) * cols.d;
            lane = c < vec_end;
        }
        r[i] = uapply<OP>(x[i], xi, lane);
    }
}

// Strided rows: a warp walks 128-column segments of one row.
template <int OP>
__global__ void __launch_bounds__(kThreads) unary_rows(float* __restrict__ r, const float* __restrict__ x,
                                                       uint64_t nseg, FastDiv segs_per_row, uint32_t cols,
                                                       uint32_t vec_end, int64_t r_s1, int64_t x_s1, float xi) {
    const int lane_id = threadIdx.x & 31;
    uint64_t warp = ((uint64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    uint64_t nwarps = ((uint64_t)gridDim.x * kThreads) >> 5;
    for (uint64_t s = warp; s < nseg; s += nwarps) {
        uint32_t ss = (uint32_t)s;
        uint32_t row = fdiv(ss, segs_per_row);
        uint32_t seg = ss - row * segs_per_row.d;
        const float* px = x + (int64_t)row * x_s1;
        float* pr = r + (int64_t)row * r_s1;
        uint32_t c0 = seg * 128u + (uint32_t)lane_id;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            uint32_t c = c0 + 32u * u;
            if (c < cols) pr[c] = uapply<OP>(px[c], xi, c < vec_end);
        }
    }
}

template <int OP>
cudaError_t launch_unary_op(float* r, const float* x, int64_t rows, int64_t cols, int64_t r_s1, int64_t x_s1,
                            float xi, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    uint64_t n = (uint64_t)rows * (uint64_t)cols;
    bool contiguous = r_s1 == cols && x_s1 == cols;
    if (rows == 1) contiguous = true;
    uint32_t vec_end = (uint32_t)(cols & ~3ll);
    bool aligned = (((uintptr_t)r | (uintptr_t)x) & 15) == 0;
    if (contiguous && (cols % 4 == 0) && aligned) {
        uint64_t n4 = n / 4;
        unary_vec4<OP><<<grid_for(n4, kThreads * 4), kThreads, 0, st>>>((float4*)r, (const float4*)x, n4, xi);
    } else if (contiguous && n < (1ull << 32)) {
        unary_flat<OP><<<grid_for(n, kThreads), kThreads, 0, st>>>(r, x, n, vec_end, make_fastdiv((uint32_t)cols), xi);
    } else {
        uint64_t spr = ((uint64_t)cols + 127) / 128;
        uint64_t nseg = (uint64_t)rows * spr;
        if (nseg >= (1ull << 32) || cols >= (1ll << 32)) return cudaErrorInvalidValue;
        unary_rows<OP><<<grid_for(nseg * 32, kThreads), kThreads, 0, st>>>(r, x, nseg, make_fastdiv((uint32_t)spr),
                                                                           (uint32_t)cols, vec_end, r_s1, x_s1, xi);
    }
    return cudaGetLastError();
}

// --------------------------------------------------------------- binary ---

// Same-shape contiguous operands.
template <int OP>
__global__ void __launch_bounds__(kThreads) binary_vec4(float4* __restrict__ r, const float4* __restrict__ x,
                                                        const float4* __restrict__ y, uint64_t n4) {
    uint64_t stride = (uint64_t)gridDim.x * kThreads;
    uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
    for (; i + stride < n4; i += 2 * stride) {
        float4 a0 = __ldcs(x + i), b0 = __ldcs(y + i);
        float4 a1 = __ldcs(x + i + stride), b1 = __ldcs(y + i + stride);
        float4 o0, o1;
        o0.x = binop<OP>(a0.x, b0.x); o0.y = binop<OP>(a0.y, b0.y); o0.z = binop<OP>(a0.z, b0.z); o0.w = binop<OP>(a0.w, b0.w);
        o1.x = binop<OP>(a1.x, b1.x); o1.y = binop<OP>(a1.y, b1.y); o1.z = binop<OP>(a1.z, b1.z); o1.w = binop<OP>(a1.w, b1.w);
        __stcs(r + i, o0);
        __stcs(r + i + stride, o1);
    }
    for (; i < n4; i += stride) {
        float4 a = __ldcs(x + i), b = __ldcs(y + i), o;
        o.x = binop<OP>(a.x, b.x); o.y = binop<OP>(a.y, b.y); o.z = binop<OP>(a.z, b.z); o.w = binop<OP>(a.w, b.w);
        __stcs(r + i, o);
    }
}

template <int OP>
__global__ void __launch_bounds__(kThreads) binary_flat(float* __restrict__ r, const float* __restrict__ x,
                                                        const float* __restrict__ y, uint64_t n) {
    uint64_t stride = (uint64_t)gridDim.x * kThreads;
    for (uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) r[i] = binop<OP>(x[i], y[i]);
}

// Iteration space: d[0] columns per row, rows = prod d[1..5].  Offsets of r,
// x and y are strides times the row indices; x and y may wrap modulo their
// own dims (x wraps only for the two-sided broadcast).
struct RowParams {
    int64_t rs[6], xs[6], ys[6];
    FastDiv dim[6];   // iteration dims
    FastDiv xdim[6];  // x dims (modulo)
    FastDiv ydim[6];  // y dims (modulo)
    FastDiv segs_per_row;
    uint64_t nseg;
    uint32_t cols;
    int y_mode;       // 0: y column == c*ys0, 1: y column fixed (y_d0 == 1), 2: c % y_d0
    int x_mod;        // x column wraps modulo x_d0 (row indices always wrap modulo x's dims)
    uint32_t seg_w;   // columns per warp iteration: 128 * steps, steps = 1..4 (row length rounded up)
    int steps;
};

__device__ __forceinline__ uint32_t mod_by(uint32_t v, const FastDiv& f) { return v - fdiv(v, f) * f.d; }


template <int OP, bool VEC>
__global__ void __launch_bounds__(kThreads, 4) binary_rows(float* __restrict__ r, const float* __restrict__ x,
                                                        const float* __restrict__ y, const RowParams p) {
    const int lane_id = threadIdx.x & 31;
    uint64_t warp = ((uint64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    uint64_t nwarps = ((uint64_t)gridDim.x * kThreads) >> 5;
    for (uint64_t s = warp; s < p.nseg; s += nwarps) {
        int64_t ro = 0, xo = 0, yo = 0;
        uint32_t seg = 0;
        if (lane_id == 0) {
            uint32_t q = (uint32_t)s;
            uint32_t row = fdiv(q, p.segs_per_row);
            seg = q - row * p.segs_per_row.d;
#pragma unroll
            for (int k = 1; k < 6; ++k) {
                uint32_t nq = fdiv(row, p.dim[k]);
                uint32_t ik = row - nq * p.dim[k].d;
                row = nq;
                ro += (int64_t)ik * p.rs[k];
                xo += (int64_t)mod_by(ik, p.xdim[k]) * p.xs[k];
                yo += (int64_t)mod_by(ik, p.ydim[k]) * p.ys[k];
            }
        }
        ro = __shfl_sync(0xffffffffu, ro, 0);
        xo = __shfl_sync(0xffffffffu, xo, 0);
        yo = __shfl_sync(0xffffffffu, yo, 0);
        seg = __shfl_sync(0xffffffffu, seg, 0);
        if constexpr (VEC) {
            float4 a[4], b[4];
            uint32_t cs[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t c = seg * p.seg_w + 128u * u + 4u * (uint32_t)lane_id;
                cs[u] = c;
                if (u < p.steps && c < p.cols) {
                    const uint32_t xc = p.x_mod ? mod_by(c, p.xdim[0]) : c;
                    a[u] = *(const float4*)(x + xo + xc);
                    if (p.y_mode == 1) {
                        const float t = y[yo];
                        b[u] = make_float4(t, t, t, t);
                    } else {
                        const uint32_t yc = p.y_mode == 0 ? c : mod_by(c, p.ydim[0]);
                        b[u] = *(const float4*)(y + yo + yc);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (u < p.steps && cs[u] < p.cols) {
                    float4 o;
                    o.x = binop<OP>(a[u].x, b[u].x); o.y = binop<OP>(a[u].y, b[u].y);
                    o.z = binop<OP>(a[u].z, b[u].z); o.w = binop<OP>(a[u].w, b[u].w);
                    __stcs((float4*)(r + ro + cs[u]), o);
                }
            }
        } else {
#pragma unroll 4
            for (int u = 0; u < 16; ++u) {
                uint32_t c = seg * p.seg_w + (uint32_t)lane_id + 32u * u;
                if (u < 4 * p.steps && c < p.cols) {
                    uint32_t xc = p.x_mod ? mod_by(c, p.xdim[0]) : c;
                    int64_t yc = p.y_mode == 0 ? (int64_t)c * p.ys[0]
                               : p.y_mode == 1 ? 0 : (int64_t)mod_by(c, p.ydim[0]) * p.ys[0];
                    r[ro + c] = binop<OP>(x[xo + xc], y[yo + yc]);
                }
            }
        }
    }
}

// Rows of at most 512 columns, vectorised: a warp walks kRowChunk consecutive
// rows; the first row's indices are decomposed once and later rows advance
// them with a carry, keeping x's and y's wrapped indices in step.
constexpr uint32_t kRowChunk = 16;

// One row's offsets, advanced by one row along dim 1 with a carry into dims 2..5; x's and
// y's wrapped indices move in step.
struct RowWalk {
    uint32_t idx[6], xi[6], yi[6];
    int64_t ro, xo, yo;

    __device__ __forceinline__ void start(uint32_t row0, const RowParams& p) {
        ro = xo = yo = 0;
        uint32_t q = row0;
#pragma unroll
        for (int k = 1; k < 6; ++k) {
            const uint32_t nq = fdiv(q, p.dim[k]);
            idx[k] = q - nq * p.dim[k].d;
            q = nq;
            xi[k] = mod_by(idx[k], p.xdim[k]);
            yi[k] = mod_by(idx[k], p.ydim[k]);
            ro += (int64_t)idx[k] * p.rs[k];
            xo += (int64_t)xi[k] * p.xs[k];
            yo += (int64_t)yi[k] * p.ys[k];
        }
    }
    __device__ __forceinline__ void next(const RowParams& p) {
#pragma unroll
        for (int k = 1; k < 6; ++k) {
            ++idx[k];
            ro += p.rs[k];
            if (++xi[k] == p.xdim[k].d) { xi[k] = 0; xo -= (int64_t)(p.xdim[k].d - 1) * p.xs[k]; } else { xo += p.xs[k]; }
            if (++yi[k] == p.ydim[k].d) { yi[k] = 0; yo -= (int64_t)(p.ydim[k].d - 1) * p.ys[k]; } else { yo += p.ys[k]; }
            if (idx[k] < p.dim[k].d) break;
            idx[k] = 0;
            ro -= (int64_t)p.dim[k].d * p.rs[k];
            // the wrapped indices of x and y restart at 0 together with idx[k]
            xo -= (int64_t)xi[k] * p.xs[k];
            yo -= (int64_t)yi[k] * p.ys[k];
            xi[k] = 0;
            yi[k] = 0;
        }
    }
};

// Rows of at most 128 * STEPS columns, vectorised: a warp walks `chunk` consecutive rows
// (kRowChunk, fewer when the tensor has few rows),
// decomposing the first row's indices once and carrying them to the next rows, with several
// rows' loads in flight before their stores.  ONCE = 1 (2): x's (y's) row is the same for every
// row of a chunk (its dim 1 has extent 1 and chunks do not cross dim 1), so it is loaded once
// per chunk and only the other operand's rows per row.
template <int OP, int STEPS, int ONCE>
__global__ void __launch_bounds__(kThreads, 2) binary_rows_chunked(float* __restrict__ r, const float* __restrict__ x,
                                                                   const float* __restrict__ y, const RowParams p,
                                                                   uint32_t nrows, uint32_t nchunks, uint32_t chunk) {
    const int lane_id = threadIdx.x & 31;
    const uint32_t warp = (uint32_t)(((uint64_t)blockIdx.x * kThreads + threadIdx.x) >> 5);
    const uint32_t nwarps = (uint32_t)(((uint64_t)gridDim.x * kThreads) >> 5);
    auto load_x = [&](int64_t xo, float4 (&a)[STEPS]) {
#pragma unroll
        for (int u = 0; u < STEPS; ++u) {
            const uint32_t c = 128u * u + 4u * (uint32_t)lane_id;
            if (c < p.cols) {
                const uint32_t xc = p.x_mod ? mod_by(c, p.xdim[0]) : c;
                a[u] = *(const float4*)(x + xo + xc);
            }
        }
    };
    auto load_y = [&](int64_t yo, float4 (&b)[STEPS]) {
#pragma unroll
        for (int u = 0; u < STEPS; ++u) {
            const uint32_t c = 128u * u + 4u * (uint32_t)lane_id;
            if (c < p.cols) {
                if (p.y_mode == 1) {
                    const float t = y[yo];
                    b[u] = make_float4(t, t, t, t);
                } else {
                    const uint32_t yc = p.y_mode == 0 ? c : mod_by(c, p.ydim[0]);
                    b[u] = *(const float4*)(y + yo + yc);
                }
            }
        }
    };
    auto store_row = [&](int64_t ro, const float4 (&a)[STEPS], const float4 (&b)[STEPS]) {
#pragma unroll
        for (int u = 0; u < STEPS; ++u) {
            const uint32_t c = 128u * u + 4u * (uint32_t)lane_id;
            if (c < p.cols) {
                float4 o;
                o.x = binop<OP>(a[u].x, b[u].x); o.y = binop<OP>(a[u].y, b[u].y);
                o.z = binop<OP>(a[u].z, b[u].z); o.w = binop<OP>(a[u].w, b[u].w);
                __stcs((float4*)(r + ro + c), o);
            }
        }
    };
    for (uint32_t ch = warp; ch < nchunks; ch += nwarps) {
        const uint32_t row0 = ch * chunk;
        RowWalk w;
        w.start(row0, p);
        const uint32_t rows_here = min(chunk, nrows - row0);
        if constexpr (ONCE != 0) {
            // one operand's row for the whole chunk, the other's R rows in flight
            constexpr int R = STEPS <= 2 ? 8 : 2;
            float4 fixed[STEPS];
            if constexpr (ONCE == 1) load_x(w.xo, fixed);
            else load_y(w.yo, fixed);
            for (uint32_t rr = 0; rr < rows_here; rr += R) {
                float4 v[R][STEPS];
                int64_t ro[R];
                const uint32_t nr = min((uint32_t)R, rows_here - rr);
#pragma unroll
                for (int k = 0; k < R; ++k) {
                    if ((uint32_t)k < nr) {
                        ro[k] = w.ro;
                        if constexpr (ONCE == 1) load_y(w.yo, v[k]);
                        else load_x(w.xo, v[k]);
                        w.next(p);
                    }
                }
#pragma unroll
                for (int k = 0; k < R; ++k) {
                    if ((uint32_t)k < nr) {
                        if constexpr (ONCE == 1) store_row(ro[k], fixed, v[k]);
                        else store_row(ro[k], v[k], fixed);
                    }
                }
            }
            continue;
        }
        // R rows' loads in flight before their stores: 4 for rows of at most 256 columns
        // (the loads are L2 latency-bound there; 114 registers allow 2 CTAs per SM), else 2
        constexpr int R = STEPS <= 2 ? 4 : 2;
        for (uint32_t rr = 0; rr < rows_here; rr += R) {
            float4 a[R][STEPS], b[R][STEPS];
            int64_t ro[R];
            const uint32_t nr = min((uint32_t)R, rows_here - rr);
#pragma unroll
            for (int k = 0; k < R; ++k) {
                if ((uint32_t)k < nr) {
                    ro[k] = w.ro;
                    load_x(w.xo, a[k]);
                    load_y(w.yo, b[k]);
                    w.next(p);
                }
            }
#pragma unroll
            for (int k = 0; k < R; ++k)
                if ((uint32_t)k < nr) store_row(ro[k], a[k], b[k]);
        }
    }
}

bool fits_u32(int64_t v) { return v >= 0 && v < (1ll << 32); }

template <int OP>
cudaError_t launch_rows(float* r, const float* x, const float* y, const int64_t* dims, const int64_t* rs,
                        const int64_t* xd, const int64_t* xs, const int64_t* yd, const int64_t* ys, bool x_mod,
                        cudaStream_t st) {
    RowParams p{};
    uint64_t rows = 1;
    for (int k = 0; k < 6; ++k) {
        if (!fits_u32(dims[k]) || !fits_u32(xd[k]) || !fits_u32(yd[k]) || dims[k] == 0 || xd[k] == 0 || yd[k] == 0)
            return cudaErrorInvalidValue;
        p.rs[k] = rs[k];
        p.xs[k] = xs[k];
        p.ys[k] = ys[k];
        p.dim[k] = make_fastdiv((uint32_t)dims[k]);
        p.xdim[k] = make_fastdiv((uint32_t)xd[k]);
        p.ydim[k] = make_fastdiv((uint32_t)yd[k]);
        if (k) rows *= (uint64_t)dims[k];
    }
    p.steps = (int)(((uint64_t)dims[0] + 127) / 128 < 4 ? ((uint64_t)dims[0] + 127) / 128 : 4);
    p.seg_w = 128u * (uint32_t)p.steps;
    uint64_t spr = ((uint64_t)dims[0] + p.seg_w - 1) / p.seg_w;
    p.segs_per_row = make_fastdiv((uint32_t)spr);
    p.nseg = rows * spr;
    if (p.nseg >= (1ull << 32)) return cudaErrorInvalidValue;
    p.cols = (uint32_t)dims[0];
    p.x_mod = x_mod && xd[0] != dims[0] ? 1 : 0;
    p.y_mode = yd[0] == dims[0] ? 0 : (yd[0] == 1 ? 1 : 2);
    bool vec = dims[0] % 4 == 0 && (((uintptr_t)r | (uintptr_t)x) & 15) == 0 && xs[0] == 1 && rs[0] == 1;
    if (x_mod) vec = vec && xd[0] % 4 == 0;
    for (int k = 1; k < 6; ++k) vec = vec && rs[k] % 4 == 0 && xs[k] % 4 == 0;
    if (p.y_mode != 1) {
        vec = vec && ys[0] == 1 && yd[0] % 4 == 0 && ((uintptr_t)y & 15) == 0;
        for (int k = 1; k < 6; ++k) vec = vec && ys[k] % 4 == 0;
    }
    if (vec && p.steps <= 4 && dims[0] <= 512 && rows >= 4 * kRowChunk && rows < (1ull << 32)) {
        // kRowChunk rows per warp, fewer when that leaves fewer than four chunks per SM
        uint32_t chunk = kRowChunk;
        while (chunk > 1 && rows / chunk < 4ull * (uint64_t)sm_count()) chunk /= 2;
        const uint32_t nchunks = (uint32_t)((rows + chunk - 1) / chunk);
        const unsigned g = grid_for((uint64_t)nchunks * 32, kThreads);
        // an operand whose dim 1 has extent 1 keeps its row across a chunk that stays inside dim 1
        const bool in_dim1 = (uint64_t)dims[1] % chunk == 0;
        const int once = !in_dim1 ? 0 : xd[1] == 1 && dims[1] > 1 ? 1 : (yd[1] == 1 && dims[1] > 1 ? 2 : 0);
#define MCU_ROWS_LAUNCH(S, O) binary_rows_chunked<OP, S, O><<<g, kThreads, 0, st>>>(r, x, y, p, (uint32_t)rows, nchunks, chunk)
#define MCU_ROWS_STEPS(S)                                \
    do {                                                 \
        if (once == 1) MCU_ROWS_LAUNCH(S, 1);            \
        else if (once == 2) MCU_ROWS_LAUNCH(S, 2);       \
        else MCU_ROWS_LAUNCH(S, 0);                      \
    } while (0)
        switch (p.steps) {
            case 1: MCU_ROWS_STEPS(1); break;
            case 2: MCU_ROWS_STEPS(2); break;
            case 3: MCU_ROWS_STEPS(3); break;
            default: MCU_ROWS_STEPS(4); break;
        }
#undef MCU_ROWS_STEPS
#undef MCU_ROWS_LAUNCH
        return cudaGetLastError();
    }
    unsigned grid = grid_for(p.nseg * 32, kThreads);
    if (vec) binary_rows<OP, true><<<grid, kThreads, 0, st>>>(r, x, y, p);
    else binary_rows<OP, false><<<grid, kThreads, 0, st>>>(r, x, y, p);
    return cudaGetLastError();
}

bool canonical(const int64_t* d, const int64_t* s) {
    int64_t acc = 1;
    for (int k = 0; k < 6; ++k) {
        if (d[k] != 1 && s[k] != acc) return false;
        acc *= d[k];
    }
    return true;
}

template <int OP>
cudaError_t launch_binary_op(float* r, const float* x, const float* y, const int64_t* xd, const int64_t* xs,
                             const int64_t* rs, const int64_t* yd, const int64_t* ys, cudaStream_t st) {
    uint64_t n = 1;
    bool same = true;
    for (int k = 0; k < 6; ++k) {
        if (xd[k] <= 0) return cudaSuccess;
        n *= (uint64_t)xd[k];
        same = same && yd[k] == xd[k];
    }
    if (same && canonical(xd, xs) && canonical(xd, rs) && canonical(yd, ys)) {
        if (n % 4 == 0 && (((uintptr_t)r | (uintptr_t)x | (uintptr_t)y) & 15) == 0) {
            uint64_t n4 = n / 4;
            binary_vec4<OP><<<grid_for(n4, kThreads * 2), kThreads, 0, st>>>((float4*)r, (const float4*)x,
                                                                             (const float4*)y, n4);
        } else {
            binary_flat<OP><<<grid_for(n, kThreads), kThreads, 0, st>>>(r, x, y, n);
        }
        return cudaGetLastError();
    }
    return launch_rows<OP>(r, x, y, xd, rs, xd, xs, yd, ys, false, st);
}

}  // namespace

#define MCU_UNARY_CASE(NAME) case OP_##NAME: return launch_unary_op<OP_##NAME>(r, x, rows, cols, r_s1, x_s1, xi, st);
#define MCU_BINARY_CASE(NAME) case OP_##NAME: return launch_binary_op<OP_##NAME>(r, x, y, xd, xs, rs, yd, ys, st);

extern "C" int mcu_launch_unary(int op, float* r, const float* x, int64_t rows, int64_t cols, int64_t r_s1,
                                int64_t x_s1, float xi, cudaStream_t st) {
    switch (op) {
        MCU_UNARY_CASE(ABS) MCU_UNARY_CASE(NEG) MCU_UNARY_CASE(LOG) MCU_UNARY_CASE(SQR) MCU_UNARY_CASE(SQRT)
        MCU_UNARY_CASE(SIN) MCU_UNARY_CASE(COS) MCU_UNARY_CASE(STEP) MCU_UNARY_CASE(SOFTMAX)
        MCU_UNARY_CASE(SOFTMAX_DV) MCU_UNARY_CASE(SIGMOID) MCU_UNARY_CASE(SIGMOID_DV) MCU_UNARY_CASE(HARD_SIGMOID)
        MCU_UNARY_CASE(SILU) MCU_UNARY_CASE(TANH) MCU_UNARY_CASE(TANH_DV) MCU_UNARY_CASE(RELU)
        MCU_UNARY_CASE(RELU_DV) MCU_UNARY_CASE(GELU) MCU_UNARY_CASE(ADDS) MCU_UNARY_CASE(SUBS)
        MCU_UNARY_CASE(MULS) MCU_UNARY_CASE(DIVS)
        default: return (int)cudaErrorInvalidValue;
    }
}

extern "C" int mcu_launch_binary(int op, float* r, const float* x, const float* y, const int64_t* xd,
                                 const int64_t* xs, const int64_t* rs, const int64_t* yd, const int64_t* ys,
                                 cudaStream_t st) {
    switch (op) {
        MCU_BINARY_CASE(ADD) MCU_BINARY_CASE(SUB) MCU_BINARY_CASE(MUL) MCU_BINARY_CASE(DIV)
        default: return (int)cudaErrorInvalidValue;
    }
}

extern "C" int mcu_launch_bcast2(int op, float* r, const float* x, const float* y, const int64_t* rd,
                                 const int64_t* xd, const int64_t* yd, cudaStream_t st) {
    int64_t rs[6], xs[6], ys[6];
    rs[0] = xs[0] = ys[0] = 1;
    for (int k = 1; k < 6; ++k) {
        rs[k] = rs[k - 1] * rd[k - 1];
        xs[k] = xs[k - 1] * xd[k - 1];
        ys[k] = ys[k - 1] * yd[k - 1];
    }
    for (int k = 0; k < 6; ++k)
        if (rd[k] <= 0 || xd[k] <= 0 || yd[k] <= 0 || rd[k] % xd[k] || rd[k] % yd[k]) return (int)cudaErrorInvalidValue;
    switch (op) {
        case OP_ADD: return launch_rows<OP_ADD>(r, x, y, rd, rs, xd, xs, yd, ys, true, st);
        case OP_SUB: return launch_rows<OP_SUB>(r, x, y, rd, rs, xd, xs, yd, ys, true, st);
        case OP_MUL: return launch_rows<OP_MUL>(r, x, y, rd, rs, xd, xs, yd, ys, true, st);
        case OP_DIV: return launch_rows<OP_DIV>(r, x, y, rd, rs, xd, xs, yd, ys, true, st);
        default: return (int)cudaErrorInvalidValue;
    }
}
