// k_reduce.cu - reductions and the row softmax.
//
// Full-tensor SUM/MEAN/MIN/MAX follow mag_blas_{sum,mean,min,max}_f32
// (magnetron/magnetron_cpu.c:1034-1152): the value goes to r[0]; sums are
// accumulated in double (mag_vsum_f64_f32, :477-492) and rounded to f32 once,
// MEAN divides the double sum by numel first; MIN/MAX use fminf/fmaxf.  The
// GPU adds in a fixed tree order (per-thread, warp shuffle, per-block, then one
// block over the block partials), so results are deterministic run to run.
//
// Row reductions and the normalised row softmax are extensions with the same
// arithmetic per row.  The softmax keeps rows of up to 65536 on chip (registers
// of one warp, or of a thread-block cluster of up to 8 CTAs that combine the row
// max and the double sum through distributed shared memory), so HBM sees one
// read and one write per element (8 B/elem) and exp is evaluated once; wider
// rows are held in L2 between a statistics pass and the output pass (still
// 8 B/elem of HBM while the resident CTAs' parts fit in L2).
#include <cuda_runtime.h>
#include <cooperative_groups.h>
#include <cstdint>
#include <cfloat>
#include <cstdlib>
#include "mcu_math.cuh"
#include "mcu_kernels.h"

namespace cg = cooperative_groups;
using namespace mcu;

namespace {

constexpr int kThreads = 256;
constexpr int kMaxPartials = 1024;

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

struct WSum { __device__ __forceinline__ double operator()(double v) const { return warp_sum(v); } };
struct WMin { __device__ __forceinline__ float operator()(float v) const { return warp_min(v); } };
struct WMax { __device__ __forceinline__ float operator()(float v) const { return warp_max(v); } };

// Block-wide combine; every thread gets the result.
// `identity` fills the lanes beyond the number of warps.
template <typename T, typename F>
__device__ __forceinline__ T block_combine(T v, F warp_fn, T* sh, T identity) {
    v = warp_fn(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    int nw = blockDim.x >> 5;
    T t = l < nw ? sh[l] : identity;
    t = warp_fn(t);
    return t;
}

struct Acc {
    double sum;
    float mn, mx;
};

__device__ __forceinline__ void acc_add(Acc& a, float v) {
    a.sum += (double)v;
    a.mn = fminf(a.mn, v);
    a.mx = fmaxf(a.mx, v);
}

// Pass 1: each block folds a grid-stride share of the elements.
// Canonical layout: elements are linear.  Otherwise rows of x_d0 elements
// start at sum_k i_k*x_sk (k = 1..5).
__global__ void __launch_bounds__(kThreads) reduce_pass1(const float* __restrict__ x, uint64_t n, int canonical,
                                                         FastDiv d0, FastDiv d1, FastDiv d2, FastDiv d3, FastDiv d4,
                                                         int64_t s1, int64_t s2, int64_t s3, int64_t s4, int64_t s5,
                                                         double* __restrict__ psum, float* __restrict__ pmin,
                                                         float* __restrict__ pmax) {
    Acc a{0.0, INFINITY, -INFINITY};
    uint64_t stride = (uint64_t)gridDim.x * kThreads;
    uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
    if (canonical) {
        const float4* x4 = (const float4*)x;
        uint64_t n4 = ((uintptr_t)x & 15) == 0 ? n / 4 : 0;
        for (uint64_t j = i; j < n4; j += stride) {
            float4 v = __ldcs(x4 + j);
            acc_add(a, v.x); acc_add(a, v.y); acc_add(a, v.z); acc_add(a, v.w);
        }
        for (uint64_t j = n4 * 4 + i; j < n; j += stride) acc_add(a, x[j]);
    } else {
        for (uint64_t j = i; j < n; j += stride) {
            uint32_t q = (uint32_t)j;
            uint32_t row = fdiv(q, d0);
            uint32_t c = q - row * d0.d;
            int64_t off = c;
            uint32_t t;
            t = fdiv(row, d1); off += (int64_t)(row - t * d1.d) * s1; row = t;
            t = fdiv(row, d2); off += (int64_t)(row - t * d2.d) * s2; row = t;
            t = fdiv(row, d3); off += (int64_t)(row - t * d3.d) * s3; row = t;
            t = fdiv(row, d4); off += (int64_t)(row - t * d4.d) * s4; row = t;
            off += (int64_t)row * s5;
            acc_add(a, x[off]);
        }
    }
    __shared__ double shd[32];
    __shared__ float shf[32];
    double s = block_combine(a.sum, WSum(), shd, 0.0);
    float mn = block_combine(a.mn, WMin(), shf, (float)INFINITY);
    float mx = block_combine(a.mx, WMax(), shf, -(float)INFINITY);
    if (threadIdx.x == 0) {
        psum[blockIdx.x] = s;
        pmin[blockIdx.x] = mn;
        pmax[blockIdx.x] = mx;
    }
}

// Pass 2: one block folds the block partials.  With `part` set it writes the
// shard's record (double sum, min, max, element count) instead of a value.
__global__ void __launch_bounds__(kThreads) reduce_pass2(int op, int nparts, double numel,
                                                         const double* __restrict__ psum, const float* __restrict__ pmin,
                                                         const float* __restrict__ pmax, float* __restrict__ r,
                                                         McuReducePart* __restrict__ part) {
    Acc a{0.0, INFINITY, -INFINITY};
    for (int i = threadIdx.x; i < nparts; i += kThreads) {
        a.sum += psum[i];
        a.mn = fminf(a.mn, pmin[i]);
        a.mx = fmaxf(a.mx, pmax[i]);
    }
    __shared__ double shd[32];
    __shared__ float shf[32];
    double s = block_combine(a.sum, WSum(), shd, 0.0);
    float mn = block_combine(a.mn, WMin(), shf, (float)INFINITY);
    float mx = block_combine(a.mx, WMax(), shf, -(float)INFINITY);
    if (threadIdx.x == 0) {
        if (part) *part = McuReducePart{s, mn, mx, (uint64_t)numel};
        else if (op == OP_SUM) r[0] = (float)s;
        else if (op == OP_MEAN) r[0] = (float)(s / numel);
        else if (op == OP_MIN) r[0] = mn;
        else r[0] = mx;
    }
}

// Shard records -> r[0].  The double sums are added one after another in record
// (rank) order, as the reference adds its row sums (mag_blas_sum_f32,
// magnetron/magnetron_cpu.c:1034-1060); MEAN divides by the total element count.
__global__ void reduce_combine(int op, const McuReducePart* __restrict__ parts, int nparts, float* __restrict__ r) {
    if (threadIdx.x != 0) return;
    double s = 0.0;
    float mn = INFINITY, mx = -INFINITY;
    uint64_t n = 0;
    for (int i = 0; i < nparts; ++i) {
        const McuReducePart p = parts[i];
        s += p.sum;
        mn = fminf(mn, p.min);
        mx = fmaxf(mx, p.max);
        n += p.count;
    }
    if (op == OP_SUM) r[0] = (float)s;
    else if (op == OP_MEAN) r[0] = (float)(s / (double)n);
    else if (op == OP_MIN) r[0] = mn;
    else r[0] = mx;
}

// -------------------------------------------------------- row reductions ---

// WIDE: unroll the vector loop by four (loads in flight per thread) for rows of at least
// 65536 columns (262144-wide SUM 6.0 -> 7.0 TB/s); narrower rows keep the compiler's choice,
// which measured faster there.  The additions keep their order either way.
template <int OP, bool WIDE = false>
__device__ __forceinline__ void row_fold(const float* __restrict__ p, uint32_t cols, int tid, int nthr, double& s,
                                         float& m) {
    bool vec = (cols % 4 == 0) && (((uintptr_t)p & 15) == 0);
    if (vec && WIDE) {
        const float4* p4 = (const float4*)p;
#pragma unroll 4
        for (uint32_t c = tid; c < cols / 4; c += nthr) {
            float4 v = __ldcs(p4 + c);
            if constexpr (OP == OP_SUM || OP == OP_MEAN) s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
            else if constexpr (OP == OP_MIN) m = fminf(fminf(m, v.x), fminf(fminf(v.y, v.z), v.w));
            else m = fmaxf(fmaxf(m, v.x), fmaxf(fmaxf(v.y, v.z), v.w));
        }
    } else if (vec) {
        const float4* p4 = (const float4*)p;
        for (uint32_t c = tid; c < cols / 4; c += nthr) {
            float4 v = __ldcs(p4 + c);
            if constexpr (OP == OP_SUM || OP == OP_MEAN) s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
            else if constexpr (OP == OP_MIN) m = fminf(fminf(m, v.x), fminf(fminf(v.y, v.z), v.w));
            else m = fmaxf(fmaxf(m, v.x), fmaxf(fmaxf(v.y, v.z), v.w));
        }
    } else {
        for (uint32_t c = tid; c < cols; c += nthr) {
            float v = p[c];
            if constexpr (OP == OP_SUM || OP == OP_MEAN) s += (double)v;
            else if constexpr (OP == OP_MIN) m = fminf(m, v);
            else m = fmaxf(m, v);
        }
    }
}

template <int OP>
__device__ __forceinline__ float row_result(double s, float m, uint32_t cols) {
    if constexpr (OP == OP_SUM) return (float)s;
    else if constexpr (OP == OP_MEAN) return (float)(s / (double)cols);
    else return m;
}

// One warp per row (short rows).
template <int OP>
__global__ void __launch_bounds__(kThreads) reduce_rows_warp(float* __restrict__ r, const float* __restrict__ x,
                                                             uint64_t rows, uint32_t cols) {
    uint64_t w = ((uint64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    uint64_t nw = ((uint64_t)gridDim.x * kThreads) >> 5;
    int l = threadIdx.x & 31;
    for (; w < rows; w += nw) {
        double s = 0.0;
        float m = OP == OP_MIN ? INFINITY : -INFINITY;
        row_fold<OP>(x + w * cols, cols, l, 32, s, m);
        s = warp_sum(s);
        m = OP == OP_MIN ? warp_min(m) : warp_max(m);
        if (l == 0) r[w] = row_result<OP>(s, m, cols);
    }
}

// One block per row (long rows).
template <int OP, bool WIDE>
__global__ void __launch_bounds__(kThreads) reduce_rows_block(float* __restrict__ r, const float* __restrict__ x,
                                                              uint64_t rows, uint32_t cols) {
    __shared__ double shd[32];
    __shared__ float shf[32];
    for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        double s = 0.0;
        float m = OP == OP_MIN ? INFINITY : -INFINITY;
        row_fold<OP, WIDE>(x + row * cols, cols, threadIdx.x, kThreads, s, m);
        s = block_combine(s, WSum(), shd, 0.0);
        m = OP == OP_MIN ? block_combine(m, WMin(), shf, (float)INFINITY) : block_combine(m, WMax(), shf, -(float)INFINITY);
        if (threadIdx.x == 0) r[row] = row_result<OP>(s, m, cols);
    }
}

template <int OP>
cudaError_t launch_rows_op(float* r, const float* x, int64_t rows, int64_t cols, cudaStream_t st) {
    unsigned cap = (unsigned)sm_count() * 8;
    if (cols < 2048) {
        uint64_t g = ((uint64_t)rows * 32 + kThreads - 1) / kThreads;
        reduce_rows_warp<OP><<<(unsigned)(g < cap ? g : cap), kThreads, 0, st>>>(r, x, (uint64_t)rows, (uint32_t)cols);
    } else {
        uint64_t g = (uint64_t)rows;
        const unsigned grid = (unsigned)(g < cap ? g : cap);
        if (cols >= 65536) reduce_rows_block<OP, true><<<grid, kThreads, 0, st>>>(r, x, (uint64_t)rows, (uint32_t)cols);
        else reduce_rows_block<OP, false><<<grid, kThreads, 0, st>>>(r, x, (uint64_t)rows, (uint32_t)cols);
    }
    return cudaGetLastError();
}

// ----------------------------------------------------------- row softmax ---
//
// Short rows (<= 2048) get one warp each and rows up to 65536 a thread-block
// cluster of 8192-element slices (one 256-thread CTA each) combining the row max
// and sum through distributed shared memory; both keep the row in registers
// between the phases (max, exp + double sum, scale), so HBM sees one read and
// one write per element.  Wider rows go to softmax_rows_l2, which keeps each
// CTA's part of the row in L2 between its statistics pass and its output pass;
// two passes over per-slice statistics (scratch) remain for a cluster shape that
// cannot be scheduled, and a three-pass kernel behind the register clusters.

constexpr int kWarpRowMax = 2048;  // rows up to this length get one warp (16 float4 per lane at most)
constexpr int kSliceVec = 8;      // float4 per thread: slices of 32 x threads elements

// The normalised row softmax (an extension: the reference has only the elementwise exp op,
// whose lanes k_elementwise.cu reproduces bit for bit) takes exp from CUDA's expf, within 2 ulp
// of exp, for every element; its results stay within 1e-6 relative of the reference-exp oracle.
// The reference's lane formula costs about 20 unfused f32 operations per element, which bounded
// these kernels below the memory roofline (32768-wide rows: 4.0 vs 4.8 TB/s).
__device__ __forceinline__ float softmax_exp(float t, uint32_t, uint32_t) { return expf(t); }

__device__ __forceinline__ float4 neg_inf4() { return make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY); }
__device__ __forceinline__ float max4(float4 v) { return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)); }

// e = exp(v - m) per component (reference lane/tail split by column), zero past the row end.
// The row sum is kept in double; the four values (each in [0, 1]) are first added pairwise in
// f32, which adds at most 2^-23 relative to the sum (about 1e-7) and saves three of every four
// f32->f64 conversions and double adds, which otherwise bound the kernel's throughput.
__device__ __forceinline__ double sum4(float4 e) {
    return (double)__fadd_rn(__fadd_rn(e.x, e.y), __fadd_rn(e.z, e.w));
}
__device__ __forceinline__ float4 exp4(float4 v, float m, uint32_t c, uint32_t cols, uint32_t vec_end, double& s) {
    float4 e;
    if (c + 3 < vec_end) {  // all four are vector lanes
        e.x = expf(fs(v.x, m));
        e.y = expf(fs(v.y, m));
        e.z = expf(fs(v.z, m));
        e.w = expf(fs(v.w, m));
        s += sum4(e);
        return e;
    }
    e.x = c < cols ? softmax_exp(fs(v.x, m), c, vec_end) : 0.0f;
    e.y = c + 1 < cols ? softmax_exp(fs(v.y, m), c + 1, vec_end) : 0.0f;
    e.z = c + 2 < cols ? softmax_exp(fs(v.z, m), c + 2, vec_end) : 0.0f;
    e.w = c + 3 < cols ? softmax_exp(fs(v.w, m), c + 3, vec_end) : 0.0f;
    s += sum4(e);
    return e;
}

// e / sum as e * rn(1/sum): within 1.5 ulp of the division, one reciprocal per row.
__device__ __forceinline__ float4 div4(float4 e, float inv) {
    return make_float4(__fmul_rn(e.x, inv), __fmul_rn(e.y, inv), __fmul_rn(e.z, inv), __fmul_rn(e.w, inv));
}

// Loads 4 consecutive elements starting at column c (c % 4 == 0 on the vector path).
__device__ __forceinline__ float4 load4(const float* px, uint32_t c, uint32_t cols, bool vec) {
    if (vec) return c < cols ? __ldcs((const float4*)(px + c)) : neg_inf4();
    float4 t;
    t.x = c < cols ? px[c] : -INFINITY;
    t.y = c + 1 < cols ? px[c + 1] : -INFINITY;
    t.z = c + 2 < cols ? px[c + 2] : -INFINITY;
    t.w = c + 3 < cols ? px[c + 3] : -INFINITY;
    return t;
}

__device__ __forceinline__ void store4(float* pr, uint32_t c, uint32_t cols, bool vec, float4 v) {
    if (vec) {
        if (c < cols) __stcs((float4*)(pr + c), v);
        return;
    }
    if (c < cols) pr[c] = v.x;
    if (c + 1 < cols) pr[c + 1] = v.y;
    if (c + 2 < cols) pr[c + 2] = v.z;
    if (c + 3 < cols) pr[c + 3] = v.w;
}

// One warp per row; lane holds columns 4*(lane + 32*i) .. +3.
template <int V>
__global__ void __launch_bounds__(256, V <= 4 ? 4 : (V <= 8 ? 3 : 1)) softmax_rows_warp(float* __restrict__ r, const float* __restrict__ x,
                                                         uint64_t rows, uint32_t cols) {
    const int lane = threadIdx.x & 31;
    const uint64_t nw = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    const uint32_t vec_end = cols & ~3u;
    for (uint64_t row = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += nw) {
        const float* px = x + row * cols;
        float* pr = r + row * cols;
        const bool vec = (cols % 4 == 0) && ((((uintptr_t)px) | ((uintptr_t)pr)) & 15) == 0;
        float4 v[V];
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = load4(px, (uint32_t)(lane + 32 * i) * 4, cols, vec);
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < V; ++i) m = fmaxf(m, max4(v[i]));
        m = warp_max(m);
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = exp4(v[i], m, (uint32_t)(lane + 32 * i) * 4, cols, vec_end, s);
        const float inv = __frcp_rn((float)warp_sum(s));
#pragma unroll
        for (int i = 0; i < V; ++i) store4(pr, (uint32_t)(lane + 32 * i) * 4, cols, vec, div4(v[i], inv));
    }
}

// One CTA per slice of 32*T*kSliceVec elements; the cluster spans the row.  Each CTA computes
// its slice's max m and sum s = sum exp(x - m) (double), pushes (m, s) into slot `rank` of every
// CTA of the cluster through distributed shared memory, and after ONE cluster barrier each CTA
// combines the slots in rank order (M = max m_q, S = sum_q s_q exp(m_q - M) in double) and
// writes its slice as exp(x - m) * (exp(m - M) / S).  After that barrier no CTA touches another's
// shared memory, so none waits for its peers before leaving.  (The barrier's relaxed arrive at
// the start orders nothing; its wait before the pushes makes sure every CTA of the cluster runs.)
template <int kSliceThreads>
__global__ void __launch_bounds__(kSliceThreads, 1024 / kSliceThreads) softmax_rows_slices(
    float* __restrict__ r, const float* __restrict__ x, uint32_t cols) {
    constexpr int kSlice = kSliceThreads * 4 * kSliceVec;
    __shared__ float sh_max[32];
    __shared__ double sh_sum[32];
    __shared__ float peer_m[16];
    __shared__ double peer_s[16];
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t crank = cluster.block_rank();
    const uint32_t csize = cluster.num_blocks();
    const uint64_t row = blockIdx.x / csize;
    const uint32_t c0 = crank * (uint32_t)kSlice;
    const float* px = x + row * cols;
    float* pr = r + row * cols;
    const uint32_t vec_end = cols & ~3u;
    const bool vec = (cols % 4 == 0) && ((((uintptr_t)px) | ((uintptr_t)pr)) & 15) == 0;
    float4 v[kSliceVec];
#pragma unroll
    for (int i = 0; i < kSliceVec; ++i) v[i] = load4(px, c0 + (uint32_t)(threadIdx.x + kSliceThreads * i) * 4, cols, vec);
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kSliceVec; ++i) m = fmaxf(m, max4(v[i]));
    m = block_combine(m, WMax(), sh_max, -(float)INFINITY);
    double s = 0.0;
    const float mm = m != -INFINITY ? m : 0.0f;  // a slice of -inf only (or past the row's end): exp(-inf) = 0
#pragma unroll
    for (int i = 0; i < kSliceVec; ++i)
        v[i] = exp4(v[i], mm, c0 + (uint32_t)(threadIdx.x + kSliceThreads * i) * 4, cols, vec_end, s);
    s = block_combine(s, WSum(), sh_sum, 0.0);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (threadIdx.x < csize) {
        *cluster.map_shared_rank(&peer_m[crank], threadIdx.x) = m;
        *cluster.map_shared_rank(&peer_s[crank], threadIdx.x) = s;
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    __shared__ float sh_f;
    if (threadIdx.x == 0) {
        float gm = -INFINITY;
        for (uint32_t k = 0; k < csize; ++k) gm = fmaxf(gm, peer_m[k]);
        double gs = 0.0;
        for (uint32_t k = 0; k < csize; ++k)
            if (peer_m[k] != -INFINITY) gs += peer_s[k] * (double)expf(peer_m[k] - gm);
        // a row of -inf only has no maximum to subtract: NaN, as exp(x - max) gives there
        sh_f = gm == -INFINITY ? __int_as_float(0x7FC00000)
                               : (m != -INFINITY ? (float)((double)expf(m - gm) / gs) : 0.0f);
    }
    __syncthreads();
    const float f = sh_f;
#pragma unroll
    for (int i = 0; i < kSliceVec; ++i) {
        const float4 e = v[i];
        store4(pr, c0 + (uint32_t)(threadIdx.x + kSliceThreads * i) * 4, cols, vec,
               make_float4(__fmul_rn(e.x, f), __fmul_rn(e.y, f), __fmul_rn(e.z, f), __fmul_rn(e.w, f)));
    }
}

// Rows wider than one CTA slice: two passes over x instead of a cluster that holds the whole
// row.  Pass 1 records each slice's max m_s and the double sum of exp(x - m_s); pass 2
// combines a row's slices in slice order (row max M, sum S = sum_s S_s * exp(m_s - M) in
// f64), then writes exp(x - M) / S with the reference's lane/tail exponential.  S differs
// from the one-pass sum only by the rounding of the rescaled terms (about 1e-7 relative).
// The row combine runs once per row in its own small kernel between the passes (HBM sees
// 12 B per element; running the passes over L2-sized chunks of rows measured slower).
struct SliceStat {
    float m;
    float pad;
    double s;
};
constexpr int kStatThreads = 256;
constexpr int kStatSlice = kStatThreads * 4 * kSliceVec;  // 8192 elements

__global__ void __launch_bounds__(kStatThreads) softmax_slice_stats(SliceStat* __restrict__ st,
                                                                    const float* __restrict__ x, uint32_t cols,
                                                                    uint32_t nslices) {
    __shared__ float sh_max[32];
    __shared__ double sh_sum[32];
    const uint64_t row = blockIdx.x / nslices;
    const uint32_t c0 = (blockIdx.x % nslices) * (uint32_t)kStatSlice;
    const float* px = x + row * cols;
    const uint32_t vec_end = cols & ~3u;
    const bool vec = (cols % 4 == 0) && ((((uintptr_t)px) & 15) == 0);
    float4 v[kSliceVec];
#pragma unroll
    for (int i = 0; i < kSliceVec; ++i)
        v[i] = load4(px, c0 + (uint32_t)(threadIdx.x + kStatThreads * i) * 4, cols, vec);
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kSliceVec; ++i) m = fmaxf(m, max4(v[i]));
    m = block_combine(m, WMax(), sh_max, -(float)INFINITY);
    double s = 0.0;
    if (m != -INFINITY) {
#pragma unroll
        for (int i = 0; i < kSliceVec; ++i)
            (void)exp4(v[i], m, c0 + (uint32_t)(threadIdx.x + kStatThreads * i) * 4, cols, vec_end, s);
    }
    s = block_combine(s, WSum(), sh_sum, 0.0);
    if (threadIdx.x == 0) st[blockIdx.x] = SliceStat{m, 0.0f, s};
}

// One thread per row: the row's max and the reciprocal of its sum from the slice statistics,
// in slice order, into the row's first SliceStat (m, and inv in `pad`).
__global__ void __launch_bounds__(256) softmax_slice_combine(SliceStat* __restrict__ st, uint64_t rows,
                                                              uint32_t nslices) {
    const uint64_t row = (uint64_t)blockIdx.x * 256 + threadIdx.x;
    if (row >= rows) return;
    SliceStat* p = st + row * nslices;
    float gm = -INFINITY;
    for (uint32_t k = 0; k < nslices; ++k) gm = fmaxf(gm, p[k].m);
    double gs = 0.0;
    for (uint32_t k = 0; k < nslices; ++k)
        if (p[k].m != -INFINITY) gs += p[k].s * exp((double)p[k].m - (double)gm);
    p[0].m = gm;
    p[0].pad = __frcp_rn((float)gs);
}

__global__ void __launch_bounds__(kStatThreads) softmax_slice_apply(float* __restrict__ r, const float* __restrict__ x,
                                                                    const SliceStat* __restrict__ st, uint32_t cols,
                                                                    uint32_t nslices) {
    const uint64_t row = blockIdx.x / nslices;
    const uint32_t c0 = (blockIdx.x % nslices) * (uint32_t)kStatSlice;
    const float gm = st[row * nslices].m, inv = st[row * nslices].pad;
    const float* px = x + row * cols;
    float* pr = r + row * cols;
    const uint32_t vec_end = cols & ~3u;
    const bool vec = (cols % 4 == 0) && ((((uintptr_t)px) | ((uintptr_t)pr)) & 15) == 0;
    double unused = 0.0;
#pragma unroll
    for (int i = 0; i < kSliceVec; ++i) {
        const uint32_t c = c0 + (uint32_t)(threadIdx.x + kStatThreads * i) * 4;
        const float4 e = exp4(load4(px, c, cols, vec), gm, c, cols, vec_end, unused);
        store4(pr, c, cols, vec, div4(e, inv));
    }
}

// Rows wider than 65536: a cluster of up to 8 CTAs per row, CTA q owning the columns
// [q * part, (q + 1) * part).  Pass 1 reads the part from HBM with the default caching (it stays
// in L2) and keeps a running max m and double sum s of exp(x - m) per thread, rescaling s by
// exp(m_old - m_new) in double when the max grows; the block and then the cluster combine
// (max, then the rescaled double sums, the cluster's in rank order through distributed shared
// memory).  Pass 2 re-reads the part, an L2 hit while the parts of the resident CTAs fit in L2,
// and writes exp(x - M) * rn(1/S) as the two-kernel path does.  HBM sees 8 B per element against
// that path's 12, with no scratch and no wait on other clusters.
// 512 threads, parts of at least 32768 columns and clusters of at most 8 measured fastest at
// 262144 columns (0.464 ms per 2^28; 256 threads 0.499, 1024 threads 0.875, parts of 16384 in
// clusters of 16: 0.488 with 256 threads, 0.566 with 512).
constexpr int kL2Threads = 512;
constexpr int kL2Unroll = 4;          // float4 loads in flight per thread in pass 1
constexpr int64_t kL2Part = 32768;    // columns per CTA at least
constexpr int kL2MaxCluster = 8;      // portable cluster size

__device__ __forceinline__ void online_add4(float4 v, float& m, double& s, uint32_t c, uint32_t cols,
                                            uint32_t vec_end) {
    const float mx = max4(v);
    if (mx > m) {
        if (m != -INFINITY) s *= exp((double)m - (double)mx);
        m = mx;
    }
    if (m != -INFINITY) (void)exp4(v, m, c, cols, vec_end, s);
}

__global__ void __launch_bounds__(kL2Threads) softmax_rows_l2(float* __restrict__ r, const float* __restrict__ x,
                                                              uint32_t cols, uint32_t part) {
    __shared__ float sh_max[32];
    __shared__ double sh_sum[32];
    __shared__ float peer_m[kL2MaxCluster];
    __shared__ double peer_s[kL2MaxCluster];
    __shared__ float sh_gm, sh_inv;
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t crank = cluster.block_rank();
    const uint32_t csize = cluster.num_blocks();
    const uint64_t row = blockIdx.x / csize;
    const uint32_t cb = crank * part;
    const uint32_t ce = cb + part < cols ? cb + part : cols;
    const float* px = x + row * cols;
    float* pr = r + row * cols;
    const uint32_t vec_end = cols & ~3u;
    const bool vec = (cols % 4 == 0) && ((((uintptr_t)px) | ((uintptr_t)pr)) & 15) == 0;
    float m = -INFINITY;
    double s = 0.0;
    if (vec) {
        constexpr uint32_t kStep = 4u * kL2Threads;
        for (uint32_t c = cb + 4u * threadIdx.x; c < ce; c += kStep * kL2Unroll) {
            float4 v[kL2Unroll];
#pragma unroll
            for (int u = 0; u < kL2Unroll; ++u)
                v[u] = c + kStep * u < ce ? *(const float4*)(px + c + kStep * u) : neg_inf4();
#pragma unroll
            for (int u = 0; u < kL2Unroll; ++u) online_add4(v[u], m, s, c + kStep * u, cols, vec_end);
        }
    } else {
        for (uint32_t c = cb + threadIdx.x; c < ce; c += kL2Threads) {
            const float v = px[c];
            if (v > m) {
                if (m != -INFINITY) s *= exp((double)m - (double)v);
                m = v;
            }
            if (m != -INFINITY) s += (double)expf(fs(v, m));
        }
    }
    const float bm = block_combine(m, WMax(), sh_max, -(float)INFINITY);
    s = block_combine(m != -INFINITY ? s * exp((double)m - (double)bm) : 0.0, WSum(), sh_sum, 0.0);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (threadIdx.x < csize) {
        *cluster.map_shared_rank(&peer_m[crank], threadIdx.x) = bm;
        *cluster.map_shared_rank(&peer_s[crank], threadIdx.x) = s;
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (threadIdx.x == 0) {
        float gm = -INFINITY;
        for (uint32_t k = 0; k < csize; ++k) gm = fmaxf(gm, peer_m[k]);
        double gs = 0.0;
        for (uint32_t k = 0; k < csize; ++k)
            if (peer_m[k] != -INFINITY) gs += peer_s[k] * exp((double)peer_m[k] - (double)gm);
        sh_gm = gm;
        sh_inv = __frcp_rn((float)gs);
    }
    __syncthreads();
    const float gm = sh_gm, inv = sh_inv;
    double unused = 0.0;
    if (vec) {
        for (uint32_t c = cb + 4u * threadIdx.x; c < ce; c += 4u * kL2Threads)
            __stcs((float4*)(pr + c), div4(exp4(__ldcs((const float4*)(px + c)), gm, c, cols, vec_end, unused), inv));
    } else {
        for (uint32_t c = cb + threadIdx.x; c < ce; c += kL2Threads) pr[c] = __fmul_rn(expf(fs(px[c], gm)), inv);
    }
}

// Rows longer than 16 slices: three passes from HBM.
constexpr int kSoftmaxThreads = 512;
__global__ void __launch_bounds__(kSoftmaxThreads) softmax_rows_global(float* __restrict__ r,
                                                                       const float* __restrict__ x, uint64_t rows,
                                                                       uint32_t cols) {
    __shared__ float sh_max[32];
    __shared__ double sh_sum[32];
    const uint32_t vec_end = cols & ~3u;
    for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float* px = x + row * cols;
        float* pr = r + row * cols;
        float m = -INFINITY;
        for (uint32_t c = threadIdx.x; c < cols; c += kSoftmaxThreads) m = fmaxf(m, px[c]);
        m = block_combine(m, WMax(), sh_max, -(float)INFINITY);
        double s = 0.0;
        for (uint32_t c = threadIdx.x; c < cols; c += kSoftmaxThreads) s += (double)softmax_exp(fs(px[c], m), c, vec_end);
        s = block_combine(s, WSum(), sh_sum, 0.0);
        const float fsum = (float)s;
        for (uint32_t c = threadIdx.x; c < cols; c += kSoftmaxThreads)
            pr[c] = __fdiv_rn(softmax_exp(fs(px[c], m), c, vec_end), fsum);
        __syncthreads();
    }
}

}  // namespace

extern "C" size_t mcu_reduce_scratch_bytes(void) {
    return (size_t)kMaxPartials * (sizeof(double) + 2 * sizeof(float));
}

static int launch_reduce(int op, float* r, McuReducePart* part, const float* x, const int64_t* xd,
                         const int64_t* xs, void* scratch, cudaStream_t st) {
    uint64_t n = 1;
    for (int k = 0; k < 6; ++k) {
        if (xd[k] <= 0) return (int)cudaErrorInvalidValue;
        n *= (uint64_t)xd[k];
    }
    int canonical = 1;
    int64_t acc = 1;
    for (int k = 0; k < 6; ++k) {
        if (xd[k] != 1 && xs[k] != acc) canonical = 0;
        acc *= xd[k];
    }
    if (!canonical && n >= (1ull << 32)) return (int)cudaErrorInvalidValue;
    uint64_t want = (n + (uint64_t)kThreads * 16 - 1) / ((uint64_t)kThreads * 16);
    int nparts = (int)(want < (uint64_t)sm_count() * 4 ? want : (uint64_t)sm_count() * 4);
    if (nparts > kMaxPartials) nparts = kMaxPartials;
    if (nparts < 1) nparts = 1;
    double* psum = (double*)scratch;
    float* pmin = (float*)(psum + kMaxPartials);
    float* pmax = pmin + kMaxPartials;
    FastDiv d[5];
    for (int k = 0; k < 5; ++k) d[k] = make_fastdiv((uint32_t)(xd[k] < (1ll << 32) ? xd[k] : 1));
    reduce_pass1<<<nparts, kThreads, 0, st>>>(x, n, canonical, d[0], d[1], d[2], d[3], d[4], xs[1], xs[2], xs[3],
                                              xs[4], xs[5], psum, pmin, pmax);
    reduce_pass2<<<1, kThreads, 0, st>>>(op, nparts, (double)n, psum, pmin, pmax, r, part);
    return (int)cudaGetLastError();
}

extern "C" int mcu_launch_reduce(int op, float* r, const float* x, const int64_t* xd, const int64_t* xs,
                                 void* scratch, cudaStream_t st) {
    return launch_reduce(op, r, nullptr, x, xd, xs, scratch, st);
}

extern "C" int mcu_launch_reduce_partial(McuReducePart* part, const float* x, const int64_t* xd, const int64_t* xs,
                                         void* scratch, cudaStream_t st) {
    return launch_reduce(OP_SUM, nullptr, part, x, xd, xs, scratch, st);
}

extern "C" int mcu_launch_reduce_combine(int op, float* r, const McuReducePart* parts, int nparts, cudaStream_t st) {
    if (nparts < 1) return (int)cudaErrorInvalidValue;
    reduce_combine<<<1, 32, 0, st>>>(op, parts, nparts, r);
    return (int)cudaGetLastError();
}

extern "C" int mcu_launch_reduce_rows(int op, float* r, const float* x, int64_t rows, int64_t cols,
                                      cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return (int)cudaSuccess;
    if (cols >= (1ll << 32)) return (int)cudaErrorInvalidValue;
    switch (op) {
        case OP_SUM: return (int)launch_rows_op<OP_SUM>(r, x, rows, cols, st);
        case OP_MEAN: return (int)launch_rows_op<OP_MEAN>(r, x, rows, cols, st);
        case OP_MIN: return (int)launch_rows_op<OP_MIN>(r, x, rows, cols, st);
        case OP_MAX: return (int)launch_rows_op<OP_MAX>(r, x, rows, cols, st);
        default: return (int)cudaErrorInvalidValue;
    }
}

// Rows wider than this go to softmax_rows_l2 (131072-wide rows: 0.445 ms per 2^28 against 0.506
// for the two-pass slice kernels and 0.61 for register-resident clusters of 16 slices); the
// two-pass slice kernels (scratch: one SliceStat per slice) remain for a cluster shape that cannot
// be scheduled.
constexpr int64_t kClusterRowMax = 8 * 8192;

// MAG_CUDA_SOFTMAX_L2=0 sends rows wider than 65536 to the two-kernel path.
static bool l2_rows_on() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("MAG_CUDA_SOFTMAX_L2");
        on = !(e && e[0] == '0');
    }
    return on != 0;
}

extern "C" size_t mcu_softmax_rows_scratch_bytes(int64_t rows, int64_t cols) {
    if (cols <= kClusterRowMax) return 0;
    return (size_t)rows * (size_t)((cols + kStatSlice - 1) / kStatSlice) * sizeof(SliceStat);
}

extern "C" int mcu_softmax_rows_kernels(int64_t rows, int64_t cols) {
    if (rows <= 0 || cols <= 0) return 0;
    return cols <= kClusterRowMax || l2_rows_on() ? 1 : 3;
}

extern "C" int mcu_launch_softmax_rows(float* r, const float* x, int64_t rows, int64_t cols, void* scratch,
                                       cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return (int)cudaSuccess;
    if (cols >= (1ll << 31) || rows >= (1ll << 31)) return (int)cudaErrorInvalidValue;
    if (cols > kClusterRowMax && l2_rows_on()) {
        // clusters of up to kL2MaxCluster CTAs, parts of at least kL2Part columns (a multiple of 4)
        int64_t cl = (cols + kL2Part - 1) / kL2Part;
        if (cl > kL2MaxCluster) cl = kL2MaxCluster;
        const int64_t part = ((cols + cl - 1) / cl + 3) & ~(int64_t)3;
        cl = (cols + part - 1) / part;
        if (rows * cl < (1ll << 31)) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)(rows * cl));
            cfg.blockDim = dim3(kL2Threads);
            cfg.dynamicSmemBytes = 0;
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)cl;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaError_t e = cudaLaunchKernelEx(&cfg, softmax_rows_l2, r, x, (uint32_t)cols, (uint32_t)part);
            if (e == cudaSuccess) return (int)cudaSuccess;
            cudaGetLastError();  // cluster shape not schedulable here: the two-kernel path below
        }
    }
    if (cols > kClusterRowMax) {
        const int64_t ns = (cols + kStatSlice - 1) / kStatSlice;
        if (!scratch || rows * ns >= (1ll << 31)) return (int)cudaErrorInvalidValue;
        SliceStat* stats = (SliceStat*)scratch;
        const unsigned blocks = (unsigned)(rows * ns);
        softmax_slice_stats<<<blocks, kStatThreads, 0, st>>>(stats, x, (uint32_t)cols, (uint32_t)ns);
        softmax_slice_combine<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(stats, (uint64_t)rows, (uint32_t)ns);
        softmax_slice_apply<<<blocks, kStatThreads, 0, st>>>(r, x, stats, (uint32_t)cols, (uint32_t)ns);
        return (int)cudaGetLastError();
    }
    if (cols <= kWarpRowMax) {
        uint64_t g = ((uint64_t)rows * 32 + 255) / 256;
        const uint64_t cap = (uint64_t)sm_count() * 16;
        const unsigned grid = (unsigned)(g < cap ? g : cap);
        if (cols <= 512) softmax_rows_warp<4><<<grid, 256, 0, st>>>(r, x, (uint64_t)rows, (uint32_t)cols);
        else if (cols <= 1024) softmax_rows_warp<8><<<grid, 256, 0, st>>>(r, x, (uint64_t)rows, (uint32_t)cols);
        else softmax_rows_warp<16><<<grid, 256, 0, st>>>(r, x, (uint64_t)rows, (uint32_t)cols);
        return (int)cudaGetLastError();
    }
    // slices of 8192 elements (256 threads) when the row fits 16 of them, else 16384 (512 threads)
    const bool small = cols <= 16 * 8192;
    const int64_t slice = small ? 8192 : 16384;
    const int64_t csize = (cols + slice - 1) / slice;
    auto kern = small ? softmax_rows_slices<256> : softmax_rows_slices<512>;
    if (csize <= 16 && rows * csize < (1ll << 31)) {
        if (csize > 8) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return (int)e;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(rows * csize));
        cfg.blockDim = dim3(small ? 256 : 512);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)csize;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, kern, r, x, (uint32_t)cols);
        if (e == cudaSuccess) return (int)cudaSuccess;
        cudaGetLastError();  // cluster shape not schedulable here: use the three-pass kernel
    }
    int g = sm_count() * 4;
    softmax_rows_global<<<(unsigned)(rows < g ? rows : g), kSoftmaxThreads, 0, st>>>(r, x, (uint64_t)rows,
                                                                                   (uint32_t)cols);
    return (int)cudaGetLastError();
}
