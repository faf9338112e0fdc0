// k_matmul_exact.cu - CUDA-core f32 matmul kernels.
//
// mag_blas_matmul_f32 (magnetron/magnetron_cpu.c:2151-2185) reads X as a
// row-major M x K buffer and Y as K x N and accumulates, for each output,
//   r = 0;  for k = 0..K-1:  r = r + X[i][k]*Y[k][j]
// with the product and the sum rounded separately (the x86 build has no FMA).
//
// matmul_exact keeps exactly that order and rounding per output: a register
// tiled kernel whose k loop runs in ascending order with __fmul_rn/__fadd_rn,
// so its results are bit-identical to the reference.  Tile sizes are picked so
// that the grid covers the GPU for small problems (the 2-layer MLP's
// 256x784x256 product runs on 64 CTAs with 32x32 tiles).
//
// matmul_skinny serves M <= 64 (matrix-vector-like products, HBM-bound on
// Y): K is split across CTAs so that all SMs stream Y, partial sums go to a
// scratch buffer and a second kernel adds the K slices in a fixed order.  It
// uses FMA and a different summation order, so it is accurate to f32
// rounding (well inside 1e-5 relative) but not bit-identical.
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include "mcu_kernels.h"
#include "mcu_math.cuh"

namespace {

constexpr int kThreads = 256;

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

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// BM x BN output tile per CTA, TM x TN per thread, BK-deep chunks of K in an S-stage ring filled
// by cp.async: chunk c + S - 1 is in flight while chunk c is consumed, so small tiles (whose
// per-chunk arithmetic is short) no longer wait a full memory latency per chunk.  Each thread
// still adds its products in k order, separately rounded, over the valid k only.
template <int BM, int BN, int TM, int TN, int BK, int S, int THREADS = (BM / TM) * (BN / TN)>
__global__ void __launch_bounds__(THREADS) matmul_exact(float* __restrict__ r, const float* __restrict__ x,
                                                         const float* __restrict__ y, int64_t M, int64_t K,
                                                         int64_t N, int64_t r_ld, int accumulate,
                                                         const float* __restrict__ bias, int64_t bias_mod, int act) {
    static_assert((BM / TM) * (BN / TN) == THREADS, "thread tiling");
    static_assert(S >= 2, "a ring of at least two stages");
    __shared__ float As[S][BK][BM + 1];
    __shared__ float Bs[S][BK][BN];
    const int64_t b = blockIdx.z;
    x += b * M * K;
    y += b * K * N;
    r += b * M * r_ld;
    const int64_t m0 = (int64_t)blockIdx.y * BM;
    const int64_t n0 = (int64_t)blockIdx.x * BN;
    const int tx = threadIdx.x % (BN / TN);
    const int ty = threadIdx.x / (BN / TN);
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            int64_t gi = m0 + ty * TM + i, gj = n0 + tx * TN + j;
            acc[i][j] = (accumulate && gi < M && gj < N) ? r[gi * r_ld + gj] : 0.0f;
        }
    const int64_t nk = (K + BK - 1) / BK;
    // each thread's elements of a chunk: fixed rows/columns and k offsets, so per chunk only the
    // k base moves (the address arithmetic had cost more instructions than the products)
    constexpr int NA = BM * BK / THREADS, NB = BN * BK / THREADS;
    static_assert(NA * THREADS == BM * BK && NB * THREADS == BN * BK, "whole chunks per thread");
    constexpr uint32_t kStageA = BK * (BM + 1) * 4, kStageB = BK * BN * 4;
    const float* xa[NA];
    const float* yb[NB];
    int kia[NA], kib[NB];
    uint32_t sa[NA], sb[NB];
#pragma unroll
    for (int j = 0; j < NA; ++j) {
        const int t = threadIdx.x + j * THREADS, mi = t / BK, ki = t % BK;
        const bool ok = m0 + mi < M;
        xa[j] = ok ? x + (m0 + mi) * K + ki : nullptr;
        kia[j] = ki;
        sa[j] = (uint32_t)__cvta_generic_to_shared(&As[0][ki][mi]);
    }
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        const int t = threadIdx.x + j * THREADS, ki = t / BN, ni = t % BN;
        const bool ok = n0 + ni < N;
        yb[j] = ok ? y + (int64_t)ki * N + n0 + ni : nullptr;
        kib[j] = ki;
        sb[j] = (uint32_t)__cvta_generic_to_shared(&Bs[0][ki][ni]);
    }
    auto issue = [&](int64_t c, int st) {  // chunk c into stage st
        const int64_t k0 = c * BK;
#pragma unroll
        for (int j = 0; j < NA; ++j) {
            const bool ok = xa[j] && k0 + kia[j] < K;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sa[j] + st * kStageA),
                         "l"(ok ? xa[j] + k0 : x), "r"(ok ? 4 : 0) : "memory");
        }
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const bool ok = yb[j] && k0 + kib[j] < K;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sb[j] + st * kStageB),
                         "l"(ok ? yb[j] + k0 * N : y), "r"(ok ? 4 : 0) : "memory");
        }
    };
#pragma unroll
    for (int c = 0; c < S - 1; ++c) {  // one commit group per chunk, empty past the last
        if (c < nk) issue(c, c);
        cp_async_commit();
    }
    int st_use = 0, st_fill = S - 1;
    for (int64_t c = 0; c < nk; ++c) {
        cp_async_wait<S - 2>();  // this thread's copies of chunk c have landed
        __syncthreads();         // everyone's have, and everyone is done with chunk c - 1's stage
        if (c + S - 1 < nk) issue(c + S - 1, st_fill);
        cp_async_commit();
        st_fill = st_fill == S - 1 ? 0 : st_fill + 1;
        const int st = st_use;
        st_use = st_use == S - 1 ? 0 : st_use + 1;
        const int64_t k0 = c * BK;
        auto step = [&](int kk) {
            float a[TM], bv[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = As[st][kk][ty * TM + i];
#pragma unroll
            for (int j = 0; j < TN; ++j) bv[j] = Bs[st][kk][tx * TN + j];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], bv[j]));
        };
        if (K - k0 >= BK) {  // a full chunk: a fixed trip count lets the shared loads run ahead
#pragma unroll 16
            for (int kk = 0; kk < BK; ++kk) step(kk);
        } else {
            const int kk_end = (int)(K - k0);
            for (int kk = 0; kk < kk_end; ++kk) step(kk);
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            int64_t gi = m0 + ty * TM + i, gj = n0 + tx * TN + j;
            if (gi < M && gj < N) {
                // a fused dense layer: the bias as the elementwise ADD indexes it (flat index,
                // or flat index mod the length of a bias broadcast along dim 0), then the
                // activation's vector-lane formula
                float v = acc[i][j];
                if (bias) {
                    const int64_t f = gi * N + gj;
                    v = __fadd_rn(v, bias[bias_mod ? f % bias_mod : f]);
                }
                if (act == 1) v = mcu::lane_op<mcu::OP_GELU>(v);
                else if (act == 2) v = mcu::lane_op<mcu::OP_SIGMOID>(v);
                r[gi * r_ld + gj] = v;
            }
        }
}

template <int BM, int BN, int TM, int TN, int BK, int S>
cudaError_t launch_exact(float* r, const float* x, const float* y, int64_t batch, int64_t M, int64_t K, int64_t N,
                         int64_t r_ld, int accumulate, cudaStream_t st, const float* bias = nullptr,
                         int64_t bias_mod = 0, int act = 0) {
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM), (unsigned)batch);
    matmul_exact<BM, BN, TM, TN, BK, S><<<grid, (BM / TM) * (BN / TN), 0, st>>>(r, x, y, M, K, N, r_ld, accumulate,
                                                                               bias, bias_mod, act);
    return cudaGetLastError();
}

// ------------------------------------------------------------- skinny ---

constexpr int kSkinnyRows = 16;           // rows per CTA (M up to 64 uses up to 4 row blocks)
constexpr int kSkinnyCols = kThreads * 4; // each thread owns 4 columns
constexpr int kSkinnyKc = 64;             // k rows per slice (multiple of 16)

// Partial product of X[m0:m0+MR, slice] and Y[slice, cols]; Y rows are
// fetched 16 (MR <= 4) or 8 at a time before any FMA, so every thread keeps
// that many 128-bit loads in flight.
template <int MR>
__global__ void __launch_bounds__(kThreads) matmul_skinny_part(float* __restrict__ part, const float* __restrict__ x,
                                                               const float* __restrict__ y, int M, int64_t K,
                                                               int64_t N, int64_t kc) {
    __shared__ float xs[MR][kSkinnyKc];
    // the slice sum may be scheduled now; it waits for this grid's completion before reading
    asm volatile("griddepcontrol.launch_dependents;");
    const int64_t c = (int64_t)blockIdx.x * kSkinnyCols + 4 * threadIdx.x;
    const int64_t k0 = (int64_t)blockIdx.y * kc;
    const int64_t k1 = (k0 + kc < K) ? k0 + kc : K;
    const int m0 = blockIdx.z * MR;
    const bool vec = (N % 4 == 0) && (((uintptr_t)y & 15) == 0) && (c + 3 < N);
    for (int t = threadIdx.x; t < MR * kSkinnyKc; t += kThreads) {
        const int m = t / kSkinnyKc, kk = t % kSkinnyKc;
        xs[m][kk] = (m0 + m < M && k0 + kk < k1) ? x[(int64_t)(m0 + m) * K + k0 + kk] : 0.0f;
    }
    __syncthreads();
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.0f;
    if (c < N) {
        auto load = [&](int64_t k) -> float4 {
            const float* py = y + k * N + c;
            if (vec) return __ldcs((const float4*)py);
            float4 t;
            t.x = py[0];
            t.y = c + 1 < N ? py[1] : 0.0f;
            t.z = c + 2 < N ? py[2] : 0.0f;
            t.w = c + 3 < N ? py[3] : 0.0f;
            return t;
        };
        constexpr int U = MR <= 4 ? 16 : 8;  // loads in flight per thread (registers permitting)
        int64_t k = k0;
        for (; k + U <= k1; k += U) {
            float4 yv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) yv[u] = load(k + u);
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int m = 0; m < MR; ++m) {
                    const float xv = xs[m][k - k0 + u];
                    acc[m][0] = fmaf(xv, yv[u].x, acc[m][0]);
                    acc[m][1] = fmaf(xv, yv[u].y, acc[m][1]);
                    acc[m][2] = fmaf(xv, yv[u].z, acc[m][2]);
                    acc[m][3] = fmaf(xv, yv[u].w, acc[m][3]);
                }
        }
        for (; k < k1; ++k) {
            const float4 yv = load(k);
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                const float xv = xs[m][k - k0];
                acc[m][0] = fmaf(xv, yv.x, acc[m][0]);
                acc[m][1] = fmaf(xv, yv.y, acc[m][1]);
                acc[m][2] = fmaf(xv, yv.z, acc[m][2]);
                acc[m][3] = fmaf(xv, yv.w, acc[m][3]);
            }
        }
        float* p = part + (int64_t)blockIdx.y * M * N;
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            if (m0 + m >= M) break;
            if (vec) {
                *(float4*)(p + (int64_t)(m0 + m) * N + c) = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (c + q < N) p[(int64_t)(m0 + m) * N + c + q] = acc[m][q];
            }
        }
    }
}

// Sum of the K slices: a CTA owns 32 consecutive outputs; warp w adds slices
// [w*S/8, (w+1)*S/8) in order (lane = output), and the eight warp sums are added in
// warp order, so the result does not depend on scheduling.
__global__ void __launch_bounds__(kThreads) matmul_skinny_sum(float* __restrict__ r, const float* __restrict__ part,
                                                              int64_t MN, int nslices, int64_t N, int64_t r_ld) {
    static_assert(kThreads == 256, "eight warps per CTA");
    __shared__ float ws[8][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t i = (int64_t)blockIdx.x * 32 + lane;
    const int s0 = (int)((int64_t)nslices * w / 8), s1 = (int)((int64_t)nslices * (w + 1) / 8);
    // launched as a programmatic dependent of the part kernel: wait until its partials are complete
    asm volatile("griddepcontrol.wait;" ::: "memory");
    float s = 0.0f;
    if (i < MN) {
#pragma unroll 8
        for (int k = s0; k < s1; ++k) s += __ldcs(part + (int64_t)k * MN + i);
    }
    ws[w][lane] = s;
    __syncthreads();
    if (w == 0 && i < MN) {
        float t = ws[0][lane];
#pragma unroll
        for (int v = 1; v < 8; ++v) t += ws[v][lane];
        r[(i / N) * r_ld + (i % N)] = t;
    }
}

// K slices so that about four CTAs per SM stream Y.
int64_t skinny_slices(int64_t M, int64_t K, int64_t N) {
    const int64_t colblocks = (N + kSkinnyCols - 1) / kSkinnyCols;
    const int64_t rowblocks = (M + kSkinnyRows - 1) / kSkinnyRows;
    int64_t want = (4 * (int64_t)sm_count() + colblocks * rowblocks - 1) / (colblocks * rowblocks);
    int64_t kc = (K + want - 1) / (want < 1 ? 1 : want);
    kc = (kc + 15) / 16 * 16;
    if (kc > kSkinnyKc) kc = kSkinnyKc;
    if (kc < 16) kc = 16;
    int64_t slices = (K + kc - 1) / kc;
    return slices < 1 ? 1 : slices;
}

int64_t skinny_kc(int64_t K, int64_t slices) {
    int64_t kc = (K + slices - 1) / slices;
    return (kc + 15) / 16 * 16;
}

cudaError_t exact_tiles(float* r, const float* x, const float* y, int64_t batch, int64_t M, int64_t K, int64_t N,
                        int64_t r_ld, int accumulate, cudaStream_t st, const float* bias, int64_t bias_mod, int act) {
    const int64_t target = 2 * (int64_t)sm_count();
    auto blocks = [&](int64_t bm, int64_t bn) { return batch * ((M + bm - 1) / bm) * ((N + bn - 1) / bn); };
    if (blocks(128, 128) >= target)
        return launch_exact<128, 128, 8, 8, 16, 2>(r, x, y, batch, M, K, N, r_ld, accumulate, st, bias, bias_mod, act);
    if (blocks(64, 64) >= target)
        return launch_exact<64, 64, 4, 4, 16, 3>(r, x, y, batch, M, K, N, r_ld, accumulate, st, bias, bias_mod, act);
    if (blocks(32, 32) >= target / 2)
        return launch_exact<32, 32, 2, 2, 32, 4>(r, x, y, batch, M, K, N, r_ld, accumulate, st, bias, bias_mod, act);
    // 64 threads of 2 x 2 outputs
    return launch_exact<16, 16, 2, 2, 64, 4>(r, x, y, batch, M, K, N, r_ld, accumulate, st, bias, bias_mod, act);
}

}  // namespace

// Row tiles are a grid dimension (at most 65535 tiles of at least 16 rows): a single product with
// more rows runs as consecutive slices of kExactRowSlice rows.
constexpr int64_t kExactRowSlice = 65535 * 16;

extern "C" int mcu_matmul_exact_kernels(int64_t batch, int64_t M) {
    return batch == 1 && M > kExactRowSlice ? (int)((M + kExactRowSlice - 1) / kExactRowSlice) : 1;
}

extern "C" int mcu_launch_matmul_exact(float* r, const float* x, const float* y, int64_t batch, int64_t M,
                                       int64_t K, int64_t N, int64_t r_ld, int accumulate, cudaStream_t st) {
    if (batch <= 0 || M <= 0 || N <= 0) return (int)cudaSuccess;
    if (batch == 1 && M > kExactRowSlice) {
        for (int64_t m0 = 0; m0 < M; m0 += kExactRowSlice) {
            const int64_t mr = M - m0 < kExactRowSlice ? M - m0 : kExactRowSlice;
            const int rc = mcu_launch_matmul_exact(r + m0 * r_ld, x + m0 * K, y, 1, mr, K, N, r_ld, accumulate, st);
            if (rc) return rc;
        }
        return (int)cudaSuccess;
    }
    if (batch >= 65536 || (M + 15) / 16 >= 65536) return (int)cudaErrorInvalidValue;
    return (int)exact_tiles(r, x, y, batch, M, K, N, r_ld, accumulate, st, nullptr, 0, 0);
}

extern "C" int mcu_launch_matmul_exact_ep(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                                          const float* bias, int64_t bias_mod, int act, cudaStream_t st) {
    if (M <= 0 || N <= 0) return (int)cudaSuccess;
    if (M > kExactRowSlice || bias_mod < 0 || act < 0 || act > 2) return (int)cudaErrorInvalidValue;
    return (int)exact_tiles(r, x, y, 1, M, K, N, N, 0, st, bias, bias_mod, act);
}

extern "C" size_t mcu_matmul_skinny_scratch_bytes(int64_t M, int64_t K, int64_t N) {
    return (size_t)skinny_slices(M, K, N) * (size_t)M * (size_t)N * sizeof(float);
}

extern "C" int mcu_launch_matmul_skinny(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                                        int64_t r_ld, void* scratch, cudaStream_t st) {
    if (M <= 0 || N <= 0) return (int)cudaSuccess;
    if (M > 4 * kSkinnyRows) return (int)cudaErrorInvalidValue;
    int64_t slices = skinny_slices(M, K, N);
    const int64_t kc = skinny_kc(K, slices);
    slices = K > 0 ? (K + kc - 1) / kc : 1;
    const unsigned rowblocks = (unsigned)((M + kSkinnyRows - 1) / kSkinnyRows);
    const int mr = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
    dim3 grid((unsigned)((N + kSkinnyCols - 1) / kSkinnyCols), (unsigned)slices, mr == 16 ? rowblocks : 1);
    float* part = (float*)scratch;
    switch (mr) {
        case 1: matmul_skinny_part<1><<<grid, kThreads, 0, st>>>(part, x, y, (int)M, K, N, kc); break;
        case 2: matmul_skinny_part<2><<<grid, kThreads, 0, st>>>(part, x, y, (int)M, K, N, kc); break;
        case 4: matmul_skinny_part<4><<<grid, kThreads, 0, st>>>(part, x, y, (int)M, K, N, kc); break;
        case 8: matmul_skinny_part<8><<<grid, kThreads, 0, st>>>(part, x, y, (int)M, K, N, kc); break;
        default: matmul_skinny_part<16><<<grid, kThreads, 0, st>>>(part, x, y, (int)M, K, N, kc); break;
    }
    const int64_t MN = M * N;
    // programmatic dependent launch: the sum's CTAs are set up while the part kernel finishes
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)((MN + 31) / 32));
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    e = cudaLaunchKernelEx(&cfg, matmul_skinny_sum, r, (const float*)part, MN, (int)slices, N, r_ld);
    return (int)e;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the skinny product.
//
// Some callers cannot allocate device memory at the moment they need a
// product: hosts that must not touch the allocator (which can block or
// synchronise the device) on a latency-critical or real-time path, and hosts
// whose device memory is carved up by a framework that owns every
// allocation.  For them the split-K partial sums live in one fixed array that
// is part of this library's device image: it is created when the library's
// device code is loaded on a GPU and stays there until the process exits.
//
// The array holds kNoAllocScratchBytes (16 MiB).  It is shared by every call
// on a device, so two calls whose kernels overlap on the GPU (different
// streams, or different host threads) race on it.  Nothing in it has to start
// at zero: every partial is written before it is read.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;
}  // namespace

static __device__ __align__(256) float g_skinny_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {
// Looked up once per device and kept for the life of the process (a cudaDeviceReset would make
// the address stale; the entry point does not support one).  Atomic: host threads may race on
// the first call.
std::atomic<void*> g_noalloc_addr[kMaxDevices];
}  // namespace

extern "C" size_t mcu_skinny_noalloc_limit(void) { return kNoAllocScratchBytes; }

// Device address of the array on the current device.  The first call on a
// device looks it up (and may make the driver load this library's device
// code there); later calls return the cached address.  Host code never uses
// the array's name as a pointer: on the host it names a stand-in object.
extern "C" int mcu_skinny_noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    void* p = g_noalloc_addr[dev].load(std::memory_order_acquire);
    if (!p) {
        e = cudaGetSymbolAddress(&p, g_skinny_noalloc_scratch);
        if (e != cudaSuccess) return (int)e;
        g_noalloc_addr[dev].store(p, std::memory_order_release);  // every thread finds the same address
    }
    *out = p;
    return (int)cudaSuccess;
}
