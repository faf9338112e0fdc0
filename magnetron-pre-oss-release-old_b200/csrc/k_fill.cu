// Seeded and constant fills on the device.
//
// The reference fills tensors on the host only (magnetron/magnetron.c:1826-1876):
// a single PCG stream (magnetron/magnetron.c:779-790) drawn element by element,
// uniform values mapped as min + (max-min) * 2^-23 * ((y >> 9) + 0.5), and normal
// values as Box-Muller pairs over that uniform stream.  Here every thread jumps
// straight to its own position in the same stream (arbitrary-stride LCG jump,
// F. Brown, "Random number generation with arbitrary strides", 1994), so the
// stream is generated in parallel, value for value the host's sequence.
//
// Layout: a thread owns float4 groups g = t, t+T, t+2T, ... (T threads in the
// grid), so each warp stores 512 contiguous bytes per round; its state moves from
// group to group by one precomputed affine jump of 4T steps.  The fill is
// HBM-write bound for the uniform stream (4 B per element).
#include "mcu_kernels.h"
#include "mcu_fill.cuh"

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace {

constexpr uint64_t kPcgMul = 6364136223846793005ull;
constexpr int kFillThreads = 256;

// s -> a*s + c (mod 2^64): k steps of the LCG compose into one such map.
struct Affine {
    uint64_t a, c;
};

// The map of n LCG steps, by binary powers of the one-step map.
__host__ __device__ inline Affine lcg_jump(uint64_t n, uint64_t inc) {
    Affine acc{1ull, 0ull}, cur{kPcgMul, inc};
    while (n) {
        if (n & 1) {
            acc.a *= cur.a;
            acc.c = acc.c * cur.a + cur.c;
        }
        cur.c = (cur.a + 1ull) * cur.c;
        cur.a *= cur.a;
        n >>= 1;
    }
    return acc;
}

// PCG output permutation of the state before the step (xorshift-high, random rotate).
__device__ __forceinline__ uint32_t pcg_out(uint64_t prev) {
    const uint32_t mixed = (uint32_t)(((prev >> 18) ^ prev) >> 27);
    const uint32_t rot = (uint32_t)(prev >> 59);
    return __funnelshift_r(mixed, mixed, rot);
}

__device__ __forceinline__ float pcg_unit(uint64_t prev) { return mcu::unit_from_bits(pcg_out(prev)); }

struct FillParams {
    uint64_t s0;          // stream state at element 0
    uint64_t inc;         // stream increment
    Affine step2, step3;  // maps of 2 and 3 steps (a one-step map is (kPcgMul, inc))
    Affine stride;        // map of 4T steps
    float p0, p1;         // uniform: min, max - min;  normal: mean, stddev
};

using mcu::box_muller;

template <bool NORMAL>
__global__ void __launch_bounds__(kFillThreads) fill_pcg(float* __restrict__ r, int64_t n, FillParams p, bool vec) {
    const uint64_t t = (uint64_t)blockIdx.x * kFillThreads + threadIdx.x;
    const uint64_t T = (uint64_t)gridDim.x * kFillThreads;
    const int64_t groups = (n + 3) >> 2;
    const Affine j = lcg_jump(4ull * t, p.inc);
    uint64_t s = j.a * p.s0 + j.c;
    for (int64_t g = (int64_t)t; g < groups; g += (int64_t)T) {
        const uint64_t q1 = kPcgMul * s + p.inc;
        const uint64_t q2 = p.step2.a * s + p.step2.c;
        const uint64_t q3 = p.step3.a * s + p.step3.c;
        float4 v = make_float4(pcg_unit(s), pcg_unit(q1), pcg_unit(q2), pcg_unit(q3));
        if constexpr (NORMAL) {
            const float2 a = box_muller(v.x, v.y, p.p0, p.p1);
            const float2 b = box_muller(v.z, v.w, p.p0, p.p1);
            v = make_float4(a.x, a.y, b.x, b.y);
        } else {
            v.x = __fadd_rn(p.p0, __fmul_rn(p.p1, v.x));
            v.y = __fadd_rn(p.p0, __fmul_rn(p.p1, v.y));
            v.z = __fadd_rn(p.p0, __fmul_rn(p.p1, v.z));
            v.w = __fadd_rn(p.p0, __fmul_rn(p.p1, v.w));
        }
        const int64_t i = g << 2;
        if (vec && i + 4 <= n) {
            __stcs(reinterpret_cast<float4*>(r + i), v);
        } else {
            r[i] = v.x;
            if (i + 1 < n) r[i + 1] = v.y;
            if (i + 2 < n) r[i + 2] = v.z;
            if (i + 3 < n) r[i + 3] = v.w;
        }
        s = p.stride.a * s + p.stride.c;
    }
}

__global__ void __launch_bounds__(kFillThreads) fill_const(float* __restrict__ r, int64_t n, float x, bool vec) {
    const int64_t T = (int64_t)gridDim.x * kFillThreads;
    const int64_t groups = (n + 3) >> 2;
    const float4 v = make_float4(x, x, x, x);
    for (int64_t g = (int64_t)blockIdx.x * kFillThreads + threadIdx.x; g < groups; g += T) {
        const int64_t i = g << 2;
        if (vec && i + 4 <= n) {
            __stcs(reinterpret_cast<float4*>(r + i), v);
        } else {
            for (int k = 0; k < 4 && i + k < n; ++k) r[i + k] = x;
        }
    }
}

int fill_blocks(int64_t n) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
            sms = 148;
    }
    const int64_t groups = (n + 3) >> 2;
    const int64_t want = (groups + kFillThreads - 1) / kFillThreads;
    const int64_t cap = (int64_t)sms * 8;  // 8 resident 256-thread CTAs per SM
    return (int)(want < cap ? want : cap);
}

}  // namespace

extern "C" uint64_t mcu_pcg_advance(uint64_t state, uint64_t inc, uint64_t n) {
    const Affine j = lcg_jump(n, inc);
    return j.a * state + j.c;
}

extern "C" int mcu_launch_fill_pcg(float* r, int64_t n, int normal, float p0, float p1, uint64_t state,
                                   uint64_t inc, cudaStream_t st) {
    if (n <= 0) return 0;
    const int blocks = fill_blocks(n);
    FillParams p;
    p.s0 = state;
    p.inc = inc;
    p.step2 = lcg_jump(2, inc);
    p.step3 = lcg_jump(3, inc);
    p.stride = lcg_jump(4ull * (uint64_t)blocks * kFillThreads, inc);
    p.p0 = p0;
    p.p1 = p1;
    const bool vec = ((uintptr_t)r & 15) == 0;
    if (normal)
        fill_pcg<true><<<blocks, kFillThreads, 0, st>>>(r, n, p, vec);
    else
        fill_pcg<false><<<blocks, kFillThreads, 0, st>>>(r, n, p, vec);
    return (int)cudaGetLastError();
}

extern "C" int mcu_launch_fill_const(float* r, int64_t n, float x, cudaStream_t st) {
    if (n <= 0) return 0;
    fill_const<<<fill_blocks(n), kFillThreads, 0, st>>>(r, n, x, ((uintptr_t)r & 15) == 0);
    return (int)cudaGetLastError();
}
