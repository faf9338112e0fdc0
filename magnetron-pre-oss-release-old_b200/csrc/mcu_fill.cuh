// Device helpers shared by the seeded fills (k_fill.cu: PCG stream, k_fill_mt.cu:
// Mersenne-twister stream).
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace mcu {

// The reference's uniform mapping of a 32-bit draw y (magnetron/magnetron.c:776, :788):
// 2^-23 * ((y >> 9) + 0.5) = (2m + 1) * 2^-24 for m = y >> 9, one of 2^23 values in (0, 1),
// formed without an int-to-float conversion as (1 + m 2^-23) - (1 - 2^-24), where both
// operands and the difference are exact in f32.
__device__ __forceinline__ float unit_from_bits(uint32_t y) {
    return __fsub_rn(__uint_as_float(0x3F800000u | (y >> 9)), 0x1.fffffep-1f);
}

// Box-Muller on one uniform pair with the reference's f32 operation order
// (magnetron/magnetron.c:1864-1872): mag = stddev * sqrtf(-2 logf(u1)); y0 = mag * cosf(2pi u2)
// + mean, y1 with sinf.  log, sin and cos are evaluated in f64 and rounded once to f32.
__device__ __forceinline__ float2 box_muller(float u1, float u2, float mean, float stddev) {
    const float l = (float)log((double)u1);
    const float mag = __fmul_rn(stddev, __fsqrt_rn(__fmul_rn(-2.0f, l)));
    const float ang = __fmul_rn((float)(2.0 * 3.14159265358979323846), u2);
    double sd, cd;
    sincos((double)ang, &sd, &cd);
    return make_float2(__fadd_rn(__fmul_rn(mag, (float)cd), mean), __fadd_rn(__fmul_rn(mag, (float)sd), mean));
}

}  // namespace mcu
