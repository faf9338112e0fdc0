// mcu_math.cuh - per-element f32 math of the magnetron forward ops, on the GPU.
//
// The reference's x86-64 build evaluates its transcendentals as SSE2
// polynomials with separately rounded multiplies and adds
// (magnetron/magnetron_cpu.c:166-244, :584-621).  These device functions
// restate the same operation sequence with __fmul_rn/__fadd_rn/__fsub_rn, which
// nvcc never contracts into FMA, so each vector-lane result is bit-identical
// to the reference.  Columns at or above (cols & ~3) of a row are the
// reference's scalar tail, which calls libm; there the value is computed in
// double precision and rounded once, which agrees with glibc's f32 functions
// to within one ulp.
#pragma once
#include <cstdint>

namespace mcu {

// op numbering of magnetron/magnetron.h:136-178
enum Op : int {
    OP_NOP, OP_CLONE, OP_VIEW, OP_TRANSPOSE, OP_PERMUTE, OP_MEAN, OP_MIN, OP_MAX, OP_SUM,
    OP_ABS, OP_NEG, OP_LOG, OP_SQR, OP_SQRT, OP_SIN, OP_COS, OP_STEP, OP_SOFTMAX, OP_SOFTMAX_DV,
    OP_SIGMOID, OP_SIGMOID_DV, OP_HARD_SIGMOID, OP_SILU, OP_SILU_DV, OP_TANH, OP_TANH_DV,
    OP_RELU, OP_RELU_DV, OP_GELU, OP_GELU_DV, OP_ADD, OP_SUB, OP_MUL, OP_DIV,
    OP_ADDS, OP_SUBS, OP_MULS, OP_DIVS, OP_MATMUL
};

__device__ __forceinline__ float fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fa(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fs(float a, float b) { return __fsub_rn(a, b); }

// mag_simd_expf, SSE2 branch (magnetron/magnetron_cpu.c:167-190), one lane.
__device__ __forceinline__ float sse_expf(float x) {
    const float r = 0x1.8p23f;
    float z = fa(fm(x, 0x1.715476p+0f), r);
    float n = fs(z, r);
    float b = fs(fs(x, fm(n, 0x1.62e4p-1f)), fm(n, 0x1.7f7d1cp-20f));
    uint32_t e = __float_as_uint(z) << 23;
    float k = __uint_as_float(e + 0x3f800000u);
    float an = fabsf(n);
    float u = fm(b, b);
    float j = fa(fm(fa(fm(fa(fm(0x1.0e4020p-7f, b), 0x1.573e2ep-5f), u),
                      fa(fm(0x1.555e66p-3f, b), 0x1.fffdb6p-2f)), u),
                 fm(0x1.ffffecp-1f, b));
    if (!(an > 126.0f)) return fa(fm(j, k), k);
    uint32_t g = (n <= 0.0f) ? 0x82000000u : 0u;
    float s1 = __uint_as_float(g + 0x7f000000u);
    float s2 = __uint_as_float(e - g);
    if (an > 192.0f) return fm(s1, s1);
    return fm(fa(fm(s2, j), s2), s1);
}

// mag_vlog_f32, SSE2 branch (magnetron/magnetron_cpu.c:584-621), one lane.
__device__ __forceinline__ float sse_logf(float x) {
    float xi = (x > 0.0f) ? x : 0.0f;
    bool invalid = xi <= 0.0f;
    uint32_t ux = __float_as_uint(xi);
    int32_t emm0 = (int32_t)(ux >> 23);
    ux = (ux & ~0x7f800000u) | 0x3f000000u;
    xi = __uint_as_float(ux);
    emm0 -= 0x7f;
    float e = fa(__int2float_rn(emm0), 1.0f);
    bool mask = xi < 0.707106781186547524f;
    float tmp = mask ? xi : 0.0f;
    xi = fs(xi, 1.0f);
    e = fs(e, mask ? 1.0f : 0.0f);
    xi = fa(xi, tmp);
    float z = fm(xi, xi);
    float y = 7.0376836292e-2f;
    y = fa(fm(y, xi), -1.1514610310e-1f);
    y = fa(fm(y, xi), 1.1676998740e-1f);
    y = fa(fm(y, xi), -1.2420140846e-1f);
    y = fa(fm(y, xi), 1.4249322787e-1f);
    y = fa(fm(y, xi), -1.6668057665e-1f);
    y = fa(fm(y, xi), 2.0000714765e-1f);
    y = fa(fm(y, xi), -2.4999993993e-1f);
    y = fa(fm(y, xi), 3.3333331174e-1f);
    y = fm(y, xi);
    y = fm(y, z);
    y = fa(fm(e, -2.12194440e-4f), y);
    y = fs(y, fm(z, 0.5f));
    xi = fa(xi, y);
    xi = fa(fm(e, 0.693359375f), xi);
    return invalid ? __uint_as_float(0xffffffffu) : xi;
}

// _mm_cvtps_epi32: nearest-even, 0x80000000 for NaN and out-of-range.
__device__ __forceinline__ int32_t cvt_rne_x86(float y) {
    if (!(y < 2147483648.0f && y >= -2147483648.0f)) return INT32_MIN;
    return __float2int_rn(y);
}

// mag_simd_sincos, SSE2 branch (magnetron/magnetron_cpu.c:206-244), one lane,
// including its equality tests on the octant.
template <bool WANT_SIN>
__device__ __forceinline__ float sse_sincosf(float xin) {
    bool sign_sin = xin < 0.0f;
    float x = __uint_as_float(__float_as_uint(xin) & 0x7fffffffu);
    float y = fm(x, 1.27323954473516f);
    int32_t emm2 = cvt_rne_x86(y);
    emm2 = (int32_t)((uint32_t)emm2 + 1u);
    emm2 &= ~1;
    y = __int2float_rn(emm2);
    bool poly = emm2 == 2;
    x = fa(x, fm(y, -0.78515625f));
    x = fa(x, fm(y, -2.4187564849853515625e-4f));
    x = fa(x, fm(y, -3.77489497744594108e-8f));
    sign_sin ^= (emm2 == 4);
    bool sign_cos = (int32_t)((uint32_t)emm2 - 2u) == 4;
    float z = fm(x, x);
    float y1 = fa(-1.388731625493765e-003f, fm(z, 2.443315711809948e-005f));
    float y2 = fa(8.3321608736e-3f, fm(z, -1.9515295891e-4f));
    y1 = fa(4.166664568298827e-002f, fm(y1, z));
    y2 = fa(-1.6666654611e-1f, fm(y2, z));
    y1 = fm(y1, z);
    y2 = fm(y2, z);
    y1 = fm(y1, z);
    y1 = fs(y1, fm(z, 0.5f));
    y2 = fa(x, fm(y2, x));
    y1 = fa(y1, 1.0f);
    if (WANT_SIN) {
        float ys = poly ? y1 : y2;
        return sign_sin ? fs(0.0f, ys) : ys;
    } else {
        float yc = poly ? y2 : y1;
        return sign_cos ? yc : fs(0.0f, yc);
    }
}

#define MCU_GELU_C1 0.79788456080286535587989211986876f
#define MCU_GELU_C2 0.044715f /* MAG_GELU_COEFF, magnetron/magnetron_internal.h:36 */

// tanh inside GELU, from tanh(y) = 1 - 2 / (e^(2y) + 1) with the hardware exp2 and reciprocal:
// absolute error below 3e-7 for every finite y (GELU's tolerance is 1e-6 max(1, |x|), the same
// bound the reference's own rcpps-based tanh is held to), +-1 past |y| ~ 9, NaN stays NaN; about
// six instructions instead of tanhf's twenty-odd, which matters in the GEMM epilogue of a
// fused dense layer.
__device__ __forceinline__ float gelu_tanh(float y) {
    const float e = __expf(2.0f * y);
    return 1.0f - __fdividef(2.0f, e + 1.0f);
}

// Ops whose value depends on the lane/tail position within a row.
__host__ __device__ constexpr bool is_lane_op(int op) {
    return op == OP_LOG || op == OP_SIN || op == OP_COS || op == OP_SOFTMAX || op == OP_SOFTMAX_DV ||
           op == OP_SIGMOID || op == OP_SILU || op == OP_TANH || op == OP_GELU;
}

// Vector-lane value (magnetron/magnetron_cpu.c:538-1000, SSE2 branches).
// tanh has no bit-exact restatement (the reference refines an x86 rcpps
// estimate); TANH uses tanhf, whose error is at most 2 ulp, GELU gelu_tanh.
template <int OP>
__device__ __forceinline__ float lane_op(float x) {
    if constexpr (OP == OP_LOG) return sse_logf(x);
    else if constexpr (OP == OP_SIN) return sse_sincosf<true>(x);
    else if constexpr (OP == OP_COS) return sse_sincosf<false>(x);
    else if constexpr (OP == OP_SOFTMAX || OP == OP_SOFTMAX_DV) return sse_expf(x);
    else if constexpr (OP == OP_SIGMOID) return __fdiv_rn(1.0f, fa(1.0f, sse_expf(fs(0.0f, x))));
    else if constexpr (OP == OP_SILU) return __fdiv_rn(x, fa(1.0f, sse_expf(fs(0.0f, x))));
    else if constexpr (OP == OP_TANH) return tanhf(x);
    else if constexpr (OP == OP_GELU) {
        float a = fa(1.0f, fm(MCU_GELU_C2, fm(x, x)));
        float b = fa(1.0f, gelu_tanh(fm(MCU_GELU_C1, fm(x, a))));
        return fm(0.5f, fm(x, b));
    } else return x;
}

// Scalar-tail value: the reference calls libm (magnetron/magnetron_cpu.c:618-620 etc.).
template <int OP>
__device__ __forceinline__ float tail_op(float x) {
    if constexpr (OP == OP_LOG) return (float)log((double)x);
    else if constexpr (OP == OP_SIN) return (float)sin((double)x);
    else if constexpr (OP == OP_COS) return (float)cos((double)x);
    else if constexpr (OP == OP_SOFTMAX || OP == OP_SOFTMAX_DV) return (float)exp((double)x);
    else if constexpr (OP == OP_SIGMOID) return __fdiv_rn(1.0f, fa(1.0f, (float)exp(-(double)x)));
    else if constexpr (OP == OP_SILU) return __fdiv_rn(x, fa(1.0f, (float)exp(-(double)x)));
    else if constexpr (OP == OP_TANH) return tanhf(x);
    else if constexpr (OP == OP_GELU) {
        float t = fm(fm(MCU_GELU_C1, x), fa(1.0f, fm(fm(MCU_GELU_C2, x), x)));
        return fm(fm(0.5f, x), fa(1.0f, gelu_tanh(t)));
    } else return x;
}

// Exact element ops (magnetron/magnetron_cpu.c:308-350, :516-534, :628-645,
// :707-715, :801-819, :911-940).
template <int OP>
__device__ __forceinline__ float exact_op(float x, float xi) {
    if constexpr (OP == OP_ABS) return fabsf(x);
    else if constexpr (OP == OP_NEG) return -x;
    else if constexpr (OP == OP_SQR) return fm(x, x);
    else if constexpr (OP == OP_SQRT) return __fsqrt_rn(x);
    else if constexpr (OP == OP_STEP) return x >= 0.0f ? 1.0f : 0.0f;
    else if constexpr (OP == OP_SIGMOID_DV) return fm(x, fs(1.0f, x));
    else if constexpr (OP == OP_HARD_SIGMOID) return fminf(1.0f, fmaxf(0.0f, __fdiv_rn(fa(x, 3.0f), 6.0f)));
    else if constexpr (OP == OP_TANH_DV) { float cx = (float)cosh((double)x); return __fdiv_rn(1.0f, fm(cx, cx)); }
    else if constexpr (OP == OP_RELU) return (x > 0.0f) ? x : 0.0f;
    else if constexpr (OP == OP_RELU_DV) return x <= 0.0f ? 0.0f : 1.0f;
    else if constexpr (OP == OP_ADDS) return fa(x, xi);
    else if constexpr (OP == OP_SUBS) return fs(x, xi);
    else if constexpr (OP == OP_MULS) return fm(x, xi);
    else if constexpr (OP == OP_DIVS) return __fdiv_rn(x, xi);
    else return x;
}

template <int OP>
__device__ __forceinline__ float binop(float a, float b) {
    if constexpr (OP == OP_ADD) return fa(a, b);
    else if constexpr (OP == OP_SUB) return fs(a, b);
    else if constexpr (OP == OP_MUL) return fm(a, b);
    else return __fdiv_rn(a, b);
}

// Unsigned 32-bit division by an invariant divisor (Granlund & Montgomery,
// "Division by Invariant Integers using Multiplication", 1994, fig. 4.1).
struct FastDiv {
    uint32_t d, m, s1, s2;
};

__host__ inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f;
    f.d = d;
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) ++l;
    f.m = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    f.s1 = l < 1 ? l : 1;
    f.s2 = l > 0 ? l - 1 : 0;
    return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
    uint32_t t = __umulhi(f.m, n);
    return (t + ((n - t) >> f.s1)) >> f.s2;
}

}  // namespace mcu
