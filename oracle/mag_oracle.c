/*
 * mag_oracle.c - CPU restatement of the magnetron f32 forward-op kernels.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker, never the product path).
 * See mag_oracle.h for the contract.  References are to files of the
 * magnetron project (MarioSieg/magnetron-pre-oss-release-old).
 *
 * Build: gcc -O2 -std=gnu11 -ffp-contract=off -fPIC -shared (oracle/Makefile).
 */
#include "mag_oracle.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>

/* op numbering of magnetron/magnetron.h:136-178 */
enum {
    OP_NOP, OP_CLONE, OP_VIEW, OP_TRANSPOSE, OP_PERMUTE, OP_MEAN, OP_MIN, OP_MAX, OP_SUM,
    OP_ABS, OP_NEG, OP_LOG, OP_SQR, OP_SQRT, OP_SIN, OP_COS, OP_STEP, OP_SOFTMAX, OP_SOFTMAX_DV,
    OP_SIGMOID, OP_SIGMOID_DV, OP_HARD_SIGMOID, OP_SILU, OP_SILU_DV, OP_TANH, OP_TANH_DV,
    OP_RELU, OP_RELU_DV, OP_GELU, OP_GELU_DV, OP_ADD, OP_SUB, OP_MUL, OP_DIV,
    OP_ADDS, OP_SUBS, OP_MULS, OP_DIVS, OP_MATMUL
};

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---------------------------------------------------------------- PRNG --- */

/* mag_prng_init, PCG branch (magnetron/magnetron.c:805-808). */
void orc_pcg_seed(orc_pcg_t* g, uint64_t seed) {
    g->state = seed ^ 0x853c49e6748fea9bull;
    g->inc = 0xda3e39cb94b95bdbull;
}

/* mag_prng_generate_n, PCG branch (magnetron/magnetron.c:779-790). */
void orc_fill_uniform(orc_pcg_t* g, float* out, int64_t n, float min, float max) {
    float span = max - min;
    for (int64_t i = 0; i < n; ++i) {
        uint64_t prev = g->state;
        g->state = prev * 6364136223846793005ull + g->inc;
        uint32_t mixed = (uint32_t)(((prev >> 18u) ^ prev) >> 27u);
        uint32_t rot = (uint32_t)(prev >> 59u);
        uint32_t y = (mixed >> rot) | (mixed << ((-rot) & 31));
        float unit = (1.f / (float)(1 << 23)) * ((float)(y >> 9) + 0.5f);
        out[i] = min + span * unit;
    }
}

/* mag_tensor_fill_random_normal: uniform pairs through Box-Muller with libm
 * logf/sqrtf/cosf/sinf (magnetron/magnetron.c:1856-1876). */
void orc_fill_normal(orc_pcg_t* g, float* out, int64_t n, float mean, float stddev) {
    orc_fill_uniform(g, out, n, 0.0f, 1.0f);
    for (int64_t i = 0; i + 1 < n; i += 2) {
        float u1 = out[i], u2 = out[i + 1];
        float mag = stddev * sqrtf(-2.0f * logf(u1));
        float ang = (float)(2.0 * M_PI) * u2;
        out[i] = mag * cosf(ang) + mean;
        out[i + 1] = mag * sinf(ang) + mean;
    }
}

/* mag_prng_init, Mersenne-twister branch (magnetron/magnetron.c:797-803): init_genrand's
 * seeding; the first draw twists. */
void orc_mt_seed(orc_mt_t* g, uint64_t seed) {
    g->state[0] = (uint32_t)seed;
    for (uint32_t i = 1; i < 624; ++i)
        g->state[i] = (uint32_t)((g->state[i - 1] ^ (g->state[i - 1] >> 30)) * 1812433253u + i);
    g->next = 0;
    g->remaining = 1;
}

/* mag_prng_generate_n, Mersenne-twister branch (magnetron/magnetron.c:751-777), as written
 * there: the twist adds the matrix constant when the low bit of y is 0 (the textbook
 * generator adds it when the bit is 1), so the stream is the reference's own. */
static void orc_mt_twist(uint32_t* st) {
    uint32_t y, i;
    for (i = 0; i < 624 - 397; ++i) {
        y = (st[i] & 0x80000000u) | (st[i + 1] & 0x7fffffffu);
        st[i] = st[i + 397] ^ (y >> 1) ^ ((y & 1) ? 0 : 0x9908b0dfu);
    }
    for (; i < 624 - 1; ++i) {
        y = (st[i] & 0x80000000u) | (st[i + 1] & 0x7fffffffu);
        st[i] = st[i + (397 - 624)] ^ (y >> 1) ^ ((y & 1) ? 0 : 0x9908b0dfu);
    }
    y = (st[623] & 0x80000000u) | (st[0] & 0x7fffffffu);
    st[623] = st[396] ^ (y >> 1) ^ ((y & 1) ? 0 : 0x9908b0dfu);
}

void orc_fill_uniform_mt(orc_mt_t* g, float* out, int64_t n, float min, float max) {
    float span = max - min;
    for (int64_t i = 0; i < n; ++i) {
        if (--g->remaining <= 0) {
            g->remaining = 624;
            g->next = 0;
            orc_mt_twist(g->state);
        }
        uint32_t y = g->state[g->next++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        y ^= y >> 18;
        float unit = (1.f / (float)(1 << 23)) * ((float)(y >> 9) + 0.5f);
        out[i] = min + span * unit;
    }
}

/* The untempered words the generator draws next, without drawing them: n words from the
 * current block on (a test helper: the stream positions a device fill continues from). */
void orc_mt_words(const orc_mt_t* g, uint32_t* out, int64_t n) {
    orc_mt_t c = *g;
    for (int64_t i = 0; i < n; ++i) {
        if (--c.remaining <= 0) {
            c.remaining = 624;
            c.next = 0;
            orc_mt_twist(c.state);
        }
        out[i] = c.state[c.next++];
    }
}

void orc_fill_normal_mt(orc_mt_t* g, float* out, int64_t n, float mean, float stddev) {
    orc_fill_uniform_mt(g, out, n, 0.0f, 1.0f);
    for (int64_t i = 0; i + 1 < n; i += 2) {
        float u1 = out[i], u2 = out[i + 1];
        float mag = stddev * sqrtf(-2.0f * logf(u1));
        float ang = (float)(2.0 * M_PI) * u2;
        out[i] = mag * cosf(ang) + mean;
        out[i + 1] = mag * sinf(ang) + mean;
    }
}

/* ------------------------------------------------- vector transcendentals --- */

/* mag_simd_expf, SSE2 branch (magnetron/magnetron_cpu.c:167-190), one lane.
 * The 4-lane fast/slow split picks the same value per lane either way
 * (k*j+k == j*k+k), so the lane is evaluated on its own. */
float orc_sse_expf(float x) {
    const float r = 0x1.8p23f;
    float z = x * 0x1.715476p+0f + r;
    float n = z - r;
    float b = (x - n * 0x1.62e4p-1f) - n * 0x1.7f7d1cp-20f;
    uint32_t e = f2u(z) << 23;
    float k = u2f(e + f2u(1.0f));
    int c = fabsf(n) > 126.0f;
    float u = b * b;
    float j = ((0x1.0e4020p-7f * b + 0x1.573e2ep-5f) * u + (0x1.555e66p-3f * b + 0x1.fffdb6p-2f)) * u
              + 0x1.ffffecp-1f * b;
    if (!c) return j * k + k;
    uint32_t g = (n <= 0.0f) ? 0x82000000u : 0u;
    float s1 = u2f(g + 0x7f000000u);
    float s2 = u2f(e - g);
    if (fabsf(n) > 192.0f) return s1 * s1;
    return (s2 * j + s2) * s1;
}

/* mag_vlog_f32, SSE2 branch (magnetron/magnetron_cpu.c:584-621), one lane.
 * Non-positive and NaN inputs give the all-ones NaN pattern, as the
 * reference's OR with the invalid mask does. */
float orc_sse_logf(float x) {
    float xi = (x > 0.0f) ? x : 0.0f;             /* _mm_max_ps(x, 0) */
    int invalid = xi <= 0.0f;
    uint32_t ux = f2u(xi);
    int32_t emm0 = (int32_t)(ux >> 23);
    ux = (ux & ~0x7f800000u) | f2u(0.5f);
    xi = u2f(ux);
    emm0 = emm0 - 0x7f;
    float e = (float)emm0;
    e = e + 1.0f;
    int mask = xi < 0.707106781186547524f;
    float tmp = mask ? xi : 0.0f;
    xi = xi - 1.0f;
    e = e - (mask ? 1.0f : 0.0f);
    xi = xi + tmp;
    float z = xi * xi;
    float y = 7.0376836292e-2f;
    y = y * xi + -1.1514610310e-1f;
    y = y * xi + 1.1676998740e-1f;
    y = y * xi + -1.2420140846e-1f;
    y = y * xi + 1.4249322787e-1f;
    y = y * xi + -1.6668057665e-1f;
    y = y * xi + 2.0000714765e-1f;
    y = y * xi + -2.4999993993e-1f;
    y = y * xi + 3.3333331174e-1f;
    y = y * xi;
    y = y * z;
    y = e * -2.12194440e-4f + y;
    y = y - z * 0.5f;
    xi = xi + y;
    xi = e * 0.693359375f + xi;
    if (invalid) return u2f(0xffffffffu);
    return xi;
}

/* _mm_cvtps_epi32 under the default rounding mode: nearest-even, and the
 * "integer indefinite" 0x80000000 for NaN or out-of-range inputs. */
static int32_t cvt_rne_i32(float y) {
    if (!(y < 2147483648.0f && y >= -2147483648.0f)) return INT32_MIN;
    return (int32_t)nearbyintf(y);
}

/* mag_simd_sincos, SSE2 branch (magnetron/magnetron_cpu.c:206-244), one lane.
 * Restated as written, including its equality tests on the octant. */
void orc_sse_sincosf(float xin, float* osin, float* ocos) {
    int sign_sin = xin < 0.0f;
    float x = u2f(f2u(xin) & 0x7fffffffu);
    float y = x * 1.27323954473516f;
    int32_t emm2 = cvt_rne_i32(y);
    emm2 = (int32_t)((uint32_t)emm2 + 1u);
    emm2 = emm2 & ~1;
    y = (float)emm2;
    int poly = emm2 == 2;
    x = x + y * -0.78515625f;
    x = x + y * -2.4187564849853515625e-4f;
    x = x + y * -3.77489497744594108e-8f;
    sign_sin ^= (emm2 == 4);
    int sign_cos = (int32_t)((uint32_t)emm2 - 2u) == 4;
    float z = x * x;
    float y1 = -1.388731625493765e-003f + z * 2.443315711809948e-005f;
    float y2 = 8.3321608736e-3f + z * -1.9515295891e-4f;
    y1 = 4.166664568298827e-002f + y1 * z;
    y2 = -1.6666654611e-1f + y2 * z;
    y1 = y1 * z;
    y2 = y2 * z;
    y1 = y1 * z;
    y1 = y1 - z * 0.5f;
    y2 = x + y2 * x;
    y1 = y1 + 1.0f;
    float ys = poly ? y1 : y2;
    float yc = poly ? y2 : y1;
    *osin = sign_sin ? (0.0f - ys) : ys;
    *ocos = sign_cos ? yc : (0.0f - yc);
}

/* Correctly rounded tanh: stands in for the reference's SSE2 tanh, whose
 * rcpps step is hardware-table dependent (magnetron/magnetron_cpu.c:192-204). */
static float tanh_cr(float x) { return (float)tanh((double)x); }

#define GELU_C1 0.79788456080286535587989211986876f
#define GELU_C2 0.044715f /* MAG_GELU_COEFF, magnetron/magnetron_internal.h:36 */

/* Vector-lane value of each transcendental op (columns below cols & ~3). */
static float lane_op(int op, float x) {
    switch (op) {
        case OP_LOG: return orc_sse_logf(x);
        case OP_SIN: { float s, c; orc_sse_sincosf(x, &s, &c); return s; }
        case OP_COS: { float s, c; orc_sse_sincosf(x, &s, &c); return c; }
        case OP_SOFTMAX: case OP_SOFTMAX_DV: return orc_sse_expf(x);
        case OP_SIGMOID: return 1.0f / (1.0f + orc_sse_expf(0.0f - x));  /* :763-770 */
        case OP_SILU: return x / (1.0f + orc_sse_expf(0.0f - x));        /* :848-855 */
        case OP_TANH: return tanh_cr(x);
        case OP_GELU: {                                                  /* :985-993 */
            float a = 1.0f + GELU_C2 * (x * x);
            float b = 1.0f + tanh_cr(GELU_C1 * (x * a));
            return 0.5f * (x * b);
        }
        default: return 0.0f;
    }
}

/* Scalar-tail value (columns at or above cols & ~3), libm as in the reference. */
static float tail_op(int op, float x) {
    switch (op) {
        case OP_LOG: return logf(x);
        case OP_SIN: return sinf(x);
        case OP_COS: return cosf(x);
        case OP_SOFTMAX: case OP_SOFTMAX_DV: return expf(x);
        case OP_SIGMOID: return 1.0f / (1.0f + expf(-x));                  /* :773 */
        case OP_SILU: return x / (1.0f + expf(-x));                        /* :858-860 */
        case OP_TANH: return tanhf(x);                                     /* :895-897 */
        case OP_GELU: return 0.5f * x * (1.0f + tanhf(GELU_C1 * x * (1.0f + GELU_C2 * x * x))); /* :995-997 */
        default: return 0.0f;
    }
}

static int is_lane_op(int op) {
    return op == OP_LOG || op == OP_SIN || op == OP_COS || op == OP_SOFTMAX || op == OP_SOFTMAX_DV ||
           op == OP_SIGMOID || op == OP_SILU || op == OP_TANH || op == OP_GELU;
}

/* Exact element ops (magnetron/magnetron_cpu.c:308-350, :516-534, :628-645,
 * :707-715, :801-819, :911-940). */
static float exact_op(int op, float x, float xi) {
    switch (op) {
        case OP_ABS: return fabsf(x);
        case OP_NEG: return -x;
        case OP_SQR: return x * x;
        case OP_SQRT: return sqrtf(x);
        case OP_STEP: return x >= 0.0f ? 1.0f : 0.0f;
        case OP_SIGMOID_DV: return x * (1.0f - x);
        case OP_HARD_SIGMOID: return fminf(1.0f, fmaxf(0.0f, (x + 3.0f) / 6.0f));
        case OP_TANH_DV: { float cx = coshf(x); return 1.0f / (cx * cx); }
        case OP_RELU: return (x > 0.0f) ? x : 0.0f;      /* mag_max(x, 0.0f) */
        case OP_RELU_DV: return x <= 0.0f ? 0.0f : 1.0f;
        case OP_ADDS: return x + xi;
        case OP_SUBS: return x - xi;
        case OP_MULS: return x * xi;
        case OP_DIVS: return x / xi;
        default: return 0.0f;
    }
}

/* Row driver shared by all unary and scalar ops, e.g. mag_blas_abs_f32
 * (magnetron/magnetron_cpu.c:1154-1175): row ri starts at ri*s1 and holds
 * cols = shape[0] consecutive elements. */
int orc_unary(int op, float* r, const float* x, int64_t rows, int64_t cols,
              int64_t r_s1, int64_t x_s1, float xi) {
    if (op == OP_SILU_DV || op == OP_GELU_DV) return (rows > 0 && cols > 0) ? -1 : 0; /* mag_panic("NYI") :873-881, :1002-1010 */
    int lane = is_lane_op(op);
    int64_t vec_end = cols & ~(int64_t)3;
    for (int64_t ri = 0; ri < rows; ++ri) {
        float* pr = r + ri * r_s1;
        const float* px = x + ri * x_s1;
        for (int64_t c = 0; c < cols; ++c) {
            float v = px[c];
            if (lane) pr[c] = (c < vec_end) ? lane_op(op, v) : tail_op(op, v);
            else pr[c] = exact_op(op, v, xi);
        }
    }
    return 0;
}

static inline float bin(int op, float a, float b) {
    switch (op) {
        case OP_ADD: return a + b;
        case OP_SUB: return a - b;
        case OP_MUL: return a * b;
        default: return a / b;
    }
}

/* mag_blas_add_f32 and siblings (magnetron/magnetron_cpu.c:1616-1714): rows
 * walk x's dims 1..5; y is tiled by index modulo its own dims. */
void orc_binary(int op, float* r, const float* x, const float* y,
                const int64_t* xd, const int64_t* xs, const int64_t* rs,
                const int64_t* yd, const int64_t* ys) {
    for (int64_t i5 = 0; i5 < xd[5]; ++i5)
    for (int64_t i4 = 0; i4 < xd[4]; ++i4)
    for (int64_t i3 = 0; i3 < xd[3]; ++i3)
    for (int64_t i2 = 0; i2 < xd[2]; ++i2)
    for (int64_t i1 = 0; i1 < xd[1]; ++i1) {
        float* pr = r + i1 * rs[1] + i2 * rs[2] + i3 * rs[3] + i4 * rs[4] + i5 * rs[5];
        const float* px = x + i1 * xs[1] + i2 * xs[2] + i3 * xs[3] + i4 * xs[4] + i5 * xs[5];
        const float* py = y + (i1 % yd[1]) * ys[1] + (i2 % yd[2]) * ys[2] + (i3 % yd[3]) * ys[3]
                            + (i4 % yd[4]) * ys[4] + (i5 % yd[5]) * ys[5];
        for (int64_t c = 0; c < xd[0]; ++c)
            pr[c] = bin(op, px[c], py[(c % yd[0]) * ys[0]]);
    }
}

/* mag_vsum_f64_f32 / mag_vmin_f32 / mag_vmax_f32 (magnetron/magnetron_cpu.c:477-514). */
static double row_sum(const float* p, int64_t n) { double s = 0.0; for (int64_t i = 0; i < n; ++i) s += (double)p[i]; return s; }
static float row_min(const float* p, int64_t n) { float m = INFINITY; for (int64_t i = 0; i < n; ++i) m = fminf(m, p[i]); return m; }
static float row_max(const float* p, int64_t n) { float m = -INFINITY; for (int64_t i = 0; i < n; ++i) m = fmaxf(m, p[i]); return m; }

/* mag_blas_{mean,min,max,sum}_f32 (magnetron/magnetron_cpu.c:1034-1152). */
float orc_reduce(int op, const float* x, const int64_t* xd, const int64_t* xs) {
    double sum = 0.0;
    float mn = INFINITY, mx = -INFINITY;
    int64_t numel = 1;
    for (int i = 0; i < 6; ++i) numel *= xd[i];
    for (int64_t i5 = 0; i5 < xd[5]; ++i5)
    for (int64_t i4 = 0; i4 < xd[4]; ++i4)
    for (int64_t i3 = 0; i3 < xd[3]; ++i3)
    for (int64_t i2 = 0; i2 < xd[2]; ++i2)
    for (int64_t i1 = 0; i1 < xd[1]; ++i1) {
        const float* p = x + i1 * xs[1] + i2 * xs[2] + i3 * xs[3] + i4 * xs[4] + i5 * xs[5];
        if (op == OP_SUM || op == OP_MEAN) sum += row_sum(p, xd[0]);
        else if (op == OP_MIN) mn = fminf(row_min(p, xd[0]), mn);
        else mx = fmaxf(row_max(p, xd[0]), mx);
    }
    if (op == OP_SUM) return (float)sum;
    if (op == OP_MEAN) return (float)(sum / (double)numel);
    return op == OP_MIN ? mn : mx;
}

/* mag_blas_matmul_f32, active i-k-j loop (magnetron/magnetron_cpu.c:2172-2185). */
void orc_matmul(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N, int64_t r_ld) {
    for (int64_t i = 0; i < M; ++i)
        for (int64_t k = 0; k < K; ++k) {
            float a = x[i * K + k];
            const float* py = y + k * N;
            float* pr = r + i * r_ld;
            for (int64_t j = 0; j < N; ++j) pr[j] += a * py[j];
        }
}

/* Rows [row0, row0+nrows) of X.Y into r (zeroed here), same arithmetic. */
void orc_matmul_rows(float* r, const float* x, const float* y, int64_t row0, int64_t nrows, int64_t K, int64_t N) {
    memset(r, 0, sizeof(float) * (size_t)(nrows * N));
    orc_matmul(r, x + row0 * K, y, nrows, K, N, N);
}

void orc_matmul_batched(float* r, const float* x, const float* y, int64_t batch, int64_t M, int64_t K, int64_t N) {
    memset(r, 0, sizeof(float) * (size_t)(batch * M * N));
    for (int64_t b = 0; b < batch; ++b)
        orc_matmul(r + b * M * N, x + b * M * K, y + b * K * N, M, K, N, N);
}

/* Two-sided tiling broadcast, r[i] = x[i mod x_d] (op) y[i mod y_d] per dim,
 * all contiguous with dim 0 fastest.  sample_idx selects linear result
 * indices (r is then packed, one value per sample); NULL means all. */
void orc_binary_bcast2(int op, float* r, const float* x, const float* y,
                       const int64_t* rd, const int64_t* xd, const int64_t* yd,
                       const int64_t* sample_idx, int64_t n_sample) {
    int64_t total = 1;
    for (int i = 0; i < 6; ++i) total *= rd[i];
    int64_t n = sample_idx ? n_sample : total;
    for (int64_t s = 0; s < n; ++s) {
        int64_t lin = sample_idx ? sample_idx[s] : s;
        int64_t rem = lin, xo = 0, yo = 0, xst = 1, yst = 1;
        for (int d = 0; d < 6; ++d) {
            int64_t id = rem % rd[d];
            rem /= rd[d];
            xo += (id % xd[d]) * xst;
            yo += (id % yd[d]) * yst;
            xst *= xd[d];
            yst *= yd[d];
        }
        r[s] = bin(op, x[xo], y[yo]);
    }
}

/* Row reductions over contiguous rows, with the reference's accumulation:
 * double sequential sum, mean = (float)(sum/cols), fminf/fmaxf scans. */
void orc_reduce_rows(int op, float* r, const float* x, int64_t rows, int64_t cols) {
    for (int64_t i = 0; i < rows; ++i) {
        const float* p = x + i * cols;
        if (op == OP_SUM) r[i] = (float)row_sum(p, cols);
        else if (op == OP_MEAN) r[i] = (float)(row_sum(p, cols) / (double)cols);
        else if (op == OP_MIN) r[i] = row_min(p, cols);
        else r[i] = row_max(p, cols);
    }
}

/* Normalised row softmax built from the reference's own pieces: the row max
 * (mag_vmax_f32), x - max in f32, the reference exp (SSE2 lanes, expf tail)
 * and a double sum (mag_vsum_f64_f32); r = e / (float)sum. */
void orc_softmax_rows(float* r, const float* x, int64_t rows, int64_t cols) {
    int64_t vec_end = cols & ~(int64_t)3;
    for (int64_t i = 0; i < rows; ++i) {
        const float* p = x + i * cols;
        float* q = r + i * cols;
        float m = row_max(p, cols);
        double s = 0.0;
        for (int64_t c = 0; c < cols; ++c) {
            float t = p[c] - m;
            float e = c < vec_end ? orc_sse_expf(t) : expf(t);
            q[c] = e;
            s += (double)e;
        }
        float fs = (float)s;
        for (int64_t c = 0; c < cols; ++c) q[c] = q[c] / fs;
    }
}
