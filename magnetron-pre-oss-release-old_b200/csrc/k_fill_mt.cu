// k_fill_mt.cu - fills from a reference context's Mersenne-twister stream, on the device.
//
// A reference context uses the Mersenne twister unless told otherwise (mag_ctx_create2 zeroes
// the context info, algorithm 0; magnetron/magnetron.c:951, magnetron/magnetron.h:67-70).  Its
// generator (magnetron/magnetron.c:751-777) draws words from a 624-word block and twists the
// block in place when it is used up.  The twist adds the matrix constant 0x9908b0df when the low
// bit of y is 0 (the textbook generator adds it when the bit is 1), so the stream is the
// reference's own and is reproduced here as written.  In stream form the word after position k is
//     w[k] = w[k-227] ^ (y >> 1) ^ (y & 1 ? 0 : A),   y = (w[k-624] & 0x80000000) | (w[k-623] & 0x7fffffff),
// an affine map of the 624 words before it; a new word depends on words at least 227 back, so
// 227 consecutive words can be formed at once.
//
// Parallel generation by jump-ahead (Haramoto, Matsumoto, Nishimura, Panneton, L'Ecuyer,
// "Efficient jump ahead for F2-linear random number generators", 2008).  With m(x) the minimal
// polynomial of the stream and q(x) = x^d mod m(x), the 624-word window d words ahead is the
// XOR of the windows i words ahead for every i with q_i = 1.  m(x) is found once by
// Berlekamp-Massey over GF(2).  (The all-ones window is the affine map's fixed point, so the
// affine constant adds the factor x + 1 to the linear part's degree-19937 polynomial, through bit
// 0 only; the low 31 bits of a window's first word feed nothing, which adds a factor x^31 that
// dies out after 31 steps, so every jump starts from a window at least one block into the
// stream.)  The future stream is cut into substreams of L words (L a multiple of 624, chosen by
// the fill's size); the windows that start them are made by doubling: window 1 from the first
// twisted block, then windows [h, 2h - 1) from windows [1, h) by a jump of (h - 1) L, so P
// substreams take about log2(P) launches.  Each jump is shared by 16 to 64 CTAs that split q's
// set bits and XOR their sums into the zeroed window.  Then one CTA per substream runs the
// recurrence forward from its window, 454 words per barrier, tempers and maps the words as the
// reference does and writes its range of the output; Box-Muller pairs are formed in a second
// pass.
//
// The fill draws exactly the words the host generator would draw: first the words left in the
// current block, then the future stream.  The state struct is left as the host generator leaves
// it (the block of the last word drawn, `next`, `remaining`); that block is read back, so the
// call waits for its kernels when it draws past the current block.
#include "mcu_kernels.h"
#include "mcu_fill.cuh"

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <vector>

namespace {

constexpr uint32_t kMtA = 0x9908b0dfu;
constexpr int kMtN = 624;
constexpr int kMtLag = 227;               // 624 - 397
constexpr int kMtMaxDegree = 19968;       // bits of a window; the minimal polynomial's degree is below
constexpr int kMtLevels = 16;             // doubling levels: up to 2^16 + 1 substreams
constexpr int kMtPolys = 1 + kMtLevels;   // x^(L - 624), then x^(L 2^v) for v = 0..15
constexpr int kMtSets = 3;                // substream lengths, chosen by the fill's size
constexpr int64_t kMtSubstream[kMtSets] = {624LL * 96, 624LL * 384, 624LL * 1536};  // substream length L
constexpr int kMtThreads = 256;
constexpr int kMtRun = 8 * 2 * kMtLag;    // words a generation CTA forms between moves of its window
constexpr int kMtChunk = kMtMaxDegree / 16;  // exponents per jump CTA: one window's jump is split 16 ways or more
constexpr int kMtJumpWords = 34 * kMtN;   // 21216 >= offset 624 + exponent 19967 + 624
constexpr int kMtOut = 208;               // jump threads: 3 window words each

__host__ __device__ __forceinline__ uint32_t mt_word(uint32_t a, uint32_t b, uint32_t c) {
    const uint32_t y = (a & 0x80000000u) | (b & 0x7fffffffu);
    return c ^ (y >> 1) ^ ((y & 1u) ? 0u : kMtA);
}

__device__ __forceinline__ float mt_value(uint32_t y, float p0, float p1) {
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return __fadd_rn(p0, __fmul_rn(p1, mcu::unit_from_bits(y)));
}

// Exponents of the jump polynomials' set bits, ascending: [set][poly][.. count).
__device__ uint16_t g_mt_idx[kMtSets][kMtPolys][kMtMaxDegree];

// Phase pairs.  Thread i < 227 forms words k = t + i and k + 227 of each 454-word step: the
// word 227 back is the thread's own previous result (a register), and the words 624 and 623
// back were formed at least one step earlier, so one barrier per step keeps them visible.

// Window dst0 + b = the jump `idx` (cnt exponents) of the stream that starts `offset` words after
// window src0 + b.  CTA (b, c) of gridDim.y adds the exponents [c cnt / Y, (c + 1) cnt / Y),
// at most kMtChunk of them; the destination window is zero before the launch.
__global__ void __launch_bounds__(kMtThreads) mt_jump(uint32_t* __restrict__ win, int src0, int dst0, int offset,
                                                      const uint16_t* __restrict__ idx, int cnt) {
    extern __shared__ uint32_t s[];  // kMtJumpWords
    __shared__ __align__(16) uint16_t sidx[kMtChunk];
    const int tid = threadIdx.x;
    const int lo = (int)((int64_t)cnt * blockIdx.y / gridDim.y);
    const int hi = (int)((int64_t)cnt * (blockIdx.y + 1) / gridDim.y);
    if (lo >= hi || hi - lo > kMtChunk) return;  // the chunk bound holds for gridDim.y >= 16
    const int need = offset + (int)idx[hi - 1] + kMtN;  // stream words s[0 .. need) are read
    if (need > kMtJumpWords) return;                    // excluded by the degree check on the host
    const uint32_t* src = win + (size_t)(src0 + blockIdx.x) * kMtN;
    for (int i = tid; i < kMtN; i += kMtThreads) s[i] = src[i];
    for (int i = tid; i < hi - lo; i += kMtThreads) sidx[i] = idx[lo + i];
    __syncthreads();
    uint32_t prev = tid < kMtLag ? s[kMtN - kMtLag + tid] : 0u;
    for (int t = kMtN; t < need; t += 2 * kMtLag) {
        const int k = t + tid;
        if (tid < kMtLag && k < need) {
            const uint32_t a0 = s[k - 624], a1 = s[k - 623], b0 = s[k - 397], b1 = s[k - 396];
            prev = mt_word(a0, a1, prev);
            s[k] = prev;
            if (k + kMtLag < need) {
                prev = mt_word(b0, b1, prev);
                s[k + kMtLag] = prev;
            }
        }
        __syncthreads();
    }
    if (tid < kMtOut) {
        const uint32_t* base = s + offset + tid;
        uint32_t a0 = 0, a1 = 0, a2 = 0;
        auto add = [&](int o) {
            a0 ^= base[o];
            a1 ^= base[o + kMtOut];
            a2 ^= base[o + 2 * kMtOut];
        };
        // exponents eight at a time (one 16-byte shared load), then the rest one by one
        const int ne = hi - lo, ne8 = ne & ~7;
        const uint4* sv = reinterpret_cast<const uint4*>(sidx);
#pragma unroll 2
        for (int e = 0; e < ne8; e += 8) {
            const uint4 w = sv[e >> 3];
            add((int)(w.x & 0xffffu));
            add((int)(w.x >> 16));
            add((int)(w.y & 0xffffu));
            add((int)(w.y >> 16));
            add((int)(w.z & 0xffffu));
            add((int)(w.z >> 16));
            add((int)(w.w & 0xffffu));
            add((int)(w.w >> 16));
        }
        for (int e = ne8; e < ne; ++e) add(sidx[e]);
        uint32_t* dst = win + (size_t)(dst0 + blockIdx.x) * kMtN + tid;
        atomicXor(dst, a0);
        atomicXor(dst + kMtOut, a1);
        atomicXor(dst + 2 * kMtOut, a2);
    }
}

struct MtGen {
    const uint32_t* win;  // window p starts substream p (future word p L); window 0 is the current block
    uint32_t* last;       // out: the block that holds the last word drawn
    float* r;
    int64_t future;       // words drawn after the current block
    int sub;              // L: words per substream
    int first;            // words still to draw from the current block, from position `next`
    int next;
    float p0, p1;         // min, max - min (0, 1 for the normal fill's uniform pass)
};

// One step of thread tid < 227: words j and j + 227 of a substream (j = t + tid), from
// q = &s[slot of word j - 624] (the buffer is linear within a run, so every access is q plus a
// constant) into o = &out[j].  CHECK: the step may pass the words formed (span) or written (keep).
template <bool CHECK>
__device__ __forceinline__ void mt_step(uint32_t* q, float* o, uint32_t& prev, int j, int span, int keep, float p0,
                                        float p1) {
    const uint32_t a0 = q[0], a1 = q[1], b0 = q[kMtLag], b1 = q[kMtLag + 1];
    if (!CHECK || j < span) {
        prev = mt_word(a0, a1, prev);
        q[kMtN] = prev;
        if (!CHECK || j < keep) o[0] = mt_value(prev, p0, p1);
        if (!CHECK || j + kMtLag < span) {
            prev = mt_word(b0, b1, prev);
            q[kMtN + kMtLag] = prev;
            if (!CHECK || j + kMtLag < keep) o[kMtLag] = mt_value(prev, p0, p1);
        }
    }
}

// CTA p writes future words [p L, min((p + 1) L, future)) to r[first + ...], running the
// stream forward from window p; CTA 0 also writes the words left in the current block.  The CTA
// that draws the last word completes and keeps its block.  Words are formed in runs of up to 8
// steps: s[0..624) holds the 624 words before the run, the run's words follow, and after each
// run its last 624 words move to the front.
__device__ __forceinline__ void mt_forward(const MtGen& g, uint32_t* s, const uint32_t* src, float* out, int keep,
                                           bool last) {
    const int tid = threadIdx.x;
    const bool act = tid < kMtLag;
    const int span = last ? ((keep - 1) / kMtN + 1) * kMtN : keep;  // words formed
    for (int i = tid; i < kMtN; i += kMtThreads) s[i] = src[i];
    __syncthreads();
    uint32_t prev = act ? s[kMtN - kMtLag + tid] : 0u;  // word tid - 227
    int j0 = 0, run = 0;
    while (j0 < span) {
        run = span - j0 < kMtRun ? span - j0 : kMtRun;
        const int clean = keep - j0 < run ? keep - j0 : run;  // words of the run that are all written
        int t = 0;
        for (; t + 2 * kMtLag <= clean; t += 2 * kMtLag) {
            if (act) mt_step<false>(s + t + tid, out + j0 + t + tid, prev, 0, 0, 0, g.p0, g.p1);
            __syncthreads();
        }
        for (; t < run; t += 2 * kMtLag) {
            if (act) mt_step<true>(s + t + tid, out + j0 + t + tid, prev, t + tid, run, keep - j0, g.p0, g.p1);
            __syncthreads();
        }
        j0 += run;
        if (j0 < span) {  // run == kMtRun >= 624: the source and destination do not overlap
            for (int i = tid; i < kMtN; i += kMtThreads) s[i] = s[run + i];
            __syncthreads();
        }
    }
    if (last)  // the last block = the last 624 words formed = s[run .. run + 624)
        for (int i = tid; i < kMtN; i += kMtThreads) g.last[i] = s[run + i];
}

__global__ void __launch_bounds__(kMtThreads) mt_generate(const MtGen g) {
    __shared__ __align__(16) uint32_t s[kMtN + kMtRun];
    const int64_t p = blockIdx.x;
    if (p == 0)
        for (int i = threadIdx.x; i < g.first; i += kMtThreads)
            g.r[i] = mt_value(g.win[g.next + i], g.p0, g.p1);
    const int64_t w0 = p * g.sub;
    if (w0 >= g.future) return;
    const int keep = (int)(g.future - w0 < g.sub ? g.future - w0 : g.sub);  // words written
    mt_forward(g, s, g.win + p * kMtN, g.r + g.first + w0, keep, w0 + keep == g.future);
}

__global__ void __launch_bounds__(kMtThreads) mt_box_muller(float* __restrict__ r, int64_t pairs, float mean,
                                                            float stddev) {
    for (int64_t k = (int64_t)blockIdx.x * kMtThreads + threadIdx.x; k < pairs;
         k += (int64_t)gridDim.x * kMtThreads) {
        const float2 v = mcu::box_muller(r[2 * k], r[2 * k + 1], mean, stddev);
        r[2 * k] = v.x;
        r[2 * k + 1] = v.y;
    }
}

// ---------------------------------------------------------------- host: GF(2) polynomials
using Poly = std::vector<uint64_t>;  // bit i = coefficient of x^i

inline int pbit(const Poly& a, int64_t i) { return (int)((a[(size_t)(i >> 6)] >> (i & 63)) & 1u); }

// dst ^= src x^sh (bits that would land past dst's end are zero by the callers' sizes)
void xor_shifted(Poly& dst, const Poly& src, int64_t sh) {
    const size_t ws = (size_t)(sh >> 6);
    const int bs = (int)(sh & 63);
    for (size_t i = 0; i < src.size() && i + ws < dst.size(); ++i) {
        dst[i + ws] ^= src[i] << bs;
        if (bs && i + ws + 1 < dst.size()) dst[i + ws + 1] ^= src[i] >> (64 - bs);
    }
}

uint64_t spread32(uint32_t v) {  // bit i -> bit 2i
    uint64_t x = v;
    x = (x | (x << 16)) & 0x0000FFFF0000FFFFull;
    x = (x | (x << 8)) & 0x00FF00FF00FF00FFull;
    x = (x | (x << 4)) & 0x0F0F0F0F0F0F0F0Full;
    x = (x | (x << 2)) & 0x3333333333333333ull;
    x = (x | (x << 1)) & 0x5555555555555555ull;
    return x;
}

struct MinPoly {
    int degree = 0;  // 0: not available
    Poly m;          // bit `degree` set; degree / 64 + 1 words
};

size_t words_of(const MinPoly& mp) { return (size_t)(mp.degree / 64 + 1); }

void reduce(Poly& a, const MinPoly& mp) {  // a mod m, a of any size
    for (int64_t e = (int64_t)a.size() * 64 - 1; e >= mp.degree; --e)
        if (pbit(a, e)) xor_shifted(a, mp.m, e - mp.degree);
    a.resize(words_of(mp), 0);
}

Poly sqr_mod(const Poly& a, const MinPoly& mp) {  // a^2 mod m: squaring over GF(2) spreads the bits
    Poly sq(2 * a.size(), 0);
    for (size_t i = 0; i < a.size(); ++i) {
        sq[2 * i] = spread32((uint32_t)a[i]);
        sq[2 * i + 1] = spread32((uint32_t)(a[i] >> 32));
    }
    reduce(sq, mp);
    return sq;
}

void mulx(Poly& a, const MinPoly& mp) {  // a <- x a mod m
    uint64_t carry = 0;
    for (size_t i = 0; i < a.size(); ++i) {
        const uint64_t c = a[i] >> 63;
        a[i] = (a[i] << 1) | carry;
        carry = c;
    }
    if (pbit(a, mp.degree))
        for (size_t i = 0; i < a.size(); ++i) a[i] ^= mp.m[i];
}

Poly powx(uint64_t e, const MinPoly& mp) {  // x^e mod m, by squaring and multiplying by x
    Poly r(words_of(mp), 0);
    r[0] = 1;
    if (mp.degree == 0) return r;
    int b = 63;
    while (b >= 0 && !((e >> b) & 1u)) --b;
    for (; b >= 0; --b) {
        r = sqr_mod(r, mp);
        if ((e >> b) & 1u) mulx(r, mp);
    }
    return r;
}

// `count` words of the stream after the window `win`, window included: out[0..624 + count).
std::vector<uint32_t> extend(const uint32_t* win, int64_t count) {
    std::vector<uint32_t> w((size_t)(kMtN + count));
    memcpy(w.data(), win, kMtN * sizeof(uint32_t));
    for (size_t k = kMtN; k < w.size(); ++k) w[k] = mt_word(w[k - 624], w[k - 623], w[k - 227]);
    return w;
}

// x^d applied to the window at w[0]: XOR of the windows w[i ..] with q_i = 1.
void apply(const Poly& q, int degree, const uint32_t* w, uint32_t* out) {
    for (int j = 0; j < kMtN; ++j) out[j] = 0;
    for (int i = 0; i < degree; ++i)
        if (pbit(q, i))
            for (int j = 0; j < kMtN; ++j) out[j] ^= w[i + j];
}

// The stream's minimal polynomial, by Berlekamp-Massey over bit 0 of the words of a seeded
// stream from its third block on (bit 0 carries the x + 1 factor of the affine constant; the
// other bits' polynomials divide it).  Checked by one jump of all 32 bits against direct
// generation; degree 0 if anything disagrees.
MinPoly find_min_poly() {
    MinPoly mp;
    const int n = 2 * kMtMaxDegree + 128;  // enough bits for a recurrence of length <= 19968
    std::vector<uint32_t> seed(kMtN);
    seed[0] = 5489u;
    for (uint32_t i = 1; i < (uint32_t)kMtN; ++i) seed[i] = (seed[i - 1] ^ (seed[i - 1] >> 30)) * 1812433253u + i;
    const std::vector<uint32_t> w = extend(seed.data(), 2 * kMtN + n);
    const uint32_t* sw = w.data() + 2 * kMtN;  // s[j] = sw[j] & 1
    // rv: bit (n - 1 - j) = s[j], so s[k - i] sits at bit (n - 1 - k) + i
    const size_t rw = (size_t)n / 64 + 4;
    Poly rv(rw, 0);
    for (int j = 0; j < n; ++j)
        if (sw[j] & 1u) rv[(size_t)(n - 1 - j) >> 6] |= 1ull << ((n - 1 - j) & 63);
    auto get64 = [&](int64_t pos) -> uint64_t {
        const size_t q = (size_t)(pos >> 6);
        const int r = (int)(pos & 63);
        const uint64_t a = q < rw ? rv[q] : 0, b = q + 1 < rw ? rv[q + 1] : 0;
        return r ? (a >> r) | (b << (64 - r)) : a;
    };
    const size_t cw = (size_t)n / 64 + 4;
    Poly c(cw, 0), b(cw, 0);
    c[0] = b[0] = 1;
    int len = 0, shift = 1;
    for (int k = 0; k < n; ++k) {
        uint64_t acc = 0;
        const int64_t base = n - 1 - k;
        for (int wd = 0; wd <= len / 64; ++wd) acc ^= c[(size_t)wd] & get64(base + 64LL * wd);
        if (!(__builtin_popcountll(acc) & 1)) {
            ++shift;
            continue;
        }
        const Poly t = 2 * len <= k ? c : Poly();
        xor_shifted(c, b, shift);
        if (2 * len <= k) {
            len = k + 1 - len;
            b = t;
            shift = 1;
        } else {
            ++shift;
        }
    }
    if (len <= 0 || len > kMtMaxDegree - 1) return mp;
    mp.degree = len;
    mp.m.assign(words_of(mp), 0);
    for (int i = 0; i <= len; ++i)  // m(x) = x^len c(1/x)
        if (pbit(c, i)) mp.m[(size_t)(len - i) >> 6] |= 1ull << ((len - i) & 63);
    // check: a jump of 30011 words from the window 700 words into the stream above
    const int64_t d = 30011;
    const Poly q = powx((uint64_t)d, mp);
    const std::vector<uint32_t> far = extend(w.data() + 700, d);
    std::vector<uint32_t> got(kMtN);
    apply(q, mp.degree, far.data(), got.data());
    if (memcmp(got.data(), far.data() + d, kMtN * sizeof(uint32_t)) != 0) mp.degree = 0;
    return mp;
}

const MinPoly& min_poly() {
    static MinPoly mp;
    static std::once_flag once;
    std::call_once(once, [] { mp = find_min_poly(); });
    return mp;
}

struct MtSet {
    int cnt[kMtPolys] = {};
    std::vector<uint16_t> idx[kMtPolys];
};

void exponents(const Poly& q, int degree, std::vector<uint16_t>& out) {
    out.clear();
    for (int i = 0; i < degree; ++i)
        if (pbit(q, i)) out.push_back((uint16_t)i);
}

const MtSet& table_set(int k) {
    static MtSet sets[kMtSets];
    static std::once_flag once[kMtSets];
    std::call_once(once[k], [k] {
        const MinPoly& mp = min_poly();
        if (!mp.degree) return;
        MtSet& s = sets[k];
        const int64_t L = kMtSubstream[k];
        exponents(powx((uint64_t)(L - kMtN), mp), mp.degree, s.idx[0]);
        Poly q = powx((uint64_t)L, mp);
        for (int v = 0; v < kMtLevels; ++v) {
            exponents(q, mp.degree, s.idx[1 + v]);
            if (v + 1 < kMtLevels) q = sqr_mod(q, mp);
        }
        for (int i = 0; i < kMtPolys; ++i) s.cnt[i] = (int)s.idx[i].size();
    });
    return sets[k];
}

constexpr int kMaxDevices = 64;
std::atomic<uint32_t> g_uploaded[kMaxDevices];  // bit k: set k is on the device
std::mutex g_upload_mu;

// The device's copy of set k's exponent lists; *base = their device address.
int upload_set(int k, const MtSet& s, uint16_t** base) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    void* sym = nullptr;
    e = cudaGetSymbolAddress(&sym, g_mt_idx);
    if (e != cudaSuccess) return (int)e;
    *base = (uint16_t*)sym + (size_t)k * kMtPolys * kMtMaxDegree;
    if (g_uploaded[dev].load(std::memory_order_acquire) & (1u << k)) return 0;
    std::lock_guard<std::mutex> lock(g_upload_mu);
    if (g_uploaded[dev].load(std::memory_order_acquire) & (1u << k)) return 0;
    for (int i = 0; i < kMtPolys; ++i) {
        const size_t off = ((size_t)k * kMtPolys + i) * kMtMaxDegree * sizeof(uint16_t);
        e = cudaMemcpyToSymbol(g_mt_idx, s.idx[i].data(), s.idx[i].size() * sizeof(uint16_t), off);
        if (e != cudaSuccess) return (int)e;
    }
    g_uploaded[dev].fetch_or(1u << k, std::memory_order_release);
    return 0;
}

struct MtPlan {
    int64_t first, future;
    int64_t subs;   // substreams (and windows), at future words 0, L, 2L, ...
    int64_t sub;    // L
    int set;
};

int plan_fill(int64_t n, uint32_t remaining, uint32_t next, MtPlan* p) {
    if (remaining < 1 || remaining > (uint32_t)kMtN || next > (uint32_t)kMtN ||
        next + (remaining - 1) > (uint32_t)kMtN)
        return (int)cudaErrorInvalidValue;  // not a state the host generator can be in
    p->first = (int64_t)remaining - 1 < n ? (int64_t)remaining - 1 : n;
    p->future = n - p->first;
    // jumps cost about 1.2 us of the GPU per window at the widest level and 11-50 us per level
    // below it; generation about 0.15-0.22 us per 454 words of one substream: these thresholds
    // keep the sum near its minimum (2^24: 70 windows of 239616 words; 2^28: 281 of 958464)
    p->set = p->future <= (1LL << 22) ? 0 : p->future <= (3LL << 24) ? 1 : 2;
    if (const char* f = getenv("MAG_CUDA_MT_SUBSTREAM_SET"))  // tests: deep jump levels at small sizes
        if (f[0] >= '0' && f[0] < '0' + kMtSets && !f[1]) p->set = f[0] - '0';
    p->sub = kMtSubstream[p->set];
    p->subs = p->future > 0 ? (p->future + p->sub - 1) / p->sub : 0;
    if (p->subs > (1LL << kMtLevels) + 1) return (int)cudaErrorInvalidValue;
    return 0;
}

}  // namespace

extern "C" int mcu_mt19937_degree(void) { return min_poly().degree; }

// Jump of a window by d words on the host, by the same polynomials the device uses (the window
// must lie at least one block into a stream): the check of the jump arithmetic.
extern "C" int mcu_mt19937_jump_host(const uint32_t* win, uint64_t d, uint32_t* out) {
    const MinPoly& mp = min_poly();
    if (!mp.degree) return (int)cudaErrorInvalidValue;
    const std::vector<uint32_t> w = extend(win, mp.degree);
    apply(powx(d, mp), mp.degree, w.data(), out);
    return 0;
}

extern "C" size_t mcu_fill_mt_scratch_bytes(int64_t n, uint32_t remaining, uint32_t next) {
    MtPlan p;
    if (n <= 0 || plan_fill(n, remaining, next, &p)) return 0;
    const int64_t wins = p.subs > 1 ? p.subs : 1;
    return (size_t)(wins + 1) * kMtN * sizeof(uint32_t);
}

// r[0..n) from the stream of st = {remaining, next, state[624]} (the context's layout); st is
// left as the host generator would leave it.  scratch: mcu_fill_mt_scratch_bytes(n, ...).
extern "C" int mcu_launch_fill_mt(float* r, int64_t n, int normal, float p0, float p1, uint32_t* st, void* scratch,
                                  cudaStream_t stream, int* launches) {
    *launches = 0;
    if (n <= 0) return 0;
    MtPlan p;
    int rc = plan_fill(n, st[0], st[1], &p);
    if (rc) return rc;
    uint32_t* win = (uint32_t*)scratch;  // [max(subs, 1)][624] windows, then the last block
    uint32_t* last = win + (size_t)(p.subs > 1 ? p.subs : 1) * kMtN;
    cudaError_t e = cudaMemcpyAsync(win, st + 2, kMtN * sizeof(uint32_t), cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return (int)e;
    int k = 0;
    if (p.subs > 1) {
        const MinPoly& mp = min_poly();
        const MtSet& s = table_set(p.set);
        if (!mp.degree || mp.degree > kMtMaxDegree - 1) return (int)cudaErrorNotSupported;
        uint16_t* idx = nullptr;
        rc = upload_set(p.set, s, &idx);
        if (rc) return rc;
        const int smem = kMtJumpWords * (int)sizeof(uint32_t);
        e = cudaFuncSetAttribute(mt_jump, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(win + kMtN, 0, (size_t)(p.subs - 1) * kMtN * sizeof(uint32_t), stream);
        if (e != cudaSuccess) return (int)e;
        // a few windows: split each jump wider, so the level's latency shrinks
        auto split = [](int64_t windows) { return windows <= 4 ? 64u : windows <= 16 ? 32u : 16u; };
        // window 1: L - 624 words past the first twisted block, which starts 624 words after window 0
        mt_jump<<<dim3(1, split(1)), kMtThreads, smem, stream>>>(win, 0, 1, kMtN, idx, s.cnt[0]);
        ++k;
        // windows [h, min(2h - 1, subs)) = windows [1, ..) jumped by (h - 1) L = L 2^v
        int v = 0;
        for (int64_t h = 2; h < p.subs; h = 2 * h - 1, ++v) {
            const int64_t cnt = (2 * h - 1 < p.subs ? 2 * h - 1 : p.subs) - h;
            const uint16_t* q = idx + (size_t)(1 + v) * kMtMaxDegree;
            mt_jump<<<dim3((unsigned)cnt, split(cnt)), kMtThreads, smem, stream>>>(win, 1, (int)h, 0, q,
                                                                                   s.cnt[1 + v]);
            ++k;
        }
    }
    MtGen g;
    g.win = win;
    g.last = last;
    g.r = r;
    g.first = (int)p.first;
    g.future = p.future;
    g.sub = (int)p.sub;
    g.next = (int)st[1];
    g.p0 = normal ? 0.0f : p0;
    g.p1 = normal ? 1.0f : p1;
    mt_generate<<<(unsigned)(p.subs > 1 ? p.subs : 1), kMtThreads, 0, stream>>>(g);
    ++k;
    if (normal) {
        const int64_t pairs = n / 2;
        int64_t blocks = (pairs + kMtThreads - 1) / kMtThreads;
        if (blocks > 148 * 8) blocks = 148 * 8;
        if (blocks > 0) {
            mt_box_muller<<<(unsigned)blocks, kMtThreads, 0, stream>>>(r, pairs, p0, p1);
            ++k;
        }
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    *launches = k;
    if (p.future > 0) {  // the block of the last word drawn, and the position after it
        e = cudaMemcpyAsync(st + 2, last, kMtN * sizeof(uint32_t), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return (int)e;
        const uint32_t t = (uint32_t)((p.future - 1) % kMtN) + 1;  // words drawn from that block
        st[1] = t;
        st[0] = (uint32_t)kMtN + 1 - t;
    } else {
        st[1] += (uint32_t)n;
        st[0] -= (uint32_t)n;
    }
    return 0;
}
