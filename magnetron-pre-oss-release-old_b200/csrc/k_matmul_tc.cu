// k_matmul_tc.cu - f32 matmul on the sm_100a tensor cores with a 3xTF32 split.
//
// R[M,N] = X[M,K] Y[K,N], all row-major f32 (the buffer interpretation of
// mag_blas_matmul_f32, magnetron/magnetron_cpu.c:2151-2185).  A TF32 product
// keeps 11 significant bits, so each operand is split into two TF32 numbers,
// x = hi + lo with hi = rna_tf32(x) and lo = rna_tf32(x - hi) (Ootomo & Yokota,
// "Recovering single precision accuracy from Tensor Cores while surpassing the
// FP32 theoretical peak performance", 2022), and the product is accumulated as
// lo*hi + hi*lo + hi*hi in f32 in tensor memory; the dropped lo*lo term is
// about 2^-22 relative, so results stay within f32 rounding of the exact
// product (the matmul tolerance is 1e-5 relative, norm-wise).
//
// Kernels
//   split_rows     X -> Xhi, Xlo     [M][Kp]    (Kp = K rounded up to 32, zero padded)
//   split_cols_t   Y -> Yhi^T, Ylo^T [N][Kp]    (transposed so both operands are K-major)
//   gemm_3xtf32    persistent, warp-specialised:
//     warp 0      TMA producer: 64B-swizzled 128x16 (X) and BNx16 (Y) tiles, hi and lo,
//                 into a 4-deep shared-memory ring (mbarrier complete_tx)
//     warp 1      TMEM allocator; lane 0 issues tcgen05.mma kind::tf32 (M=128, N=BN, K=8),
//                 three per k-step, and tcgen05.commit to free ring slots / publish tiles
//     warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns -> registers -> global,
//                 from one of two TMEM accumulators so it overlaps the next tile's MMAs
// Every mbarrier wait is bounded: on expiry the kernel records a status code,
// all roles leave their loops, and TMEM is released before the CTA exits.
// No load uses cluster multicast; the same kernel serves multi-GPU runs.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cstdint>
#include "mcu_kernels.h"

namespace {

constexpr int BM = 128;          // UMMA M (one CTA, TMEM lanes 0..127)
constexpr int BK = 16;           // f32 per 64-byte swizzle row (one ring stage holds K = 16)
constexpr int KPAD = 32;         // K padding of the split operands
constexpr int kEpiWarps = 8;   // two per TMEM lane quadrant, each owning half of the tile's columns
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kWaitLimit = 1u << 22;

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

// ------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

struct Abort {
    volatile int* flag;  // shared: set once any role gives up
    int* status;         // global status word
};

// Bounded wait on the phase of `parity`.  False when this or another role gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const Abort& ab, int code) {
    for (uint32_t i = 0;; ++i) {
        if (mbar_test(bar, parity)) return true;
        if (*ab.flag) return false;
        if (i >= kWaitLimit) {
            *ab.flag = 1;
            atomicCAS(ab.status, 0, code);
            return false;
        }
        if (i > 32) __nanosleep(64);
    }
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem) * B(smem)^T, kind::tf32, issued by one thread.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Shared-memory matrix descriptor: K-major rows of BK*4 bytes, swizzled (64B
// or 128B), 8-row atoms 8*BK*4 bytes apart.
__device__ __forceinline__ uint64_t sw_desc(uint32_t saddr) {
    constexpr uint32_t row_bytes = BK * 4;
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                         // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)((8 * row_bytes) >> 4) << 32;    // stride byte offset between 8-row atoms
    d |= (uint64_t)1 << 46;                         // descriptor version for tcgen05
    d |= (uint64_t)(row_bytes == 128 ? 2 : 4) << 61; // SWIZZLE_128B or SWIZZLE_64B
    return d;
}

// Instruction descriptor, kind::tf32: D f32, A/B tf32, both K-major, M=128, N=BN.
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------ tile order
// Groups of kGroupM row-blocks sweep all column blocks, so a wave of CTAs
// shares few X panels and the Y panels stay hot in L2.
constexpr int kGroupM = 16;

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int first = g * kGroupM;
    const int gsz = min(num_m - first, kGroupM);
    const int local = t - g * per_group;
    mb = first + local % gsz;
    nb = local / gsz;
}

// ------------------------------------------------------------ the GEMM
template <int BN, int STAGES>
struct Cfg {
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BN * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 512;
    static_assert(TMEM_COLS <= 512, "two accumulators must fit TMEM");
};

// Epilogue of a fused dense layer: out = act(acc + bias) and, for the next
// product, its tf32 hi/lo split in [M][Kp_out] layout.
struct Epi {
    const float* bias;  // same row-major index as the result, or null
    float* out_hi;      // split output (null: none)
    float* out_lo;
    int64_t kp_out;
    int act;            // 0 none, 1 GELU (the reference's vector-lane formula)
};

__device__ __forceinline__ float rna_tf32_dev(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ float gelu_lane(float x) {
    // GELU lane of mag_vgelu_f32 (magnetron/magnetron_cpu.c:985-993), tanh by tanhf
    const float a = __fadd_rn(1.0f, __fmul_rn(0.044715f, __fmul_rn(x, x)));
    const float b = __fadd_rn(1.0f, tanhf(__fmul_rn(0.79788456080286535587989211986876f, __fmul_rn(x, a))));
    return __fmul_rn(0.5f, __fmul_rn(x, b));
}

template <int BN, int STAGES, bool FUSED>
__global__ void __maxnreg__(168)
    gemm_3xtf32(const __grid_constant__ CUtensorMap map_xhi, const __grid_constant__ CUtensorMap map_xlo,
                const __grid_constant__ CUtensorMap map_yhi, const __grid_constant__ CUtensorMap map_ylo,
                float* __restrict__ r, int M, int N, int Kp, int64_t ldr, int* status, const Epi epi,
                int seg_kb, int batch) {
    using C = Cfg<BN, STAGES>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* ring = smem;
    uint64_t* full = (uint64_t*)(smem + STAGES * C::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint32_t* tmem_slot = (uint32_t*)(drain + 1);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + BN - 1) / BN;
    const int tiles_per_batch = num_m * num_n;
    const int tiles = tiles_per_batch * batch;  // batch b's operands start at rows b*M (X) and b*N (Y)
    const int nk = Kp / BK;
    Abort ab{abort_flag, status};

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 32 * kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_xhi) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_xlo) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_yhi) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_ylo) : "memory");
            uint32_t it = 0;
            for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
                int mb, nb;
                const int bt = t / tiles_per_batch;
                tile_coords(t - bt * tiles_per_batch, num_m, num_n, mb, nb);
                const int xrow = bt * M + mb * BM, yrow = bt * N + nb * BN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const uint32_t s = it % STAGES, round = it / STAGES;
                    if (!mbar_wait(&empty[s], (round & 1) ^ 1, ab, 1)) goto done;
                    uint8_t* st = ring + s * C::STAGE_BYTES;
                    mbar_expect_tx(&full[s], C::STAGE_BYTES);
                    tma_load_2d(&map_xhi, &full[s], st, kb * BK, xrow);
                    tma_load_2d(&map_xlo, &full[s], st + C::A_BYTES, kb * BK, xrow);
                    tma_load_2d(&map_yhi, &full[s], st + 2 * C::A_BYTES, kb * BK, yrow);
                    tma_load_2d(&map_ylo, &full[s], st + 2 * C::A_BYTES + C::B_BYTES, kb * BK, yrow);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer: one TMEM accumulator per K segment, two in flight
            constexpr uint32_t idesc = idesc_tf32(BN);
            uint32_t it = 0, gseg = 0;
            for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
                for (int kb0 = 0; kb0 < nk; kb0 += seg_kb, ++gseg) {
                    const uint32_t b = gseg & 1, bround = gseg >> 1;
                    if (!mbar_wait(&acc_empty[b], (bround & 1) ^ 1, ab, 2)) goto done;
                    tc_fence_after();
                    const uint32_t d = tmem_base + b * BN;
                    const int kb1 = min(kb0 + seg_kb, nk);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const uint32_t s = it % STAGES, round = it / STAGES;
                        if (!mbar_wait(&full[s], round & 1, ab, 3)) goto done;
                        tc_fence_after();
                        const uint32_t base = smem_u32(ring + s * C::STAGE_BYTES);
#pragma unroll
                        for (int kk = 0; kk < BK / 8; ++kk) {
                            const uint64_t xhi = sw_desc(base + kk * 32);
                            const uint64_t xlo = sw_desc(base + C::A_BYTES + kk * 32);
                            const uint64_t yhi = sw_desc(base + 2 * C::A_BYTES + kk * 32);
                            const uint64_t ylo = sw_desc(base + 2 * C::A_BYTES + C::B_BYTES + kk * 32);
                            umma_tf32(d, xlo, yhi, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                            umma_tf32(d, xhi, ylo, idesc, 1);
                            umma_tf32(d, xhi, yhi, idesc, 1);
                        }
                        umma_commit(&empty[s]);
                    }
                    umma_commit(&acc_full[b]);
                }
            }
        }
    } else {  // ---- epilogue warps: TMEM lanes 32*(warp%4) .. +31, columns [h*BN/2, (h+1)*BN/2)
        constexpr int HC = BN / 2;   // columns per thread
        const int q = warp & 3;
        const int h = (warp - 2) >> 2;
        uint32_t gseg = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            int mb, nb;
            const int bt = t / tiles_per_batch;
            tile_coords(t - bt * tiles_per_batch, num_m, num_n, mb, nb);
            if constexpr (FUSED) {
                // bring this thread's bias row slice toward L2 now; it is read after the last segment
                const int prow = mb * BM + q * 32 + lane;
                if (epi.bias && prow < M) {
                    const float* pb = epi.bias + (int64_t)prow * N + nb * BN + h * HC;
#pragma unroll
                    for (int j = 0; j < HC; j += 32)
                        if (nb * BN + h * HC + j < N) asm volatile("prefetch.global.L2 [%0];" ::"l"(pb + j));
                }
            }
            // segment sums are added in registers with round-to-nearest
            float sum[HC];
            for (int kb0 = 0; kb0 < nk; kb0 += seg_kb, ++gseg) {
                const uint32_t b = gseg & 1, bround = gseg >> 1;
                if (!mbar_wait(&acc_full[b], bround & 1, ab, 4)) goto done;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < HC / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + b * BN + h * HC + c * 32, v);
                    if (kb0 == 0) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[c * 32 + j] = __uint_as_float(v[j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[c * 32 + j] = __fadd_rn(sum[c * 32 + j], __uint_as_float(v[j]));
                    }
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[b]);
            }
            const int row = mb * BM + q * 32 + lane;
            if (row >= M) continue;
            const int colh = nb * BN + h * HC;
            float* out = r + (int64_t)bt * M * ldr + (int64_t)row * ldr + colh;
            const bool vec = ((ldr & 3) == 0) && ((((uintptr_t)r) & 15) == 0);
#pragma unroll
            for (int c = 0; c < HC / 32; ++c) {
                float* v = sum + c * 32;
                const int cb = colh + c * 32;
                const bool full = cb + 32 <= N;
                if constexpr (FUSED) {
                    if (epi.bias) {
                        const float* pb = epi.bias + (int64_t)row * N + cb;
                        if (full && vec) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4) {
                                const float4 b4 = __ldcs((const float4*)(pb + j));
                                v[j] = __fadd_rn(v[j], b4.x);
                                v[j + 1] = __fadd_rn(v[j + 1], b4.y);
                                v[j + 2] = __fadd_rn(v[j + 2], b4.z);
                                v[j + 3] = __fadd_rn(v[j + 3], b4.w);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (cb + j < N) v[j] = __fadd_rn(v[j], pb[j]);
                        }
                    }
                    if (epi.act == 1) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = gelu_lane(v[j]);
                    }
                    if (epi.out_hi && full) {
                        float* ph = epi.out_hi + (int64_t)row * epi.kp_out + cb;
                        float* pl = epi.out_lo + (int64_t)row * epi.kp_out + cb;
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            float4 hh, ll;
                            hh.x = rna_tf32_dev(v[j]);     ll.x = rna_tf32_dev(v[j] - hh.x);
                            hh.y = rna_tf32_dev(v[j + 1]); ll.y = rna_tf32_dev(v[j + 1] - hh.y);
                            hh.z = rna_tf32_dev(v[j + 2]); ll.z = rna_tf32_dev(v[j + 2] - hh.z);
                            hh.w = rna_tf32_dev(v[j + 3]); ll.w = rna_tf32_dev(v[j + 3] - hh.w);
                            *(float4*)(ph + j) = hh;
                            *(float4*)(pl + j) = ll;
                        }
                    }
                }
                if (vec && full) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *(float4*)(out + c * 32 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (cb + j < N) out[c * 32 + j] = v[j];
                }
            }
        }
    }
done:
    __syncthreads();
    if (warp == 1) {
        if (*abort_flag && lane == 0) {
            // let MMAs still in flight finish before the accumulator is released
            umma_commit(drain);
            for (uint32_t i = 0; i < kWaitLimit && !mbar_test(drain, 0); ++i) __nanosleep(64);
        }
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"((uint32_t)C::TMEM_COLS));
    }
}

// ------------------------------------------------------------ split kernels
__device__ __forceinline__ float rna_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// X[M][K] -> hi/lo [M][Kp]; one thread per 4 consecutive k.
__global__ void __launch_bounds__(256) split_rows(const float* __restrict__ x, float* __restrict__ hi,
                                                  float* __restrict__ lo, int64_t M, int64_t K, int64_t Kp) {
    const int64_t q = Kp / 4;
    const int64_t n = M * q;
    const bool vec = (K % 4 == 0) && ((((uintptr_t)x) & 15) == 0);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / q, k = (i - m * q) * 4;
        float v[4];
        if (vec && k + 4 <= K) {
            float4 t = __ldcs((const float4*)(x + m * K + k));
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = (k + j < K) ? x[m * K + k + j] : 0.0f;
        }
        float4 h, l;
        h.x = rna_tf32(v[0]); l.x = rna_tf32(v[0] - h.x);
        h.y = rna_tf32(v[1]); l.y = rna_tf32(v[1] - h.y);
        h.z = rna_tf32(v[2]); l.z = rna_tf32(v[2] - h.z);
        h.w = rna_tf32(v[3]); l.w = rna_tf32(v[3] - h.w);
        *(float4*)(hi + m * Kp + k) = h;
        *(float4*)(lo + m * Kp + k) = l;
    }
}

// Y[K][N] -> hi/lo transposed [N][Kp] through a 32x32 shared tile.
__global__ void __launch_bounds__(256) split_cols_t(const float* __restrict__ y, float* __restrict__ hi,
                                                    float* __restrict__ lo, int64_t K, int64_t N, int64_t Kp) {
    __shared__ float tile[32][33];
    y += (int64_t)blockIdx.z * K * N;   // batch b: Y[b] is K x N, its split rows start at b*N
    hi += (int64_t)blockIdx.z * N * Kp;
    lo += (int64_t)blockIdx.z * N * Kp;
    const int64_t k0 = (int64_t)blockIdx.y * 32, n0 = (int64_t)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int j = ty; j < 32; j += 8) {
        const int64_t k = k0 + j, n = n0 + tx;
        tile[j][tx] = (k < K && n < N) ? y[k * N + n] : 0.0f;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        const int64_t n = n0 + j, k = k0 + tx;
        if (n < N && k < Kp) {
            const float v = tile[tx][j];
            const float h = rna_tf32(v);
            hi[n * Kp + k] = h;
            lo[n * Kp + k] = rna_tf32(v - h);
        }
    }
}

// ------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// 2-D map over a [rows][Kp] f32 array, box = box_rows x 32, 128-byte swizzle.
bool make_map(CUtensorMap* m, const float* base, int64_t rows, int64_t kp, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(kp * 4)};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, BK == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

struct Layout {
    int64_t kp;
    size_t xhi, xlo, yhi, ylo, total;
};

Layout layout(int64_t M, int64_t K, int64_t N) {
    Layout l;
    l.kp = round_up(K < 1 ? 1 : K, KPAD);
    size_t xs = (size_t)round_up(M * l.kp * 4, 1024), ys = (size_t)round_up(N * l.kp * 4, 1024);
    l.xhi = 0;
    l.xlo = xs;
    l.yhi = 2 * xs;
    l.ylo = 2 * xs + ys;
    l.total = 2 * xs + 2 * ys;
    return l;
}

constexpr int kBN = 256;
constexpr int kStages = 4;

// K per TMEM accumulation segment (MAG_CUDA_TC_SEGMENT, default 256).  Tensor-core
// f32 accumulation truncates; restarting the accumulator every segment and
// adding segments with round-to-nearest bounds that error by the segment length
// instead of K.  0 = one segment spanning K.
int segment_kb() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("MAG_CUDA_TC_SEGMENT");
        int k = (e && *e) ? atoi(e) : 256;
        v = k <= 0 ? (1 << 30) : (k + BK - 1) / BK;
    }
    return v;
}

}  // namespace

extern "C" int mcu_matmul_tc_supported(void) {
    if (getenv("MAG_CUDA_NO_TC")) return 0;
    return encode_fn() != nullptr;
}

extern "C" size_t mcu_matmul_tc_scratch_bytes(int64_t M, int64_t K, int64_t N) { return layout(M, K, N).total; }

static int launch_tc(float* r, const float* x, const float* y, int64_t B, int64_t M, int64_t K, int64_t N,
                     void* scratch, int* status, cudaStream_t st, const mcu_tc_epilogue* ep);

extern "C" int mcu_launch_matmul_tc_ex(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                                       void* scratch, int* status, cudaStream_t st, const mcu_tc_epilogue* ep) {
    return launch_tc(r, x, y, 1, M, K, N, scratch, status, st, ep);
}

extern "C" size_t mcu_matmul_tc_batched_scratch_bytes(int64_t B, int64_t M, int64_t K, int64_t N) {
    return layout(B * M, K, B * N).total;
}

extern "C" int mcu_launch_matmul_tc_batched(float* r, const float* x, const float* y, int64_t B, int64_t M, int64_t K,
                                            int64_t N, void* scratch, int* status, cudaStream_t st) {
    return launch_tc(r, x, y, B, M, K, N, scratch, status, st, nullptr);
}

static int launch_tc(float* r, const float* x, const float* y, int64_t B, int64_t M, int64_t K, int64_t N,
                     void* scratch, int* status, cudaStream_t st, const mcu_tc_epilogue* ep) {
    if (B <= 0 || M <= 0 || N <= 0) return (int)cudaSuccess;
    if (B * M >= (1ll << 31) || B * N >= (1ll << 31) || K >= (1ll << 21) || !scratch) return (int)cudaErrorInvalidValue;
    if (B > 1 && ep) return (int)cudaErrorInvalidValue;
    const Layout l = layout(B * M, K, B * N);
    char* base = (char*)scratch;
    float* xhi = (float*)(base + l.xhi);
    float* xlo = (float*)(base + l.xlo);
    float* yhi = (float*)(base + l.yhi);
    float* ylo = (float*)(base + l.ylo);
    const bool presplit = ep && ep->a_hi && ep->a_lo;
    if (presplit) {
        xhi = (float*)ep->a_hi;
        xlo = (float*)ep->a_lo;
    } else {
        int64_t n = B * M * (l.kp / 4);  // X of all batches is one (B*M) x K row-major matrix
        int64_t g = (n + 255) / 256;
        if (g > 8 * sm_count()) g = 8 * sm_count();
        split_rows<<<(unsigned)g, 256, 0, st>>>(x, xhi, xlo, B * M, K, l.kp);
    }
    {
        dim3 grid((unsigned)((N + 31) / 32), (unsigned)(l.kp / 32), (unsigned)B);
        split_cols_t<<<grid, 256, 0, st>>>(y, yhi, ylo, K, N, l.kp);
    }
    CUtensorMap mxh, mxl, myh, myl;
    if (!make_map(&mxh, xhi, B * M, l.kp, BM) || !make_map(&mxl, xlo, B * M, l.kp, BM) ||
        !make_map(&myh, yhi, B * N, l.kp, kBN) || !make_map(&myl, ylo, B * N, l.kp, kBN))
        return (int)cudaErrorInvalidValue;
    using C = Cfg<kBN, kStages>;
    const int64_t tiles = B * ((M + BM - 1) / BM) * ((N + kBN - 1) / kBN);
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    Epi epi{};
    const bool fused = ep && (ep->bias || ep->act || ep->out_hi);
    if (fused) {
        if (ep->out_hi && (N % 32 != 0 || ep->kp_out != round_up(N, KPAD))) return (int)cudaErrorInvalidValue;
        epi.bias = ep->bias;
        epi.out_hi = ep->out_hi;
        epi.out_lo = ep->out_lo;
        epi.kp_out = ep->kp_out;
        epi.act = ep->act;
        auto kern = gemm_3xtf32<kBN, kStages, true>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return (int)e;
        kern<<<grid, kThreads, C::SMEM, st>>>(mxh, mxl, myh, myl, r, (int)M, (int)N, (int)l.kp, (int64_t)N, status, epi,
                                              segment_kb(), (int)B);
    } else {
        auto kern = gemm_3xtf32<kBN, kStages, false>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return (int)e;
        kern<<<grid, kThreads, C::SMEM, st>>>(mxh, mxl, myh, myl, r, (int)M, (int)N, (int)l.kp, (int64_t)N, status, epi,
                                              segment_kb(), (int)B);
    }
    return (int)cudaGetLastError();
}

extern "C" int mcu_launch_matmul_tc(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                                    void* scratch, int* status, cudaStream_t st) {
    return mcu_launch_matmul_tc_ex(r, x, y, M, K, N, scratch, status, st, nullptr);
}
