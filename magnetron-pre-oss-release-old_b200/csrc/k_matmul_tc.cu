// k_matmul_tc.cu - f32 matmul on the sm_100a tensor cores with a three-product split.
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
// The same split in f16 (11 significant bits, like tf32) runs the kind::f16
// tensor-core path at twice the kind::tf32 rate.  f16's narrow exponent range is
// handled by exact power-of-two scaling: each row of X and each column of Y is
// scaled so its largest magnitude lies in [2^14, 2^15) before the split, and the
// epilogue multiplies the sum by 2^-(row exponent + column exponent).  Errors are
// then bounded relative to the row and column maxima, as for tf32.
//
// Kernels
//   split_rows[_f16]     X -> Xhi, Xlo     [M][Kp]  (Kp = K rounded up to 32, zero padded)
//   split_cols_t[_f16]   Y -> Yhi^T, Ylo^T [N][Kp]  (transposed so both operands are K-major)
//   gemm_3x              persistent, warp-specialised:
//     warp 0      TMA producer: 64B-swizzled 128-row (X) and BN-row (Y) tiles of 64 bytes of K
//                 (16 tf32 or 32 f16), hi and lo, into a 4-deep shared-memory ring
//     warp 1      TMEM allocator; lane 0 issues tcgen05.mma kind::tf32 or kind::f16
//                 (M=128, N=BN, 32 bytes of K), three per k-step, and tcgen05.commit to
//                 free ring slots / publish accumulators
//     warps 4..11 epilogue: tcgen05.ld 32 lanes x 32 columns -> registers -> global,
//                 from one of two TMEM accumulators so it overlaps the next segment's MMAs;
//                 a fused layer's bias arrives by TMA in 32 x 32 chunks staged in shared memory
//   Warpgroup 0 (producer, MMA issuer, two idle warps) gives registers to the two epilogue
//   warpgroups with setmaxnreg, so the 128 per-thread segment sums never spill.
// Every mbarrier wait is bounded: on expiry the kernel records a status code,
// all roles leave their loops, and TMEM is released before the CTA exits.
// No load uses cluster multicast; the same kernel serves multi-GPU runs.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cstdint>
#include <cstring>
#include "mcu_kernels.h"
#include "mcu_math.cuh"

#include <utility>

namespace {

constexpr int BM = 128;          // UMMA M (one CTA, TMEM lanes 0..127)
constexpr int ROW_BYTES = 64;    // K bytes per swizzled smem row: one ring stage holds 64 bytes of K
constexpr int BK = 16;           // f32 per 64-byte row (the tf32 split)
constexpr int BK16 = 32;         // f16 per 64-byte row (the f16 split)
constexpr int KPAD = 32;         // K padding of the split operands
constexpr int kEpiWarps = 8;   // two per TMEM lane quadrant, each owning half of the tile's columns
constexpr int kEpiWarp0 = 4;   // warpgroup 0: producer, MMA issuer, two idle warps; warpgroups 1-2: epilogue
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
// Register split (setmaxnreg): the launch gives every thread kLaunchRegs; warpgroup 0 drops to
// kCtrlRegs and the two epilogue warpgroups rise to kEpiRegs, so the epilogue holds its
// 128-column segment sums without spilling.  128*kCtrlRegs + 256*kEpiRegs == kThreads*kLaunchRegs.
constexpr int kLaunchRegs = 168, kCtrlRegs = 40, kEpiRegs = 232;
static_assert(128 * kCtrlRegs + 256 * kEpiRegs == kThreads * kLaunchRegs, "register split must match the launch");
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

__device__ __forceinline__ float4 lds4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a) : "memory");
    return v;
}

__device__ __forceinline__ void sts4(uint32_t a, float x, float y, float z, float w) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}

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

// Programmatic dependent launch: every kernel of a product's chain after the first is launched so
// that it may be scheduled while its predecessor finishes; each kernel waits for the previous
// grid's completion (and memory) before it touches memory, and lets its own dependents be
// scheduled at once.  Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
}

// ---- CTA pairs (2-CTA clusters): the leader (rank 0) issues the MMAs for both CTAs
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of `saddr` (a shared::cta address) in the CTA of rank `rank`.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an mbarrier of
// either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t bar_caddr, void* dst, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"((uint64_t)map), "r"(bar_caddr), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem) * B(smem)^T, kind::tf32 or kind::f16 (both operands the same
// type), issued by one thread.
template <bool F16, bool PAIR = false>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
    if constexpr (PAIR) {  // M = 256 across the pair: A rows and half of B from each CTA's shared memory
        if constexpr (F16) {
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
                "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
        } else {
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
                "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
        }
    } else if constexpr (F16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
    }
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// Pair form: arrives on the barrier at the same offset in both CTAs of the pair.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}
// Pair form, this CTA's barrier only.
__device__ __forceinline__ void umma_commit_pair_local(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Shared-memory matrix descriptor: K-major rows of ROW_BYTES bytes, swizzled (64B
// or 128B), 8-row atoms 8*ROW_BYTES bytes apart.
template <int RB = ROW_BYTES>
__device__ __forceinline__ uint64_t sw_desc(uint32_t saddr) {
    constexpr uint32_t row_bytes = RB;
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                         // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)((8 * row_bytes) >> 4) << 32;    // stride byte offset between 8-row atoms
    d |= (uint64_t)1 << 46;                         // descriptor version for tcgen05
    d |= (uint64_t)(row_bytes == 128 ? 2 : 4) << 61; // SWIZZLE_128B or SWIZZLE_64B
    return d;
}

// Instruction descriptor: D f32, A/B tf32 (format 2, kind::tf32) or f16 (format 0,
// kind::f16), both K-major, M = 128 (one CTA) or 256 (a CTA pair), N=BN.
__host__ __device__ constexpr uint32_t idesc_3x(int n, bool f16, int m = BM) {
    const uint32_t fmt = f16 ? 0u : 2u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// v * 2^-s for s in [-252, 252] (row and column exponents lie in [-113, 126]): two
// multiplications by normal powers of two that scale the same way, so the product is
// exact unless the result is subnormal or overflows, and then rounded once.
__device__ __forceinline__ float unscale(float v, int s) {
    const int s1 = s >> 1, s2 = s - s1;
    return __fmul_rn(__fmul_rn(v, __int_as_float((127 - s1) << 23)), __int_as_float((127 - s2) << 23));
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
template <int BN, int STAGES, bool PAIR = false, int RB = ROW_BYTES>
struct Cfg {
    static constexpr int A_BYTES = BM * RB;
    static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * RB;  // a pair splits Y's rows between its CTAs
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 512;
    // fused epilogue: each epilogue warp stages its 32 x 32 f32 bias chunk (4 KB, 128B-swizzled)
    static constexpr int BIAS_BYTES = kEpiWarps * 32 * 32 * 4;
    static constexpr int SMEM_BIAS = STAGES * STAGE_BYTES + 1024 + BIAS_BYTES + 1024;
    static_assert(TMEM_COLS <= 512, "two accumulators must fit TMEM");
    static_assert(SMEM <= 227 * 1024, "the ring must fit shared memory");
};

// Epilogue of a fused dense layer: out = act(acc + bias) and, for the next
// product, its tf32 hi/lo split in [M][Kp_out] layout.
struct Epi {
    const float* bias;  // same row-major index as the result, or null
    float* out_hi;      // split output (null: none; tf32 split only)
    float* out_lo;
    int64_t kp_out;
    int act;            // 0 none, 1 GELU (the reference's vector-lane formula)
    const int* row_exp; // f16 split: power-of-two exponents of X's rows ([B*M]) and Y's columns ([B*N])
    const int* col_exp;
    int bias_map;       // the bias is also described by map_bias (32 x 32 boxes): staged through shared memory
    int bias_zero;      // no bias read: the bias is known to be zero, and x + 0.0f (-0 -> +0) stands for it
    // f16 split: floor-element counts of X's rows ([B*M]) and of Y's 32-column chunks
    // ([B*ceil(N/32)]), and where outputs that fail the floor check are listed (floor_check)
    const int* row_floor;
    const int* col_floor;
    int2* chk_list;     // (global row, column) of each listed output, up to chk_cap
    int* chk_count;     // [0] outputs listed (may pass chk_cap), [1] rows listed
    int* chk_rflag;     // [B*M] a row has a listed output
    int* chk_rows;      // [B*M] those rows
    int chk_cap;
};

__device__ __forceinline__ float rna_tf32_dev(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ float gelu_lane(float x) {
    // GELU lane of mag_vgelu_f32 (magnetron/magnetron_cpu.c:985-993), the same arithmetic as the
    // elementwise GELU kernel (lane_op<OP_GELU>), so fused and unfused layers agree bit for bit
    return mcu::lane_op<mcu::OP_GELU>(x);
}

// The floor of the f16 split.  For a scaled element s = x * 2^e (row maximum in [2^14, 2^15)),
// hi + lo represents s within 2^-22 |s| while lo is a normal f16, i.e. for |s| >= 2^-3; below
// that ("floor elements") lo is subnormal and the error is at most 2^-25, absolute, in scaled
// units.  So an output's error beyond the 2^-22-relative terms is at most
//     2^-25 (nF_i 2^-e_i max_k|y_kj| + nG_j 2^-f_j max_k|x_ik|) <= 2^-10 2^-(e_i+f_j) (nF_i + nG_j)
// (nF_i, nG_j: floor elements of row i of X and column j of Y; the maxima are below 2^(15-e)),
// which is at most 2^-18 (3.8e-6) of the output whenever its scaled sum |acc| = 2^(e_i+f_j) |C_ij|
// is at least 2^8 (nF_i + nG_j); with the other error terms (2^-21 relative to |X||Y| for the
// split and the dropped lo*lo product, about 2e-6 for the segment-wise accumulation) an output
// stays within 1e-5 of |X||Y|.  Outputs below that are listed and recomputed exactly
// (fix_outputs): in ordinary data a few hundred per large product, for a row whose large entries
// meet zeros in Y (all its products then carried by elements far below its maximum) the whole
// row.  The GEMM epilogue bounds nG_j by the largest count of the output's 32-column chunk.
__device__ __forceinline__ float floor_threshold(int n) { return n > 0 ? 256.0f * (float)n : 0.0f; }

// Largest floor count of the 32 columns of chunk cb (per column counts in cf; a warp-wide
// reduction, every lane gets it).
__device__ __forceinline__ int chunk_floor(const int* cf, int64_t cb, int64_t N, int lane) {
    return __reduce_max_sync(0xffffffffu, cb + lane < N ? __ldg(cf + cb + lane) : 0);
}

__device__ __noinline__ void list_output(int2* list, int* count, int* rflag, int* rows, int cap, int64_t grow,
                                        int64_t col) {
    const int i = atomicAdd(count, 1);
    if (i < cap) list[i] = make_int2((int)grow, (int)col);
    if (atomicExch(rflag + grow, 1) == 0) rows[atomicAdd(count + 1, 1)] = (int)grow;
}
#define LIST_OUTPUT(epi, grow, col) \
    list_output((epi).chk_list, (epi).chk_count, (epi).chk_rflag, (epi).chk_rows, (epi).chk_cap, (grow), (col))

// Work unit u -> tile t, part, and its K stages [kbeg, kend) (see the work-unit comment in gemm_3x).
__device__ __forceinline__ void decode_unit(int u, int split_from, int kparts, int kpc, int nk, int& t, int& part,
                                            int& kbeg, int& kend) {
    if (u < split_from) {
        t = u;
        part = 0;
        kbeg = 0;
        kend = nk;
    } else {
        const int v = u - split_from;
        const int j = v / kparts;
        t = split_from + j;
        part = v - j * kparts;
        kbeg = part * kpc;
        kend = min(nk, kbeg + kpc);
    }
}

template <int BN, int STAGES, bool FUSED, bool F16, bool PAIR, int RB = ROW_BYTES>
__global__ void __maxnreg__(kLaunchRegs)
    gemm_3x(const __grid_constant__ CUtensorMap map_xhi, const __grid_constant__ CUtensorMap map_xlo,
                const __grid_constant__ CUtensorMap map_yhi, const __grid_constant__ CUtensorMap map_ylo,
                const __grid_constant__ CUtensorMap map_bias, float* __restrict__ r, int M, int N, int Kp, int64_t ldr, int* status, const Epi epi,
                int seg_kb, int first_kb, int batch, int kparts, int kpc, int split_from, float* __restrict__ part_out,
                float* __restrict__ tail_out, int stall) {
    pdl_begin();
    using C = Cfg<BN, STAGES, PAIR, RB>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* ring = smem;
    uint64_t* full = (uint64_t*)(smem + STAGES * C::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint64_t* bias_full = drain + 1;  // one per epilogue warp
    uint32_t* tmem_slot = (uint32_t*)(bias_full + kEpiWarps);
    uint8_t* bias_smem = smem + STAGES * C::STAGE_BYTES + 1024;  // 1024-aligned for the 128B swizzle
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // a pair computes 256-row tiles: CTA `rank` owns rows [128*rank, 128*rank + 128) of each
    // and loads Y's rows [BN/2*rank, BN/2*rank + BN/2) of its column block
    constexpr int TM = PAIR ? 2 * BM : BM;
    const uint32_t rank = PAIR ? cluster_rank() : 0;
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // this CTA's (pair's) tile stream
    const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int num_m = (M + TM - 1) / TM;
    const int num_n = (N + BN - 1) / BN;
    const int tiles_per_batch = num_m * num_n;
    const int tiles = tiles_per_batch * batch;  // batch b's operands start at rows b*M (X) and b*N (Y)
    constexpr int KE = RB / (F16 ? 2 : 4);       // K elements per ring stage
    const int nk = Kp / KE;
    // Work units: tiles [0, split_from) whole, one unit each; tiles [split_from, tiles) cut into
    // kparts units of kpc K stages (kparts > 1, one batch, no fused epilogue).  split_from == 0:
    // split K for products with few tiles, parts in part_out as [part][M][N]; split_from > 0: only
    // the tiles of a last, partly filled wave are split, parts in tail_out as [tile][part][TM][BN].
    // Either way the parts are summed afterwards in a fixed order.
    const int work = split_from + (tiles - split_from) * kparts;
    Abort ab{abort_flag, status};

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], PAIR ? 2 * kEpiWarps : 32 * kEpiWarps);  // a pair: one arrive per warp
        }
        mbar_init(drain, 1);
        for (int e = 0; e < kEpiWarps; ++e) mbar_init(&bias_full[e], 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        if constexpr (PAIR) {  // warp 1 of both CTAs: each gets the same columns in its own TMEM
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(tmem_slot)),
                         "r"((uint32_t)C::TMEM_COLS));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(tmem_slot)),
                         "r"((uint32_t)C::TMEM_COLS));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();  // barriers of both CTAs are initialised before any remote use
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp < kEpiWarp0) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
      if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_xhi) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_xlo) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_yhi) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_ylo) : "memory");
            uint32_t it = 0;
            for (int u = unit; u < work; u += units) {
                int t, part, kbeg, kend;
                decode_unit(u, split_from, kparts, kpc, nk, t, part, kbeg, kend);
                int mb, nb;
                const int bt = t / tiles_per_batch;
                tile_coords(t - bt * tiles_per_batch, num_m, num_n, mb, nb);
                const int xrow = bt * M + mb * TM + (int)rank * BM;
                const int yrow = bt * N + nb * BN + (int)rank * (BN / 2) * (PAIR ? 1 : 0);
                for (int kb = kbeg; kb < kend; ++kb, ++it) {
                    const uint32_t s = it % STAGES, round = it / STAGES;
                    // stall (a test of the bounded waits): the first wait is for a phase that
                    // nothing completes, so it expires before any copy or MMA is issued
                    const uint32_t want = ((round & 1) ^ 1) ^ (stall && it == 0 ? 1u : 0u);
                    if (!mbar_wait(&empty[s], want, ab, 1)) goto done;
                    uint8_t* st = ring + s * C::STAGE_BYTES;
                    if constexpr (PAIR) {
                        // both CTAs' loads complete on the leader's full barrier, which expects both
                        const uint32_t fb = mapa_rank(smem_u32(&full[s]), 0);
                        if (rank == 0) mbar_expect_tx(&full[s], 2 * C::STAGE_BYTES);
                        tma_load_2d_pair(&map_xhi, fb, st, kb * KE, xrow);
                        tma_load_2d_pair(&map_xlo, fb, st + C::A_BYTES, kb * KE, xrow);
                        tma_load_2d_pair(&map_yhi, fb, st + 2 * C::A_BYTES, kb * KE, yrow);
                        tma_load_2d_pair(&map_ylo, fb, st + 2 * C::A_BYTES + C::B_BYTES, kb * KE, yrow);
                    } else {
                        mbar_expect_tx(&full[s], C::STAGE_BYTES);
                        tma_load_2d(&map_xhi, &full[s], st, kb * KE, xrow);
                        tma_load_2d(&map_xlo, &full[s], st + C::A_BYTES, kb * KE, xrow);
                        tma_load_2d(&map_yhi, &full[s], st + 2 * C::A_BYTES, kb * KE, yrow);
                        tma_load_2d(&map_ylo, &full[s], st + 2 * C::A_BYTES + C::B_BYTES, kb * KE, yrow);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {  // ---- MMA issuer (a pair's leader): one TMEM accumulator per K segment, two in flight
            constexpr uint32_t idesc = idesc_3x(BN, F16, TM);
            uint32_t it = 0, gseg = 0;
            for (int u = unit; u < work; u += units) {
                int t, part, kbeg, kend;
                decode_unit(u, split_from, kparts, kpc, nk, t, part, kbeg, kend);
                for (int kb0 = kbeg, sl = first_kb; kb0 < kend; kb0 += sl, sl = seg_kb, ++gseg) {
                    const uint32_t b = gseg & 1, bround = gseg >> 1;
                    if (!mbar_wait(&acc_empty[b], (bround & 1) ^ 1, ab, 2)) goto done;
                    tc_fence_after();
                    const uint32_t d = tmem_base + b * BN;
                    const int kb1 = min(kb0 + sl, kend);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const uint32_t s = it % STAGES, round = it / STAGES;
                        if (!mbar_wait(&full[s], round & 1, ab, 3)) goto done;
                        tc_fence_after();
                        const uint32_t base = smem_u32(ring + s * C::STAGE_BYTES);
#pragma unroll
                        for (int kk = 0; kk < RB / 32; ++kk) {  // one MMA consumes 32 bytes of K
                            const uint64_t xhi = sw_desc<RB>(base + kk * 32);
                            const uint64_t xlo = sw_desc<RB>(base + C::A_BYTES + kk * 32);
                            const uint64_t yhi = sw_desc<RB>(base + 2 * C::A_BYTES + kk * 32);
                            const uint64_t ylo = sw_desc<RB>(base + 2 * C::A_BYTES + C::B_BYTES + kk * 32);
                            umma<F16, PAIR>(d, xlo, yhi, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                            umma<F16, PAIR>(d, xhi, ylo, idesc, 1);
                            umma<F16, PAIR>(d, xhi, yhi, idesc, 1);
                        }
                        if constexpr (PAIR) umma_commit_pair(&empty[s]);  // frees the stage in both CTAs
                        else umma_commit(&empty[s]);
                    }
                    if constexpr (PAIR) umma_commit_pair(&acc_full[b]);
                    else umma_commit(&acc_full[b]);
                }
            }
        }
      }
    } else {  // ---- epilogue warps: TMEM lanes 32*(warp%4) .. +31, columns [h*BN/2, (h+1)*BN/2)
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kEpiRegs));
        constexpr int HC = BN / 2;   // columns per thread
        const int q = warp & 3;
        const int h = (warp - kEpiWarp0) >> 2;
        const int ew = warp - kEpiWarp0;  // this warp's bias staging slot and barrier
        uint8_t* bbuf = bias_smem + ew * 4096;
        uint32_t bphase = 0;
        const bool vec = ((ldr & 3) == 0) && ((((uintptr_t)r) & 15) == 0);
        uint32_t gseg = 0;
        for (int u = unit; u < work; u += units) {
            int t, part, kbeg, kend;
            decode_unit(u, split_from, kparts, kpc, nk, t, part, kbeg, kend);
            // output: a whole tile goes to r; a split tile's part to part_out (every tile split,
            // split_from == 0) or to tail_out (only the last wave's tiles split)
            const bool tail = split_from > 0 && t >= split_from;
            float* const rb = (kparts > 1 && split_from == 0) ? part_out + (int64_t)part * M * N : r;
            int mb, nb;
            const int bt = t / tiles_per_batch;
            tile_coords(t - bt * tiles_per_batch, num_m, num_n, mb, nb);
            const int mrow = mb * TM + (int)rank * BM;  // this CTA's first row of the tile
            if constexpr (FUSED) {
                // bring this thread's bias row slice toward L2 now; it is read after the last segment
                const int prow = mrow + q * 32 + lane;
                if (epi.bias && prow < M) {
                    const float* pb = epi.bias + (int64_t)prow * N + nb * BN + h * HC;
#pragma unroll
                    for (int j = 0; j < HC; j += 32)
                        if (nb * BN + h * HC + j < N) asm volatile("prefetch.global.L2 [%0];" ::"l"(pb + j));
                }
            }
            const int row0 = mrow + q * 32;  // this warp's first row
            const int colh = nb * BN + h * HC;
            // the bias chunk of 32 columns goes through shared memory when the map covers it
            auto stage_bias = [&](int cb) {
                if (lane == 0) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier reads of the slot
                    mbar_expect_tx(&bias_full[ew], 32 * 32 * 4);
                    tma_load_2d(&map_bias, &bias_full[ew], bbuf, cb, row0);
                }
            };
            const bool map_ok = FUSED && epi.bias_map && vec && row0 < M;
            bool staged0 = false;
            // segment sums are added in registers with round-to-nearest
            float sum[HC];
            for (int kb0 = kbeg, sl = first_kb; kb0 < kend; kb0 += sl, sl = seg_kb, ++gseg) {
                const uint32_t b = gseg & 1, bround = gseg >> 1;
                if (map_ok && !staged0 && kb0 + sl >= kend && colh + 32 <= N) {
                    stage_bias(colh);  // the first chunk loads while the last segment accumulates
                    staged0 = true;
                }
                if (!mbar_wait(&acc_full[b], bround & 1, ab, 4)) goto done;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < HC / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + b * BN + h * HC + c * 32, v);
                    if (kb0 == kbeg) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[c * 32 + j] = __uint_as_float(v[j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) sum[c * 32 + j] = __fadd_rn(sum[c * 32 + j], __uint_as_float(v[j]));
                    }
                }
                tc_fence_before();
                if constexpr (PAIR) {  // release the accumulator on the leader's barrier, once per warp
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_rank(smem_u32(&acc_empty[b]), 0));
                } else {
                    mbar_arrive(&acc_empty[b]);
                }
            }
            if (row0 >= M) continue;  // the whole warp is past the last row
            const int row = row0 + lane;
            const bool row_ok = row < M;
            const int rowc = row_ok ? row : row0;  // lanes past M compute but store nothing
            int ea = 0;
            if constexpr (F16) ea = epi.row_exp[(int64_t)bt * M + rowc];
            if constexpr (FUSED) {
                // Every 32-column chunk passes through this warp's 4 KB slot.  Phase A: lane = row
                // writes its unscaled sums (plus the staged bias) in place, in the slot's 128-byte
                // swizzle.  Phase B: a rolled loop walks the slot four rows at a time, eight lanes to
                // a row, through the unstaged bias, GELU, the tf32 split and the stores, so each
                // row's 128 bytes leave as one coalesced store and the per-element code exists once.
                // (a fused product is one unsplit product: its tiles write r, batch 0)
                const bool bvec = ((((uintptr_t)epi.bias) & 15) == 0) && (N & 3) == 0;
                const int cc = (lane & 7) * 4;
                const uint32_t sbuf = smem_u32(bbuf);
#pragma unroll
                for (int c = 0; c < HC / 32; ++c) {
                    const int cb = colh + c * 32;
                    if (cb >= N) break;
                    const bool full = cb + 32 <= N;
                    const bool staged = map_ok && full;
                    if (staged) {
                        if (c > 0 || !staged0) stage_bias(cb);
                        if (!mbar_wait(&bias_full[ew], bphase, ab, 5)) goto done;
                        bphase ^= 1;
                    }
                    const int* ce = F16 ? epi.col_exp + (int64_t)bt * N + cb : nullptr;
                    float thr = 0.0f;  // floor check of this lane's row (threshold on the scaled sums)
                    if constexpr (F16) {  // every lane takes part in the chunk's reduction
                        const int cm = chunk_floor(epi.col_floor, cb, N, lane);
                        thr = row_ok ? floor_threshold(__ldg(epi.row_floor + row) + cm) : 0.0f;
                    }
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const uint32_t slot = sbuf + lane * 128 + (((j >> 2) ^ (lane & 7)) << 4);
                        float a[4] = {sum[c * 32 + j], sum[c * 32 + j + 1], sum[c * 32 + j + 2], sum[c * 32 + j + 3]};
                        if constexpr (F16) {
                            const bool lo4 = fabsf(a[0]) < thr || fabsf(a[1]) < thr || fabsf(a[2]) < thr || fabsf(a[3]) < thr;
                            if (__any_sync(0xffffffffu, lo4)) {  // rare: listed for the exact recomputation
#pragma unroll
                                for (int u = 0; u < 4; ++u)
                                    if (fabsf(a[u]) < thr && cb + j + u < N) LIST_OUTPUT(epi, row, cb + j + u);
                            }
                        }
                        if constexpr (F16) {  // undo the operands' power-of-two scaling
                            int e[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u) e[u] = cb + j + u < N ? __ldg(ce + j + u) : 0;
#pragma unroll
                            for (int u = 0; u < 4; ++u) a[u] = unscale(a[u], ea + e[u]);
                        }
                        if (staged) {
                            const float4 b4 = lds4(slot);
                            a[0] = __fadd_rn(a[0], b4.x);
                            a[1] = __fadd_rn(a[1], b4.y);
                            a[2] = __fadd_rn(a[2], b4.z);
                            a[3] = __fadd_rn(a[3], b4.w);
                        }
                        sts4(slot, a[0], a[1], a[2], a[3]);
                    }
                    __syncwarp();
#pragma unroll 1
                    for (int i = 0; i < 8; ++i) {
                        const int rr = 4 * i + (lane >> 3);
                        const int grow = row0 + rr;
                        const int col = cb + cc;
                        const float4 s4 = lds4(sbuf + rr * 128 + (((lane & 7) ^ (rr & 7)) << 4));
                        if (grow >= M || col >= N) continue;
                        const bool vq = vec && col + 4 <= N;
                        const bool gbias = epi.bias && !staged;
                        float a[4] = {s4.x, s4.y, s4.z, s4.w};
                        if (epi.bias_zero) {
#pragma unroll
                            for (int u = 0; u < 4; ++u) a[u] = __fadd_rn(a[u], 0.0f);
                        }
                        if (gbias) {
                            const float* q = epi.bias + (int64_t)grow * N + col;
                            if (vq && bvec) {
                                const float4 b4 = __ldcs((const float4*)q);
                                a[0] = __fadd_rn(a[0], b4.x);
                                a[1] = __fadd_rn(a[1], b4.y);
                                a[2] = __fadd_rn(a[2], b4.z);
                                a[3] = __fadd_rn(a[3], b4.w);
                            } else {
#pragma unroll
                                for (int u = 0; u < 4; ++u)
                                    if (col + u < N) a[u] = __fadd_rn(a[u], q[u]);
                            }
                        }
                        if (epi.act == 1) {
#pragma unroll
                            for (int u = 0; u < 4; ++u) a[u] = gelu_lane(a[u]);
                        }
                        if constexpr (!F16) {  // the host admits a split output only for N % 32 == 0
                            if (epi.out_hi) {
                                float hh[4], ll[4];
#pragma unroll
                                for (int u = 0; u < 4; ++u) {
                                    hh[u] = rna_tf32_dev(a[u]);
                                    ll[u] = rna_tf32_dev(a[u] - hh[u]);
                                }
                                float* oh = epi.out_hi + (int64_t)grow * epi.kp_out + col;
                                float* ol = epi.out_lo + (int64_t)grow * epi.kp_out + col;
                                if (vq) {
                                    *(float4*)oh = make_float4(hh[0], hh[1], hh[2], hh[3]);
                                    *(float4*)ol = make_float4(ll[0], ll[1], ll[2], ll[3]);
                                } else {
#pragma unroll
                                    for (int u = 0; u < 4; ++u) {
                                        if (col + u < N) {
                                            oh[u] = hh[u];
                                            ol[u] = ll[u];
                                        }
                                    }
                                }
                            }
                        }
                        float* o = r + (int64_t)grow * ldr + col;
                        if (vq) {
                            *(float4*)o = make_float4(a[0], a[1], a[2], a[3]);
                        } else {
#pragma unroll
                            for (int u = 0; u < 4; ++u)
                                if (col + u < N) o[u] = a[u];
                        }
                    }
                    // every lane is done with the slot before the next chunk's bias load refills it
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                }
                continue;
            }
            float* out = tail ? tail_out + ((int64_t)((t - split_from) * kparts + part) * TM + (rowc - mb * TM)) * BN +
                                    (colh - nb * BN)
                              : rb + (int64_t)bt * M * ldr + (int64_t)rowc * ldr + colh;
            const bool vec_u = tail || vec;  // the tail buffer's rows are BN floats, 16-byte aligned
            // whole-tile outputs get the floor check here; split tiles' parts after their sum
            const bool check = F16 && !tail && !(kparts > 1 && split_from == 0);
#pragma unroll
            for (int c = 0; c < HC / 32; ++c) {
                float* v = sum + c * 32;
                const int cb = colh + c * 32;
                const bool full = cb + 32 <= N;
                if (F16 && check && cb < N) {  // warp-uniform: the chunk's largest column count needs every lane
                    const int cm = chunk_floor(epi.col_floor + (int64_t)bt * N, cb, N, lane);
                    const float thr = row_ok ? floor_threshold(__ldg(epi.row_floor + (int64_t)bt * M + row) + cm) : 0.0f;
                    uint32_t low = 0;
#pragma unroll
                    for (int j = 0; j < 32; ++j) low |= (fabsf(v[j]) < thr ? 1u : 0u) << j;
                    for (uint32_t m = low; m; m &= m - 1) {
                        const int j = __ffs(m) - 1;
                        if (cb + j < N) LIST_OUTPUT(epi, (int64_t)bt * M + row, cb + j);
                    }
                }
                const bool fast = full && vec_u && (!F16 || ((((int64_t)bt * N) & 3) == 0));
                if (fast) {
                    // one float4 at a time through unscale and store: short live ranges keep the
                    // 128-column segment sum in registers without spills
                    const int* ce = F16 ? epi.col_exp + (int64_t)bt * N + cb : nullptr;
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float a[4] = {v[j], v[j + 1], v[j + 2], v[j + 3]};
                        if constexpr (F16) {  // undo the operands' power-of-two scaling
                            const int4 e4 = *(const int4*)(ce + j);
                            a[0] = unscale(a[0], ea + e4.x);
                            a[1] = unscale(a[1], ea + e4.y);
                            a[2] = unscale(a[2], ea + e4.z);
                            a[3] = unscale(a[3], ea + e4.w);
                        }
                        if (row_ok) {
                            const float4 o4 = make_float4(a[0], a[1], a[2], a[3]);
                            // the product's result is not read again here: evict it first, so it
                            // displaces the split operands of later tiles as little as possible
                            if (tail) *(float4*)(out + c * 32 + j) = o4;
                            else __stcs((float4*)(out + c * 32 + j), o4);
                        }
                    }
                    continue;
                }
                if (!row_ok) continue;
                // ragged edge or unaligned result: element by element
                const int* ce = F16 ? epi.col_exp + (int64_t)bt * N + cb : nullptr;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (cb + j >= N) break;
                    float a = v[j];
                    if constexpr (F16) a = unscale(a, ea + ce[j]);
                    out[c * 32 + j] = a;
                }
            }
        }
    }
done:
    __syncthreads();
    if (warp == 1 && lane == 0 && rank == 0 && *abort_flag) {
        // let MMAs still in flight finish before the accumulators are released
        if constexpr (PAIR) umma_commit_pair_local(drain);
        else umma_commit(drain);
        for (uint32_t i = 0; i < kWaitLimit && !mbar_test(drain, 0); ++i) __nanosleep(64);
    }
    if constexpr (PAIR) {  // neither CTA leaves while its peer may still signal it or write its TMEM
        tc_fence_before();
        cluster_sync();
    }
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                         "r"((uint32_t)C::TMEM_COLS));
        else
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
    pdl_begin();
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
    pdl_begin();
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

// f16 split with power-of-two scaling: a row (or column) with largest magnitude
// m = f * 2^E, f in [1, 2), is multiplied by 2^(14 - E) so it peaks in [2^14, 2^15),
// inside f16's range with 2^-24 absolute resolution left for the lo parts.
__device__ __forceinline__ int scale_exp(float amax) {
    if (!(amax > 0.0f) || isinf(amax)) return 0;  // zero row, or inf/NaN that no scaling keeps finite
    int e = 14 - ilogbf(amax);
    return e > 126 ? 126 : e;  // 2^e stays a normal f32
}

__device__ __forceinline__ uint32_t pack2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// Returns whether v is a floor element (below).
__device__ __forceinline__ bool split_f16(float v, float scale, __half& hi, __half& lo) {
    const float s = __fmul_rn(v, scale);  // exact: a power of two (unless it underflows)
    hi = __float2half_rn(s);
    lo = __float2half_rn(__fsub_rn(s, __half2float(hi)));  // the difference is exact in f32
    return v != 0.0f && fabsf(s) < 0.125f;
}


// X[M][K] -> hi/lo [M][Kp] f16 and row_exp[M]: one warp per row, the row read twice
// (the second read hits L2).
__global__ void __launch_bounds__(256) split_rows_f16(const float* __restrict__ x, __half* __restrict__ hi,
                                                      __half* __restrict__ lo, int* __restrict__ row_exp, int64_t M,
                                                      int64_t K, int64_t Kp, int* __restrict__ row_floor) {
    pdl_begin();
    const int64_t m = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (m >= M) return;
    const float* xr = x + m * K;
    const bool vec = (K % 4 == 0) && ((((uintptr_t)x) & 15) == 0);
    float amax = 0.0f;
    if (vec) {
        for (int64_t k = lane * 4; k < K; k += 128) {
            const float4 t = *(const float4*)(xr + k);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
        }
    } else {
        for (int64_t k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(xr[k]));
    }
    // (fmaxf skips NaN: a NaN element stays NaN through the split and its outputs are NaN)
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const int e = scale_exp(amax);
    const float scale = __int_as_float((127 + e) << 23);
    if (lane == 0) row_exp[m] = e;
    __half* hr = hi + m * Kp;
    __half* lr = lo + m * Kp;
    int nf = 0;
    for (int64_t k = lane * 4; k < Kp; k += 128) {
        float v[4];
        if (vec && k + 4 <= K) {
            const float4 t = __ldcs((const float4*)(xr + k));
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = (k + j < K) ? xr[k + j] : 0.0f;
        }
        __half h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) nf += split_f16(v[j], scale, h[j], l[j]);
        *(uint2*)(hr + k) = make_uint2(pack2(h[0], h[1]), pack2(h[2], h[3]));
        *(uint2*)(lr + k) = make_uint2(pack2(l[0], l[1]), pack2(l[2], l[3]));
    }
    nf = __reduce_add_sync(0xffffffffu, nf);
    if (lane == 0) row_floor[m] = nf;
}

// The same split for rows of up to 128*V elements (V <= 8): one warp per row, the row in
// registers, eight rows per CTA.
template <int V>
__global__ void __launch_bounds__(256) split_rows_f16_warp(const float* __restrict__ x, __half* __restrict__ hi,
                                                           __half* __restrict__ lo, int* __restrict__ row_exp,
                                                           int64_t M, int64_t K, int64_t Kp, int* __restrict__ row_floor) {
    pdl_begin();
    const int64_t m = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (m >= M) return;
    const float* xr = x + m * K;
    const bool vec = (K % 4 == 0) && ((((uintptr_t)x) & 15) == 0);
    float4 v[V];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int64_t k = ((int64_t)i * 32 + lane) * 4;
        if (vec && k + 4 <= K) {
            v[i] = __ldcs((const float4*)(xr + k));
        } else {
            v[i].x = k < K ? xr[k] : 0.0f;
            v[i].y = k + 1 < K ? xr[k + 1] : 0.0f;
            v[i].z = k + 2 < K ? xr[k + 2] : 0.0f;
            v[i].w = k + 3 < K ? xr[k + 3] : 0.0f;
        }
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const int e = scale_exp(amax);
    const float scale = __int_as_float((127 + e) << 23);
    if (lane == 0) row_exp[m] = e;
    __half* hr = hi + m * Kp;
    __half* lr = lo + m * Kp;
    int nf = 0;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int64_t k = ((int64_t)i * 32 + lane) * 4;
        if (k >= Kp) break;
        __half h[4], l[4];
        nf += split_f16(v[i].x, scale, h[0], l[0]);
        nf += split_f16(v[i].y, scale, h[1], l[1]);
        nf += split_f16(v[i].z, scale, h[2], l[2]);
        nf += split_f16(v[i].w, scale, h[3], l[3]);
        *(uint2*)(hr + k) = make_uint2(pack2(h[0], h[1]), pack2(h[2], h[3]));
        *(uint2*)(lr + k) = make_uint2(pack2(l[0], l[1]), pack2(l[2], l[3]));
    }
    nf = __reduce_add_sync(0xffffffffu, nf);
    if (lane == 0) row_floor[m] = nf;
}

// The same split for rows of up to 1024*V elements: one 256-thread CTA per row keeps the row
// in registers (V float4 per thread), so X is read from HBM once.
template <int V>
__global__ void __launch_bounds__(256) split_rows_f16_block(const float* __restrict__ x, __half* __restrict__ hi,
                                                            __half* __restrict__ lo, int* __restrict__ row_exp,
                                                            int64_t K, int64_t Kp, int* __restrict__ row_floor) {
    pdl_begin();
    __shared__ float wmax[8];
    __shared__ int wfloor[8];
    const int64_t m = blockIdx.x;
    const float* xr = x + m * K;
    const bool vec = (K % 4 == 0) && ((((uintptr_t)x) & 15) == 0);
    float4 v[V];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int64_t k = ((int64_t)i * 256 + threadIdx.x) * 4;
        if (vec && k + 4 <= K) {
            v[i] = __ldcs((const float4*)(xr + k));
        } else {
            v[i].x = k < K ? xr[k] : 0.0f;
            v[i].y = k + 1 < K ? xr[k + 1] : 0.0f;
            v[i].z = k + 2 < K ? xr[k + 2] : 0.0f;
            v[i].w = k + 3 < K ? xr[k + 3] : 0.0f;
        }
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) amax = fmaxf(amax, wmax[w]);
    const int e = scale_exp(amax);
    const float scale = __int_as_float((127 + e) << 23);
    if (threadIdx.x == 0) row_exp[m] = e;
    __half* hr = hi + m * Kp;
    __half* lr = lo + m * Kp;
    int nf = 0;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int64_t k = ((int64_t)i * 256 + threadIdx.x) * 4;
        if (k >= Kp) break;
        __half h[4], l[4];
        nf += split_f16(v[i].x, scale, h[0], l[0]);
        nf += split_f16(v[i].y, scale, h[1], l[1]);
        nf += split_f16(v[i].z, scale, h[2], l[2]);
        nf += split_f16(v[i].w, scale, h[3], l[3]);
        *(uint2*)(hr + k) = make_uint2(pack2(h[0], h[1]), pack2(h[2], h[3]));
        *(uint2*)(lr + k) = make_uint2(pack2(l[0], l[1]), pack2(l[2], l[3]));
    }
    nf = __reduce_add_sync(0xffffffffu, nf);
    if ((threadIdx.x & 31) == 0) wfloor[threadIdx.x >> 5] = nf;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += wfloor[w];
        row_floor[m] = t;
    }
}

// Split-K: r = part[0] + part[1] + ... in that order (f32 adds, so the result does not
// depend on which parts finished first), then a fused layer's bias, GELU and tf32 operand
// split exactly as the GEMM epilogue (and the separate ADD and GELU ops) apply them.
// Floor check of a finished (unscaled) output at flat index i of an [M][N] result, batch 0 (the
// same bound as the GEMM epilogue's, in unscaled units).  M * N < 2^31 for the products that
// reach it (split along K: fewer tiles than CTAs; last-wave tails: under 8 waves of tiles).
__device__ __forceinline__ void check_output(const Epi& epi, float c, int64_t row, int64_t col, int64_t N) {
    const int n = epi.row_floor[row] + epi.col_floor[col];
    if (n > 0 && fabsf(c) < unscale(floor_threshold(n), epi.row_exp[row] + epi.col_exp[col]))
        LIST_OUTPUT(epi, row, col);
}

__global__ void __launch_bounds__(256) sum_parts(float* __restrict__ r, const float* __restrict__ part, int64_t M,
                                                 int64_t N, int parts, const Epi epi) {
    pdl_begin();
    const int64_t n = M * N;
    if (!epi.out_hi && (n & 3) == 0 && ((((uintptr_t)r) & 15) == 0) && (!epi.bias || ((((uintptr_t)epi.bias) & 15) == 0))) {
        for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n / 4; i += (int64_t)gridDim.x * 256) {
            float4 a = __ldcs((const float4*)part + i);
            for (int p = 1; p < parts; ++p) {
                const float4 b = __ldcs((const float4*)(part + (int64_t)p * n) + i);
                a.x = __fadd_rn(a.x, b.x); a.y = __fadd_rn(a.y, b.y);
                a.z = __fadd_rn(a.z, b.z); a.w = __fadd_rn(a.w, b.w);
            }
            if (epi.chk_count) {
                const uint32_t e0 = (uint32_t)(4 * i), row = e0 / (uint32_t)N;
                uint32_t col = e0 - row * (uint32_t)N;
                const float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t rr = col < (uint32_t)N ? row : row + 1, cc = col < (uint32_t)N ? col : col - (uint32_t)N;
                    check_output(epi, v[u], rr, cc, N);
                    ++col;
                }
            }
            if (epi.bias) {
                const float4 b = ((const float4*)epi.bias)[i];
                a.x = __fadd_rn(a.x, b.x); a.y = __fadd_rn(a.y, b.y);
                a.z = __fadd_rn(a.z, b.z); a.w = __fadd_rn(a.w, b.w);
            } else if (epi.bias_zero) {
                a.x = __fadd_rn(a.x, 0.0f); a.y = __fadd_rn(a.y, 0.0f);
                a.z = __fadd_rn(a.z, 0.0f); a.w = __fadd_rn(a.w, 0.0f);
            }
            if (epi.act == 1) {
                a.x = gelu_lane(a.x); a.y = gelu_lane(a.y); a.z = gelu_lane(a.z); a.w = gelu_lane(a.w);
            }
            ((float4*)r)[i] = a;
        }
        return;
    }
    for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
        float a = __ldcs(part + i);
        for (int p = 1; p < parts; ++p) a = __fadd_rn(a, __ldcs(part + (int64_t)p * n + i));
        if (epi.chk_count) {
            const uint32_t row = (uint32_t)i / (uint32_t)N;
            check_output(epi, a, row, (uint32_t)i - row * (uint32_t)N, N);
        }
        if (epi.bias) a = __fadd_rn(a, epi.bias[i]);
        else if (epi.bias_zero) a = __fadd_rn(a, 0.0f);
        if (epi.act == 1) a = gelu_lane(a);
        r[i] = a;
        if (epi.out_hi) {
            const int64_t row = (uint32_t)i / (uint32_t)N, col = i - row * N;  // M * N < 2^31
            const float hh = rna_tf32_dev(a);
            epi.out_hi[row * epi.kp_out + col] = hh;
            epi.out_lo[row * epi.kp_out + col] = rna_tf32_dev(a - hh);
        }
    }
}

// Last-wave split: r = part[0] + part[1] + ... (in that order) over the tiles [split_from, ...)
// whose K range was cut into kparts units; parts laid out [tile][part][TM][BN].  One thread per
// four consecutive columns of a tile row.
template <int BN>
__global__ void __launch_bounds__(256) sum_tail(float* __restrict__ r, const float* __restrict__ tail, int M, int N,
                                                int TM, int num_m, int num_n, int split_from, int kparts,
                                                const Epi chk) {
    pdl_begin();
    const int per_tile = TM * BN / 4;
    const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
    const int j = (int)(idx / per_tile);
    const int local = (int)(idx - (int64_t)j * per_tile);
    const int lr = local / (BN / 4), lc = (local - lr * (BN / 4)) * 4;
    const int t = split_from + j, tpb = num_m * num_n;
    const int bt = t / tpb;  // batch b's result starts at row b*M
    int mb, nb;
    tile_coords(t - bt * tpb, num_m, num_n, mb, nb);
    const int row = mb * TM + lr, col = nb * BN + lc;
    if (row >= M || col >= N) return;
    r += (int64_t)bt * M * N;
    const float* p = tail + ((int64_t)j * kparts * TM + lr) * BN + lc;
    float4 a = __ldcs((const float4*)p);
    for (int q = 1; q < kparts; ++q) {
        const float4 b = __ldcs((const float4*)(p + (int64_t)q * TM * BN));
        a.x = __fadd_rn(a.x, b.x); a.y = __fadd_rn(a.y, b.y);
        a.z = __fadd_rn(a.z, b.z); a.w = __fadd_rn(a.w, b.w);
    }
    if (chk.chk_count) {  // f16 split: the floor check of the split tiles' outputs
        const float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (col + u >= N) break;
            const int64_t grow = (int64_t)bt * M + row, gcol = (int64_t)bt * N + col + u;
            const int nf = chk.row_floor[grow] + chk.col_floor[gcol];
            if (nf > 0 && fabsf(v[u]) < unscale(floor_threshold(nf), chk.row_exp[grow] + chk.col_exp[gcol]))
                LIST_OUTPUT(chk, grow, col + u);
        }
    }
    float* o = r + (int64_t)row * N + col;
    if ((N & 3) == 0 && (((uintptr_t)r) & 15) == 0 && col + 4 <= N) {
        *(float4*)o = a;
    } else {
        o[0] = a.x;
        if (col + 1 < N) o[1] = a.y;
        if (col + 2 < N) o[2] = a.z;
        if (col + 3 < N) o[3] = a.w;
    }
}

// Column maxima of Y[b][K][N] as f32 bits (|y| compares as an unsigned integer; NaN above inf).
// A block covers 128 columns x 128 rows: 32 lanes take four consecutive columns each (one
// float4 per row, so a warp reads 512 contiguous bytes), 8 warps take every 8th row; the warps'
// maxima meet in shared memory and one atomicMax per column leaves the block.
constexpr int kColMaxRows = 128;
__global__ void __launch_bounds__(256) col_absmax(const float* __restrict__ y, unsigned* __restrict__ cmax, int64_t K,
                                                  int64_t N) {
    pdl_begin();
    __shared__ unsigned part[8][128];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t n = (int64_t)blockIdx.x * 128 + lane * 4;
    y += (int64_t)blockIdx.z * K * N;
    cmax += (int64_t)blockIdx.z * N;
    const int64_t k0 = (int64_t)blockIdx.y * kColMaxRows, k1 = k0 + kColMaxRows < K ? k0 + kColMaxRows : K;
    const bool vec = (N % 4 == 0) && ((((uintptr_t)y) & 15) == 0);
    unsigned m0 = 0, m1 = 0, m2 = 0, m3 = 0;
    if (n < N) {
        if (vec) {
#pragma unroll 4
            for (int64_t k = k0 + w; k < k1; k += 8) {
                const float4 v = __ldg((const float4*)(y + k * N + n));
                m0 = max(m0, __float_as_uint(v.x) & 0x7FFFFFFFu);
                m1 = max(m1, __float_as_uint(v.y) & 0x7FFFFFFFu);
                m2 = max(m2, __float_as_uint(v.z) & 0x7FFFFFFFu);
                m3 = max(m3, __float_as_uint(v.w) & 0x7FFFFFFFu);
            }
        } else {
            for (int64_t k = k0 + w; k < k1; k += 8) {
                const float* p = y + k * N + n;
                m0 = max(m0, __float_as_uint(__ldg(p)) & 0x7FFFFFFFu);
                if (n + 1 < N) m1 = max(m1, __float_as_uint(__ldg(p + 1)) & 0x7FFFFFFFu);
                if (n + 2 < N) m2 = max(m2, __float_as_uint(__ldg(p + 2)) & 0x7FFFFFFFu);
                if (n + 3 < N) m3 = max(m3, __float_as_uint(__ldg(p + 3)) & 0x7FFFFFFFu);
            }
        }
    }
    part[w][lane * 4] = m0;
    part[w][lane * 4 + 1] = m1;
    part[w][lane * 4 + 2] = m2;
    part[w][lane * 4 + 3] = m3;
    __syncthreads();
    if (threadIdx.x < 128) {
        const int64_t c = (int64_t)blockIdx.x * 128 + threadIdx.x;
        unsigned m = part[0][threadIdx.x];
#pragma unroll
        for (int i = 1; i < 8; ++i) m = max(m, part[i][threadIdx.x]);
        if (c < N) atomicMax(cmax + c, m);
    }
}

// Y[K][N] -> hi/lo transposed [N][Kp] f16 through a 64 (k) x 64 (n) shared tile, scaled per
// column.  Each thread loads four float4 of Y's rows and stores eight consecutive k of one
// column as one 16-byte word of hi and one of lo.  col_exp[N] is written by the first k-block.
__global__ void __launch_bounds__(256) split_cols_t_f16(const float* __restrict__ y, const unsigned* __restrict__ cmax,
                                                        __half* __restrict__ hi, __half* __restrict__ lo,
                                                        int* __restrict__ col_exp, int64_t K, int64_t N, int64_t Kp,
                                                        int* __restrict__ col_floor) {
    pdl_begin();
    __shared__ float tile[64][65];
    __shared__ float scl[64];
    y += (int64_t)blockIdx.z * K * N;
    hi += (int64_t)blockIdx.z * N * Kp;
    lo += (int64_t)blockIdx.z * N * Kp;
    cmax += (int64_t)blockIdx.z * N;
    col_exp += (int64_t)blockIdx.z * N;
    const int64_t k0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
    if (threadIdx.x < 64 && n0 + threadIdx.x < N) {
        const unsigned b = cmax[n0 + threadIdx.x];
        const int e = b > 0x7F800000u ? 0 : scale_exp(__uint_as_float(b));
        scl[threadIdx.x] = __int_as_float((127 + e) << 23);
        if (blockIdx.y == 0) col_exp[n0 + threadIdx.x] = e;
    }
    // 64 rows of 16 float4: thread t takes float4 t & 15 of rows (t >> 4) + 16 i
    const bool vec = (N % 4 == 0) && ((((uintptr_t)y) & 15) == 0);
    const int c4 = (threadIdx.x & 15) * 4, r0 = threadIdx.x >> 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int j = r0 + 16 * i;
        const int64_t k = k0 + j, n = n0 + c4;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k < K) {
            const float* py = y + k * N + n;
            if (vec && n + 4 <= N) {
                v = __ldcs((const float4*)py);  // Y's last read: evict first, keep the split halves in L2
            } else {
                v.x = n < N ? py[0] : 0.0f;
                v.y = n + 1 < N ? py[1] : 0.0f;
                v.z = n + 2 < N ? py[2] : 0.0f;
                v.w = n + 3 < N ? py[3] : 0.0f;
            }
        }
        tile[j][c4] = v.x;
        tile[j][c4 + 1] = v.y;
        tile[j][c4 + 2] = v.z;
        tile[j][c4 + 3] = v.w;
    }
    __syncthreads();
    // 64 columns x 8 runs of 8 k: two per thread; a warp writes four columns' 128-byte runs
#pragma unroll
    for (int q2 = 0; q2 < 2; ++q2) {
        const int item = threadIdx.x + 256 * q2;
        const int j = item >> 3, kc = (item & 7) * 8;
        const int64_t n = n0 + j, k = k0 + kc;
        if (n < N && k < Kp) {  // Kp is a multiple of 32: k .. k + 7 are all inside
            const float sc = scl[j];
            __half h[8], l[8];
            int nf = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) nf += split_f16(tile[kc + q][j], sc, h[q], l[q]);
            // floor elements, counted per column (zeroed before the split; the partial counts of
            // every k-block add up)
            if (nf) atomicAdd(col_floor + (int64_t)blockIdx.z * N + n, nf);
            *(uint4*)(hi + n * Kp + k) = make_uint4(pack2(h[0], h[1]), pack2(h[2], h[3]), pack2(h[4], h[5]),
                                                    pack2(h[6], h[7]));
            *(uint4*)(lo + n * Kp + k) = make_uint4(pack2(l[0], l[1]), pack2(l[2], l[3]), pack2(l[4], l[5]),
                                                    pack2(l[6], l[7]));
        }
    }
}

// The outputs listed by the floor check, recomputed exactly: one CTA per output, thread t summing
// the f32 products (exact in double) over k = t, t + 256, ... in double (four loads in flight),
// then a fixed tree over the CTA; rounded once, then a fused layer's bias and GELU as the
// epilogue applies them.  When more outputs were listed than the list holds, every output of
// the listed rows is recomputed.  Either way the result depends only on the inputs.
__global__ void __launch_bounds__(256) fix_outputs(const float* __restrict__ x, const float* __restrict__ y,
                                                   float* __restrict__ r, int64_t M, int64_t K, int64_t N,
                                                   const Epi epi) {
    pdl_begin();
    __shared__ double part[8];
    const int listed = epi.chk_count[0];
    const bool by_rows = listed > epi.chk_cap;
    const int64_t items = by_rows ? (int64_t)epi.chk_count[1] * N : (int64_t)listed;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
        int64_t gi, j;
        if (by_rows) {
            gi = epi.chk_rows[it / N];
            j = it - (it / N) * N;
        } else {
            const int2 p = epi.chk_list[it];
            gi = p.x;
            j = p.y;
        }
        const int64_t bt = gi / M;
        const float* xr = x + gi * K;
        const float* yc = y + bt * K * N + j;
        double acc = 0.0;
#pragma unroll 4
        for (int64_t k = threadIdx.x; k < K; k += 256) acc += (double)__ldg(xr + k) * (double)__ldg(yc + k * N);
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
        if (lane == 0) part[w] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = part[0];
#pragma unroll
            for (int q = 1; q < 8; ++q) t += part[q];
            float c = (float)t;
            if (epi.bias) c = __fadd_rn(c, epi.bias[gi * N + j]);
            else if (epi.bias_zero) c = __fadd_rn(c, 0.0f);
            if (epi.act == 1) c = gelu_lane(c);
            r[gi * N + j] = c;
        }
        __syncthreads();  // part[] is rewritten by the next output
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

// 2-D map over a [rows][Kp] array of f32 or f16, box = box_rows x rb bytes (64 or 128), swizzled
// by rb bytes.
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t kp, int box_rows, bool f16,
              int rb = ROW_BYTES) {
    auto fn = encode_fn();
    if (!fn) return false;
    const int es = f16 ? 2 : 4;
    cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(kp * es)};
    cuuint32_t box[2] = {(cuuint32_t)(rb / es), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    rb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Scratch of one product: split operands, and for the f16 split the row/column
// exponents and column maxima.  Sized for the tf32 split, which needs the most.
constexpr int kCheckCap = 1 << 16;  // outputs the floor check lists individually

struct Layout {
    int64_t kp;
    size_t xhi, xlo, yhi, ylo, rexp, cexp, cmax, parts, tail, total;
    // f16 split's floor check: [cmax | cfloor | counters | chk_rflag] is cleared by one memset
    size_t cfloor, counters, chk_rflag, clear_bytes, rfloor, chk_rows, chk_list;
    int kparts;  // split-K factor of an unfused single product (1: none)
    int kpc;     // its ring stages per part
};

// The last wave of a persistent product of 1 to 8 waves: when the tiles left after the full
// waves fill at most half of the CTAs (pairs), split each of them along K into parts (at least 4
// ring stages each, at most 8 parts, parts x tiles <= CTAs), so that wave finishes in about
// 1/parts of a tile time.
struct TailPlan {
    int parts = 1, kpc = 0, split_from = 0;
};

constexpr int kStagesPair = 6;  // 32 KB stages: A rows and half of Y's rows per CTA

// Tensor-core products use CTA pairs (M = 256 per MMA, half of Y per CTA, so each SM
// stages a third less per k-step) unless MAG_CUDA_TC_PAIR=0.
bool use_pairs() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("MAG_CUDA_TC_PAIR");
        v = (e && *e == '0') ? 0 : 1;
    }
    return v == 1;
}

// Pair products of the f16 split stage 128 bytes of K per row (64 f16, 128-byte swizzle, three
// 64 KB stages): half the TMA rows of 64-byte stages for the same bytes, 2-4 % faster on every
// size measured.  MAG_CUDA_TC_ROW128=0 (unfused products) and MAG_CUDA_TC_ROW128_FUSED=0 (fused
// layers) return to 64-byte rows.
bool wide_rows(bool fused) {
    static int v[2] = {-2, -2};
    if (v[fused] == -2) {
        const char* e = getenv(fused ? "MAG_CUDA_TC_ROW128_FUSED" : "MAG_CUDA_TC_ROW128");
        v[fused] = (e && *e == '0') ? 0 : 1;
    }
    return v[fused] == 1;
}

// Pairs compute 256-row tiles: products with fewer rows run one CTA per 128-row tile.
bool pair_for(int64_t M, bool f16) { return f16 && use_pairs() && M >= 2 * BM; }

// Split K when a single product has too few tiles to occupy the GPU: up to 16 parts of
// at least 4 ring stages each, so tiles x parts approaches the number of CTAs (pairs).
int choose_parts(int64_t M, int64_t K, int64_t N, bool f16) {
    const bool pair = pair_for(M, f16);
    const int64_t tm = pair ? 256 : 128;
    const int64_t tiles = ((M + tm - 1) / tm) * ((N + 255) / 256);
    const int64_t units = pair ? sm_count() / 2 : sm_count();
    const int64_t kp = (K + KPAD - 1) / KPAD * KPAD;
    const int64_t nk = kp / (f16 ? BK16 : BK);
    int64_t parts = units / (tiles ? tiles : 1);
    if (parts > nk / 4) parts = nk / 4;
    if (parts > 16) parts = 16;
    if (parts < 2) return 1;
    const int64_t kpc = (nk + parts - 1) / parts;
    return (int)((nk + kpc - 1) / kpc);  // no empty part
}

TailPlan plan_tail(int64_t B, int64_t M, int64_t K, int64_t N, bool f16, int ke = 0) {
    TailPlan tp;
    const bool pair = pair_for(M, f16);
    const int64_t tm = pair ? 2 * BM : BM;
    const int64_t tiles = B * ((M + tm - 1) / tm) * ((N + 255) / 256);
    const int64_t units = pair ? sm_count() / 2 : sm_count();
    const int64_t kp = (K + KPAD - 1) / KPAD * KPAD;
    const int64_t nk = kp / (ke ? ke : (f16 ? BK16 : BK));
    // (from 8 waves on, a mostly empty last wave costs under 1/16 of the product)
    if (tiles <= units || tiles >= 8 * units) return tp;
    const int64_t rem = tiles % units;
    if (rem == 0 || 2 * rem > units) return tp;
    int64_t parts = units / rem;
    if (parts > 8) parts = 8;
    if (parts > nk / 4) parts = nk / 4;
    if (parts < 2) return tp;
    const int64_t kpc = (nk + parts - 1) / parts;
    parts = (nk + kpc - 1) / kpc;
    if (parts < 2) return tp;
    tp.parts = (int)parts;
    tp.kpc = (int)kpc;
    tp.split_from = (int)(tiles - rem);
    return tp;
}

size_t tail_bytes(int64_t B, int64_t M, int64_t K, int64_t N, bool f16) {
    const TailPlan tp = plan_tail(B, M, K, N, f16);
    if (tp.parts < 2) return 0;
    const int64_t tm = pair_for(M, f16) ? 2 * BM : BM;
    const int64_t tiles = B * ((M + tm - 1) / tm) * ((N + 255) / 256);
    return (size_t)((tiles - tp.split_from) * tp.parts * tm * 256 * 4);
}

// Scratch of B products of M x K times K x N (operands of all batches split into one array each).
Layout layout(int64_t B, int64_t M, int64_t K, int64_t N, bool f16) {
    Layout l;
    l.kp = round_up(K < 1 ? 1 : K, KPAD);
    const int es = f16 ? 2 : 4;
    const int64_t rows = B * M, cols = B * N;
    size_t xs = (size_t)round_up(rows * l.kp * es, 1024), ys = (size_t)round_up(cols * l.kp * es, 1024);
    l.xhi = 0;
    l.xlo = xs;
    l.yhi = 2 * xs;
    l.ylo = 2 * xs + ys;
    l.rexp = 2 * xs + 2 * ys;
    l.cexp = l.rexp + (size_t)round_up(rows * 4, 256);
    l.cmax = l.cexp + (size_t)round_up(cols * 4, 256);
    l.cfloor = l.cmax + (size_t)round_up(cols * 4, 256);
    l.counters = l.cfloor + (size_t)round_up(cols * 4, 256);
    l.chk_rflag = l.counters + 256;
    l.clear_bytes = l.chk_rflag + (size_t)round_up(rows * 4, 256) - l.cmax;
    l.rfloor = l.chk_rflag + (size_t)round_up(rows * 4, 256);
    l.chk_rows = l.rfloor + (size_t)round_up(rows * 4, 256);
    l.chk_list = l.chk_rows + (size_t)round_up(rows * 4, 256);
    l.parts = l.chk_list + (size_t)kCheckCap * 8;
    l.kparts = B == 1 ? choose_parts(M, K, N, f16) : 1;
    {
        const int64_t nk = l.kp / (f16 ? BK16 : BK);
        l.kpc = (int)((nk + l.kparts - 1) / l.kparts);
    }
    l.tail = l.parts + (l.kparts > 1 ? (size_t)round_up((int64_t)l.kparts * M * N * 4, 256) : 0);
    l.total = l.tail + (l.kparts > 1 ? 0 : (size_t)round_up((int64_t)tail_bytes(B, M, K, N, f16), 256));
    return l;
}

size_t scratch_bytes(int64_t B, int64_t M, int64_t K, int64_t N) {
    const size_t a = layout(B, M, K, N, false).total, b = layout(B, M, K, N, true).total;
    return a > b ? a : b;
}

constexpr int kBN = 256;
constexpr int kStages = 4;

// K per TMEM accumulation segment (MAG_CUDA_TC_SEGMENT; default 512 for the f16 split,
// 256 for tf32).  Tensor-core f32 accumulation truncates; restarting the accumulator
// every segment and adding segments with round-to-nearest bounds that error by the
// segment length instead of K (at K = 16384: 2.0e-6 of max|C| for f16 at 512, 2.1e-6 for
// tf32 at 256).  Longer segments give the epilogue more time per accumulator.  0 = one
// segment spanning K.  Returned in ring stages.
int segment_kb(bool f16, int ke = 0) {
    static int k = -2;
    if (k == -2) {
        const char* e = getenv("MAG_CUDA_TC_SEGMENT");
        k = (e && *e) ? atoi(e) : -1;
    }
    const int seg = k == -1 ? (f16 ? 512 : 256) : k;
    if (!ke) ke = f16 ? BK16 : BK;
    return seg <= 0 ? (1 << 30) : (seg + ke - 1) / ke;
}

// K of a tile's first segment (MAG_CUDA_TC_SEGMENT_FIRST; default: the segment length), in ring
// stages.  The epilogue's stores of one tile overlap the MMAs of the next tile's first two
// segments, so a long first segment hides them while short later segments keep the truncation
// of the tensor-core accumulator small.
int segment_first_kb(bool f16, int ke = 0) {
    static int k = -2;
    if (k == -2) {
        const char* e = getenv("MAG_CUDA_TC_SEGMENT_FIRST");
        k = (e && *e) ? atoi(e) : -1;
    }
    if (k == -1) return segment_kb(f16, ke);
    if (!ke) ke = f16 ? BK16 : BK;
    return k <= 0 ? (1 << 30) : (k + ke - 1) / ke;
}

// 2-D map over the fused epilogue's row-major [M][N] f32 bias, box 32 x 32, 128-byte swizzle.
bool make_bias_map(CUtensorMap* m, const float* bias, int64_t M, int64_t N) {
    auto fn = encode_fn();
    if (!fn || (N & 3) || (((uintptr_t)bias) & 15)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)(N * 4)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)bias, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// MAG_CUDA_TC_TEST_STALL=1 makes the GEMM's first wait one that never completes (read at each
// launch): a test of the bounded waits and the status word without any fault.
int test_stall() {
    const char* e = getenv("MAG_CUDA_TC_TEST_STALL");
    return e && e[0] == '1';
}

// A kernel of a product's chain launched as a programmatic dependent of the previous kernel on the
// stream (it waits in the kernel, pdl_begin, before touching memory).
template <typename... KArgs, typename... Args>
cudaError_t launch_dep(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <bool FUSED, bool F16, bool PAIR, int RB = ROW_BYTES>
int launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, const CUtensorMap& d,
                const CUtensorMap& bias, float* r, int64_t M, int64_t N, int64_t kp, int* status, const Epi& epi,
                int64_t B, cudaStream_t st, int kparts, int kpc, int split_from, float* part_out, float* tail_out) {
    // 128-byte rows double a stage: three of them fit beside the barriers
    constexpr int STG = RB == 128 ? 3 : PAIR ? (FUSED ? kStagesPair : kStagesPair + 1) : kStages;
    using C = Cfg<kBN, STG, PAIR, RB>;
    static_assert(!FUSED || C::SMEM_BIAS <= 227 * 1024, "ring and bias staging must fit shared memory");
    constexpr int KE = RB / (F16 ? 2 : 4);
    auto kern = gemm_3x<kBN, STG, FUSED, F16, PAIR, RB>;
    const int smem = FUSED ? C::SMEM_BIAS : C::SMEM;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    const int64_t tm = PAIR ? 2 * BM : BM;
    const int64_t all = B * ((M + tm - 1) / tm) * ((N + kBN - 1) / kBN);
    if (kparts <= 1) split_from = (int)all;
    const int64_t tiles = split_from + (all - split_from) * kparts;  // work units
    if constexpr (!PAIR) {
        const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
        return (int)launch_dep(kern, dim3(grid), dim3(kThreads), (size_t)smem, st, a, b, c, d, bias, r, (int)M, (int)N,
                               (int)kp, (int64_t)N, status, epi, segment_kb(F16, KE), segment_first_kb(F16, KE), (int)B,
                               kparts, kpc, split_from, part_out, tail_out, test_stall());
    } else {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = 1;  // the occupancy query below takes the cluster shape only
        cfg.gridDim = dim3((unsigned)sm_count());
        int max_clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg) != cudaSuccess || max_clusters <= 0) {
            cudaGetLastError();
            max_clusters = sm_count() / 2;
        }
        const int64_t clusters = tiles < max_clusters ? tiles : max_clusters;
        cfg.gridDim = dim3((unsigned)(2 * clusters));
        cfg.numAttrs = 2;  // and a programmatic dependent of the split kernels
        e = cudaLaunchKernelEx(&cfg, kern, a, b, c, d, bias, r, (int)M, (int)N, (int)kp, (int64_t)N, status, epi,
                               segment_kb(F16, KE), segment_first_kb(F16, KE), (int)B, kparts, kpc, split_from, part_out,
                               tail_out, test_stall());
        return (int)e;
    }
}

}  // namespace

extern "C" int mcu_matmul_tc_supported(void) {
    if (getenv("MAG_CUDA_NO_TC")) return 0;
    return encode_fn() != nullptr;
}

extern "C" size_t mcu_matmul_tc_scratch_bytes(int64_t M, int64_t K, int64_t N) { return scratch_bytes(1, M, K, N); }

extern "C" int mcu_matmul_tc_kernels(int64_t M, int64_t K, int64_t N, int f16, int flags) {
    // flags: bit 0 = X arrives split by the previous layer (tf32), bit 1 = fused epilogue
    const int split = f16 ? 3 : ((flags & 1) ? 1 : 2);  // operand split kernels
    const bool parts = choose_parts(M, K, N, f16 != 0) > 1;
    const bool tail = !parts && !(flags & 2) && plan_tail(1, M, K, N, f16 != 0).parts > 1;
    return split + 1 + (parts || tail ? 1 : 0) + (f16 ? 1 : 0);  // f16: the floor check's recomputation
}

static int launch_tc(float* r, const float* x, const float* y, int64_t B, int64_t M, int64_t K, int64_t N,
                     void* scratch, int* status, cudaStream_t st, const mcu_tc_epilogue* ep, int f16);

extern "C" int mcu_launch_matmul_tc_ex(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                                       void* scratch, int* status, cudaStream_t st, const mcu_tc_epilogue* ep,
                                       int f16) {
    return launch_tc(r, x, y, 1, M, K, N, scratch, status, st, ep, f16);
}

extern "C" size_t mcu_matmul_tc_batched_scratch_bytes(int64_t B, int64_t M, int64_t K, int64_t N) {
    return scratch_bytes(B, M, K, N);
}

extern "C" int mcu_matmul_tc_batched_kernels(int64_t B, int64_t M, int64_t K, int64_t N, int f16) {
    return (f16 ? 4 : 2) + 1 + (plan_tail(B, M, K, N, f16 != 0).parts > 1 ? 1 : 0);
}

extern "C" int mcu_launch_matmul_tc_batched(float* r, const float* x, const float* y, int64_t B, int64_t M, int64_t K,
                                            int64_t N, void* scratch, int* status, cudaStream_t st, int f16) {
    return launch_tc(r, x, y, B, M, K, N, scratch, status, st, nullptr, f16);
}

static int launch_tc(float* r, const float* x, const float* y, int64_t B, int64_t M, int64_t K, int64_t N,
                     void* scratch, int* status, cudaStream_t st, const mcu_tc_epilogue* ep, int f16) {
    if (B <= 0 || M <= 0 || N <= 0) return (int)cudaSuccess;
    if (B * M >= (1ll << 31) || B * N >= (1ll << 31) || K > MCU_TC_MAX_K || !scratch) return (int)cudaErrorInvalidValue;
    if (B > 1 && ep) return (int)cudaErrorInvalidValue;
    const Layout l = layout(B, M, K, N, f16 != 0);
    char* base = (char*)scratch;
    void* xhi = base + l.xhi;
    void* xlo = base + l.xlo;
    void* yhi = base + l.yhi;
    void* ylo = base + l.ylo;
    int* rexp = (int*)(base + l.rexp);
    int* cexp = (int*)(base + l.cexp);
    unsigned* cmax = (unsigned*)(base + l.cmax);
    // the tf32 split can take X already split by the previous layer's epilogue; the f16
    // split scales whole rows, so it always splits X itself
    const bool presplit = !f16 && ep && ep->a_hi && ep->a_lo;
    int* rfloor = (int*)(base + l.rfloor);
    int* cfloor = (int*)(base + l.cfloor);
    if (presplit) {
        xhi = (void*)ep->a_hi;
        xlo = (void*)ep->a_lo;
    } else if (f16) {
        // column maxima, floor counts of column chunks, the check's counters and row flags start at zero
        cudaError_t e = cudaMemsetAsync(cmax, 0, l.clear_bytes, st);
        if (e != cudaSuccess) return (int)e;
        __half *h16 = (__half*)xhi, *l16 = (__half*)xlo;
        const unsigned rows = (unsigned)(B * M);
        const unsigned wrows = (rows + 7) / 8;
        if (l.kp <= 128) split_rows_f16_warp<1><<<wrows, 256, 0, st>>>(x, h16, l16, rexp, B * M, K, l.kp, rfloor);
        else if (l.kp <= 256) split_rows_f16_warp<2><<<wrows, 256, 0, st>>>(x, h16, l16, rexp, B * M, K, l.kp, rfloor);
        else if (l.kp <= 512) split_rows_f16_warp<4><<<wrows, 256, 0, st>>>(x, h16, l16, rexp, B * M, K, l.kp, rfloor);
        else if (l.kp <= 1024) split_rows_f16_warp<8><<<wrows, 256, 0, st>>>(x, h16, l16, rexp, B * M, K, l.kp, rfloor);
        else if (l.kp <= 2048) split_rows_f16_block<2><<<rows, 256, 0, st>>>(x, h16, l16, rexp, K, l.kp, rfloor);
        else if (l.kp <= 4096) split_rows_f16_block<4><<<rows, 256, 0, st>>>(x, h16, l16, rexp, K, l.kp, rfloor);
        else if (l.kp <= 8192) split_rows_f16_block<8><<<rows, 256, 0, st>>>(x, h16, l16, rexp, K, l.kp, rfloor);
        else split_rows_f16<<<(unsigned)((B * M + 7) / 8), 256, 0, st>>>(x, h16, l16, rexp, B * M, K, l.kp, rfloor);
    } else {
        int64_t n = B * M * (l.kp / 4);  // X of all batches is one (B*M) x K row-major matrix
        int64_t g = (n + 255) / 256;
        if (g > 8 * sm_count()) g = 8 * sm_count();
        split_rows<<<(unsigned)g, 256, 0, st>>>(x, (float*)xhi, (float*)xlo, B * M, K, l.kp);
    }
    if (f16) {
        dim3 gm((unsigned)((N + 127) / 128), (unsigned)((K + kColMaxRows - 1) / kColMaxRows), (unsigned)B);
        cudaError_t e = launch_dep(col_absmax, gm, dim3(256), 0, st, y, cmax, K, N);
        if (e != cudaSuccess) return (int)e;
        dim3 grid((unsigned)((N + 63) / 64), (unsigned)((l.kp + 63) / 64), (unsigned)B);
        e = launch_dep(split_cols_t_f16, grid, dim3(256), 0, st, y, (const unsigned*)cmax, (__half*)yhi, (__half*)ylo, cexp,
                       K, N, l.kp, cfloor);
        if (e != cudaSuccess) return (int)e;
    } else {
        dim3 grid((unsigned)((N + 31) / 32), (unsigned)(l.kp / 32), (unsigned)B);
        cudaError_t e = launch_dep(split_cols_t, grid, dim3(256), 0, st, y, (float*)yhi, (float*)ylo, K, N, l.kp);
        if (e != cudaSuccess) return (int)e;
    }
    CUtensorMap mxh, mxl, myh, myl;
    const bool h = f16 != 0;
    const bool pair = pair_for(M, h);
    const int yrows = pair ? kBN / 2 : kBN;
    // unfused, unsplit pair products may stage 128 bytes of K per row (64 f16)
    const bool any_fused = ep && (ep->bias || ep->bias_zero || ep->act || (ep->out_hi && !f16));
    const bool wide = h && pair && (B == 1 ? l.kparts : 1) == 1 && l.kp % 64 == 0 && wide_rows(any_fused);
    const int rb = wide ? 128 : ROW_BYTES;
    if (!make_map(&mxh, xhi, B * M, l.kp, BM, h, rb) || !make_map(&mxl, xlo, B * M, l.kp, BM, h, rb) ||
        !make_map(&myh, yhi, B * N, l.kp, yrows, h, rb) || !make_map(&myl, ylo, B * N, l.kp, yrows, h, rb))
        return (int)cudaErrorInvalidValue;
    Epi chk{};  // the f16 split's floor check (no fields for tf32)
    chk.row_exp = rexp;
    chk.col_exp = cexp;
    if (f16) {
        chk.row_floor = rfloor;
        chk.col_floor = cfloor;
        chk.chk_list = (int2*)(base + l.chk_list);
        chk.chk_count = (int*)(base + l.counters);
        chk.chk_rflag = (int*)(base + l.chk_rflag);
        chk.chk_rows = (int*)(base + l.chk_rows);
        chk.chk_cap = kCheckCap;
    }
    Epi epi = chk;
    const bool fused = ep && (ep->bias || ep->bias_zero || ep->act || (ep->out_hi && !f16));
    const int kparts = B == 1 ? l.kparts : 1;
    float* part = kparts > 1 ? (float*)(base + l.parts) : nullptr;
    // f16 split: the listed outputs recomputed exactly, after every other kernel of the product
    auto fix = [&]() -> int {
        if (!f16) return (int)cudaSuccess;
        Epi fe = chk;
        if (fused) {
            fe.bias = ep->bias;
            fe.bias_zero = ep->bias_zero;
            fe.act = ep->act;
        }
        return (int)launch_dep(fix_outputs, dim3((unsigned)(4 * sm_count())), dim3(256), 0, st, x, y, r, M, K, N, fe);
    };
    if (fused && kparts == 1) {
        if (!f16 && ep->out_hi && (N % 32 != 0 || ep->kp_out != round_up(N, KPAD))) return (int)cudaErrorInvalidValue;
        epi.bias = ep->bias;
        epi.bias_zero = ep->bias ? 0 : ep->bias_zero;
        epi.out_hi = f16 ? nullptr : ep->out_hi;
        epi.out_lo = f16 ? nullptr : ep->out_lo;
        epi.kp_out = ep->kp_out;
        epi.act = ep->act;
        CUtensorMap mb;
        memset(&mb, 0, sizeof(mb));
        epi.bias_map = ep->bias && make_bias_map(&mb, ep->bias, M, N);
        int rc;
        if (wide)
            rc = launch_gemm<true, true, true, 128>(mxh, mxl, myh, myl, mb, r, M, N, l.kp, status, epi, B, st, 1, 0, 0,
                                                    nullptr, nullptr);
        else if (pair)
            rc = launch_gemm<true, true, true>(mxh, mxl, myh, myl, mb, r, M, N, l.kp, status, epi, B, st, 1, 0, 0,
                                               nullptr, nullptr);
        else
            rc = f16 ? launch_gemm<true, true, false>(mxh, mxl, myh, myl, mb, r, M, N, l.kp, status, epi, B, st, 1, 0,
                                                      0, nullptr, nullptr)
                     : launch_gemm<true, false, false>(mxh, mxl, myh, myl, mb, r, M, N, l.kp, status, epi, B, st, 1, 0,
                                                       0, nullptr, nullptr);
        return rc ? rc : fix();
    }
    Epi plain = chk;
    // an unfused single product whose last wave is mostly empty splits that wave's tiles along K
    int gparts = kparts, gkpc = l.kpc, split_from = 0;
    float* tail = nullptr;
    if (kparts == 1 && !fused) {
        const TailPlan tp = plan_tail(B, M, K, N, h, wide ? 64 : 0);  // no more parts than the buffer holds
        if (tp.parts > 1) {
            gparts = tp.parts;
            gkpc = tp.kpc;
            split_from = tp.split_from;
            tail = (float*)(base + l.tail);
        }
    }
    int rc = wide ? launch_gemm<false, true, true, 128>(mxh, mxl, myh, myl, mxh, r, M, N, l.kp, status, plain, B, st,
                                                        gparts, gkpc, split_from, part, tail)
         : pair ? launch_gemm<false, true, true>(mxh, mxl, myh, myl, mxh, r, M, N, l.kp, status, plain, B, st, gparts,
                                                 gkpc, split_from, part, tail)
         : f16 ? launch_gemm<false, true, false>(mxh, mxl, myh, myl, mxh, r, M, N, l.kp, status, plain, B, st, gparts,
                                                 gkpc, split_from, part, tail)
               : launch_gemm<false, false, false>(mxh, mxl, myh, myl, mxh, r, M, N, l.kp, status, plain, B, st, gparts,
                                                  gkpc, split_from, part, tail);
    if (rc) return rc;
    if (tail) {
        const int tm = pair ? 2 * BM : BM;
        const int num_m = (int)((M + tm - 1) / tm), num_n = (int)((N + kBN - 1) / kBN);
        const int64_t ntail = B * num_m * num_n - split_from;
        const int64_t blocks = ntail * tm * kBN / 4 / 256;
        rc = (int)launch_dep(sum_tail<kBN>, dim3((unsigned)blocks), dim3(256), 0, st, r, (const float*)tail, (int)M,
                             (int)N, tm, num_m, num_n, split_from, gparts, chk);
        return rc ? rc : fix();
    }
    if (kparts == 1) return fix();
    // a fused layer whose product was split: its epilogue runs after the sum, in the same order
    Epi fe = chk;
    if (fused) {
        if (!f16 && ep->out_hi && (N % 32 != 0 || ep->kp_out != round_up(N, KPAD))) return (int)cudaErrorInvalidValue;
        fe.bias = ep->bias;
        fe.bias_zero = ep->bias ? 0 : ep->bias_zero;
        fe.act = ep->act;
        fe.out_hi = f16 ? nullptr : ep->out_hi;
        fe.out_lo = f16 ? nullptr : ep->out_lo;
        fe.kp_out = ep->kp_out;
    }
    const int64_t n = M * N;
    int64_t g = (n + 255) / 256;
    if (g > 8 * sm_count()) g = 8 * sm_count();
    rc = (int)launch_dep(sum_parts, dim3((unsigned)(g ? g : 1)), dim3(256), 0, st, r, (const float*)part, M, N, kparts,
                         fe);
    return rc ? rc : fix();
}

extern "C" int mcu_launch_matmul_tc(float* r, const float* x, const float* y, int64_t M, int64_t K, int64_t N,
                                    void* scratch, int* status, cudaStream_t st, int f16) {
    return mcu_launch_matmul_tc_ex(r, x, y, M, K, N, scratch, status, st, nullptr, f16);
}
