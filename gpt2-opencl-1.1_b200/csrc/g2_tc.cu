// g2_tc.cu -- tensor-core GEMM (tcgen05 + TMA) for many-row passes.
//
// out[r][n] = epilogue(sum_k X[r][k] W[k][n]) for the R rows of a prefill
// (the runtime matmul of prefill, main.c:593-684 via launch_matmul
// main.c:1518, with its bias / gelu / add_inplace / split_kv epilogues,
// main.c:1759-1786) or of a batched decode step (one token of each of R
// sequences).
//
// Mapping onto tcgen05.mma (cta_group::1, M = 128):
//   * MMA A = W^T: 128 output features x K.  The Conv1D weights [K][N] are
//     feature-contiguous, which is the MN-major operand layout, so they are
//     used in place: TMA boxes of 128 bytes of features x BK rows, 128-byte
//     swizzle.
//   * MMA B = X^T: K x BN rows, K-major (X [R][K] rows are K-contiguous).
//   * D (fp32) lives in tensor memory: 128 lanes (features) x BN columns
//     (rows); the epilogue warps read it with tcgen05.ld and store
//     feature-contiguous, coalesced rows.
// One CTA computes a 128 x BN tile over a range of K (split-K when the tiles
// alone cannot fill the SMs); partial tiles go to a scratch buffer and one
// small kernel sums the splits in order and applies the epilogue, so results
// do not depend on timing.
//
// Warp roles: warp 0 lane 0 issues the TMA loads of a STAGES-deep ring,
// warp 1 lane 0 issues the MMAs (tcgen05.commit releases a stage when the
// MMAs that read it complete), all four warps run the epilogue.  For 3xTF32
// the weights are either two tf32 copies in HBM (hi and lo, both loaded by
// TMA), or, with TcArgs::wsplit, the fp32 weights themselves: the tile then
// arrives once and warps 2 and 3 split it in shared memory into hi =
// x truncated to tf32 (in place) and lo = x - hi before the MMAs read the
// stage (half the HBM bytes, more shared-memory traffic).  Every wait
// is bounded; on expiry the kernel records G2_ERR_TIMEOUT in *err, drains its
// own copies, frees its tensor memory and returns.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "g2_device.cuh"
#include "g2_tc.h"
#include "gpt2b200.h"

namespace g2 {

namespace {

constexpr int kThreads = 256;   // 8 warps: all run the epilogue, warps 2-7 split fp32 weights (wsplit)
constexpr int kSplitWarps = 6;
typedef unsigned long long u64;

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ u64 gtime() {
    u64 t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(u64 *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(u64 *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(u64 *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ bool mbar_try(u64 *b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of parity `parity`, at most 1 s.
__device__ __forceinline__ bool mbar_wait(u64 *b, unsigned parity) {
    if (mbar_try(b, parity)) return true;
    const u64 limit = gtime() + 1000000000ull;
    for (;;) {
        if (mbar_try(b, parity)) return true;
        if (gtime() > limit) return false;
    }
}
// One contiguous bulk copy global -> shared (16-byte aligned, size a multiple of 16), L2 policy `pol`.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, unsigned bytes, u64 *bar, u64 pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, u64 *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<u64>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor (version 1) with a 128-byte swizzle: layout
// type 2 (16-byte granules, 8-row atoms) or, for MN-major 32-bit operands, type 1
// (128-byte swizzle of 32-byte granules, 4-row atoms).
__device__ __forceinline__ u64 sw128_desc(unsigned saddr, unsigned lbo, unsigned sbo, unsigned layout = 2) {
    return (u64)((saddr >> 4) & 0x3FFFu) | ((u64)((lbo >> 4) & 0x3FFFu) << 16) | ((u64)((sbo >> 4) & 0x3FFFu) << 32) |
           (1ull << 46) | ((u64)layout << 61);
}

// Instruction descriptor: D f32; A, B tf32 or f16; A MN-major (Conv1D weights)
// or K-major (AK: rows of wte), B K-major; N = BN, M = 128.
template <int KIND, int BN, bool AK>
__host__ __device__ constexpr unsigned make_idesc() {
    return (1u << 4) | ((KIND == TC_TF32X3 ? 2u : 0u) << 7) | ((KIND == TC_TF32X3 ? 2u : 0u) << 10) |
           ((AK ? 0u : 1u) << 15) | ((unsigned)(BN >> 3) << 17) | ((unsigned)(kTcTileF >> 4) << 24);
}

template <int KIND>
__device__ __forceinline__ void mma(unsigned tmem_d, u64 adesc, u64 bdesc, unsigned idesc, unsigned accum) {
    if (KIND == TC_TF32X3) {
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
    } else {
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
    }
}
__device__ __forceinline__ void mma_commit(u64 *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 tensor-memory lanes.
__device__ __forceinline__ void tmem_ld32(unsigned taddr, float (&v)[32]) {
    unsigned r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// 16 consecutive fp32 columns of this warp's 32 tensor-memory lanes.
__device__ __forceinline__ void tmem_ld16(unsigned taddr, float (&v)[16]) {
    unsigned r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

template <typename WT>
struct TcArgs {
    int N, R;
    int kb_total, kb_per;   // K blocks in total and per split (uniform splits)
    int splits;
    SplitInfo si;           // si.G > 0: balanced split over si.G CTAs (one row tile), else si.splits == splits
    float *part;            // [partials][R][N] when the GEMM is split
    int *err;
    int wsplit;             // 3xTF32 only: the weight map is the fp32 weights, split in shared memory
    const unsigned char *img_hi, *img_lo;   // stage images of the weights (TcWeights), or nullptr
    Epi<WT> e;              // bias / GELU / residual / K,V append, out
    OperandOut op;          // the output also as the next GEMM's operand (row stride N)
};

template <int KIND>
struct TcShape {
    static constexpr int NPASS = KIND == TC_TF32X3 ? 2 : 1;   // hi and lo copies
    static constexpr int ELEM = KIND == TC_TF32X3 ? 4 : 2;
    static constexpr int BK = 128 / ELEM;                      // K per stage: one 128-byte row
    static constexpr int BOX_F = 128 / ELEM;                   // features per weight box
    static constexpr int NBOX = kTcTileF / BOX_F;              // weight boxes per stage and copy
    static constexpr int A_BYTES = kTcTileF * BK * ELEM;       // 16 KB
    static constexpr int KSTEP = KIND == TC_TF32X3 ? 8 : 16;   // K per MMA
    static constexpr int NSTEP = BK / KSTEP;
    // the weights (MN-major A): tf32 needs the 32-byte-granule swizzle (4-row atoms of 512 B)
    static constexpr unsigned A_LAYOUT = KIND == TC_TF32X3 ? 1u : 2u;
    static constexpr unsigned A_SBO = KIND == TC_TF32X3 ? 512u : 1024u;
};

template <int KIND, int BN>
struct TcCfg {
    using S = TcShape<KIND>;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE = S::NPASS * (S::A_BYTES + B_BYTES);
    // Ring stages within 216 KB of shared memory (at most 8).  The fp16 128-row tiles of
    // prefill keep to ~100 KB so that two CTAs share an SM: one's epilogue then overlaps
    // the other's main loop.
    static constexpr int BUDGET = (KIND == TC_F16 && BN == 128) ? 102400 : 221184;
    static constexpr int STAGES = (BUDGET / STAGE) < 8 ? (BUDGET / STAGE) : 8;
    static constexpr size_t SMEM = (size_t)STAGES * STAGE + 1024 + 256;
};

template <int KIND, int BN, typename WT, bool AK>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mw_hi, const __grid_constant__ CUtensorMap mw_lo,
                   const __grid_constant__ CUtensorMap mx_hi, const __grid_constant__ CUtensorMap mx_lo,
                   TcArgs<WT> a) {
    using S = TcShape<KIND>;
    using C = TcCfg<KIND, BN>;
    constexpr int STAGES = C::STAGES;
    // 3xTF32 with wsplit: the weight tile is loaded once (fp32) and split in shared memory.
    const bool kSplitW = KIND == TC_TF32X3 && a.wsplit;
    const int WPASS = kSplitW ? 1 : S::NPASS;                              // weight copies loaded by TMA
    const unsigned kTx = kSplitW ? C::STAGE - S::A_BYTES : C::STAGE;        // TMA bytes per stage
    extern __shared__ unsigned char smem_raw[];
    unsigned char *base =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    u64 *full = reinterpret_cast<u64 *>(base + (size_t)STAGES * C::STAGE);
    u64 *empty = full + STAGES;
    u64 *done = empty + STAGES;
    u64 *conv = done + 1;   // [STAGES]: the stage's weight tile is split (kSplitW)
    unsigned *tslot = reinterpret_cast<unsigned *>(conv + STAGES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // This CTA's work: one segment (tile, first K block, K blocks, partial index), or,
    // under the balanced split, the end of one tile and the start of the next (the
    // planner keeps a share under one tile's K blocks, so never more than two).
    int sf0, sf1, sk0, sk1, sn0, sn1 = 0, sj0, sj1 = 0;   // segments 0 and 1 (scalars, no local-memory arrays)
    const int r0 = a.si.G ? 0 : blockIdx.y * BN;
    if (a.si.G) {
        const long long U = a.si.U, KB = a.si.KB;
        const long long u0 = (long long)blockIdx.x * U / a.si.G, u1 = (long long)(blockIdx.x + 1) * U / a.si.G;
        const int t0 = (int)(u0 / KB);
        const long long e0 = min(u1, (long long)(t0 + 1) * KB);
        sf0 = t0 * kTcTileF;
        sk0 = (int)(u0 - t0 * KB);
        sn0 = (int)(e0 - u0);
        sj0 = (int)blockIdx.x - a.si.cta_of((long long)t0 * KB);
        sf1 = sf0 + kTcTileF;
        sk1 = 0;
        sn1 = (int)(u1 - e0);   // the next tile's first K blocks, if any (partial 0 of that tile)
    } else {
        sf0 = blockIdx.x * kTcTileF;
        sk0 = blockIdx.z * a.kb_per;
        sn0 = min(a.kb_per, a.kb_total - sk0);   // >= 1 (the planner guarantees it)
        sj0 = blockIdx.z;
        sf1 = sf0;
        sk1 = 0;
    }
    const int nkb = sn0 + sn1;
    const unsigned tcols = a.si.G ? 2u * BN : (unsigned)BN;   // one BN-column accumulator per segment

    if (threadIdx.x == 0) {
        // the TMA descriptors (kernel parameters) are fetched while the barriers are set up
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<u64>(&mw_hi)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<u64>(&mx_hi)) : "memory");
        if (KIND == TC_TF32X3) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<u64>(&mw_lo)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<u64>(&mx_lo)) : "memory");
        }
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&conv[s], kSplitWarps);   // one arrival per splitting warp
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                     "r"(tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tmem = *tslot;

    if (threadIdx.x == 0) {
        // ---- TMA producer ----
        // The weights are no earlier kernel's output: the first stages' weight
        // tiles are requested before waiting for the previous kernel, the rows
        // (its output) after.
        const int pre = nkb < STAGES ? nkb : STAGES;
        u64 pol;   // weights are read once per pass: L2 evict-first
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
        for (int i = 0; i < pre; ++i) {
            unsigned char *st = base + (size_t)i * C::STAGE;
            const int sg = i < sn0 ? 0 : 1, f0 = sg ? sf1 : sf0;
            const int k = ((sg ? sk1 : sk0) + i - (sg ? sn0 : 0)) * S::BK;
            mbar_expect_tx(&full[i], kTx);
#pragma unroll 2
            for (int p = 0; p < WPASS; ++p) {
                if (AK) {
                    tma_load_2d(st + p * S::A_BYTES, p ? &mw_lo : &mw_hi, k, f0, &full[i]);
                } else if (a.img_hi) {   // the stage image: one bulk copy
                    bulk_load(st + p * S::A_BYTES,
                              (p ? a.img_lo : a.img_hi) + ((size_t)(f0 / kTcTileF) * a.kb_total + k / S::BK) * S::A_BYTES,
                              S::A_BYTES, &full[i], pol);
                } else {
#pragma unroll
                    for (int b = 0; b < S::NBOX; ++b)
                        tma_load_2d(st + p * S::A_BYTES + b * (S::BK * 128), p ? &mw_lo : &mw_hi, f0 + b * S::BOX_F,
                                    k, &full[i]);
                }
            }
        }
        pdl_wait();
        pdl_launch();
        for (int i = 0; i < pre; ++i) {
            unsigned char *st = base + (size_t)i * C::STAGE;
            const int sg = i < sn0 ? 0 : 1;
            const int k = ((sg ? sk1 : sk0) + i - (sg ? sn0 : 0)) * S::BK;
#pragma unroll
            for (int p = 0; p < S::NPASS; ++p)
                tma_load_2d(st + S::NPASS * S::A_BYTES + p * C::B_BYTES, p ? &mx_lo : &mx_hi, k, r0, &full[i]);
        }
        int issued = pre;
        for (int i = pre; i < nkb; ++i) {
            const int s = i % STAGES;
            if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1)) {
                atomicCAS(a.err, 0, G2_ERR_TIMEOUT);
                break;
            }
            unsigned char *st = base + (size_t)s * C::STAGE;
            const int sg = i < sn0 ? 0 : 1, f0 = sg ? sf1 : sf0;
            const int k = ((sg ? sk1 : sk0) + i - (sg ? sn0 : 0)) * S::BK;
            mbar_expect_tx(&full[s], kTx);
#pragma unroll 2
            for (int p = 0; p < WPASS; ++p) {
                if (AK) {   // 128 rows x 128 bytes of K in one box
                    tma_load_2d(st + p * S::A_BYTES, p ? &mw_lo : &mw_hi, k, f0, &full[s]);
                } else if (a.img_hi) {
                    bulk_load(st + p * S::A_BYTES,
                              (p ? a.img_lo : a.img_hi) + ((size_t)(f0 / kTcTileF) * a.kb_total + k / S::BK) * S::A_BYTES,
                              S::A_BYTES, &full[s], pol);
                } else {
#pragma unroll
                    for (int b = 0; b < S::NBOX; ++b)
                        tma_load_2d(st + p * S::A_BYTES + b * (S::BK * 128), p ? &mw_lo : &mw_hi, f0 + b * S::BOX_F,
                                    k, &full[s]);
                }
            }
#pragma unroll
            for (int p = 0; p < S::NPASS; ++p)
                tma_load_2d(st + S::NPASS * S::A_BYTES + p * C::B_BYTES, p ? &mx_lo : &mx_hi, k, r0, &full[s]);
            ++issued;
        }
        // every copy issued must land before the CTA may exit
        for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
    } else {
        pdl_wait();
        pdl_launch();
    }
    if (threadIdx.x == 32) {
        // ---- MMA issuer ----
        constexpr unsigned idesc = make_idesc<KIND, BN, AK>();
        for (int i = 0; i < nkb; ++i) {
            const int s = i % STAGES;
            if (!mbar_wait(&full[s], (i / STAGES) & 1) || (kSplitW && !mbar_wait(&conv[s], (i / STAGES) & 1))) {
                atomicCAS(a.err, 0, G2_ERR_TIMEOUT);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const unsigned a_hi = smem_u32(base + (size_t)s * C::STAGE);
            const unsigned b_hi = a_hi + S::NPASS * S::A_BYTES;
            const int sg = i < sn0 ? 0 : 1, ki = i - (sg ? sn0 : 0);   // segment, K block within it
            const unsigned td = tmem + (unsigned)(sg * BN);
#pragma unroll
            for (int j = 0; j < S::NSTEP; ++j) {
                const unsigned ao = AK ? j * S::KSTEP * S::ELEM : j * S::KSTEP * 128, bo = j * S::KSTEP * S::ELEM;
                const u64 ad = AK ? sw128_desc(a_hi + ao, 16, 1024) : sw128_desc(a_hi + ao, S::BK * 128, S::A_SBO, S::A_LAYOUT);
                const u64 bd = sw128_desc(b_hi + bo, 16, 1024);
                const unsigned acc = (ki | j) != 0;
                mma<KIND>(td, ad, bd, idesc, acc);
                if (KIND == TC_TF32X3) {
                    const u64 ad_lo = AK ? sw128_desc(a_hi + S::A_BYTES + ao, 16, 1024)
                                         : sw128_desc(a_hi + S::A_BYTES + ao, S::BK * 128, S::A_SBO, S::A_LAYOUT);
                    const u64 bd_lo = sw128_desc(b_hi + C::B_BYTES + bo, 16, 1024);
                    mma<KIND>(td, ad, bd_lo, idesc, 1u);
                    mma<KIND>(td, ad_lo, bd, idesc, 1u);
                }
            }
            mma_commit(&empty[s]);
        }
        mma_commit(done);
    }
    if (kSplitW && warp >= 2) {
        // ---- weight split: fp32 tile -> hi = x truncated to tf32 (in place), lo = x - hi ----
        const int ct = threadIdx.x - 64;   // 0 .. 32 kSplitWarps - 1
        for (int i = 0; i < nkb; ++i) {
            const int s = i % STAGES;
            if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
                atomicCAS(a.err, 0, G2_ERR_TIMEOUT);
                break;
            }
            float4 *hi = reinterpret_cast<float4 *>(base + (size_t)s * C::STAGE);
            float4 *lo = reinterpret_cast<float4 *>(base + (size_t)s * C::STAGE + S::A_BYTES);
#pragma unroll 4
            for (int k = ct; k < S::A_BYTES / 16; k += 32 * kSplitWarps) {
                const float4 w = hi[k];
                const float4 h = make_float4(__uint_as_float(__float_as_uint(w.x) & 0xFFFFE000u),
                                             __uint_as_float(__float_as_uint(w.y) & 0xFFFFE000u),
                                             __uint_as_float(__float_as_uint(w.z) & 0xFFFFE000u),
                                             __uint_as_float(__float_as_uint(w.w) & 0xFFFFE000u));
                hi[k] = h;
                lo[k] = make_float4(w.x - h.x, w.y - h.y, w.z - h.z, w.w - h.w);   // exact
            }
            // the generic-proxy writes become visible to the tensor cores' (async proxy) reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[s]);
        }
    }
    __syncwarp();

    // ---- epilogue: tensor memory -> output (one split) or partial tile ----
    const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0));   // warp-uniform: tcgen05.ld is .sync.aligned
    if (!ok && lane == 0) atomicCAS(a.err, 0, G2_ERR_TIMEOUT);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // Warp w reads tensor-memory lanes 32 (w % 4) .. (its lane quarter: features f0 + 32 (w % 4) + lane)
    // and columns (w / 4) BN / 2 .. of them (rows r0 + ...): two warps per quarter.  One
    // accumulator per segment; a split GEMM writes the segment's partial of its tile.
    const int q = warp & 3, ch = warp >> 2;
    const bool direct = !a.si.G && a.splits == 1;
    if (ok) {
        constexpr int HALF = BN / 2;
        constexpr int CW = HALF < 32 ? HALF : 32;   // columns per tensor-memory load
#pragma unroll 1
        for (int sg = 0; sg < 2; ++sg) {
            if ((sg ? sn1 : sn0) == 0) continue;
            const int f = (sg ? sf1 : sf0) + q * 32 + lane;
            float *dst = a.part + (size_t)(sg ? sj1 : sj0) * a.R * a.N;
#pragma unroll 1
            for (int c0 = ch * HALF; c0 < (ch + 1) * HALF; c0 += CW) {
                float v[32];
                const unsigned ta = tmem + ((unsigned)(q * 32) << 16) + (unsigned)(sg * BN + c0);
                if (CW == 32) {
                    tmem_ld32(ta, v);
                } else {
                    float v16[16];
                    tmem_ld16(ta, v16);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = v16[j];
                }
                if (f < a.N) {
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        const int r = r0 + c0 + j;
                        if (r >= a.R) continue;
                        if (direct) put_operand(a.op, (size_t)r * a.N + f, a.e.apply(r, f, v[j]));
                        else dst[(size_t)r * a.N + f] = v[j];
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tcols));
}

// Sum of the split-K partials part[s][i .. i+3] in split order.  The loads of up
// to kSumBatch splits are issued together (the sum stays in order), so the
// reduce waits one memory latency per batch rather than one per split.
constexpr int kSumBatch = 8;
__device__ __forceinline__ float4 split_sum(const float *part, int splits, long long total, long long i) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < splits; s0 += kSumBatch) {
        float4 p[kSumBatch];
#pragma unroll
        for (int k = 0; k < kSumBatch; ++k)
            if (s0 + k < splits) p[k] = *reinterpret_cast<const float4 *>(part + (size_t)(s0 + k) * total + i);
#pragma unroll
        for (int k = 0; k < kSumBatch; ++k)
            if (s0 + k < splits) {
                if (s0 + k == 0) {
                    acc = p[0];
                } else {
                    acc.x += p[k].x;
                    acc.y += p[k].y;
                    acc.z += p[k].z;
                    acc.w += p[k].w;
                }
            }
    }
    return acc;
}

// Ordered sum of the splits + epilogue (+ the next GEMM's operand), 4 outputs
// per thread (N % 4 == 0); used when a GEMM ran with split-K.
template <typename WT>
__global__ void tc_reduce_kernel(const float *part, SplitInfo si, int R, int N, Epi<WT> e, OperandOut op) {
    const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    const long long total = (long long)R * N;
    const bool in = i < total;
    const int r = in ? (int)(i / N) : 0, n = in ? (int)(i % N) : 0;
    // the bias is not written by the previous kernels: read it before the wait
    float bv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (in && (e.epi & EPI_BIAS))
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = tof(e.bias[n + j]);
    pdl_wait();
    pdl_launch();
    if (!in) return;
    Epi<WT> en = e;   // the rest of the epilogue, with the bias added here
    en.epi &= ~EPI_BIAS;
    const float4 acc = split_sum(part, si.at(n), total, i);
    put_operand(op, (size_t)i, en.apply(r, n, acc.x + bv[0]));
    put_operand(op, (size_t)i + 1, en.apply(r, n + 1, acc.y + bv[1]));
    put_operand(op, (size_t)i + 2, en.apply(r, n + 2, acc.z + bv[2]));
    put_operand(op, (size_t)i + 3, en.apply(r, n + 3, acc.w + bv[3]));
}

// The same for a GEMM whose output rows (the residual stream) feed a
// LayerNorm: one CTA per row sums the splits, applies the epilogue (out =
// the residual stream; no K/V append), then takes the row's LayerNorm
// (math.cl:283-311: mean, then the mean square deviation, eps 1e-5) and writes
// the normalised row, times gamma plus beta, as the next GEMM's operand.
// N % 4 == 0, N <= 2048.  The bias, gamma and beta (not written by the
// previous kernels) are read before the wait for the previous kernel; after it,
// the partials of both of a thread's column groups and the residual are all
// requested before any is summed, so the row costs one memory round trip.
// NG: groups of 1024 columns a CTA covers (N <= 1024 NG); the one-group instantiation
// (small and medium widths) keeps two CTAs per SM for many-row prefill passes.
template <typename WT, int NG>
__global__ void __launch_bounds__(256, NG == 1 ? 2 : 1)
    tc_reduce_ln_kernel(const float *part, SplitInfo si, int R, int N, Epi<WT> e, const WT *g, const WT *b,
                        OperandOut op) {
    __shared__ float sh[8];
    const int r = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const long long total = (long long)R * N;
    int nn[NG];
    bool in[NG];
    float wb[4 * NG], wg[4 * NG], wbe[4 * NG];
#pragma unroll
    for (int k = 0; k < NG; ++k) {
        nn[k] = (t + k * 256) * 4;
        in[k] = nn[k] < N;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            wb[4 * k + j] = in[k] && (e.epi & EPI_BIAS) ? tof(e.bias[nn[k] + j]) : 0.0f;
            wg[4 * k + j] = in[k] ? tof(g[nn[k] + j]) : 0.0f;
            wbe[4 * k + j] = in[k] ? tof(b[nn[k] + j]) : 0.0f;
        }
    }
    pdl_wait();
    pdl_launch();
    float4 res[NG], acc[NG];
    int ns[NG];
#pragma unroll
    for (int k = 0; k < NG; ++k) {
        res[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        ns[k] = in[k] ? si.at(nn[k]) : 0;
        if (in[k] && (e.epi & EPI_RESID))
            res[k] = *reinterpret_cast<const float4 *>(e.resid + (size_t)r * N + nn[k]);
    }
    int nsm = 0;
#pragma unroll
    for (int k = 0; k < NG; ++k) nsm = ns[k] > nsm ? ns[k] : nsm;
    for (int s0 = 0; s0 < nsm; s0 += kSumBatch) {   // in split order, as split_sum
        float4 p[NG][kSumBatch];
#pragma unroll
        for (int k = 0; k < kSumBatch; ++k)
#pragma unroll
            for (int c = 0; c < NG; ++c)
                if (s0 + k < ns[c])
                    p[c][k] = *reinterpret_cast<const float4 *>(part + (size_t)(s0 + k) * total + (size_t)r * N + nn[c]);
#pragma unroll
        for (int k = 0; k < kSumBatch; ++k)
#pragma unroll
            for (int c = 0; c < NG; ++c)
                if (s0 + k < ns[c]) {
                    if (s0 + k == 0) {
                        acc[c] = p[c][0];
                    } else {
                        acc[c].x += p[c][k].x;
                        acc[c].y += p[c][k].y;
                        acc[c].z += p[c][k].z;
                        acc[c].w += p[c][k].w;
                    }
                }
    }
    // the epilogue (Epi::apply without the K/V append): + bias, GELU, residual + v, stored
    float v[4 * NG];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < NG; ++k) {
        if (!in[k]) continue;
        const float a4[4] = {acc[k].x, acc[k].y, acc[k].z, acc[k].w};
        const float r4[4] = {res[k].x, res[k].y, res[k].z, res[k].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float x = a4[j];
            if (e.epi & EPI_BIAS) x += wb[4 * k + j];
            if (e.epi & EPI_GELU) x = gelu_f(x);
            if (e.epi & EPI_RESID) x = r4[j] + x;
            v[4 * k + j] = x;
        }
        if (!(e.epi & EPI_NOSTORE))
            *reinterpret_cast<float4 *>(e.out + (size_t)r * N + nn[k]) =
                make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        s += (v[4 * k] + v[4 * k + 1]) + (v[4 * k + 2] + v[4 * k + 3]);
    }
    auto block_sum = [&](float x) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        __syncthreads();
        if (lane == 0) sh[warp] = x;
        __syncthreads();
        float y = lane < 8 ? sh[lane] : 0.0f;   // every lane ends with the total
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        return y;
    };
    const float mean = block_sum(s) / (float)N;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < NG; ++k)
        if (in[k])
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float d = v[4 * k + j] - mean;
                q = fmaf(d, d, q);
            }
    const float rstd = 1.0f / sqrtf(block_sum(q) / (float)N + 1e-5f);
#pragma unroll
    for (int k = 0; k < NG; ++k)
        if (in[k])
#pragma unroll
            for (int j = 0; j < 4; ++j)
                put_operand(op, (size_t)r * N + nn[k] + j, (v[4 * k + j] - mean) * rstd * wg[4 * k + j] + wbe[4 * k + j]);
}

// x -> (hi, lo) tf32 pair, or x -> fp16.
__global__ void tc_prep_kernel(int kind, const float4 *x, float4 *hi, float4 *lo, __half2 *h16, long long n4) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 v = x[i];
        if (kind == TC_TF32X3) {
            float h[4], l[4];
            const float in[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                unsigned t;
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(in[j]));
                h[j] = __uint_as_float(t);
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(in[j] - h[j]));
                l[j] = __uint_as_float(t);
            }
            hi[i] = make_float4(h[0], h[1], h[2], h[3]);
            lo[i] = make_float4(l[0], l[1], l[2], l[3]);
        } else {
            h16[2 * i] = __floats2half2_rn(v.x, v.y);
            h16[2 * i + 1] = __floats2half2_rn(v.z, v.w);
        }
    }
}

// ---- stage images -------------------------------------------------------------
// Element positions of one stage's weight tile as the tiled TMA loads of the
// GEMM place them: the NBOX boxes of BOX_F features x BK rows of a tensor
// whose element (row, feature) holds row * 128 + feature are loaded exactly as
// the producer loads a weight stage (same box shapes, swizzle and shared-memory
// alignment), then copied out, so table[p] names the element at position p.
template <int KIND>
__global__ void tc_perm_kernel(const __grid_constant__ CUtensorMap m, unsigned *table, int *err) {
    using S = TcShape<KIND>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *base =
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    u64 *bar = reinterpret_cast<u64 *>(base + S::A_BYTES);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_expect_tx(bar, S::A_BYTES);
        for (int b = 0; b < S::NBOX; ++b) tma_load_2d(base + b * (S::BK * 128), &m, b * S::BOX_F, 0, bar);
    }
    __syncthreads();
    const bool ok = mbar_wait(bar, 0);
    if (!ok) {
        if (threadIdx.x == 0) atomicCAS(err, 0, G2_ERR_TIMEOUT);
        return;
    }
    for (int i = threadIdx.x; i < S::A_BYTES / S::ELEM; i += blockDim.x)
        table[i] = S::ELEM == 4 ? reinterpret_cast<const unsigned *>(base)[i]
                                : (unsigned)reinterpret_cast<const unsigned short *>(base)[i];
}

__global__ void tc_iota_kernel(unsigned *idx32, unsigned short *idx16, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (idx32) idx32[i] = (unsigned)i;
        else idx16[i] = (unsigned short)i;
    }
}

// img[(t KB + kb) PER + p] = W[kb BK + row][t 128 + feature], (row, feature) = table[p]
// (zero past N; a table entry outside the stage also gives zero).  TC_TF32X3:
// tf32 hi / lo images split as tc_prep_kernel does, or the fp32 image when
// img_lo is null.  TC_F16: the fp16 image.
__global__ void tc_image_kernel(int kind, const void *W, void *img_hi, void *img_lo, const unsigned *table, int K,
                                int N, long long total) {
    const int BK = kind == TC_TF32X3 ? 32 : 64;
    const int PER = kind == TC_TF32X3 ? 4096 : 8192;   // elements per 16 KB stage
    const int KB = K / BK;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long st = i / PER;
        const unsigned e = table[(int)(i - st * PER)];
        const int row = (int)(e >> 7), col = (int)(e & 127u);
        const int t = (int)(st / KB), kb = (int)(st - (long long)t * KB);
        const int k = kb * BK + row, n = t * kTcTileF + col;
        const bool in = row < BK && n < N;
        if (kind == TC_TF32X3) {
            const float x = in ? reinterpret_cast<const float *>(W)[(size_t)k * N + n] : 0.0f;
            if (img_lo) {
                unsigned u;
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
                const float h = __uint_as_float(u);
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x - h));
                reinterpret_cast<float *>(img_hi)[i] = h;
                reinterpret_cast<float *>(img_lo)[i] = __uint_as_float(u);
            } else {
                reinterpret_cast<float *>(img_hi)[i] = x;
            }
        } else {
            reinterpret_cast<__half *>(img_hi)[i] =
                in ? reinterpret_cast<const __half *>(W)[(size_t)k * N + n] : __float2half_rn(0.0f);
        }
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Row-tile height (BN) and split count for R rows x N outputs over kb_total K blocks.
struct TcPlan {
    int bn, splits, kb_per;
};
TcPlan plan(int R, int N, int kb_total, int sms) {
    TcPlan p;
    p.bn = R <= 32 ? 32 : R <= 64 ? 64 : 128;
    const int tiles = ((N + kTcTileF - 1) / kTcTileF) * ((R + p.bn - 1) / p.bn);
    int s = (sms + tiles - 1) / tiles;                     // one wave of CTAs
    s = s < 1 ? 1 : s;
    const int max_s = kb_total / 2 > 0 ? kb_total / 2 : 1;   // at least two K blocks per split
    s = s > max_s ? max_s : s;
    s = s > 32 ? 32 : s;
    p.kb_per = (kb_total + s - 1) / s;
    p.splits = (kb_total + p.kb_per - 1) / p.kb_per;       // no empty split
    return p;
}

// Balanced split (SplitInfo) for R rows of an N-output projection over
// kb_total K blocks: when the rows fit one tile height and the 128-feature
// tiles are fewer than the SMs, the tiles' K blocks are shared out equally
// over min(sms, U / 2) CTAs (at least two K blocks each), so that every SM
// streams weights; each share then spans at most two tiles.  Uniform splits
// of each tile leave SMs idle whenever tiles x splits misses the SM count
// (76 to 104 of 148 CTAs on the 32-row GEMMs of GPT-2 XL).  Measured on
// B200: the balanced GEMMs' main loops are up to twice as short; their extra
// partials (up to 13 per column) cost the LayerNorm-fused reduces about as
// much, so a GEMM whose reduce takes a LayerNorm keeps uniform splits.  For the
// others (c_attn, c_fc) it pays on the 3xTF32 GEMMs (c5 +3.7%) and not on the
// fp16 ones (c4 -7%): by default it applies to 3xTF32 GEMMs of up to 32 rows;
// G2_TC_BALANCED sets the largest row count for both precisions (0 = never).
SplitInfo balanced_plan(int R, int N, int kb_total, int bn, int sms, int kind, bool ln) {
    static const int env_rows = getenv("G2_TC_BALANCED") ? atoi(getenv("G2_TC_BALANCED")) : -1;
    const int max_rows = env_rows >= 0 ? env_rows : (kind == TC_TF32X3 ? 32 : 0);
    SplitInfo si;
    if (ln) return si;
    const int tiles = (N + kTcTileF - 1) / kTcTileF;
    const long long U = (long long)tiles * kb_total;
    if (R > max_rows || R > bn || N % 4 || tiles >= sms || kb_total < 2) return si;
    const int G = (int)(U / 2 < sms ? U / 2 : sms);
    if (G <= tiles) return si;
    si.G = G;
    si.KB = kb_total;
    si.U = U;
    return si;
}
// The most partials any output column of the plan has.
int max_partials(const SplitInfo &si, int N) {
    int m = si.splits;
    if (si.G)
        for (int n = 0; n < N; n += kTcTileF) m = std::max(m, si.at(n));
    return m;
}

template <int KIND, int BN, typename WT, bool AK>
void launch_kernel(const TcWeights &w, const TcRowsOperand &x, int bn_idx, const TcArgs<WT> &a, cudaStream_t st) {
    using C = TcCfg<KIND, BN>;
    static unsigned long long attr_set = 0;   // devices on which this instantiation's smem limit was raised
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !(__atomic_load_n(&attr_set, __ATOMIC_ACQUIRE) >> dev & 1ull)) {
        cudaFuncSetAttribute(tc_gemm_kernel<KIND, BN, WT, AK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
        __atomic_fetch_or(&attr_set, 1ull << dev, __ATOMIC_RELEASE);
    } else if (dev >= 64) {
        cudaFuncSetAttribute(tc_gemm_kernel<KIND, BN, WT, AK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    }
    const dim3 grid = a.si.G ? dim3((unsigned)a.si.G) : dim3((a.N + kTcTileF - 1) / kTcTileF, (a.R + BN - 1) / BN, a.splits);
    launch_pdl(tc_gemm_kernel<KIND, BN, WT, AK>, grid, dim3(kThreads), C::SMEM, st, w.hi, KIND == TC_TF32X3 ? w.lo : w.hi,
               x.hi[bn_idx], KIND == TC_TF32X3 ? x.lo[bn_idx] : x.hi[bn_idx], a);
}

}  // namespace

int tc_encode(CUtensorMap *map, CUtensorMapDataType dt, const void *base, unsigned long long inner,
              unsigned long long outer, unsigned box_inner, unsigned box_outer, bool atom32) {
    EncodeTiledFn fn = encoder();
    if (!fn) return G2_ERR_CUDA;
    const unsigned elem = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT16 ? 2 : 4;
    if (box_inner * elem != 128 || ((uintptr_t)base & 15) || (inner * elem) % 16) return G2_ERR_ARG;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * elem};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? G2_OK : G2_ERR_CUDA;
}

int tc_weights(TcWeights *w, int kind, const void *hi, const void *lo, int K, int N) {
    const bool t = kind == TC_TF32X3;
    const CUtensorMapDataType dt = t ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const unsigned bf = t ? 32 : 64, bk = t ? 32 : 64;
    w->K = K;
    w->N = N;
    w->kmajor = false;
    w->wsplit = t && !lo;
    int rc = tc_encode(&w->hi, dt, hi, N, K, bf, bk, t);
    if (!rc && t && lo) rc = tc_encode(&w->lo, dt, lo, N, K, bf, bk, t);
    else w->lo = w->hi;
    return rc;
}

int tc_stage_perm(int kind, void *idx, unsigned *table, int *err, cudaStream_t st) {
    // The table depends only on the weight kind: it is recorded once per process
    // and kind, checked on the host to be a permutation of the stage's elements,
    // and uploaded for every later engine.
    static std::mutex mu;
    static std::vector<unsigned> cached[2];
    const bool t = kind == TC_TF32X3;
    const int BK = t ? 32 : 64, n = BK * kTcTileF;   // one stage: BK rows x 128 features
    std::lock_guard<std::mutex> lk(mu);
    std::vector<unsigned> &c = cached[t ? 1 : 0];
    if (c.empty()) {
        tc_iota_kernel<<<(n + 255) / 256, 256, 0, st>>>(t ? reinterpret_cast<unsigned *>(idx) : nullptr,
                                                        t ? nullptr : reinterpret_cast<unsigned short *>(idx), n);
        CUtensorMap m;
        const int rc = tc_encode(&m, t ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, idx, kTcTileF,
                                 BK, t ? 32 : 64, BK, t);
        if (rc) return rc;
        const size_t smem = 16384 + 1024 + 64;
        if (t) {
            cudaFuncSetAttribute(tc_perm_kernel<TC_TF32X3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            tc_perm_kernel<TC_TF32X3><<<1, 256, smem, st>>>(m, table, err);
        } else {
            cudaFuncSetAttribute(tc_perm_kernel<TC_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            tc_perm_kernel<TC_F16><<<1, 256, smem, st>>>(m, table, err);
        }
        std::vector<unsigned> h(n);
        int e = 0;
        if (cudaMemcpyAsync(h.data(), table, sizeof(unsigned) * n, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(&e, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess || e)
            return G2_ERR_CUDA;
        std::vector<char> seen(n, 0);
        for (unsigned v : h) {
            if (v >= (unsigned)n || seen[v]) return G2_ERR_CUDA;   // not a permutation
            seen[v] = 1;
        }
        c = h;
        return G2_OK;
    }
    return cudaMemcpyAsync(table, c.data(), sizeof(unsigned) * n, cudaMemcpyHostToDevice, st) == cudaSuccess ? G2_OK
                                                                                                          : G2_ERR_CUDA;
}

size_t tc_image_elems(int kind, int K, int N) {
    (void)kind;
    return (size_t)((N + kTcTileF - 1) / kTcTileF) * kTcTileF * K;
}

void launch_tc_image(int kind, const void *W, void *img_hi, void *img_lo, const unsigned *table, int K, int N,
                     cudaStream_t st) {
    const long long total = (long long)tc_image_elems(kind, K, N);
    const int blocks = (int)((total + 255) / 256 < 8192 ? (total + 255) / 256 : 8192);
    tc_image_kernel<<<blocks, 256, 0, st>>>(kind, W, img_hi, img_lo, table, K, N, total);
}

int tc_weights_kmajor(TcWeights *w, int kind, const void *hi, const void *lo, int K, int N) {
    const bool t = kind == TC_TF32X3;
    const CUtensorMapDataType dt = t ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const unsigned bk = t ? 32 : 64;
    w->K = K;
    w->N = N;
    w->kmajor = true;
    w->wsplit = t && !lo;
    int rc = tc_encode(&w->hi, dt, hi, K, N, bk, kTcTileF, false);
    if (!rc && t && lo) rc = tc_encode(&w->lo, dt, lo, K, N, bk, kTcTileF, false);
    else w->lo = w->hi;
    return rc;
}

int tc_rows_operand(TcRowsOperand *x, int kind, const void *hi, const void *lo, int K, int R) {
    const bool t = kind == TC_TF32X3;
    const CUtensorMapDataType dt = t ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const unsigned bk = t ? 32 : 64;
    x->K = K;
    x->R = R;
    const unsigned bn[3] = {32, 64, 128};
    for (int i = 0; i < 3; ++i) {
        int rc = tc_encode(&x->hi[i], dt, hi, K, R, bk, bn[i], false);
        if (!rc && t) rc = tc_encode(&x->lo[i], dt, lo, K, R, bk, bn[i], false);
        if (rc) return rc;
        if (!t) x->lo[i] = x->hi[i];
    }
    return G2_OK;
}

void launch_tc_prep(int kind, const float *x, float *hi, float *lo, __half *h16, long long n, cudaStream_t st) {
    const long long n4 = n / 4;
    const int blocks = (int)((n4 + 255) / 256 < 4096 ? (n4 + 255) / 256 : 4096);
    tc_prep_kernel<<<blocks > 0 ? blocks : 1, 256, 0, st>>>(kind, reinterpret_cast<const float4 *>(x),
                                                          reinterpret_cast<float4 *>(hi), reinterpret_cast<float4 *>(lo),
                                                          reinterpret_cast<__half2 *>(h16), n4);
}

size_t tc_partial_floats(int R_max, int N, int K, int kind, int sms) {
    const int kb_total = K / (kind == TC_TF32X3 ? 32 : 64);
    size_t m = 0;
    for (int R = 1; R <= R_max; ++R) {
        const TcPlan p = plan(R, N, kb_total, sms);
        const SplitInfo si = balanced_plan(R, N, kb_total, p.bn, sms, kind, false);
        // room for either plan (a GEMM followed by a LayerNorm reduce keeps uniform splits)
        const size_t f = (size_t)std::max(si.G ? max_partials(si, N) : 0, p.splits) * R * N;
        m = f > m ? f : m;
    }
    return m;
}

template <typename WT>
int launch_tc_gemm(int kind, const TcWeights &w, const TcRowsOperand &x, int R, float *partial, size_t partial_floats,
                   unsigned *tile_ctr, int *err, const WT *bias, const float *resid, float *out, int epi,
                   const KVLayout *kv, int layer, Rows rows, int sms, cudaStream_t st, OperandOut op, int out_stride,
                   const WT *ln_g, const WT *ln_b, OperandOut ln_op, bool *ln_done, bool defer_reduce,
                   SplitInfo *si_out) {
    const int bk = kind == TC_TF32X3 ? 32 : 64;
    const int kb_total = w.K / bk;
    TcPlan p = plan(R, w.N, kb_total, sms);
    if (w.N % 4) {   // the reduce kernel works in float4s: no split-K (the LM head's 393 tiles need none)
        p.splits = 1;
        p.kb_per = kb_total;
    }
    // Split caps measured on B200 for 32-row batched steps: more splits add
    // partial-tile traffic and reduce time faster than they add streaming
    // CTAs.  A reduce fused with a LayerNorm (one CTA per row) takes up to 8;
    // a plain reduce up to 3 (fp16) or 2 (3xTF32, twice the partial bytes
    // per weight byte).
    {
        // G2_TC_CAP / G2_TC_CAP_LN override the caps (measurement sweeps)
        static const int cap_env = getenv("G2_TC_CAP") ? atoi(getenv("G2_TC_CAP")) : 0;
        static const int cap_ln_env = getenv("G2_TC_CAP_LN") ? atoi(getenv("G2_TC_CAP_LN")) : 0;
        int cap = ln_g ? 8 : kind == TC_TF32X3 ? 2 : 3;
        if (ln_g && cap_ln_env > 0) cap = cap_ln_env;
        if (!ln_g && cap_env > 0) cap = cap_env;
        if (p.splits > cap) {
            p.kb_per = (kb_total + cap - 1) / cap;
            p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
        }
    }
    // fewer splits if the scratch is smaller than the plan needs (one split needs none)
    while (p.splits > 1 && (size_t)p.splits * R * w.N > partial_floats) {
        p.kb_per = (kb_total + p.splits - 2) / (p.splits - 1);
        p.splits = (kb_total + p.kb_per - 1) / p.kb_per;
    }
    TcArgs<WT> a;
    a.N = w.N;
    a.R = R;
    a.kb_total = kb_total;
    a.kb_per = p.kb_per;
    a.splits = p.splits;
    a.si.splits = p.splits;
    if (!w.kmajor) {   // the balanced split, where it applies and its partials fit the scratch
        const SplitInfo si = balanced_plan(R, w.N, kb_total, p.bn, sms, kind, ln_g != nullptr);
        if (si.G && (size_t)max_partials(si, w.N) * R * w.N <= partial_floats) a.si = si;
    }
    a.part = partial;
    a.err = err;
    a.wsplit = w.wsplit ? 1 : 0;
    a.img_hi = w.kmajor ? nullptr : reinterpret_cast<const unsigned char *>(w.img_hi);
    a.img_lo = w.kmajor ? nullptr : reinterpret_cast<const unsigned char *>(w.img_lo);
    (void)tile_ctr;
    a.e.bias = bias;
    a.e.resid = resid;
    a.e.out = out;
    a.e.N = out_stride > 0 ? out_stride : w.N;   // row stride of out (and resid)
    a.e.epi = epi;
    if (kv) a.e.kv = *kv;
    a.e.layer = layer;
    a.e.pos = rows.pos;
    a.e.slot = rows.slot;
    a.e.E = w.N / 3;
    a.op = op;
    const int bi = p.bn == 32 ? 0 : p.bn == 64 ? 1 : 2;
    if (w.kmajor) {   // the LM head (rows of wte): one row tile of 32 per launch suffices for batched steps
        if (kind == TC_TF32X3) {
            if (p.bn == 32) launch_kernel<TC_TF32X3, 32, WT, true>(w, x, bi, a, st);
            else if (p.bn == 64) launch_kernel<TC_TF32X3, 64, WT, true>(w, x, bi, a, st);
            else launch_kernel<TC_TF32X3, 128, WT, true>(w, x, bi, a, st);
        } else {
            if (p.bn == 32) launch_kernel<TC_F16, 32, WT, true>(w, x, bi, a, st);
            else if (p.bn == 64) launch_kernel<TC_F16, 64, WT, true>(w, x, bi, a, st);
            else launch_kernel<TC_F16, 128, WT, true>(w, x, bi, a, st);
        }
    } else if (kind == TC_TF32X3) {
        if (p.bn == 32) launch_kernel<TC_TF32X3, 32, WT, false>(w, x, bi, a, st);
        else if (p.bn == 64) launch_kernel<TC_TF32X3, 64, WT, false>(w, x, bi, a, st);
        else launch_kernel<TC_TF32X3, 128, WT, false>(w, x, bi, a, st);
    } else {
        if (p.bn == 32) launch_kernel<TC_F16, 32, WT, false>(w, x, bi, a, st);
        else if (p.bn == 64) launch_kernel<TC_F16, 64, WT, false>(w, x, bi, a, st);
        else launch_kernel<TC_F16, 128, WT, false>(w, x, bi, a, st);
    }
    if (ln_done) *ln_done = false;
    if (si_out) *si_out = a.si;
    if (!a.si.split()) return 1;   // the GEMM applied the epilogue itself
    if (defer_reduce) return 1;    // the consumer sums the partials
    if (ln_g && w.N <= 2048 && (w.N % 4) == 0 && !(a.e.epi & EPI_KV)) {   // splits, epilogue and the next LayerNorm
        if (w.N <= 1024)
            launch_pdl(tc_reduce_ln_kernel<WT, 1>, dim3((unsigned)R), dim3(256), 0, st, (const float *)partial, a.si, R,
                       w.N, a.e, ln_g, ln_b, ln_op);
        else
            launch_pdl(tc_reduce_ln_kernel<WT, 2>, dim3((unsigned)R), dim3(256), 0, st, (const float *)partial, a.si, R,
                       w.N, a.e, ln_g, ln_b, ln_op);
        if (ln_done) *ln_done = true;
        return 2;
    }
    const long long n4 = (long long)R * w.N / 4;
    launch_pdl(tc_reduce_kernel<WT>, dim3((unsigned)((n4 + 255) / 256)), dim3(256), 0, st, (const float *)partial, a.si,
               R, w.N, a.e, op);
    return 2;
}

template int launch_tc_gemm<float>(int, const TcWeights &, const TcRowsOperand &, int, float *, size_t, unsigned *,
                                   int *, const float *, const float *, float *, int, const KVLayout *, int, Rows, int,
                                   cudaStream_t, OperandOut, int, const float *, const float *, OperandOut, bool *, bool,
                                   SplitInfo *);
template int launch_tc_gemm<__half>(int, const TcWeights &, const TcRowsOperand &, int, float *, size_t, unsigned *,
                                    int *, const __half *, const float *, float *, int, const KVLayout *, int, Rows, int,
                                    cudaStream_t, OperandOut, int, const __half *, const __half *, OperandOut, bool *,
                                    bool, SplitInfo *);

#ifdef G2_CHECK
int check_flag_tc() {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g2_check_flag, sizeof(int));
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g2_check_flag, &z, sizeof(int));
    }
    return v;
}
#else
int check_flag_tc() { return 0; }
#endif

}  // namespace g2
