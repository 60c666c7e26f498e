// g2_mega.cu -- persistent B = 1 decode kernel (fp32): every layer and every
// greedy step of a generation in one cooperative launch.
//
// It replaces the per-token kernel sequence of decode() (main.c:1792-1833)
// and the greedy branch of sample_next_token (main.c:1898-1904).
//
// Structure (one CTA per SM; 15 consumer warps + 1 producer warp):
//
//  * A token is a chain of dependent cross-CTA exchanges; their latency, not
//    HBM bandwidth, bounds B = 1 decode.  A layer takes three:
//      A  LN1 + c_attn + K/V append      needs x (the residual stream)
//      B  attention + attn.c_proj        needs q, k, v of one head
//      D  LN2 + c_fc + GELU + mlp.c_proj needs x + attention output
//    B and D compute their projection split over K: a B unit (head h, column
//    slice j) runs the whole attention of head h (every unit of head h repeats
//    it, reading the head's K/V rows from L2) and multiplies the head's 64
//    outputs by rows 64h..64h+63 of attn.c_proj, slice j.  A D unit computes a
//    strip of c_fc columns, applies GELU in shared memory and multiplies the
//    strip by the same rows of mlp.c_proj, for all E outputs.  No unit waits
//    for another unit's partial: the partial sums meet in an accumulator.
//  * Accumulators are 64-bit words holding count * 2^55 + sum(round(v * 2^32))
//    modulo 2^64.  A contribution is one red.add of 2^55 + round(v * 2^32).
//    Integer addition is exact and order-independent, so the sum does not
//    depend on timing, and the count field tells a reader when every
//    contributor has added.  The representable range is |sum| < 2^22 (GPT-2
//    activations stay orders of magnitude below it); a contribution is
//    clamped to +-2^21.  Each accumulator vector is used once per launch (the
//    host zeroes them before the launch).
//  * Every CTA keeps the residual stream x in shared memory and applies the
//    same update from the accumulators, x += acc + bias (add_inplace after
//    the projection, math.cl:314), so all CTAs hold bit-identical copies.
//  * A units are column strips of c_attn over the full K, followed by a bias
//    row and a column-sum row.  LN1 (and LN2 in D) are folded in:
//    W' = diag(gamma) W, b' = b + beta W, and LN(x) W' + b' =
//    rstd (x W' - mean colsum(W')) + b', so the statistics are reduced in the
//    same pass as the products.  q, k, v reach the B units as 64-bit words
//    (epoch << 32 | float bits): readiness costs one L2 round trip.
//  * Unit g of a layer belongs to CTA g % gridDim.x, counting A, then B, then
//    D units.  For the LM head every CTA takes an equal contiguous share of
//    the wte rows, in units of up to 15 rows (one per consumer warp), so all
//    CTAs finish it together.  The producer warp streams the CTA's units, in
//    consumption order, through an 8-slot shared-memory ring with
//    cp.async.bulk (mbarrier full/empty, L2 evict-first).  The stream waits on
//    no activation, so it runs ahead across layer and token boundaries.
//  * Then LN_f + LM head with a per-CTA argmax; every CTA reads all CTA
//    partials and derives the next token.  The K/V rows a step appends are
//    read by later steps only; one fence pair per step at that exchange
//    orders them.
//  * Every wait is bounded (globaltimer, MegaParams::timeout_ns per wait, 2 s
//    unless the engine was opened with a shorter limit).  On expiry the thread
//    records an error code; the consumer warps leave together at the next
//    uniform check, the producer stops issuing and drains its in-flight
//    copies, and the host reports G2_ERR_TIMEOUT.  A contribution clamped at
//    +-2^21 is recorded the same way (kErrClamp) and reported as
//    G2_ERR_RANGE.
#include <cfloat>
#include <climits>
#include <cstdint>

#include "g2_mega.h"

namespace g2 {

namespace {

constexpr int kWarps = 15;                 // consumer warps: with the producer, 16 warps (128 registers each)
constexpr int kCons = kWarps * 32;         // consumer threads
constexpr int kThreads = kCons + 32;       // + producer warp
constexpr int kSlots = 8;
constexpr int kSlotBytes = 24832;          // 194 * 128: whole rows at every strip width (16 to 128 B)
constexpr int kConsBar = 1;                // named barrier of the consumer warps
constexpr int kMaxKeys = 1024;             // attention keys (positions) per head
constexpr int kKeysPerPass = kCons / 4;    // 4 threads per key in the score pass
constexpr int kPvGroups = kCons / 16;      // key groups of the P.V pass (16 threads = 64 dims per key)
constexpr int kPart = 2048;                // partial-sum scratch (floats)
// Reduction scratch (floats): two alternating halves for strip units, then the
// argmax partials, the attention scalars and the LayerNorm partials.
constexpr int kRedHalf = 512;
constexpr int kRedArg = 1024;              // 16 values, then 16 indices
constexpr int kRedAtt = 1056;              // 32
constexpr int kRedLn = 1088;               // 32
constexpr int kRedFloats = 1120;
// Per-CTA constants computed once at launch (ints), so that no unit divides by
// a runtime value: strip geometries of the A and D units, block geometries of
// the B and D units, the B-unit slice count, and the first unit of each layer.
constexpr int kGeoA = 0, kGeoDs = 8;       // strip: CG, RG, RPC, nfull, magic(CG), cw
constexpr int kGeoB = 16, kGeoDb = 24;     // block: CG, RG, RPC, magic(CG), NB, RG * CG
constexpr int kCfgMnq = 32, kCfgNq = 33;   // magic(nq), nq
constexpr int kCfgOffB = 34, kCfgOffD = 35;   // nA % G, (nA + nB) % G
constexpr int kCfgInvE = 36;               // 1 / E (float bits)
constexpr int kCfgLm0 = 37, kCfgLm1 = 38;  // this CTA's wte rows [lm0, lm1)
constexpr int kCfgFirst = 40;              // [l] = first unit of layer l's count on this CTA, l < L
constexpr int kCfgInts = (kCfgFirst + kMegaMaxLayers + 3) / 4 * 4;   // a whole number of 16-byte words
constexpr int kMaxJ = 4;                   // vector words per consumer thread (E <= kMaxJ * kCons)
// n / d for 0 <= n < 2048 and 1 <= d <= 480 as (n * magic(d)) >> 20, with
// magic(d) = ceil(2^20 / d) (exact in that range: n (magic * d - 2^20) < 2^20).
__host__ __device__ constexpr int magic20(int d) { return ((1 << 20) + d - 1) / d; }
__device__ __forceinline__ int mdiv(int n, int m) { return (n * m) >> 20; }

typedef unsigned long long u64;

constexpr u64 kAccOne = 1ull << 55;        // one contribution in the count field
constexpr float kAccMax = 2097152.0f;      // 2^21: clamp of one contribution

__device__ __forceinline__ u64 gtime() {
    u64 t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ u64 ld_tag(const u64 *p) {
    u64 v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_tag(u64 *p, float v, unsigned ep) {
    const u64 w = ((u64)ep << 32) | (u64)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ bool tag_is(u64 w, unsigned ep) { return (unsigned)(w >> 32) == ep; }
__device__ __forceinline__ float tag_val(u64 w) { return __uint_as_float((unsigned)w); }

// Accumulator words: count * 2^55 + sum of round(v * 2^32), modulo 2^64.
// A contribution beyond +-2^21 is clamped and recorded in *err (kErrClamp),
// so that a lost range is reported rather than silent.
__device__ __forceinline__ void acc_add(u64 *dst, float v, int *err) {
    if (!(fabsf(v) <= kAccMax)) atomicCAS(err, 0, kErrClamp);
    v = fminf(fmaxf(v, -kAccMax), kAccMax);
    const long long q = __float2ll_rn(v * 4294967296.0f);   // exact scaling by 2^32, one rounding
    const u64 c = kAccOne + (u64)q;
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(dst), "l"(c) : "memory");
}
__device__ __forceinline__ unsigned acc_count(u64 w) { return (unsigned)((w + (1ull << 54)) >> 55); }

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync %0, %1;" ::"n"(kConsBar), "n"(kCons) : "memory"); }
__device__ __forceinline__ int cons_and(int pred) {
    int r;
    asm volatile(
        "{ .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.s32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"(pred), "n"(kConsBar), "n"(kCons)
        : "memory");
    return r;
}

// ---- mbarrier / bulk copy --------------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
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
// Wait for the phase of parity `parity` to complete, for at most ns.
__device__ __forceinline__ bool mbar_wait(u64 *b, unsigned parity, u64 ns) {
    if (mbar_try(b, parity)) return true;
    const u64 limit = gtime() + ns;
    for (;;) {
        if (mbar_try(b, parity)) return true;
        if (gtime() > limit) return false;
    }
}
// The producer's wait: the same, sleeping between tries so that the waiting
// warp leaves its scheduler's issue slots to the consumer warps.
__device__ __forceinline__ bool mbar_wait_idle(u64 *b, unsigned parity, u64 ns) {
    if (mbar_try(b, parity)) return true;
    const u64 limit = gtime() + ns;
    for (;;) {
        __nanosleep(64);
        if (mbar_try(b, parity)) return true;
        if (gtime() > limit) return false;
    }
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, unsigned bytes, u64 *bar, u64 policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
    return v1 > v2 || (v1 == v2 && i1 < i2);
}
// Butterfly argmax over a warp under the order of better(): every lane ends
// with the unique maximum of the lanes' (value, index) pairs.
__device__ __forceinline__ void warp_argmax(float &v, int &i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}
__device__ __forceinline__ float gelu_f(float v) {
    return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
}
__device__ __forceinline__ void fma4(float4 &acc, float x, const float4 &w) {
    acc.x = fmaf(x, w.x, acc.x);
    acc.y = fmaf(x, w.y, acc.y);
    acc.z = fmaf(x, w.z, acc.z);
    acc.w = fmaf(x, w.w, acc.w);
}

// ---- the per-step unit schedule (the same in producer and consumers) ------------------
struct Sched {
    int nA, nB, nD;        // units per phase
    int per_layer;         // nA + nB + nD
    int G;                 // CTAs
    // first unit of a phase starting at global unit index g0 that belongs to CTA c
    __device__ __forceinline__ int first(int g0, int c) const {
        const int r = (c - g0) % G;
        return r < 0 ? r + G : r;
    }
    __device__ __forceinline__ int a_first(int l, int c) const { return first(l * per_layer, c); }
    __device__ __forceinline__ int b_first(int l, int c) const { return first(l * per_layer + nA, c); }
    __device__ __forceinline__ int d_first(int l, int c) const { return first(l * per_layer + nA + nB, c); }
};

struct Smem {
    float *xs;     // input vector of the current phase (E + 4 floats)
    float *xres;   // the residual stream x (E floats)
    float *red;    // reduction scratch (kRedFloats)
    float *attp;   // attention scores, then probabilities (kMaxKeys)
    float *attq;   // q, k, v of the head at pos (192)
    float *atta;   // attention output of the head (64); GELU outputs of a D unit
    float *part;   // partial sums of the P.V and block passes (kPart)
    int *cfg;      // per-CTA constants (kCfgInts)
    u64 *trc;      // trace accumulators (thread 0 only)
    u64 *full, *empty;
    unsigned char *ring;
};

// Trace layout in shared memory (u64): see g2_mega.h; [20] phase-begin stamp,
// [21] inputs stamp, [22] timeline count, [32..160) timeline stamps (CTA 0, one step).
struct Cx {
    const MegaParams *p;
    Smem s;
    int cta, ctid, warp, lane;
    unsigned chunk_i;   // next ring chunk to consume
    unsigned upar;      // parity of the next strip unit's reduction scratch
    int failed;         // this thread saw an expired wait
    bool tr;            // tracing (consumer thread 0)
    bool tl;            // timeline stamps (CTA 0, one step)
    u64 t0;
};

__device__ __forceinline__ void tr_stamp(Cx &cx) {
    if (cx.tl) {
        const u64 n = cx.s.trc[22];
        if (n < (u64)(kTraceSlots - 32)) {
            cx.s.trc[32 + n] = gtime() - cx.t0;
            cx.s.trc[22] = n + 1;
        }
    }
}
__device__ __forceinline__ void tr_begin(Cx &cx) {
    if (cx.tr) {
        cx.s.trc[20] = gtime();
        tr_stamp(cx);
    }
}
__device__ __forceinline__ void tr_inputs(Cx &cx, int ph) {
    if (cx.tr) {
        const u64 t = gtime();
        cx.s.trc[21] = t;
        cx.s.trc[ph] += t - cx.s.trc[20];
        tr_stamp(cx);
    }
}
__device__ __forceinline__ void tr_end(Cx &cx, int ph) {
    if (cx.tr) {
        cx.s.trc[8 + ph] += gtime() - cx.s.trc[21];
        tr_stamp(cx);
    }
}

__device__ __forceinline__ void fail(Cx &cx, int code) {
    cx.failed = 1;
    atomicCAS(cx.p->err, 0, code);
}

// Poll n tagged words into dst until all carry `ep`.  All consumer threads.
// Each warp polls its own words round after round with no barrier in between
// (a warp leaves when all of its lanes have their words); one barrier at the
// end, which also carries the failure flag.  The deadline is checked every 64
// rounds.
__device__ __forceinline__ bool poll_vec(Cx &cx, const u64 *src, float *dst, int n, unsigned ep, int code) {
    const u64 limit = gtime() + cx.p->timeout_ns;
    // bit j of `pending`: word ctid + j * kCons not yet seen with the right epoch (n <= 32 * kCons)
    unsigned pending = 0;
    if (!cx.failed)
        for (int j = 0, i = cx.ctid; i < n; ++j, i += kCons) pending |= 1u << j;
    for (unsigned round = 0; __any_sync(0xffffffffu, pending != 0); ++round) {
        if ((round & 63u) == 63u && __any_sync(0xffffffffu, gtime() > limit)) {
            fail(cx, code);
            break;
        }
        for (unsigned m = pending; m; m &= m - 1) {
            const int j = __ffs(m) - 1, i = cx.ctid + j * kCons;
            const u64 w = ld_tag(src + i);
            if (tag_is(w, ep)) {
                dst[i] = tag_val(w);
                pending &= ~(1u << j);
            }
        }
    }
    return cons_and(!cx.failed);
}

// Poll the accumulator at src (ncopy copies of E words; copy c collects the
// units u with u % ncopy == c of the nunits contributors) until every word
// holds its count, then x[i] = x[i] + (sum over copies in order + bias[i]) in
// xres and xs.  The bias is loaded before the first round, so no load waits
// after the accumulator turns ready.  The copies' fixed-point values are added
// as integers (exact), then rounded to float once.  Rounds per warp, one
// barrier at the end, as in poll_vec.  All consumer threads.
__device__ __forceinline__ bool poll_acc(Cx &cx, const u64 *src, int ncopy, int nunits, const float *bias, int E,
                                         int code) {
    const u64 limit = gtime() + cx.p->timeout_ns;
    unsigned pending = 0;
    float bv[kMaxJ];
#pragma unroll
    for (int j = 0; j < kMaxJ; ++j) {
        const int i = cx.ctid + j * kCons;
        bv[j] = i < E ? __ldg(bias + i) : 0.0f;
        if (i < E) pending |= 1u << j;
    }
    if (cx.failed) pending = 0;
    for (unsigned round = 0; __any_sync(0xffffffffu, pending != 0); ++round) {
        if ((round & 63u) == 63u && __any_sync(0xffffffffu, gtime() > limit)) {
            fail(cx, code);
            break;
        }
#pragma unroll
        for (int j = 0; j < kMaxJ; ++j) {
            if (!(pending & (1u << j))) continue;
            const int i = cx.ctid + j * kCons;
            u64 w[kAccCopies];
            bool ready = true;
#pragma unroll
            for (int c = 0; c < kAccCopies; ++c) {
                if (c >= ncopy) break;
                w[c] = ld_tag(src + (size_t)c * E + i);
                ready = ready && acc_count(w[c]) == (unsigned)((nunits - c + ncopy - 1) / ncopy);
            }
            if (ready) {   // the copies' fixed-point values summed exactly, then one rounding
                long long s = (long long)(w[0] - ((u64)acc_count(w[0]) << 55));
#pragma unroll
                for (int c = 1; c < kAccCopies; ++c)
                    if (c < ncopy) s += (long long)(w[c] - ((u64)acc_count(w[c]) << 55));
                const float v = __ll2float_rn(s) * 2.3283064365386963e-10f;
                const float x = cx.s.xres[i] + (v + bv[j]);
                cx.s.xres[i] = x;
                cx.s.xs[i] = x;
                pending &= ~(1u << j);
            }
        }
    }
    return cons_and(!cx.failed);
}

// Per-thread sums of xs[0..n) and of its squares, in a fixed order.
__device__ __forceinline__ void ln_sums(const Cx &cx, int n, float &s, float &q) {
    s = 0.0f;
    q = 0.0f;
    for (int i = cx.ctid; i < n; i += kCons) {
        const float v = cx.s.xs[i];
        s += v;
        q = fmaf(v, v, q);
    }
}
// LayerNorm statistics (math.cl:297-308) from the CTA totals of x and x * x:
// mean and rstd = 1 / sqrt(var + 1e-5).  The one-pass variance is taken in
// fp32; it loses precision only when |mean| is many times the spread of x.
__device__ __forceinline__ void ln_finish(float S, float Q, float inv_n, float &mean, float &rstd) {
    mean = S * inv_n;
    const float var = fmaxf(Q * inv_n - mean * mean, 0.0f);
    rstd = rsqrtf(var + 1e-5f);
}
// LayerNorm statistics of xs[0..n) in every consumer thread.  One barrier.
__device__ __forceinline__ void ln_stats(Cx &cx, int n, float &mean, float &rstd) {
    float s, q;
    ln_sums(cx, n, s, q);
    s = warp_sum(s);
    q = warp_sum(q);
    float *st = cx.s.red + kRedLn;
    if (cx.lane == 0) {
        st[cx.warp] = s;
        st[16 + cx.warp] = q;
    }
    cons_sync();
    // each half-warp sums the kWarps partials (both halves end with the totals)
    const int h = cx.lane & 15;
    float S = h < kWarps ? st[h] : 0.0f, Q = h < kWarps ? st[16 + h] : 0.0f;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        S += __shfl_xor_sync(0xffffffffu, S, o);
        Q += __shfl_xor_sync(0xffffffffu, Q, o);
    }
    ln_finish(S, Q, __int_as_float(cx.s.cfg[kCfgInvE]), mean, rstd);
}

// Ring chunk cx.chunk_i + k (waits for its bytes).  On an expired wait the
// thread is marked failed and computes on whatever the slot holds; the
// phase's uniform check discards the result.
__device__ __forceinline__ const float4 *chunk_wait(Cx &cx, unsigned k = 0) {
    const unsigned i = cx.chunk_i + k, slot = i % kSlots, par = (i / kSlots) & 1u;
    if (!mbar_wait(&cx.s.full[slot], par, cx.p->timeout_ns)) fail(cx, 4);
    return reinterpret_cast<const float4 *>(cx.s.ring + (size_t)slot * kSlotBytes);
}
// Release the next n chunks to the producer (each consumer warp arrives once).
__device__ __forceinline__ void chunk_done(Cx &cx, unsigned n = 1) {
    __syncwarp();
    if (cx.lane == 0)
        for (unsigned k = 0; k < n; ++k) mbar_arrive(&cx.s.empty[(cx.chunk_i + k) % kSlots]);
    cx.chunk_i += n;
}

// One strip unit of K weight rows plus its bias row and column-sum row, for
// its cw columns (4 CG with CG in 1..6 or 8, so that CG divides kCons), with
// the LayerNorm folded in:
// y = rstd * (xs . W' - mean * colsum(W')) + b', the statistics reduced in the
// same pass as the products (one barrier for the whole unit).  The result is
// in threads ctid < cw.  Thread (rg, cg) = (ctid / CG, ctid % CG) takes rows
// rg + i RG (i < 3, and i = 3 where the chunk has it) of float4 column group
// cg: in a chunk of RPC rows its weights are float4s ctid + i kCons (3 RG <=
// RPC <= 4 RG at every width).  Chunks of weight rows only are taken two at a
// time without masks; the chunk with the bias and column-sum rows is masked.
__device__ __forceinline__ float strip_unit(Cx &cx, int K, int geo) {
    const int *gm = cx.s.cfg + geo;
    const int CG = gm[0];                           // float4 column groups (cw / 4)
    const int RG = gm[1];                           // row groups (RG * CG == kCons)
    const int RPC = gm[2];                          // rows per chunk
    const int cw = gm[5];
    const int rg = mdiv(cx.ctid, gm[4]), t = cx.ctid;
    const int rows = K + 2;
    const bool has4 = rg + 3 * RG < RPC;
    const float *xs = cx.s.xs;
    float s, q;
    ln_sums(cx, K, s, q);
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    float bias = 0.0f, csum = 0.0f;
    const int nfull = gm[3];   // chunks of weight rows only (K / RPC)
    int c = 0, r0 = 0;
    for (; c + 1 < nfull; c += 2, r0 += 2 * RPC) {
        const float4 *w = chunk_wait(cx, 0), *v = chunk_wait(cx, 1);
        const float *x = xs + r0 + rg, *y = x + RPC;
        float4 w0 = w[t], w1 = w[t + kCons], w2 = w[t + 2 * kCons], w3 = make_float4(0.f, 0.f, 0.f, 0.f);
        float4 v0 = v[t], v1 = v[t + kCons], v2 = v[t + 2 * kCons], v3 = w3;
        float x3 = 0.0f, y3 = 0.0f;
        if (has4) {
            w3 = w[t + 3 * kCons];
            v3 = v[t + 3 * kCons];
            x3 = x[3 * RG];
            y3 = y[3 * RG];
        }
        fma4(a0, x[0], w0);
        fma4(a1, x[RG], w1);
        fma4(a0, x[2 * RG], w2);
        fma4(a1, x3, w3);
        fma4(a0, y[0], v0);
        fma4(a1, y[RG], v1);
        fma4(a0, y[2 * RG], v2);
        fma4(a1, y3, v3);
        chunk_done(cx, 2);
    }
    for (; r0 < rows; r0 += RPC) {
        const float4 *w = chunk_wait(cx);
        const int nr = min(RPC, rows - r0);
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int r = rg + it * RG;
            if (r < nr && r0 + r < K) fma4(it & 1 ? a1 : a0, xs[r0 + r], w[t + it * kCons]);
        }
        if (t < cw) {   // the bias and column-sum rows (possibly in different chunks)
            const float *ch = reinterpret_cast<const float *>(w);
            if (K >= r0 && K < r0 + nr) bias = ch[(K - r0) * cw + t];
            if (K + 1 >= r0 && K + 1 < r0 + nr) csum = ch[(K + 1 - r0) * cw + t];
        }
        chunk_done(cx);
    }
    tr_stamp(cx);
    float4 acc = make_float4(a0.x + a1.x, a0.y + a1.y, a0.z + a1.z, a0.w + a1.w);
    // Lanes congruent mod CG hold the same column group ((32 warp + lane) % CG):
    // fold them into lanes 0..CG-1 of the warp, then add across warps.
    for (int o = CG; o < 32; o <<= 1) {
        const float4 u = make_float4(__shfl_down_sync(0xffffffffu, acc.x, o), __shfl_down_sync(0xffffffffu, acc.y, o),
                                     __shfl_down_sync(0xffffffffu, acc.z, o), __shfl_down_sync(0xffffffffu, acc.w, o));
        if (cx.lane + o < 32) {
            acc.x += u.x;
            acc.y += u.y;
            acc.z += u.z;
            acc.w += u.w;
        }
    }
    s = warp_sum(s);
    q = warp_sum(q);
    float *red = cx.s.red + (cx.upar & 1) * kRedHalf;   // [warp][32] products, then [480 + 2 warp] sums
    cx.upar ^= 1u;
    if (cx.lane < CG) reinterpret_cast<float4 *>(red)[cx.warp * 8 + (cx.warp * 32 + cx.lane) % CG] = acc;
    if (cx.lane == 0) {
        red[480 + 2 * cx.warp] = s;
        red[481 + 2 * cx.warp] = q;
    }
    cons_sync();
    tr_stamp(cx);
    float y = 0.0f;
    if (t < cw) {
        float tt[kWarps];
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tt[w] = red[w * 32 + t];
#pragma unroll
        for (int st = 1; st < kWarps; st <<= 1)
#pragma unroll
            for (int w = 0; w + st < kWarps; w += 2 * st) tt[w] += tt[w + st];
        float S = 0.0f, Q = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            S += red[480 + 2 * w];
            Q += red[481 + 2 * w];
        }
        float mean, rstd;
        ln_finish(S, Q, __int_as_float(cx.s.cfg[kCfgInvE]), mean, rstd);
        y = fmaf(rstd, fmaf(-mean, csum, tt[0]), bias);
    }
    return y;
}

// One row block: y[n] = sum_r a[r] W[r][n] for `rows` rows of NB floats
// streamed from the ring (NB a multiple of 4, NB / 4 <= kCons, NB * 4 <=
// kSlotBytes), each y[n] added to the accumulator word dst[n].  Thread
// (rg, cg) = (ctid / CG, ctid % CG) sums rows rg, rg + RG, ... of float4
// column group cg (float4s ctid, ctid + RG CG, ... of a chunk); the RG
// partials are then added in a fixed order.  a is in shared memory.
__device__ __forceinline__ void block_unit(Cx &cx, const float *a, int rows, int geo, u64 *dst) {
    const int *gm = cx.s.cfg + geo;
    const int RG = gm[1], RPC = gm[2], NB = gm[4], RGCG = gm[5];   // RPC: rows per chunk
    const int t = cx.ctid, rg = mdiv(t, gm[3]);
    const bool act = t < RGCG;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    for (int r0 = 0; r0 < rows; r0 += RPC) {
        const float4 *w = chunk_wait(cx);
        const int nr = min(RPC, rows - r0);
        if (act) {
            const float *ar = a + r0 + rg;
            int k = 0;
            for (; rg + (k + 3) * RG < nr; k += 4) {   // four rows in flight
                const float4 w0 = w[t + k * RGCG], w1 = w[t + (k + 1) * RGCG], w2 = w[t + (k + 2) * RGCG],
                             w3 = w[t + (k + 3) * RGCG];
                fma4(a0, ar[k * RG], w0);
                fma4(a1, ar[(k + 1) * RG], w1);
                fma4(a0, ar[(k + 2) * RG], w2);
                fma4(a1, ar[(k + 3) * RG], w3);
            }
            for (; rg + k * RG < nr; ++k) fma4(k & 1 ? a1 : a0, ar[k * RG], w[t + k * RGCG]);
        }
        chunk_done(cx);
    }
    tr_stamp(cx);
    float *part = cx.s.part;   // [RG][NB], RG * NB <= 4 * kCons <= kPart
    if (act) reinterpret_cast<float4 *>(part)[t] = make_float4(a0.x + a1.x, a0.y + a1.y, a0.z + a1.z, a0.w + a1.w);
    cons_sync();
    for (int n = t; n < NB; n += kCons) {
        float y = part[n];
        for (int g = 1; g < RG; ++g) y += part[g * NB + n];
        acc_add(dst + n, y, cx.p->err);
    }
}

__device__ __forceinline__ unsigned epoch_of(const MegaParams &p, int step, int layer, int ph) {
    return p.epoch0 + (unsigned)step * (unsigned)((p.L + 1) * 8) + (unsigned)(layer * 8 + ph);
}
// Accumulator of layer l in step `step`: w = 0 after B (attention
// projection, one copy of E words), w = 1 after D (MLP projection,
// kAccCopies copies of E words; D unit u adds into copy u % kAccCopies, which
// cuts the contention on each word).
__device__ __forceinline__ u64 *acc_of(const MegaParams &p, int step, int l, int w) {
    return p.acc + ((size_t)(step * p.L + l) * (1 + kAccCopies) + (w ? 1 : 0)) * p.E;
}

// ---- producer: the CTA's weight stream for all steps ------------------------------------
// Streams `bytes` from src in whole rows of row_bytes per ring chunk.
__device__ __forceinline__ bool produce(Cx &cx, const char *src, size_t bytes, size_t row_bytes, unsigned &i,
                                        u64 policy) {
    const MegaParams &p = *cx.p;
    const size_t chunk = (kSlotBytes / row_bytes) * row_bytes;
    for (size_t off = 0; off < bytes; off += chunk) {
        const unsigned nb = (unsigned)(bytes - off < chunk ? bytes - off : chunk);
        const unsigned slot = i % kSlots;
        if (!mbar_wait_idle(&cx.s.empty[slot], ((i / kSlots) & 1u) ^ 1u, p.timeout_ns)) {
            fail(cx, 1);
            return false;
        }
        // Keep at most max_inflight copies outstanding.
        if (i >= (unsigned)p.max_inflight) {
            const unsigned j = i - p.max_inflight;
            if (!mbar_wait_idle(&cx.s.full[j % kSlots], (j / kSlots) & 1u, p.timeout_ns)) {
                fail(cx, 1);
                return false;
            }
        }
        mbar_expect_tx(&cx.s.full[slot], nb);
        bulk_load(cx.s.ring + (size_t)slot * kSlotBytes, src + off, nb, &cx.s.full[slot], policy);
        ++i;
    }
    return true;
}

__device__ __forceinline__ void producer(Cx &cx, const Sched &S) {
    const MegaParams &p = *cx.p;
    u64 policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    const int E = p.E, L = p.L, G = S.G, cwq = p.cw_qkv, cwf = p.cw_fc, NB = E / p.nq;
    const size_t ua = (size_t)(E + 2) * cwq * 4, ub = (size_t)64 * NB * 4;
    const size_t ud_strip = (size_t)(E + 2) * cwf * 4, ud_block = (size_t)cwf * E * 4;
    unsigned i = 0;
    bool ok = true;
    for (int step = 0; step < p.n_steps && ok; ++step) {
        for (int l = 0; l < L && ok; ++l) {
            const char *pa = reinterpret_cast<const char *>(p.packed + p.layer_off[l * 3 + 0]);
            const char *pb = reinterpret_cast<const char *>(p.packed + p.layer_off[l * 3 + 1]);
            const char *pd = reinterpret_cast<const char *>(p.packed + p.layer_off[l * 3 + 2]);
            for (int u = S.a_first(l, cx.cta); u < S.nA && ok; u += G) ok = produce(cx, pa + u * ua, ua, cwq * 4, i, policy);
            for (int u = S.b_first(l, cx.cta); u < S.nB && ok; u += G)
                ok = produce(cx, pb + u * ub, ub, (size_t)NB * 4, i, policy);
            for (int u = S.d_first(l, cx.cta); u < S.nD && ok; u += G) {
                const char *src = pd + u * (ud_strip + ud_block);
                ok = produce(cx, src, ud_strip, cwf * 4, i, policy) &&
                     produce(cx, src + ud_strip, ud_block, (size_t)E * 4, i, policy);
            }
        }
        const char *lm = reinterpret_cast<const char *>(p.lm);
        const int r1 = (int)((long long)(cx.cta + 1) * p.V / G);
        for (int v0 = (int)((long long)cx.cta * p.V / G); v0 < r1 && ok; v0 += p.lm_rows) {
            const size_t bytes = (size_t)min(p.lm_rows, r1 - v0) * E * sizeof(float);
            ok = produce(cx, lm + (size_t)v0 * E * sizeof(float), bytes, (size_t)E * 4, i, policy);
        }
    }
    // Every copy issued must land before the CTA may exit (the ring is its destination).
    for (unsigned j = i > kSlots ? i - kSlots : 0; j < i; ++j)
        mbar_wait(&cx.s.full[j % kSlots], (j / kSlots) & 1u, p.timeout_ns);
}

// ---- consumer units --------------------------------------------------------------------

// Single-query attention of head h over positions 0..pos (attn_scores_1q,
// attn_softmax_1q, attn_out_1q, math.cl:388-476) into atta[0..64).  The
// cached keys and values are read from the cache (L2); the first pass of keys
// is loaded before the wait for q.  The key and value at pos come from the
// qkv vector.
//
// Up to p.split_t positions, every B unit of head h (slice j of nq) runs the
// whole attention of the head.  Past it (long contexts, where one SM reading
// the head's whole K and V is the slow part) unit j takes only keys
// [j c, (j + 1) c), c = ceil(T / nq), and publishes its partial (running max
// m_j, sum l_j of exp(s - m_j), unnormalised output o_j) as tagged words;
// each unit then polls the head's nq partials and merges them in slice order
// (M = max m_j, out = sum_j o_j e^(m_j - M) / sum_j l_j e^(m_j - M)), so every
// unit of the head derives the same output (flash-decoding).
__device__ __forceinline__ bool attention(Cx &cx, int h, int jslice, int step, int l, int pos) {
    const MegaParams &p = *cx.p;
    const int E = p.E, T = pos + 1;
    const bool split = T > p.split_t;
    const int nq = p.nq;
    int k0 = 0, k1 = T;
    if (split) {
        const int c = (T + nq - 1) / nq;
        k0 = min(T, jslice * c);
        k1 = min(T, k0 + c);
    }
    const unsigned ep_in = epoch_of(p, step, l, 0);
    float *q = cx.s.attq, *pr = cx.s.attp, *a = cx.s.atta, *part = cx.s.part;
    float *rb = cx.s.red + kRedAtt;   // [0, 15) warp maxima, [16, 31) warp sums
    const int key = cx.ctid >> 2, k4 = cx.ctid & 3;   // score pass: 4 threads per key, 16 dims each
    const int dq = cx.ctid & 15, grp = cx.ctid >> 4;  // P.V pass: float4 dq of 64 dims, key group grp
    const size_t hb = (size_t)l * p.layer_stride + (size_t)h * p.max_seq * 64;
    const float4 *K4 = reinterpret_cast<const float4 *>(p.kc + hb);
    const float4 *V4 = reinterpret_cast<const float4 *>(p.vc + hb);
    float4 kr[4];
    {
        const int j = k0 + key;
        const bool c = j < k1 && j != pos;
#pragma unroll
        for (int t = 0; t < 4; ++t) kr[t] = c ? K4[(size_t)j * 16 + k4 * 4 + t] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    {   // q, k, v of head h at pos
        const u64 limit = gtime() + cx.p->timeout_ns;
        bool pend = cx.ctid < 192 && !cx.failed;
        for (unsigned round = 0; __any_sync(0xffffffffu, pend); ++round) {
            if ((round & 63u) == 63u && __any_sync(0xffffffffu, gtime() > limit)) {
                fail(cx, 5);
                break;
            }
            if (pend) {
                const u64 w = ld_tag(p.t_qkv + (cx.ctid >> 6) * E + h * 64 + (cx.ctid & 63));
                if (tag_is(w, ep_in)) {
                    q[cx.ctid] = tag_val(w);
                    pend = false;
                }
            }
        }
        if (!cons_and(!cx.failed)) return false;
    }
    tr_inputs(cx, 1);
    // scores s_j = q . k_j / 8 (the key at pos comes from the qkv vector)
    float mloc = -FLT_MAX;
    for (int j0 = k0; j0 < k1; j0 += kKeysPerPass) {
        const int j = j0 + key;
        if (j0 > k0) {
            const bool c = j < k1 && j != pos;
#pragma unroll
            for (int t = 0; t < 4; ++t) kr[t] = c ? K4[(size_t)j * 16 + k4 * 4 + t] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (j == pos) {
#pragma unroll
            for (int t = 0; t < 4; ++t)
                kr[t] = make_float4(q[64 + k4 * 16 + 4 * t], q[64 + k4 * 16 + 4 * t + 1], q[64 + k4 * 16 + 4 * t + 2],
                                    q[64 + k4 * 16 + 4 * t + 3]);
        }
        const float *qq = q + k4 * 16;
        float s = 0.0f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            s = fmaf(kr[t].x, qq[4 * t], s);
            s = fmaf(kr[t].y, qq[4 * t + 1], s);
            s = fmaf(kr[t].z, qq[4 * t + 2], s);
            s = fmaf(kr[t].w, qq[4 * t + 3], s);
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s *= 0.125f;   // 1 / sqrt(64)
        if (j < k1) {
            if (k4 == 0) pr[j - k0] = s;
            mloc = fmaxf(mloc, s);
        }
    }
    float m = warp_max(mloc);
    if (cx.lane == 0) rb[cx.warp] = m;
    cons_sync();
    m = rb[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) m = fmaxf(m, rb[w]);
    float lsum = 0.0f;
    for (int j = k0 + cx.ctid; j < k1; j += kCons) {
        const float e = expf(pr[j - k0] - m);
        pr[j - k0] = e;
        lsum += e;
    }
    lsum = warp_sum(lsum);
    if (cx.lane == 0) rb[16 + cx.warp] = lsum;
    cons_sync();
    tr_stamp(cx);
    float Lt = rb[16];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) Lt += rb[16 + w];
    // P.V: thread (grp, dq) sums keys grp, grp + kPvGroups, ... of dims 4 dq .. 4 dq + 3
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = k0 + grp; j0 < k1; j0 += 8 * kPvGroups) {   // eight keys per round: their rows in flight together
        float4 vv[8];
        float pp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + u * kPvGroups;
            const bool in = j < k1;
            vv[u] = (in && j != pos) ? V4[(size_t)j * 16 + dq] : make_float4(0.f, 0.f, 0.f, 0.f);
            if (j == pos)
                vv[u] = make_float4(q[128 + 4 * dq], q[128 + 4 * dq + 1], q[128 + 4 * dq + 2], q[128 + 4 * dq + 3]);
            pp[u] = in ? pr[j - k0] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) fma4(o, pp[u], vv[u]);
    }
    reinterpret_cast<float4 *>(part)[grp * 16 + dq] = o;   // [kPvGroups][64]
    cons_sync();
    float y = 0.0f;
    if (cx.ctid < 64) {
        y = part[cx.ctid];
        for (int g = 1; g < kPvGroups; ++g) y += part[g * 64 + cx.ctid];
    }
    if (split) {
        // publish this slice's (o, m, l); merge the head's nq slices in slice order.
        // pr (the probabilities) is free again after the barrier above.
        const unsigned ep1 = epoch_of(p, step, l, 1);
        u64 *ta = p.t_att + (size_t)h * nq * 66;
        if (cx.ctid < 64) st_tag(ta + jslice * 66 + cx.ctid, y, ep1);
        else if (cx.ctid == 64) st_tag(ta + jslice * 66 + 64, m, ep1);
        else if (cx.ctid == 65) st_tag(ta + jslice * 66 + 65, Lt, ep1);
        if (!poll_vec(cx, ta, pr, nq * 66, ep1, 7)) return false;
        if (cx.ctid < 64) {
            float M = -FLT_MAX;
            for (int jj = 0; jj < nq; ++jj) M = fmaxf(M, pr[jj * 66 + 64]);
            float L = 0.0f, acc = 0.0f;
            for (int jj = 0; jj < nq; ++jj) {
                const float w = expf(pr[jj * 66 + 64] - M);
                L = fmaf(pr[jj * 66 + 65], w, L);
                acc = fmaf(pr[jj * 66 + cx.ctid], w, acc);
            }
            a[cx.ctid] = acc / L;
        }
    } else if (cx.ctid < 64) {
        a[cx.ctid] = y / Lt;
    }
    cons_sync();
    tr_stamp(cx);
    return true;
}

// The units of this CTA in one half of layer l, each kind through one copy of
// its code (the loop stays in the instruction cache):
//   half 0: A units -- LN1 + c_attn strip -> tagged qkv words, and the K and
//           V columns appended to the cache at pos (split_kv,
//           math.cl:367-383); then B units -- attention of head h, then its
//           64 outputs times rows 64h.. of attn.c_proj, column slice j, into
//           the attention accumulator;
//   half 1: D units -- LN2 + c_fc strip, GELU (math.cl:21-23), then the cw
//           values times the matching cw rows of mlp.c_proj (all E outputs)
//           into the MLP accumulator.
// xs holds the input x.
__device__ __forceinline__ bool run_units(Cx &cx, const Sched &S, int step, int l, int pos, int half) {
    const MegaParams &p = *cx.p;
    const int E = p.E, t = cx.ctid;
    const int *cf = cx.s.cfg;
    for (int kind = half ? 2 : 0; kind <= (half ? 2 : 1); ++kind) {
        const int n = kind == 0 ? S.nA : kind == 1 ? S.nB : S.nD;
        int u = cf[kCfgFirst + l] - (kind == 0 ? 0 : cf[kind == 1 ? kCfgOffB : kCfgOffD]);
        if (u < 0) u += S.G;
        u64 *acc = acc_of(p, step, l, kind == 1 ? 0 : 1);
        const unsigned ep = epoch_of(p, step, l, 0);
        const int ph = kind == 0 ? 0 : kind == 1 ? 1 : 3;   // trace slot
        float *av = cx.s.atta;
        for (; u < n; u += S.G) {
            tr_begin(cx);
            int rows, geo;
            u64 *dst;
            if (kind != 1) {
                tr_inputs(cx, ph);
                const float v = strip_unit(cx, E, kind == 0 ? kGeoA : kGeoDs);
                if (kind == 0) {
                    if (t < p.cw_qkv) {
                        const int col = u * p.cw_qkv + t;
                        if (col >= E) {   // K or V of head m / 64
                            int m = col - E;
                            float *kv = m >= E ? p.vc : p.kc;
                            if (m >= E) m -= E;
                            kv[(size_t)l * p.layer_stride + ((size_t)(m >> 6) * p.max_seq + pos) * 64 + (m & 63)] = v;
                        }
                        st_tag(p.t_qkv + col, v, ep);
                    }
                    tr_end(cx, ph);
                    continue;
                }
                if (t < p.cw_fc) av[t] = gelu_f(v);
                cons_sync();
                rows = p.cw_fc;
                geo = kGeoDb;
                dst = acc + (size_t)(u % kAccCopies) * E;
            } else {
                const int h = mdiv(u, cf[kCfgMnq]), j = u - h * cf[kCfgNq];
                if (!attention(cx, h, j, step, l, pos)) return false;
                rows = 64;
                geo = kGeoB;
                dst = acc + j * cf[kGeoB + 4];
            }
            block_unit(cx, av, rows, geo, dst);
            tr_end(cx, ph);
        }
        // An expired wait inside a unit is caught at the next poll, whose exit
        // barrier also carries the failure flag.
        tr_stamp(cx);
    }
    return true;
}

}  // namespace

// kTr: the traced instantiation (phase stamps when P.trace is set); in the
// other one every trace branch folds away at compile time.
template <bool kTr>
__global__ void __launch_bounds__(kThreads, 1) mega_decode_kernel(MegaParams P) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const MegaParams &p = P;
    Cx cx;
    cx.p = &P;
    cx.cta = blockIdx.x;
    cx.warp = threadIdx.x >> 5;
    cx.lane = threadIdx.x & 31;
    cx.ctid = threadIdx.x;   // consumers: 0..479
    cx.failed = 0;
    cx.chunk_i = 0;
    cx.upar = 0;
    cx.tr = kTr && p.trace != nullptr && threadIdx.x == 0;
    cx.tl = false;
    cx.t0 = cx.tr ? gtime() : 0;
    const int G = gridDim.x, E = p.E, L = p.L;
    unsigned char *sp = smem_raw;
    cx.s.ring = sp;
    sp += kSlots * kSlotBytes;
    cx.s.full = reinterpret_cast<u64 *>(sp);
    cx.s.empty = cx.s.full + kSlots;
    sp += 2 * kSlots * sizeof(u64);
    cx.s.trc = reinterpret_cast<u64 *>(sp);
    sp += kTraceSlots * sizeof(u64);
    cx.s.red = reinterpret_cast<float *>(sp);
    sp += kRedFloats * sizeof(float);
    cx.s.attp = reinterpret_cast<float *>(sp);
    sp += kMaxKeys * sizeof(float);
    cx.s.attq = reinterpret_cast<float *>(sp);
    sp += 192 * sizeof(float);
    cx.s.atta = reinterpret_cast<float *>(sp);
    sp += 64 * sizeof(float);
    cx.s.part = reinterpret_cast<float *>(sp);
    sp += kPart * sizeof(float);
    cx.s.xres = reinterpret_cast<float *>(sp);
    sp += (size_t)E * sizeof(float);
    cx.s.xs = reinterpret_cast<float *>(sp);   // 16-byte aligned: the LM rows read it as float4
    sp += (size_t)(E + 4) * sizeof(float);
    cx.s.cfg = reinterpret_cast<int *>(sp);    // last, so that it moves no other array

    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&cx.s.full[i], 1);
            mbar_init(&cx.s.empty[i], kWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < kTraceSlots; i += kThreads) cx.s.trc[i] = 0;

    Sched S;
    S.nA = 3 * E / p.cw_qkv;
    S.nB = p.NH * p.nq;
    S.nD = p.F / p.cw_fc;
    S.per_layer = S.nA + S.nB + S.nD;
    S.G = G;
    if (threadIdx.x == 0) {   // the per-CTA constants: every runtime division of the units, once
        int *cf = cx.s.cfg;
        for (int s = 0; s < 2; ++s) {   // strips of width cw over E rows (+ bias and column-sum rows)
            const int cw = s ? p.cw_fc : p.cw_qkv, CG = cw >> 2, RPC = kSlotBytes / (cw * 4);
            int *g = cf + (s ? kGeoDs : kGeoA);
            g[0] = CG;
            g[1] = kCons / CG;
            g[2] = RPC;
            g[3] = E / RPC;
            g[4] = magic20(CG);
            g[5] = cw;
        }
        for (int b = 0; b < 2; ++b) {   // blocks of NB columns
            const int NB = b ? E : E / p.nq, CG = NB >> 2;
            int *g = cf + (b ? kGeoDb : kGeoB);
            g[0] = CG;
            g[1] = kCons / CG;
            g[2] = kSlotBytes / (NB * 4);
            g[3] = magic20(CG);
            g[4] = NB;
            g[5] = (kCons / CG) * CG;
        }
        cf[kCfgMnq] = magic20(p.nq);
        cf[kCfgNq] = p.nq;
        cf[kCfgOffB] = S.nA % G;
        cf[kCfgOffD] = (S.nA + S.nB) % G;
        cf[kCfgInvE] = __float_as_int(1.0f / (float)E);
        cf[kCfgLm0] = (int)((long long)cx.cta * p.V / G);
        cf[kCfgLm1] = (int)((long long)(cx.cta + 1) * p.V / G);
        for (int l = 0; l < L; ++l) cf[kCfgFirst + l] = S.first(l * S.per_layer, cx.cta);
    }
    __syncthreads();

    if (cx.warp == kWarps) {   // producer warp: one thread issues, the rest are idle
        if (cx.lane == 0) producer(cx, S);
        return;
    }

    // ======================= consumer warps =======================
    float *xs = cx.s.xs;
    int tok = p.state->token, pos = p.state->pos;
    const int step_base = p.state->step, min_new = p.state->min_new;
    for (int step = 0; step < p.n_steps; ++step) {
        cx.tl = kTr && cx.tr && cx.cta == 0 && step == min(3, p.n_steps - 1);
        // the host bounds the steps so that pos stays inside the cache; clamp regardless
        if (!G2_BOUNDS(tok >= 0 && tok < p.V && pos >= 0 && pos < p.max_seq, 106)) {
            tok = min(max(tok, 0), p.V - 1);
            pos = min(max(pos, 0), p.max_seq - 1);
        }
        // x = wte[tok] + wpe[pos] (embed, math.cl:333)
        for (int i = cx.ctid; i < E; i += kCons) {
            const float x = p.wte[(size_t)tok * E + i] + p.wpe[(size_t)pos * E + i];
            xs[i] = x;
            cx.s.xres[i] = x;
        }
        cons_sync();
        // Per layer: A and B units on x; x += attention; D units; x += MLP.
        // The last pass (l == L) only takes in the MLP output of the last layer.
        float lg[kMaxJ], lb[kMaxJ];   // LN_f gamma and beta, loaded before the last layer's exchange
        for (int l = 0; l <= L; ++l) {
            for (int half = 0; half < 2; ++half) {
                if (l == L && half == 1) break;
                if (l > 0 || half == 1) {   // x += (MLP of layer l - 1 | attention of layer l) + bias
                    const int lp = half ? l : l - 1;
                    if (l == L) {
#pragma unroll
                        for (int j = 0; j < kMaxJ; ++j) {
                            const int i = cx.ctid + j * kCons;
                            lg[j] = i < E ? __ldg(p.lnf_g + i) : 0.0f;
                            lb[j] = i < E ? __ldg(p.lnf_b + i) : 0.0f;
                        }
                    }
                    tr_begin(cx);
                    if (!poll_acc(cx, acc_of(p, step, lp, 1 - half), half ? 1 : kAccCopies, half ? p.NH : S.nD,
                                  half ? p.layers[lp].proj_b : p.layers[lp].fc2_b, E, half ? 6 : 2))
                        goto out;
                    tr_inputs(cx, half ? 4 : l == L ? 5 : 2);
                }
                if (l == L) break;
                if (!run_units(cx, S, step, l, pos, half)) goto out;
            }
        }
        // ---------------- LN_f + LM head + greedy argmax ----------------
        {
            // this CTA's wte rows [v0, r1): an equal share, in units of up to lm_rows rows
            int v0 = cx.s.cfg[kCfgLm0];
            const int r1 = cx.s.cfg[kCfgLm1];
            const bool forbid = (step_base + step) < min_new;
            float best = -FLT_MAX;
            int besti = INT_MAX;
            if (v0 < r1) {
                tr_begin(cx);
                tr_inputs(cx, 5);
                float mean, rstd;
                ln_stats(cx, E, mean, rstd);
                // normalise in place with gamma / beta (math.cl:310); the rows read it 16 times
#pragma unroll
                for (int j = 0; j < kMaxJ; ++j) {
                    const int i = cx.ctid + j * kCons;
                    if (i < E) xs[i] = (xs[i] - mean) * rstd * lg[j] + lb[j];
                }
                cons_sync();
                // A unit holds up to kWarps rows over one or more chunks: all of its
                // chunks are waited for, then warp w takes row w.
                const int RPC = kSlotBytes / (E * 4);
                const int E4 = E / 4;
                const float4 *x4 = reinterpret_cast<const float4 *>(xs);
                for (; v0 < r1; v0 += p.lm_rows) {
                    const int rows = min(p.lm_rows, r1 - v0);
                    const int nch = (rows + RPC - 1) / RPC;
                    for (int k = 0; k < nch; ++k) chunk_wait(cx, k);
                    if (cx.warp < rows) {
                        const float4 *w4 = reinterpret_cast<const float4 *>(
                                               cx.s.ring + (size_t)((cx.chunk_i + cx.warp / RPC) % kSlots) * kSlotBytes) +
                                           (size_t)(cx.warp % RPC) * E4;
                        float s0 = 0.0f, s1 = 0.0f;
                        int j = cx.lane;
                        for (; j + 32 < E4; j += 64) {
                            const float4 w = w4[j], xv = x4[j], w2 = w4[j + 32], xv2 = x4[j + 32];
                            s0 = fmaf(w.x, xv.x, s0);
                            s1 = fmaf(w2.x, xv2.x, s1);
                            s0 = fmaf(w.y, xv.y, s0);
                            s1 = fmaf(w2.y, xv2.y, s1);
                            s0 = fmaf(w.z, xv.z, s0);
                            s1 = fmaf(w2.z, xv2.z, s1);
                            s0 = fmaf(w.w, xv.w, s0);
                            s1 = fmaf(w2.w, xv2.w, s1);
                        }
                        if (j < E4) {
                            const float4 w = w4[j], xv = x4[j];
                            s0 = fmaf(w.x, xv.x, s0);
                            s0 = fmaf(w.y, xv.y, s0);
                            s0 = fmaf(w.z, xv.z, s0);
                            s0 = fmaf(w.w, xv.w, s0);
                        }
                        const float sacc = warp_sum(s0 + s1);
                        const int v = v0 + cx.warp;
                        if (cx.lane == 0) p.logits[v] = sacc;
                        if (!(forbid && v == kEos) && better(sacc, v, best, besti)) {
                            best = sacc;
                            besti = v;
                        }
                    }
                    chunk_done(cx, nch);
                }
                if (!cons_and(!cx.failed)) goto out;
            }
            tr_end(cx, 5);
            // this CTA's best -> tagged partial; then every CTA reduces all partials
            float *rv = cx.s.red + kRedArg;
            int *ri = reinterpret_cast<int *>(cx.s.red) + kRedArg + 16;
            cons_sync();
            if (cx.lane == 0) {
                rv[cx.warp] = best;
                ri[cx.warp] = besti;
            }
            cons_sync();
            // The partials alternate between two halves by step parity: a CTA whose
            // own work is not on another CTA's path may still be reading step s
            // when that CTA writes step s + 1; step s + 2 needs its step s + 1 partial.
            const unsigned ep = epoch_of(p, step, L, 0);
            u64 *tb = p.t_best + (size_t)(step & 1) * 2 * G;
            if (cx.warp == 0) {   // the CTA's best of its warps' bests
                best = cx.lane < kWarps ? rv[cx.lane] : -FLT_MAX;
                besti = cx.lane < kWarps ? ri[cx.lane] : INT_MAX;
                warp_argmax(best, besti);
                if (cx.lane == 0) {
                    // release: this CTA's K/V rows of the step (ordered before this
                    // thread by the barrier above) become visible with the partial
                    __threadfence();
                    st_tag(tb + 2 * cx.cta, best, ep);
                    st_tag(tb + 2 * cx.cta + 1, __int_as_float(besti), ep);
                }
            }
            float *bv = cx.s.part;                                  // 2 * G <= kPart floats
            int *bi = reinterpret_cast<int *>(cx.s.attq);           // [0] token
            tr_begin(cx);
            if (!poll_vec(cx, tb, bv, 2 * G, ep, 3)) goto out;
            __threadfence();   // acquire: every CTA's K/V rows of this step, for the steps that follow
            tr_inputs(cx, 6);
            if (cx.warp == 0) {   // the best of all CTAs' bests: lanes take CTAs c = lane mod 32
                float gb = -FLT_MAX;
                int gi = INT_MAX;
                for (int c = cx.lane; c < G; c += 32) {
                    const int ix = __float_as_int(bv[2 * c + 1]);
                    if (better(bv[2 * c], ix, gb, gi)) {
                        gb = bv[2 * c];
                        gi = ix;
                    }
                }
                warp_argmax(gb, gi);
                if (gi == INT_MAX) gi = 0;   // every logit NaN: never hand an invalid id to the next step
                if (cx.lane == 0) bi[0] = gi;
                if (cx.cta == 0 && cx.lane == 0) {
                    p.out_tokens[step_base + step] = gi;
                    if (step == p.n_steps - 1) {
                        p.result[0] = gi;
                        p.result[1] = __float_as_int(gb);
                    }
                }
            }
            cons_sync();
            tok = bi[0];
            pos += 1;
            cons_sync();
            tr_end(cx, 6);
        }
    }
    if (cx.cta == 0 && cx.ctid == 0) {
        p.state->token = tok;
        p.state->pos = pos;
        p.state->step = step_base + p.n_steps;
    }
out:
    if (cx.tr) {
        u64 *t = p.trace + (size_t)cx.cta * kTraceSlots;
        for (int i = 0; i < kTraceSlots; ++i) t[i] = cx.s.trc[i];
        t[17] = gtime() - cx.t0;
    }
    return;
}

size_t mega_smem_bytes(int E) {
    return (size_t)kSlots * kSlotBytes + 2 * kSlots * sizeof(unsigned long long) + kTraceSlots * sizeof(unsigned long long) +
           (kRedFloats + kMaxKeys + 192 + 64 + kPart + kCfgInts) * sizeof(float) + (size_t)(2 * E + 4) * sizeof(float);
}
int mega_threads() { return kThreads; }
const void *mega_kernel_ptr(bool traced) {
    return traced ? (const void *)mega_decode_kernel<true> : (const void *)mega_decode_kernel<false>;
}
int mega_slot_bytes() { return kSlotBytes; }
int mega_max_keys() { return kMaxKeys; }

#ifdef G2_CHECK
int check_flag_mega() {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g2_check_flag, sizeof(int));
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g2_check_flag, &z, sizeof(int));
    }
    return v;
}
#else
int check_flag_mega() { return 0; }
#endif

}  // namespace g2
