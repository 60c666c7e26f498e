// g2_mega.cu -- persistent B = 1 decode kernel (fp32): every layer and every
// greedy step of a generation in one cooperative launch.
//
// It replaces the per-token kernel sequence of decode() (main.c:1792-1833)
// and the greedy branch of sample_next_token (main.c:1898-1904).
//
// Structure (one CTA per SM; 15 consumer warps + 1 producer warp):
//
//  * Weights are repacked at load time into "units": a column strip of a
//    projection over its full K (so no output needs a cross-CTA reduction),
//    followed by a bias row and a column-sum row.  For qkv and fc the
//    preceding LayerNorm's gamma and beta are folded in (W' = diag(gamma) W,
//    b' = b + beta W), and the normalisation itself is applied after the
//    products: LN(x) W' + b' = rstd (x W' - mean colsum(W')) + b'.  The strip
//    width of each projection (4 to 32 columns) is the narrowest that gives
//    every CTA at most one unit per phase.  LM-head units are 16-row blocks of
//    wte.  Unit g of a step belongs to CTA g % gridDim.x, counting across all
//    phases of the step, so the CTAs share each layer's bytes evenly.
//  * The producer warp streams the CTA's units, in consumption order, through
//    an 8-slot shared-memory ring with cp.async.bulk (mbarrier full/empty,
//    L2 evict-first).  The stream is the same every step and waits on no
//    activation, so it runs ahead across layer and token boundaries.
//  * Activations move between CTAs as 64-bit words (epoch << 32 | float
//    bits).  A consumer polls the vector it needs until every word carries the
//    epoch of the producing phase: readiness costs one L2 round trip, with no
//    grid barrier and no atomics.  A buffer is rewritten only after every
//    reader of its previous contents has produced the outputs the rewrite
//    depends on, so a reader never sees a newer epoch than it waits for.  The
//    values a phase needs besides its input vector (residuals) are fetched in
//    the same polling pass; nothing else on the critical path reads DRAM.
//  * Per layer: A = LN1 + qkv + K/V append, B = attention per (head, 64-key
//    chunk) with online-softmax partials (the current position's K/V come
//    from the qkv vector itself), C = combine + proj + residual, D = LN2 +
//    fc + GELU, E = fc2 + residual.  Then LN_f + LM head with a per-CTA
//    argmax; every CTA reads all CTA partials and derives the next token.
//    The K/V rows a step appends are read by later steps only; one fence pair
//    per step at that exchange orders them.
//  * Barriers per phase are few: a strip unit takes one, which also reduces
//    the LayerNorm sums of x and x * x (double-buffered scratch; the summing
//    threads finish the statistics and store the outputs).
//  * Every wait is bounded (globaltimer, 2 s per wait).  On expiry the thread
//    records an error code; the consumer warps leave together at the next
//    uniform check, the producer stops issuing and drains its in-flight
//    copies, and the host reports G2_ERR_TIMEOUT.
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
constexpr unsigned long long kTimeoutNs = 2000000000ull;
constexpr int kConsBar = 1;                // named barrier of the consumer warps
constexpr int kMaxChunks = 16;             // attention chunks per head (1024 / 64)
constexpr int kRes = 64;                   // residual values a CTA prefetches per phase
// Reduction scratch (floats): two alternating halves for strip units, then the
// argmax partials, the attention scalars and the LayerNorm partials.
constexpr int kRedHalf = 512;
constexpr int kRedArg = 1024;              // 16 values, then 16 indices
constexpr int kRedAtt = 1056;              // 32
constexpr int kRedLn = 1088;               // 32
constexpr int kRedFloats = 1120;

typedef unsigned long long u64;

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
__device__ __forceinline__ int cons_or(int pred) {
    int r;
    asm volatile(
        "{ .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.s32 %0, 1, 0, q; }"
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
// Wait for the phase of parity `parity` to complete, for at most kTimeoutNs.
__device__ __forceinline__ bool mbar_wait(u64 *b, unsigned parity) {
    if (mbar_try(b, parity)) return true;
    const u64 limit = gtime() + kTimeoutNs;
    for (;;) {
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
__device__ __forceinline__ float gelu_f(float v) {
    return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
}

// ---- the per-step unit schedule (the same in producer and consumers) ------------------
struct Sched {
    int nA, nC, nD, nE, nLM;   // units per phase
    int per_layer;             // nA + nC + nD + nE
    int G;                     // CTAs
    // first unit of a phase starting at global unit index g0 that belongs to CTA c
    __device__ __forceinline__ int first(int g0, int c) const {
        const int r = (c - g0) % G;
        return r < 0 ? r + G : r;
    }
    __device__ __forceinline__ int count(int first, int n) const { return first < n ? (n - first + G - 1) / G : 0; }
};

struct Smem {
    float *xs;     // input vector of the current phase (max(E, F) + 1 floats)
    float *red;    // reduction scratch: 2 x [16 warps][16] unit partials, then [512,560) stats/ints
    float *att;    // attention / argmax scratch (1024 floats)
    float *res;    // residual values of this CTA's units (kRes floats)
    float *lnf;    // final LayerNorm gamma [E] and beta [E]
    u64 *trc;      // trace accumulators (thread 0 only)
    u64 *full, *empty;
    unsigned char *ring;
};

// Trace layout in shared memory (u64): [0..8) poll ns per phase, [8..16) work ns,
// [16] chunk-wait ns, [18] units, [19] chunks, [20] phase-begin stamp, [21] inputs stamp,
// [24] timeline count, [32..64) timeline stamps (CTA 0, step 0).
struct Cx {
    const MegaParams *p;
    Smem s;
    int cta, ctid, warp, lane;
    unsigned chunk_i;   // next ring chunk to consume
    unsigned upar;      // parity of the next strip unit's reduction scratch
    int failed;         // this thread saw an expired wait
    bool tr;            // tracing (consumer thread 0)
    bool tl;            // timeline stamps (CTA 0, step 0)
    u64 t0;
};

__device__ __forceinline__ void tr_stamp(Cx &cx) {
    if (cx.tl) {
        const u64 n = cx.s.trc[24];
        if (n < 32) {
            cx.s.trc[32 + n] = gtime() - cx.t0;
            cx.s.trc[24] = n + 1;
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

// Uniform deadline check of a polling loop, every 64 rounds (a barrier round).
__device__ __forceinline__ bool poll_expired(Cx &cx, unsigned round, u64 limit, int code) {
    if ((round & 63u) != 63u) return false;
    if (cons_or(gtime() > limit)) {
        fail(cx, code);
        return true;
    }
    return false;
}

// Poll n tagged words into dst until all carry `ep`, together with the
// residual words of this CTA's units (nunits units of cw columns, the first
// unit index first, tagged res_ep) into cx.s.res.  All consumer threads.
__device__ __forceinline__ bool poll_vec(Cx &cx, const u64 *src, float *dst, int n, unsigned ep,
                                         const u64 *res_src = nullptr, int first = 0, int cw = 0, int nunits = 0,
                                         unsigned res_ep = 0) {
    const u64 limit = gtime() + kTimeoutNs;
    const int G = gridDim.x;
    const int nres = cw * nunits;
    // bit j of `pending`: word ctid + j * kCons not yet seen with the right epoch
    // (n <= 31 * kCons); bit 31: this thread's residual word
    unsigned pending = 0;
    for (int j = 0, i = cx.ctid; i < n; ++j, i += kCons) pending |= 1u << j;
    if (cx.ctid < nres) pending |= 1u << 31;
    for (unsigned round = 0;; ++round) {
        for (unsigned m = pending & 0x7fffffffu; m; m &= m - 1) {
            const int j = __ffs(m) - 1, i = cx.ctid + j * kCons;
            const u64 w = ld_tag(src + i);
            if (tag_is(w, ep)) {
                dst[i] = tag_val(w);
                pending &= ~(1u << j);
            }
        }
        if (pending >> 31) {
            const int col = (first + (cx.ctid / cw) * G) * cw + cx.ctid % cw;
            const u64 w = ld_tag(res_src + col);
            if (tag_is(w, res_ep)) {
                cx.s.res[cx.ctid] = tag_val(w);
                pending &= 0x7fffffffu;
            }
        }
        if (cons_and(pending == 0)) return true;
        if (poll_expired(cx, round, limit, 2)) return false;
    }
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
__device__ __forceinline__ void ln_finish(float S, float Q, int n, float &mean, float &rstd) {
    mean = S / (float)n;
    const float var = fmaxf(Q / (float)n - mean * mean, 0.0f);
    rstd = 1.0f / sqrtf(var + 1e-5f);
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
    ln_finish(S, Q, n, mean, rstd);
}

// Next ring chunk (waits for its bytes).  On an expired wait the thread is
// marked failed and computes on whatever the slot holds; the phase's uniform
// check discards the result.
__device__ __forceinline__ const float *chunk_begin(Cx &cx) {
    const unsigned slot = cx.chunk_i % kSlots, par = (cx.chunk_i / kSlots) & 1u;
    if (cx.tr) {
        const u64 t = gtime();
        if (!mbar_wait(&cx.s.full[slot], par)) fail(cx, 4);
        cx.s.trc[16] += gtime() - t;
        cx.s.trc[19] += 1;
    } else if (!mbar_wait(&cx.s.full[slot], par)) {
        fail(cx, 4);
    }
    return reinterpret_cast<const float *>(cx.s.ring + (size_t)slot * kSlotBytes);
}
__device__ __forceinline__ void chunk_end(Cx &cx) {
    __syncwarp();
    if (cx.lane == 0) mbar_arrive(&cx.s.empty[cx.chunk_i % kSlots]);
    ++cx.chunk_i;
}

// One strip unit of K weight rows plus its bias row and column-sum row, for
// its cw columns (4, 8, 16 or 32).  Without LayerNorm it returns
// y = xs . W + b; with `ln` the input is normalised implicitly,
// y = rstd * (xs . W' - mean * colsum(W')) + b', so that the statistics are
// reduced in the same pass as the products (one barrier for the whole unit).
// The result is in threads ctid < cw.  Every row of a chunk is loaded before
// any product (four rows per thread and chunk cover a slot at every width).
// The width is a run-time value so that every phase runs this one copy of the
// code (it stays in the instruction cache across phases).
__device__ __forceinline__ float strip_unit(Cx &cx, int K, int cw, bool ln) {
    const int lg = cw == 32 ? 3 : cw == 16 ? 2 : cw == 8 ? 1 : 0;   // log2 of the float4 column groups
    const int CG = 1 << lg, RG = kCons >> lg;
    const int RPC = kSlotBytes / (cw * 4);          // rows per chunk; RPC <= 4 * RG
    const int cg = cx.ctid & (CG - 1), rg = cx.ctid >> lg;
    const int rows = K + 2;
    const float *xs = cx.s.xs;
    long long c0 = cx.tr ? clock64() : 0;
    float s = 0.0f, q = 0.0f;
    if (ln) ln_sums(cx, K, s, q);
    if (cx.tr) {
        const long long c = clock64();
        cx.s.trc[22] += c - c0;
        c0 = c;
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float bias = 0.0f, csum = 0.0f;
    for (int r0 = 0; r0 < rows; r0 += RPC) {
        const float *ch = chunk_begin(cx);
        const float4 *w4 = reinterpret_cast<const float4 *>(ch);
        const int nr = min(RPC, rows - r0);
        float xv[4];
        float4 w[4];
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int r = min(rg + it * RG, nr - 1);   // in this chunk's rows; masked below
            xv[it] = xs[r0 + r];                       // r0 + r <= K + 1 < size of xs
            w[it] = w4[(r << lg) + cg];
        }
        if (cx.ctid < cw) {   // the bias and column-sum rows (possibly in different chunks)
            if (K >= r0 && K < r0 + nr) bias = ch[(K - r0) * cw + cx.ctid];
            if (K + 1 >= r0 && K + 1 < r0 + nr) csum = ch[(K + 1 - r0) * cw + cx.ctid];
        }
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int r = rg + it * RG;
            const bool in = r < nr && r0 + r < K;
            const float x = in ? xv[it] : 0.0f;
            const float4 ww = in ? w[it] : make_float4(0.f, 0.f, 0.f, 0.f);
            acc.x = fmaf(x, ww.x, acc.x);
            acc.y = fmaf(x, ww.y, acc.y);
            acc.z = fmaf(x, ww.z, acc.z);
            acc.w = fmaf(x, ww.w, acc.w);
        }
        chunk_end(cx);
    }
    if (cx.tr) {
        const long long c = clock64();
        cx.s.trc[23] += c - c0;
        c0 = c;
    }
    // lanes with equal lane % CG hold the same columns: reduce within the warp, then across warps
    for (int o = CG; o < 32; o <<= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
    }
    if (ln) {
        s = warp_sum(s);
        q = warp_sum(q);
    }
    float *red = cx.s.red + (cx.upar & 1) * kRedHalf;   // [warp][32] products, then [480 + 2 warp] sums
    cx.upar ^= 1u;
    if (cx.lane < CG) reinterpret_cast<float4 *>(red)[cx.warp * 8 + cx.lane] = acc;
    if (ln && cx.lane == 0) {
        red[480 + 2 * cx.warp] = s;
        red[481 + 2 * cx.warp] = q;
    }
    cons_sync();
    float y = 0.0f;
    if (cx.ctid < cw) {
        float t[kWarps];
#pragma unroll
        for (int w = 0; w < kWarps; ++w) t[w] = red[w * 32 + cx.ctid];
#pragma unroll
        for (int st = 1; st < kWarps; st <<= 1)
#pragma unroll
            for (int w = 0; w + st < kWarps; w += 2 * st) t[w] += t[w + st];
        if (ln) {
            float S = 0.0f, Q = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                S += red[480 + 2 * w];
                Q += red[481 + 2 * w];
            }
            float mean, rstd;
            ln_finish(S, Q, K, mean, rstd);
            y = fmaf(rstd, fmaf(-mean, csum, t[0]), bias);
        } else {
            y = t[0] + bias;
        }
    }
    if (cx.tr) {
        cx.s.trc[25] += clock64() - c0;
        cx.s.trc[27] += 1;
    }
    return y;
}

__device__ __forceinline__ unsigned epoch_of(const MegaParams &p, int step, int layer, int ph) {
    return p.epoch0 + (unsigned)step * (unsigned)((p.L + 1) * 8) + (unsigned)(layer * 8 + ph);
}

// ---- producer: the CTA's weight stream for all steps ------------------------------------
__device__ __forceinline__ void producer(Cx &cx, const Sched &S) {
    const MegaParams &p = *cx.p;
    u64 policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    const int E = p.E, F = p.F, L = p.L, G = S.G;
    unsigned i = 0;
    bool ok = true;
    for (int step = 0; step < p.n_steps && ok; ++step) {
        for (int l = 0; l <= L && ok; ++l) {
            const int nph = l < L ? 4 : 1;
            for (int ph = 0; ph < nph && ok; ++ph) {
                int g0, n;
                const char *base;
                size_t ubytes, row_bytes;
                if (l < L) {
                    g0 = l * S.per_layer + (ph > 0 ? S.nA : 0) + (ph > 1 ? S.nC : 0) + (ph > 2 ? S.nD : 0);
                    n = ph == 0 ? S.nA : ph == 1 ? S.nC : ph == 2 ? S.nD : S.nE;
                    base = reinterpret_cast<const char *>(p.packed + p.layer_off[l * 4 + ph]);
                    ubytes = (size_t)((ph == 3 ? F : E) + 2) * p.cw[ph] * sizeof(float);
                    row_bytes = (size_t)p.cw[ph] * sizeof(float);
                } else {
                    g0 = L * S.per_layer;
                    n = S.nLM;
                    base = reinterpret_cast<const char *>(p.lm);
                    ubytes = (size_t)p.lm_rows * E * sizeof(float);
                    row_bytes = (size_t)E * sizeof(float);
                }
                const size_t chunk = (kSlotBytes / row_bytes) * row_bytes;
                for (int u = S.first(g0, cx.cta); u < n && ok; u += G) {
                    const char *src = base + (size_t)u * ubytes;
                    size_t bytes = ubytes;
                    if (l == L) bytes = (size_t)min(p.lm_rows, p.V - u * p.lm_rows) * E * sizeof(float);
                    for (size_t off = 0; off < bytes; off += chunk) {
                        const unsigned nb = (unsigned)(bytes - off < chunk ? bytes - off : chunk);
                        const unsigned slot = i % kSlots;
                        if (!mbar_wait(&cx.s.empty[slot], ((i / kSlots) & 1u) ^ 1u)) {
                            fail(cx, 1);
                            ok = false;
                            break;
                        }
                        // Keep at most max_inflight copies outstanding.
                        if (i >= (unsigned)p.max_inflight) {
                            const unsigned j = i - p.max_inflight;
                            if (!mbar_wait(&cx.s.full[j % kSlots], (j / kSlots) & 1u)) {
                                fail(cx, 1);
                                ok = false;
                                break;
                            }
                        }
                        mbar_expect_tx(&cx.s.full[slot], nb);
                        bulk_load(cx.s.ring + (size_t)slot * kSlotBytes, src + off, nb, &cx.s.full[slot], policy);
                        ++i;
                    }
                }
            }
        }
    }
    // Every copy issued must land before the CTA may exit (the ring is its destination).
    for (unsigned j = i > kSlots ? i - kSlots : 0; j < i; ++j) mbar_wait(&cx.s.full[j % kSlots], (j / kSlots) & 1u);
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) mega_decode_kernel(MegaParams P) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const MegaParams &p = P;
    Cx cx;
    cx.p = &P;
    cx.cta = blockIdx.x;
    cx.warp = threadIdx.x >> 5;
    cx.lane = threadIdx.x & 31;
    cx.ctid = threadIdx.x;   // consumers: 0..511
    cx.failed = 0;
    cx.chunk_i = 0;
    cx.upar = 0;
    cx.tr = p.trace != nullptr && threadIdx.x == 0;
    cx.tl = cx.tr && blockIdx.x == 0;
    cx.t0 = cx.tr ? gtime() : 0;
    const int G = gridDim.x, E = p.E, F = p.F, L = p.L;
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
    cx.s.att = reinterpret_cast<float *>(sp);
    sp += 1024 * sizeof(float);
    cx.s.res = reinterpret_cast<float *>(sp);
    sp += kRes * sizeof(float);
    cx.s.lnf = reinterpret_cast<float *>(sp);
    sp += 2 * (size_t)E * sizeof(float);
    cx.s.xs = reinterpret_cast<float *>(sp);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&cx.s.full[i], 1);
            mbar_init(&cx.s.empty[i], kWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < kTraceSlots; i += kThreads) cx.s.trc[i] = 0;
    for (int i = threadIdx.x; i < E; i += kThreads) {
        cx.s.lnf[i] = p.lnf_g[i];
        cx.s.lnf[E + i] = p.lnf_b[i];
    }
    __syncthreads();

    Sched S;
    S.nA = 3 * E / p.cw[0];
    S.nC = E / p.cw[1];
    S.nD = F / p.cw[2];
    S.nE = E / p.cw[3];
    S.nLM = (p.V + p.lm_rows - 1) / p.lm_rows;
    S.per_layer = S.nA + S.nC + S.nD + S.nE;
    S.G = G;

    if (cx.warp == kWarps) {   // producer warp: one thread issues, the rest are idle
        if (cx.lane == 0) producer(cx, S);
        return;
    }

    // ======================= consumer warps =======================
    float *xs = cx.s.xs;
    int tok = p.state->token, pos = p.state->pos;
    const int step_base = p.state->step, min_new = p.state->min_new;
    for (int step = 0; step < p.n_steps; ++step) {
        const int T = pos + 1;
        const int nch = (T + 63) / 64;
        for (int l = 0; l < L; ++l) {
            const int gl = l * S.per_layer;
            // Phases in order A (LN1 + qkv + K/V append), B (attention), C (combine
            // + proj + residual), D (LN2 + fc + GELU), E (fc2 + residual).  A, C, D
            // and E share one body below; only their inputs and epilogues differ.
            for (int ph = 0; ph < 5; ++ph) {
                if (ph == 1) {
            {
                const int nB = p.NH * nch;
                const unsigned ep_in = epoch_of(p, step, l, 0), ep = epoch_of(p, step, l, 1);
                const int shift = (l * 37) % G;
                for (int b = S.first(shift, cx.cta); b < nB; b += G) {
                    const int h = b / nch, c = b % nch;
                    // q, k_new, v_new of head h at pos (192); P (64); P.V partials (256)
                    float *q = cx.s.att, *pr = cx.s.att + 192, *pv = cx.s.att + 256;
                    tr_begin(cx);
                    // threads 0..255: scores with 4 threads per key (16 dims each), then P.V with
                    // thread (d, grp) over keys grp*16 .. grp*16+15.  The cached keys and values
                    // (positions before pos, written by earlier steps) are loaded before the
                    // wait for q; the key and value at pos come from the qkv vector (q + 64, q + 128).
                    const size_t hb = (size_t)l * p.layer_stride + (size_t)h * p.max_seq * 64;
                    const float *K = p.kc + hb, *V = p.vc + hb;
                    const int j0 = c * 64, nj = min(64, T - j0);
                    const bool act = cx.ctid < 256;
                    const int key = (cx.ctid >> 2) & 63, part = cx.ctid & 3;
                    const int d = cx.ctid & 63, grp = (cx.ctid >> 6) & 3;
                    const bool kcached = act && key < nj && j0 + key != pos;
                    float4 kr[4];
#pragma unroll
                    for (int t = 0; t < 4; ++t)
                        kr[t] = kcached ? reinterpret_cast<const float4 *>(K + (size_t)(j0 + key) * 64 + part * 16)[t]
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
                    float vv[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const int jj = grp * 16 + t, j = j0 + jj;
                        vv[t] = (act && jj < nj && j != pos) ? V[(size_t)j * 64 + d] : 0.0f;
                    }
                    {
                        const u64 limit = gtime() + kTimeoutNs;
                        bool pend = cx.ctid < 192;
                        for (unsigned round = 0;; ++round) {
                            if (pend) {
                                const u64 w = ld_tag(p.t_qkv + (cx.ctid >> 6) * E + h * 64 + (cx.ctid & 63));
                                if (tag_is(w, ep_in)) {
                                    q[cx.ctid] = tag_val(w);
                                    pend = false;
                                }
                            }
                            if (cons_and(!pend)) break;
                            if (poll_expired(cx, round, limit, 5)) goto out;
                        }
                    }
                    tr_inputs(cx, 1);
                    float s = 0.0f;
                    if (act && key < nj) {
                        const float *qq = q + part * 16;
                        if (!kcached) {   // the key at pos
#pragma unroll
                            for (int t = 0; t < 16; ++t) s = fmaf(q[64 + part * 16 + t], qq[t], s);
                        } else {
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                s = fmaf(kr[t].x, qq[4 * t], s);
                                s = fmaf(kr[t].y, qq[4 * t + 1], s);
                                s = fmaf(kr[t].z, qq[4 * t + 2], s);
                                s = fmaf(kr[t].w, qq[4 * t + 3], s);
                            }
                        }
                    }
#pragma unroll
                    for (int t = 0; t < 16; ++t)   // the value at pos (constant indices keep vv in registers)
                        if (act && j0 + grp * 16 + t == pos) vv[t] = q[128 + d];
                    s += __shfl_xor_sync(0xffffffffu, s, 1);
                    s += __shfl_xor_sync(0xffffffffu, s, 2);
                    s *= 0.125f;   // 1 / sqrt(64)
                    const bool valid = act && key < nj;
                    float m = warp_max(valid ? s : -FLT_MAX);
                    float *rb = cx.s.red + kRedAtt;   // 32 floats
                    if (cx.lane == 0 && cx.warp < 8) rb[cx.warp] = m;
                    cons_sync();
                    m = -FLT_MAX;
                    for (int w = 0; w < 8; ++w) m = fmaxf(m, rb[w]);
                    const float e = valid ? expf(s - m) : 0.0f;
                    if (act && part == 0) pr[key] = e;
                    const float lsum = warp_sum(act && part == 0 ? e : 0.0f);
                    if (cx.lane == 0 && cx.warp < 8) rb[16 + cx.warp] = lsum;
                    cons_sync();
                    if (act) {
                        float o = 0.0f;
#pragma unroll
                        for (int t = 0; t < 16; ++t) o = fmaf(pr[grp * 16 + t], vv[t], o);
                        pv[grp * 64 + d] = o;
                    }
                    cons_sync();
                    u64 *rec = p.t_part + ((size_t)h * kMaxChunks + c) * 66;
                    if (cx.ctid < 64) {
                        float acc = 0.0f;
                        for (int g2 = 0; g2 < 4; ++g2) acc += pv[g2 * 64 + cx.ctid];
                        st_tag(rec + 2 + cx.ctid, acc, ep);
                    } else if (cx.ctid == 64) {
                        float lt = 0.0f;
                        for (int w = 0; w < 8; ++w) lt += rb[16 + w];
                        st_tag(rec, m, ep);
                        st_tag(rec + 1, lt, ep);
                    }
                    cons_sync();
                    tr_end(cx, 1);
                }
            }
                    continue;
                }
                // strip phase: ph 0 = A, 2 = C, 3 = D, 4 = E
                const int g0 = gl + (ph >= 2 ? S.nA : 0) + (ph >= 3 ? S.nC : 0) + (ph >= 4 ? S.nD : 0);
                const int n = ph == 0 ? S.nA : ph == 2 ? S.nC : ph == 3 ? S.nD : S.nE;
                int u = S.first(g0, cx.cta);
                if (u >= n) continue;
                const int cw = p.cw[ph == 0 ? 0 : ph - 1], K = ph == 4 ? F : E;
                const int tph = ph == 0 ? 0 : ph;    // trace slot
                tr_begin(cx);
                // ---- inputs ----
                if (ph == 2) {
                    const int nres = S.count(u, S.nC) * cw;
                    const unsigned ep_b = epoch_of(p, step, l, 1), ep_res = epoch_of(p, step, l - 1, 4);
                    // attn[h*64 + d] = sum_c acc_c[d] e^(m_c - M) / sum_c l_c e^(m_c - M), and the residuals
                    const u64 limit = gtime() + kTimeoutNs;
                    // pending: bit j for output ctid + j * kCons, bit 31 for the residual word
                    unsigned pending = 0;
                    for (int j = 0, i = cx.ctid; i < E; ++j, i += kCons) pending |= 1u << j;
                    if (cx.ctid < nres) pending |= 1u << 31;
                    for (unsigned round = 0;; ++round) {
                        for (unsigned mk = pending & 0x7fffffffu; mk; mk &= mk - 1) {
                            const int j = __ffs(mk) - 1, i = cx.ctid + j * kCons;
                            const int h = i >> 6, dd = i & 63;
                            // merge the chunks' (m, l, acc) in one pass, rescaling to the running max
                            float M = -FLT_MAX, Lt = 0.0f, O = 0.0f;
                            bool ok = true;
                            for (int c = 0; c < nch; ++c) {
                                const u64 *rec = p.t_part + ((size_t)h * kMaxChunks + c) * 66;
                                const u64 w0 = ld_tag(rec), w1 = ld_tag(rec + 1), w2 = ld_tag(rec + 2 + dd);
                                ok = ok && tag_is(w0, ep_b) && tag_is(w1, ep_b) && tag_is(w2, ep_b);
                                const float mc = tag_val(w0), lc = tag_val(w1), ac = tag_val(w2);
                                if (mc > M) {
                                    const float sc = expf(M - mc);   // 0 on the first chunk
                                    Lt = fmaf(Lt, sc, lc);
                                    O = fmaf(O, sc, ac);
                                    M = mc;
                                } else {
                                    const float wgt = expf(mc - M);
                                    Lt = fmaf(lc, wgt, Lt);
                                    O = fmaf(ac, wgt, O);
                                }
                            }
                            if (!ok) continue;
                            xs[i] = O / Lt;
                            pending &= ~(1u << j);
                        }
                        if (pending >> 31) {
                            const int n = (u + (cx.ctid / cw) * G) * cw + cx.ctid % cw;
                            if (l == 0) {
                                cx.s.res[cx.ctid] = p.wte[(size_t)tok * E + n] + p.wpe[(size_t)pos * E + n];
                                pending &= 0x7fffffffu;
                            } else {
                                const u64 w = ld_tag(p.t_hb + n);
                                if (tag_is(w, ep_res)) {
                                    cx.s.res[cx.ctid] = tag_val(w);
                                    pending &= 0x7fffffffu;
                                }
                            }
                        }
                        if (cons_and(pending == 0)) break;
                        if (poll_expired(cx, round, limit, 6)) goto out;
                    }
                } else if (ph == 0 && l == 0) {
                    for (int i = cx.ctid; i < E; i += kCons)
                        xs[i] = p.wte[(size_t)tok * E + i] + p.wpe[(size_t)pos * E + i];
                    cons_sync();
                } else {
                    // A: h'' of the previous layer; D: h'; E: f, with the residuals h' of its columns
                    const u64 *src = ph == 0 ? p.t_hb : ph == 3 ? p.t_ha : p.t_f;
                    const unsigned ep_in = ph == 0 ? epoch_of(p, step, l - 1, 4) : epoch_of(p, step, l, ph == 3 ? 2 : 3);
                    if (!poll_vec(cx, src, xs, ph == 4 ? F : E, ep_in, p.t_ha, u, cw, ph == 4 ? S.count(u, S.nE) : 0,
                                  epoch_of(p, step, l, 2)))
                        goto out;
                }
                tr_inputs(cx, tph);
                // ---- units ----
                {
                    const unsigned ep = epoch_of(p, step, l, ph == 0 ? 0 : ph == 2 ? 2 : ph == 3 ? 3 : 4);
                    u64 *dst = ph == 0 ? p.t_qkv : ph == 2 ? p.t_ha : ph == 3 ? p.t_f : p.t_hb;
                    for (int k = 0; u < n; u += G, ++k) {
                        float v = strip_unit(cx, K, cw, ph == 0 || ph == 3);   // LN1 / LN2 folded in
                        if (cx.ctid < cw) {
                            const int col = u * cw + cx.ctid;
                            if (ph == 0) {
                                if (col >= E) {   // K or V of head m / 64: append at pos (math.cl:367-383)
                                    int m = col - E;
                                    float *kv = m >= E ? p.vc : p.kc;
                                    if (m >= E) m -= E;
                                    kv[(size_t)l * p.layer_stride + ((size_t)(m >> 6) * p.max_seq + pos) * 64 + (m & 63)] = v;
                                }
                            } else if (ph == 3) {
                                v = gelu_f(v);
                            } else {
                                v += cx.s.res[k * cw + cx.ctid];   // C, E: residual
                            }
                            st_tag(dst + col, v, ep);
                        }
                        if (cx.tr) cx.s.trc[18] += 1;
                    }
                }
                if (!cons_and(!cx.failed)) goto out;
                tr_end(cx, tph);
            }
        }
        // ---------------- LN_f + LM head + greedy argmax ----------------
        {
            int u = S.first(L * S.per_layer, cx.cta);
            const bool forbid = (step_base + step) < min_new;
            float best = -FLT_MAX;
            int besti = INT_MAX;
            if (u < S.nLM) {
                tr_begin(cx);
                if (!poll_vec(cx, p.t_hb, xs, E, epoch_of(p, step, L - 1, 4))) goto out;
                tr_inputs(cx, 5);
                float mean, rstd;
                ln_stats(cx, E, mean, rstd);
                // normalise in place with gamma / beta (math.cl:310); the rows read it 16 times
                for (int i = cx.ctid; i < E; i += kCons) xs[i] = (xs[i] - mean) * rstd * cx.s.lnf[i] + cx.s.lnf[E + i];
                cons_sync();
                const int RPC = kSlotBytes / (E * 4);
                const int E4 = E / 4;
                const float4 *x4 = reinterpret_cast<const float4 *>(xs);
                for (; u < S.nLM; u += G) {
                    const int v0 = u * p.lm_rows, rows = min(p.lm_rows, p.V - v0);
                    for (int r0 = 0; r0 < rows; r0 += RPC) {
                        const float *ch = chunk_begin(cx);
                        const int nr = min(RPC, rows - r0);
                        for (int r = cx.warp; r < nr; r += kWarps) {
                            const float4 *w4 = reinterpret_cast<const float4 *>(ch + (size_t)r * E);
                            float sacc = 0.0f;
                            for (int j = cx.lane; j < E4; j += 32) {
                                const float4 w = w4[j], xv = x4[j];
                                sacc = fmaf(w.x, xv.x, sacc);
                                sacc = fmaf(w.y, xv.y, sacc);
                                sacc = fmaf(w.z, xv.z, sacc);
                                sacc = fmaf(w.w, xv.w, sacc);
                            }
                            sacc = warp_sum(sacc);
                            const int v = v0 + r0 + r;
                            if (cx.lane == 0) p.logits[v] = sacc;
                            if (!(forbid && v == kEos) && better(sacc, v, best, besti)) {
                                best = sacc;
                                besti = v;
                            }
                        }
                        chunk_end(cx);
                    }
                }
                if (!cons_and(!cx.failed)) goto out;
                tr_end(cx, 5);
            }
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
            if (cx.ctid == 0) {
                for (int w = 0; w < kWarps; ++w)
                    if (better(rv[w], ri[w], best, besti)) {
                        best = rv[w];
                        besti = ri[w];
                    }
                // release: this CTA's K/V rows of the step (ordered before this
                // thread by the barrier above) become visible with the partial
                __threadfence();
                st_tag(tb + 2 * cx.cta, best, ep);
                st_tag(tb + 2 * cx.cta + 1, __int_as_float(besti), ep);
            }
            float *bv = cx.s.att;                                    // 2 * G <= 512 floats
            int *bi = reinterpret_cast<int *>(cx.s.att + 512);      // [0] token
            tr_begin(cx);
            if (!poll_vec(cx, tb, bv, 2 * G, ep)) goto out;
            __threadfence();   // acquire: every CTA's K/V rows of this step, for the steps that follow
            tr_inputs(cx, 6);
            if (cx.ctid == 0) {
                float gb = -FLT_MAX;
                int gi = INT_MAX;
                for (int c = 0; c < G; ++c) {
                    const int ix = __float_as_int(bv[2 * c + 1]);
                    if (better(bv[2 * c], ix, gb, gi)) {
                        gb = bv[2 * c];
                        gi = ix;
                    }
                }
                if (gi == INT_MAX) gi = 0;   // every logit NaN: never hand an invalid id to the next step
                bi[0] = gi;
                if (cx.cta == 0) {
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
            cx.tl = false;
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

size_t mega_smem_bytes(int E, int F) {
    const int xs = (E > F ? E : F) + 4;
    return (size_t)kSlots * kSlotBytes + 2 * kSlots * sizeof(unsigned long long) + kTraceSlots * sizeof(unsigned long long) +
           kRedFloats * sizeof(float) + 1024 * sizeof(float) + kRes * sizeof(float) + 2 * (size_t)E * sizeof(float) +
           (size_t)xs * sizeof(float);
}
int mega_threads() { return kThreads; }
const void *mega_kernel_ptr() { return (const void *)mega_decode_kernel; }
int mega_slot_bytes() { return kSlotBytes; }

}  // namespace g2
