// g2_mega.cu -- persistent B = 1 decode kernel (fp32): every layer and every
// greedy step of a generation in one cooperative launch.
//
// It replaces the per-token kernel sequence of decode() (main.c:1792-1833)
// and the greedy branch of sample_next_token (main.c:1898-1904).
//
// Structure (one CTA per SM; 16 consumer warps + 1 producer warp):
//
//  * Weights are repacked at load time into "units": column strips of a
//    projection over its full K (so no output needs a cross-CTA reduction),
//    about 48 KB each, and 16-row blocks of wte for the LM head.  Unit g of a
//    step belongs to CTA g % gridDim.x, counting across all phases of the
//    step, so every SM streams the same bytes per layer to within one unit.
//  * The producer warp streams the CTA's units, in consumption order, through
//    an 8 x 24 KB shared-memory ring with cp.async.bulk (mbarrier full/empty,
//    L2 evict-first).  The stream is the same every step and waits on no
//    activation, so it runs ahead across layer and token boundaries.
//  * Activations move between CTAs as 64-bit words (epoch << 32 | float
//    bits).  A consumer polls the vector it needs until every word carries the
//    epoch of the producing phase: readiness costs one L2 round trip, with no
//    grid barrier and no atomics.  A buffer is rewritten only after every
//    reader of its previous contents has produced the outputs the rewrite
//    depends on, so a reader never sees a newer epoch than it waits for.
//  * Per layer: A = LN1 + qkv + K/V append, B = attention per (head, 64-key
//    chunk) with online-softmax partials, C = combine + proj + residual,
//    D = LN2 + fc + GELU, E = fc2 + residual.  Then LN_f + LM head with a per-CTA
//    argmax; every CTA reads all CTA partials and derives the next token.
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

constexpr int kCons = 512;                 // consumer threads
constexpr int kThreads = kCons + 32;       // + producer warp
constexpr int kSlots = 8;
constexpr int kSlotBytes = 24576;
constexpr unsigned long long kTimeoutNs = 2000000000ull;
constexpr int kConsBar = 1;                // named barrier of the consumer warps
constexpr int kMaxChunks = 16;             // attention chunks per head (1024 / 64)

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
};

struct Smem {
    float *xs;     // input vector of the current phase (max(E, F) floats)
    float *red;    // reduction scratch: [0,256) per-warp partials, [256,272) unit results, [288,320) ints
    float *att;    // attention / argmax scratch (1024 floats)
    u64 *full, *empty;
    unsigned char *ring;
};

// Optional phase trace kept by consumer thread 0 of each CTA (MegaParams::trace).
struct Trace {
    bool on;
    bool timeline;            // CTA 0, step 0: also record phase stamps of layers 0 and 1
    u64 t0, tb, tm;
    u64 poll[8], work[8], chunkw;
    unsigned units, chunks;
    int ntl;
    u64 tl[32];
};

struct Cx {
    const MegaParams *p;
    Smem s;
    int cta, ctid, warp, lane;
    unsigned chunk_i;   // next ring chunk to consume
    int failed;         // this thread saw an expired wait
    Trace tr;
};

// Trace points (no-ops unless tracing): phase begins, its inputs have arrived, phase ends.
__device__ __forceinline__ void tr_stamp(Cx &cx) {
    if (cx.tr.timeline && cx.tr.ntl < 32) cx.tr.tl[cx.tr.ntl++] = gtime() - cx.tr.t0;
}
__device__ __forceinline__ void tr_begin(Cx &cx) {
    if (cx.tr.on) {
        cx.tr.tb = gtime();
        tr_stamp(cx);
    }
}
__device__ __forceinline__ void tr_inputs(Cx &cx, int ph) {
    if (cx.tr.on) {
        cx.tr.tm = gtime();
        cx.tr.poll[ph] += cx.tr.tm - cx.tr.tb;
        tr_stamp(cx);
    }
}
__device__ __forceinline__ void tr_end(Cx &cx, int ph) {
    if (cx.tr.on) {
        cx.tr.work[ph] += gtime() - cx.tr.tm;
        tr_stamp(cx);
    }
}

__device__ __forceinline__ void fail(Cx &cx, int code) {
    cx.failed = 1;
    atomicCAS(cx.p->err, 0, code);
}

// Poll n tagged words into dst until all carry `ep` (all consumer threads).
__device__ bool poll_vec(Cx &cx, const u64 *src, float *dst, int n, unsigned ep) {
    const u64 limit = gtime() + kTimeoutNs;
    for (;;) {
        int ok = 1;
        for (int i = cx.ctid; i < n; i += kCons) {
            const u64 w = ld_tag(src + i);
            if (!tag_is(w, ep)) ok = 0;
            else dst[i] = tag_val(w);
        }
        if (cons_and(ok)) return true;
        if (cons_or(gtime() > limit)) {
            fail(cx, 2);
            return false;
        }
        __nanosleep(32);
    }
}
// One tagged word (a single thread; failures surface at the next uniform check).
__device__ float poll_one(Cx &cx, const u64 *src, unsigned ep) {
    u64 w = ld_tag(src);
    if (tag_is(w, ep)) return tag_val(w);
    const u64 limit = gtime() + kTimeoutNs;
    for (;;) {
        __nanosleep(20);
        w = ld_tag(src);
        if (tag_is(w, ep)) return tag_val(w);
        if (gtime() > limit) {
            fail(cx, 3);
            return 0.0f;
        }
    }
}

// LayerNorm of xs[0..n) in place: two passes, eps 1e-5 (math.cl:297-310).
__device__ void ln_inplace(Cx &cx, int n, const float *g, const float *b) {
    float s = 0.0f;
    for (int i = cx.ctid; i < n; i += kCons) s += cx.s.xs[i];
    s = warp_sum(s);
    if (cx.lane == 0) cx.s.red[cx.warp] = s;
    cons_sync();
    float tot = 0.0f;
    for (int w = 0; w < 16; ++w) tot += cx.s.red[w];
    const float mean = tot / (float)n;
    cons_sync();
    float v = 0.0f;
    for (int i = cx.ctid; i < n; i += kCons) {
        const float d = cx.s.xs[i] - mean;
        v += d * d;
    }
    v = warp_sum(v);
    if (cx.lane == 0) cx.s.red[cx.warp] = v;
    cons_sync();
    float var = 0.0f;
    for (int w = 0; w < 16; ++w) var += cx.s.red[w];
    var /= (float)n;
    const float rstd = 1.0f / sqrtf(var + 1e-5f);
    for (int i = cx.ctid; i < n; i += kCons) cx.s.xs[i] = (cx.s.xs[i] - mean) * rstd * g[i] + b[i];
    cons_sync();
}

// Next ring chunk (waits for its bytes).  On an expired wait the thread is
// marked failed and computes on whatever the slot holds; the caller's uniform
// check discards the result.
__device__ __forceinline__ const float *chunk_begin(Cx &cx) {
    const unsigned slot = cx.chunk_i % kSlots, par = (cx.chunk_i / kSlots) & 1u;
    if (cx.tr.on) {
        const u64 t = gtime();
        if (!mbar_wait(&cx.s.full[slot], par)) fail(cx, 4);
        cx.tr.chunkw += gtime() - t;
        ++cx.tr.chunks;
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

// One strip unit: sum_k xs[k] * W[k][c] for its CW columns over K rows that
// arrive in ring chunks.  Leaves the CW sums in red[256 .. 256 + CW).
template <int CW>
__device__ void strip_unit(Cx &cx, int K) {
    constexpr int CG = CW / 4, RG = kCons / CG;
    constexpr int RPC = kSlotBytes / (CW * 4);   // rows per chunk
    const int cg = cx.ctid % CG, rg = cx.ctid / CG;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < K; r0 += RPC) {
        const float4 *w4 = reinterpret_cast<const float4 *>(chunk_begin(cx));
        const int nr = min(RPC, K - r0);
        const float *x = cx.s.xs + r0;
        for (int r = rg; r < nr; r += RG) {
            const float xv = x[r];
            const float4 w = w4[r * CG + cg];
            acc.x = fmaf(xv, w.x, acc.x);
            acc.y = fmaf(xv, w.y, acc.y);
            acc.z = fmaf(xv, w.z, acc.z);
            acc.w = fmaf(xv, w.w, acc.w);
        }
        chunk_end(cx);
    }
    // lanes with equal lane % CG hold the same columns: reduce within the warp, then across warps
#pragma unroll
    for (int o = CG; o < 32; o <<= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
    }
    cons_sync();   // previous users of red[] are done
    if (cx.lane < CG) {
        float *r = cx.s.red + cx.warp * 16 + cx.lane * 4;
        r[0] = acc.x;
        r[1] = acc.y;
        r[2] = acc.z;
        r[3] = acc.w;
    }
    cons_sync();
    if (cx.ctid < CW) {
        float tot = 0.0f;
        for (int w = 0; w < 16; ++w) tot += cx.s.red[w * 16 + cx.ctid];
        cx.s.red[256 + cx.ctid] = tot;
    }
    cons_sync();
}

__device__ __forceinline__ void strip_e(Cx &cx, int K) {
    if (cx.p->cw_e == 16) strip_unit<16>(cx, K);
    else strip_unit<8>(cx, K);
}

__device__ __forceinline__ unsigned epoch_of(const MegaParams &p, int step, int layer, int ph) {
    return p.epoch0 + (unsigned)step * (unsigned)((p.L + 1) * 8) + (unsigned)(layer * 8 + ph);
}

// ---- producer: the CTA's weight stream for all steps ------------------------------------
__device__ void producer(Cx &cx, const Sched &S) {
    const MegaParams &p = *cx.p;
    u64 policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    const int E = p.E, F = p.F, L = p.L, G = S.G;
    const size_t ue = (size_t)E * p.cw_e * sizeof(float), uf = (size_t)F * p.cw_f * sizeof(float);
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
                    const int counts[4] = {S.nA, S.nC, S.nD, S.nE};
                    g0 = l * S.per_layer;
                    for (int q = 0; q < ph; ++q) g0 += counts[q];
                    n = counts[ph];
                    base = reinterpret_cast<const char *>(p.packed + p.layer_off[l * 4 + ph]);
                    ubytes = ph == 3 ? uf : ue;
                    row_bytes = (size_t)(ph == 3 ? p.cw_f : p.cw_e) * sizeof(float);
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
    cx.tr.on = p.trace != nullptr && threadIdx.x == 0;
    cx.tr.timeline = cx.tr.on && blockIdx.x == 0;
    cx.tr.ntl = 0;
    cx.tr.chunkw = 0;
    cx.tr.units = cx.tr.chunks = 0;
    for (int i = 0; i < 8; ++i) cx.tr.poll[i] = cx.tr.work[i] = 0;
    cx.tr.t0 = cx.tr.on ? gtime() : 0;
    unsigned char *sp = smem_raw;
    cx.s.ring = sp;
    sp += kSlots * kSlotBytes;
    cx.s.full = reinterpret_cast<u64 *>(sp);
    cx.s.empty = cx.s.full + kSlots;
    sp += 2 * kSlots * sizeof(u64);
    cx.s.red = reinterpret_cast<float *>(sp);
    sp += 320 * sizeof(float);
    cx.s.att = reinterpret_cast<float *>(sp);
    sp += 1024 * sizeof(float);
    cx.s.xs = reinterpret_cast<float *>(sp);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&cx.s.full[i], 1);
            mbar_init(&cx.s.empty[i], 16);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int G = gridDim.x, E = p.E, F = p.F, L = p.L;
    Sched S;
    S.nA = 3 * E / p.cw_e;
    S.nC = E / p.cw_e;
    S.nD = F / p.cw_e;
    S.nE = E / p.cw_f;
    S.nLM = (p.V + p.lm_rows - 1) / p.lm_rows;
    S.per_layer = S.nA + S.nC + S.nD + S.nE;
    S.G = G;

    if (cx.warp == 16) {   // producer warp: one thread issues, the rest are idle
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
            const LayerPtrs &lw = p.layers[l];
            const int gl = l * S.per_layer;
            // ---------------- phase A: LN1 + qkv + K/V append (split_kv) ----------------
            {
                int u = S.first(gl, cx.cta);
                if (u < S.nA) {
                    tr_begin(cx);
                    if (l == 0) {
                        for (int i = cx.ctid; i < E; i += kCons)
                            xs[i] = p.wte[(size_t)tok * E + i] + p.wpe[(size_t)pos * E + i];
                        cons_sync();
                    } else if (!poll_vec(cx, p.t_hb, xs, E, epoch_of(p, step, l - 1, 4))) {
                        goto out;
                    }
                    tr_inputs(cx, 0);
                    ln_inplace(cx, E, lw.ln1_g, lw.ln1_b);
                    const unsigned ep = epoch_of(p, step, l, 0);
                    for (; u < S.nA; u += G) {
                        strip_e(cx, E);
                        if (cx.ctid < p.cw_e) {
                            const int n = u * p.cw_e + cx.ctid;
                            const float v = cx.s.red[256 + cx.ctid] + lw.qkv_b[n];
                            if (n >= E) {   // K or V of head m / 64: append at pos (math.cl:367-383)
                                int m = n - E;
                                float *dst = m >= E ? p.vc : p.kc;
                                if (m >= E) m -= E;
                                dst[(size_t)l * p.layer_stride + ((size_t)(m >> 6) * p.max_seq + pos) * 64 + (m & 63)] = v;
                                __threadfence();   // cache row visible before the tag that announces it
                            }
                            st_tag(p.t_qkv + n, v, ep);
                        }
                        if (!cons_and(!cx.failed)) goto out;
                        if (cx.tr.on) ++cx.tr.units;
                    }
                    tr_end(cx, 0);
                }
            }
            // ---------------- phase B: attention units (head, 64-key chunk) ----------------
            {
                const int nB = p.NH * nch;
                const unsigned ep_in = epoch_of(p, step, l, 0), ep = epoch_of(p, step, l, 1);
                const int shift = (l * 37) % G;
                for (int b = S.first(shift, cx.cta); b < nB; b += G) {
                    const int h = b / nch, c = b % nch;
                    float *q = cx.s.att, *pr = cx.s.att + 192, *pv = cx.s.att + 256;   // pv: 512 floats
                    tr_begin(cx);
                    {
                        const u64 limit = gtime() + kTimeoutNs;
                        for (;;) {
                            int ok = 1;
                            if (cx.ctid < 192) {   // q, k, v of head h at pos
                                const u64 w = ld_tag(p.t_qkv + (cx.ctid >> 6) * E + h * 64 + (cx.ctid & 63));
                                if (!tag_is(w, ep_in)) ok = 0;
                                else q[cx.ctid] = tag_val(w);
                            }
                            if (cons_and(ok)) break;
                            if (cons_or(gtime() > limit)) {
                                fail(cx, 5);
                                goto out;
                            }
                            __nanosleep(32);
                        }
                        __threadfence();   // K/V rows written before those tags are visible
                    }
                    tr_inputs(cx, 1);
                    const size_t hb = (size_t)l * p.layer_stride + (size_t)h * p.max_seq * 64;
                    const float *K = p.kc + hb, *V = p.vc + hb;
                    const int j0 = c * 64, nj = min(64, T - j0);
                    // scores: 8 threads per key, 8 dims each
                    const int key = cx.ctid >> 3, part = cx.ctid & 7;
                    float s = 0.0f;
                    if (key < nj) {
                        const float4 *kr = reinterpret_cast<const float4 *>(K + (size_t)(j0 + key) * 64 + part * 8);
                        const float4 a = kr[0], bq = kr[1];
                        const float *qq = q + part * 8;
                        s = a.x * qq[0] + a.y * qq[1] + a.z * qq[2] + a.w * qq[3] + bq.x * qq[4] + bq.y * qq[5] +
                            bq.z * qq[6] + bq.w * qq[7];
                    }
                    // V for the P.V pass: thread (d, grp) takes keys grp*8 .. grp*8+7
                    const int d = cx.ctid & 63, grp = cx.ctid >> 6;
                    float vv[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const int jj = grp * 8 + t;
                        vv[t] = jj < nj ? V[(size_t)(j0 + jj) * 64 + d] : 0.0f;
                    }
                    s += __shfl_xor_sync(0xffffffffu, s, 1);
                    s += __shfl_xor_sync(0xffffffffu, s, 2);
                    s += __shfl_xor_sync(0xffffffffu, s, 4);
                    s *= 0.125f;   // 1 / sqrt(64)
                    float m = warp_max(key < nj ? s : -FLT_MAX);
                    if (cx.lane == 0) cx.s.red[cx.warp] = m;
                    cons_sync();
                    m = -FLT_MAX;
                    for (int w = 0; w < 16; ++w) m = fmaxf(m, cx.s.red[w]);
                    const float e = key < nj ? expf(s - m) : 0.0f;
                    if (part == 0) pr[key] = e;
                    const float lsum = warp_sum(part == 0 ? e : 0.0f);
                    cons_sync();
                    if (cx.lane == 0) cx.s.red[cx.warp] = lsum;
                    float o = 0.0f;
#pragma unroll
                    for (int t = 0; t < 8; ++t) o = fmaf(pr[grp * 8 + t], vv[t], o);
                    pv[grp * 64 + d] = o;
                    cons_sync();
                    u64 *rec = p.t_part + ((size_t)h * kMaxChunks + c) * 66;
                    if (cx.ctid < 64) {
                        float acc = 0.0f;
                        for (int g2 = 0; g2 < 8; ++g2) acc += pv[g2 * 64 + cx.ctid];
                        st_tag(rec + 2 + cx.ctid, acc, ep);
                    } else if (cx.ctid == 64) {
                        float lt = 0.0f;
                        for (int w = 0; w < 16; ++w) lt += cx.s.red[w];
                        st_tag(rec, m, ep);
                        st_tag(rec + 1, lt, ep);
                    }
                    cons_sync();
                    tr_end(cx, 1);
                }
            }
            // ---------------- phase C: combine attention + proj + residual ----------------
            {
                int u = S.first(gl + S.nA, cx.cta);
                if (u < S.nC) {
                    tr_begin(cx);
                    const unsigned ep_b = epoch_of(p, step, l, 1);
                    // attn[h*64 + d] = sum_c acc_c[d] e^(m_c - M) / sum_c l_c e^(m_c - M)
                    const u64 limit = gtime() + kTimeoutNs;
                    for (;;) {
                        int ok = 1;
                        for (int i = cx.ctid; i < E; i += kCons) {
                            const int h = i >> 6, dd = i & 63;
                            float mc[kMaxChunks], lc[kMaxChunks], ac[kMaxChunks];
                            float M = -FLT_MAX;
                            for (int c = 0; c < nch; ++c) {
                                const u64 *rec = p.t_part + ((size_t)h * kMaxChunks + c) * 66;
                                const u64 w0 = ld_tag(rec), w1 = ld_tag(rec + 1), w2 = ld_tag(rec + 2 + dd);
                                if (!tag_is(w0, ep_b) || !tag_is(w1, ep_b) || !tag_is(w2, ep_b)) ok = 0;
                                mc[c] = tag_val(w0);
                                lc[c] = tag_val(w1);
                                ac[c] = tag_val(w2);
                                M = fmaxf(M, mc[c]);
                            }
                            float Lt = 0.0f, O = 0.0f;
                            for (int c = 0; c < nch; ++c) {
                                const float wgt = expf(mc[c] - M);
                                Lt = fmaf(lc[c], wgt, Lt);
                                O = fmaf(ac[c], wgt, O);
                            }
                            xs[i] = O / Lt;
                        }
                        if (cons_and(ok)) break;
                        if (cons_or(gtime() > limit)) {
                            fail(cx, 6);
                            goto out;
                        }
                        __nanosleep(32);
                    }
                    tr_inputs(cx, 2);
                    const unsigned ep = epoch_of(p, step, l, 2), ep_res = epoch_of(p, step, l - 1, 4);
                    for (; u < S.nC; u += G) {
                        strip_e(cx, E);
                        if (cx.ctid < p.cw_e) {
                            const int n = u * p.cw_e + cx.ctid;
                            const float res = l == 0 ? p.wte[(size_t)tok * E + n] + p.wpe[(size_t)pos * E + n]
                                                     : poll_one(cx, p.t_hb + n, ep_res);
                            st_tag(p.t_ha + n, res + (cx.s.red[256 + cx.ctid] + lw.proj_b[n]), ep);
                        }
                        if (!cons_and(!cx.failed)) goto out;
                        if (cx.tr.on) ++cx.tr.units;
                    }
                    tr_end(cx, 2);
                }
            }
            // ---------------- phase D: LN2 + fc + GELU ----------------
            {
                int u = S.first(gl + S.nA + S.nC, cx.cta);
                if (u < S.nD) {
                    tr_begin(cx);
                    if (!poll_vec(cx, p.t_ha, xs, E, epoch_of(p, step, l, 2))) goto out;
                    tr_inputs(cx, 3);
                    ln_inplace(cx, E, lw.ln2_g, lw.ln2_b);
                    const unsigned ep = epoch_of(p, step, l, 3);
                    for (; u < S.nD; u += G) {
                        strip_e(cx, E);
                        if (cx.ctid < p.cw_e) {
                            const int n = u * p.cw_e + cx.ctid;
                            st_tag(p.t_f + n, gelu_f(cx.s.red[256 + cx.ctid] + lw.fc_b[n]), ep);
                        }
                        if (!cons_and(!cx.failed)) goto out;
                        if (cx.tr.on) ++cx.tr.units;
                    }
                    tr_end(cx, 3);
                }
            }
            // ---------------- phase E: fc2 + residual ----------------
            {
                int u = S.first(gl + S.nA + S.nC + S.nD, cx.cta);
                if (u < S.nE) {
                    tr_begin(cx);
                    if (!poll_vec(cx, p.t_f, xs, F, epoch_of(p, step, l, 3))) goto out;
                    tr_inputs(cx, 4);
                    const unsigned ep = epoch_of(p, step, l, 4), ep_res = epoch_of(p, step, l, 2);
                    for (; u < S.nE; u += G) {
                        strip_unit<4>(cx, F);
                        if (cx.ctid < 4) {
                            const int n = u * 4 + cx.ctid;
                            const float res = poll_one(cx, p.t_ha + n, ep_res);
                            st_tag(p.t_hb + n, res + (cx.s.red[256 + cx.ctid] + lw.fc2_b[n]), ep);
                        }
                        if (!cons_and(!cx.failed)) goto out;
                        if (cx.tr.on) ++cx.tr.units;
                    }
                    tr_end(cx, 4);
                }
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
                ln_inplace(cx, E, p.lnf_g, p.lnf_b);
                const int RPC = kSlotBytes / (E * 4);
                const int E4 = E / 4;
                const float4 *x4 = reinterpret_cast<const float4 *>(xs);
                for (; u < S.nLM; u += G) {
                    const int v0 = u * p.lm_rows, rows = min(p.lm_rows, p.V - v0);
                    for (int r0 = 0; r0 < rows; r0 += RPC) {
                        const float *ch = chunk_begin(cx);
                        const int nr = min(RPC, rows - r0);
                        for (int r = cx.warp; r < nr; r += 16) {
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
            int *redi = reinterpret_cast<int *>(cx.s.red) + 288;
            cons_sync();
            if (cx.lane == 0) {
                cx.s.red[cx.warp] = best;
                redi[cx.warp] = besti;
            }
            cons_sync();
            // The partials alternate between two halves by step parity: a CTA whose
            // own work is not on another CTA's path may still be reading step s
            // when that CTA writes step s + 1; step s + 2 needs its step s + 1 partial.
            const unsigned ep = epoch_of(p, step, L, 0);
            u64 *tb = p.t_best + (size_t)(step & 1) * 2 * G;
            if (cx.ctid == 0) {
                for (int w = 0; w < 16; ++w)
                    if (better(cx.s.red[w], redi[w], best, besti)) {
                        best = cx.s.red[w];
                        besti = redi[w];
                    }
                st_tag(tb + 2 * cx.cta, best, ep);
                st_tag(tb + 2 * cx.cta + 1, __int_as_float(besti), ep);
            }
            float *bv = cx.s.att;                                    // 2 * G <= 512 floats
            int *bi = reinterpret_cast<int *>(cx.s.att + 512);      // [0] token
            tr_begin(cx);
            if (!poll_vec(cx, tb, bv, 2 * G, ep)) goto out;
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
            if (step == 0 && cx.tr.timeline) cx.tr.timeline = false;
        }
    }
    if (cx.cta == 0 && cx.ctid == 0) {
        p.state->token = tok;
        p.state->pos = pos;
        p.state->step = step_base + p.n_steps;
    }
out:
    if (cx.tr.on) {
        u64 *t = p.trace + (size_t)cx.cta * kTraceSlots;
        for (int i = 0; i < 8; ++i) {
            t[i] = cx.tr.poll[i];
            t[8 + i] = cx.tr.work[i];
        }
        t[16] = cx.tr.chunkw;
        t[17] = gtime() - cx.tr.t0;
        t[18] = cx.tr.units;
        t[19] = cx.tr.chunks;
        for (int i = 0; i < cx.tr.ntl; ++i) t[32 + i] = cx.tr.tl[i];
    }
    return;
}

size_t mega_smem_bytes(int E, int F) {
    const int xs = E > F ? E : F;
    return (size_t)kSlots * kSlotBytes + 2 * kSlots * sizeof(unsigned long long) + 320 * sizeof(float) +
           1024 * sizeof(float) + (size_t)xs * sizeof(float);
}
int mega_threads() { return kThreads; }
const void *mega_kernel_ptr() { return (const void *)mega_decode_kernel; }

}  // namespace g2
