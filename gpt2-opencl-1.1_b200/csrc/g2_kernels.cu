// g2_kernels.cu -- sm_100a kernels of the GPT-2 decode/prefill path.
//
// Each kernel replaces one or more of the reference's OpenCL kernels
// (math.cl) with the neighbouring element-wise work fused in:
//
//   gemv_kernel       matvec4 / matvec4_sk + reduce_partial (math.cl:185-280)
//                     with layernorm (math.cl:283) fused as a prologue and
//                     bias / GELU / residual / split_kv (math.cl:367) as the
//                     epilogue.  B = 1 decode.
//   gemm_kernel       the prefill matmul (main.c:593-684) + gelu / add_inplace /
//                     split_kv epilogues, for any number of rows (prefill and
//                     batched decode).
//   attn_kernel       attn_scores_1q + attn_softmax_1q + attn_out_1q
//                     (math.cl:388-476): one query per row, keys split over
//                     CTAs (flash-decoding), online softmax, deterministic
//                     in-order combine by the last CTA of each head.
//   lm_head_kernel    final layernorm + lm_head matvec (main.c:1828-1832) +
//                     the greedy argmax of sample_next_token (main.c:1898-1904).
//   embed_kernel      embed (math.cl:333).
//
// Arithmetic is fp32 with fp32 accumulation (fp16 weights are widened on
// load).  Summation orders differ from the reference (parallel reductions);
// parity is checked against the oracle within the stated tolerances.
#include <cuda.h>

#include <cfloat>
#include <cstdlib>
#include <climits>

#include "g2_device.cuh"
#include "gpt2b200.h"

namespace g2 {

// ------------------------------------------------------------------------------
// helpers
// ------------------------------------------------------------------------------
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
// Block-wide sum; `sh` holds >= 32 floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float *sh) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = (l < nw) ? sh[l] : 0.0f;
    t = warp_sum(t);
    return t;
}
__device__ __forceinline__ float block_max(float v, float *sh) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float t = (l < nw) ? sh[l] : -FLT_MAX;
    return warp_max(t);
}

// Two-pass LayerNorm statistics of x[0..n) (math.cl:297-308), block-wide.
__device__ __forceinline__ void ln_stats(const float *x, int n, float *sh, float &mean, float &rstd) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
    mean = block_sum(s, sh) / (float)n;
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float d = x[i] - mean;
        v += d * d;
    }
    const float var = block_sum(v, sh) / (float)n;
    rstd = 1.0f / sqrtf(var + 1e-5f);
}

// 16-byte streaming load of weights (read once per step: no L1 allocation).
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

template <typename WT>
struct Vec;
template <>
struct Vec<float> {
    static constexpr int n = 4;
};
template <>
struct Vec<__half> {
    static constexpr int n = 8;
};

// acc[0..n) += x * w[0..n), w packed in 16 bytes.
__device__ __forceinline__ void fma_vec(float *acc, uint4 w, float x, float) {
    acc[0] = fmaf(x, __uint_as_float(w.x), acc[0]);
    acc[1] = fmaf(x, __uint_as_float(w.y), acc[1]);
    acc[2] = fmaf(x, __uint_as_float(w.z), acc[2]);
    acc[3] = fmaf(x, __uint_as_float(w.w), acc[3]);
}
__device__ __forceinline__ void fma_vec(float *acc, uint4 w, float x, __half) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        acc[2 * i] = fmaf(x, f.x, acc[2 * i]);
        acc[2 * i + 1] = fmaf(x, f.y, acc[2 * i + 1]);
    }
}
// 16 bytes of cache elements as fp32
__device__ __forceinline__ void unpack_vec(uint4 w, float *f, float) {
    f[0] = __uint_as_float(w.x);
    f[1] = __uint_as_float(w.y);
    f[2] = __uint_as_float(w.z);
    f[3] = __uint_as_float(w.w);
}
__device__ __forceinline__ void unpack_vec(uint4 w, float *f, __half) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(h[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}
// dot of 16 bytes of weights with xs[0..n)
__device__ __forceinline__ float dot_vec(uint4 w, const float *xs, float) {
    return __uint_as_float(w.x) * xs[0] + __uint_as_float(w.y) * xs[1] + __uint_as_float(w.z) * xs[2] +
           __uint_as_float(w.w) * xs[3];
}
__device__ __forceinline__ float dot_vec(uint4 w, const float *xs, __half) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&w);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        s = fmaf(f.x, xs[2 * i], s);
        s = fmaf(f.y, xs[2 * i + 1], s);
    }
    return s;
}

// ------------------------------------------------------------------------------
// embed (math.cl:333-350)
// ------------------------------------------------------------------------------
template <typename WT>
__global__ void embed_kernel(const WT *wte, const WT *wpe, Rows rows, float *h, int E, int V, int n_pos) {
    pdl_wait();
    pdl_launch();
    const int r = blockIdx.x;
    // ids and positions are validated on the host; clamp so that a bad value
    // can never address outside the tables (and report it in the checked build)
    const int tok0 = rows.tok[r], pos0 = rows.pos[r];
    if (threadIdx.x == 0) {
        (void)G2_BOUNDS(tok0 >= 0 && tok0 < V, 101);
        (void)G2_BOUNDS(pos0 >= 0 && pos0 < n_pos, 102);
    }
    const int tok = min(max(tok0, 0), V - 1), pos = min(max(pos0, 0), n_pos - 1);
    for (int i = threadIdx.x; i < E; i += blockDim.x)
        h[(size_t)r * E + i] = tof(wte[(size_t)tok * E + i]) + tof(wpe[(size_t)pos * E + i]);
}

// layernorm (math.cl:283-311), one CTA per row.
template <typename WT>
__global__ void __launch_bounds__(256) layernorm_kernel(const float *x, float *out, const WT *g, const WT *b, int E,
                                                        OperandOut op) {
    pdl_wait();
    pdl_launch();
    __shared__ float sh[32];
    const float *xr = x + (size_t)blockIdx.x * E;
    float mean, rstd;
    ln_stats(xr, E, sh, mean, rstd);
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        const float v = (xr[i] - mean) * rstd * tof(g[i]) + tof(b[i]);
        const size_t o = (size_t)blockIdx.x * E + i;
        out[o] = v;
        put_operand(op, o, v);
    }
}

// ------------------------------------------------------------------------------
// B = 1 GEMV with split-K across CTAs and an in-order last-CTA reduction
// ------------------------------------------------------------------------------
template <typename WT>
struct GemvArgs {
    const float *x;
    const WT *W;
    const WT *ln_g, *ln_b;
    float *partial;
    unsigned *counters;
    int N, K;
    Epi<WT> e;
};

template <typename WT>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs<WT> a) {
    pdl_wait();
    pdl_launch();
    constexpr int VN = Vec<WT>::n, BN = 16 * VN;
    extern __shared__ float smem[];
    __shared__ float sh[32];
    __shared__ int s_last;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int tile = blockIdx.x, ks = blockIdx.y, ksplit = gridDim.y;
    const int kchunk = a.K / ksplit, k0 = ks * kchunk;
    float *xs = smem;
    float *red = smem + kchunk;

    float mean = 0.0f, rstd = 1.0f;
    if (a.ln_g) ln_stats(a.x, a.K, sh, mean, rstd);
    for (int i = tid; i < kchunk; i += 256) {
        float v = a.x[k0 + i];
        if (a.ln_g) v = (v - mean) * rstd * tof(a.ln_g[k0 + i]) + tof(a.ln_b[k0 + i]);
        xs[i] = v;
    }
    __syncthreads();

    const int n0 = tile * BN + tx * VN;
    float acc[VN];
#pragma unroll
    for (int c = 0; c < VN; ++c) acc[c] = 0.0f;
    if (n0 < a.N) {
        const WT *wp = a.W + (size_t)(k0 + ty) * a.N + n0;
        const size_t step = (size_t)16 * a.N;
        const int iters = kchunk >> 4;
        int it = 0;
        for (; it + 4 <= iters; it += 4) {
            uint4 w0 = ld_stream(wp), w1 = ld_stream(wp + step), w2 = ld_stream(wp + 2 * step),
                  w3 = ld_stream(wp + 3 * step);
            wp += 4 * step;
            fma_vec(acc, w0, xs[ty + (it + 0) * 16], WT());
            fma_vec(acc, w1, xs[ty + (it + 1) * 16], WT());
            fma_vec(acc, w2, xs[ty + (it + 2) * 16], WT());
            fma_vec(acc, w3, xs[ty + (it + 3) * 16], WT());
        }
        for (; it < iters; ++it) {
            uint4 w0 = ld_stream(wp);
            wp += step;
            fma_vec(acc, w0, xs[ty + it * 16], WT());
        }
    }
#pragma unroll
    for (int c = 0; c < VN; ++c) red[ty * BN + tx * VN + c] = acc[c];
    __syncthreads();
    float colsum = 0.0f;
    const int n = tile * BN + tid;
    if (tid < BN) {
        for (int t = 0; t < 16; ++t) colsum += red[t * BN + tid];
    }
    if (ksplit == 1) {
        if (tid < BN && n < a.N) a.e.apply(0, n, colsum);
        return;
    }
    if (tid < BN && n < a.N) a.partial[(size_t)ks * a.N + n] = colsum;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.counters[tile], 1u) == (unsigned)(ksplit - 1));
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid < BN && n < a.N) {
        float s = 0.0f;
        for (int k = 0; k < ksplit; ++k) s += __ldcg(&a.partial[(size_t)k * a.N + n]);
        a.e.apply(0, n, s);
    }
    if (tid == 0) a.counters[tile] = 0u;
}

// ------------------------------------------------------------------------------
// Rows GEMM (SIMT fp32): C[M][N] = A[M][K] * W, W either [K][N] or (BT) [N][K]
// ------------------------------------------------------------------------------
template <typename WT>
struct GemmArgs {
    const float *A;
    const WT *W;
    int M, N, K;
    Epi<WT> e;
};

template <typename WT, int BM, bool BT>
__global__ void __launch_bounds__(256) gemm_kernel(GemmArgs<WT> a) {
    pdl_wait();
    pdl_launch();
    constexpr int BN = 64, BK = 16, TM = BM / 16;
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[TM][4];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int k0 = 0; k0 < a.K; k0 += BK) {
        // A tile: BM rows x 16 k as float4 (BM*4 vectors)
        for (int idx = tid; idx < BM * 4; idx += 256) {
            const int row = idx >> 2, c4 = idx & 3;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m0 + row < a.M) v = *reinterpret_cast<const float4 *>(a.A + (size_t)(m0 + row) * a.K + k0 + c4 * 4);
            As[c4 * 4 + 0][row] = v.x;
            As[c4 * 4 + 1][row] = v.y;
            As[c4 * 4 + 2][row] = v.z;
            As[c4 * 4 + 3][row] = v.w;
        }
        if (!BT) {
            // W [K][N]: 16 rows x 64 columns
            for (int idx = tid; idx < BK * BN; idx += 256) {
                const int row = idx >> 6, col = idx & 63;
                const int n = n0 + col;
                Bs[row][col] = n < a.N ? tof(a.W[(size_t)(k0 + row) * a.N + n]) : 0.0f;
            }
        } else {
            // W [N][K]: 64 rows (outputs) x 16 k
            for (int idx = tid; idx < BK * BN; idx += 256) {
                const int col = idx >> 4, kk = idx & 15;
                const int n = n0 + col;
                Bs[kk][col] = n < a.N ? tof(a.W[(size_t)n * a.K + k0 + kk]) : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float av[TM];
#pragma unroll
            for (int i = 0; i < TM; ++i) av[i] = As[kk][ty * TM + i];
            const float4 bv = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
#pragma unroll
            for (int i = 0; i < TM; ++i) {
                acc[i][0] = fmaf(av[i], bv.x, acc[i][0]);
                acc[i][1] = fmaf(av[i], bv.y, acc[i][1]);
                acc[i][2] = fmaf(av[i], bv.z, acc[i][2]);
                acc[i][3] = fmaf(av[i], bv.w, acc[i][3]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int r = m0 + ty * TM + i;
        if (r >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < a.N) a.e.apply(r, n, acc[i][j]);
        }
    }
}

// ------------------------------------------------------------------------------
// Single-query attention, flash-decoding split over keys
// ------------------------------------------------------------------------------
template <typename KT>
struct AttnArgs {
    const float *qkv;
    int qkv_stride;
    KVLayout kv;
    int layer;
    Rows rows;
    float *out;
    int out_stride;
    float *partial;      // [rows][heads][max_splits][66]
    unsigned *counters;  // [rows][heads]
    int max_splits;
    OperandOut op;       // the output also as the next GEMM's operand (row stride out_stride)
    const float *qpart;  // c_attn split-K partials [partials][rows][qkv_stride], or nullptr (qkv holds the sums)
    SplitInfo qsi;       // partials per column
    long long qtotal;    // rows * qkv_stride
    const KT *qbias;     // c_attn bias [3E]
    int *err;            // attn_stream_kernel: G2_ERR_TIMEOUT if a wait expired
};

template <typename KT>
__global__ void __launch_bounds__(128, sizeof(KT) == 4 ? 3 : 4) attn_kernel(AttnArgs<KT> a) {
    pdl_wait();
    pdl_launch();
    constexpr int CH = kAttnChunk;              // keys per chunk: one per thread in the score pass
    constexpr int VN = 16 / sizeof(KT);         // elements per 16-byte load
    constexpr int DG = kHeadDim / VN;           // 16-byte groups per 64-dim row (8 fp16, 16 fp32)
    constexpr int KG = 128 / DG;                // key groups of the P.V pass
    constexpr int VPT = CH / KG;                // V slices per thread in the P.V pass
    constexpr int VPF = VPT <= 8 ? VPT : 8;     // of which requested together with the keys
    static_assert(CH == 128, "one key per thread");
    __shared__ float q[kHeadDim];
    __shared__ float p[CH];
    __shared__ float red[KG][kHeadDim];
    __shared__ float sh[32];
    __shared__ int s_last;
    __shared__ float knew[2][kHeadDim];   // k and v at pos, when summed here from the c_attn partials
    const int h = blockIdx.x, sp = blockIdx.y, r = blockIdx.z, tid = threadIdx.x;
    const int NH = a.kv.n_head;
    const int T = a.rows.pos[r] + 1;
    if (!G2_BOUNDS(T >= 1 && T <= a.kv.max_seq && a.rows.slot[r] >= 0 && a.rows.slot[r] < a.kv.n_slots, 104)) return;
    const int nsplit = (T + CH - 1) / CH;   // chunks; CTA sp takes chunks sp, sp + Y, ...
    const int Y = gridDim.y;
    if (sp >= nsplit) return;
    const int nparts = nsplit < Y ? nsplit : Y;
    const int slot = a.rows.slot[r];
    const int pos = T - 1;
    const long long base = (long long)slot * a.kv.slot_stride + (long long)a.layer * a.kv.layer_stride +
                           (long long)h * a.kv.max_seq * kHeadDim;
    const bool fused = a.qpart != nullptr;
    if (!fused) {
        if (tid < kHeadDim) q[tid] = a.qkv[(size_t)r * a.qkv_stride + h * kHeadDim + tid] * 0.125f;  // 1/sqrt(64)
    } else {
        // c_attn output = (sum of the splits in order) + bias, as its reduce would give
        const int E = a.qkv_stride / 3;
        const bool kv_here = sp == (nsplit - 1) % Y;   // this CTA takes the chunk with pos: k, v and their append
        for (int c = tid; c < (kv_here ? 3 : 1) * kHeadDim; c += blockDim.x) {
            const int part = c / kHeadDim, d = c % kHeadDim;   // 0 q, 1 k, 2 v
            const size_t col = (size_t)part * E + h * kHeadDim + d;
            // the partials' loads are issued eight at a time; the sum stays in split order
            const float *pc = a.qpart + (size_t)r * a.qkv_stride + col;
            const int ns = a.qsi.at((int)col);
            float acc = 0.0f;
            for (int s0 = 0; s0 < ns; s0 += 8) {
                float pv[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) pv[k] = s0 + k < ns ? pc[(size_t)(s0 + k) * a.qtotal] : 0.0f;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (s0 + k < ns) acc = s0 + k == 0 ? pv[0] : acc + pv[k];
            }
            const float v = acc + tof(a.qbias[col]);
            if (part == 0) {
                q[d] = v * 0.125f;
            } else {   // K / V append (split_kv, math.cl:367-383), kept at the cache's precision
                const KT st = fromf<KT>(v);
                KT *dst = reinterpret_cast<KT *>(part == 1 ? a.kv.k : a.kv.v) + base + (size_t)pos * kHeadDim + d;
                *dst = st;
                knew[part - 1][d] = tof(st);
            }
        }
    }
    const KT *K = reinterpret_cast<const KT *>(a.kv.k) + base;
    const KT *V = reinterpret_cast<const KT *>(a.kv.v) + base;
    const int dg = tid % DG, kg = tid / DG;
    // running online-softmax state over this CTA's chunks (acc: threads < 64, one dim each)
    float Mr = -FLT_MAX, Lr = 0.0f, acc = 0.0f;
    for (int ch = sp; ch < nsplit; ch += Y) {
        const int j0 = ch * CH;
        const int nj = min(CH, T - j0);
        // scores: one key per thread, its 64 dims in 16-byte loads issued together
        uint4 kw[DG];
        if (tid < nj) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(K + (size_t)(j0 + tid) * kHeadDim);
#pragma unroll
            for (int i = 0; i < DG; ++i) kw[i] = kr[i];
        }
        // The V slices this thread multiplies in the P.V pass (keys kg, kg + KG, ... of dims
        // dg * VN ..) do not depend on the scores: the first VPF of them are requested
        // with the keys, the rest right after the scores, so the pass waits for no load.
        // (With fused c_attn partials the value at pos comes from shared memory instead.)
        const int jpos = fused ? pos - j0 : -1;
        uint4 vw[VPT];
#pragma unroll
        for (int i = 0; i < VPF; ++i) {
            const int jj = kg + i * KG;
            if (jj < nj && jj != jpos) vw[i] = *reinterpret_cast<const uint4 *>(V + (size_t)(j0 + jj) * kHeadDim + dg * VN);
        }
        __syncthreads();   // q (and k, v at pos); the previous chunk's readers of p and red are done
        float s = -FLT_MAX;
        if (tid < nj) {
            float d = 0.0f;
            if (fused && j0 + tid == pos) {   // the key this pass appended: from shared memory
                for (int i = 0; i < kHeadDim; ++i) d = fmaf(knew[0][i], q[i], d);
            } else {
#pragma unroll
                for (int i = 0; i < DG; ++i) d += dot_vec(kw[i], q + i * VN, KT());
            }
            s = d;
        }
        asm volatile("" ::: "memory");   // the second half of the V slices after the key rows are dead
#pragma unroll
        for (int i = VPF; i < VPT; ++i) {
            const int jj = kg + i * KG;
            if (jj < nj && jj != jpos) vw[i] = *reinterpret_cast<const uint4 *>(V + (size_t)(j0 + jj) * kHeadDim + dg * VN);
        }
        const float m = block_max(s, sh);
        const float e = tid < nj ? expf(s - m) : 0.0f;
        p[tid] = e;
        const float l = block_sum(e, sh);   // its barriers also publish p
        // P.V: thread (kg, dg) sums keys kg, kg + KG, ... of dims dg * VN .. dg * VN + VN - 1
        float o[VN], o2[VN];
#pragma unroll
        for (int i = 0; i < VN; ++i) o[i] = o2[i] = 0.0f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int jj = kg + i * KG;
            if (jj >= nj) continue;
            if (jj == jpos) {
#pragma unroll
                for (int e = 0; e < VN; ++e) o[e] = fmaf(p[jj], knew[1][dg * VN + e], o[e]);
            } else if (i & 1) {
                fma_vec(o2, vw[i], p[jj], KT());
            } else {
                fma_vec(o, vw[i], p[jj], KT());
            }
        }
#pragma unroll
        for (int i = 0; i < VN; ++i) red[kg][dg * VN + i] = o[i] + o2[i];
        __syncthreads();
        float ac = 0.0f;
        if (tid < kHeadDim)
#pragma unroll
            for (int g = 0; g < KG; ++g) ac += red[g][tid];
        // merge this chunk into the running state
        const float Mn = fmaxf(Mr, m);
        const float so = expf(Mr - Mn), sn = expf(m - Mn);   // so = 0 on the first chunk
        acc = acc * so + ac * sn;
        Lr = Lr * so + l * sn;
        Mr = Mn;
    }
    if (nparts == 1) {
        if (tid < kHeadDim) {
            const size_t o = (size_t)r * a.out_stride + h * kHeadDim + tid;
            const float v = acc / Lr;
            a.out[o] = v;
            put_operand(a.op, o, v);
        }
        return;
    }
    float *P = a.partial + (((size_t)r * NH + h) * a.max_splits + sp) * (kHeadDim + 2);
    if (tid < kHeadDim) P[2 + tid] = acc;
    if (tid == 0) {
        P[0] = Mr;
        P[1] = Lr;
    }
    __threadfence();
    __syncthreads();
    unsigned *ctr = a.counters + (size_t)r * NH + h;
    if (tid == 0) s_last = (atomicAdd(ctr, 1u) == (unsigned)(nparts - 1));
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid < kHeadDim) {
        const float *P0 = a.partial + ((size_t)r * NH + h) * a.max_splits * (kHeadDim + 2);
        float M = -FLT_MAX;
        for (int i = 0; i < nparts; ++i) M = fmaxf(M, __ldcg(P0 + (size_t)i * (kHeadDim + 2)));
        float L = 0.0f, O = 0.0f;
        for (int i = 0; i < nparts; ++i) {
            const float *Pi = P0 + (size_t)i * (kHeadDim + 2);
            const float w = expf(__ldcg(Pi) - M);
            L = fmaf(__ldcg(Pi + 1), w, L);
            O = fmaf(__ldcg(Pi + 2 + tid), w, O);
        }
        const size_t o = (size_t)r * a.out_stride + h * kHeadDim + tid;
        a.out[o] = O / L;
        put_operand(a.op, o, O / L);
    }
    if (tid == 0) *ctr = 0u;
}

// ------------------------------------------------------------------------------
// Single-query attention of a batched decode step, streamed (attn_scores_1q,
// attn_softmax_1q, attn_out_1q, math.cl:388-476, for one token of each of R
// sequences), used when the attention sums c_attn's split-K partials itself.
//
// The work items are (row, head, 128-key chunk), row-major then head-major.
// CTA c of G takes items [c I / G, (c + 1) I / G), so every SM streams about the
// same number of K and V bytes.  A CTA stages its items' K and V chunks in a
// two-stage shared-memory ring with one bulk copy each (the rows are
// contiguous), computes each chunk from shared memory and merges consecutive
// chunks of one (row, head) with the online softmax.  A (row, head) whose
// chunks span several CTAs is finished by the last of them to arrive (partials
// in slice order, as attn_kernel does).  The first stages are requested before
// the wait for the previous kernel: the cached K and V rows before the step's
// position were written by earlier steps, and the row at the position comes from
// the summed c_attn partials, not from the cache.  Every wait is bounded; on
// expiry the CTA records G2_ERR_TIMEOUT in a.err, waits (bounded) for its own
// copies in flight and returns.
// ------------------------------------------------------------------------------
namespace {
constexpr int kAsThreads = 256;
constexpr int kAsStages = 2;
constexpr int kAsMaxRows = 256;        // rows (sequences) one launch may take
typedef unsigned long long u64a;
__device__ __forceinline__ unsigned as_smem(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ u64a as_time() {
    u64a t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool as_try(u64a *b, unsigned par) {
    unsigned ok;
    asm volatile("{ .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok)
                 : "r"(as_smem(b)), "r"(par)
                 : "memory");
    return ok != 0;
}
// Wait for phase `par` of b for at most 1 s.
__device__ __forceinline__ bool as_wait(u64a *b, unsigned par) {
    if (as_try(b, par)) return true;
    const u64a lim = as_time() + 1000000000ull;
    for (;;) {
        if (as_try(b, par)) return true;
        if (as_time() > lim) return false;
    }
}
// 2-D tiled TMA load of box (x, y) of map into shared memory (signals bar)
__device__ __forceinline__ void as_tma2d(void *dst, const CUtensorMap *map, int x, int y, u64a *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            as_smem(dst)),
        "l"(reinterpret_cast<u64a>(map)), "r"(x), "r"(y), "r"(as_smem(bar))
        : "memory");
}
// Tensor-core pieces of the fp16 path: m16n8k16 (fp16 operands, fp32 accumulation),
// ldmatrix of 8 x 8 fp16 tiles, and the byte offset of 16-byte chunk c of row r in
// a tile of 128-byte rows stored with the 128-byte swizzle (what the TMA load writes).
__device__ __forceinline__ void mma16816(float (&d)[4], const unsigned (&a)[4], unsigned b0, unsigned b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(unsigned (&r)[4], unsigned addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(unsigned (&r)[4], unsigned addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ unsigned swz128(int r, int c) { return (unsigned)(r * 128 + ((c ^ (r & 7)) << 4)); }
__device__ __forceinline__ unsigned pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const unsigned *>(&h);
}
__device__ __forceinline__ void as_bulk(void *dst, const void *src, unsigned bytes, u64a *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     as_smem(dst)),
                 "l"(src), "r"(bytes), "r"(as_smem(bar))
                 : "memory");
}
}  // namespace

// Keys per item: 128 for fp16 caches, 64 for fp32 (a two-stage ring of 32 KB
// stages either way, so that three CTAs share an SM).
template <typename KT>
__host__ __device__ constexpr int as_chunk() {
    return sizeof(KT) == 2 ? 128 : 64;
}
// Dynamic shared memory: the ring (1 KB more for the alignment of the swizzled tiles).
size_t attn_stream_smem(int elem) { return (size_t)kAsStages * 2 * (elem == 2 ? 128 : 64) * kHeadDim * elem + 1024; }

// MMA (fp16 caches with their tensor maps mk, mv): each K and V chunk arrives by one
// tiled TMA load in the 128-byte swizzle, and each warp computes its 16 keys' scores
// (K tile x q) and P.V (P x V tile, V read transposed by ldmatrix) with m16n8k16
// tensor-core operations, fp16 operands (q and the probabilities rounded to fp16, as
// the fp16 engine's GEMM operands are) and fp32 accumulation.  The cache row at the
// step's position is patched into the staged tiles from the summed c_attn partials.
template <typename KT, bool MMA>
__global__ void __launch_bounds__(kAsThreads, 3)
    attn_stream_kernel(AttnArgs<KT> a, int nrows, const __grid_constant__ CUtensorMap mk,
                       const __grid_constant__ CUtensorMap mv) {
    constexpr int CH = as_chunk<KT>();               // keys per item
    constexpr int NW = kAsThreads / 32;              // warps
    constexpr int KPW = CH / NW;                     // keys per warp: 16 (fp16) or 8 (fp32)
    constexpr int TPK = 32 / KPW;                    // threads per key in the score pass: 2 or 4
    constexpr int EPC = 16 / sizeof(KT);             // elements per 16-byte chunk of a key row
    constexpr int CB = CH * kHeadDim * sizeof(KT);   // bytes of a full K (or V) chunk
    static_assert(kHeadDim * sizeof(KT) == TPK * 64, "each thread of a key reads four 16-byte chunks");
    static_assert(!MMA || sizeof(KT) == 2, "the tensor-core path takes fp16 caches");
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char *ring =                            // [stage][K chunk, V chunk], 1024-byte aligned
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ u64a full[kAsStages];
    __shared__ float q[kHeadDim];
    __shared__ float wo[NW][kHeadDim], wm[NW], wl[NW];   // per-warp partial (o, max, sum)
    __shared__ float knew[2][kHeadDim];
    __shared__ int nch[kAsMaxRows], off[kAsMaxRows + 1], rpos[kAsMaxRows], rslot[kAsMaxRows];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, NH = a.kv.n_head;
    if (tid == 0) {
        for (int s = 0; s < kAsStages; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(as_smem(&full[s])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // items per row (chunks of its keys, per head), their prefix sums, positions and slots
    for (int r = tid; r < nrows; r += kAsThreads) {
        const int T = a.rows.pos[r] + 1, sl = a.rows.slot[r];
        const bool ok = G2_BOUNDS(T >= 1 && T <= a.kv.max_seq && sl >= 0 && sl < a.kv.n_slots, 107);
        nch[r] = ok ? (T + CH - 1) / CH : 0;
        rpos[r] = T - 1;
        rslot[r] = sl;
    }
    __syncthreads();
    if (tid == 0) {
        off[0] = 0;
        for (int r = 0; r < nrows; ++r) off[r + 1] = off[r] + NH * nch[r];
    }
    __syncthreads();
    // the items are shared over G = min(grid, I) CTAs, so that every CTA of the
    // partition holds at least one (the part counts of the merge rely on it)
    const long long I = off[nrows];
    const int G = (int)(I < (long long)gridDim.x ? I : (long long)gridDim.x), c = blockIdx.x;
    const int i0 = c < G ? (int)((long long)c * I / G) : 0, i1 = c < G ? (int)((long long)(c + 1) * I / G) : 0;
    // A cursor over (row, head, chunk): placed by one scan, then advanced in O(1).
    struct Cur {
        int r, h, ch;
    };
    auto place = [&](int i) {
        Cur u;
        u.r = 0;
        while (off[u.r + 1] <= i) ++u.r;
        const int j = i - off[u.r];
        u.h = j / nch[u.r];
        u.ch = j - u.h * nch[u.r];
        return u;
    };
    auto next = [&](Cur &u) {
        if (++u.ch == nch[u.r]) {
            u.ch = 0;
            if (++u.h == NH) {
                u.h = 0;
                do ++u.r;
                while (u.r < nrows && nch[u.r] == 0);
            }
        }
    };
    auto kv_base = [&](int r, int h) -> long long {
        return (long long)rslot[r] * a.kv.slot_stride + (long long)a.layer * a.kv.layer_stride +
               (long long)h * a.kv.max_seq * kHeadDim;
    };
    // thread 0: request item (cursor u, index i)'s K and V rows into stage (i - i0) % kAsStages
    auto issue = [&](const Cur &u, int i) {
        const int T = rpos[u.r] + 1, j0 = u.ch * CH, nj = min(CH, T - j0);
        const int s = (i - i0) % kAsStages;
        u64a *bar = &full[s];
        if (MMA) {   // 64-row boxes covering the chunk's keys (rows past them: weighted 0)
            const int nbox = (nj + 63) / 64;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(as_smem(bar)),
                         "r"((unsigned)(nbox * CB))
                         : "memory");
            const int row = (int)((kv_base(u.r, u.h) + (long long)j0 * kHeadDim) / kHeadDim);
            for (int b = 0; b < nbox; ++b) {
                as_tma2d(ring + (size_t)s * 2 * CB + b * (CB / 2), &mk, 0, row + 64 * b, bar);
                as_tma2d(ring + (size_t)s * 2 * CB + CB + b * (CB / 2), &mv, 0, row + 64 * b, bar);
            }
            return;
        }
        const unsigned bytes = (unsigned)(nj * kHeadDim * sizeof(KT));
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(as_smem(bar)), "r"(2 * bytes)
                     : "memory");
        const long long b = kv_base(u.r, u.h) + (long long)j0 * kHeadDim;
        as_bulk(ring + (size_t)s * 2 * CB, reinterpret_cast<const KT *>(a.kv.k) + b, bytes, bar);
        as_bulk(ring + (size_t)s * 2 * CB + CB, reinterpret_cast<const KT *>(a.kv.v) + b, bytes, bar);
    };
    if (MMA) {   // the ring starts as zeros: rows a short chunk leaves unloaded are read with weight 0
        uint4 *z = reinterpret_cast<uint4 *>(ring);
        for (int k = tid; k < kAsStages * 2 * CB / 16; k += kAsThreads) z[k] = make_uint4(0u, 0u, 0u, 0u);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // before the TMA writes
        __syncthreads();
    }
    Cur iu{0, 0, 0};   // thread 0's issue cursor
    if (tid == 0 && i0 < i1) {
        iu = place(i0);
        for (int i = i0; i < i1 && i < i0 + kAsStages; ++i) {
            issue(iu, i);
            next(iu);
        }
    }
    pdl_wait();
    pdl_launch();
    const int E = a.qkv_stride / 3;
    // score pass: lane (kl, part) of warp w takes key w KPW + kl, 16-byte chunks 4 part .. 4 part + 3
    // of its row, read in an order rotated by the key (bank-conflict free); q in that order in registers
    const int kl = lane / TPK, part = lane % TPK;
    int rot[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) rot[t] = part * 4 + ((t + kl + (TPK == 4 && part >= 2 ? 2 : 0)) & 3);
    float qr[4][EPC];
    unsigned qb[4][2];   // MMA: q as the B operand of the score products
    float Mr = -FLT_MAX, Lr = 0.0f, acc = 0.0f;      // running softmax of the current (row, head), threads < 64
    Cur u{0, 0, 0};
    if (i0 < i1) u = place(i0);
    for (int i = i0; i < i1; ++i, next(u)) {
        const int r = u.r, h = u.h, ch = u.ch;
        const int T = rpos[r] + 1, pos = T - 1, j0 = ch * CH, nj = min(CH, T - j0);
        const int s = (i - i0) % kAsStages;
        const bool fresh = i == i0 || ch == 0;       // a new (row, head) run of this CTA
        if (fresh) {
            Mr = -FLT_MAX;
            Lr = 0.0f;
            acc = 0.0f;
        }
        {   // q at a run's start, and at the chunk with pos also k and v (appended), from c_attn's partials
            const bool kv_here = ch == nch[r] - 1;
            for (int cc = tid; cc < 3 * kHeadDim; cc += kAsThreads) {
                const int pt = cc / kHeadDim, d = cc % kHeadDim;
                if (pt == 0 ? !fresh : !kv_here) continue;
                const size_t col = (size_t)pt * E + h * kHeadDim + d;
                const float *pc = a.qpart + (size_t)r * a.qkv_stride + col;
                const int ns = a.qsi.at((int)col);
                float sum = 0.0f;
                for (int s0 = 0; s0 < ns; s0 += 8) {   // loads issued eight at a time, summed in split order
                    float pv[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) pv[k] = s0 + k < ns ? pc[(size_t)(s0 + k) * a.qtotal] : 0.0f;
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (s0 + k < ns) sum = s0 + k == 0 ? pv[0] : sum + pv[k];
                }
                const float v = sum + tof(a.qbias[col]);
                if (pt == 0) {
                    q[d] = v * 0.125f;   // 1/sqrt(64)
                } else {   // K / V append (split_kv, math.cl:367-383), kept at the cache's precision
                    const KT stv = fromf<KT>(v);
                    KT *dst = reinterpret_cast<KT *>(pt == 1 ? a.kv.k : a.kv.v) + kv_base(r, h) + (size_t)pos * kHeadDim + d;
                    *dst = stv;
                    knew[pt - 1][d] = tof(stv);
                }
            }
        }
        // this item's K and V in shared memory (bounded wait; a failure is carried by the barrier)
        const int fail = as_wait(&full[s], (unsigned)(((i - i0) / kAsStages) & 1)) ? 0 : 1;
        if (__syncthreads_or(fail)) {
            if (tid == 0) {
                atomicCAS(a.err, 0, G2_ERR_TIMEOUT);
                // copies this CTA issued and nobody consumed: wait for them (bounded) before exiting
                for (int k = i + 1; k < i1 && k < i + kAsStages; ++k)
                    as_wait(&full[(k - i0) % kAsStages], (unsigned)(((k - i0) / kAsStages) & 1));
            }
            return;
        }
        if constexpr (MMA) {
            const unsigned kb = as_smem(ring + (size_t)s * 2 * CB), vb = kb + CB;
            const int jpos = pos - j0;   // the key at pos (this step's), if in this chunk
            if (jpos >= 0 && jpos < nj) {   // its K and V rows into the staged tiles, from the summed partials
                if (tid < 2 * kHeadDim) {
                    const int d = tid & (kHeadDim - 1), w = tid >> 6;
                    __half *dst = reinterpret_cast<__half *>(ring + (size_t)s * 2 * CB + (w ? CB : 0) +
                                                             swz128(jpos, d >> 3) + (d & 7) * 2);
                    *dst = __float2half_rn(knew[w][d]);
                }
                // these generic writes come before the TMA that next fills this stage
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncthreads();
            }
            const int g = lane >> 2, t = lane & 3, q8 = lane >> 3;
            if (fresh) {   // q as the B operand: column 0 only (lanes of group 0), fp16
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    qb[k][0] = g == 0 ? pack_h2(q[16 * k + 2 * t], q[16 * k + 2 * t + 1]) : 0u;
                    qb[k][1] = g == 0 ? pack_h2(q[16 * k + 8 + 2 * t], q[16 * k + 9 + 2 * t]) : 0u;
                }
            }
            const int r0 = warp * 16;                              // this warp's 16 keys of the chunk
            const int lrow = r0 + (q8 & 1) * 8 + (lane & 7);       // the row this lane addresses for ldmatrix
            float sd[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k = 0; k < 4; ++k) {   // dims 16 k .. 16 k + 15
                unsigned af[4];
                ldsm_x4(af, kb + swz128(lrow, 2 * k + (q8 >> 1)));
                mma16816(sd, af, qb[k][0], qb[k][1]);
            }
            // column 0 (lanes t == 0): sd[0] = score of key r0 + g, sd[2] = of key r0 + g + 8
            const bool va = t == 0 && r0 + g < nj, vb8 = t == 0 && r0 + g + 8 < nj;
            const float m = warp_max(fmaxf(va ? sd[0] : -FLT_MAX, vb8 ? sd[2] : -FLT_MAX));
            const float p0 = va ? expf(sd[0] - m) : 0.0f, p1 = vb8 ? expf(sd[2] - m) : 0.0f;
            const float l = warp_sum(p0 + p1);
            // P as the A operand: row 0 holds keys r0 .. r0 + 15 (lanes of group 0), fp16
            const float pa = __shfl_sync(0xffffffffu, p0, 8 * t), pb = __shfl_sync(0xffffffffu, p0, 8 * t + 4);
            const float pc = __shfl_sync(0xffffffffu, p1, 8 * t), pd = __shfl_sync(0xffffffffu, p1, 8 * t + 4);
            const unsigned pf[4] = {g == 0 ? pack_h2(pa, pb) : 0u, 0u, g == 0 ? pack_h2(pc, pd) : 0u, 0u};
            float o[8][4];
#pragma unroll
            for (int nb = 0; nb < 8; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {   // dims 16 u .. 16 u + 15: two n-blocks of 8
                unsigned bf[4];
                ldsm_x4_t(bf, vb + swz128(lrow, 2 * u + (q8 >> 1)));
                mma16816(o[2 * u], pf, bf[0], bf[1]);
                mma16816(o[2 * u + 1], pf, bf[2], bf[3]);
            }
            if (g == 0)   // row 0 of each n-block: dims 8 nb + 2 t, + 1
#pragma unroll
                for (int nb = 0; nb < 8; ++nb) {
                    wo[warp][8 * nb + 2 * t] = o[nb][0];
                    wo[warp][8 * nb + 2 * t + 1] = o[nb][1];
                }
            if (lane == 0) {
                wm[warp] = m;
                wl[warp] = l;
            }
        } else {
        if (fresh) {
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
                for (int e = 0; e < EPC; ++e) qr[t][e] = q[rot[t] * EPC + e];
        }
        const KT *Ks = reinterpret_cast<const KT *>(ring + (size_t)s * 2 * CB);
        const KT *Vs = reinterpret_cast<const KT *>(ring + (size_t)s * 2 * CB + CB);
        const int jpos = pos - j0;   // the key at pos (this step's), if in this chunk: from knew
        const int j = warp * KPW + kl;
        float sc = 0.0f;
        if (j < nj) {
            if (j == jpos) {
#pragma unroll
                for (int t = 0; t < 4; ++t)
#pragma unroll
                    for (int e = 0; e < EPC; ++e) sc = fmaf(knew[0][rot[t] * EPC + e], qr[t][e], sc);
            } else {
                const uint4 *kr = reinterpret_cast<const uint4 *>(Ks + (size_t)j * kHeadDim);
                uint4 w[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) w[t] = kr[rot[t]];
#pragma unroll
                for (int t = 0; t < 4; ++t) sc += dot_vec(w[t], qr[t], KT());
            }
        }
#pragma unroll
        for (int o = 1; o < TPK; o <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
        // the warp's softmax over its keys, then P.V: lane l takes dims 2 l, 2 l + 1
        const float m = warp_max(j < nj ? sc : -FLT_MAX);
        const float pj = j < nj ? expf(sc - m) : 0.0f;
        const float l = warp_sum(part == 0 ? pj : 0.0f);
        // every slot of the warp is read (rows past nj hold stale data: their weight
        // and value are selected to 0, so nothing of them reaches the sums), so that
        // the loop has no exit and its loads and shuffles are issued ahead
        const int kmax = nj - warp * KPW;   // valid keys of this warp (may be <= 0)
        float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int k = 0; k < KPW; ++k) {
            const int jj = warp * KPW + k;
            const bool in = k < kmax;
            const float ps = __shfl_sync(0xffffffffu, pj, k * TPK);
            const float pk = in ? ps : 0.0f;
            float2 f;
            if (sizeof(KT) == 2)
                f = __half22float2(reinterpret_cast<const __half2 *>(Vs + (size_t)jj * kHeadDim)[lane]);
            else
                f = reinterpret_cast<const float2 *>(Vs + (size_t)jj * kHeadDim)[lane];
            if (jj == jpos) f = make_float2(knew[1][2 * lane], knew[1][2 * lane + 1]);
            o0 = fmaf(pk, in ? f.x : 0.0f, o0);
            o1 = fmaf(pk, in ? f.y : 0.0f, o1);
        }
        wo[warp][2 * lane] = o0;
        wo[warp][2 * lane + 1] = o1;
        if (lane == 0) {
            wm[warp] = m;
            wl[warp] = l;
        }
        }   // the CUDA-core path
        __syncthreads();
        // the stage is free again: request the item kAsStages ahead into it
        if (tid == 0 && i + kAsStages < i1) {
            issue(iu, i + kAsStages);
            next(iu);
        }
        if (tid < kHeadDim) {   // the warps' partials merged in warp order, then into the run
            float M = -FLT_MAX;
#pragma unroll
            for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w]);
            float lc = 0.0f, oc = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float f = expf(wm[w] - M);   // 0 for a warp without keys
                lc = fmaf(wl[w], f, lc);
                oc = fmaf(wo[w][tid], f, oc);
            }
            const float Mn = fmaxf(Mr, M);
            const float so = expf(Mr - Mn), sn = expf(M - Mn);   // so = 0 on a run's first chunk
            acc = acc * so + oc * sn;
            Lr = Lr * so + lc * sn;
            Mr = Mn;
        }
        // the end of this (row, head) in this CTA: finish it, or hand in a partial
        if (ch == nch[r] - 1 || i == i1 - 1) {
            const long long u0 = off[r] + (long long)h * nch[r];     // the (row, head)'s first item
            const int c0 = (int)(((u0 + 1) * G - 1) / I);            // CTAs holding its first and last items
            const int c1 = (int)(((u0 + nch[r]) * G - 1) / I);
            const int nparts = c1 - c0 + 1, seg = c - c0;
            const size_t o = (size_t)r * a.out_stride + h * kHeadDim + tid;
            if (nparts == 1) {
                if (tid < kHeadDim) {
                    a.out[o] = acc / Lr;
                    put_operand(a.op, o, acc / Lr);
                }
            } else {
                float *P = a.partial + (((size_t)r * NH + h) * a.max_splits + seg) * (kHeadDim + 2);
                if (tid < kHeadDim) P[2 + tid] = acc;
                if (tid == 0) {
                    P[0] = Mr;
                    P[1] = Lr;
                }
                // the CTA barrier orders every thread's partial before thread 0's release;
                // the last arrival's acquire (then the barrier) orders the reads after all
                __syncthreads();
                unsigned *ctr = a.counters + (size_t)r * NH + h;
                if (tid == 0) {
                    unsigned prev;
                    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
                    s_last = prev == (unsigned)(nparts - 1);
                }
                __syncthreads();
                if (s_last) {
                    if (tid < kHeadDim) {
                        const float *P0 = a.partial + ((size_t)r * NH + h) * a.max_splits * (kHeadDim + 2);
                        float M = -FLT_MAX;
                        for (int k = 0; k < nparts; ++k) M = fmaxf(M, __ldcg(P0 + (size_t)k * (kHeadDim + 2)));
                        float L = 0.0f, O = 0.0f;
                        for (int k = 0; k < nparts; ++k) {
                            const float *Pk = P0 + (size_t)k * (kHeadDim + 2);
                            const float w = expf(__ldcg(Pk) - M);
                            L = fmaf(__ldcg(Pk + 1), w, L);
                            O = fmaf(__ldcg(Pk + 2 + tid), w, O);
                        }
                        a.out[o] = O / L;
                        put_operand(a.op, o, O / L);
                    }
                    if (tid == 0) *ctr = 0u;
                }
            }
        }
        __syncthreads();   // q, knew and the warp partials are reused by the next item
    }
}

// ------------------------------------------------------------------------------
// Single-query attention of a batched decode step over fp16 caches, one warp per
// run of keys (attn_scores_1q, attn_softmax_1q, attn_out_1q, math.cl:388-476, for
// one token of each of R sequences).
//
// The work items are (row, head, 64-key chunk), row-major then head-major, and
// warp w of W takes items [w I / W, (w + 1) I / W).  W is the number of (row,
// head) runs times the whole number of warps each can have (at least one; fewer
// warps than runs: the warps' shares hold several runs), so when the rows have
// equal positions every warp streams exactly one run, or an equal share of one.
// Each warp:
//   * requests its chunks' K and V tiles (64 rows x 128 B, 128-byte swizzle) by
//     TMA into its own three-stage ring, the first stages before the wait for
//     the previous kernel (the cached rows before each step's position were
//     written by earlier steps);
//   * sums q from c_attn's split-K partials at a run's start, together with the
//     new K and V rows when its share holds the run's last chunk; it appends
//     those to the cache (split_kv, math.cl:367-383) and patches them into the
//     staged tile at the step's position;
//   * computes the chunk's scores (K tile x q: the keys on the MMA's m, q as
//     column 0 of B) and P.V as V^T P (the dims on m, the V tile read transposed
//     by ldmatrix as the A operand, P as column 0 of B) with m16n8k16 tensor-core
//     operations -- 32 a chunk, each using one column of its 8, which is why
//     the time of a chunk follows their count -- fp16 operands (q and the
//     probabilities rounded to fp16, as the fp16 engine's GEMM operands are) and
//     fp32 accumulation, and keeps the run's online softmax -- running maximum,
//     sum and the 64 outputs, the latter in the MMA accumulators -- in registers;
//   * at the end of its share of a run writes the output (and the next GEMM's
//     operand), or hands in a partial that the last warp of the run to arrive
//     merges in slice order.
// After the set-up no CTA-wide barrier is taken: a warp never waits for another.
// Every wait is bounded; on expiry the warp records G2_ERR_TIMEOUT in a.err, waits
// (bounded) for its own copies in flight and returns.
// ------------------------------------------------------------------------------
namespace {
constexpr int kAwWarps = 4;                        // warps per CTA
constexpr int kAwStages = 3;                       // ring stages per warp
constexpr int kAwChunk = 64;                       // keys per item (one 64-row TMA box of K and of V)
constexpr int kAwTile = kAwChunk * kHeadDim * 2;   // bytes of one staged K (or V) tile: 8 KB
constexpr int kAwCols = 3 * kHeadDim / 32;         // q, k, v columns of a head per lane: 6
}  // namespace
size_t attn_warp_smem() { return (size_t)kAwWarps * kAwStages * 2 * kAwTile + 1024; }

__global__ void __launch_bounds__(kAwWarps * 32, 1)
    attn_warp_kernel(AttnArgs<__half> a, int nrows, int wmax, const __grid_constant__ CUtensorMap mk,
                     const __grid_constant__ CUtensorMap mv) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char *ring =   // [warp][stage][K tile, V tile], 1024-byte aligned
        reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ u64a full[kAwWarps][kAwStages];
    __shared__ float qs[kAwWarps][kHeadDim];
    __shared__ float knew[kAwWarps][2][kHeadDim];
    __shared__ int nch[kAsMaxRows], off[kAsMaxRows + 1], rpos[kAsMaxRows], rslot[kAsMaxRows];
    __shared__ int s_runs;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, NH = a.kv.n_head;
    if (tid == 0) {
        for (int w = 0; w < kAwWarps; ++w)
            for (int s = 0; s < kAwStages; ++s)
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(as_smem(&full[w][s])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // chunks per row (of its keys, per head), their prefix sums, positions and slots
    for (int r = tid; r < nrows; r += kAwWarps * 32) {
        const int T = a.rows.pos[r] + 1, sl = a.rows.slot[r];
        const bool ok = G2_BOUNDS(T >= 1 && T <= a.kv.max_seq && sl >= 0 && sl < a.kv.n_slots, 108);
        nch[r] = ok ? (T + kAwChunk - 1) / kAwChunk : 0;
        rpos[r] = T - 1;
        rslot[r] = sl;
    }
    __syncthreads();
    if (tid == 0) {
        int runs = 0;
        off[0] = 0;
        for (int r = 0; r < nrows; ++r) {
            off[r + 1] = off[r] + NH * nch[r];
            runs += nch[r] ? NH : 0;
        }
        s_runs = runs;
    }
    __syncthreads();
    // W <= I, so that every warp of the partition holds at least one item (the part
    // counts of the merge rely on it)
    const long long I = off[nrows];
    const int runs = s_runs;
    long long Wl = runs == 0 ? 0 : (runs <= wmax ? (long long)runs * (wmax / runs) : (long long)wmax);
    if (Wl > I) Wl = I;
    const int W = (int)Wl, w = blockIdx.x * kAwWarps + warp;
    const int i0 = w < W ? (int)((long long)w * I / W) : 0, i1 = w < W ? (int)((long long)(w + 1) * I / W) : 0;
    unsigned char *wring = ring + (size_t)warp * kAwStages * 2 * kAwTile;
    u64a *wfull = full[warp];
    struct Cur {
        int r, h, ch;
    };
    auto place = [&](int i) {
        Cur u;
        u.r = 0;
        while (off[u.r + 1] <= i) ++u.r;
        const int j = i - off[u.r];
        u.h = j / nch[u.r];
        u.ch = j - u.h * nch[u.r];
        return u;
    };
    auto next = [&](Cur &u) {
        if (++u.ch == nch[u.r]) {
            u.ch = 0;
            if (++u.h == NH) {
                u.h = 0;
                do ++u.r;
                while (u.r < nrows && nch[u.r] == 0);
            }
        }
    };
    auto kv_base = [&](int r, int h) -> long long {
        return (long long)rslot[r] * a.kv.slot_stride + (long long)a.layer * a.kv.layer_stride +
               (long long)h * a.kv.max_seq * kHeadDim;
    };
    // lane 0: request item (cursor u, index i)'s K and V tiles into stage (i - i0) % kAwStages
    auto issue = [&](const Cur &u, int i) {
        const int s = (i - i0) % kAwStages;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(as_smem(&wfull[s])),
                     "r"((unsigned)(2 * kAwTile))
                     : "memory");
        const int row = (int)(kv_base(u.r, u.h) / kHeadDim) + u.ch * kAwChunk;
        as_tma2d(wring + (size_t)s * 2 * kAwTile, &mk, 0, row, &wfull[s]);
        as_tma2d(wring + (size_t)s * 2 * kAwTile + kAwTile, &mv, 0, row, &wfull[s]);
    };
    Cur iu{0, 0, 0};   // lane 0's issue cursor
    if (lane == 0 && i0 < i1) {
        iu = place(i0);
        for (int i = i0; i < i1 && i < i0 + kAwStages; ++i) {
            issue(iu, i);
            next(iu);
        }
    }
    pdl_wait();
    pdl_launch();
    if (i0 >= i1) return;   // a warp without items
    const int E = a.qkv_stride / 3;
    const int g = lane >> 2, t = lane & 3, q8 = lane >> 3;
    const int lrow = (q8 & 1) * 8 + (lane & 7);   // tile row (within 16) this lane addresses: K (A of the scores)
    const int krow = (q8 >> 1) * 8 + (lane & 7);  // and V (A of V^T P, read transposed)
    // P.V accumulators: column 0 (lanes t == 0) of m-tile dm holds dims 16 dm + g (o[dm][0]) and
    // 16 dm + g + 8 (o[dm][2])
    float o[4][4];
    float Mr = -FLT_MAX, Lr = 0.0f;               // the run's running maximum and sum
    unsigned qb[4][2];                            // q (column 0 of the scores' B operand): dims 16 k + 2 t, + 8
    Cur u = place(i0);
    for (int i = i0; i < i1; ++i, next(u)) {
        const int r = u.r, h = u.h, ch = u.ch;
        const int T = rpos[r] + 1, pos = T - 1, j0 = ch * kAwChunk, nj = min(kAwChunk, T - j0);
        const int s = (i - i0) % kAwStages;
        const bool fresh = i == i0 || ch == 0;   // a new (row, head) run of this warp
        if (fresh) {
            Mr = -FLT_MAX;
            Lr = 0.0f;
#pragma unroll
            for (int dm = 0; dm < 4; ++dm) o[dm][0] = o[dm][1] = o[dm][2] = o[dm][3] = 0.0f;
            // q, and the new k and v when this warp's share holds the run's last chunk (the one
            // with the step's position), from c_attn's partials: lane takes columns lane + 32 j
            // of the head's 192; all their partial loads are issued before any is summed, and
            // each column is summed in split order
            const bool kv_mine = off[r] + (long long)h * nch[r] + nch[r] - 1 < i1;
            const float *pcv[kAwCols];
            int nsv[kAwCols], nsmax = 0;
            float acc[kAwCols];
#pragma unroll
            for (int j = 0; j < kAwCols; ++j) {
                const int cc = lane + 32 * j, pt = cc >> 6, d = cc & (kHeadDim - 1);
                const size_t col = (size_t)pt * E + h * kHeadDim + d;
                const bool need = pt == 0 || kv_mine;
                pcv[j] = a.qpart + (size_t)r * a.qkv_stride + col;
                nsv[j] = need ? a.qsi.at((int)col) : 0;
                nsmax = max(nsmax, nsv[j]);
                acc[j] = 0.0f;
            }
            constexpr int QB = 8;   // partials per column per round
            for (int s0 = 0; s0 < nsmax; s0 += QB) {
                float pv[kAwCols][QB];
#pragma unroll
                for (int j = 0; j < kAwCols; ++j)
#pragma unroll
                    for (int k = 0; k < QB; ++k) pv[j][k] = s0 + k < nsv[j] ? pcv[j][(size_t)(s0 + k) * a.qtotal] : 0.0f;
#pragma unroll
                for (int j = 0; j < kAwCols; ++j)
#pragma unroll
                    for (int k = 0; k < QB; ++k)
                        if (s0 + k < nsv[j]) acc[j] = s0 + k == 0 ? pv[j][k] : acc[j] + pv[j][k];
            }
#pragma unroll
            for (int j = 0; j < kAwCols; ++j) {
                if (!nsv[j]) continue;
                const int cc = lane + 32 * j, pt = cc >> 6, d = cc & (kHeadDim - 1);
                const float v = acc[j] + tof(a.qbias[(size_t)pt * E + h * kHeadDim + d]);
                if (pt == 0) {
                    qs[warp][d] = v * 0.125f;   // 1/sqrt(64)
                } else {   // K / V append at the cache's precision
                    const __half stv = __float2half_rn(v);
                    __half *dst = reinterpret_cast<__half *>(pt == 1 ? a.kv.k : a.kv.v) + kv_base(r, h) +
                                  (size_t)pos * kHeadDim + d;
                    *dst = stv;
                    knew[warp][pt - 1][d] = __half2float(stv);
                }
            }
            __syncwarp();
            // q as column 0 of the scores' B operand (lanes of group 0), fp16
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                qb[k][0] = g == 0 ? pack_h2(qs[warp][16 * k + 2 * t], qs[warp][16 * k + 2 * t + 1]) : 0u;
                qb[k][1] = g == 0 ? pack_h2(qs[warp][16 * k + 8 + 2 * t], qs[warp][16 * k + 9 + 2 * t]) : 0u;
            }
        }
        // this item's K and V tiles (bounded wait)
        const bool ok = as_wait(&wfull[s], (unsigned)(((i - i0) / kAwStages) & 1));
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) {
                atomicCAS(a.err, 0, G2_ERR_TIMEOUT);
                // copies this warp issued and nobody consumed: wait for them (bounded) before exiting
                for (int k = i + 1; k < i1 && k < i + kAwStages; ++k)
                    as_wait(&wfull[(k - i0) % kAwStages], (unsigned)(((k - i0) / kAwStages) & 1));
            }
            return;
        }
        const unsigned kb = as_smem(wring + (size_t)s * 2 * kAwTile), vb = kb + kAwTile;
        const int jpos = pos - j0;   // the key at pos (this step's), if in this chunk
        if (jpos >= 0 && jpos < nj) {   // its K and V rows into the staged tiles, from the summed partials
#pragma unroll
            for (int e = lane; e < 2 * kHeadDim; e += 32) {
                const int d = e & (kHeadDim - 1), w2 = e >> 6;
                __half *dst = reinterpret_cast<__half *>(wring + (size_t)s * 2 * kAwTile + (w2 ? kAwTile : 0) +
                                                         swz128(jpos, d >> 3) + (d & 7) * 2);
                *dst = __float2half_rn(knew[warp][w2][d]);
            }
            // these generic writes come before the TMA that next fills this stage
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        }
        // scores with the keys on the MMA's m and q as column 0 of B: keys 16 mt + g (sd[mt][0])
        // and 16 mt + g + 8 (sd[mt][2]) in lanes t == 0
        float sd[4][4];
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            sd[mt][0] = sd[mt][1] = sd[mt][2] = sd[mt][3] = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {   // dims 16 k .. 16 k + 15
                unsigned af[4];
                ldsm_x4(af, kb + swz128(16 * mt + lrow, 2 * k + (q8 >> 1)));
                mma16816(sd[mt], af, qb[k][0], qb[k][1]);
            }
        }
        // online softmax over the run, among the lanes t == 0 (the others take no part)
        float mloc = -FLT_MAX;
        if (t == 0) {
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                if (nj == kAwChunk || 16 * mt + g < nj) mloc = fmaxf(mloc, sd[mt][0]);
                if (nj == kAwChunk || 16 * mt + g + 8 < nj) mloc = fmaxf(mloc, sd[mt][2]);
            }
        }
        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 4));
        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 8));
        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 16));
        const float mn = fmaxf(Mr, mloc);
        const float sc = __expf(Mr - mn);   // 0 at a run's first chunk
        float p0[4], p1[4], ls = 0.0f;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            p0[mt] = t == 0 && (nj == kAwChunk || 16 * mt + g < nj) ? __expf(sd[mt][0] - mn) : 0.0f;
            p1[mt] = t == 0 && (nj == kAwChunk || 16 * mt + g + 8 < nj) ? __expf(sd[mt][2] - mn) : 0.0f;
            ls += p0[mt] + p1[mt];
        }
        ls += __shfl_xor_sync(0xffffffffu, ls, 4);
        ls += __shfl_xor_sync(0xffffffffu, ls, 8);
        ls += __shfl_xor_sync(0xffffffffu, ls, 16);
        Lr = Lr * sc + ls;
        Mr = mn;
#pragma unroll
        for (int dm = 0; dm < 4; ++dm) {   // columns 1-7 of the accumulators stay 0
            o[dm][0] *= sc;
            o[dm][2] *= sc;
        }
        // P.V as V^T P: the dims on the MMA's m (V read transposed by ldmatrix as the A operand),
        // P as column 0 of B (lanes of group 0 hold keys 2 t, + 1 and 2 t + 8, + 9 of each step)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {   // keys 16 kk .. 16 kk + 15
            const float pa = __shfl_sync(0xffffffffu, p0[kk], 8 * t), pb = __shfl_sync(0xffffffffu, p0[kk], 8 * t + 4);
            const float pc = __shfl_sync(0xffffffffu, p1[kk], 8 * t), pd = __shfl_sync(0xffffffffu, p1[kk], 8 * t + 4);
            const unsigned b0 = g == 0 ? pack_h2(pa, pb) : 0u, b1 = g == 0 ? pack_h2(pc, pd) : 0u;
#pragma unroll
            for (int dm = 0; dm < 4; ++dm) {   // dims 16 dm .. 16 dm + 15
                unsigned af[4];
                ldsm_x4_t(af, vb + swz128(16 * kk + krow, 2 * dm + (q8 & 1)));
                mma16816(o[dm], af, b0, b1);
            }
        }
        // the stage is read: request the item kAwStages ahead into it
        __syncwarp();
        if (lane == 0 && i + kAwStages < i1) {
            issue(iu, i + kAwStages);
            next(iu);
        }
        // the end of this (row, head) in this warp: finish it, or hand in a partial
        if (ch == nch[r] - 1 || i == i1 - 1) {
            const long long u0 = off[r] + (long long)h * nch[r];   // the run's first item
            const int c0 = (int)(((u0 + 1) * W - 1) / I);          // warps holding its first and last items
            const int c1 = (int)(((u0 + nch[r]) * W - 1) / I);
            const int nparts = c1 - c0 + 1, seg = w - c0;
            const size_t ob = (size_t)r * a.out_stride + h * kHeadDim;
            if (nparts == 1) {
                if (t == 0) {
                    const float inv = 1.0f / Lr;
#pragma unroll
                    for (int dm = 0; dm < 4; ++dm)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const size_t oi = ob + 16 * dm + g + 8 * e;
                            const float v = o[dm][2 * e] * inv;
                            a.out[oi] = v;
                            put_operand(a.op, oi, v);
                        }
                }
            } else {
                float *P = a.partial + (((size_t)r * NH + h) * a.max_splits + seg) * (kHeadDim + 2);
                if (t == 0)
#pragma unroll
                    for (int dm = 0; dm < 4; ++dm) {
                        P[2 + 16 * dm + g] = o[dm][0];
                        P[2 + 16 * dm + g + 8] = o[dm][2];
                    }
                if (lane == 0) {
                    P[0] = Mr;
                    P[1] = Lr;
                }
                __threadfence();   // this warp's partial before its arrival
                __syncwarp();
                unsigned *ctr = a.counters + (size_t)r * NH + h;
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(ctr, 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == (unsigned)(nparts - 1)) {   // the last to arrive: merge the parts in slice order
                    __threadfence();
                    const float *P0 = a.partial + ((size_t)r * NH + h) * a.max_splits * (kHeadDim + 2);
                    float M = -FLT_MAX;
                    for (int k = 0; k < nparts; ++k) M = fmaxf(M, __ldcg(P0 + (size_t)k * (kHeadDim + 2)));
#pragma unroll
                    for (int dd = 0; dd < 2; ++dd) {
                        const int d = lane + 32 * dd;
                        float L = 0.0f, O = 0.0f;
                        for (int k = 0; k < nparts; ++k) {
                            const float *Pk = P0 + (size_t)k * (kHeadDim + 2);
                            const float wk = expf(__ldcg(Pk) - M);
                            L = fmaf(__ldcg(Pk + 1), wk, L);
                            O = fmaf(__ldcg(Pk + 2 + d), wk, O);
                        }
                        a.out[ob + d] = O / L;
                        put_operand(a.op, ob + d, O / L);
                    }
                    __syncwarp();
                    if (lane == 0) *ctr = 0u;
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------
// Causal attention of a prompt (prefill): the per-query loop of prefill()
// (main.c:1759-1763 over attn_scores_1q, attn_softmax_1q, attn_out_1q,
// math.cl:388-476) for all query rows of one slot in one launch.
// ------------------------------------------------------------------------------
struct PrefillAttnArgs {
    const float *qkv;    // [rows][qkv_stride]; q of head h at column 64 h
    int qkv_stride;
    KVLayout kv;         // the rows' K and V are in the cache already
    int layer;
    Rows rows;           // pos[r]: the row's position; slot: the same for every row of the pass
    int nrows;
    float *out;
    int out_stride;
    OperandOut op;
};
constexpr int kPaTile = 64;                 // query rows and keys per tile
constexpr int kPaLd = kHeadDim + 4;         // row stride of the shared-memory tiles (floats)
constexpr size_t kPaSmem = 4ull * kPaTile * kPaLd * sizeof(float);   // Q, K, V and P tiles

// CTA (h, t) takes query rows 64 t .. 64 t + 63 of head h and walks the keys
// 0 .. (largest position of its rows) in tiles of 64.  Each K and V tile is
// staged in shared memory once for the 64 queries (the single-query kernel
// reads it again for every row); thread (ty, tx) holds the scores of rows
// 4 ty .. 4 ty + 3 for keys tx + 16 j (j < 4) and the outputs of the same rows
// for dims 4 tx .. 4 tx + 3.  The softmax of each row is merged online across
// the key tiles.  Keys after a row's position are masked (causal); keys past
// the tile's largest position are staged as zeros.  All arithmetic in fp32.
template <typename KT>
__global__ void __launch_bounds__(256) prefill_attn_kernel(PrefillAttnArgs a) {
    pdl_wait();
    pdl_launch();
    constexpr int QT = kPaTile, LD = kPaLd;
    constexpr int VN = 16 / sizeof(KT);   // cache elements per 16-byte load
    constexpr int G = kHeadDim / VN;      // 16-byte loads per key row
    extern __shared__ __align__(16) float pa_sm[];
    float *Qs = pa_sm, *Ks = Qs + QT * LD, *Vs = Ks + QT * LD, *Ps = Vs + QT * LD;
    __shared__ int spos[QT];
    const int h = blockIdx.x, r0 = blockIdx.y * QT, tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    const int nr = min(QT, a.nrows - r0);
    if (tid < QT) spos[tid] = tid < nr ? a.rows.pos[r0 + tid] : -1;
    for (int i = tid; i < QT * (kHeadDim / 4); i += blockDim.x) {   // q / sqrt(64)
        const int row = i / (kHeadDim / 4), c4 = i % (kHeadDim / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < nr) v = reinterpret_cast<const float4 *>(a.qkv + (size_t)(r0 + row) * a.qkv_stride + h * kHeadDim)[c4];
        reinterpret_cast<float4 *>(Qs + row * LD)[c4] = make_float4(v.x * 0.125f, v.y * 0.125f, v.z * 0.125f, v.w * 0.125f);
    }
    __syncthreads();
    int pmax = -1;
    for (int i = 0; i < nr; ++i) pmax = max(pmax, spos[i]);
    if (!G2_BOUNDS(pmax < a.kv.max_seq && a.rows.slot[r0] >= 0 && a.rows.slot[r0] < a.kv.n_slots, 105)) return;
    int mypos[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) mypos[i] = spos[ty * 4 + i];
    const long long base = (long long)a.rows.slot[r0] * a.kv.slot_stride + (long long)a.layer * a.kv.layer_stride +
                           (long long)h * a.kv.max_seq * kHeadDim;
    const KT *K = reinterpret_cast<const KT *>(a.kv.k) + base;
    const KT *V = reinterpret_cast<const KT *>(a.kv.v) + base;
    float m[4], l[4], o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; ++c) o[i][c] = 0.0f;
    }
    for (int j0 = 0; j0 <= pmax; j0 += QT) {
        for (int i = tid; i < QT * G; i += blockDim.x) {   // stage keys j0 .. j0 + 63 as fp32
            const int row = i / G, g = i % G;
            float f[VN];
            if (j0 + row <= pmax) {
                const uint4 kw = *reinterpret_cast<const uint4 *>(K + (size_t)(j0 + row) * kHeadDim + g * VN);
                const uint4 vw = *reinterpret_cast<const uint4 *>(V + (size_t)(j0 + row) * kHeadDim + g * VN);
                unpack_vec(kw, f, KT());
#pragma unroll
                for (int e = 0; e < VN; ++e) Ks[row * LD + g * VN + e] = f[e];
                unpack_vec(vw, f, KT());
#pragma unroll
                for (int e = 0; e < VN; ++e) Vs[row * LD + g * VN + e] = f[e];
            } else {
#pragma unroll
                for (int e = 0; e < VN; ++e) Ks[row * LD + g * VN + e] = Vs[row * LD + g * VN + e] = 0.0f;
            }
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 4
        for (int k = 0; k < kHeadDim; k += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4 *>(Qs + (ty * 4 + i) * LD + k);
#pragma unroll
            for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4 *>(Ks + (tx + 16 * j) * LD + k);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
                    s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
                    s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
                    s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
                }
        }
        // online softmax per row: the row's 64 keys are spread over the 16 lanes of a half-warp
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mt = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j0 + tx + 16 * j > mypos[i]) s[i][j] = -INFINITY;
                mt = fmaxf(mt, s[i][j]);
            }
#pragma unroll
            for (int x = 8; x > 0; x >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, x));
            const float mn = fmaxf(m[i], mt);
            const bool none = mn == -INFINITY;   // no key of this row yet (or a padding row)
            const float sc = none ? 1.0f : expf(m[i] - mn);
            float ls = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float pj = s[i][j] == -INFINITY ? 0.0f : expf(s[i][j] - mn);
                s[i][j] = pj;
                ls += pj;
            }
#pragma unroll
            for (int x = 8; x > 0; x >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, x);
            l[i] = l[i] * sc + ls;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < 4; ++c) o[i][c] *= sc;
#pragma unroll
            for (int j = 0; j < 4; ++j) Ps[(ty * 4 + i) * LD + tx + 16 * j] = s[i][j];
        }
        __syncthreads();
#pragma unroll 4
        for (int j = 0; j < QT; j += 4) {   // O += P V
            float4 pv[4], vv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4 *>(Ps + (ty * 4 + i) * LD + j);
#pragma unroll
            for (int u = 0; u < 4; ++u) vv[u] = *reinterpret_cast<const float4 *>(Vs + (j + u) * LD + tx * 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pp[4] = {pv[i].x, pv[i].y, pv[i].z, pv[i].w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    o[i][0] = fmaf(pp[u], vv[u].x, o[i][0]);
                    o[i][1] = fmaf(pp[u], vv[u].y, o[i][1]);
                    o[i][2] = fmaf(pp[u], vv[u].z, o[i][2]);
                    o[i][3] = fmaf(pp[u], vv[u].w, o[i][3]);
                }
            }
        }
        __syncthreads();   // the next tile overwrites K, V and P
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = ty * 4 + i;
        if (row >= nr) continue;
        const float inv = 1.0f / l[i];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const size_t oi = (size_t)(r0 + row) * a.out_stride + h * kHeadDim + tx * 4 + c;
            const float v = o[i][c] * inv;
            a.out[oi] = v;
            put_operand(a.op, oi, v);
        }
    }
}

template <typename KT>
void launch_prefill_attention(const float *qkv, int qkv_stride, const KVLayout &kv, int layer, Rows rows, int nrows,
                              float *out, int out_stride, cudaStream_t st, OperandOut op) {
    // More than 48 KB of dynamic shared memory: the opt-in is a per-device attribute,
    // so it is made once on every device this process launches on.
    static unsigned long long attr_set = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(__atomic_load_n(&attr_set, __ATOMIC_ACQUIRE) >> dev & 1ull)) {
        cudaFuncSetAttribute(prefill_attn_kernel<KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPaSmem);
        if (dev < 64) __atomic_fetch_or(&attr_set, 1ull << dev, __ATOMIC_RELEASE);
    }
    PrefillAttnArgs a;
    a.qkv = qkv;
    a.qkv_stride = qkv_stride;
    a.kv = kv;
    a.layer = layer;
    a.rows = rows;
    a.nrows = nrows;
    a.out = out;
    a.out_stride = out_stride;
    a.op = op;
    dim3 grid(kv.n_head, (nrows + kPaTile - 1) / kPaTile);
    launch_pdl(prefill_attn_kernel<KT>, grid, dim3(256), kPaSmem, st, a);
}

// ------------------------------------------------------------------------------
// LM head (one row) with the final LayerNorm and greedy argmax fused
// ------------------------------------------------------------------------------
template <typename WT>
struct LmArgs {
    const float *x;
    const WT *wte, *g, *b;
    float *logits;
    int E, V, Vp, forbid_eos;
    float *pval;
    int *pidx;
    unsigned *counter;
    int *result;
    StepState *state;
    int *out_tokens;
};

// (v1, i1) beats (v2, i2): larger value, or equal value and smaller index.
__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
    return v1 > v2 || (v1 == v2 && i1 < i2);
}

constexpr int kLmBlocks = 148 * 4;

template <typename WT>
__global__ void __launch_bounds__(256) lm_head_kernel(LmArgs<WT> a) {
    pdl_wait();
    pdl_launch();
    constexpr int VN = Vec<WT>::n;
    extern __shared__ float xs[];
    __shared__ float sh[32];
    __shared__ float wv[8];
    __shared__ int wi[8];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int forbid = a.forbid_eos || (a.state && a.state->step < a.state->min_new);
    float mean, rstd;
    ln_stats(a.x, a.E, sh, mean, rstd);
    for (int i = tid; i < a.E; i += 256) xs[i] = (a.x[i] - mean) * rstd * tof(a.g[i]) + tof(a.b[i]);
    __syncthreads();
    float best = -FLT_MAX;
    int besti = INT_MAX;
    const int nw = gridDim.x * 8;
    for (int v = blockIdx.x * 8 + warp; v < a.V; v += nw) {
        const WT *row = a.wte + (size_t)v * a.E;
        float s = 0.0f;
        for (int i = lane * VN; i < a.E; i += 32 * VN) s += dot_vec(ld_stream(row + i), xs + i, WT());
        s = warp_sum(s);
        if (lane == 0) a.logits[v] = s;
        if (!(forbid && v == kEos) && better(s, v, best, besti)) {
            best = s;
            besti = v;
        }
    }
    if (blockIdx.x == 0)
        for (int v = a.V + tid; v < a.Vp; v += 256) a.logits[v] = 0.0f;
    if (lane == 0) {
        wv[warp] = best;
        wi[warp] = besti;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 8; ++w)
            if (better(wv[w], wi[w], best, besti)) {
                best = wv[w];
                besti = wi[w];
            }
        a.pval[blockIdx.x] = best;
        a.pidx[blockIdx.x] = besti;
        __threadfence();
        s_last = (atomicAdd(a.counter, 1u) == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last || tid != 0) return;
    __threadfence();
    float bv = -FLT_MAX;
    int bi = INT_MAX;
    for (int c = 0; c < (int)gridDim.x; ++c) {
        const float v = __ldcg(a.pval + c);
        const int i = __ldcg(a.pidx + c);
        if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    if (bi == INT_MAX) bi = 0;   // every logit NaN: never hand an invalid id to the next step
    a.result[0] = bi;
    a.result[1] = __float_as_int(bv);
    if (a.state) {
        a.out_tokens[a.state->step] = bi;
        a.state->token = bi;
        a.state->pos += 1;
        a.state->step += 1;
    }
    *a.counter = 0u;
}

// Argmax per row of logits [rows][Vp] (one CTA per row).
constexpr int kArgThreads = 1024;   // a row of GPT-2's 50,257 logits in two rounds of loads
constexpr int kArgLoads = 8;        // float4 chunks in flight per thread and round
__global__ void __launch_bounds__(kArgThreads) argmax_rows_kernel(const float *logits, int V, int Vp, int forbid_eos,
                                                                  int *tokens, float *values, int *tok_next,
                                                                  int *pos_next, int *out_tokens, int out_stride,
                                                                  const int *step_ptr) {
    pdl_wait();
    pdl_launch();
    __shared__ float wv[kArgThreads / 32];
    __shared__ int wi[kArgThreads / 32];
    const int r = blockIdx.x, tid = threadIdx.x;
    const float *L = logits + (size_t)r * Vp;
    float best = -FLT_MAX;
    int besti = INT_MAX;
    // float4 chunks (rows are Vp = multiple of 4 floats, 16-byte aligned), kArgLoads in flight per thread
    const float4 *L4 = reinterpret_cast<const float4 *>(L);
    const int n4 = (V + 3) / 4;
    for (int c0 = tid; c0 < n4; c0 += kArgLoads * kArgThreads) {
        float4 q[kArgLoads];
#pragma unroll
        for (int u = 0; u < kArgLoads; ++u) {
            const int c = c0 + u * kArgThreads;
            q[u] = c < n4 ? L4[c] : make_float4(-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX);
        }
#pragma unroll
        for (int u = 0; u < kArgLoads; ++u) {
            const int c = c0 + u * kArgThreads;
            const float vals[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int v = 4 * c + k;
                if (c >= n4 || v >= V || (forbid_eos && v == kEos)) continue;
                if (better(vals[k], v, best, besti)) {
                    best = vals[k];
                    besti = v;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (better(ov, oi, best, besti)) {
            best = ov;
            besti = oi;
        }
    }
    if ((tid & 31) == 0) {
        wv[tid >> 5] = best;
        wi[tid >> 5] = besti;
    }
    __syncthreads();
    if (tid < 32) {   // the warps' bests; the first-maximum order makes any reduction order give the same
        best = wv[tid];
        besti = wi[tid];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
            if (better(ov, oi, best, besti)) {
                best = ov;
                besti = oi;
            }
        }
    }
    if (tid == 0) {
        if (besti == INT_MAX) besti = 0;   // every logit NaN
        if (tokens) tokens[r] = besti;
        if (values) values[r] = best;
        if (tok_next) tok_next[r] = besti;
        if (pos_next) pos_next[r] += 1;
        if (out_tokens) out_tokens[(size_t)r * out_stride + *step_ptr] = besti;
    }
}

__global__ void copy_kernel(const float *src, float *dst, int n) {
    pdl_wait();
    pdl_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = src[i];
}
__global__ void step_advance_kernel(int *step) {
    pdl_wait();
    pdl_launch();
    *step += 1;
}

// ------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------
template <typename WT>
void launch_embed(const WT *wte, const WT *wpe, Rows rows, float *h, int E, int V, int n_pos, int nrows,
                  cudaStream_t st) {
    launch_pdl(embed_kernel<WT>, dim3(nrows), dim3(256), 0, st, wte, wpe, rows, h, E, V, n_pos);
}

template <typename WT>
void launch_layernorm(const float *x, float *out, const WT *g, const WT *b, int E, int nrows, cudaStream_t st,
                      OperandOut op) {
    launch_pdl(layernorm_kernel<WT>, dim3(nrows), dim3(256), 0, st, x, out, g, b, E, op);
}

template <typename WT>
GemvPlan gemv_plan(int N, int K, int sms) {
    constexpr int BN = 16 * Vec<WT>::n;
    GemvPlan p;
    p.tiles = (N + BN - 1) / BN;
    const int target = sms * 4;
    const int units = K / 16;  // ksplit must divide K/16
    int best = 1;
    for (int d = 1; d <= units; ++d) {
        if (units % d) continue;
        if (p.tiles * d <= target) best = d;
    }
    p.ksplit = best;
    p.smem_bytes = (size_t)(K / p.ksplit + 16 * BN) * sizeof(float);
    return p;
}

template <typename WT>
void launch_gemv(const float *x, const WT *W, const WT *bias, const float *resid, float *y, int N, int K, int epi,
                 const WT *ln_g, const WT *ln_b, float *partial, unsigned *counters, GemvPlan plan,
                 const KVLayout *kv, int layer, const int *pos_ptr, const int *slot_ptr, cudaStream_t st) {
    constexpr int BN = 16 * Vec<WT>::n;
    GemvArgs<WT> a;
    a.x = x;
    a.W = W;
    a.ln_g = ln_g;
    a.ln_b = ln_b;
    a.partial = partial;
    a.counters = counters;
    a.N = N;
    a.K = K;
    a.e.bias = bias;
    a.e.resid = resid;
    a.e.out = y;
    a.e.N = N;
    a.e.epi = epi;
    if (kv) a.e.kv = *kv;
    a.e.layer = layer;
    a.e.pos = pos_ptr;
    a.e.slot = slot_ptr;
    a.e.E = N / 3;
    dim3 grid(plan.tiles, plan.ksplit);
    launch_pdl(gemv_kernel<WT>, grid, dim3(256), plan.smem_bytes, st, a);
}

template <typename WT>
void launch_gemm_rows(const float *A, const WT *W, const WT *bias, const float *resid, float *C, int M, int N, int K,
                      int epi, const KVLayout *kv, int layer, Rows rows, cudaStream_t st) {
    GemmArgs<WT> a;
    a.A = A;
    a.W = W;
    a.M = M;
    a.N = N;
    a.K = K;
    a.e.bias = bias;
    a.e.resid = resid;
    a.e.out = C;
    a.e.N = N;
    a.e.epi = epi;
    if (kv) a.e.kv = *kv;
    a.e.layer = layer;
    a.e.pos = rows.pos;
    a.e.slot = rows.slot;
    a.e.E = N / 3;
    if (M <= 32) {
        dim3 grid((N + 63) / 64, (M + 31) / 32);
        launch_pdl(gemm_kernel<WT, 32, false>, grid, dim3(256), 0, st, a);
    } else {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        launch_pdl(gemm_kernel<WT, 64, false>, grid, dim3(256), 0, st, a);
    }
}

size_t attn_partial_floats(int nrows, int n_head, int max_seq) {
    const int ms = (max_seq + 63) / 64;   // the streamed kernel's 64-key chunks of fp32 caches
    return (size_t)nrows * n_head * ms * (kHeadDim + 2);
}
size_t attn_counter_count(int nrows, int n_head) { return (size_t)nrows * n_head; }

// One streamed-attention launch: G = SMs x resident CTAs (per device and instantiation,
// with the shared-memory limit raised once per device).
template <typename KT, bool MMA>
static void launch_attn_stream(const AttnArgs<KT> &a, int nrows, const CUtensorMap &mk, const CUtensorMap &mv,
                               cudaStream_t st) {
    static unsigned long long attr_set = 0;
    static int per_sm[64];
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = attn_stream_smem((int)sizeof(KT));
    if (dev >= 64 || !(__atomic_load_n(&attr_set, __ATOMIC_ACQUIRE) >> dev & 1ull)) {
        cudaFuncSetAttribute(attn_stream_kernel<KT, MMA>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_stream_kernel<KT, MMA>, kAsThreads, smem);
        if (dev < 64) {
            per_sm[dev] = n > 0 ? n : 1;
            __atomic_fetch_or(&attr_set, 1ull << dev, __ATOMIC_RELEASE);
        }
    }
    const int G = sms * (dev < 64 ? per_sm[dev] : 1);
    launch_pdl(attn_stream_kernel<KT, MMA>, dim3((unsigned)G), dim3(kAsThreads), smem, st, a, nrows, mk, mv);
}

// One warp-per-run attention launch (fp16 caches): as many CTAs as fit at once, wmax =
// their warps (per device, with the shared-memory limit raised once per device).
static void launch_attn_warp(const AttnArgs<__half> &a, int nrows, const CUtensorMap &mk, const CUtensorMap &mv,
                             cudaStream_t st) {
    static unsigned long long attr_set = 0;
    static int per_sm[64];
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = attn_warp_smem();
    if (dev >= 64 || !(__atomic_load_n(&attr_set, __ATOMIC_ACQUIRE) >> dev & 1ull)) {
        cudaFuncSetAttribute(attn_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_warp_kernel, kAwWarps * 32, smem);
        if (dev < 64) {
            per_sm[dev] = n > 0 ? n : 1;
            __atomic_fetch_or(&attr_set, 1ull << dev, __ATOMIC_RELEASE);
        }
    }
    const int G = sms * (dev < 64 ? per_sm[dev] : 1);
    launch_pdl(attn_warp_kernel, dim3((unsigned)G), dim3(kAwWarps * 32), smem, st, a, nrows, G * kAwWarps, mk, mv);
}

// G2_ATTN_STREAM=1: fp16 decode attention by the streamed kernel instead of the warp-per-run one.
static bool attn_stream_forced() {
    static const int v = [] {
        const char *e = getenv("G2_ATTN_STREAM");
        return e && atoi(e) > 0 ? 1 : 0;
    }();
    return v != 0;
}

template <typename KT>
void launch_attention(const float *qkv, int qkv_stride, const KVLayout &kv, int layer, Rows rows, int nrows,
                      float *out, int out_stride, float *partial, unsigned *counters, int max_pos_hint,
                      cudaStream_t st, OperandOut op, QkvPartials qp) {
    AttnArgs<KT> a;
    a.op = op;
    a.qpart = qp.part;
    a.qsi = qp.si;
    a.qtotal = (long long)nrows * qkv_stride;
    a.qbias = reinterpret_cast<const KT *>(qp.bias);
    a.qkv = qkv;
    a.qkv_stride = qkv_stride;
    a.kv = kv;
    a.layer = layer;
    a.rows = rows;
    a.out = out;
    a.out_stride = out_stride;
    a.partial = partial;
    a.counters = counters;
    a.max_splits = (kv.max_seq + kAttnChunk - 1) / kAttnChunk;
    a.err = qp.err;
    if (qp.part && qp.err && nrows <= kAsMaxRows) {
        // decode rows with c_attn's partials: the streamed kernel, as many CTAs as fit at once
        // (fp16 caches with their tensor maps: the tensor-core instantiation)
        a.max_splits = (kv.max_seq + as_chunk<KT>() - 1) / as_chunk<KT>();   // partial slots per (row, head)
        if constexpr (sizeof(KT) == 2) {
            if (qp.kmap && qp.vmap && !attn_stream_forced()) {
                a.max_splits = (kv.max_seq + kAwChunk - 1) / kAwChunk;
                launch_attn_warp(a, nrows, *static_cast<const CUtensorMap *>(qp.kmap),
                                 *static_cast<const CUtensorMap *>(qp.vmap), st);
                return;
            }
        }
        if (sizeof(KT) == 2 && qp.kmap && qp.vmap)
            launch_attn_stream<KT, sizeof(KT) == 2>(a, nrows, *static_cast<const CUtensorMap *>(qp.kmap),
                                                     *static_cast<const CUtensorMap *>(qp.vmap), st);
        else
            launch_attn_stream<KT, false>(a, nrows, CUtensorMap{}, CUtensorMap{}, st);
        return;
    }
    const int splits = max_pos_hint < 0 ? a.max_splits : (max_pos_hint + kAttnChunk) / kAttnChunk;
    dim3 grid(kv.n_head, splits, nrows);
    launch_pdl(attn_kernel<KT>, grid, dim3(128), 0, st, a);
}

int lm_head_blocks() { return kLmBlocks; }

// Four ints written on the device (row descriptors of single-query calls), so
// that no host-memory copy is needed and the call can be captured in a graph.
__global__ void set_ints_kernel(int *p, int a, int b, int c, int d) {
    p[0] = a;
    p[1] = b;
    p[2] = c;
    p[3] = d;
}
void launch_set_ints(int *p, int a, int b, int c, int d, cudaStream_t st) { set_ints_kernel<<<1, 1, 0, st>>>(p, a, b, c, d); }

bool pdl_enabled() {
    static const bool on = [] {
        const char *v = getenv("G2_NO_PDL");
        return !(v && v[0] == '1');
    }();
    return on;
}

template <typename WT>
void launch_lm_head(const float *x, const WT *wte, const WT *lnf_g, const WT *lnf_b, float *logits, int E, int V,
                    int Vp, int forbid_eos, float *partial, unsigned *counter, int *result, StepState *state,
                    int *out_tokens, cudaStream_t st) {
    LmArgs<WT> a;
    a.x = x;
    a.wte = wte;
    a.g = lnf_g;
    a.b = lnf_b;
    a.logits = logits;
    a.E = E;
    a.V = V;
    a.Vp = Vp;
    a.forbid_eos = forbid_eos;
    a.pval = partial;
    a.pidx = reinterpret_cast<int *>(partial + kLmBlocks);
    a.counter = counter;
    a.result = result;
    a.state = state;
    a.out_tokens = out_tokens;
    launch_pdl(lm_head_kernel<WT>, dim3(kLmBlocks), dim3(256), (size_t)E * sizeof(float), st, a);
}

template <typename WT>
void launch_lm_head_rows(const float *x, const WT *wte, float *logits, int E, int V, int Vp, int nrows,
                         cudaStream_t st) {
    GemmArgs<WT> a;
    a.A = x;
    a.W = wte;
    a.M = nrows;
    a.N = V;
    a.K = E;
    a.e.bias = nullptr;
    a.e.resid = nullptr;
    a.e.out = logits;
    a.e.N = Vp;
    a.e.epi = EPI_NONE;
    a.e.E = 0;
    if (nrows <= 32) {
        dim3 grid((V + 63) / 64, (nrows + 31) / 32);
        launch_pdl(gemm_kernel<WT, 32, true>, grid, dim3(256), 0, st, a);
    } else {
        dim3 grid((V + 63) / 64, (nrows + 63) / 64);
        launch_pdl(gemm_kernel<WT, 64, true>, grid, dim3(256), 0, st, a);
    }
}

void launch_argmax_rows(const float *logits, int V, int Vp, int nrows, int forbid_eos, int *tokens, float *values,
                        int *tok_next, int *pos_next, int *out_tokens, int out_stride, const int *step_ptr,
                        cudaStream_t st) {
    launch_pdl(argmax_rows_kernel, dim3(nrows), dim3(kArgThreads), 0, st, logits, V, Vp, forbid_eos, tokens, values, tok_next, pos_next,
                                              out_tokens, out_stride, step_ptr);
}

void launch_copy_row(const float *src, float *dst, int n, cudaStream_t st) {
    launch_pdl(copy_kernel, dim3((n + 255) / 256), dim3(256), 0, st, src, dst, n);
}
__global__ void add_ints_kernel(int *p, int n, int add) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] += add;
}
void launch_add_ints(int *p, int n, int add, cudaStream_t st) {
    add_ints_kernel<<<(n + 255) / 256, 256, 0, st>>>(p, n, add);
}
void launch_step_advance(int *step_ptr, cudaStream_t st) { launch_pdl(step_advance_kernel, dim3(1), dim3(1), 0, st, step_ptr); }

// 32 x 32 tiles through shared memory (one padding column against bank
// conflicts): both the reads of src rows and the writes of dst rows are
// coalesced.  Block (32, 8); each thread moves four elements.
template <typename WT>
__global__ void transpose_kernel(const float *__restrict__ src, WT *__restrict__ dst, int rows, int cols) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = src[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + threadIdx.x;   // dst row c, column r
        if (r < rows && c < cols) dst[(size_t)c * rows + r] = fromf<WT>(tile[threadIdx.x][i]);
    }
}

template <typename WT>
void launch_transpose(const float *src, WT *dst, int rows, int cols, cudaStream_t st) {
    dim3 grid((cols + 31) / 32, (rows + 31) / 32);
    transpose_kernel<WT><<<grid, dim3(32, 8), 0, st>>>(src, dst, rows, cols);
}

// explicit instantiations
#define G2_INST(WT)                                                                                                   \
    template void launch_embed<WT>(const WT *, const WT *, Rows, float *, int, int, int, int, cudaStream_t);         \
    template void launch_layernorm<WT>(const float *, float *, const WT *, const WT *, int, int, cudaStream_t,       \
                                       OperandOut);                                                                   \
    template GemvPlan gemv_plan<WT>(int, int, int);                                                                    \
    template void launch_gemv<WT>(const float *, const WT *, const WT *, const float *, float *, int, int, int,      \
                                  const WT *, const WT *, float *, unsigned *, GemvPlan, const KVLayout *, int,     \
                                  const int *, const int *, cudaStream_t);                                           \
    template void launch_gemm_rows<WT>(const float *, const WT *, const WT *, const float *, float *, int, int, int, \
                                       int, const KVLayout *, int, Rows, cudaStream_t);                              \
    template void launch_prefill_attention<WT>(const float *, int, const KVLayout &, int, Rows, int, float *, int,   \
                                               cudaStream_t, OperandOut);                                              \
    template void launch_attention<WT>(const float *, int, const KVLayout &, int, Rows, int, float *, int, float *,  \
                                       unsigned *, int, cudaStream_t, OperandOut, QkvPartials);                       \
    template void launch_lm_head<WT>(const float *, const WT *, const WT *, const WT *, float *, int, int, int, int, \
                                     float *, unsigned *, int *, StepState *, int *, cudaStream_t);                  \
    template void launch_lm_head_rows<WT>(const float *, const WT *, float *, int, int, int, int, cudaStream_t);  \
    template void launch_transpose<WT>(const float *, WT *, int, int, cudaStream_t);
G2_INST(float)
G2_INST(__half)

#ifdef G2_CHECK
int check_flag_kernels() {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g2_check_flag, sizeof(int));
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g2_check_flag, &z, sizeof(int));
    }
    return v;
}
#else
int check_flag_kernels() { return 0; }
#endif

}  // namespace g2
