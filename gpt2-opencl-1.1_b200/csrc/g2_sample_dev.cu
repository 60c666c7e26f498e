// g2_sample_dev.cu -- the reference's sample_next_token (main.c:1872-1939) on
// the device, so that a sampled token costs a 4-byte read instead of the
// 201 KB logits read of main.c:1878.
//
// One CTA of 1024 threads over the V logits of a slot:
//   1. copy to a work buffer; EOS masked to -1e30 when forbidden (main.c:1882);
//   2. repetition penalty over the unique context ids (main.c:1885-1895):
//      one thread per context position, applied at an id's first occurrence
//      only, so no two threads touch the same logit;
//   3. temperature <= 0: first maximum (main.c:1898-1904);
//   4. else scale by 1 / T, then the k-th largest value (main.c:1839-1868) by
//      an exact radix select over order-preserving integer keys (4 passes of
//      8 bits with shared-memory histograms) and everything strictly below
//      it masked (main.c:1913-1918);
//   5. the maximum, exp(l - max) of the survivors (masked entries count 0)
//      and their sum in double (main.c:1920-1931);
//   6. the first index whose running sum reaches u * sum (main.c:1933-1938),
//      u supplied by the caller (the reference draws rand() / (RAND_MAX + 1)).
//      Each thread owns a contiguous block; block sums are scanned in order.
#include <cfloat>

#include "g2_device.cuh"
#include "gpt2b200.h"

namespace g2 {

namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ unsigned float_key(float f) {
    const unsigned b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);   // ascending floats -> ascending keys
}
__device__ __forceinline__ float key_float(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SampleArgs {
    const float *logits;
    float *work;          // [V]
    int V;
    const int *ctx;       // [n_ctx] (device)
    int n_ctx;
    int forbid_eos;
    float temperature;
    int top_k;
    float rep_penalty;
    double u;             // uniform draw in [0, 1)
    int *out;             // [0] token
};

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
    __shared__ unsigned hist[256];
    __shared__ double dsum[kThreads];
    __shared__ float fred[32];
    __shared__ int ired[32];
    __shared__ unsigned sel[2];   // prefix, remaining rank
    __shared__ double total_s;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int V = a.V;
    float *w = a.work;
    for (int i = t; i < V; i += kThreads) w[i] = a.logits[i];
    __syncthreads();
    if (t == 0 && a.forbid_eos && G2_EOS < V) w[G2_EOS] = -1e30f;
    __syncthreads();
    if (a.rep_penalty > 1.0f) {
        for (int i = t; i < a.n_ctx; i += kThreads) {
            const int tk = a.ctx[i];
            if (tk < 0 || tk >= V) continue;
            bool dup = false;
            for (int j = 0; j < i && !dup; ++j) dup = a.ctx[j] == tk;
            if (dup) continue;
            const float l = w[tk];
            w[tk] = l > 0.0f ? l / a.rep_penalty : l * a.rep_penalty;
        }
    }
    __syncthreads();

    if (a.temperature <= 0.0f) {   // greedy: first maximum
        float bv = -FLT_MAX;
        int bi = INT_MAX;
        for (int i = t; i < V; i += kThreads) {   // increasing i: strict > keeps the first
            const float l = w[i];
            if (bi == INT_MAX || l > bv) {
                bv = l;
                bi = i;
            }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            fred[warp] = bv;
            ired[warp] = bi;
        }
        __syncthreads();
        if (t == 0) {
            bv = fred[0];
            bi = ired[0];
            for (int q = 1; q < kThreads / 32; ++q)
                if (ired[q] != INT_MAX && (bi == INT_MAX || fred[q] > bv || (fred[q] == bv && ired[q] < bi))) {
                    bv = fred[q];
                    bi = ired[q];
                }
            a.out[0] = bi == INT_MAX ? 0 : bi;
        }
        return;
    }

    const float inv_t = 1.0f / a.temperature;
    for (int i = t; i < V; i += kThreads) w[i] *= inv_t;
    int k = a.top_k;
    if (k <= 0 || k > V) k = V;
    if (k > G2_MAX_TOPK) k = G2_MAX_TOPK;
    __syncthreads();
    if (k < V) {
        // k-th largest: the key with (#keys > key) < k <= (#keys >= key), digit by digit from the top
        if (t == 0) {
            sel[0] = 0;
            sel[1] = (unsigned)k;
        }
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            for (int b = t; b < 256; b += kThreads) hist[b] = 0;
            __syncthreads();
            const unsigned prefix = sel[0];
            const unsigned hmask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
            for (int i = t; i < V; i += kThreads) {
                const unsigned key = float_key(w[i]);
                if ((key & hmask) == (prefix & hmask)) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (t == 0) {
                unsigned need = sel[1];
                int b = 255;
                for (; b > 0; --b) {
                    if (hist[b] >= need) break;
                    need -= hist[b];
                }
                sel[0] = prefix | ((unsigned)b << shift);
                sel[1] = need;
            }
            __syncthreads();
        }
        const float thresh = key_float(sel[0]);
        for (int i = t; i < V; i += kThreads)
            if (w[i] < thresh) w[i] = -1e30f;
        __syncthreads();
    }
    // maximum
    float mx = -1e30f;
    for (int i = t; i < V; i += kThreads) mx = fmaxf(mx, w[i]);
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) fred[warp] = mx;
    __syncthreads();
    mx = fred[0];
    for (int q = 1; q < kThreads / 32; ++q) mx = fmaxf(mx, fred[q]);
    // exps and the in-order running sum: thread t owns [lo, hi)
    const int per = (V + kThreads - 1) / kThreads, lo = min(V, t * per), hi = min(V, lo + per);
    double s = 0.0;
    for (int i = lo; i < hi; ++i) {
        const float l = w[i];
        float e = 0.0f;
        if (l > -1e29f) e = expf(l - mx);
        w[i] = e;
        s += e;
    }
    dsum[t] = s;
    __syncthreads();
    // exclusive scan of the block sums, in order (thread 0; 1024 doubles)
    if (t == 0) {
        double acc = 0.0;
        for (int q = 0; q < kThreads; ++q) {
            const double v = dsum[q];
            dsum[q] = acc;
            acc += v;
        }
        ired[0] = INT_MAX;
        total_s = acc;
    }
    __syncthreads();
    const double total = total_s;
    const double r = a.u * total;
    double acc = dsum[t];
    int found = INT_MAX;
    for (int i = lo; i < hi; ++i) {
        acc += w[i];
        if (acc >= r) {
            found = i;
            break;
        }
    }
    for (int o = 16; o; o >>= 1) found = min(found, __shfl_xor_sync(0xffffffffu, found, o));
    __syncthreads();
    if (lane == 0) atomicMin(&ired[0], found);
    __syncthreads();
    if (t == 0) a.out[0] = ired[0] == INT_MAX ? V - 1 : ired[0];
}

// The k (<= G2_MAX_TOPK) largest of logits[0..V), in the order of the reference's
// first-maximum scan (main.c:1898-1904): the larger value first, equal values by
// the smaller index.  One CTA:
//   1. the k-th largest key by the radix select of sample_kernel (kth_largest,
//      main.c:1839-1868): T, and `need`, how many keys equal to T belong to the
//      top k (every key above T does: there are k - need of them);
//   2. each thread owns a contiguous block of indices; block counts of keys above
//      T and equal to T are scanned in index order, so each selected logit gets
//      its output slot and the keys equal to T are taken in increasing index;
//   3. a bitonic sort of the k (key, index) pairs in shared memory.
// -0.0 is keyed as +0.0 (they compare equal as floats); logits are finite.
constexpr int kTopkThreads = 1024;
__device__ __forceinline__ unsigned logit_key(float f) { return float_key(f == 0.0f ? 0.0f : f); }

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const float *logits, int V, int k, float *vals, int *idx) {
    __shared__ unsigned hist[256];
    __shared__ unsigned sel[2];                       // prefix, remaining rank
    __shared__ int wtot[2][32];
    __shared__ unsigned long long cand[G2_MAX_TOPK];  // (key << 32) | (0xffffffff - index)
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    if (t == 0) {
        sel[0] = 0;
        sel[1] = (unsigned)k;
    }
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int b = t; b < 256; b += kTopkThreads) hist[b] = 0;
        __syncthreads();
        const unsigned prefix = sel[0];
        const unsigned hmask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
        for (int i = t; i < V; i += kTopkThreads) {
            const unsigned key = logit_key(logits[i]);
            if ((key & hmask) == (prefix & hmask)) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (t == 0) {
            unsigned need = sel[1];
            int b = 255;
            for (; b > 0; --b) {
                if (hist[b] >= need) break;
                need -= hist[b];
            }
            sel[0] = prefix | ((unsigned)b << shift);
            sel[1] = need;
        }
        __syncthreads();
    }
    const unsigned T = sel[0];
    const int need = (int)sel[1];
    const int per = (V + kTopkThreads - 1) / kTopkThreads, lo = min(V, t * per), hi = min(V, lo + per);
    int ngt = 0, neq = 0;
    for (int i = lo; i < hi; ++i) {
        const unsigned key = logit_key(logits[i]);
        ngt += key > T;
        neq += key == T;
    }
    // exclusive prefix sums of both counts over the threads, in index order
    int sg = ngt, se = neq;
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, sg, o), b = __shfl_up_sync(0xffffffffu, se, o);
        if (lane >= o) {
            sg += a;
            se += b;
        }
    }
    if (lane == 31) {
        wtot[0][warp] = sg;
        wtot[1][warp] = se;
    }
    __syncthreads();
    if (warp == 0) {
        int a = wtot[0][lane], b = wtot[1][lane];
        for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
            if (lane >= o) {
                a += x;
                b += y;
            }
        }
        wtot[0][lane] = a - wtot[0][lane];   // exclusive, per warp
        wtot[1][lane] = b - wtot[1][lane];
    }
    __syncthreads();
    int pg = wtot[0][warp] + sg - ngt, pe = wtot[1][warp] + se - neq;   // this thread's first slots
    const int base_eq = k - need;
    for (int i = lo; i < hi && (pg < base_eq || pe < need); ++i) {
        const unsigned key = logit_key(logits[i]);
        const unsigned long long c = ((unsigned long long)key << 32) | (0xffffffffu - (unsigned)i);
        if (key > T) {
            cand[pg++] = c;
        } else if (key == T) {
            if (pe < need) cand[base_eq + pe] = c;
            ++pe;
        }
    }
    int P = 1;
    while (P < k) P <<= 1;
    for (int i = k + t; i < P; i += kTopkThreads) cand[i] = 0ull;   // below every real entry
    __syncthreads();
    // bitonic sort, decreasing
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = t; i < P; i += kTopkThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const unsigned long long x = cand[i], y = cand[j];
                    if ((i & size) == 0 ? x < y : x > y) {
                        cand[i] = y;
                        cand[j] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int r = t; r < k; r += kTopkThreads) {
        const int id = (int)(0xffffffffu - (unsigned)(cand[r] & 0xffffffffu));
        idx[r] = id;
        vals[r] = logits[id];
    }
}

}  // namespace

void launch_topk(const float *logits, int V, int k, float *vals, int *idx, cudaStream_t st) {
    topk_kernel<<<1, kTopkThreads, 0, st>>>(logits, V, k, vals, idx);
}

void launch_sample(const float *logits, float *work, int V, const int *ctx, int n_ctx, int forbid_eos,
                   float temperature, int top_k, float rep_penalty, double u, int *out, cudaStream_t st) {
    SampleArgs a{logits, work, V, ctx, n_ctx, forbid_eos, temperature, top_k, rep_penalty, u, out};
    sample_kernel<<<1, kThreads, 0, st>>>(a);
}

}  // namespace g2
