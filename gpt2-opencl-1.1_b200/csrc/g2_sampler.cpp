// g2_sampler.cpp -- host token sampler with the semantics of the reference's
// sample_next_token (main.c:1872-1939) and kth_largest (main.c:1839-1868).
//
// The logits are copied, so the caller's buffer is left unchanged.  Steps:
// EOS masked to -1e30 when forbidden; repetition penalty over the unique
// context ids (divide positive logits, multiply the rest); then greedy
// (first maximum) or temperature scaling, a top-k threshold (the k-th largest
// value; everything strictly below it is dropped), softmax accumulated in
// double, and an inverse-CDF draw with the C library's rand().
#include <cmath>
#include <cstdlib>
#include <vector>

#include "gpt2b200.h"

namespace {

// k-th largest value of a[0..n) (k <= G2_MAX_TOPK) with a min-heap of the k
// largest seen so far.
float kth_largest(const float *a, int n, int k) {
    float heap[G2_MAX_TOPK];
    int size = 0;
    auto sift_down = [&](int j) {
        for (;;) {
            const int l = 2 * j + 1, r = l + 1;
            int m = j;
            if (l < size && heap[l] < heap[m]) m = l;
            if (r < size && heap[r] < heap[m]) m = r;
            if (m == j) return;
            std::swap(heap[j], heap[m]);
            j = m;
        }
    };
    for (int i = 0; i < n; ++i) {
        const float v = a[i];
        if (size < k) {
            int j = size++;
            heap[j] = v;
            while (j > 0 && heap[(j - 1) / 2] > heap[j]) {
                std::swap(heap[(j - 1) / 2], heap[j]);
                j = (j - 1) / 2;
            }
        } else if (v > heap[0]) {
            heap[0] = v;
            sift_down(0);
        }
    }
    return heap[0];
}

}  // namespace

extern "C" int g2_sample(const float *logits_in, int vocab_size, const int *ctx, int n_ctx, int forbid_eos,
                         float temperature, int top_k, float rep_penalty, int *out_token) {
    if (!logits_in || !out_token || vocab_size <= 0 || n_ctx < 0 || (n_ctx > 0 && !ctx)) return G2_ERR_ARG;
    const int V = vocab_size;
    std::vector<float> logits(logits_in, logits_in + V);
    if (forbid_eos && G2_EOS < V) logits[G2_EOS] = -1e30f;
    if (rep_penalty > 1.0f) {
        for (int i = 0; i < n_ctx; ++i) {
            const int t = ctx[i];
            if (t < 0 || t >= V) continue;
            bool seen = false;
            for (int j = 0; j < i && !seen; ++j) seen = ctx[j] == t;
            if (seen) continue;
            if (logits[t] > 0.0f) logits[t] /= rep_penalty;
            else logits[t] *= rep_penalty;
        }
    }
    if (temperature <= 0.0f) {
        int best = 0;
        for (int i = 1; i < V; ++i)
            if (logits[i] > logits[best]) best = i;
        *out_token = best;
        return G2_OK;
    }
    const float inv_t = 1.0f / temperature;
    for (float &l : logits) l *= inv_t;
    int k = top_k;
    if (k <= 0 || k > V) k = V;
    if (k > G2_MAX_TOPK) k = G2_MAX_TOPK;
    if (k < V) {
        const float thresh = kth_largest(logits.data(), V, k);
        for (float &l : logits)
            if (l < thresh) l = -1e30f;
    }
    float mx = -1e30f;
    for (float l : logits) mx = l > mx ? l : mx;
    double sum = 0.0;
    for (float &l : logits) {
        if (l <= -1e29f) {
            l = 0.0f;
            continue;
        }
        l = expf(l - mx);
        sum += l;
    }
    const double r = ((double)rand() / ((double)RAND_MAX + 1.0)) * sum;
    double acc = 0.0;
    int chosen = V - 1;
    for (int i = 0; i < V; ++i) {
        acc += logits[i];
        if (acc >= r) {
            chosen = i;
            break;
        }
    }
    *out_token = chosen;
    return G2_OK;
}
