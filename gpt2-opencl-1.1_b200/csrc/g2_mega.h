// g2_mega.h -- parameters of the persistent B = 1 decode kernel (g2_mega.cu).
#pragma once
#include <cstddef>

#include "g2_internal.h"

namespace g2 {

// Per-layer vectors (biases and LayerNorm parameters), device pointers.
struct LayerPtrs {
    const float *ln1_g, *ln1_b, *qkv_b, *proj_b, *ln2_g, *ln2_b, *fc_b, *fc2_b;
};

struct MegaParams {
    int L, E, F, NH, V, max_seq;
    int cw[4];           // strip widths (columns per unit) of qkv, proj, fc and fc2
    int lm_rows;         // wte rows per LM unit
    int n_steps;         // greedy decode steps in this launch
    long long layer_stride;                 // KV elements per layer of one slot
    const float *packed;                    // strip-packed projection weights
    const long long *layer_off;             // [L][4] float offsets of qkv, proj, fc, fc2 strips
    const LayerPtrs *layers;                // [L]
    const float *wte, *wpe, *lnf_g, *lnf_b, *lm;
    float *kc, *vc;                         // this slot's KV cache bases
    unsigned long long *t_qkv, *t_part, *t_ha, *t_hb, *t_f, *t_best;   // tagged activations
    float *logits;                          // [V_pad] of this slot
    int *out_tokens;                        // this slot's token row
    int *result;                            // [0] last token, [1] its logit bits
    StepState *state;                       // token / pos / step / min_new in and out
    int *err;                               // 0, or the code of the first expired wait
    unsigned epoch0;
    int max_inflight;   // bulk copies a CTA keeps outstanding (1..8); the ring holds 8 slots regardless
    // Optional phase trace (nullptr = off): per CTA kTraceSlots words, see g2_mega.cu.
    unsigned long long *trace;
};

constexpr int kTraceSlots = 64;
// Trace words per CTA: [0..8) ns spent polling inputs per phase (A, B, C, D, E, LM, argmax),
// [8..16) ns of work after the inputs arrived per phase, [16] ns waiting for ring chunks,
// [17] kernel ns, [18] units, [19] chunks, [22] / [23] / [25] SM cycles of strip units in
// LayerNorm sums / row products (chunk waits included) / reduction, [27] strip units,
// [32..64) CTA 0 only: step-0 timeline of layer 0 (phase start/end stamps relative to kernel start).

size_t mega_smem_bytes(int E, int F);
int mega_threads();
const void *mega_kernel_ptr();
int mega_slot_bytes();
// Packed floats of one projection: N / CW units of (K + 2) rows x CW.  Rows
// 0..K-1 are the weights, row K the bias, row K + 1 the column sums of the
// weights (used when a LayerNorm is folded in, zero otherwise).
inline long long mega_packed_floats(int K, int N) { return (long long)(K + 2) * N; }
// Strip width of a projection with N outputs on G CTAs: the narrowest of 4, 8,
// 16 and 32 columns that gives every CTA at most one unit, else 32 (every CTA
// then streams several units).  0 if N is not a multiple of 4.
inline int mega_cw(int N, int G) {
    for (int cw = 4; cw <= 32; cw *= 2)
        if (N % cw == 0 && N / cw <= G) return cw;
    return N % 32 == 0 ? 32 : N % 16 == 0 ? 16 : N % 8 == 0 ? 8 : N % 4 == 0 ? 4 : 0;
}
inline int mega_lm_rows(int E) {
    const int rpc = 24576 / (E * 4);
    return rpc < 1 ? 1 : 2 * rpc;
}
// Epochs one launch of n_steps uses.
inline unsigned mega_epochs(int L, int n_steps) { return (unsigned)n_steps * (unsigned)((L + 1) * 8) + 8u; }

}  // namespace g2
