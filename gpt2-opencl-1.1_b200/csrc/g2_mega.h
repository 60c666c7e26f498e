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
    int cw_qkv, cw_fc;   // strip widths (columns per unit) of c_attn and c_fc
    int nq;              // column slices of attn.c_proj per head (B units = NH * nq)
    int lm_rows;         // wte rows per LM unit
    int n_steps;         // greedy decode steps in this launch
    long long layer_stride;                 // KV elements per layer of one slot
    const float *packed;                    // unit-packed projection weights
    const long long *layer_off;             // [L][3] float offsets of the A, B and D units
    const LayerPtrs *layers;                // [L]
    const float *wte, *wpe, *lnf_g, *lnf_b, *lm;
    float *kc, *vc;                         // this slot's KV cache bases
    unsigned long long *t_qkv, *t_best;     // tagged activations: q, k, v; argmax partials
    unsigned long long *t_att;              // [NH][nq][66] tagged attention partials (o[64], m, l)
    int split_t;                            // past this many positions a head's keys are split over its nq units
    unsigned long long *acc;                // mega_acc_words(n_steps, L, E) accumulator words, zero at launch
    float *logits;                          // [V_pad] of this slot
    int *out_tokens;                        // this slot's token row
    int *result;                            // [0] last token, [1] its logit bits
    StepState *state;                       // token / pos / step / min_new in and out
    int *err;                               // 0, or the code of the first expired wait (or kErrClamp)
    unsigned long long timeout_ns;          // limit of every device-side wait
    unsigned epoch0;
    int max_inflight;   // bulk copies a CTA keeps outstanding (1..8); the ring holds 8 slots regardless
    // Optional phase trace (nullptr = off): per CTA kTraceSlots words, see g2_mega.cu.
    unsigned long long *trace;
};

// MegaParams::err code of a clamped accumulator contribution (wait sites use 1..6).
constexpr int kErrClamp = 16;
constexpr unsigned long long kMegaTimeoutNs = 2000000000ull;   // default wait limit: 2 s

constexpr int kTraceSlots = 160;
// Trace words per CTA: [0..8) ns spent waiting for inputs: [1] B (q, k, v), [2] x after
// the MLP, [4] x after attention, [5] LM head, [6] argmax; [8..16) ns of work after the
// inputs arrived: [8] A, [9] B, [11] D, [13] LM head, [14] argmax; [17] kernel ns; [22]
// timeline stamps taken; [32..160) CTA 0 only: the timeline of one step (step 3, or the last
// step of a shorter launch): phase start/end stamps relative to kernel start.

size_t mega_smem_bytes(int E);
int mega_threads();
// The kernel; `traced` selects the instantiation that records the phase trace.
const void *mega_kernel_ptr(bool traced);
int mega_slot_bytes();
int mega_max_keys();
// Steps per launch (the accumulators of one launch are sized for this many).
constexpr int kMegaMaxSteps = 256;
// Layers the kernel's per-CTA schedule table holds.
constexpr int kMegaMaxLayers = 64;
// Copies of the MLP accumulator (D units spread their additions over them).
constexpr int kAccCopies = 4;
// Accumulator words of one launch of n steps: per step and layer, one
// attention vector and kAccCopies MLP vectors of E words.
inline size_t mega_acc_words(int n, int L, int E) { return (size_t)n * L * (1 + kAccCopies) * E; }
// Packed floats of a layer's units:
//  A: 3E / cw_qkv strips of (E + 2) rows x cw_qkv (weights with ln_1's gamma
//     folded in, then the bias row with beta folded in, then the column sums);
//  B: NH * nq blocks of 64 rows x E / nq (rows 64h.. of attn.c_proj, one
//     column slice);
//  D: F / cw_fc units, each a c_fc strip (as in A, with ln_2) followed by
//     the matching cw_fc rows of mlp.c_proj (E floats each).
inline long long mega_packed_a(int E) { return (long long)(E + 2) * 3 * E; }
inline long long mega_packed_b(int E) { return (long long)E * E; }
inline long long mega_packed_d(int E, int F) { return (long long)(E + 2) * F + (long long)F * E; }
// Strip width of a projection with N outputs on G CTAs: the narrowest of 4,
// 8, 12, 16, 20, 24 and 32 columns (cw / 4 float4 groups dividing the 480
// consumer threads) that gives every CTA at most one unit, else the widest
// that divides N.  0 if none divides N.
inline int mega_cw(int N, int G) {
    static const int widths[7] = {4, 8, 12, 16, 20, 24, 32};
    for (int cw : widths)
        if (N % cw == 0 && N / cw <= G) return cw;
    for (int k = 6; k >= 0; --k)
        if (N % widths[k] == 0) return widths[k];
    return 0;
}
// wte rows per LM-head unit: one per consumer warp (15), over at most a few
// ring chunks.
inline int mega_lm_rows(int E) {
    (void)E;
    return 15;
}
// Column slices of attn.c_proj per head (B units = NH * nq): a slice is a
// whole number of float4 groups, at most one per consumer thread.
inline bool mega_nq_ok(int E, int nq) { return nq >= 1 && E % nq == 0 && (E / nq) % 4 == 0 && E / nq / 4 <= 480; }
// Default: 8 (measured best for GPT-2 small: one ring chunk of attn.c_proj
// per B unit), else the largest of 4, 3, 2, 1 that is valid, keeping NH * nq
// within the G CTAs (G2_MEGA_NQ overrides).
inline int mega_nq(int E, int NH, int G) {
    if (mega_nq_ok(E, 8) && NH * 8 <= G) return 8;
    for (int nq = 4; nq >= 1; --nq)
        if (mega_nq_ok(E, nq)) return nq;
    return 0;
}
// Epochs one launch of n_steps uses.
inline unsigned mega_epochs(int L, int n_steps) { return (unsigned)n_steps * (unsigned)((L + 1) * 8) + 8u; }

}  // namespace g2
