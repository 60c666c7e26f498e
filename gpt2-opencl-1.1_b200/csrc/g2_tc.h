// g2_tc.h -- tensor-core GEMM (tcgen05) for many-row passes: prefill and
// batched decode.  See g2_tc.cu.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "g2_internal.h"

namespace g2 {

// Operand precision of a tensor-core GEMM.
//  TC_TF32X3: fp32 operands split as x = hi + lo (hi = x rounded to tf32, lo =
//             the rest rounded to tf32); three tf32 products hi*hi + hi*lo +
//             lo*hi with fp32 accumulation, which keeps fp32-level accuracy.
//             The activations arrive split (their producer writes hi and
//             lo); the weights are two tf32 copies made at load, or the fp32
//             weights split tile by tile in shared memory (TcWeights::wsplit).
//  TC_F16:    fp16 operands (fp16 weights of the fp16 engine; activations
//             rounded to fp16), fp32 accumulation.
enum TcKind { TC_F16 = 0, TC_TF32X3 = 1 };

constexpr int kTcTileF = 128;   // output features per CTA (the MMA's M)

// Encode a 2-D row-major tensor [outer][inner] of `dt` elements with a
// 128-byte-swizzled box of box_inner x box_outer elements (box_inner * elem
// must be 128 bytes); atom32 selects the swizzle of 32-byte granules that
// MN-major tf32 operands need.  Returns 0 or a G2_ERR_* code.
int tc_encode(CUtensorMap *map, CUtensorMapDataType dt, const void *base, unsigned long long inner,
              unsigned long long outer, unsigned box_inner, unsigned box_outer, bool atom32);

// Weight operand of one projection W [K][N]: tensor maps of its tf32 hi and lo
// copies (TC_TF32X3), or with lo == nullptr of the fp32 weights themselves,
// split in the kernel (wsplit), or of the fp16 weights (TC_F16, lo unused).
// img_hi / img_lo (optional, [K][N] weights only): the weights as stage
// images, the exact shared-memory bytes of one ring stage's weight tile for
// tile t and K block kb at ((t * K / BK) + kb) * 16 KB, so that one bulk copy
// fills a stage (four to eight tiled TMA boxes otherwise; a ring CTA then
// streams about twice the bytes per second).  With wsplit, img_hi is the fp32
// image, split in shared memory; otherwise the tf32 hi / lo images (or the
// fp16 image).
struct TcWeights {
    CUtensorMap hi, lo;
    int K, N;
    bool kmajor;   // false: [K][N] (Conv1D, feature-contiguous); true: [N][K] (rows of wte)
    bool wsplit;   // TC_TF32X3 with the fp32 weights in `hi` (or the fp32 image)
    const void *img_hi = nullptr, *img_lo = nullptr;
};
int tc_weights(TcWeights *w, int kind, const void *hi, const void *lo, int K, int N);

// Stage images.  tc_stage_perm records, on the device, where a tiled TMA load
// of one stage's weight boxes puts each element: table[p] = row * 128 +
// feature of the element at element position p of the stage (4096 fp32 or
// 8192 fp16 positions), found by loading a tensor whose elements hold their
// own coordinates (idx: 16 KB of device scratch, 16-byte aligned).
// tc_image_elems is the size of one projection's image in elements;
// launch_tc_image gathers W [K][N] into it (features past N zero), as tf32
// hi / lo (TC_TF32X3 with img_lo), fp32 (img_lo == nullptr) or fp16.
int tc_stage_perm(int kind, void *idx, unsigned *table, int *err, cudaStream_t st);
size_t tc_image_elems(int kind, int K, int N);
void launch_tc_image(int kind, const void *W, void *img_hi, void *img_lo, const unsigned *table, int K, int N,
                     cudaStream_t st);
// The same for a [N][K] row-major weight (K-contiguous), e.g. the tied LM head wte.
int tc_weights_kmajor(TcWeights *w, int kind, const void *hi, const void *lo, int K, int N);

// Activation operand X [R][K] (hi / lo fp32 copies, or fp16): maps for every
// row-tile height the planner may pick.
struct TcRowsOperand {
    CUtensorMap hi[3], lo[3];   // box heights 32, 64, 128
    int K, R;
};
int tc_rows_operand(TcRowsOperand *x, int kind, const void *hi, const void *lo, int K, int R);

// Split an fp32 [n] array into tf32 hi / lo copies (TC_TF32X3) or round it to
// fp16 (TC_F16: h16 written, hi / lo unused).  n % 4 == 0.
void launch_tc_prep(int kind, const float *x, float *hi, float *lo, __half *h16, long long n, cudaStream_t st);

// Floats of partial-sum scratch the planner uses for up to R_max rows of an
// N x K projection on `sms` SMs.
size_t tc_partial_floats(int R_max, int N, int K, int kind, int sms);

// Output tiles one GEMM may have (tile counters to allocate, zeroed).
constexpr int kTcMaxTiles = 4096;

// out[r][n] = epilogue(sum_k X[r][k] W[k][n]) for r < R (bias / GELU /
// residual / K,V append of g2_device.cuh); `op` optionally also writes the
// output as the next GEMM's operand.  With one K split the GEMM applies the
// epilogue from tensor memory (one launch); with split-K the partials go to
// `partial` and one kernel sums them in split order (two launches).
// `tile_ctr` is reserved (kTcMaxTiles zeroed counters).  out_stride > 0 sets
// the row stride of out and resid (else N).  With ln_g / ln_b, a split-K GEMM
// also takes the LayerNorm of each output row (gamma ln_g, beta ln_b) and
// writes it as ln_op, the next GEMM's operand; *ln_done then says whether it
// did (a single-split GEMM does not: its caller runs the LayerNorm).  With
// defer_reduce a split-K GEMM leaves its partial tiles in `partial` for the
// consumer to sum; *si_out receives where the partials are (si_out->split()
// false: the GEMM applied the epilogue itself).  `err` receives an error code
// if a wait inside the kernel expires.  Returns the launch count.
template <typename WT>
int launch_tc_gemm(int kind, const TcWeights &w, const TcRowsOperand &x, int R, float *partial, size_t partial_floats,
                   unsigned *tile_ctr, int *err, const WT *bias, const float *resid, float *out, int epi,
                   const KVLayout *kv, int layer, Rows rows, int sms, cudaStream_t st, OperandOut op = OperandOut(),
                   int out_stride = 0, const WT *ln_g = nullptr, const WT *ln_b = nullptr, OperandOut ln_op = OperandOut(),
                   bool *ln_done = nullptr, bool defer_reduce = false, SplitInfo *si_out = nullptr);

}  // namespace g2
