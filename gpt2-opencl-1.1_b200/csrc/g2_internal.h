// g2_internal.h -- device-side types and kernel launchers shared by the
// engine (g2_engine.cu) and the kernels (g2_kernels.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace g2 {

// Launch a kernel with programmatic dependent launch (it may start while the
// previous kernel of the stream finishes; it calls pdl_wait() before touching
// that kernel's data).  G2_NO_PDL=1 turns it off (plain stream order).
bool pdl_enabled();
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

constexpr int kHeadDim = 64;        // GPT-2 head size (all family members)
constexpr int kAttnChunk = 128;     // keys per attention CTA (flash-decoding split)
constexpr int kMaxSeq = 1024;       // KV positions per slot (main.c:51)
constexpr int kEos = 50256;         // main.c:58

// Per-token decode state in device memory.  The B=1 decode graph reads the
// token and position from here and its last kernel writes the next greedy
// token back, so one captured graph serves every step.
struct StepState {
    int token;       // token to embed this step
    int pos;         // its position
    int slot;        // KV slot
    int step;        // tokens generated so far (index into out_tokens)
    int min_new;     // EOS is excluded from the argmax while step < min_new
    int pad[3];
};

// KV cache addressing: element (slot, layer, head, pos, d) of K (or V) is at
// base + slot*slot_stride + layer*layer_stride + (head*max_seq + pos)*64 + d.
struct KVLayout {
    void *k, *v;                 // cache bases (float or __half)
    long long slot_stride;       // elements
    long long layer_stride;      // elements
    int max_seq;
    int n_head;
    int n_slots = 1;             // sequence slots the cache holds
};

// Bounds-checked build (-DG2_CHECK, `make check`): device code tests the
// data-dependent indexes it is about to use (token ids, positions, slots, key
// counts) with G2_BOUNDS(ok, site); a failed test records `site` in this
// translation unit's flag (first failure wins) and the access is skipped, in
// place of a device assert.  The host reads and clears the flags with
// check_flags() at its synchronising calls and reports G2_ERR_RANGE.  In the
// normal build G2_BOUNDS(ok, site) is just `ok` (the same guards, unreported).
#ifdef G2_CHECK
#ifdef __CUDACC__
static __device__ int g2_check_flag;
__device__ __forceinline__ bool g2_bounds(bool ok, int site) {
    if (!ok) atomicCAS(&g2_check_flag, 0, site);
    return ok;
}
#define G2_BOUNDS(ok, site) ::g2::g2_bounds((ok), (site))
#endif
#else
#define G2_BOUNDS(ok, site) (ok)
#endif
// The first failed bounds test of each kernel file since the last call (0: none),
// cleared; always 0 in the normal build.
int check_flags();
int check_flag_kernels();
int check_flag_mega();
int check_flag_tc();

// Row descriptors of a batched pass: row r embeds tok[r] at pos[r] of slot[r].
struct Rows {
    const int *tok;
    const int *pos;
    const int *slot;
};

// EPI_NOSTORE: the result goes only to the next GEMM's operand (OperandOut), not to `out`.
enum Epilogue { EPI_NONE = 0, EPI_BIAS = 1, EPI_GELU = 2, EPI_RESID = 4, EPI_KV = 8, EPI_NOSTORE = 16 };

// A kernel's output also written as the next tensor-core GEMM's operand (row
// stride = that GEMM's K): kind 1 = tf32 hi / lo pair (TC_TF32X3), 0 = fp16
// (TC_F16), -1 = not written.
struct OperandOut {
    int kind = -1;
    float *hi = nullptr, *lo = nullptr;
    __half *h16 = nullptr;
};

// ---- launchers (g2_kernels.cu); all asynchronous on `st` ------------------------
// p[0..4) = a, b, c, d on the device (g2_kernels.cu).
void launch_set_ints(int *p, int a, int b, int c, int d, cudaStream_t st);
// sample_next_token on the device (g2_sample_dev.cu): token -> out[0].
void launch_sample(const float *logits, float *work, int V, const int *ctx, int n_ctx, int forbid_eos,
                   float temperature, int top_k, float rep_penalty, double u, int *out, cudaStream_t st);
// The k (<= G2_MAX_TOPK) largest of logits[0..V) on the device (g2_sample_dev.cu):
// vals / idx [k], the larger value first, equal values by the smaller index.
void launch_topk(const float *logits, int V, int k, float *vals, int *idx, cudaStream_t st);

template <typename WT>
void launch_embed(const WT *wte, const WT *wpe, Rows rows, float *h, int E, int V, int n_pos, int nrows,
                  cudaStream_t st);

template <typename WT>
void launch_layernorm(const float *x, float *out, const WT *g, const WT *b, int E, int nrows, cudaStream_t st,
                      OperandOut op = OperandOut());

// B=1 GEMV: y = x' W (+bias)(GELU)(+resid)(KV append), x' = LN(x) if ln_g.
// partial: [ksplit][N] floats, counters: [N / cols-per-CTA] zeroed uints.
struct GemvPlan {
    int ksplit;
    int tiles;
    // dynamic shared memory of one CTA: its x slice plus the column-tile partials
    // (the launch keeps the default 48 KB limit; entry points refuse larger shapes)
    size_t smem_bytes;
};
constexpr size_t kGemvMaxSmem = 48 * 1024;
template <typename WT>
GemvPlan gemv_plan(int N, int K, int sms);
template <typename WT>
void launch_gemv(const float *x, const WT *W, const WT *bias, const float *resid, float *y, int N, int K,
                 int epi, const WT *ln_g, const WT *ln_b, float *partial, unsigned *counters, GemvPlan plan,
                 const KVLayout *kv, int layer, const int *pos_ptr, const int *slot_ptr, cudaStream_t st);

// Rows GEMM: C[M][N] = A[M][K] W[K][N] with the same epilogues (KV append per row).
template <typename WT>
void launch_gemm_rows(const float *A, const WT *W, const WT *bias, const float *resid, float *C, int M, int N,
                      int K, int epi, const KVLayout *kv, int layer, Rows rows, cudaStream_t st);

// Single-query attention for nrows rows: row r attends to positions
// 0..pos[r] of its slot. partial/counters: scratch (see attn_workspace_*).
size_t attn_partial_floats(int nrows, int n_head, int max_seq);
size_t attn_counter_count(int nrows, int n_head);

// How many split-K partials a tensor-core GEMM left for an output column, and
// where.  Partial j of column n is at part[j][row][n] either way.
//  * Uniform splits (G == 0): every 128-feature tile has `splits` partials.
//  * Balanced split (G > 0): the tiles' K blocks, tile-major (U = tiles * KB
//    units), are cut into G contiguous equal shares, one per CTA, so a CTA
//    may finish one tile and start the next.  CTA c takes units
//    [floor(c U / G), floor((c + 1) U / G)); its piece of tile t is partial
//    c - cta_of(t KB) of that tile, so the pieces of a tile are summed in
//    K order.
struct SplitInfo {
    int splits = 1;
    int G = 0;
    int KB = 0;
    long long U = 0;
    // the CTA whose share holds unit u
    __host__ __device__ int cta_of(long long u) const { return (int)(((u + 1) * G - 1) / U); }
    // partials of output column n (tiles of 128 features)
    __host__ __device__ int at(int n) const {
        if (!G) return splits;
        const long long u0 = (long long)(n >> 7) * KB;
        return cta_of(u0 + KB - 1) - cta_of(u0) + 1;
    }
    __host__ __device__ bool split() const { return G > 0 || splits > 1; }
};

// The c_attn output of a batched decode step still as split-K partial tiles
// ([partials][rows][3E], row stride qkv_stride, counted by si) plus the c_attn bias: the
// attention sums them itself (and appends the new K and V to the cache), so
// the GEMM needs no reduce launch.  Only for rows of distinct sequences: a
// row's attention then reads no K/V row that another row of the pass appends.
struct QkvPartials {
    const float *part = nullptr;
    SplitInfo si;
    const void *bias = nullptr;   // [3E] of the engine's weight type
    int *err = nullptr;           // where an expired wait of the streamed attention is recorded
    // fp16 caches: CUtensorMaps of K and V as [rows][64] (box 64 x 64, 128-byte
    // swizzle) for the tensor-core path of the streamed attention, or nullptr
    const void *kmap = nullptr, *vmap = nullptr;
};

template <typename KT>
void launch_attention(const float *qkv, int qkv_stride, const KVLayout &kv, int layer, Rows rows, int nrows,
                      float *out, int out_stride, float *partial, unsigned *counters, int max_pos_hint,
                      cudaStream_t st, OperandOut op = OperandOut(), QkvPartials qp = QkvPartials());

// Causal attention of a prompt's rows (prefill of one slot: every row has the
// same slot, row r attends to positions 0..pos[r], whose K and V are already in
// the cache).  Tiles of 64 query rows x 64 keys with K and V staged in shared
// memory; out[r][h*64 + d] (and `op`, the next GEMM's operand).
template <typename KT>
void launch_prefill_attention(const float *qkv, int qkv_stride, const KVLayout &kv, int layer, Rows rows, int nrows,
                              float *out, int out_stride, cudaStream_t st, OperandOut op = OperandOut());

// LM head on one row x (fp32 [E]) with the final LayerNorm fused:
// logits[v] = LN_f(x) . wte[v]; argmax over v < V (first index on ties,
// EOS excluded while state->step < state->min_new when state != NULL, or
// when forbid_eos).  Writes logits[0..Vp), best (token, value) to result[0..1]
// and, if state, appends the token to out_tokens and advances state.
template <typename WT>
void launch_lm_head(const float *x, const WT *wte, const WT *lnf_g, const WT *lnf_b, float *logits, int E,
                    int V, int Vp, int forbid_eos, float *partial, unsigned *counter, int *result,
                    StepState *state, int *out_tokens, cudaStream_t st);
int lm_head_blocks();

// Batched LM head: logits[r][v] = x_r . wte[v] for rows of x (already
// normalised), then argmax per row into tokens[r] (and optional state update).
template <typename WT>
void launch_lm_head_rows(const float *x, const WT *wte, float *logits, int E, int V, int Vp, int nrows,
                         cudaStream_t st);
void launch_argmax_rows(const float *logits, int V, int Vp, int nrows, int forbid_eos, int *tokens, float *values,
                        int *tok_next, int *pos_next, int *out_tokens, int out_stride, const int *step_ptr,
                        cudaStream_t st);

void launch_copy_row(const float *src, float *dst, int n, cudaStream_t st);
// p[0..n) += add
void launch_add_ints(int *p, int n, int add, cudaStream_t st);

// dst[c][r] = src[r][c] for a [rows][cols] fp32 matrix, converted to WT: the
// load-time transpose of an nn.Linear [out][in] weight into the Conv1D
// [in][out] layout the kernels read (main.c:1252-1300 does it on the host).
template <typename WT>
void launch_transpose(const float *src, WT *dst, int rows, int cols, cudaStream_t st);

// Record `msg` as the calling thread's g2_last_error(); returns `code`.
int set_error(int code, const char *msg);
void launch_step_advance(int *step_ptr, cudaStream_t st);

}  // namespace g2
