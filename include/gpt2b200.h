/* gpt2b200.h -- C ABI of the B200 GPT-2 inference engine.
 *
 * Drop-in for the host seam of GPT2-OpenCL-1.1's main.c, the static functions
 * between its generation loop and its OpenCL launch helpers:
 *
 *   load_config + load_model + preallocate_buffers  (main.c:294, 1339, 1451)
 *                                  -> g2_open
 *   prefill(ids, prompt_len)        (main.c:1739)   -> g2_prefill
 *   decode(new_token_id, start_pos) (main.c:1792)   -> g2_decode, g2_decode_batch
 *   logits read in sample_next_token (main.c:1878)  -> g2_logits, g2_argmax
 *   sample_next_token               (main.c:1872)   -> g2_sample
 *   the greedy loop of main()       (main.c:2106-2150) -> g2_generate
 *
 * and of its launch helpers (main.c:1518-1733) for single kernels on device
 * pointers: g2k_*.
 *
 * Conventions (the reference exits the process on any error, main.c:189-195;
 * this library never does):
 *  - every call returns int status: G2_OK (0) or a negative G2_ERR_*;
 *    g2_last_error() gives the message of the calling thread's last failure;
 *  - the engine owns device memory; the caller owns host buffers;
 *  - one engine per GPU; calls on one engine are serialised by the caller;
 *    engines on different GPUs may be driven from different host threads;
 *  - weights are safetensors in GPT-2's Conv1D [in, out] layout (nn.Linear
 *    [out, in] is detected and transposed), F32 or F16; the LM head is tied to
 *    wte unless lm_head.weight exists; logits have padded_vocab = (V+3)&~3
 *    entries, the padding being 0 (main.c:326, 1302-1337).
 */
#ifndef GPT2B200_H
#define GPT2B200_H
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G2_OK 0
#define G2_ERR_ARG (-1)      /* null pointer, bad size or flag */
#define G2_ERR_IO (-2)       /* model file missing or unreadable */
#define G2_ERR_FORMAT (-3)   /* malformed config/safetensors, missing tensor, bad shape or dtype */
#define G2_ERR_CUDA (-4)     /* CUDA error, no sm_100 device */
#define G2_ERR_OOM (-5)      /* host or device allocation failed */
#define G2_ERR_RANGE (-6)    /* token id, position, slot or length out of range */
#define G2_ERR_STATE (-7)    /* call out of order (e.g. decode at a position not yet filled) */
#define G2_ERR_TIMEOUT (-8)  /* a bounded device-side wait expired */

#define G2_F32 0             /* fp32 weights, activations, KV (the reference's arithmetic type) */
#define G2_F16 1             /* fp16 weights and KV, fp32 accumulation and activations */

#define G2_EOS 50256         /* main.c:58 */
#define G2_MAX_TOPK 256      /* main.c:55 */

typedef struct g2_engine g2_engine;

typedef struct g2_config {
    int n_layer, n_embd, n_head, n_ctx, vocab_size, ffn_dim, padded_vocab;
    int dtype;       /* G2_F32 / G2_F16 */
    int max_batch;   /* sequence slots */
    int device;
    size_t weight_bytes;   /* bytes of weights streamed per decode step (for GB/s) */
    size_t device_bytes;   /* device memory held by the engine */
    int persistent;        /* 1: B = 1 decode runs the persistent kernel (one launch per
                              g2_decode / g2_generate); 0: per-layer kernels in a CUDA graph */
} g2_config;

const char *g2_last_error(void);

/* config.json + model.safetensors from model_dir onto CUDA device `device`,
 * with KV caches for `max_batch` independent sequences (slots 0..max_batch-1).
 * Replaces load_config / init_opencl / load_model / preallocate_buffers. */
int g2_open(const char *model_dir, int device, int max_batch, int dtype, g2_engine **out);
int g2_close(g2_engine *e);
int g2_get_config(const g2_engine *e, g2_config *out);

/* prefill (main.c:1739): run ids[0..n) at positions 0..n-1 of `slot`, fill its
 * KV cache, leave the logits of the last row in the slot's logits buffer. */
int g2_prefill(g2_engine *e, int slot, const int *ids, int n);

/* decode (main.c:1792): one token at `pos` of `slot` (pos must equal the
 * number of positions already in the slot's cache). */
int g2_decode(g2_engine *e, int slot, int token, int pos);
/* decode for n slots at once (one token each, each at its own position). */
int g2_decode_batch(g2_engine *e, int n, const int *slots, const int *tokens, const int *pos);

/* The LM head split over several GPUs by vocabulary rows (the optional
 * column-sharded GPT-2 XL head: each GPU takes a range of wte's rows for the
 * rows of every GPU and the best per row is exchanged).
 * g2_decode_batch_rows: decode() (main.c:1792-1830) for n sequences without
 * the LM head matvec (main.c:1831); writes the final LayerNorm of each row,
 * [n][n_embd] fp32, to `rows` (device memory, 16-byte aligned).  No logits are
 * written.  Returns once the rows are complete.
 * g2_lm_head_rows: the LM head matvec (main.c:1831) over wte rows [v0, v1)
 * (v0 a multiple of 4) for nrows (<= max(n_ctx, max_batch)) normalised rows in
 * device memory; best_value[r] / best_index[r] (device memory) receive the
 * row's first maximum in that range (main.c:1898-1904) and its index in the
 * whole vocabulary.  Returns once they are complete. */
int g2_decode_batch_rows(g2_engine *e, int n, const int *slots, const int *tokens, const int *pos, float *rows);
int g2_lm_head_rows(g2_engine *e, int nrows, const float *rows, int v0, int v1, float *best_value, int *best_index);

/* Copy the first n (<= padded_vocab) logits of `slot` to host memory. */
int g2_logits(g2_engine *e, int slot, float *host, int n);
/* Device argmax over logits[0..vocab_size) of `slot`, first index on ties
 * (main.c:1898-1904); forbid_eos excludes G2_EOS (main.c:1882). */
int g2_argmax(g2_engine *e, int slot, int forbid_eos, int *token, float *value);

/* The k largest logits of `slot` over logits[0..vocab_size), found on the
 * device (1 <= k <= min(G2_MAX_TOPK, vocab_size)): values[0..k) in decreasing
 * order with their token ids, equal values by increasing id (the order of the
 * first-maximum scan, main.c:1898-1904), so values[k-1] is kth_largest(logits,
 * k) (main.c:1839-1868) and ids[0] is the greedy token.  values and ids are host
 * arrays of k entries; 2 k values come back instead of the vocab_size logits. */
int g2_topk(g2_engine *e, int slot, int k, float *values, int *ids);

/* sample_next_token (main.c:1872-1939) on host logits[0..vocab_size): EOS mask,
 * repetition penalty over the unique context ids, then greedy (temperature
 * <= 0, first max) or temperature + top-k (<= G2_MAX_TOPK) + C rand() draw. */
int g2_sample(const float *logits, int vocab_size, const int *context_ids, int n_context,
              int forbid_eos, float temperature, int top_k, float rep_penalty, int *out_token);

/* sample_next_token (main.c:1872-1939) on the device, on the logits of `slot`
 * (left unchanged): the same EOS mask, repetition penalty over the unique ids
 * context_ids[0..n_context) (host array, n_context <= n_ctx), greedy first
 * maximum for temperature <= 0, else 1/temperature scaling, the top-k
 * threshold (k-th largest; k clamped to G2_MAX_TOPK) and the inverse-CDF draw
 * at u01 * sum.  The caller supplies the uniform draw u01 in [0, 1) -- the
 * reference uses rand() / (RAND_MAX + 1.0).  Only the token comes back to the
 * host (4 bytes instead of the vocab_size logits). */
int g2_sample_device(g2_engine *e, int slot, const int *context_ids, int n_context, int forbid_eos,
                     float temperature, int top_k, float rep_penalty, double u01, int *out_token);

/* ---- tokenizer (tokenizer.c:442-579): GPT-2 byte-level BPE ----
 * vocab.json + merges.txt from `dir`; the same pre-tokenization, merges and
 * byte mapping as the reference, so the same ids and bytes. */
typedef struct g2_tokenizer g2_tokenizer;
int g2_tokenizer_load(const char *dir, g2_tokenizer **out);
void g2_tokenizer_free(g2_tokenizer *t);
int g2_tokenizer_vocab_size(const g2_tokenizer *t);
/* UTF-8 text -> at most max_ids ids; returns the count (or a negative code). */
int g2_tok_encode(const g2_tokenizer *t, const char *text, int *ids, int max_ids);
/* ids -> bytes, NUL-terminated within max_bytes; returns the bytes written. */
int g2_tok_decode(const g2_tokenizer *t, const int *ids, int n, char *out, int max_bytes);

/* Greedy generation on the device (main.c:2106-2150 with --greedy,
 * --rep-penalty 1): prefill `prompt`, then argmax/decode until n_new tokens
 * (the prefill's token included) are in out_tokens.  EOS is excluded from the
 * argmax for the first `min_new` tokens and ends generation after that.
 * Returns the number of tokens written (>= 1) or a negative status. */
int g2_generate(g2_engine *e, int slot, const int *prompt, int n_prompt, int n_new, int min_new,
                int *out_tokens);

/* Greedy generation for `n` slots at once with batched decode steps
 * (prompts concatenated in `prompts`, lengths in `prompt_lens`); every slot
 * generates exactly n_new tokens with EOS excluded.  out_tokens is [n][n_new]. */
int g2_generate_batch(g2_engine *e, int n, const int *slots, const int *prompts,
                      const int *prompt_lens, int n_new, int *out_tokens);

int g2_synchronize(g2_engine *e);
/* Device time (ms) of the last g2_generate / g2_generate_batch decode phase
 * and prefill phase, measured with CUDA events on the engine's stream. */
int g2_last_timing(g2_engine *e, float *prefill_ms, float *decode_ms, int *decode_steps);
/* Kernel launches issued by this engine since open. */
long long g2_launch_count(const g2_engine *e);

/* ---- single kernels on device pointers (main.c:1518-1733) -----------------
 * All pointers are device pointers on the current device; `stream` is a
 * cudaStream_t (NULL = legacy default stream).  fp32 throughout. */

/* Bytes of scratch g2k_matvec needs for an N x K product. */
size_t g2k_matvec_workspace(int N, int K);
/* launch_matvec / launch_matvec_splitk (main.c:1554-1618):
 * y[n] = sum_k x'[k] * W[k*N + n] (+bias[n]) (+residual[n]) (then GELU),
 * where x' = LayerNorm(x; ln_gamma, ln_beta, eps 1e-5) when ln_gamma is not
 * NULL (the decode layernorm, main.c:1620, fused in), else x.  residual may
 * alias y.  N % 4 == 0, K % 16 == 0; a K slice that would not fit one
 * CTA's 48 KB of shared memory (very wide N with K over ~11,000) gives
 * G2_ERR_RANGE.  `workspace` must hold
 * g2k_matvec_workspace(N, K) bytes, 256-byte aligned, and be zero-filled
 * before its first use; the call leaves it ready for the next one. */
int g2k_matvec(const float *x, const float *W, const float *bias, const float *residual, float *y,
               int N, int K, int apply_gelu, const float *ln_gamma, const float *ln_beta,
               void *workspace, size_t workspace_bytes, void *stream);

/* g2k_matvec without a workspace argument, for callers that cannot allocate
 * device memory (an FFI binding with no device allocator of its own, an
 * application whose device memory belongs to another allocator, or a path
 * that must not take cudaMalloc's implicit synchronisation).  This entry has
 * no counterpart in the reference.  Its scratch is a fixed 256 KiB device
 * array inside this library (held on every GPU that loads it until exit);
 * shapes whose split-K scratch would exceed it return G2_ERR_RANGE.  The
 * first call on a device looks the array up (make it before any stream
 * capture); that address does not survive cudaDeviceReset, so make no call
 * on a device after resetting it in the same process.  Every call clears the
 * array's counters before its kernel; calls that overlap on the GPU share
 * the array and race, so serialise them.
 * Same arguments and results as g2k_matvec otherwise. */
int g2k_matvec_noalloc(const float *x, const float *W, const float *bias, const float *residual, float *y,
                       int N, int K, int apply_gelu, const float *ln_gamma, const float *ln_beta, void *stream);

/* launch_matmul (main.c:1518) + launch_gelu / launch_add (main.c:1635-1654):
 * C[m][n] = sum_k A[m][k] * B[k][n] (+bias[n]) (GELU if apply_gelu) (+residual[m][n]).
 * residual may alias C.  N % 4 == 0, K % 4 == 0. */
int g2k_matmul(const float *A, const float *B, const float *bias, const float *residual, float *C,
               int M, int N, int K, int apply_gelu, void *stream);

/* The same product on the tensor cores (tcgen05): the runtime matmul of
 * prefill (main.c:593-684) for many rows.  precision G2_F32 splits every
 * operand into tf32 hi + lo and sums three tf32 products (fp32-level
 * accuracy); G2_F16 rounds both operands to fp16.  fp32 accumulation either
 * way.  K % 64 == 0, N % 8 == 0, A / B / C 16-byte aligned.  `workspace`
 * (256-byte aligned) holds g2k_matmul_tc_workspace() bytes; its first int
 * becomes G2_ERR_TIMEOUT if a wait inside the kernel expired. */
size_t g2k_matmul_tc_workspace(int M, int N, int K, int precision);
int g2k_matmul_tc(const float *A, const float *B, const float *bias, const float *residual, float *C,
                  int M, int N, int K, int apply_gelu, int precision, void *workspace,
                  size_t workspace_bytes, void *stream);

/* launch_layernorm (main.c:1620): rows of n_embd, eps 1e-5. */
int g2k_layernorm(const float *x, float *out, const float *gamma, const float *beta, int n_embd,
                  int rows, void *stream);

/* Bytes of scratch g2k_attention needs for n_head heads. */
size_t g2k_attention_workspace(int n_head, int max_seq);
/* launch_attn_scores + launch_attn_softmax + launch_attn_out (main.c:1687-1733)
 * for one query: out[h*64+d] = sum_j softmax_j(q_h . K[h][j] / 8) * V[h][j][d]
 * over j = 0..T_kv-1.  q: [n_head*64]; K, V: [n_head][max_seq][64] (this
 * engine's cache layout, position-major per head).  T_kv <= max_seq <= 1024.
 * Workspace rules as g2k_matvec. */
int g2k_attention(const float *q, const float *K, const float *V, float *out, int n_head,
                  int max_seq, int T_kv, void *workspace, size_t workspace_bytes, void *stream);

/* The kernel of g2_topk on device pointers: the k (1 <= k <= min(G2_MAX_TOPK, n))
 * largest of logits[0..n), values[0..k) decreasing with their indices ids[0..k),
 * equal values by increasing index (-0.0 and +0.0 are equal; logits finite).
 * Asynchronous on `stream`. */
int g2k_topk(const float *logits, int n, int k, float *values, int *ids, void *stream);

#ifdef __cplusplus
}
#endif
#endif
