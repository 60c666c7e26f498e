/* ref_cpu.h -- CPU restatement of the GPT2-OpenCL-1.1 hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity oracle for the
 * CUDA engine: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The engine never links or calls it.
 *
 * Every function restates one piece of the reference (citations are
 * file:line in the reference project) with the reference's summation
 * order: serial-k dot products, strided split-K partials reduced in slice
 * order, the 64-lane tree softmax, one work-item per output.  It is built
 * with -ffp-contract=off so no multiply-add is fused, which makes it
 * bit-identical to the reference's math.cl compiled for the host CPU with
 * the same flag (oracle/_ref, see oracle/Makefile).
 *
 * Parity pin: tests/test_oracle_pin.py checks each kernel and the whole
 * prefill/decode/sample flow bit-exactly against the reference's own code
 * (math.cl and main.c compiled from their sources into oracle/_ref with a
 * CPU OpenCL shim), and tests/golden/ holds fixtures produced that way.
 */
#ifndef REF_CPU_H
#define REF_CPU_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define REF_MAX_SEQ 1024   /* KV and score row stride, main.c:51 / math.cl:18 */
#define REF_EOS 50256      /* main.c:58 */
#define REF_MAX_TOPK 256   /* main.c:55 */
#define REF_MAX_KSLICE 8   /* main.c:54 */

/* ---- kernels (math.cl) -------------------------------------------------- */
void ref_matvec(const float *A, const float *B, const float *bias, const float *residual,
                float *C, int N, int K, int apply_gelu);                    /* math.cl:152 */
void ref_matvec4(const float *A, const float *B, const float *bias, const float *residual,
                 float *C, int N, int K, int apply_gelu);                   /* math.cl:185 */
void ref_matvec4_sk(const float *A, const float *B, float *partial, int N, int K,
                    int kslice);                                            /* math.cl:229 */
void ref_reduce_partial(const float *partial, const float *bias, const float *residual,
                        float *C, int N, int kslice, int apply_gelu);       /* math.cl:249 */
void ref_layernorm(const float *x, float *out, const float *gamma, const float *beta,
                   int n_embd, int seq_len);                                /* math.cl:283 */
void ref_add_inplace(float *a, const float *b, int n);                      /* math.cl:314 */
void ref_gelu(float *x, int n);                                             /* math.cl:325 */
float ref_gelu_f(float v);                                                  /* math.cl:21  */
void ref_embed(const float *wte, const float *wpe, float *out, int n_embd, int seq_len,
               int start_pos, const int *ids);                              /* math.cl:333 */
void ref_split_kv(const float *qkv, float *k_cache, float *v_cache, int start_pos, int T,
                  int D, int max_seq);                                      /* math.cl:367 */
void ref_attn_scores_1q(const float *qkv, const float *k_cache, float *scores, int q_base,
                        int T_kv, int D, int DH, int NH, int max_seq, float scale); /* math.cl:388 */
void ref_attn_softmax_1q(float *scores, int T_kv, int NH, int lws);         /* math.cl:415 */
void ref_attn_out_1q(const float *scores, const float *v_cache, float *out, int T_kv, int D,
                     int DH, int out_base);                                 /* math.cl:459 */
void ref_matmul(const float *A, const float *B, const float *bias, float *C, int M, int N,
                int K);                                                     /* main.c:593-684 */

/* launch_matvec / launch_matvec_splitk dispatch (main.c:1554-1618). */
void ref_launch_matvec(const float *A, const float *B, const float *bias, const float *residual,
                       float *C, int N, int K, int apply_gelu);
void ref_launch_matvec_splitk(const float *A, const float *B, const float *bias,
                              const float *residual, float *C, int N, int K, int ks,
                              int apply_gelu, float *partial_scratch);

/* ---- model --------------------------------------------------------------- */
typedef struct {
    int n_layer, n_embd, n_head, n_ctx, vocab_size, ffn_dim, padded_vocab;
} ref_config;

typedef struct ref_model ref_model;
typedef struct ref_seq ref_seq;

const char *ref_last_error(void);
/* load_config (main.c:294-331) with the ceilings of main.c:47-52 lifted, except
 * n_ctx <= REF_MAX_SEQ, which fixes the KV stride. */
int ref_load_config(const char *dir, ref_config *out);
/* load_model (main.c:1339-1417): F32 as in the reference, plus F16/BF16 widened
 * to float (the fp16 configuration runs the fp32 oracle on fp16-rounded weights). */
int ref_model_open(const char *dir, ref_model **out);
void ref_model_close(ref_model *m);
void ref_model_get_config(const ref_model *m, ref_config *out);
/* Pinned tuning: split-K slices for attn_proj and ffn2 (main.c:1815, 1824) and the
 * softmax work-group size (main.c:124).  Defaults 8, 8, 64. */
void ref_model_set_tuning(ref_model *m, int ks_attn_proj, int ks_ffn2, int attn_lws);
const float *ref_model_lm_head(const ref_model *m);   /* [E, V_pad], main.c:1302 */

int ref_seq_new(const ref_model *m, ref_seq **out);
void ref_seq_free(ref_seq *s);
int ref_prefill(ref_seq *s, const int *ids, int prompt_len);   /* main.c:1739-1790 */
int ref_decode(ref_seq *s, int token, int pos);                 /* main.c:1792-1833 */
const float *ref_seq_logits(const ref_seq *s);                  /* buf_logits[V_pad] */
const float *ref_seq_hidden(const ref_seq *s);                  /* buf_hidden (row 0 after decode) */
const float *ref_seq_kcache(const ref_seq *s, int layer);       /* [E, 1024] transposed */
const float *ref_seq_vcache(const ref_seq *s, int layer);       /* [1024, E] */

/* ---- sampler (main.c:1839-1939) ------------------------------------------ */
float ref_kth_largest(const float *a, int n, int k);
/* sample_next_token on a copy of logits[0..vocab_size). Uses the C library rand(). */
int ref_sample_next_token(const float *logits, int vocab_size, const int *context_ids,
                          int n_context, int forbid_eos, float temperature, int top_k,
                          float rep_penalty);
void ref_srand(unsigned seed);

/* Greedy generation as main.c:2106-2150 (rep_penalty/min_tokens as given). Writes up
 * to max_new tokens into out, returns the number generated or <0 on error. */
int ref_generate(ref_seq *s, const int *prompt, int prompt_len, int max_new, int min_new,
                 float temperature, int top_k, float rep_penalty, int *out);

int ref_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
