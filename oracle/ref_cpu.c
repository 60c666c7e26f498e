/* ref_cpu.c -- CPU restatement of the GPT2-OpenCL-1.1 hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity oracle for the CUDA engine (see
 * ref_cpu.h).  Built with -O3 -ffp-contract=off -fopenmp; OpenMP splits only
 * independent work-items (output columns, rows, heads), so every output is
 * produced by the same sequence of float operations as one OpenCL work-item
 * of the reference.
 */
#define _POSIX_C_SOURCE 200809L
#define _FILE_OFFSET_BITS 64
#include "ref_cpu.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static char g_err[512];
static int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}
const char *ref_last_error(void) { return g_err; }

int ref_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ========================================================================
 * Kernels (math.cl)
 * ======================================================================== */

/* math.cl:21-23 */
float ref_gelu_f(float v) {
    return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
}

#define COLCHUNK 256

/* Epilogue shared by matvec4 / reduce_partial: +bias, +residual, GELU, in that
 * order (math.cl:212-225, 266-279). */
static inline float epi(float s, const float *bias, const float *residual, int n, int gelu) {
    if (bias) s += bias[n];
    if (residual) s += residual[n];
    if (gelu) s = ref_gelu_f(s);
    return s;
}

/* math.cl:185-226.  Work-item col4 owns columns 4*col4..+3 and accumulates
 * s += A[k] * B[k][c] for k = 0..K-1 in order.  Iterating k outside and the
 * columns inside gives each column exactly that sequence. */
void ref_matvec4(const float *A, const float *B, const float *bias, const float *residual,
                 float *C, int N, int K, int apply_gelu) {
#pragma omp parallel for schedule(static)
    for (int n0 = 0; n0 < N; n0 += COLCHUNK) {
        const int n1 = n0 + COLCHUNK < N ? n0 + COLCHUNK : N;
        float acc[COLCHUNK];
        for (int n = n0; n < n1; ++n) acc[n - n0] = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float a = A[k];
            const float *b = B + (size_t)k * N;
            for (int n = n0; n < n1; ++n) acc[n - n0] += a * b[n];
        }
        for (int n = n0; n < n1; ++n) C[n] = epi(acc[n - n0], bias, residual, n, apply_gelu);
    }
}

/* math.cl:152-182: four interleaved partial sums, tail into s0, then
 * ((s0 + s1) + s2) + s3. */
void ref_matvec(const float *A, const float *B, const float *bias, const float *residual,
                float *C, int N, int K, int apply_gelu) {
#pragma omp parallel for schedule(static)
    for (int col = 0; col < N; ++col) {
        const float *Bc = B + col;
        float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
        int k = 0;
        for (; k + 4 <= K; k += 4) {
            s0 += A[k + 0] * Bc[(size_t)(k + 0) * N];
            s1 += A[k + 1] * Bc[(size_t)(k + 1) * N];
            s2 += A[k + 2] * Bc[(size_t)(k + 2) * N];
            s3 += A[k + 3] * Bc[(size_t)(k + 3) * N];
        }
        for (; k < K; ++k) s0 += A[k] * Bc[(size_t)k * N];
        float sum = s0 + s1 + s2 + s3;
        C[col] = epi(sum, bias, residual, col, apply_gelu);
    }
}

/* math.cl:229-246: slice ks sums k = ks, ks+kslice, ... (strided). */
void ref_matvec4_sk(const float *A, const float *B, float *partial, int N, int K, int kslice) {
    const int nchunk = (N + COLCHUNK - 1) / COLCHUNK;
#pragma omp parallel for collapse(2) schedule(static)
    for (int ks = 0; ks < kslice; ++ks) {
        for (int ci = 0; ci < nchunk; ++ci) {
            const int n0 = ci * COLCHUNK;
            const int n1 = n0 + COLCHUNK < N ? n0 + COLCHUNK : N;
            float acc[COLCHUNK];
            for (int n = n0; n < n1; ++n) acc[n - n0] = 0.0f;
            for (int k = ks; k < K; k += kslice) {
                const float a = A[k];
                const float *b = B + (size_t)k * N;
                for (int n = n0; n < n1; ++n) acc[n - n0] += a * b[n];
            }
            float *p = partial + (size_t)ks * N;
            for (int n = n0; n < n1; ++n) p[n] = acc[n - n0];
        }
    }
}

/* math.cl:249-280: s = 0 + p[0] + p[1] + ... then the epilogue. */
void ref_reduce_partial(const float *partial, const float *bias, const float *residual,
                        float *C, int N, int kslice, int apply_gelu) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        float s = 0.0f;
        for (int ks = 0; ks < kslice; ++ks) s += partial[(size_t)ks * N + n];
        C[n] = epi(s, bias, residual, n, apply_gelu);
    }
}

/* launch_matvec (main.c:1554-1576): matvec4 when N % 4 == 0, else scalar. */
void ref_launch_matvec(const float *A, const float *B, const float *bias, const float *residual,
                       float *C, int N, int K, int apply_gelu) {
    if ((N & 3) == 0) ref_matvec4(A, B, bias, residual, C, N, K, apply_gelu);
    else ref_matvec(A, B, bias, residual, C, N, K, apply_gelu);
}

/* launch_matvec_splitk (main.c:1578-1618): falls back to launch_matvec unless
 * 1 < ks <= MAX_KSLICE and N % 4 == 0. */
void ref_launch_matvec_splitk(const float *A, const float *B, const float *bias,
                              const float *residual, float *C, int N, int K, int ks,
                              int apply_gelu, float *partial) {
    if ((N & 3) != 0 || ks <= 1 || ks > REF_MAX_KSLICE) {
        ref_launch_matvec(A, B, bias, residual, C, N, K, apply_gelu);
        return;
    }
    ref_matvec4_sk(A, B, partial, N, K, ks);
    ref_reduce_partial(partial, bias, residual, C, N, ks, apply_gelu);
}

/* math.cl:283-311: one work-item per row, two serial passes. */
void ref_layernorm(const float *x, float *out, const float *gamma, const float *beta, int n_embd,
                   int seq_len) {
#pragma omp parallel for schedule(static)
    for (int s = 0; s < seq_len; ++s) {
        const float *xi = x + (size_t)s * n_embd;
        float *xo = out + (size_t)s * n_embd;
        float mean = 0.0f;
        for (int i = 0; i < n_embd; ++i) mean += xi[i];
        mean /= (float)n_embd;
        float var = 0.0f;
        for (int i = 0; i < n_embd; ++i) {
            float d = xi[i] - mean;
            var += d * d;
        }
        var /= (float)n_embd;
        const float inv_std = 1.0f / sqrtf(var + 1e-5f);
        for (int i = 0; i < n_embd; ++i) xo[i] = (xi[i] - mean) * inv_std * gamma[i] + beta[i];
    }
}

/* math.cl:314-322 */
void ref_add_inplace(float *a, const float *b, int n) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) a[i] += b[i];
}

/* math.cl:325-330 */
void ref_gelu(float *x, int n) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) x[i] = ref_gelu_f(x[i]);
}

/* math.cl:333-350 */
void ref_embed(const float *wte, const float *wpe, float *out, int n_embd, int seq_len,
               int start_pos, const int *ids) {
    for (int i = 0; i < seq_len; ++i) {
        const int pos = start_pos + i, tok = ids[i];
        for (int d = 0; d < n_embd; ++d)
            out[(size_t)i * n_embd + d] = wte[(size_t)tok * n_embd + d] + wpe[(size_t)pos * n_embd + d];
    }
}

/* math.cl:367-383: K transposed [D, max_seq], V row-major [max_seq, D]. */
void ref_split_kv(const float *qkv, float *k_cache, float *v_cache, int start_pos, int T, int D,
                  int max_seq) {
    for (int i = 0; i < T; ++i) {
        const int pos = start_pos + i;
        for (int d = 0; d < D; ++d) {
            k_cache[(size_t)d * max_seq + pos] = qkv[(size_t)i * 3 * D + D + d];
            v_cache[(size_t)pos * D + d] = qkv[(size_t)i * 3 * D + 2 * D + d];
        }
    }
}

/* math.cl:388-412: s = sum_k q[h*DH+k] * K^T[h*DH+k][j], then * scale. */
void ref_attn_scores_1q(const float *qkv, const float *k_cache, float *scores, int q_base,
                        int T_kv, int D, int DH, int NH, int max_seq, float scale) {
    (void)D;
    const float *q = qkv + q_base;
#pragma omp parallel for collapse(2) schedule(static) if (T_kv * NH > 4096)
    for (int h = 0; h < NH; ++h) {
        for (int j = 0; j < T_kv; ++j) {
            const int off = h * DH;
            float s = 0;
            for (int k = 0; k < DH; ++k) s += q[off + k] * k_cache[(size_t)(off + k) * max_seq + j];
            scores[(size_t)h * max_seq + j] = s * scale;
        }
    }
}

/* math.cl:415-456 with lws lanes: lane-strided partial max / exp-sum, tree
 * reductions halving s each step, then row *= 1/sum.  A tree step reads only
 * slots >= s, which that step does not write, so running the lanes of a step
 * in order reproduces the work-group. */
void ref_attn_softmax_1q(float *scores, int T_kv, int NH, int lws) {
#pragma omp parallel for schedule(static) if (NH * T_kv > 4096)
    for (int h = 0; h < NH; ++h) {
        float scratch[256];
        float *row = scores + (size_t)h * REF_MAX_SEQ;
        for (int lid = 0; lid < lws; ++lid) {
            float mx = -1e30f;
            for (int j = lid; j < T_kv; j += lws)
                if (row[j] > mx) mx = row[j];
            scratch[lid] = mx;
        }
        for (int s = lws >> 1; s > 0; s >>= 1)
            for (int lid = 0; lid < s; ++lid) {
                float a = scratch[lid], b = scratch[lid + s];
                scratch[lid] = a > b ? a : b;
            }
        const float m = scratch[0];
        for (int lid = 0; lid < lws; ++lid) {
            float sum = 0;
            for (int j = lid; j < T_kv; j += lws) {
                float e = expf(row[j] - m);
                row[j] = e;
                sum += e;
            }
            scratch[lid] = sum;
        }
        for (int s = lws >> 1; s > 0; s >>= 1)
            for (int lid = 0; lid < s; ++lid) scratch[lid] += scratch[lid + s];
        const float inv = 1.0f / scratch[0];
        for (int j = 0; j < T_kv; ++j) row[j] *= inv;
    }
}

/* math.cl:459-476: out[d] = sum_j p[h(d)][j] * V[j][d], serial in j. */
void ref_attn_out_1q(const float *scores, const float *v_cache, float *out, int T_kv, int D,
                     int DH, int out_base) {
#pragma omp parallel for schedule(static) if (D * T_kv > 65536)
    for (int d = 0; d < D; ++d) {
        const int h = d / DH;
        const float *srow = scores + (size_t)h * REF_MAX_SEQ;
        float s = 0;
        for (int j = 0; j < T_kv; ++j) s += srow[j] * v_cache[(size_t)j * D + d];
        out[out_base + d] = s;
    }
}

/* The runtime-built matmul (main.c:593-684): each C[r][c] accumulates
 * acc += A[r][k] * B[k][c] for k in order (zero-padded k beyond K adds +0),
 * then v = acc + bias[c].  The tile shape does not change this sequence. */
void ref_matmul(const float *A, const float *B, const float *bias, float *C, int M, int N, int K) {
    const int nchunk = (N + COLCHUNK - 1) / COLCHUNK;
#pragma omp parallel for collapse(2) schedule(static)
    for (int r = 0; r < M; ++r) {
        for (int ci = 0; ci < nchunk; ++ci) {
            const int n0 = ci * COLCHUNK;
            const int n1 = n0 + COLCHUNK < N ? n0 + COLCHUNK : N;
            float acc[COLCHUNK];
            for (int n = n0; n < n1; ++n) acc[n - n0] = 0.0f;
            const float *a = A + (size_t)r * K;
            for (int k = 0; k < K; ++k) {
                const float av = a[k];
                const float *b = B + (size_t)k * N;
                for (int n = n0; n < n1; ++n) acc[n - n0] += av * b[n];
            }
            for (int n = n0; n < n1; ++n) {
                float v = acc[n - n0];
                if (bias) v += bias[n];
                C[(size_t)r * N + n] = v;
            }
        }
    }
}

/* ========================================================================
 * Config and safetensors loading (main.c:272-331, 1141-1417)
 * ======================================================================== */

static char *slurp(const char *path, long *len) {
    FILE *fp = fopen(path, "rb");
    if (!fp) return NULL;
    fseek(fp, 0, SEEK_END);
    long n = ftell(fp);
    fseek(fp, 0, SEEK_SET);
    char *b = malloc((size_t)n + 1);
    if (!b) { fclose(fp); return NULL; }
    if (fread(b, 1, (size_t)n, fp) != (size_t)n) { free(b); fclose(fp); return NULL; }
    fclose(fp);
    b[n] = 0;
    if (len) *len = n;
    return b;
}

/* json_get_int_any (main.c:272-287): first '"key"', then ':', then atoi. */
static int json_int(const char *json, const char *const *keys, int nkeys, int defval) {
    for (int i = 0; i < nkeys; ++i) {
        char pat[128];
        snprintf(pat, sizeof pat, "\"%s\"", keys[i]);
        const char *p = strstr(json, pat);
        if (!p) continue;
        p = strchr(p, ':');
        if (!p) continue;
        p++;
        while (*p == ' ' || *p == '\t') p++;
        return atoi(p);
    }
    return defval;
}

int ref_load_config(const char *dir, ref_config *c) {
    char path[1024];
    snprintf(path, sizeof path, "%s/config.json", dir);
    char *json = slurp(path, NULL);
    if (!json) {
        c->n_layer = 12; c->n_embd = 768; c->n_head = 12;
        c->n_ctx = 1024; c->vocab_size = 50257; c->ffn_dim = 3072;
    } else {
        const char *k1[1];
        k1[0] = "n_layer"; c->n_layer = json_int(json, k1, 1, 12);
        k1[0] = "n_embd"; c->n_embd = json_int(json, k1, 1, 768);
        k1[0] = "n_head"; c->n_head = json_int(json, k1, 1, 12);
        const char *ctx_keys[2] = {"n_positions", "n_ctx"};
        c->n_ctx = json_int(json, ctx_keys, 2, 1024);
        k1[0] = "vocab_size"; c->vocab_size = json_int(json, k1, 1, 50257);
        k1[0] = "n_inner";
        int inner = json_int(json, k1, 1, 0);
        c->ffn_dim = inner > 0 ? inner : 4 * c->n_embd;
        free(json);
    }
    if (c->n_layer <= 0 || c->n_embd <= 0 || c->n_head <= 0 || c->vocab_size <= 0 ||
        c->ffn_dim <= 0 || c->n_embd % c->n_head != 0)
        return fail(-3, "config: invalid dimensions");
    if (c->n_ctx > REF_MAX_SEQ || c->n_ctx <= 0) return fail(-3, "config: n_ctx %d exceeds %d", c->n_ctx, REF_MAX_SEQ);
    c->padded_vocab = (c->vocab_size + 3) & ~3;
    return 0;
}

/* --- a small safetensors header reader ------------------------------------ */
enum { DT_F32, DT_F16, DT_BF16, DT_OTHER };
typedef struct {
    char name[160];
    int dtype, ndim;
    int64_t shape[4];
    int64_t begin, end;
} st_tensor;
typedef struct {
    FILE *fp;
    int64_t data_start;
    int n;
    st_tensor *t;
} st_file;

static void skip_ws(const char **p) { while (**p == ' ' || **p == '\n' || **p == '\r' || **p == '\t') (*p)++; }
static int parse_str(const char **p, char *out, int cap) {
    skip_ws(p);
    if (**p != '"') return -1;
    (*p)++;
    int n = 0;
    while (**p && **p != '"') {
        char ch = **p;
        if (ch == '\\') { (*p)++; ch = **p; if (!ch) return -1; }
        if (n + 1 < cap) out[n++] = ch;
        (*p)++;
    }
    if (**p != '"') return -1;
    (*p)++;
    out[n] = 0;
    return n;
}
static int skip_value(const char **p) {
    skip_ws(p);
    char c = **p;
    if (c == '"') { char tmp[8]; return parse_str(p, tmp, sizeof tmp) < 0 ? -1 : 0; }
    if (c == '{' || c == '[') {
        char close = c == '{' ? '}' : ']';
        (*p)++;
        skip_ws(p);
        if (**p == close) { (*p)++; return 0; }
        for (;;) {
            if (c == '{') {
                char tmp[8];
                if (parse_str(p, tmp, sizeof tmp) < 0) return -1;
                skip_ws(p);
                if (**p != ':') return -1;
                (*p)++;
            }
            if (skip_value(p)) return -1;
            skip_ws(p);
            if (**p == ',') { (*p)++; continue; }
            if (**p == close) { (*p)++; return 0; }
            return -1;
        }
    }
    while (**p && **p != ',' && **p != '}' && **p != ']') (*p)++;
    return 0;
}
static int parse_ints(const char **p, int64_t *v, int cap) {
    skip_ws(p);
    if (**p != '[') return -1;
    (*p)++;
    int n = 0;
    skip_ws(p);
    if (**p == ']') { (*p)++; return 0; }
    for (;;) {
        skip_ws(p);
        char *e;
        long long x = strtoll(*p, &e, 10);
        if (e == *p) return -1;
        *p = e;
        if (n < cap) v[n] = x;
        n++;
        skip_ws(p);
        if (**p == ',') { (*p)++; continue; }
        if (**p == ']') { (*p)++; return n; }
        return -1;
    }
}

static int st_open(const char *dir, st_file *f) {
    char path[1024];
    snprintf(path, sizeof path, "%s/model.safetensors", dir);
    memset(f, 0, sizeof *f);
    f->fp = fopen(path, "rb");
    if (!f->fp) return fail(-2, "cannot open %s", path);
    unsigned char lb[8];
    if (fread(lb, 1, 8, f->fp) != 8) return fail(-3, "short header length");
    uint64_t hl = 0;
    for (int i = 7; i >= 0; --i) hl = (hl << 8) | lb[i];
    if (hl > (1u << 30)) return fail(-3, "header length implausible");
    char *h = malloc(hl + 1);
    if (!h) return fail(-5, "oom header");
    if (fread(h, 1, hl, f->fp) != hl) { free(h); return fail(-3, "short header"); }
    h[hl] = 0;
    f->data_start = 8 + (int64_t)hl;
    int cap = 64;
    f->t = malloc(sizeof(st_tensor) * cap);
    const char *p = h;
    skip_ws(&p);
    int rc = 0;
    if (*p != '{') { rc = fail(-3, "header not an object"); goto out; }
    p++;
    for (;;) {
        skip_ws(&p);
        if (*p == '}') break;
        char key[160];
        if (parse_str(&p, key, sizeof key) < 0) { rc = fail(-3, "bad key"); goto out; }
        skip_ws(&p);
        if (*p != ':') { rc = fail(-3, "missing ':'"); goto out; }
        p++;
        if (strcmp(key, "__metadata__") == 0) {
            if (skip_value(&p)) { rc = fail(-3, "bad metadata"); goto out; }
        } else {
            if (f->n == cap) { cap *= 2; f->t = realloc(f->t, sizeof(st_tensor) * cap); }
            st_tensor *t = &f->t[f->n++];
            memset(t, 0, sizeof *t);
            snprintf(t->name, sizeof t->name, "%s", key);
            t->dtype = -1; t->begin = -1;
            skip_ws(&p);
            if (*p != '{') { rc = fail(-3, "tensor entry not an object"); goto out; }
            p++;
            for (;;) {
                skip_ws(&p);
                if (*p == '}') { p++; break; }
                char f2[32];
                if (parse_str(&p, f2, sizeof f2) < 0) { rc = fail(-3, "bad field"); goto out; }
                skip_ws(&p);
                if (*p != ':') { rc = fail(-3, "missing ':'"); goto out; }
                p++;
                if (strcmp(f2, "dtype") == 0) {
                    char dt[16];
                    if (parse_str(&p, dt, sizeof dt) < 0) { rc = fail(-3, "bad dtype"); goto out; }
                    t->dtype = !strcmp(dt, "F32") ? DT_F32 : !strcmp(dt, "F16") ? DT_F16 : !strcmp(dt, "BF16") ? DT_BF16 : DT_OTHER;
                } else if (strcmp(f2, "shape") == 0) {
                    t->ndim = parse_ints(&p, t->shape, 4);
                    if (t->ndim < 0 || t->ndim > 4) { rc = fail(-3, "bad shape"); goto out; }
                } else if (strcmp(f2, "data_offsets") == 0) {
                    int64_t o[2];
                    if (parse_ints(&p, o, 2) != 2) { rc = fail(-3, "bad offsets"); goto out; }
                    t->begin = o[0]; t->end = o[1];
                } else if (skip_value(&p)) { rc = fail(-3, "bad value"); goto out; }
                skip_ws(&p);
                if (*p == ',') p++;
            }
            if (t->dtype < 0 || t->begin < 0 || t->end < t->begin) { rc = fail(-3, "incomplete tensor %s", t->name); goto out; }
        }
        skip_ws(&p);
        if (*p == ',') { p++; continue; }
        if (*p == '}') break;
        rc = fail(-3, "malformed header");
        goto out;
    }
out:
    free(h);
    return rc;
}
static void st_close(st_file *f) {
    if (f->fp) fclose(f->fp);
    free(f->t);
    memset(f, 0, sizeof *f);
}
/* lookup_flexible (main.c:1194-1207): name, "transformer."+name, "model."+name. */
static st_tensor *st_lookup(st_file *f, const char *name) {
    const char *pre[3] = {"", "transformer.", "model."};
    for (int k = 0; k < 3; ++k) {
        char buf[256];
        snprintf(buf, sizeof buf, "%s%s", pre[k], name);
        for (int i = 0; i < f->n; ++i)
            if (strcmp(f->t[i].name, buf) == 0) return &f->t[i];
    }
    return NULL;
}
static int64_t st_numel(const st_tensor *t) {
    int64_t n = 1;
    for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
    return n;
}
static float half_to_float(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0) u = s;
        else {
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; sh++; }
            m &= 0x3ff;
            u = s | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) u = s | 0x7f800000u | (m << 13);
    else u = s | ((e + 112) << 23) | (m << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}
/* Read a tensor as float (F32 as stored; F16/BF16 widened exactly). */
static float *st_read(st_file *f, const st_tensor *t) {
    int64_t n = st_numel(t);
    int es = t->dtype == DT_F32 ? 4 : (t->dtype == DT_F16 || t->dtype == DT_BF16) ? 2 : 0;
    if (!es) { fail(-3, "tensor %s: unsupported dtype", t->name); return NULL; }
    if (t->end - t->begin != n * es) { fail(-3, "tensor %s: size mismatch", t->name); return NULL; }
    float *out = malloc((size_t)n * sizeof(float));
    if (!out) { fail(-5, "oom"); return NULL; }
    if (fseeko(f->fp, (off_t)(f->data_start + t->begin), SEEK_SET) != 0) { free(out); fail(-2, "seek"); return NULL; }
    if (es == 4) {
        if (fread(out, 4, (size_t)n, f->fp) != (size_t)n) { free(out); fail(-2, "short read %s", t->name); return NULL; }
    } else {
        uint16_t *tmp = malloc((size_t)n * 2);
        if (!tmp || fread(tmp, 2, (size_t)n, f->fp) != (size_t)n) { free(tmp); free(out); fail(-2, "short read %s", t->name); return NULL; }
        for (int64_t i = 0; i < n; ++i) {
            if (t->dtype == DT_F16) out[i] = half_to_float(tmp[i]);
            else { uint32_t u = (uint32_t)tmp[i] << 16; memcpy(&out[i], &u, 4); }
        }
        free(tmp);
    }
    return out;
}

struct ref_model {
    ref_config c;
    float *wte, *wpe, *lnf_w, *lnf_b, *lm_head;
    float **ln1_w, **ln1_b, **qkv_w, **qkv_b, **proj_w, **proj_b;
    float **ln2_w, **ln2_b, **fc_w, **fc_b, **fc2_w, **fc2_b;
    int ks_attn_proj, ks_ffn2, attn_lws;
};

static float *load_vec(st_file *f, const char *name, int64_t numel, int *rc) {
    if (*rc) return NULL;
    st_tensor *t = st_lookup(f, name);
    if (!t) { *rc = fail(-3, "tensor '%s' not found", name); return NULL; }
    if (st_numel(t) != numel) { *rc = fail(-3, "tensor '%s': expected %lld elements", name, (long long)numel); return NULL; }
    float *v = st_read(f, t);
    if (!v) *rc = -3;
    return v;
}
/* load_linear_weight (main.c:1252-1300): keep Conv1D [in,out]; transpose Linear [out,in]. */
static float *load_linear(st_file *f, const char *name, int out_dim, int in_dim, int conv1d, int *rc) {
    if (*rc) return NULL;
    st_tensor *t = st_lookup(f, name);
    if (!t) { *rc = fail(-3, "tensor '%s' not found", name); return NULL; }
    if (t->ndim != 2) { *rc = fail(-3, "tensor '%s': not 2-D", name); return NULL; }
    int fr = (int)t->shape[0], fc = (int)t->shape[1];
    if (conv1d ? (fr != in_dim || fc != out_dim) : (fr != out_dim || fc != in_dim)) {
        *rc = fail(-3, "tensor '%s': expected [%d,%d], got [%d,%d]", name, conv1d ? in_dim : out_dim,
                   conv1d ? out_dim : in_dim, fr, fc);
        return NULL;
    }
    float *raw = st_read(f, t);
    if (!raw) { *rc = -3; return NULL; }
    if (conv1d) return raw;
    float *tr = malloc((size_t)out_dim * in_dim * sizeof(float));
    for (int n = 0; n < out_dim; ++n)
        for (int k = 0; k < in_dim; ++k) tr[(size_t)k * out_dim + n] = raw[(size_t)n * in_dim + k];
    free(raw);
    return tr;
}
/* make_padded_lm_head (main.c:1302-1337): [V,E] source -> [E, V_pad], zero columns past V. */
static float *padded_lm_head(const float *src, int K, int V, int Vp) {
    float *o = malloc((size_t)K * Vp * sizeof(float));
    if (!o) return NULL;
    for (int k = 0; k < K; ++k)
        for (int n = 0; n < Vp; ++n) o[(size_t)k * Vp + n] = n < V ? src[(size_t)n * K + k] : 0.0f;
    return o;
}

static float **alloc_ptrs(int n) { return calloc((size_t)n, sizeof(float *)); }

int ref_model_open(const char *dir, ref_model **out) {
    *out = NULL;
    ref_model *m = calloc(1, sizeof *m);
    if (!m) return fail(-5, "oom");
    int rc = ref_load_config(dir, &m->c);
    if (rc) { free(m); return rc; }
    m->ks_attn_proj = 8; m->ks_ffn2 = 8; m->attn_lws = 64;
    st_file f;
    rc = st_open(dir, &f);
    if (rc) { st_close(&f); free(m); return rc; }
    const int L = m->c.n_layer, E = m->c.n_embd, F = m->c.ffn_dim, V = m->c.vocab_size;
    /* detect_weight_layout (main.c:1234-1250) */
    st_tensor *probe = st_lookup(&f, "h.0.attn.c_attn.weight");
    int conv1d = 1;
    if (!probe || probe->ndim != 2) rc = fail(-3, "cannot find h.0.attn.c_attn.weight");
    else if (probe->shape[0] == E && probe->shape[1] == 3 * E) conv1d = 1;
    else if (probe->shape[0] == 3 * E && probe->shape[1] == E) conv1d = 0;
    else rc = fail(-3, "unexpected c_attn shape");
    m->wte = load_vec(&f, "wte.weight", (int64_t)V * E, &rc);
    m->wpe = load_vec(&f, "wpe.weight", (int64_t)m->c.n_ctx * E, &rc);
    m->ln1_w = alloc_ptrs(L); m->ln1_b = alloc_ptrs(L); m->qkv_w = alloc_ptrs(L); m->qkv_b = alloc_ptrs(L);
    m->proj_w = alloc_ptrs(L); m->proj_b = alloc_ptrs(L); m->ln2_w = alloc_ptrs(L); m->ln2_b = alloc_ptrs(L);
    m->fc_w = alloc_ptrs(L); m->fc_b = alloc_ptrs(L); m->fc2_w = alloc_ptrs(L); m->fc2_b = alloc_ptrs(L);
    for (int l = 0; l < L && !rc; ++l) {
        char n[256];
#define NM(s) (snprintf(n, sizeof n, "h.%d.%s", l, s), n)
        m->ln1_w[l] = load_vec(&f, NM("ln_1.weight"), E, &rc);
        m->ln1_b[l] = load_vec(&f, NM("ln_1.bias"), E, &rc);
        m->qkv_w[l] = load_linear(&f, NM("attn.c_attn.weight"), 3 * E, E, conv1d, &rc);
        m->qkv_b[l] = load_vec(&f, NM("attn.c_attn.bias"), 3 * E, &rc);
        m->proj_w[l] = load_linear(&f, NM("attn.c_proj.weight"), E, E, conv1d, &rc);
        m->proj_b[l] = load_vec(&f, NM("attn.c_proj.bias"), E, &rc);
        m->ln2_w[l] = load_vec(&f, NM("ln_2.weight"), E, &rc);
        m->ln2_b[l] = load_vec(&f, NM("ln_2.bias"), E, &rc);
        m->fc_w[l] = load_linear(&f, NM("mlp.c_fc.weight"), F, E, conv1d, &rc);
        m->fc_b[l] = load_vec(&f, NM("mlp.c_fc.bias"), F, &rc);
        m->fc2_w[l] = load_linear(&f, NM("mlp.c_proj.weight"), E, F, conv1d, &rc);
        m->fc2_b[l] = load_vec(&f, NM("mlp.c_proj.bias"), E, &rc);
#undef NM
    }
    m->lnf_w = load_vec(&f, "ln_f.weight", E, &rc);
    m->lnf_b = load_vec(&f, "ln_f.bias", E, &rc);
    if (!rc) {
        /* tied or separate lm_head (main.c:1374-1414) */
        st_tensor *lt = st_lookup(&f, "lm_head.weight");
        if (!lt) m->lm_head = padded_lm_head(m->wte, E, V, m->c.padded_vocab);
        else {
            float *src = st_read(&f, lt);
            if (!src) rc = -3;
            else if (lt->ndim == 2 && lt->shape[0] == V && lt->shape[1] == E)
                m->lm_head = padded_lm_head(src, E, V, m->c.padded_vocab);
            else if (lt->ndim == 2 && lt->shape[0] == E && lt->shape[1] == V) {
                float *tmp = malloc((size_t)V * E * sizeof(float));
                for (int v = 0; v < V; ++v)
                    for (int k = 0; k < E; ++k) tmp[(size_t)v * E + k] = src[(size_t)k * V + v];
                m->lm_head = padded_lm_head(tmp, E, V, m->c.padded_vocab);
                free(tmp);
            } else rc = fail(-3, "lm_head.weight: unexpected shape");
            free(src);
        }
        if (!rc && !m->lm_head) rc = fail(-5, "oom lm_head");
    }
    st_close(&f);
    if (rc) { ref_model_close(m); return rc; }
    *out = m;
    return 0;
}

void ref_model_close(ref_model *m) {
    if (!m) return;
    free(m->wte); free(m->wpe); free(m->lnf_w); free(m->lnf_b); free(m->lm_head);
    float **arrs[12] = {m->ln1_w, m->ln1_b, m->qkv_w, m->qkv_b, m->proj_w, m->proj_b,
                        m->ln2_w, m->ln2_b, m->fc_w, m->fc_b, m->fc2_w, m->fc2_b};
    for (int a = 0; a < 12; ++a) {
        if (!arrs[a]) continue;
        for (int l = 0; l < m->c.n_layer; ++l) free(arrs[a][l]);
        free(arrs[a]);
    }
    free(m);
}

void ref_model_get_config(const ref_model *m, ref_config *out) { *out = m->c; }
void ref_model_set_tuning(ref_model *m, int ks_attn_proj, int ks_ffn2, int attn_lws) {
    m->ks_attn_proj = ks_attn_proj;
    m->ks_ffn2 = ks_ffn2;
    m->attn_lws = attn_lws;
}
const float *ref_model_lm_head(const ref_model *m) { return m->lm_head; }

/* ========================================================================
 * Sequence state and the forward passes (main.c:1451-1490, 1739-1833)
 * ======================================================================== */

struct ref_seq {
    const ref_model *m;
    float *hidden, *ln_out, *attn, *attn_proj, *ffn1, *ffn2, *qkv_new, *qkv_full;
    float *last_hidden, *logits, *partial, *scores;
    float **k_cache, **v_cache;
};

int ref_seq_new(const ref_model *m, ref_seq **out) {
    const size_t E = m->c.n_embd, F = m->c.ffn_dim, T = 3 * E, S = REF_MAX_SEQ,
                 V = m->c.padded_vocab, NH = m->c.n_head;
    ref_seq *s = calloc(1, sizeof *s);
    s->m = m;
    s->hidden = calloc(S * E, 4); s->ln_out = calloc(S * E, 4); s->attn = calloc(S * E, 4);
    s->attn_proj = calloc(S * E, 4); s->ffn1 = calloc(S * F, 4); s->ffn2 = calloc(S * E, 4);
    s->qkv_new = calloc(T, 4); s->qkv_full = calloc(S * T, 4); s->last_hidden = calloc(E, 4);
    s->logits = calloc(V, 4);
    size_t pn = (size_t)REF_MAX_KSLICE * (V > F ? V : F);
    s->partial = calloc(pn, 4);
    s->scores = calloc(NH * S, 4);
    s->k_cache = calloc(m->c.n_layer, sizeof(float *));
    s->v_cache = calloc(m->c.n_layer, sizeof(float *));
    int ok = s->hidden && s->ln_out && s->attn && s->attn_proj && s->ffn1 && s->ffn2 && s->qkv_new &&
             s->qkv_full && s->last_hidden && s->logits && s->partial && s->scores;
    for (int l = 0; l < m->c.n_layer && ok; ++l) {
        s->k_cache[l] = calloc(E * S, 4);
        s->v_cache[l] = calloc(S * E, 4);
        ok = s->k_cache[l] && s->v_cache[l];
    }
    if (!ok) { ref_seq_free(s); *out = NULL; return fail(-5, "oom sequence buffers"); }
    *out = s;
    return 0;
}

void ref_seq_free(ref_seq *s) {
    if (!s) return;
    free(s->hidden); free(s->ln_out); free(s->attn); free(s->attn_proj); free(s->ffn1); free(s->ffn2);
    free(s->qkv_new); free(s->qkv_full); free(s->last_hidden); free(s->logits); free(s->partial); free(s->scores);
    for (int l = 0; s->k_cache && l < s->m->c.n_layer; ++l) { free(s->k_cache[l]); free(s->v_cache[l]); }
    free(s->k_cache); free(s->v_cache);
    free(s);
}

const float *ref_seq_logits(const ref_seq *s) { return s->logits; }
const float *ref_seq_hidden(const ref_seq *s) { return s->hidden; }
const float *ref_seq_kcache(const ref_seq *s, int l) { return s->k_cache[l]; }
const float *ref_seq_vcache(const ref_seq *s, int l) { return s->v_cache[l]; }

static void attention_1q(ref_seq *s, int l, const float *qkv, int q_base, int T_kv, float *out, int out_base) {
    const ref_config *c = &s->m->c;
    const int E = c->n_embd, DH = E / c->n_head;
    const float scale = 1.0f / sqrtf((float)DH);   /* main.c:1692 */
    ref_attn_scores_1q(qkv, s->k_cache[l], s->scores, q_base, T_kv, E, DH, c->n_head, REF_MAX_SEQ, scale);
    ref_attn_softmax_1q(s->scores, T_kv, c->n_head, s->m->attn_lws);
    ref_attn_out_1q(s->scores, s->v_cache[l], out, T_kv, E, DH, out_base);
}

/* main.c:1739-1790 */
int ref_prefill(ref_seq *s, const int *ids, int n) {
    const ref_model *m = s->m;
    const ref_config *c = &m->c;
    const int E = c->n_embd, T = 3 * E, F = c->ffn_dim;
    if (n <= 0 || n > c->n_ctx) return fail(-6, "prompt length %d out of range", n);
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= c->vocab_size) return fail(-6, "token id %d out of range", ids[i]);
    ref_embed(m->wte, m->wpe, s->hidden, E, n, 0, ids);
    for (int l = 0; l < c->n_layer; ++l) {
        ref_layernorm(s->hidden, s->ln_out, m->ln1_w[l], m->ln1_b[l], E, n);
        ref_matmul(s->ln_out, m->qkv_w[l], m->qkv_b[l], s->qkv_full, n, T, E);
        ref_split_kv(s->qkv_full, s->k_cache[l], s->v_cache[l], 0, n, E, REF_MAX_SEQ);
        for (int i = 0; i < n; ++i) attention_1q(s, l, s->qkv_full, i * 3 * E, i + 1, s->attn, i * E);
        ref_matmul(s->attn, m->proj_w[l], m->proj_b[l], s->attn_proj, n, E, E);
        ref_add_inplace(s->hidden, s->attn_proj, n * E);
        ref_layernorm(s->hidden, s->ln_out, m->ln2_w[l], m->ln2_b[l], E, n);
        ref_matmul(s->ln_out, m->fc_w[l], m->fc_b[l], s->ffn1, n, F, E);
        ref_gelu(s->ffn1, n * F);
        ref_matmul(s->ffn1, m->fc2_w[l], m->fc2_b[l], s->ffn2, n, E, F);
        ref_add_inplace(s->hidden, s->ffn2, n * E);
    }
    ref_layernorm(s->hidden, s->ln_out, m->lnf_w, m->lnf_b, E, n);
    memcpy(s->last_hidden, s->ln_out + (size_t)(n - 1) * E, (size_t)E * 4);
    ref_launch_matvec(s->last_hidden, m->lm_head, NULL, NULL, s->logits, c->padded_vocab, E, 0);
    return 0;
}

/* main.c:1792-1833 */
int ref_decode(ref_seq *s, int tok, int pos) {
    const ref_model *m = s->m;
    const ref_config *c = &m->c;
    const int E = c->n_embd, T = 3 * E, F = c->ffn_dim;
    if (tok < 0 || tok >= c->vocab_size) return fail(-6, "token id %d out of range", tok);
    if (pos < 0 || pos >= c->n_ctx) return fail(-6, "position %d out of range", pos);
    ref_embed(m->wte, m->wpe, s->hidden, E, 1, pos, &tok);
    for (int l = 0; l < c->n_layer; ++l) {
        ref_layernorm(s->hidden, s->ln_out, m->ln1_w[l], m->ln1_b[l], E, 1);
        ref_launch_matvec(s->ln_out, m->qkv_w[l], m->qkv_b[l], NULL, s->qkv_new, T, E, 0);
        ref_split_kv(s->qkv_new, s->k_cache[l], s->v_cache[l], pos, 1, E, REF_MAX_SEQ);
        attention_1q(s, l, s->qkv_new, 0, pos + 1, s->attn, 0);
        ref_launch_matvec_splitk(s->attn, m->proj_w[l], m->proj_b[l], s->hidden, s->hidden, E, E,
                                 m->ks_attn_proj, 0, s->partial);
        ref_layernorm(s->hidden, s->ln_out, m->ln2_w[l], m->ln2_b[l], E, 1);
        ref_launch_matvec(s->ln_out, m->fc_w[l], m->fc_b[l], NULL, s->ffn1, F, E, 1);
        ref_launch_matvec_splitk(s->ffn1, m->fc2_w[l], m->fc2_b[l], s->hidden, s->hidden, E, F,
                                 m->ks_ffn2, 0, s->partial);
    }
    ref_layernorm(s->hidden, s->ln_out, m->lnf_w, m->lnf_b, E, 1);
    ref_launch_matvec(s->ln_out, m->lm_head, NULL, NULL, s->logits, c->padded_vocab, E, 0);
    return 0;
}

/* ========================================================================
 * Sampler (main.c:1839-1939)
 * ======================================================================== */

/* main.c:1839-1868: min-heap of the k largest, returns its root. */
float ref_kth_largest(const float *a, int n, int k) {
    float heap[REF_MAX_TOPK];
    int hn = 0;
    for (int i = 0; i < n; ++i) {
        const float v = a[i];
        if (hn < k) {
            int j = hn++;
            heap[j] = v;
            while (j > 0) {
                const int p = (j - 1) >> 1;
                if (heap[p] <= heap[j]) break;
                const float t = heap[p]; heap[p] = heap[j]; heap[j] = t;
                j = p;
            }
        } else if (v > heap[0]) {
            heap[0] = v;
            int j = 0;
            for (;;) {
                const int l = 2 * j + 1, r = 2 * j + 2;
                int mm = j;
                if (l < k && heap[l] < heap[mm]) mm = l;
                if (r < k && heap[r] < heap[mm]) mm = r;
                if (mm == j) break;
                const float t = heap[j]; heap[j] = heap[mm]; heap[mm] = t;
                j = mm;
            }
        }
    }
    return heap[0];
}

void ref_srand(unsigned seed) { srand(seed); }

/* main.c:1872-1939 on a private copy of the logits. */
int ref_sample_next_token(const float *logits_in, int V, const int *ctx, int n_ctx, int forbid_eos,
                          float temperature, int top_k, float rep_penalty) {
    float *logits = malloc((size_t)V * sizeof(float));
    if (!logits) return fail(-5, "oom");
    memcpy(logits, logits_in, (size_t)V * sizeof(float));
    if (forbid_eos && REF_EOS < V) logits[REF_EOS] = -1e30f;
    if (rep_penalty > 1.0f) {
        for (int i = 0; i < n_ctx; ++i) {
            const int tk = ctx[i];
            if (tk < 0 || tk >= V) continue;
            int dup = 0;
            for (int j = 0; j < i; ++j)
                if (ctx[j] == tk) { dup = 1; break; }
            if (dup) continue;
            if (logits[tk] > 0.0f) logits[tk] /= rep_penalty;
            else logits[tk] *= rep_penalty;
        }
    }
    int chosen;
    if (temperature <= 0.0f) {
        int best = 0;
        float bv = logits[0];
        for (int i = 1; i < V; ++i)
            if (logits[i] > bv) { bv = logits[i]; best = i; }
        chosen = best;
    } else {
        const float inv_T = 1.0f / temperature;
        for (int i = 0; i < V; ++i) logits[i] *= inv_T;
        int k = top_k;
        if (k <= 0 || k > V) k = V;
        if (k > REF_MAX_TOPK) k = REF_MAX_TOPK;
        if (k < V) {
            const float thresh = ref_kth_largest(logits, V, k);
            for (int i = 0; i < V; ++i)
                if (logits[i] < thresh) logits[i] = -1e30f;
        }
        float max_v = -1e30f;
        for (int i = 0; i < V; ++i)
            if (logits[i] > max_v) max_v = logits[i];
        double sum = 0.0;
        for (int i = 0; i < V; ++i) {
            if (logits[i] <= -1e29f) { logits[i] = 0.0f; continue; }
            const float e = expf(logits[i] - max_v);
            logits[i] = e;
            sum += e;
        }
        const double r = ((double)rand() / ((double)RAND_MAX + 1.0)) * sum;
        double acc = 0.0;
        chosen = V - 1;
        for (int i = 0; i < V; ++i) {
            acc += logits[i];
            if (acc >= r) { chosen = i; break; }
        }
    }
    free(logits);
    return chosen;
}

/* The generation loop of main.c:2106-2150 without text output. */
int ref_generate(ref_seq *s, const int *prompt, int prompt_len, int max_new, int min_new,
                 float temperature, int top_k, float rep_penalty, int *out) {
    const int V = s->m->c.vocab_size;
    if (prompt_len <= 0 || prompt_len >= REF_MAX_SEQ) return fail(-6, "prompt length");
    int *ids = malloc(sizeof(int) * REF_MAX_SEQ);
    memcpy(ids, prompt, sizeof(int) * (size_t)prompt_len);
    int seq_len = prompt_len, n = 0;
    int rc = ref_prefill(s, ids, seq_len);
    if (rc) { free(ids); return rc; }
    int next = ref_sample_next_token(s->logits, V, ids, seq_len, 0 < min_new, temperature, top_k, rep_penalty);
    ids[seq_len++] = next;
    out[n++] = next;
    int generated = 1;
    while (generated < max_new && next != REF_EOS && seq_len < REF_MAX_SEQ) {
        rc = ref_decode(s, ids[seq_len - 1], seq_len - 1);
        if (rc) { free(ids); return rc; }
        next = ref_sample_next_token(s->logits, V, ids, seq_len, generated < min_new, temperature, top_k,
                                     rep_penalty);
        ids[seq_len++] = next;
        generated++;
        out[n++] = next;
        if (next == REF_EOS) break;
    }
    free(ids);
    return n;
}
