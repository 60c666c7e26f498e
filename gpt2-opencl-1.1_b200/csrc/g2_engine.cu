// g2_engine.cu -- the C ABI (include/gpt2b200.h): model loading, KV caches,
// prefill / decode orchestration, CUDA-graph decode steps, device greedy loop.
//
// Orchestration follows the reference's prefill() and decode()
// (main.c:1739-1833), with its 147 launches per decoded token replaced by
// 2 + 5 * n_layer fused kernels captured once in a CUDA graph; the token and
// position live in device memory (StepState) so one graph serves every step,
// and greedy generation runs with no host round trip per token.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <map>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "g2_internal.h"
#include "g2_loader.h"
#include "g2_mega.h"
#include "g2_tc.h"
#include "gpt2b200.h"

using namespace g2;

// NVTX range over an entry point (prefill, decode, sampling, generation), for
// profiler timelines; header-only NVTX, a no-op unless a tool is attached.
namespace {
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
};
}  // namespace

// ------------------------------------------------------------------------------
// errors
// ------------------------------------------------------------------------------
static thread_local std::string t_err;

static int set_err(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    return code;
}

extern "C" const char *g2_last_error(void) { return t_err.c_str(); }

namespace g2 {
int set_error(int code, const char *msg) { return set_err(code, "%s", msg); }
}  // namespace g2

#define CK(call)                                                                                              \
    do {                                                                                                      \
        cudaError_t e_ = (call);                                                                              \
        if (e_ != cudaSuccess)                                                                                \
            return set_err(e_ == cudaErrorMemoryAllocation ? G2_ERR_OOM : G2_ERR_CUDA, "%s: %s (%s:%d)", #call, \
                           cudaGetErrorString(e_), __FILE__, __LINE__);                                       \
    } while (0)
#define CKL()                                                                                        \
    do {                                                                                             \
        cudaError_t e_ = cudaGetLastError();                                                         \
        if (e_ != cudaSuccess)                                                                       \
            return set_err(G2_ERR_CUDA, "kernel launch: %s (%s:%d)", cudaGetErrorString(e_), __FILE__, \
                           __LINE__);                                                                \
    } while (0)

// ------------------------------------------------------------------------------
// engine state
// ------------------------------------------------------------------------------
struct LayerOff {
    size_t ln1_g, ln1_b, qkv_w, qkv_b, proj_w, proj_b, ln2_g, ln2_b, fc_w, fc_b, fc2_w, fc2_b;
};

struct g2_engine {
    int device = 0, dtype = G2_F32, max_batch = 1, sms = 148;
    ModelConfig c;
    cudaStream_t st = nullptr;
    // weights: one allocation, element offsets per tensor
    void *wbuf = nullptr;
    size_t welem = 0, esize = 4;
    size_t wte = 0, wpe = 0, lnf_g = 0, lnf_b = 0, lm = 0;
    std::vector<LayerOff> L;
    size_t stream_bytes = 0, device_bytes = 0;
    // KV caches
    void *kbuf = nullptr, *vbuf = nullptr;
    KVLayout kv{};
    // fp16 caches as 2-D tensors ([rows][64], one row per (slot, layer, head,
    // position)) for the batched attention's swizzled TMA loads
    CUtensorMap kv_kmap{}, kv_vmap{};
    bool kv_maps = false;
    // workspaces
    int R = 0;   // rows capacity
    float *h = nullptr, *xln = nullptr, *qkv = nullptr, *attn = nullptr, *ffn = nullptr;
    float *logits = nullptr, *logits_rows = nullptr;
    float *gemv_partial = nullptr, *attn_partial = nullptr, *lm_partial = nullptr;
    unsigned *gemv_ctr = nullptr, *attn_ctr = nullptr, *lm_ctr = nullptr;
    size_t gemv_ctr_n = 0, attn_ctr_n = 0;   // counters in each array (zeroed again after an expired wait)
    int *rows_tok = nullptr, *rows_pos = nullptr, *rows_slot = nullptr;
    int *result = nullptr, *argmax_out = nullptr, *batch_step = nullptr, *out_tokens = nullptr;
    StepState *state = nullptr;
    // pinned staging
    int *h_rows = nullptr;          // [3][R]
    StepState *h_state = nullptr;   // ring
    int h_state_i = 0;
    int *h_small = nullptr;         // results; its last two ints receive the error words (sync_and_check)
    cudaEvent_t staged = nullptr;
    GemvPlan plan_qkv{}, plan_proj{}, plan_fc{}, plan_fc2{};
    std::vector<int> filled;        // positions present in each slot's cache
    int result_slot = -1;           // slot whose lm_head argmax is in `result`
    // graphs
    std::vector<cudaGraphExec_t> dec_graph;
    int dec_graph_kernels = 0;
    cudaGraphExec_t batch_graph = nullptr;
    // prefill graphs by prompt length: a length is run eagerly on first use and
    // captured on the second (G2_NO_PREFILL_GRAPH=1 keeps it eager)
    struct PrefillGraph {
        cudaGraphExec_t exec = nullptr;
        long long kernels = 0;
        int uses = 0;
    };
    std::map<int, PrefillGraph> prefill_graphs;
    bool prefill_graph_on = true;
    int batch_graph_n = 0, batch_graph_kernels = 0;
    // Largest position a captured batch step may reach: it sizes the attention grid
    // (128-key chunks per row), so the graph is re-captured when a generation needs more.
    int batch_graph_pos = -1, batch_pos_hint = -1;
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    float last_prefill_ms = 0, last_decode_ms = 0;
    int last_decode_steps = 0;
    long long launches = 0;
    // persistent B = 1 decode kernel (fp32)
    bool mega = false;
    float *packed = nullptr;            // unit-packed projection weights
    std::vector<long long> layer_off;   // [L][3] float offsets into packed (A, B, D units)
    long long *d_layer_off = nullptr;
    LayerPtrs *d_layers = nullptr;
    unsigned long long *t_qkv = nullptr, *t_best = nullptr, *t_att = nullptr;
    int mega_split_t = 320;   // positions past which a head's keys are split over its units (G2_MEGA_SPLIT_T)
    unsigned long long *mega_acc = nullptr;   // mega_acc_words(kMegaMaxSteps, L, E) accumulator words
    int *d_err = nullptr;
    unsigned long long *d_trace = nullptr;   // phase trace, when G2_MEGA_TRACE names an output file
    std::string trace_path;
    unsigned mega_epoch = 0;
    // Limit of every device-side wait (G2_WAIT_LIMIT_MS overrides the 2 s default;
    // tests shorten it to exercise the expiry path quickly).
    unsigned long long wait_ns = kMegaTimeoutNs;
    // Test hook (G2_TEST_STALL=acc at open): the next persistent launch gets one
    // accumulator word that can never turn ready, so its waits expire; one-shot.
    int test_stall = 0;
    int mega_inflight = 3;   // outstanding bulk copies per CTA (G2_MEGA_INFLIGHT overrides)
    int mega_grid = 0;
    int mega_cw[2] = {0, 0};   // strip widths of c_attn and c_fc
    int mega_nq = 0;           // attn.c_proj column slices per head
    bool lnf_done = false;     // the last many-row pass wrote the ln_f operand of its rows
    size_t mega_smem = 0;
    // tensor-core GEMMs of the many-row passes (prefill, batched decode)
    bool tc = false;
    int tc_kind = TC_TF32X3;
    float *tc_xhi = nullptr, *tc_xlo = nullptr;     // GEMM input rows with K = E: hi / lo (fp32) or fp16 (in tc_xhi)
    float *tc_x2hi = nullptr, *tc_x2lo = nullptr;   // fc2's input rows (K = F), written by the fc GEMM
    unsigned *tc_ctr = nullptr;                    // split-K tile counters
    float *tc_part = nullptr;                 // split-K partial sums
    float *tc_w = nullptr;                    // fp32 engine without wsplit: tf32 hi / lo copies of the projections
    float *tc_lm_w = nullptr;                 // fp32 engine without wsplit: tf32 hi / lo copies of wte
    void *tc_img = nullptr;                   // stage images of the projections (TcWeights::img_hi / img_lo)
    void *tc_idx = nullptr;                   // 16 KB: the coordinate tensor of tc_stage_perm
    unsigned *tc_perm = nullptr;              // stage element positions (tc_stage_perm)
    size_t tc_part_floats = 0;
    int *tc_err = nullptr;
    // device sampler
    float *sample_work = nullptr;   // [padded_vocab]
    int *sample_ctx = nullptr;      // [n_ctx] context ids
    int *topk_out = nullptr;        // g2_topk: [G2_MAX_TOPK] values (as float) then [G2_MAX_TOPK] ids
    int *h_ctx = nullptr;           // pinned staging of the context ids
    std::vector<TcWeights> tc_maps;           // [L][4]: qkv, proj, fc, fc2
    TcWeights tc_lm{};                        // the tied LM head: wte [V][E] as a K-major operand
    // LM head over one range of vocabulary rows (g2_lm_head_rows): its operand map and logits
    TcWeights tc_lm_shard{};
    int shard_v0 = -1, shard_v1 = -1;
    float *shard_logits = nullptr;            // [rows][stride] of the last g2_lm_head_rows
    size_t shard_cap = 0;                     // floats shard_logits holds
    TcRowsOperand tc_x_e{}, tc_x_f{};         // input rows with K = E (tc_x*) and K = F (tc_x2*)

    template <typename WT>
    const WT *w(size_t off) const {
        return reinterpret_cast<const WT *>(wbuf) + off;
    }
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static uint16_t f2h_bits(float f) {
    __half h = __float2half_rn(f);
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

// ------------------------------------------------------------------------------
// open / close
// ------------------------------------------------------------------------------
static void free_engine(g2_engine *e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->st) cudaStreamSynchronize(e->st);
    for (auto g : e->dec_graph)
        if (g) cudaGraphExecDestroy(g);
    if (e->batch_graph) cudaGraphExecDestroy(e->batch_graph);
    for (auto &kv : e->prefill_graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    void *dev_ptrs[] = {e->shard_logits, e->sample_work, e->sample_ctx, e->topk_out, e->tc_w, e->tc_lm_w, e->tc_img, e->tc_idx, e->tc_perm, e->tc_xhi, e->tc_xlo, e->tc_x2hi, e->tc_x2lo, e->tc_ctr, e->tc_part, e->tc_err, e->d_trace, e->packed, e->d_layer_off, e->d_layers, e->t_qkv, e->mega_acc,
                        e->t_best, e->t_att, e->d_err, e->wbuf, e->kbuf, e->vbuf, e->h, e->xln, e->qkv, e->attn, e->ffn, e->logits,
                        e->logits_rows, e->gemv_partial, e->attn_partial, e->lm_partial, e->gemv_ctr,
                        e->attn_ctr, e->lm_ctr, e->rows_tok, e->rows_pos, e->rows_slot, e->result,
                        e->argmax_out, e->batch_step, e->out_tokens, e->state};
    for (void *p : dev_ptrs)
        if (p) cudaFree(p);
    if (e->h_rows) cudaFreeHost(e->h_rows);
    if (e->h_state) cudaFreeHost(e->h_state);
    if (e->h_small) cudaFreeHost(e->h_small);
    if (e->h_ctx) cudaFreeHost(e->h_ctx);
    if (e->staged) cudaEventDestroy(e->staged);
    for (auto &ev : e->ev)
        if (ev) cudaEventDestroy(ev);
    if (e->st) cudaStreamDestroy(e->st);
    delete e;
}

template <typename T>
static int dalloc(g2_engine *e, T **p, size_t count) {
    const size_t bytes = align_up(count * sizeof(T), 256);
    cudaError_t r = cudaMalloc((void **)p, bytes);
    if (r != cudaSuccess)
        return set_err(G2_ERR_OOM, "cudaMalloc(%zu bytes): %s", bytes, cudaGetErrorString(r));
    e->device_bytes += bytes;
    // The zeroing runs on the legacy default stream, which the engine's
    // non-blocking stream does not wait for: it must be complete before the
    // caller hands the buffer to that stream, or it could land after the
    // stream's first writes.
    r = cudaMemset(*p, 0, bytes);
    if (r == cudaSuccess) r = cudaDeviceSynchronize();
    if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "cudaMemset: %s", cudaGetErrorString(r));
    return G2_OK;
}

// Element (k, n) of a projection W with K inputs and N outputs, stored either
// Conv1D [K][N] (lin false) or nn.Linear [N][K] (lin true).
static inline float w_at(const float *W, int K, int N, bool lin, int k, int n) {
    return lin ? W[(size_t)n * K + k] : W[(size_t)k * N + n];
}

// One projection W (K inputs, N outputs) packed for the persistent decode
// kernel: unit u (columns u*CW .. u*CW + CW - 1) is (K + 2) rows x CW, rows
// k < K holding g[k] * W[k][n], row K holding b[n] + sum_k beta[k] * W[k][n]
// and row K + 1 the column sums of the stored rows.  With g and beta the
// preceding LayerNorm's parameters this folds the LayerNorm's affine part into
// the projection: (norm(x) * g + beta) W + b = norm(x) (diag(g) W) +
// (beta W + b).  Without a LayerNorm (g = beta = nullptr) the rows are W and b.
static void pack_strips(const float *W, bool lin, const float *b, const float *g, const float *beta, int K, int N,
                        int CW, float *out) {
    for (int u = 0; u < N / CW; ++u) {
        float *o = out + (size_t)u * (K + 2) * CW;
        for (int k = 0; k < K; ++k) {
            const float gk = g ? g[k] : 1.0f;
            for (int cc = 0; cc < CW; ++cc) o[(size_t)k * CW + cc] = gk * w_at(W, K, N, lin, k, u * CW + cc);
        }
        for (int cc = 0; cc < CW; ++cc) {
            const int n = u * CW + cc;
            double acc = b[n], cs = 0.0;
            if (beta)
                for (int k = 0; k < K; ++k) acc += (double)beta[k] * (double)w_at(W, K, N, lin, k, n);
            if (g)   // sums of the stored (rounded) W' column: x W' - mean * sum_k W'[k] = (x - mean) W'
                for (int k = 0; k < K; ++k) cs += (double)o[(size_t)k * CW + cc];
            o[(size_t)K * CW + cc] = (float)acc;
            o[(size_t)(K + 1) * CW + cc] = (float)cs;
        }
    }
}

// Units of one layer for the persistent decode kernel, part q (0: A, 1: B,
// 2: D; layout in g2_mega.h).  T holds the layer's twelve tensors in file
// order: ln_1.w/b, c_attn.w/b, attn.c_proj.w/b, ln_2.w/b, c_fc.w/b,
// mlp.c_proj.w/b, the projections as stored in the file (Conv1D [in][out],
// or nn.Linear [out][in] when lin).  The projection biases of B and D are
// not packed: the kernel adds them when it reads the accumulators.
static void pack_mega_layer(const std::vector<float> *T, bool lin, int E, int F, int NH, int cwq, int cwf, int nq,
                            int q, std::vector<float> &out) {
    if (q == 0) {
        out.resize((size_t)mega_packed_a(E));
        pack_strips(T[2].data(), lin, T[3].data(), T[0].data(), T[1].data(), E, 3 * E, cwq, out.data());
    } else if (q == 1) {
        out.resize((size_t)mega_packed_b(E));
        const int NB = E / nq;
        const float *W = T[4].data();   // E x E
        float *o = out.data();
        for (int h = 0; h < NH; ++h)
            for (int j = 0; j < nq; ++j)
                for (int d = 0; d < 64; ++d)
                    for (int n = 0; n < NB; ++n) *o++ = w_at(W, E, E, lin, h * 64 + d, j * NB + n);
    } else {
        out.resize((size_t)mega_packed_d(E, F));
        std::vector<float> strips((size_t)(E + 2) * F);
        pack_strips(T[8].data(), lin, T[9].data(), T[6].data(), T[7].data(), E, F, cwf, strips.data());
        const float *W2 = T[10].data();   // F inputs x E outputs
        float *o = out.data();
        for (int u = 0; u < F / cwf; ++u) {
            const float *st = strips.data() + (size_t)u * (E + 2) * cwf;
            o = std::copy(st, st + (size_t)(E + 2) * cwf, o);
            for (int f = u * cwf; f < (u + 1) * cwf; ++f)
                for (int n = 0; n < E; ++n) *o++ = w_at(W2, F, E, lin, f, n);
        }
    }
}

// Load every tensor into one device buffer, converted to the engine dtype.
static int load_weights(g2_engine *e, const std::string &dir) {
    std::string err;
    SafeTensors sf;
    int rc = sf.open(dir + "/model.safetensors", err);
    if (rc) return set_err(rc, "%s", err.c_str());
    const ModelConfig &c = e->c;
    const int E = c.n_embd, F = c.ffn_dim, V = c.vocab_size;
    // detect_weight_layout (main.c:1234-1250)
    const StTensor *probe = sf.find("h.0.attn.c_attn.weight");
    if (!probe || probe->shape.size() != 2) return set_err(G2_ERR_FORMAT, "cannot find h.0.attn.c_attn.weight");
    bool conv1d;
    if (probe->shape[0] == E && probe->shape[1] == 3 * E) conv1d = true;
    else if (probe->shape[0] == 3 * E && probe->shape[1] == E) conv1d = false;
    else return set_err(G2_ERR_FORMAT, "h.0.attn.c_attn.weight: unexpected shape [%lld,%lld]",
                        (long long)probe->shape[0], (long long)probe->shape[1]);
    const StTensor *lmt = sf.find("lm_head.weight");

    // layout plan
    struct Item {
        std::string name;
        size_t *off;
        int rows, cols;      // as stored on the device: [rows][cols]
        int kind;            // 0 vector/plain, 1 linear weight [in][out], 2 lm_head
        int layer, ph;       // linear weights: layer and phase (0 qkv, 1 proj, 2 fc, 3 fc2)
    };
    std::vector<Item> items;
    e->L.resize(c.n_layer);
    items.push_back({"wte.weight", &e->wte, V, E, 0});
    items.push_back({"wpe.weight", &e->wpe, c.n_ctx, E, 0});
    for (int l = 0; l < c.n_layer; ++l) {
        LayerOff &o = e->L[l];
        const std::string p = "h." + std::to_string(l) + ".";
        items.push_back({p + "ln_1.weight", &o.ln1_g, 1, E, 0});
        items.push_back({p + "ln_1.bias", &o.ln1_b, 1, E, 0});
        items.push_back({p + "attn.c_attn.weight", &o.qkv_w, E, 3 * E, 1, l, 0});
        items.push_back({p + "attn.c_attn.bias", &o.qkv_b, 1, 3 * E, 0});
        items.push_back({p + "attn.c_proj.weight", &o.proj_w, E, E, 1, l, 1});
        items.push_back({p + "attn.c_proj.bias", &o.proj_b, 1, E, 0});
        items.push_back({p + "ln_2.weight", &o.ln2_g, 1, E, 0});
        items.push_back({p + "ln_2.bias", &o.ln2_b, 1, E, 0});
        items.push_back({p + "mlp.c_fc.weight", &o.fc_w, E, F, 1, l, 2});
        items.push_back({p + "mlp.c_fc.bias", &o.fc_b, 1, F, 0});
        items.push_back({p + "mlp.c_proj.weight", &o.fc2_w, F, E, 1, l, 3});
        items.push_back({p + "mlp.c_proj.bias", &o.fc2_b, 1, E, 0});
    }
    items.push_back({"ln_f.weight", &e->lnf_g, 1, E, 0});
    items.push_back({"ln_f.bias", &e->lnf_b, 1, E, 0});
    if (lmt) items.push_back({"lm_head.weight", &e->lm, V, E, 2});
    size_t off = 0;
    for (auto &it : items) {
        *it.off = off;
        off = align_up(off + (size_t)it.rows * it.cols, 128);
    }
    if (!lmt) e->lm = e->wte;   // tied head (main.c:1374-1386)
    e->welem = off;
    const size_t bytes = off * e->esize;
    cudaError_t r = cudaMalloc(&e->wbuf, bytes);
    if (r != cudaSuccess) return set_err(G2_ERR_OOM, "cudaMalloc weights (%zu bytes): %s", bytes, cudaGetErrorString(r));
    e->device_bytes += bytes;
    // Unit-packed copy of the projections for the persistent decode kernel
    // (pack_mega_layer): each unit is one contiguous run of floats.
    const int *cw = e->mega_cw;
    if (e->mega) {
        e->layer_off.assign((size_t)c.n_layer * 3, 0);
        long long po = 0;
        for (int l = 0; l < c.n_layer; ++l) {
            const long long sz[3] = {mega_packed_a(E), mega_packed_b(E), mega_packed_d(E, F)};
            for (int q = 0; q < 3; ++q) {
                e->layer_off[(size_t)l * 3 + q] = po;
                po += (sz[q] + 63) / 64 * 64;
            }
        }
        r = cudaMalloc(&e->packed, (size_t)po * 4);
        if (r != cudaSuccess) return set_err(G2_ERR_OOM, "cudaMalloc packed weights: %s", cudaGetErrorString(r));
        e->device_bytes += (size_t)po * 4;
    }
    // host copies of the current layer's tensors until all twelve are read
    std::vector<std::vector<float>> layer_t(12);
    int layer_have = 0;

    std::vector<float> tmp, pk;
    std::vector<uint16_t> hv;
    // nn.Linear [out][in] projections (and an [E][V] lm_head) are transposed on
    // the device: the file's values go to this staging buffer, and a transpose
    // kernel writes them into the weight buffer in the kernels' layout.
    float *stage = nullptr;
    size_t stage_n = 0;
    struct StageFree {
        float *&p;
        ~StageFree() {
            if (p) cudaFree(p);
        }
    } stage_free{stage};
    for (auto &it : items) {
        const StTensor *t = sf.find(it.name);
        if (!t) return set_err(G2_ERR_FORMAT, "tensor '%s' not found", it.name.c_str());
        const size_t n = (size_t)it.rows * it.cols;
        if ((size_t)t->numel() != n) return set_err(G2_ERR_FORMAT, "tensor '%s': %lld elements, expected %zu",
                                                    it.name.c_str(), (long long)t->numel(), n);
        tmp.resize(n);
        rc = sf.read_f32(*t, tmp.data(), err);
        if (rc) return set_err(rc, "%s", err.c_str());
        const float *src = tmp.data();
        int tr_rows = 0, tr_cols = 0;   // > 0: transpose [tr_rows][tr_cols] on the device
        if (it.kind == 1) {
            // Conv1D [in,out] is kept; nn.Linear [out,in] is transposed (main.c:1252-1300)
            const int in = it.rows, out = it.cols;
            if (t->shape.size() != 2) return set_err(G2_ERR_FORMAT, "tensor '%s' is not 2-D", it.name.c_str());
            if (conv1d) {
                if (t->shape[0] != in || t->shape[1] != out)
                    return set_err(G2_ERR_FORMAT, "tensor '%s': expected [%d,%d]", it.name.c_str(), in, out);
            } else {
                if (t->shape[0] != out || t->shape[1] != in)
                    return set_err(G2_ERR_FORMAT, "tensor '%s': expected [%d,%d]", it.name.c_str(), out, in);
                tr_rows = out;
                tr_cols = in;
            }
        } else if (it.kind == 2) {
            // lm_head.weight [V,E] is kept; [E,V] is transposed (main.c:1387-1410)
            if (t->shape.size() != 2) return set_err(G2_ERR_FORMAT, "lm_head.weight is not 2-D");
            if (t->shape[0] == E && t->shape[1] == V) {
                tr_rows = E;
                tr_cols = V;
            } else if (!(t->shape[0] == V && t->shape[1] == E)) {
                return set_err(G2_ERR_FORMAT, "lm_head.weight: unexpected shape");
            }
        }
        if (e->mega && it.name.compare(0, 2, "h.") == 0) {
            // the layer's tensors arrive in the order ln_1.w/b, c_attn.w/b, attn.c_proj.w/b,
            // ln_2.w/b, c_fc.w/b, mlp.c_proj.w/b; pack the four projections once all are here
            layer_t[layer_have].assign(src, src + n);
            if (++layer_have == 12) {
                const int l = atoi(it.name.c_str() + 2);   // "h.<l>.mlp.c_proj.bias"
                const std::vector<float> *T = layer_t.data();
                for (int q = 0; q < 3; ++q) {
                    pack_mega_layer(T, !conv1d, E, F, c.n_head, cw[0], cw[1], e->mega_nq, q, pk);
                    r = cudaMemcpy(e->packed + e->layer_off[(size_t)l * 3 + q], pk.data(), pk.size() * 4,
                                   cudaMemcpyHostToDevice);
                    if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "upload packed layer %d: %s", l, cudaGetErrorString(r));
                }
                layer_have = 0;
            }
        }
        void *dst = (char *)e->wbuf + *it.off * e->esize;
        if (tr_rows > 0) {
            if (n > stage_n) {
                if (stage) cudaFree(stage);
                stage = nullptr;
                r = cudaMalloc(&stage, n * 4);
                if (r != cudaSuccess) return set_err(G2_ERR_OOM, "cudaMalloc transpose staging: %s", cudaGetErrorString(r));
                stage_n = n;
            }
            r = cudaMemcpy(stage, src, n * 4, cudaMemcpyHostToDevice);
            if (r == cudaSuccess) {
                if (e->dtype == G2_F32) launch_transpose<float>(stage, (float *)dst, tr_rows, tr_cols, 0);
                else launch_transpose<__half>(stage, (__half *)dst, tr_rows, tr_cols, 0);
                r = cudaGetLastError();
            }
            if (r == cudaSuccess) r = cudaDeviceSynchronize();   // the staging buffer is reused by the next tensor
        } else if (e->dtype == G2_F32) {
            r = cudaMemcpy(dst, src, n * 4, cudaMemcpyHostToDevice);
        } else {
            hv.resize(n);
            for (size_t i = 0; i < n; ++i) hv[i] = f2h_bits(src[i]);
            r = cudaMemcpy(dst, hv.data(), n * 2, cudaMemcpyHostToDevice);
        }
        if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "upload '%s': %s", it.name.c_str(), cudaGetErrorString(r));
    }
    // A cudaMemcpy from pageable host memory may return before its DMA has landed,
    // and the engine's stream does not wait for the legacy default stream: every
    // upload must be complete before the first kernel on that stream reads the
    // weights (the tensor-core weight images are built right after this).
    if ((r = cudaDeviceSynchronize()) != cudaSuccess)
        return set_err(G2_ERR_CUDA, "weight upload: %s", cudaGetErrorString(r));
    // Algorithmic bytes streamed per decode step (weights + biases + LN + lm head).
    const size_t es = e->esize;
    e->stream_bytes = es * ((size_t)c.n_layer * ((size_t)4 * E * E + (size_t)2 * E * F) + (size_t)E * c.padded_vocab) +
                      es * ((size_t)c.n_layer * (9 * (size_t)E + F) + 2 * (size_t)E);
    return G2_OK;
}

extern "C" int g2_open(const char *model_dir, int device, int max_batch, int dtype, g2_engine **out) {
    if (!model_dir || !out) return set_err(G2_ERR_ARG, "g2_open: null argument");
    *out = nullptr;
    if (max_batch < 1 || max_batch > 4096) return set_err(G2_ERR_ARG, "g2_open: max_batch out of range");
    if (dtype != G2_F32 && dtype != G2_F16) return set_err(G2_ERR_ARG, "g2_open: dtype must be G2_F32 or G2_F16");
    {
        // Validate the files before touching a device (format errors are reported first).
        ModelConfig c;
        std::string err;
        int rc = load_config(model_dir, c, err);
        if (!rc) rc = validate_gpt2(model_dir, c, err);
        if (rc) return set_err(rc, "%s", err.c_str());
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return set_err(G2_ERR_CUDA, "g2_open: no CUDA device");
    if (device < 0 || device >= ndev) return set_err(G2_ERR_ARG, "g2_open: device %d of %d", device, ndev);
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) return set_err(G2_ERR_CUDA, "g2_open: device %d is sm_%d%d; this build targets sm_100a",
                                        device, prop.major, prop.minor);
    auto *e = new g2_engine;
    e->device = device;
    e->dtype = dtype;
    e->esize = dtype == G2_F32 ? 4 : 2;
    e->max_batch = max_batch;
    e->sms = prop.multiProcessorCount;
    int rc;
    std::string err;
    if ((rc = load_config(model_dir, e->c, err))) {
        delete e;
        return set_err(rc, "%s", err.c_str());
    }
#define TRY(x)                \
    do {                      \
        if ((rc = (x))) {     \
            free_engine(e);   \
            return rc;        \
        }                     \
    } while (0)
    {
        cudaError_t r = cudaSetDevice(device);
        if (r != cudaSuccess) {
            delete e;
            return set_err(G2_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(r));
        }
        r = cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking);
        if (r != cudaSuccess) {
            delete e;
            return set_err(G2_ERR_CUDA, "cudaStreamCreate: %s", cudaGetErrorString(r));
        }
    }
    {
        // The persistent B = 1 decode kernel: fp32, one co-resident CTA per SM,
        // its shared-memory ring and input vector within the opt-in limit.
        const char *off = getenv("G2_NO_MEGA");
        int coop = 0, optin = 0;
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        const size_t smem = mega_smem_bytes(e->c.n_embd);
        const int G = e->sms, E = e->c.n_embd, F = e->c.ffn_dim;
        int *cw = e->mega_cw;
        cw[0] = mega_cw(3 * E, G);
        cw[1] = mega_cw(F, G);
        e->mega_nq = mega_nq(E, e->c.n_head, G);
        if (const char *nq = getenv("G2_MEGA_NQ"))
            if (mega_nq_ok(E, atoi(nq))) e->mega_nq = atoi(nq);
        // every row (E floats) fits a ring slot, an E-wide block has at most one
        // float4 group per consumer thread, and the context fits the score buffer
        e->mega = dtype == G2_F32 && !(off && off[0] == '1') && coop && smem <= (size_t)optin && G <= 256 && cw[0] &&
                  cw[1] && e->mega_nq && E * 4 <= mega_slot_bytes() && E / 4 <= 480 && e->c.n_ctx <= mega_max_keys() &&
                  e->c.n_head * 64 == E && e->c.n_layer <= kMegaMaxLayers;
        e->mega_smem = smem;
        if (const char *st = getenv("G2_MEGA_SPLIT_T"))
            if (atoi(st) >= 64) e->mega_split_t = atoi(st);   // >= 64: every slice then has keys
        if (const char *w = getenv("G2_WAIT_LIMIT_MS"))
            if (atoi(w) > 0) e->wait_ns = (unsigned long long)atoi(w) * 1000000ull;
        if (const char *t = getenv("G2_TEST_STALL"))
            if (!strcmp(t, "acc")) e->test_stall = 1;
    }
    TRY(load_weights(e, model_dir));
    const ModelConfig &c = e->c;
    const int E = c.n_embd, F = c.ffn_dim, NH = c.n_head, S = c.n_ctx, Vp = c.padded_vocab;
    // KV caches [slot][layer][head][pos][64]
    e->kv.max_seq = S;
    e->kv.n_head = NH;
    e->kv.n_slots = max_batch;
    e->kv.layer_stride = (long long)NH * S * kHeadDim;
    e->kv.slot_stride = e->kv.layer_stride * c.n_layer;
    const size_t kv_elems = (size_t)e->kv.slot_stride * max_batch;
    {
        const size_t bytes = kv_elems * e->esize;
        cudaError_t r1 = cudaMalloc(&e->kbuf, bytes);
        cudaError_t r2 = r1 == cudaSuccess ? cudaMalloc(&e->vbuf, bytes) : r1;
        if (r2 != cudaSuccess) {
            free_engine(e);
            return set_err(G2_ERR_OOM, "KV cache (%zu bytes x 2): %s", bytes, cudaGetErrorString(r2));
        }
        e->device_bytes += 2 * bytes;
        e->kv.k = e->kbuf;
        e->kv.v = e->vbuf;
        // zeroed once: positions a sequence has not written hold zeros, never stale bit
        // patterns of other data (the batched attention reads whole 128-key tiles)
        r1 = cudaMemset(e->kbuf, 0, bytes);
        if (r1 == cudaSuccess) r1 = cudaMemset(e->vbuf, 0, bytes);
        if (r1 == cudaSuccess) r1 = cudaDeviceSynchronize();
        if (r1 != cudaSuccess) {
            free_engine(e);
            return set_err(G2_ERR_CUDA, "KV cache zeroing: %s", cudaGetErrorString(r1));
        }
        if (dtype == G2_F16) {
            const unsigned long long rows = kv_elems / kHeadDim;
            if (tc_encode(&e->kv_kmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, e->kbuf, kHeadDim, rows, kHeadDim, 64,
                          false) == G2_OK &&
                tc_encode(&e->kv_vmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, e->vbuf, kHeadDim, rows, kHeadDim, 64,
                          false) == G2_OK)
                e->kv_maps = true;
        }
    }
    e->R = S > max_batch ? S : max_batch;
    const int R = e->R;
    TRY(dalloc(e, &e->h, (size_t)R * E));
    TRY(dalloc(e, &e->xln, (size_t)R * E));
    TRY(dalloc(e, &e->qkv, (size_t)R * 3 * E));
    TRY(dalloc(e, &e->attn, (size_t)R * E));
    TRY(dalloc(e, &e->ffn, (size_t)R * F));
    TRY(dalloc(e, &e->logits, (size_t)max_batch * Vp));
    TRY(dalloc(e, &e->logits_rows, (size_t)max_batch * Vp));
    if (dtype == G2_F32) {
        e->plan_qkv = gemv_plan<float>(3 * E, E, e->sms);
        e->plan_proj = gemv_plan<float>(E, E, e->sms);
        e->plan_fc = gemv_plan<float>(F, E, e->sms);
        e->plan_fc2 = gemv_plan<float>(E, F, e->sms);
    } else {
        e->plan_qkv = gemv_plan<__half>(3 * E, E, e->sms);
        e->plan_proj = gemv_plan<__half>(E, E, e->sms);
        e->plan_fc = gemv_plan<__half>(F, E, e->sms);
        e->plan_fc2 = gemv_plan<__half>(E, F, e->sms);
    }
    size_t gp = 0, gt = 0;
    const GemvPlan plans[4] = {e->plan_qkv, e->plan_proj, e->plan_fc, e->plan_fc2};
    const int Ns[4] = {3 * E, E, F, E};
    for (int i = 0; i < 4; ++i) {
        gp = std::max(gp, (size_t)plans[i].ksplit * Ns[i]);
        gt = std::max(gt, (size_t)plans[i].tiles);
    }
    TRY(dalloc(e, &e->gemv_partial, gp));
    TRY(dalloc(e, &e->gemv_ctr, gt));
    e->gemv_ctr_n = gt;
    TRY(dalloc(e, &e->attn_partial, attn_partial_floats(R, NH, S)));
    TRY(dalloc(e, &e->attn_ctr, attn_counter_count(R, NH)));
    e->attn_ctr_n = attn_counter_count(R, NH);
    TRY(dalloc(e, &e->lm_partial, (size_t)2 * lm_head_blocks()));
    TRY(dalloc(e, &e->lm_ctr, 1));
    TRY(dalloc(e, &e->rows_tok, R));
    TRY(dalloc(e, &e->rows_pos, R));
    TRY(dalloc(e, &e->rows_slot, R));
    TRY(dalloc(e, &e->result, 2));
    TRY(dalloc(e, &e->argmax_out, 2 * (size_t)max_batch));
    TRY(dalloc(e, &e->batch_step, 1));
    TRY(dalloc(e, &e->out_tokens, (size_t)max_batch * S));
    TRY(dalloc(e, &e->state, 1));
    TRY(dalloc(e, &e->sample_work, (size_t)Vp));
    TRY(dalloc(e, &e->sample_ctx, (size_t)S));
    TRY(dalloc(e, &e->topk_out, (size_t)2 * G2_MAX_TOPK));
    {
        cudaError_t r = cudaMallocHost(&e->h_rows, sizeof(int) * 3 * (size_t)R);
        if (r == cudaSuccess) r = cudaMallocHost(&e->h_state, sizeof(StepState) * 64);
        if (r == cudaSuccess) r = cudaMallocHost(&e->h_small, sizeof(int) * 4 * (size_t)max_batch + 64);
        if (r == cudaSuccess) r = cudaMallocHost(&e->h_ctx, sizeof(int) * (size_t)S);
        if (r == cudaSuccess) r = cudaEventCreateWithFlags(&e->staged, cudaEventDisableTiming);
        for (auto &ev : e->ev)
            if (r == cudaSuccess) r = cudaEventCreate(&ev);
        if (r != cudaSuccess) {
            free_engine(e);
            return set_err(G2_ERR_CUDA, "host staging: %s", cudaGetErrorString(r));
        }
    }
    e->filled.assign(max_batch, 0);
    e->dec_graph.assign(max_batch, nullptr);
    if (e->mega) {
        TRY(dalloc(e, &e->t_qkv, (size_t)3 * E));
        TRY(dalloc(e, &e->mega_acc, mega_acc_words(kMegaMaxSteps, c.n_layer, E)));
        TRY(dalloc(e, &e->t_best, (size_t)4 * e->sms));
        TRY(dalloc(e, &e->t_att, (size_t)c.n_head * e->mega_nq * 66));
        TRY(dalloc(e, &e->d_err, 1));
        TRY(dalloc(e, &e->d_layer_off, e->layer_off.size()));
        TRY(dalloc(e, &e->d_layers, (size_t)c.n_layer));
        std::vector<LayerPtrs> lp(c.n_layer);
        for (int l = 0; l < c.n_layer; ++l) {
            const LayerOff &o = e->L[l];
            lp[l] = LayerPtrs{e->w<float>(o.ln1_g), e->w<float>(o.ln1_b), e->w<float>(o.qkv_b), e->w<float>(o.proj_b),
                              e->w<float>(o.ln2_g), e->w<float>(o.ln2_b), e->w<float>(o.fc_b), e->w<float>(o.fc2_b)};
        }
        cudaError_t r = cudaMemcpy(e->d_layers, lp.data(), sizeof(LayerPtrs) * lp.size(), cudaMemcpyHostToDevice);
        if (r == cudaSuccess)
            r = cudaMemcpy(e->d_layer_off, e->layer_off.data(), sizeof(long long) * e->layer_off.size(),
                           cudaMemcpyHostToDevice);
        const bool traced = getenv("G2_MEGA_TRACE") != nullptr;
        for (int k = 0; k < 2 && r == cudaSuccess; ++k)
            r = cudaFuncSetAttribute(mega_kernel_ptr(k == 1), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)e->mega_smem);
        int per_sm = 0;
        if (r == cudaSuccess)
            r = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mega_kernel_ptr(traced), mega_threads(),
                                                              e->mega_smem);
        if (r != cudaSuccess) {
            free_engine(e);
            return set_err(G2_ERR_CUDA, "decode kernel setup: %s", cudaGetErrorString(r));
        }
        if (per_sm < 1) {
            e->mega = false;   // cannot be co-resident: keep the graph path
        }
        e->mega_grid = e->sms;
        if (const char *fl = getenv("G2_MEGA_INFLIGHT")) {
            const int v = atoi(fl);
            if (v >= 1 && v <= 8) e->mega_inflight = v;
        }
        if (const char *tp = getenv("G2_MEGA_TRACE")) {
            e->trace_path = tp;
            TRY(dalloc(e, &e->d_trace, (size_t)e->mega_grid * kTraceSlots));
        }
    }
    {
        // Tensor-core GEMMs for prefill and batched decode: every K a multiple of
        // 64 and every N of 8 (the projections of all GPT-2 sizes qualify).
        const char *npg = getenv("G2_NO_PREFILL_GRAPH");
        e->prefill_graph_on = !(npg && npg[0] == '1');
        const char *notc = getenv("G2_NO_TC");
        e->tc = !(notc && notc[0] == '1') && E % 64 == 0 && F % 64 == 0 && E % 8 == 0;
        if (e->tc) {
            e->tc_kind = dtype == G2_F32 ? TC_TF32X3 : TC_F16;
            const int Ks[4] = {E, E, E, F}, Ns[4] = {3 * E, E, F, E};
            // fp32 engines stream the projections as stage images (TcWeights::img_hi),
            // one bulk copy per ring stage: tf32 hi / lo images (or, with
            // G2_TC_WSPLIT=1, the fp32 image split in shared memory), in place of
            // tf32 hi / lo copies read by tiled TMA boxes (G2_TC_IMG=0).  fp16 engines
            // read their weights in place by tiled boxes (G2_TC_IMG=1 makes an fp16
            // image; measured no faster, so it is not worth the second copy).
            const char *ws_env = getenv("G2_TC_WSPLIT");
            const bool wsplit = e->tc_kind == TC_TF32X3 && ws_env && ws_env[0] == '1';
            const char *img_env = getenv("G2_TC_IMG");
            const bool img = img_env ? img_env[0] == '1' : e->tc_kind == TC_TF32X3;
            const int ncopy = e->tc_kind == TC_TF32X3 && !wsplit ? 2 : 1;
            const size_t elem = e->tc_kind == TC_TF32X3 ? 4 : 2;
            size_t per_layer = 0, img_layer = 0;
            for (int q = 0; q < 4; ++q) {
                per_layer += align_up((size_t)Ks[q] * Ns[q], 64);
                img_layer += tc_image_elems(e->tc_kind, Ks[q], Ns[q]) * elem;
            }
            if (img) {
                TRY(dalloc(e, reinterpret_cast<unsigned char **>(&e->tc_img), ncopy * img_layer * c.n_layer));
                TRY(dalloc(e, reinterpret_cast<unsigned char **>(&e->tc_idx), (size_t)16384));
                TRY(dalloc(e, &e->tc_perm, (size_t)8192));
                TRY(dalloc(e, &e->tc_err, 1));
                if (tc_stage_perm(e->tc_kind, e->tc_idx, e->tc_perm, e->tc_err, e->st)) {
                    free_engine(e);
                    return set_err(G2_ERR_CUDA, "stage permutation of the tensor-core weights");
                }
            } else if (e->tc_kind == TC_TF32X3 && !wsplit) {
                TRY(dalloc(e, &e->tc_w, 2 * per_layer * c.n_layer));
            }
            e->tc_maps.resize((size_t)c.n_layer * 4);
            size_t o = 0, io = 0;
            for (int l = 0; l < c.n_layer; ++l) {
                const LayerOff &lo = e->L[l];
                const size_t wo[4] = {lo.qkv_w, lo.proj_w, lo.fc_w, lo.fc2_w};
                for (int q = 0; q < 4; ++q) {
                    const size_t n = (size_t)Ks[q] * Ns[q];
                    TcWeights &tw = e->tc_maps[(size_t)l * 4 + q];
                    int rc;
                    if (img) {
                        // the maps stay valid descriptors of the weights; the GEMM reads the images
                        const size_t ib = tc_image_elems(e->tc_kind, Ks[q], Ns[q]) * elem;
                        unsigned char *ih = reinterpret_cast<unsigned char *>(e->tc_img) + io;
                        unsigned char *il = ncopy == 2 ? ih + img_layer * c.n_layer : nullptr;
                        if (e->tc_kind == TC_TF32X3) {
                            rc = tc_weights(&tw, TC_TF32X3, e->w<float>(wo[q]), nullptr, Ks[q], Ns[q]);
                            launch_tc_image(TC_TF32X3, e->w<float>(wo[q]), ih, il, e->tc_perm, Ks[q], Ns[q], e->st);
                            tw.wsplit = wsplit;
                        } else {
                            rc = tc_weights(&tw, TC_F16, e->w<__half>(wo[q]), nullptr, Ks[q], Ns[q]);
                            launch_tc_image(TC_F16, e->w<__half>(wo[q]), ih, nullptr, e->tc_perm, Ks[q], Ns[q], e->st);
                        }
                        tw.img_hi = ih;
                        tw.img_lo = il;
                        io += ib;
                    } else if (e->tc_kind == TC_TF32X3 && !wsplit) {
                        float *hi = e->tc_w + o, *lo_ = e->tc_w + per_layer * c.n_layer + o;
                        launch_tc_prep(TC_TF32X3, e->w<float>(wo[q]), hi, lo_, nullptr, (long long)n, e->st);
                        rc = tc_weights(&tw, TC_TF32X3, hi, lo_, Ks[q], Ns[q]);
                    } else if (wsplit) {
                        rc = tc_weights(&tw, TC_TF32X3, e->w<float>(wo[q]), nullptr, Ks[q], Ns[q]);
                    } else {
                        rc = tc_weights(&tw, TC_F16, e->w<__half>(wo[q]), nullptr, Ks[q], Ns[q]);
                    }
                    if (rc) {
                        free_engine(e);
                        return set_err(rc, "tensor map of layer %d projection %d", l, q);
                    }
                    o += align_up(n, 64);
                }
            }
            {
                const size_t n = (size_t)c.vocab_size * E;
                int rc;
                if (e->tc_kind == TC_TF32X3 && !wsplit) {
                    TRY(dalloc(e, &e->tc_lm_w, 2 * align_up(n, 64)));
                    float *hi = e->tc_lm_w, *lo_ = e->tc_lm_w + align_up(n, 64);
                    launch_tc_prep(TC_TF32X3, e->w<float>(e->lm), hi, lo_, nullptr, (long long)n, e->st);
                    rc = tc_weights_kmajor(&e->tc_lm, TC_TF32X3, hi, lo_, E, c.vocab_size);
                } else if (wsplit) {
                    rc = tc_weights_kmajor(&e->tc_lm, TC_TF32X3, e->w<float>(e->lm), nullptr, E, c.vocab_size);
                } else {
                    rc = tc_weights_kmajor(&e->tc_lm, TC_F16, e->w<__half>(e->lm), nullptr, E, c.vocab_size);
                }
                if (rc) {
                    free_engine(e);
                    return set_err(rc, "tensor map of the LM head");
                }
            }
            TRY(dalloc(e, &e->tc_xhi, (size_t)R * E));
            TRY(dalloc(e, &e->tc_x2hi, (size_t)R * F));
            if (e->tc_kind == TC_TF32X3) {
                TRY(dalloc(e, &e->tc_xlo, (size_t)R * E));
                TRY(dalloc(e, &e->tc_x2lo, (size_t)R * F));
            }
            TRY(dalloc(e, &e->tc_ctr, (size_t)kTcMaxTiles));
            int rc = tc_rows_operand(&e->tc_x_e, e->tc_kind, e->tc_xhi, e->tc_xlo, E, R);
            if (!rc) rc = tc_rows_operand(&e->tc_x_f, e->tc_kind, e->tc_x2hi, e->tc_x2lo, F, R);
            if (rc) {
                free_engine(e);
                return set_err(rc, "tensor maps of the GEMM input rows");
            }
            for (int q = 0; q < 4; ++q)
                e->tc_part_floats = std::max(e->tc_part_floats, tc_partial_floats(R, Ns[q], Ks[q], e->tc_kind, e->sms));
            TRY(dalloc(e, &e->tc_part, e->tc_part_floats));
            if (!e->tc_err) TRY(dalloc(e, &e->tc_err, 1));
            cudaError_t r = cudaStreamSynchronize(e->st);
            if (r != cudaSuccess) {
                free_engine(e);
                return set_err(G2_ERR_CUDA, "tensor-core weight split: %s", cudaGetErrorString(r));
            }
            int perm_err = 0;   // an expired wait in tc_stage_perm
            if (cudaMemcpy(&perm_err, e->tc_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess || perm_err) {
                free_engine(e);
                return set_err(perm_err ? perm_err : G2_ERR_CUDA, "tensor-core weight images: the stage permutation failed");
            }
        }
    }
#undef TRY
    // the remaining uploads of set-up (row tables, packed units) are complete
    // before any call runs work on the engine's stream
    if (cudaDeviceSynchronize() != cudaSuccess) {
        free_engine(e);
        return set_err(G2_ERR_CUDA, "g2_open: engine set-up failed");
    }
    *out = e;
    return G2_OK;
}

extern "C" int g2_close(g2_engine *e) {
    if (!e) return set_err(G2_ERR_ARG, "g2_close: null engine");
    free_engine(e);
    return G2_OK;
}

extern "C" int g2_get_config(const g2_engine *e, g2_config *out) {
    if (!e || !out) return set_err(G2_ERR_ARG, "g2_get_config: null argument");
    out->n_layer = e->c.n_layer;
    out->n_embd = e->c.n_embd;
    out->n_head = e->c.n_head;
    out->n_ctx = e->c.n_ctx;
    out->vocab_size = e->c.vocab_size;
    out->ffn_dim = e->c.ffn_dim;
    out->padded_vocab = e->c.padded_vocab;
    out->dtype = e->dtype;
    out->max_batch = e->max_batch;
    out->device = e->device;
    out->weight_bytes = e->stream_bytes;
    out->device_bytes = e->device_bytes;
    out->persistent = e->mega ? 1 : 0;
    return G2_OK;
}

extern "C" long long g2_launch_count(const g2_engine *e) { return e ? e->launches : -1; }

// ------------------------------------------------------------------------------
// forward passes
// ------------------------------------------------------------------------------

// Stage row descriptors (tok, pos, slot) into the device row arrays.
static int stage_rows(g2_engine *e, int n, const int *tok, const int *pos, const int *slot) {
    CK(cudaEventSynchronize(e->staged));   // previous staging copy has been consumed
    int *hr = e->h_rows;
    memcpy(hr, tok, sizeof(int) * n);
    memcpy(hr + e->R, pos, sizeof(int) * n);
    memcpy(hr + 2 * e->R, slot, sizeof(int) * n);
    CK(cudaMemcpyAsync(e->rows_tok, hr, sizeof(int) * n, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->rows_pos, hr + e->R, sizeof(int) * n, cudaMemcpyHostToDevice, e->st));
    CK(cudaMemcpyAsync(e->rows_slot, hr + 2 * e->R, sizeof(int) * n, cudaMemcpyHostToDevice, e->st));
    CK(cudaEventRecord(e->staged, e->st));
    return G2_OK;
}

// All layers over `nrows` rows described by the device row arrays (prefill of
// one slot, or one decode token for each of several slots).  Leaves the
// residual stream in e->h.
// Where a kernel writes the next tensor-core GEMM's operand: the rows with
// K = E (LN and attention outputs) or fc2's rows (fc's output).
static OperandOut operand_e(const g2_engine *e) {
    OperandOut o;
    if (e->tc) {
        o.kind = e->tc_kind;
        o.hi = e->tc_xhi;
        o.lo = e->tc_xlo;
        o.h16 = reinterpret_cast<__half *>(e->tc_xhi);
    }
    return o;
}
static OperandOut operand_f(const g2_engine *e) {
    OperandOut o;
    if (e->tc) {
        o.kind = e->tc_kind;
        o.hi = e->tc_x2hi;
        o.lo = e->tc_x2lo;
        o.h16 = reinterpret_cast<__half *>(e->tc_x2hi);
    }
    return o;
}

// One projection of a many-row pass: out[r] = epilogue(X[r] W), on the tensor
// cores (X already written as the operand by its producer) or by the SIMT GEMM.
// With ln_g / ln_b (the LayerNorm that follows this residual-stream update),
// a split-K tensor-core GEMM also writes the LayerNorm of its output rows as
// ln_op; returns whether it did (else the caller runs the LayerNorm).
template <typename WT>
static bool rows_gemm(g2_engine *e, int l, int q, const float *X, int nrows, const WT *W, const WT *bias,
                      const float *resid, float *out, int N, int K, int epi, const KVLayout *kv, Rows rows,
                      OperandOut op = OperandOut(), const WT *ln_g = nullptr, const WT *ln_b = nullptr,
                      OperandOut ln_op = OperandOut()) {
    bool ln_done = false;
    if (e->tc) {
        e->launches += launch_tc_gemm<WT>(e->tc_kind, e->tc_maps[(size_t)l * 4 + q],
                                          K == e->c.n_embd ? e->tc_x_e : e->tc_x_f, nrows, e->tc_part,
                                          e->tc_part_floats, e->tc_ctr, e->tc_err, bias, resid, out, epi, kv, l, rows,
                                          e->sms, e->st, op, 0, ln_g, ln_b, ln_op, &ln_done);
    } else {
        launch_gemm_rows<WT>(X, W, bias, resid, out, nrows, N, K, epi, kv, l, rows, e->st);
        e->launches += 1;
    }
    return ln_done;
}

// All layers over `nrows` rows described by the device row arrays (prefill of
// one slot, or one decode token for each of several slots: decode_rows).
// Leaves the residual stream in e->h.  With the tensor cores, LayerNorm and
// attention write the next GEMM's operand themselves, fc writes fc2's, the
// residual-stream reduces take the next LayerNorm, and for decode rows the
// attention sums c_attn's split-K partials itself: a layer is five to seven
// launches.
template <typename WT>
static int forward_rows(g2_engine *e, int nrows, int max_pos, bool decode_rows = false) {
    const ModelConfig &c = e->c;
    const int E = c.n_embd, F = c.ffn_dim;
    cudaStream_t st = e->st;
    Rows rows{e->rows_tok, e->rows_pos, e->rows_slot};
    const OperandOut ope = operand_e(e), opf = operand_f(e);
    launch_embed<WT>(e->w<WT>(e->wte), e->w<WT>(e->wpe), rows, e->h, E, c.vocab_size, c.n_ctx, nrows, st);
    e->launches += 1;
    bool ln1_done = false;   // the previous layer's fc2 wrote this layer's ln_1 operand
    for (int l = 0; l < c.n_layer; ++l) {
        const LayerOff &o = e->L[l];
        if (!ln1_done) {
            launch_layernorm<WT>(e->h, e->xln, e->w<WT>(o.ln1_g), e->w<WT>(o.ln1_b), E, nrows, st, ope);
            e->launches += 1;
        }
        QkvPartials qp;
        if (e->tc && decode_rows) {   // c_attn without its reduce: the attention sums the partials
            SplitInfo si;
            e->launches += launch_tc_gemm<WT>(e->tc_kind, e->tc_maps[(size_t)l * 4], e->tc_x_e, nrows, e->tc_part,
                                              e->tc_part_floats, e->tc_ctr, e->tc_err, e->w<WT>(o.qkv_b), nullptr,
                                              e->qkv, EPI_BIAS | EPI_KV, &e->kv, l, rows, e->sms, st, OperandOut(), 0,
                                              nullptr, nullptr, OperandOut(), nullptr, true, &si);
            if (si.split()) {
                qp.part = e->tc_part;
                qp.si = si;
                qp.err = e->tc_err;
                if (e->kv_maps) {
                    qp.kmap = &e->kv_kmap;
                    qp.vmap = &e->kv_vmap;
                }
                qp.bias = e->w<WT>(o.qkv_b);
            }
        } else {
            rows_gemm<WT>(e, l, 0, e->xln, nrows, e->w<WT>(o.qkv_w), e->w<WT>(o.qkv_b), nullptr, e->qkv, 3 * E, E,
                          EPI_BIAS | EPI_KV, &e->kv, rows);
        }
        // A prompt of more than 64 rows: causal attention in 64 x 64 tiles (each K/V tile read once per
        // 64 queries).  Decode rows (one query per sequence) and short prompts (whose tiles would
        // give one CTA per head): one CTA per (head, 128-key chunk, row).
        if (!decode_rows && nrows > 64)
            launch_prefill_attention<WT>(e->qkv, 3 * E, e->kv, l, rows, nrows, e->attn, E, st, ope);
        else
            launch_attention<WT>(e->qkv, 3 * E, e->kv, l, rows, nrows, e->attn, E, e->attn_partial, e->attn_ctr,
                                 max_pos, st, ope, qp);
        e->launches += 1;
        const bool ln2_done = rows_gemm<WT>(e, l, 1, e->attn, nrows, e->w<WT>(o.proj_w), e->w<WT>(o.proj_b), e->h,
                                            e->h, E, E, EPI_BIAS | EPI_RESID, nullptr, rows, OperandOut(),
                                            e->w<WT>(o.ln2_g), e->w<WT>(o.ln2_b), ope);
        if (!ln2_done) {
            launch_layernorm<WT>(e->h, e->xln, e->w<WT>(o.ln2_g), e->w<WT>(o.ln2_b), E, nrows, st, ope);
            e->launches += 1;
        }
        rows_gemm<WT>(e, l, 2, e->xln, nrows, e->w<WT>(o.fc_w), e->w<WT>(o.fc_b), nullptr, e->ffn, F, E,
                      // on the tensor cores only fc2's operand is read, not the fp32 rows
                      EPI_BIAS | EPI_GELU | (e->tc ? EPI_NOSTORE : 0), nullptr, rows, opf);
        // the next LayerNorm: ln_1 of layer l + 1, or ln_f after the last layer
        const bool last = l + 1 == c.n_layer;
        const WT *ng = e->w<WT>(last ? e->lnf_g : e->L[l + 1].ln1_g), *nb = e->w<WT>(last ? e->lnf_b : e->L[l + 1].ln1_b);
        ln1_done = rows_gemm<WT>(e, l, 3, e->ffn, nrows, e->w<WT>(o.fc2_w), e->w<WT>(o.fc2_b), e->h, e->h, E, F,
                                 EPI_BIAS | EPI_RESID, nullptr, rows, OperandOut(), ng, nb, ope);
    }
    e->lnf_done = ln1_done;
    CKL();
    return G2_OK;
}

// ln_f + the tied LM head over the `nrows` rows of e->h (one token of each
// sequence of a batched step) into e->logits_rows (row stride padded_vocab):
// on the tensor cores, ln_f writes the operand and the GEMM reads wte's rows.
template <typename WT>
static void lm_head_rows(g2_engine *e, int nrows) {
    const ModelConfig &c = e->c;
    if (!(e->tc && e->lnf_done)) {   // else the last fc2 wrote the ln_f operand
        launch_layernorm<WT>(e->h, e->xln, e->w<WT>(e->lnf_g), e->w<WT>(e->lnf_b), c.n_embd, nrows, e->st, operand_e(e));
        e->launches += 1;
    }
    if (e->tc) {
        Rows rows{e->rows_tok, e->rows_pos, e->rows_slot};
        e->launches += launch_tc_gemm<WT>(e->tc_kind, e->tc_lm, e->tc_x_e, nrows, e->tc_part, e->tc_part_floats,
                                          e->tc_ctr, e->tc_err, nullptr, nullptr, e->logits_rows, 0, nullptr, 0, rows,
                                          e->sms, e->st, OperandOut(), c.padded_vocab);
    } else {
        launch_lm_head_rows<WT>(e->xln, e->w<WT>(e->lm), e->logits_rows, c.n_embd, c.vocab_size, c.padded_vocab,
                                nrows, e->st);
        e->launches += 1;
    }
}

// LM head on row `row` of e->h for `slot`, optionally advancing the step state.
template <typename WT>
static int lm_head_row(g2_engine *e, int row, int slot, StepState *state) {
    const ModelConfig &c = e->c;
    launch_lm_head<WT>(e->h + (size_t)row * c.n_embd, e->w<WT>(e->lm), e->w<WT>(e->lnf_g), e->w<WT>(e->lnf_b),
                       e->logits + (size_t)slot * c.padded_vocab, c.n_embd, c.vocab_size, c.padded_vocab, 0,
                       e->lm_partial, e->lm_ctr, e->result, state,
                       state ? e->out_tokens + (size_t)slot * c.n_ctx : nullptr, e->st);
    e->launches += 1;
    e->result_slot = slot;
    CKL();
    return G2_OK;
}

// One B = 1 decode step driven by e->state (kernels only; captured in a graph).
template <typename WT>
static void record_decode_step(g2_engine *e, int slot) {
    const ModelConfig &c = e->c;
    const int E = c.n_embd, F = c.ffn_dim;
    cudaStream_t st = e->st;
    StepState *s = e->state;
    Rows rows{&s->token, &s->pos, &s->slot};
    launch_embed<WT>(e->w<WT>(e->wte), e->w<WT>(e->wpe), rows, e->h, E, c.vocab_size, c.n_ctx, 1, st);
    for (int l = 0; l < c.n_layer; ++l) {
        const LayerOff &o = e->L[l];
        launch_gemv<WT>(e->h, e->w<WT>(o.qkv_w), e->w<WT>(o.qkv_b), nullptr, e->qkv, 3 * E, E, EPI_BIAS | EPI_KV,
                        e->w<WT>(o.ln1_g), e->w<WT>(o.ln1_b), e->gemv_partial, e->gemv_ctr, e->plan_qkv, &e->kv, l,
                        &s->pos, &s->slot, st);
        launch_attention<WT>(e->qkv, 3 * E, e->kv, l, rows, 1, e->attn, E, e->attn_partial, e->attn_ctr, -1, st);
        launch_gemv<WT>(e->attn, e->w<WT>(o.proj_w), e->w<WT>(o.proj_b), e->h, e->h, E, E, EPI_BIAS | EPI_RESID,
                        nullptr, nullptr, e->gemv_partial, e->gemv_ctr, e->plan_proj, nullptr, l, nullptr, nullptr,
                        st);
        launch_gemv<WT>(e->h, e->w<WT>(o.fc_w), e->w<WT>(o.fc_b), nullptr, e->ffn, F, E, EPI_BIAS | EPI_GELU,
                        e->w<WT>(o.ln2_g), e->w<WT>(o.ln2_b), e->gemv_partial, e->gemv_ctr, e->plan_fc, nullptr, l,
                        nullptr, nullptr, st);
        launch_gemv<WT>(e->ffn, e->w<WT>(o.fc2_w), e->w<WT>(o.fc2_b), e->h, e->h, E, F, EPI_BIAS | EPI_RESID,
                        nullptr, nullptr, e->gemv_partial, e->gemv_ctr, e->plan_fc2, nullptr, l, nullptr, nullptr,
                        st);
    }
    launch_lm_head<WT>(e->h, e->w<WT>(e->lm), e->w<WT>(e->lnf_g), e->w<WT>(e->lnf_b),
                       e->logits + (size_t)slot * c.padded_vocab, E, c.vocab_size, c.padded_vocab, 0, e->lm_partial,
                       e->lm_ctr, e->result, s, e->out_tokens + (size_t)slot * c.n_ctx, st);
}

static int decode_graph(g2_engine *e, int slot, cudaGraphExec_t *out) {
    if (e->dec_graph[slot]) {
        *out = e->dec_graph[slot];
        return G2_OK;
    }
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    if (e->dtype == G2_F32) record_decode_step<float>(e, slot);
    else record_decode_step<__half>(e, slot);
    cudaError_t le = cudaGetLastError();
    cudaError_t r = cudaStreamEndCapture(e->st, &g);
    if (le != cudaSuccess) return set_err(G2_ERR_CUDA, "decode capture launch: %s", cudaGetErrorString(le));
    if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "decode capture: %s", cudaGetErrorString(r));
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    r = cudaGraphInstantiate(&e->dec_graph[slot], g, 0);
    cudaGraphDestroy(g);
    if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(r));
    e->dec_graph_kernels = (int)nn;
    *out = e->dec_graph[slot];
    return G2_OK;
}

// The persistent decode kernel for n_steps greedy steps of `slot`, starting
// from e->state (token, pos, step, min_new) and leaving it advanced.
static int launch_mega(g2_engine *e, int slot, int n_steps) {
    const ModelConfig &c = e->c;
    if (e->mega_epoch > 0xF0000000u) {   // epochs are 32-bit: restart them on cleared buffers
        CK(cudaMemsetAsync(e->t_qkv, 0, (size_t)3 * c.n_embd * 8, e->st));
        CK(cudaMemsetAsync(e->t_best, 0, (size_t)4 * e->sms * 8, e->st));
        CK(cudaMemsetAsync(e->t_att, 0, (size_t)c.n_head * e->mega_nq * 66 * 8, e->st));
        e->mega_epoch = 0;
    }
    MegaParams P;
    P.L = c.n_layer;
    P.E = c.n_embd;
    P.F = c.ffn_dim;
    P.NH = c.n_head;
    P.V = c.vocab_size;
    P.max_seq = e->kv.max_seq;
    P.cw_qkv = e->mega_cw[0];
    P.cw_fc = e->mega_cw[1];
    P.nq = e->mega_nq;
    P.lm_rows = mega_lm_rows(P.E);
    P.n_steps = n_steps;
    P.layer_stride = e->kv.layer_stride;
    P.packed = e->packed;
    P.layer_off = e->d_layer_off;
    P.layers = e->d_layers;
    P.wte = e->w<float>(e->wte);
    P.wpe = e->w<float>(e->wpe);
    P.lnf_g = e->w<float>(e->lnf_g);
    P.lnf_b = e->w<float>(e->lnf_b);
    P.lm = e->w<float>(e->lm);
    P.kc = reinterpret_cast<float *>(e->kbuf) + (size_t)slot * e->kv.slot_stride;
    P.vc = reinterpret_cast<float *>(e->vbuf) + (size_t)slot * e->kv.slot_stride;
    P.t_qkv = e->t_qkv;
    P.acc = e->mega_acc;
    P.t_best = e->t_best;
    P.t_att = e->t_att;
    P.split_t = e->mega_split_t;
    P.logits = e->logits + (size_t)slot * c.padded_vocab;
    P.out_tokens = e->out_tokens + (size_t)slot * c.n_ctx;
    P.result = e->result;
    P.state = e->state;
    P.err = e->d_err;
    P.trace = e->d_trace;
    P.max_inflight = e->mega_inflight;
    P.timeout_ns = e->wait_ns;
    // launches of at most kMegaMaxSteps steps, each on zeroed accumulators
    for (int done = 0; done < n_steps;) {
        const int n = std::min(kMegaMaxSteps, n_steps - done);
        CK(cudaMemsetAsync(e->mega_acc, 0, mega_acc_words(n, c.n_layer, c.n_embd) * 8, e->st));
        if (e->test_stall) {
            // Word 0 of step 0's layer-0 attention accumulator starts with 128 in its
            // count field: its NH contributions never bring it to NH, so every CTA's
            // wait for that vector expires (the kernel then returns G2_ERR_TIMEOUT).
            CK(cudaMemsetAsync(reinterpret_cast<char *>(e->mega_acc) + 7, 0x40, 1, e->st));
            e->test_stall = 0;
        }
        P.n_steps = n;
        P.epoch0 = e->mega_epoch + 1;
        e->mega_epoch += mega_epochs(c.n_layer, n);
        void *args[] = {&P};
        CK(cudaLaunchCooperativeKernel(mega_kernel_ptr(e->d_trace != nullptr), dim3(e->mega_grid), dim3(mega_threads()),
                                       args, e->mega_smem, e->st));
        e->launches += 1;
        done += n;
    }
    return G2_OK;
}

// After a synchronised traced launch: append the per-CTA phase trace as one JSON line.
static void dump_trace(g2_engine *e, int n_steps) {
    if (!e->d_trace) return;
    std::vector<unsigned long long> t((size_t)e->mega_grid * kTraceSlots);
    if (cudaMemcpy(t.data(), e->d_trace, t.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return;
    FILE *f = fopen(e->trace_path.c_str(), "a");
    if (!f) return;
    fprintf(f, "{\"steps\": %d, \"ctas\": [", n_steps);
    for (int c = 0; c < e->mega_grid; ++c) {
        fprintf(f, "%s[", c ? "," : "");
        for (int i = 0; i < kTraceSlots; ++i) fprintf(f, "%s%llu", i ? "," : "", t[(size_t)c * kTraceSlots + i]);
        fprintf(f, "]");
    }
    fprintf(f, "]}\n");
    fclose(f);
}

namespace g2 {
int check_flags() {
    int v = check_flag_kernels();
    const int t = check_flag_tc(), m = check_flag_mega();
    if (!v) v = t;
    if (!v) v = m;
    return v;
}
}  // namespace g2

// Synchronise the engine's stream and report what its kernels recorded: an
// expired bounded wait of a tensor-core GEMM or of the decode kernel, a clamped
// accumulator contribution, and (bounds-checked build) a failed bounds test of
// any kernel.  The two error words are copied to pinned memory behind the
// caller's own copies on the stream, so one synchronisation serves both (a
// token of the host loop pays one host round trip, not three).
// After an expired wait: a kernel that gave up may have left a cross-CTA (or
// cross-warp) arrival counter part-way, so every counter array is zeroed on the
// stream before the next kernel.
static int reset_counters(g2_engine *e) {
    if (e->gemv_ctr) CK(cudaMemsetAsync(e->gemv_ctr, 0, e->gemv_ctr_n * sizeof(unsigned), e->st));
    if (e->attn_ctr) CK(cudaMemsetAsync(e->attn_ctr, 0, e->attn_ctr_n * sizeof(unsigned), e->st));
    if (e->lm_ctr) CK(cudaMemsetAsync(e->lm_ctr, 0, sizeof(unsigned), e->st));
    if (e->tc_ctr) CK(cudaMemsetAsync(e->tc_ctr, 0, (size_t)kTcMaxTiles * sizeof(unsigned), e->st));
    return G2_OK;
}

static int sync_and_check(g2_engine *e) {
    int *h = e->h_small + 4 * (size_t)e->max_batch;   // the two spare ints
    h[0] = h[1] = 0;
    if (e->tc) CK(cudaMemcpyAsync(&h[0], e->tc_err, sizeof(int), cudaMemcpyDeviceToHost, e->st));
    if (e->mega) CK(cudaMemcpyAsync(&h[1], e->d_err, sizeof(int), cudaMemcpyDeviceToHost, e->st));
    CK(cudaStreamSynchronize(e->st));
    if (const int site = check_flags())
        return set_err(G2_ERR_RANGE, "bounds check failed in a kernel (site %d, G2_CHECK build)", site);
    if (h[0]) {
        CK(cudaMemsetAsync(e->tc_err, 0, sizeof(int), e->st));   // ordered before the stream's next kernels
        if (const int rc = reset_counters(e)) return rc;
        return set_err(G2_ERR_TIMEOUT, "tensor-core GEMM or batched attention: a bounded device-side wait expired");
    }
    if (const int code = h[1]) {
        CK(cudaMemsetAsync(e->d_err, 0, sizeof(int), e->st));
        if (code != kErrClamp)
            if (const int rc = reset_counters(e)) return rc;
        if (code == kErrClamp)
            return set_err(G2_ERR_RANGE, "decode kernel: an accumulator contribution exceeded +-2^21 and was clamped");
        return set_err(G2_ERR_TIMEOUT, "decode kernel: a bounded device-side wait expired (site %d)", code);
    }
    return G2_OK;
}

static int check_slot(const g2_engine *e, int slot) {
    if (slot < 0 || slot >= e->max_batch) return set_err(G2_ERR_RANGE, "slot %d out of range [0,%d)", slot, e->max_batch);
    return G2_OK;
}

static int check_ids(const g2_engine *e, const int *ids, int n) {
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= e->c.vocab_size)
            return set_err(G2_ERR_RANGE, "token id %d at index %d out of range [0,%d)", ids[i], i, e->c.vocab_size);
    return G2_OK;
}

// One many-row prefill pass over `n` staged-ready rows (tok, pos, slot per row):
// all layers, K/V appended to each row's slot.  The forward reads its rows from
// device arrays, so one graph per row count serves every slot and prompt (a pass
// of several prompts has the same kernels as one prompt of as many rows, since
// passes of more than 64 rows use the tiled attention, whose tiles each take
// the slot of their first row).
static int prefill_rows(g2_engine *e, int n, const int *tok, const int *pos, const int *sl, int max_pos) {
    int rc;
    if ((rc = stage_rows(e, n, tok, pos, sl))) return rc;
    auto run = [&]() { return e->dtype == G2_F32 ? forward_rows<float>(e, n, max_pos) : forward_rows<__half>(e, n, max_pos); };
    g2_engine::PrefillGraph *pg = nullptr;
    if (e->prefill_graph_on && n > 1) {
        pg = &e->prefill_graphs[n];
        if (!pg->exec && pg->uses >= 1 && e->prefill_graphs.size() <= 64) {
            cudaGraph_t g;
            const long long before = e->launches;
            CK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
            rc = run();
            cudaError_t r = cudaStreamEndCapture(e->st, &g);
            if (rc) return rc;
            if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "prefill capture: %s", cudaGetErrorString(r));
            r = cudaGraphInstantiate(&pg->exec, g, 0);
            cudaGraphDestroy(g);
            if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "prefill graph instantiate: %s", cudaGetErrorString(r));
            pg->kernels = e->launches - before;
            e->launches = before;
        }
        ++pg->uses;
    }
    if (pg && pg->exec) {
        CK(cudaGraphLaunch(pg->exec, e->st));
        e->launches += pg->kernels;
    } else if ((rc = run())) {
        return rc;
    }
    return G2_OK;
}

static int prefill_impl(g2_engine *e, int slot, const int *ids, int n) {
    int rc;
    if ((rc = check_slot(e, slot))) return rc;
    if (!ids || n <= 0 || n > e->c.n_ctx) return set_err(G2_ERR_RANGE, "prefill length %d out of range [1,%d]", n, e->c.n_ctx);
    if ((rc = check_ids(e, ids, n))) return rc;
    std::vector<int> pos(n), sl(n, slot);
    for (int i = 0; i < n; ++i) pos[i] = i;
    if ((rc = prefill_rows(e, n, ids, pos.data(), sl.data(), n - 1))) return rc;
    e->filled[slot] = n;
    return G2_OK;
}

extern "C" int g2_prefill(g2_engine *e, int slot, const int *ids, int n) {
    NvtxRange nvtx_range("g2_prefill");
    if (!e) return set_err(G2_ERR_ARG, "null engine");
    CK(cudaSetDevice(e->device));
    int rc = prefill_impl(e, slot, ids, n);
    if (rc) return rc;
    return e->dtype == G2_F32 ? lm_head_row<float>(e, n - 1, slot, nullptr) : lm_head_row<__half>(e, n - 1, slot, nullptr);
}

extern "C" int g2_decode(g2_engine *e, int slot, int token, int pos) {
    NvtxRange nvtx_range("g2_decode");
    if (!e) return set_err(G2_ERR_ARG, "null engine");
    int rc;
    if ((rc = check_slot(e, slot))) return rc;
    if (token < 0 || token >= e->c.vocab_size) return set_err(G2_ERR_RANGE, "token id %d out of range", token);
    if (pos < 0 || pos >= e->c.n_ctx) return set_err(G2_ERR_RANGE, "position %d out of range [0,%d)", pos, e->c.n_ctx);
    if (pos > e->filled[slot]) return set_err(G2_ERR_STATE, "position %d but slot %d holds %d positions", pos, slot, e->filled[slot]);
    CK(cudaSetDevice(e->device));
    cudaGraphExec_t g = nullptr;
    if (!e->mega && (rc = decode_graph(e, slot, &g))) return rc;
    if (e->h_state_i == 0) CK(cudaStreamSynchronize(e->st));   // ring of pinned states wrapped
    StepState *hs = e->h_state + e->h_state_i;
    e->h_state_i = (e->h_state_i + 1) % 64;
    *hs = StepState{token, pos, slot, 0, 0, {0, 0, 0}};
    CK(cudaMemcpyAsync(e->state, hs, sizeof(StepState), cudaMemcpyHostToDevice, e->st));
    if (e->mega) {
        if ((rc = launch_mega(e, slot, 1))) return rc;
    } else {
        CK(cudaGraphLaunch(g, e->st));
        e->launches += e->dec_graph_kernels;
    }
    e->filled[slot] = pos + 1;
    e->result_slot = slot;
    return G2_OK;
}

extern "C" int g2_decode_batch(g2_engine *e, int n, const int *slots, const int *tokens, const int *pos) {
    NvtxRange nvtx_range("g2_decode_batch");
    if (!e || !slots || !tokens || !pos) return set_err(G2_ERR_ARG, "g2_decode_batch: null argument");
    if (n < 1 || n > e->max_batch) return set_err(G2_ERR_RANGE, "batch %d out of range [1,%d]", n, e->max_batch);
    int rc, maxp = 0;
    std::vector<int> seen(e->max_batch, 0);
    for (int i = 0; i < n; ++i) {
        if ((rc = check_slot(e, slots[i]))) return rc;
        if (seen[slots[i]]++) return set_err(G2_ERR_ARG, "slot %d repeated in batch", slots[i]);
        if (pos[i] < 0 || pos[i] >= e->c.n_ctx) return set_err(G2_ERR_RANGE, "position %d out of range", pos[i]);
        if (pos[i] > e->filled[slots[i]]) return set_err(G2_ERR_STATE, "slot %d: position %d beyond %d filled", slots[i], pos[i], e->filled[slots[i]]);
        maxp = std::max(maxp, pos[i]);
    }
    if ((rc = check_ids(e, tokens, n))) return rc;
    CK(cudaSetDevice(e->device));
    if ((rc = stage_rows(e, n, tokens, pos, slots))) return rc;
    const ModelConfig &c = e->c;
    if (e->dtype == G2_F32) {
        if ((rc = forward_rows<float>(e, n, maxp, true))) return rc;
        lm_head_rows<float>(e, n);
    } else {
        if ((rc = forward_rows<__half>(e, n, maxp, true))) return rc;
        lm_head_rows<__half>(e, n);
    }
    for (int i = 0; i < n; ++i)
        launch_copy_row(e->logits_rows + (size_t)i * c.padded_vocab, e->logits + (size_t)slots[i] * c.padded_vocab,
                        c.vocab_size, e->st);
    e->launches += n;
    CKL();
    for (int i = 0; i < n; ++i) e->filled[slots[i]] = pos[i] + 1;
    e->result_slot = -1;
    return G2_OK;
}

// ------------------------------------------------------------------------------
// LM head split by vocabulary rows (the optional column-sharded XL head): the
// layers of a batched step without their LM head, and the LM head over one
// range of wte rows for any set of normalised rows.  Several GPUs each take a
// range and exchange the per-row best (gpt2b200.lmshard).
// ------------------------------------------------------------------------------
extern "C" int g2_decode_batch_rows(g2_engine *e, int n, const int *slots, const int *tokens, const int *pos,
                                    float *rows) {
    NvtxRange nvtx_range("g2_decode_batch_rows");
    if (!e || !slots || !tokens || !pos || !rows) return set_err(G2_ERR_ARG, "g2_decode_batch_rows: null argument");
    if (((uintptr_t)rows) & 15) return set_err(G2_ERR_ARG, "g2_decode_batch_rows: rows not 16-byte aligned");
    if (n < 1 || n > e->max_batch) return set_err(G2_ERR_RANGE, "batch %d out of range [1,%d]", n, e->max_batch);
    int rc, maxp = 0;
    std::vector<int> seen(e->max_batch, 0);
    for (int i = 0; i < n; ++i) {
        if ((rc = check_slot(e, slots[i]))) return rc;
        if (seen[slots[i]]++) return set_err(G2_ERR_ARG, "slot %d repeated in batch", slots[i]);
        if (pos[i] < 0 || pos[i] >= e->c.n_ctx) return set_err(G2_ERR_RANGE, "position %d out of range", pos[i]);
        if (pos[i] > e->filled[slots[i]]) return set_err(G2_ERR_STATE, "slot %d: position %d beyond %d filled", slots[i], pos[i], e->filled[slots[i]]);
        maxp = std::max(maxp, pos[i]);
    }
    if ((rc = check_ids(e, tokens, n))) return rc;
    CK(cudaSetDevice(e->device));
    if ((rc = stage_rows(e, n, tokens, pos, slots))) return rc;
    const ModelConfig &c = e->c;
    // the residual stream after the last layer, then ln_f (math.cl:283-311) into the caller's rows
    if (e->dtype == G2_F32) {
        if ((rc = forward_rows<float>(e, n, maxp, true))) return rc;
        launch_layernorm<float>(e->h, rows, e->w<float>(e->lnf_g), e->w<float>(e->lnf_b), c.n_embd, n, e->st);
    } else {
        if ((rc = forward_rows<__half>(e, n, maxp, true))) return rc;
        launch_layernorm<__half>(e->h, rows, e->w<__half>(e->lnf_g), e->w<__half>(e->lnf_b), c.n_embd, n, e->st);
    }
    e->launches += 1;
    CKL();
    for (int i = 0; i < n; ++i) e->filled[slots[i]] = pos[i] + 1;
    e->result_slot = -1;
    return sync_and_check(e);   // the caller's collectives run on another stream
}

extern "C" int g2_lm_head_rows(g2_engine *e, int nrows, const float *rows, int v0, int v1, float *best_value,
                               int *best_index) {
    NvtxRange nvtx_range("g2_lm_head_rows");
    if (!e || !rows || !best_value || !best_index) return set_err(G2_ERR_ARG, "g2_lm_head_rows: null argument");
    const ModelConfig &c = e->c;
    const int E = c.n_embd;
    if (nrows < 1 || nrows > e->R) return set_err(G2_ERR_RANGE, "g2_lm_head_rows: %d rows (at most %d)", nrows, e->R);
    if (v0 < 0 || v1 <= v0 || v1 > c.vocab_size || v0 % 4)
        return set_err(G2_ERR_RANGE, "g2_lm_head_rows: rows [%d, %d) of %d (v0 a multiple of 4)", v0, v1, c.vocab_size);
    if (((uintptr_t)rows) & 15) return set_err(G2_ERR_ARG, "g2_lm_head_rows: rows not 16-byte aligned");
    CK(cudaSetDevice(e->device));
    const int W = v1 - v0, Ws = (W + 3) / 4 * 4;   // logits row stride: whole float4s for the argmax
    if ((size_t)nrows * Ws > e->shard_cap) {
        if (e->shard_logits) cudaFree(e->shard_logits);
        e->shard_logits = nullptr;
        e->shard_cap = 0;
        int rc = dalloc(e, &e->shard_logits, (size_t)nrows * Ws);
        if (rc) return rc;
        e->shard_cap = (size_t)nrows * Ws;
    }
    if (e->tc) {
        if (v0 != e->shard_v0 || v1 != e->shard_v1) {   // the operand map of rows [v0, v1) of the head
            int rc;
            const size_t n = (size_t)c.vocab_size * E;
            if (e->tc_kind == TC_TF32X3 && e->tc_lm_w)
                rc = tc_weights_kmajor(&e->tc_lm_shard, TC_TF32X3, e->tc_lm_w + (size_t)v0 * E,
                                       e->tc_lm_w + align_up(n, 64) + (size_t)v0 * E, E, W);
            else if (e->tc_kind == TC_TF32X3)
                rc = tc_weights_kmajor(&e->tc_lm_shard, TC_TF32X3, e->w<float>(e->lm) + (size_t)v0 * E, nullptr, E, W);
            else
                rc = tc_weights_kmajor(&e->tc_lm_shard, TC_F16, e->w<__half>(e->lm) + (size_t)v0 * E, nullptr, E, W);
            if (rc) return set_err(rc, "g2_lm_head_rows: tensor map of vocabulary rows [%d, %d)", v0, v1);
            e->shard_v0 = v0;
            e->shard_v1 = v1;
        }
        // the rows as the GEMM operand (tf32 hi / lo, or fp16), then logits = rows . wte[v0..v1)
        launch_tc_prep(e->tc_kind, rows, e->tc_xhi, e->tc_xlo, reinterpret_cast<__half *>(e->tc_xhi),
                       (long long)nrows * E, e->st);
        Rows rr{e->rows_tok, e->rows_pos, e->rows_slot};
        e->launches += 1 + (e->dtype == G2_F32
                                ? launch_tc_gemm<float>(e->tc_kind, e->tc_lm_shard, e->tc_x_e, nrows, e->tc_part,
                                                        e->tc_part_floats, e->tc_ctr, e->tc_err, nullptr, nullptr,
                                                        e->shard_logits, 0, nullptr, 0, rr, e->sms, e->st, OperandOut(), Ws)
                                : launch_tc_gemm<__half>(e->tc_kind, e->tc_lm_shard, e->tc_x_e, nrows, e->tc_part,
                                                         e->tc_part_floats, e->tc_ctr, e->tc_err, nullptr, nullptr,
                                                         e->shard_logits, 0, nullptr, 0, rr, e->sms, e->st, OperandOut(),
                                                         Ws));
    } else if (e->dtype == G2_F32) {
        launch_lm_head_rows<float>(rows, e->w<float>(e->lm) + (size_t)v0 * E, e->shard_logits, E, W, Ws, nrows, e->st);
        e->launches += 1;
    } else {
        launch_lm_head_rows<__half>(rows, e->w<__half>(e->lm) + (size_t)v0 * E, e->shard_logits, E, W, Ws, nrows, e->st);
        e->launches += 1;
    }
    // per row the first maximum of the range (main.c:1898-1904), as an index into the whole vocabulary
    launch_argmax_rows(e->shard_logits, W, Ws, nrows, 0, best_index, best_value, nullptr, nullptr, nullptr, 0, nullptr,
                       e->st);
    launch_add_ints(best_index, nrows, v0, e->st);
    e->launches += 2;
    CKL();
    return sync_and_check(e);
}

extern "C" int g2_logits(g2_engine *e, int slot, float *host, int n) {
    if (!e || !host) return set_err(G2_ERR_ARG, "g2_logits: null argument");
    int rc;
    if ((rc = check_slot(e, slot))) return rc;
    if (n < 0 || n > e->c.padded_vocab) return set_err(G2_ERR_RANGE, "g2_logits: n %d > padded_vocab", n);
    CK(cudaSetDevice(e->device));
    CK(cudaMemcpyAsync(host, e->logits + (size_t)slot * e->c.padded_vocab, sizeof(float) * n, cudaMemcpyDeviceToHost, e->st));
    return sync_and_check(e);
}

extern "C" int g2_argmax(g2_engine *e, int slot, int forbid_eos, int *token, float *value) {
    NvtxRange nvtx_range("g2_argmax");
    if (!e || !token) return set_err(G2_ERR_ARG, "g2_argmax: null argument");
    int rc;
    if ((rc = check_slot(e, slot))) return rc;
    CK(cudaSetDevice(e->device));
    if (e->result_slot == slot) {
        // the LM-head kernel's argmax (no EOS exclusion); it also answers the
        // EOS-excluding query whenever its token is not EOS
        CK(cudaMemcpyAsync(e->h_small, e->result, 2 * sizeof(int), cudaMemcpyDeviceToHost, e->st));
        if ((rc = sync_and_check(e))) return rc;
        if (!forbid_eos || e->h_small[0] != kEos) {
            *token = e->h_small[0];
            if (value) memcpy(value, &e->h_small[1], 4);
            return G2_OK;
        }
    }
    launch_argmax_rows(e->logits + (size_t)slot * e->c.padded_vocab, e->c.vocab_size, e->c.padded_vocab, 1, forbid_eos,
                       e->argmax_out, reinterpret_cast<float *>(e->argmax_out + 1), nullptr, nullptr, nullptr, 0,
                       nullptr, e->st);
    e->launches += 1;
    CKL();
    CK(cudaMemcpyAsync(e->h_small, e->argmax_out, 2 * sizeof(int), cudaMemcpyDeviceToHost, e->st));
    if ((rc = sync_and_check(e))) return rc;
    *token = e->h_small[0];
    if (value) memcpy(value, &e->h_small[1], 4);
    return G2_OK;
}

extern "C" int g2_sample_device(g2_engine *e, int slot, const int *context_ids, int n_context, int forbid_eos,
                                float temperature, int top_k, float rep_penalty, double u01, int *out_token) {
    NvtxRange nvtx_range("g2_sample_device");
    if (!e || !out_token || n_context < 0 || (n_context > 0 && !context_ids))
        return set_err(G2_ERR_ARG, "g2_sample_device: bad argument");
    int rc;
    if ((rc = check_slot(e, slot))) return rc;
    if (n_context > e->c.n_ctx) return set_err(G2_ERR_RANGE, "g2_sample_device: %d context ids > n_ctx %d", n_context, e->c.n_ctx);
    if (!(u01 >= 0.0 && u01 < 1.0)) return set_err(G2_ERR_ARG, "g2_sample_device: u01 must be in [0, 1)");
    if (e->filled[slot] == 0) return set_err(G2_ERR_STATE, "g2_sample_device: slot %d has no logits yet", slot);
    CK(cudaSetDevice(e->device));
    if (n_context > 0) {
        memcpy(e->h_ctx, context_ids, sizeof(int) * n_context);
        CK(cudaMemcpyAsync(e->sample_ctx, e->h_ctx, sizeof(int) * n_context, cudaMemcpyHostToDevice, e->st));
    }
    launch_sample(e->logits + (size_t)slot * e->c.padded_vocab, e->sample_work, e->c.vocab_size, e->sample_ctx,
                  n_context, forbid_eos, temperature, top_k, rep_penalty, u01, e->argmax_out, e->st);
    e->launches += 1;
    CKL();
    CK(cudaMemcpyAsync(e->h_small, e->argmax_out, sizeof(int), cudaMemcpyDeviceToHost, e->st));
    if ((rc = sync_and_check(e))) return rc;
    *out_token = e->h_small[0];
    return G2_OK;
}

extern "C" int g2_topk(g2_engine *e, int slot, int k, float *values, int *ids) {
    NvtxRange nvtx_range("g2_topk");
    if (!e || !values || !ids) return set_err(G2_ERR_ARG, "g2_topk: null argument");
    int rc;
    if ((rc = check_slot(e, slot))) return rc;
    if (k < 1 || k > G2_MAX_TOPK || k > e->c.vocab_size)
        return set_err(G2_ERR_RANGE, "g2_topk: k %d out of range [1,%d]", k, std::min(G2_MAX_TOPK, e->c.vocab_size));
    if (e->filled[slot] == 0) return set_err(G2_ERR_STATE, "g2_topk: slot %d has no logits yet", slot);
    CK(cudaSetDevice(e->device));
    float *dv = reinterpret_cast<float *>(e->topk_out);
    int *di = e->topk_out + G2_MAX_TOPK;
    launch_topk(e->logits + (size_t)slot * e->c.padded_vocab, e->c.vocab_size, k, dv, di, e->st);
    e->launches += 1;
    CKL();
    CK(cudaMemcpyAsync(values, dv, sizeof(float) * k, cudaMemcpyDeviceToHost, e->st));
    CK(cudaMemcpyAsync(ids, di, sizeof(int) * k, cudaMemcpyDeviceToHost, e->st));
    return sync_and_check(e);
}

extern "C" int g2_synchronize(g2_engine *e) {
    if (!e) return set_err(G2_ERR_ARG, "null engine");
    CK(cudaSetDevice(e->device));
    return sync_and_check(e);
}

extern "C" int g2_last_timing(g2_engine *e, float *prefill_ms, float *decode_ms, int *decode_steps) {
    if (!e) return set_err(G2_ERR_ARG, "null engine");
    if (prefill_ms) *prefill_ms = e->last_prefill_ms;
    if (decode_ms) *decode_ms = e->last_decode_ms;
    if (decode_steps) *decode_steps = e->last_decode_steps;
    return G2_OK;
}

extern "C" int g2_generate(g2_engine *e, int slot, const int *prompt, int n_prompt, int n_new, int min_new,
                           int *out_tokens) {
    NvtxRange nvtx_range("g2_generate");
    if (!e || !prompt || !out_tokens) return set_err(G2_ERR_ARG, "g2_generate: null argument");
    if (n_new < 1) return set_err(G2_ERR_ARG, "g2_generate: n_new must be >= 1");
    int rc;
    if ((rc = check_slot(e, slot))) return rc;
    if (n_prompt < 1 || n_prompt >= e->c.n_ctx) return set_err(G2_ERR_RANGE, "prompt length %d out of range", n_prompt);
    // main.c:2126: generation stops when the sequence reaches the context size
    const int cap = e->c.n_ctx - n_prompt;
    if (n_new > cap) n_new = cap;
    CK(cudaSetDevice(e->device));
    cudaGraphExec_t g = nullptr;
    if (!e->mega && (rc = decode_graph(e, slot, &g))) return rc;
    CK(cudaStreamSynchronize(e->st));
    StepState *hs = e->h_state + e->h_state_i;
    e->h_state_i = (e->h_state_i + 1) % 64;
    *hs = StepState{0, n_prompt - 1, slot, 0, min_new, {0, 0, 0}};
    CK(cudaEventRecord(e->ev[0], e->st));
    CK(cudaMemcpyAsync(e->state, hs, sizeof(StepState), cudaMemcpyHostToDevice, e->st));
    if ((rc = prefill_impl(e, slot, prompt, n_prompt))) return rc;
    rc = e->dtype == G2_F32 ? lm_head_row<float>(e, n_prompt - 1, slot, e->state)
                            : lm_head_row<__half>(e, n_prompt - 1, slot, e->state);
    if (rc) return rc;
    CK(cudaEventRecord(e->ev[1], e->st));
    if (e->mega) {
        if (n_new > 1 && (rc = launch_mega(e, slot, n_new - 1))) return rc;
    } else {
        for (int i = 1; i < n_new; ++i) CK(cudaGraphLaunch(g, e->st));
        e->launches += (long long)(n_new - 1) * e->dec_graph_kernels;
    }
    CK(cudaEventRecord(e->ev[2], e->st));
    CK(cudaMemcpyAsync(out_tokens, e->out_tokens + (size_t)slot * e->c.n_ctx, sizeof(int) * n_new,
                       cudaMemcpyDeviceToHost, e->st));
    if ((rc = sync_and_check(e))) return rc;
    if (e->mega && n_new > 1) dump_trace(e, n_new - 1);
    CK(cudaEventElapsedTime(&e->last_prefill_ms, e->ev[0], e->ev[1]));
    CK(cudaEventElapsedTime(&e->last_decode_ms, e->ev[1], e->ev[2]));
    e->last_decode_steps = n_new - 1;
    e->filled[slot] = n_prompt + n_new - 1;
    e->result_slot = slot;
    // EOS ends generation once it is allowed (main.c:2126, 2135)
    for (int i = 0; i < n_new; ++i)
        if (out_tokens[i] == kEos && i >= min_new) return i + 1;
    return n_new;
}

// One batched greedy decode step for the rows in the device row arrays.
template <typename WT>
static int record_batch_step(g2_engine *e, int n) {
    const ModelConfig &c = e->c;
    int rc = forward_rows<WT>(e, n, e->batch_pos_hint, true);
    if (rc) return rc;
    lm_head_rows<WT>(e, n);
    launch_argmax_rows(e->logits_rows, c.vocab_size, c.padded_vocab, n, 1, nullptr, nullptr, e->rows_tok,
                       e->rows_pos, e->out_tokens, c.n_ctx, e->batch_step, e->st);
    launch_step_advance(e->batch_step, e->st);
    e->launches += 2;
    return G2_OK;
}

extern "C" int g2_generate_batch(g2_engine *e, int n, const int *slots, const int *prompts, const int *prompt_lens,
                                 int n_new, int *out_tokens) {
    NvtxRange nvtx_range("g2_generate_batch");
    if (!e || !slots || !prompts || !prompt_lens || !out_tokens) return set_err(G2_ERR_ARG, "g2_generate_batch: null argument");
    if (n < 1 || n > e->max_batch) return set_err(G2_ERR_RANGE, "batch %d out of range", n);
    if (n_new < 1) return set_err(G2_ERR_ARG, "n_new must be >= 1");
    int rc;
    std::vector<int> seen(e->max_batch, 0);
    for (int i = 0; i < n; ++i) {
        if ((rc = check_slot(e, slots[i]))) return rc;
        if (seen[slots[i]]++) return set_err(G2_ERR_ARG, "slot %d repeated", slots[i]);
        if (prompt_lens[i] < 1 || prompt_lens[i] + n_new - 1 > e->c.n_ctx)
            return set_err(G2_ERR_RANGE, "prompt %d: length %d + %d new exceeds context %d", i, prompt_lens[i], n_new, e->c.n_ctx);
    }
    CK(cudaSetDevice(e->device));
    CK(cudaStreamSynchronize(e->st));
    const ModelConfig &c = e->c;
    CK(cudaEventRecord(e->ev[0], e->st));
    // Prefill; each sequence's greedy token goes to row i of the batch.  Prompts
    // that are whole 64-row tiles share many-row passes of up to R rows (the
    // tensor-core GEMMs then run on more rows at once); others go one by one.
    size_t off = 0;
    bool tiles = e->tc;
    for (int i = 0; i < n; ++i) tiles = tiles && prompt_lens[i] % 64 == 0;
    for (int i = 0; i < n;) {
        int j = i + 1, rows = prompt_lens[i];
        if (tiles)
            while (j < n && rows + prompt_lens[j] <= e->R) rows += prompt_lens[j++];
        if (j == i + 1) {
            if ((rc = prefill_impl(e, slots[i], prompts + off, prompt_lens[i]))) return rc;
        } else {
            std::vector<int> pos(rows), sl(rows);
            int maxp = 0;
            for (int q = i, r = 0; q < j; ++q) {
                for (int t = 0; t < prompt_lens[q]; ++t, ++r) {
                    pos[r] = t;
                    sl[r] = slots[q];
                }
                maxp = std::max(maxp, prompt_lens[q] - 1);
            }
            if ((rc = check_ids(e, prompts + off, rows))) return rc;
            if ((rc = prefill_rows(e, rows, prompts + off, pos.data(), sl.data(), maxp))) return rc;
            for (int q = i; q < j; ++q) e->filled[slots[q]] = prompt_lens[q];
        }
        for (int q = i, r = 0; q < j; r += prompt_lens[q], ++q) {
            rc = e->dtype == G2_F32 ? lm_head_row<float>(e, r + prompt_lens[q] - 1, slots[q], nullptr)
                                    : lm_head_row<__half>(e, r + prompt_lens[q] - 1, slots[q], nullptr);
            if (rc) return rc;
            launch_argmax_rows(e->logits + (size_t)slots[q] * c.padded_vocab, c.vocab_size, c.padded_vocab, 1, 1,
                               e->argmax_out + q, nullptr, nullptr, nullptr, nullptr, 0, nullptr, e->st);
            e->launches += 1;
        }
        for (int q = i; q < j; ++q) off += prompt_lens[q];
        i = j;
    }
    CKL();
    // rows for the decode steps: tok from the prefill argmax, pos = prompt length
    CK(cudaStreamSynchronize(e->st));
    std::vector<int> tok(n), pos(n), sl(n);
    CK(cudaMemcpy(tok.data(), e->argmax_out, sizeof(int) * n, cudaMemcpyDeviceToHost));
    for (int i = 0; i < n; ++i) {
        pos[i] = prompt_lens[i];
        sl[i] = slots[i];
        out_tokens[(size_t)i * n_new] = tok[i];
    }
    if ((rc = stage_rows(e, n, tok.data(), pos.data(), sl.data()))) return rc;
    int one = 1;
    CK(cudaMemcpyAsync(e->batch_step, &one, sizeof(int), cudaMemcpyHostToDevice, e->st));
    CK(cudaEventRecord(e->ev[1], e->st));
    if (n_new > 1) {
        // this generation's last decode position, rounded up to a whole attention chunk
        int last = 0;
        for (int i = 0; i < n; ++i) last = std::max(last, prompt_lens[i] + n_new - 2);
        const int hint = std::min((last / kAttnChunk + 1) * kAttnChunk - 1, e->c.n_ctx - 1);
        if (!e->batch_graph || e->batch_graph_n != n || e->batch_graph_pos < hint) {
            e->batch_pos_hint = hint;
            if (e->batch_graph) cudaGraphExecDestroy(e->batch_graph);
            e->batch_graph = nullptr;
            cudaGraph_t g;
            const long long before = e->launches;
            CK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
            rc = e->dtype == G2_F32 ? record_batch_step<float>(e, n) : record_batch_step<__half>(e, n);
            cudaError_t r = cudaStreamEndCapture(e->st, &g);
            if (rc) return rc;
            if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "batch capture: %s", cudaGetErrorString(r));
            r = cudaGraphInstantiate(&e->batch_graph, g, 0);
            cudaGraphDestroy(g);
            if (r != cudaSuccess) return set_err(G2_ERR_CUDA, "batch graph instantiate: %s", cudaGetErrorString(r));
            e->batch_graph_kernels = (int)(e->launches - before);
            e->launches = before;
            e->batch_graph_n = n;
            e->batch_graph_pos = hint;
        }
        for (int s = 1; s < n_new; ++s) CK(cudaGraphLaunch(e->batch_graph, e->st));
        e->launches += (long long)(n_new - 1) * e->batch_graph_kernels;
    }
    CK(cudaEventRecord(e->ev[2], e->st));
    if ((rc = sync_and_check(e))) return rc;   // an expired GEMM wait of any step is reported here
    for (int i = 0; i < n; ++i) {
        CK(cudaMemcpy(out_tokens + (size_t)i * n_new + 1, e->out_tokens + (size_t)i * c.n_ctx + 1,
                      sizeof(int) * (n_new - 1), cudaMemcpyDeviceToHost));
        e->filled[slots[i]] = prompt_lens[i] + n_new - 1;
    }
    CK(cudaEventElapsedTime(&e->last_prefill_ms, e->ev[0], e->ev[1]));
    CK(cudaEventElapsedTime(&e->last_decode_ms, e->ev[1], e->ev[2]));
    e->last_decode_steps = n_new - 1;
    e->result_slot = -1;
    return G2_OK;
}

// ------------------------------------------------------------------------------
// single-kernel entry points (device pointers)
// ------------------------------------------------------------------------------
static int current_sms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

extern "C" size_t g2k_matvec_workspace(int N, int K) {
    if (N <= 0 || K <= 0) return 0;
    GemvPlan p = gemv_plan<float>(N, K, current_sms());
    return align_up((size_t)p.tiles * 4, 256) + align_up((size_t)p.ksplit * N * 4, 256);
}

extern "C" int g2k_matvec(const float *x, const float *W, const float *bias, const float *residual, float *y, int N,
                          int K, int apply_gelu, const float *ln_gamma, const float *ln_beta, void *workspace,
                          size_t workspace_bytes, void *stream) {
    if (!x || !W || !y || !workspace) return set_err(G2_ERR_ARG, "g2k_matvec: null argument");
    if (N <= 0 || K <= 0 || N % 4 || K % 16) return set_err(G2_ERR_ARG, "g2k_matvec: need N %% 4 == 0, K %% 16 == 0");
    if ((ln_gamma == nullptr) != (ln_beta == nullptr)) return set_err(G2_ERR_ARG, "g2k_matvec: ln_gamma and ln_beta go together");
    if (workspace_bytes < g2k_matvec_workspace(N, K)) return set_err(G2_ERR_ARG, "g2k_matvec: workspace too small");
    if ((uintptr_t)workspace % 256) return set_err(G2_ERR_ARG, "g2k_matvec: workspace not 256-byte aligned");
    GemvPlan p = gemv_plan<float>(N, K, current_sms());
    if (p.smem_bytes > kGemvMaxSmem)
        return set_err(G2_ERR_RANGE, "g2k_matvec: K = %d is too long for one column tile's shared memory at N = %d", K, N);
    unsigned *ctr = reinterpret_cast<unsigned *>(workspace);
    float *partial = reinterpret_cast<float *>((char *)workspace + align_up((size_t)p.tiles * 4, 256));
    const int epi = (bias ? EPI_BIAS : 0) | (apply_gelu ? EPI_GELU : 0) | (residual ? EPI_RESID : 0);
    launch_gemv<float>(x, W, bias, residual, y, N, K, epi, ln_gamma, ln_beta, partial, ctr, p, nullptr, 0, nullptr,
                       nullptr, (cudaStream_t)stream);
    CKL();
    return G2_OK;
}

extern "C" int g2k_matmul(const float *A, const float *B, const float *bias, const float *residual, float *C, int M,
                          int N, int K, int apply_gelu, void *stream) {
    if (!A || !B || !C) return set_err(G2_ERR_ARG, "g2k_matmul: null argument");
    if (M <= 0 || N <= 0 || K <= 0 || K % 16) return set_err(G2_ERR_ARG, "g2k_matmul: need K %% 16 == 0");
    const int epi = (bias ? EPI_BIAS : 0) | (apply_gelu ? EPI_GELU : 0) | (residual ? EPI_RESID : 0);
    launch_gemm_rows<float>(A, B, bias, residual, C, M, N, K, epi, nullptr, 0, Rows{nullptr, nullptr, nullptr},
                            (cudaStream_t)stream);
    CKL();
    return G2_OK;
}

// Workspace of g2k_matmul_tc: [err + tile counters | A hi | A lo | B hi | B lo | partial sums],
// 256-byte aligned parts.
static size_t tc_ws_layout(int M, int N, int K, int precision, int sms, size_t off[6]) {
    const int kind = precision == G2_F16 ? TC_F16 : TC_TF32X3;
    const size_t es = kind == TC_F16 ? 2 : 4;
    const size_t sz[6] = {256 + (size_t)kTcMaxTiles * 4, (size_t)M * K * es, kind == TC_F16 ? 0 : (size_t)M * K * 4,
                          (size_t)K * N * es, kind == TC_F16 ? 0 : (size_t)K * N * 4,
                          tc_partial_floats(M, N, K, kind, sms) * 4};
    size_t o = 0;
    for (int i = 0; i < 6; ++i) {
        off[i] = o;
        o += align_up(sz[i], 256);
    }
    return o;
}
static int device_sms() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

extern "C" size_t g2k_matmul_tc_workspace(int M, int N, int K, int precision) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    size_t off[6];
    return tc_ws_layout(M, N, K, precision, device_sms(), off);
}

extern "C" int g2k_matmul_tc(const float *A, const float *B, const float *bias, const float *residual, float *C, int M,
                             int N, int K, int apply_gelu, int precision, void *workspace, size_t workspace_bytes,
                             void *stream) {
    if (!A || !B || !C || !workspace) return set_err(G2_ERR_ARG, "g2k_matmul_tc: null argument");
    if (precision != G2_F32 && precision != G2_F16) return set_err(G2_ERR_ARG, "g2k_matmul_tc: bad precision");
    if (M <= 0 || N <= 0 || K <= 0 || K % 64 || N % 8)
        return set_err(G2_ERR_ARG, "g2k_matmul_tc: need K %% 64 == 0 and N %% 8 == 0");
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)C) & 15) return set_err(G2_ERR_ARG, "g2k_matmul_tc: pointers not 16-byte aligned");
    if ((uintptr_t)workspace % 256) return set_err(G2_ERR_ARG, "g2k_matmul_tc: workspace not 256-byte aligned");
    const int sms = device_sms();
    size_t off[6];
    if (workspace_bytes < tc_ws_layout(M, N, K, precision, sms, off)) return set_err(G2_ERR_ARG, "g2k_matmul_tc: workspace too small");
    const int kind = precision == G2_F16 ? TC_F16 : TC_TF32X3;
    char *ws = static_cast<char *>(workspace);
    cudaStream_t st = (cudaStream_t)stream;
    int *err = reinterpret_cast<int *>(ws);
    unsigned *ctr = reinterpret_cast<unsigned *>(ws + 256);
    CK(cudaMemsetAsync(ws, 0, 256 + (size_t)kTcMaxTiles * 4, st));
    float *ahi = reinterpret_cast<float *>(ws + off[1]), *alo = reinterpret_cast<float *>(ws + off[2]);
    float *bhi = reinterpret_cast<float *>(ws + off[3]), *blo = reinterpret_cast<float *>(ws + off[4]);
    launch_tc_prep(kind, A, ahi, alo, reinterpret_cast<__half *>(ahi), (long long)M * K, st);
    launch_tc_prep(kind, B, bhi, blo, reinterpret_cast<__half *>(bhi), (long long)K * N, st);
    TcWeights w;
    TcRowsOperand x;
    int rc = tc_weights(&w, kind, bhi, blo, K, N);
    if (!rc) rc = tc_rows_operand(&x, kind, ahi, alo, K, M);
    if (rc) return set_err(rc, "g2k_matmul_tc: tensor map encoding failed");
    const int epi = (bias ? EPI_BIAS : 0) | (apply_gelu ? EPI_GELU : 0) | (residual ? EPI_RESID : 0);
    if (((size_t)(N + kTcTileF - 1) / kTcTileF) * ((M + 31) / 32) > (size_t)kTcMaxTiles)
        return set_err(G2_ERR_RANGE, "g2k_matmul_tc: more than %d output tiles", kTcMaxTiles);
    launch_tc_gemm<float>(kind, w, x, M, reinterpret_cast<float *>(ws + off[5]),
                          tc_partial_floats(M, N, K, kind, sms), ctr, err, bias, residual, C, epi, nullptr, 0,
                          Rows{nullptr, nullptr, nullptr}, sms, st);
    CKL();
    return G2_OK;
}

extern "C" int g2k_layernorm(const float *x, float *out, const float *gamma, const float *beta, int n_embd, int rows,
                             void *stream) {
    if (!x || !out || !gamma || !beta) return set_err(G2_ERR_ARG, "g2k_layernorm: null argument");
    if (n_embd <= 0 || rows <= 0) return set_err(G2_ERR_ARG, "g2k_layernorm: bad size");
    launch_layernorm<float>(x, out, gamma, beta, n_embd, rows, (cudaStream_t)stream);
    CKL();
    return G2_OK;
}

extern "C" int g2k_topk(const float *logits, int n, int k, float *values, int *ids, void *stream) {
    if (!logits || !values || !ids) return set_err(G2_ERR_ARG, "g2k_topk: null argument");
    if (n < 1 || k < 1 || k > G2_MAX_TOPK || k > n)
        return set_err(G2_ERR_RANGE, "g2k_topk: need 1 <= k <= min(%d, n), n >= 1 (k %d, n %d)", G2_MAX_TOPK, k, n);
    launch_topk(logits, n, k, values, ids, (cudaStream_t)stream);
    CKL();
    return G2_OK;
}

extern "C" size_t g2k_attention_workspace(int n_head, int max_seq) {
    if (n_head <= 0 || max_seq <= 0) return 0;
    return 256 + align_up(attn_counter_count(1, n_head) * 4, 256) + align_up(attn_partial_floats(1, n_head, max_seq) * 4, 256);
}

extern "C" int g2k_attention(const float *q, const float *K, const float *V, float *out, int n_head, int max_seq,
                             int T_kv, void *workspace, size_t workspace_bytes, void *stream) {
    if (!q || !K || !V || !out || !workspace) return set_err(G2_ERR_ARG, "g2k_attention: null argument");
    if (n_head <= 0 || max_seq <= 0 || max_seq > kMaxSeq || T_kv < 1 || T_kv > max_seq)
        return set_err(G2_ERR_RANGE, "g2k_attention: need 1 <= T_kv <= max_seq <= %d", kMaxSeq);
    if (workspace_bytes < g2k_attention_workspace(n_head, max_seq)) return set_err(G2_ERR_ARG, "g2k_attention: workspace too small");
    if ((uintptr_t)workspace % 256) return set_err(G2_ERR_ARG, "g2k_attention: workspace not 256-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    int *rowinfo = reinterpret_cast<int *>(workspace);   // [0] = pos, [1] = slot, [2] = token
    unsigned *ctr = reinterpret_cast<unsigned *>((char *)workspace + 256);
    float *partial = reinterpret_cast<float *>((char *)workspace + 256 + align_up(attn_counter_count(1, n_head) * 4, 256));
    launch_set_ints(rowinfo, T_kv - 1, 0, 0, 0, st);   // pos, slot, token (no host copy: graph-capturable)
    KVLayout kv;
    kv.k = const_cast<float *>(K);
    kv.v = const_cast<float *>(V);
    kv.slot_stride = 0;
    kv.layer_stride = 0;
    kv.max_seq = max_seq;
    kv.n_head = n_head;
    launch_attention<float>(q, n_head * kHeadDim, kv, 0, Rows{rowinfo + 2, rowinfo, rowinfo + 1}, 1, out,
                            n_head * kHeadDim, partial, ctr, T_kv - 1, st);
    CKL();
    return G2_OK;
}
