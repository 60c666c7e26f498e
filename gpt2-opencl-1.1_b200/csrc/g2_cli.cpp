// g2_cli.cpp -- command-line text generation on the engine: the host flow of
// the reference's main() (main.c:1966-2160) over the C ABI.
//
//   gpt2b200 --model DIR [--device N] [--temperature T] [--top-k K]
//            [--rep-penalty P] [--max-tokens N] [--min-tokens N] [--seed N]
//            [--greedy] [--prompt TEXT] [--host-sampler]
//   gpt2b200 --list-devices
//
// Same flags and defaults as the reference (temperature 0.8, top-k 40,
// repetition penalty 1.1, 32 tokens, EOS forbidden for the first token, seed
// from time()).  Per prompt: encode (at most n_ctx - 1 ids), prefill, sample
// the first token (EOS forbidden while fewer than --min-tokens are out), then
// decode + sample until --max-tokens, EOS or a full context.  Sampling runs on
// the device (g2_sample_device) with the uniform draw taken from the C
// library's rand() seeded by --seed -- rand() is drawn only for a stochastic
// pick, as in the reference, so the sequence of draws is the reference's;
// --host-sampler copies the logits back and samples on the host (g2_sample)
// instead.  Generated text is printed incrementally: the generated ids are
// re-decoded and only the new bytes written (the reference's emit_new_bytes).
// Without --prompt, prompts are read one per line from standard input.
#include <cuda_runtime.h>
#include <sys/time.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <string>
#include <vector>

#include "gpt2b200.h"

namespace {

double now_s() {
    struct timeval tv;
    gettimeofday(&tv, nullptr);
    return (double)tv.tv_sec + 1e-6 * (double)tv.tv_usec;
}

struct Opts {
    const char *model = nullptr, *prompt = nullptr;
    int device = 0, top_k = 40, max_tokens = 32, min_tokens = 1;
    float temperature = 0.8f, rep_penalty = 1.1f;
    unsigned seed = 0;
    bool seed_set = false, list_devices = false, host_sampler = false;
};

int usage(const char *argv0) {
    fprintf(stderr,
            "Usage: %s --model <dir> [options]\n"
            "       %s --list-devices\n"
            "Options:\n"
            "  --device N         CUDA device index (default 0)\n"
            "  --temperature T    sampling temperature (default 0.8; 0 = greedy)\n"
            "  --top-k K          top-K filter (default 40; 0 = off)\n"
            "  --rep-penalty P    repetition penalty (default 1.1; 1.0 = off)\n"
            "  --max-tokens N     stop after N generated tokens (default 32)\n"
            "  --min-tokens N     forbid EOS for the first N tokens (default 1)\n"
            "  --seed N           RNG seed (default: time(NULL))\n"
            "  --greedy           shorthand for --temperature 0\n"
            "  --prompt TEXT      run one generation and exit\n"
            "  --host-sampler     sample on the host from copied logits\n",
            argv0, argv0);
    return EXIT_FAILURE;
}

int parse(int argc, char **argv, Opts &o) {
    for (int i = 1; i < argc; ++i) {
        const char *a = argv[i];
        const bool has = i + 1 < argc;
        if (!strcmp(a, "--model") && has) o.model = argv[++i];
        else if (!strcmp(a, "--device") && has) o.device = atoi(argv[++i]);
        else if (!strcmp(a, "--list-devices")) o.list_devices = true;
        else if (!strcmp(a, "--temperature") && has) o.temperature = (float)atof(argv[++i]);
        else if (!strcmp(a, "--top-k") && has) o.top_k = atoi(argv[++i]);
        else if (!strcmp(a, "--rep-penalty") && has) o.rep_penalty = (float)atof(argv[++i]);
        else if (!strcmp(a, "--max-tokens") && has) o.max_tokens = atoi(argv[++i]) < 1 ? 1 : atoi(argv[i]);
        else if (!strcmp(a, "--min-tokens") && has) o.min_tokens = atoi(argv[++i]) < 1 ? 1 : atoi(argv[i]);
        else if (!strcmp(a, "--seed") && has) {
            o.seed = (unsigned)strtoul(argv[++i], nullptr, 10);
            o.seed_set = true;
        } else if (!strcmp(a, "--greedy")) o.temperature = 0.0f;
        else if (!strcmp(a, "--prompt") && has) o.prompt = argv[++i];
        else if (!strcmp(a, "--host-sampler")) o.host_sampler = true;
        else if (!o.model && !o.list_devices && a[0] != '-') o.model = a;
        else return -1;
    }
    return 0;
}

// One sampled token from the logits of slot 0 (main.c:1872-1939).
int sample(g2_engine *e, const Opts &o, const std::vector<int> &ctx, int forbid_eos, int vocab, std::vector<float> &lg,
           int *tok) {
    if (o.host_sampler) {
        int rc = g2_logits(e, 0, lg.data(), vocab);
        if (rc) return rc;
        return g2_sample(lg.data(), vocab, ctx.data(), (int)ctx.size(), forbid_eos, o.temperature, o.top_k,
                         o.rep_penalty, tok);
    }
    const double u = o.temperature > 0.0f ? (double)rand() / ((double)RAND_MAX + 1.0) : 0.0;
    return g2_sample_device(e, 0, ctx.data(), (int)ctx.size(), forbid_eos, o.temperature, o.top_k, o.rep_penalty, u,
                            tok);
}

void emit_new(const g2_tokenizer *tk, const std::vector<int> &gen, std::vector<char> &buf, int &printed) {
    const int n = g2_tok_decode(tk, gen.data(), (int)gen.size(), buf.data(), (int)buf.size());
    if (n > printed) {
        fwrite(buf.data() + printed, 1, (size_t)(n - printed), stdout);
        fflush(stdout);
        printed = n;
    }
}

}  // namespace

int main(int argc, char **argv) {
    Opts o;
    if (parse(argc, argv, o) || (!o.model && !o.list_devices)) return usage(argv[0]);
    if (o.list_devices) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
        for (int d = 0; d < n; ++d) {
            cudaDeviceProp p;
            if (cudaGetDeviceProperties(&p, d) == cudaSuccess)
                printf("[%d] %s  sm_%d%d  %d SMs  %.1f GiB\n", d, p.name, p.major, p.minor, p.multiProcessorCount,
                       (double)p.totalGlobalMem / (1024.0 * 1024.0 * 1024.0));
        }
        if (n == 0) printf("no CUDA devices\n");
        return EXIT_SUCCESS;
    }
    if (!o.seed_set) o.seed = (unsigned)time(nullptr);
    srand(o.seed);
    if (o.temperature <= 0.0f)
        printf("Sampling: greedy min_tokens=%d%s\n", o.min_tokens, o.rep_penalty > 1.0f ? " (with repetition penalty)" : "");
    else
        printf("Sampling: temperature=%.3f top_k=%d rep_penalty=%.3f min_tokens=%d seed=%u\n", o.temperature, o.top_k,
               o.rep_penalty, o.min_tokens, o.seed);
    if (o.top_k > G2_MAX_TOPK) fprintf(stderr, "Warning: top-k clamped from %d to %d (MAX_TOPK).\n", o.top_k, G2_MAX_TOPK);

    g2_engine *e = nullptr;
    if (g2_open(o.model, o.device, 1, G2_F32, &e)) {
        fprintf(stderr, "Failed to load the model from %s: %s\n", o.model, g2_last_error());
        return EXIT_FAILURE;
    }
    g2_config cfg;
    g2_get_config(e, &cfg);
    g2_tokenizer *tk = nullptr;
    if (g2_tokenizer_load(o.model, &tk)) {
        fprintf(stderr, "Failed to load tokenizer from %s\n", o.model);
        g2_close(e);
        return EXIT_FAILURE;
    }
    printf("Tokenizer: %d tokens.\n", g2_tokenizer_vocab_size(tk));
    const bool interactive = isatty(STDIN_FILENO) && !o.prompt;
    const int S = cfg.n_ctx;
    std::vector<int> ids(S), gen;
    std::vector<float> lg(cfg.padded_vocab);
    std::vector<char> text((size_t)16 * S + 16);
    int status = EXIT_SUCCESS;
    std::string line;
    for (;;) {
        if (interactive) {
            printf("> ");
            fflush(stdout);
        }
        if (o.prompt) {
            line = o.prompt;
        } else {
            char buf[1024];
            if (!fgets(buf, sizeof buf, stdin)) break;
            buf[strcspn(buf, "\n")] = 0;
            line = buf;
        }
        if (line.empty()) {
            if (!interactive) break;
            continue;
        }
        const int n_prompt = g2_tok_encode(tk, line.c_str(), ids.data(), S - 1);   // one slot left for a token
        if (n_prompt <= 0) {
            if (!interactive) {
                status = EXIT_FAILURE;
                break;
            }
            continue;
        }
        std::vector<int> ctx(ids.begin(), ids.begin() + n_prompt);
        gen.clear();
        int printed = 0, next = 0, rc;
        const double t0 = now_s();
        if ((rc = g2_prefill(e, 0, ctx.data(), n_prompt)) ||
            (rc = sample(e, o, ctx, 0 < o.min_tokens, cfg.vocab_size, lg, &next))) {
            fprintf(stderr, "generation failed: %s\n", g2_last_error());
            status = EXIT_FAILURE;
            break;
        }
        ctx.push_back(next);
        if (next != G2_EOS) {
            gen.push_back(next);
            emit_new(tk, gen, text, printed);
        }
        const double t1 = now_s();
        int generated = 1;
        while (generated < o.max_tokens && next != G2_EOS && (int)ctx.size() < S) {
            if ((rc = g2_decode(e, 0, ctx.back(), (int)ctx.size() - 1)) ||
                (rc = sample(e, o, ctx, generated < o.min_tokens, cfg.vocab_size, lg, &next))) {
                fprintf(stderr, "generation failed: %s\n", g2_last_error());
                status = EXIT_FAILURE;
                break;
            }
            ctx.push_back(next);
            ++generated;
            if (next == G2_EOS) break;
            gen.push_back(next);
            emit_new(tk, gen, text, printed);
        }
        const double t2 = now_s();
        printf("\n");
        const int steps = generated - 1;
        printf("[%d prompt tokens, prefill %.2f ms; %d decode steps, %.3f ms/token, %.1f tok/s]\n", n_prompt,
               1e3 * (t1 - t0), steps, steps > 0 ? 1e3 * (t2 - t1) / steps : 0.0, steps > 0 ? steps / (t2 - t1) : 0.0);
        if (status != EXIT_SUCCESS || o.prompt) break;
    }
    g2_tokenizer_free(tk);
    g2_close(e);
    return status;
}
