// g2_loader.h -- config.json and safetensors reading for the engine.
#pragma once
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

namespace g2 {

struct ModelConfig {
    int n_layer = 12, n_embd = 768, n_head = 12, n_ctx = 1024, vocab_size = 50257, ffn_dim = 3072;
    int padded_vocab = 50260;
};

// load_config (main.c:294-331): integer keys found by name, GPT-2 small
// defaults when config.json is absent; n_ctx from "n_positions" or "n_ctx";
// ffn = n_inner or 4 * n_embd.  The reference's compile-time ceilings
// (main.c:47-52) are not imposed except n_ctx <= 1024 and head size 64.
// Returns 0 or a G2_ERR_* code with `err` set.
int load_config(const std::string &dir, ModelConfig &c, std::string &err);

enum StDtype { ST_F32 = 0, ST_F16 = 1, ST_BF16 = 2, ST_OTHER = 3 };

struct StTensor {
    std::string name;
    int dtype = ST_OTHER;
    std::vector<int64_t> shape;
    int64_t begin = -1, end = -1;
    int64_t numel() const {
        int64_t n = 1;
        for (auto s : shape) n *= s;
        return n;
    }
};

class SafeTensors {
  public:
    ~SafeTensors();
    int open(const std::string &path, std::string &err);
    // Lookup with the reference's prefixes (main.c:1194-1207): name,
    // "transformer." + name, "model." + name.
    const StTensor *find(const std::string &name) const;
    // Read a tensor and convert to float.
    int read_f32(const StTensor &t, float *out, std::string &err);
    const std::vector<StTensor> &tensors() const { return tensors_; }

  private:
    FILE *fp_ = nullptr;
    int64_t data_start_ = 0;
    int64_t file_size_ = 0;
    std::vector<StTensor> tensors_;
};

// Check config + model.safetensors without touching a device: every GPT-2
// tensor present, with the element count and 2-D shape (Conv1D or Linear
// layout, main.c:1234-1300) the config implies and a float dtype.
int validate_gpt2(const std::string &dir, const ModelConfig &c, std::string &err);

}  // namespace g2
