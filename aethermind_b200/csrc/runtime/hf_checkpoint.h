// Hugging Face checkpoint directory reader (host side): config.json plus
// model.safetensors, or model.safetensors.index.json and its shards.
//
// Follows the reference's HF loader contract (src/model/model_loader.cpp:12-55,
// src/model/formats/hf/hf_directory_reader.cpp:425-576,
// hf_safetensors_file.cpp, hf_safetensors_index.cpp, hf_weight_resolver.cpp):
// the directory layouts it accepts, the Llama config fields it reads and the
// tensor names it resolves (model.embed_tokens.weight, model.norm.weight,
// lm_head.weight optional when tied, model.layers.<i>.{input_layernorm,
// post_attention_layernorm, self_attn.{q,k,v,o}_proj, mlp.{gate,up,down}_proj}
// .weight). Tensor payloads are memory-mapped read-only; nothing is copied
// until the caller uploads a tensor to the device.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "runtime/status.h"

namespace aethermind {
namespace hf {

enum class TensorDtype { kF32, kBF16, kF16 };

struct TensorInfo {
    TensorDtype dtype = TensorDtype::kF32;
    std::vector<int64_t> shape;
    const uint8_t* data = nullptr;  // inside the file's read-only mapping
    size_t bytes = 0;
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
};

struct LlamaConfig {
    int64_t vocab = 0, hidden = 0, layers = 0, n_q_heads = 0, n_kv_heads = 0, head_dim = 0, inter = 0;
    int64_t max_position_embeddings = 0;
    double rope_theta = 10000.0;
    float rms_eps = 1e-5f;
    bool tied_embeddings = false;
};

class MappedFile;

class Checkpoint {
public:
    ~Checkpoint();
    // Opens a checkpoint directory: parses config.json and every safetensors
    // header. NotFound for a missing directory or file, InvalidArgument for
    // malformed JSON, headers, dtypes or shapes.
    static StatusOr<std::unique_ptr<Checkpoint>> Open(const std::string& dir);

    const LlamaConfig& config() const { return config_; }
    // The named tensor; InvalidArgument naming it when it is absent.
    StatusOr<const TensorInfo*> Get(const std::string& name) const;
    bool Has(const std::string& name) const { return tensors_.count(name) != 0; }
    size_t size() const { return tensors_.size(); }

private:
    Status AddFile(const std::string& path);
    LlamaConfig config_;
    std::vector<std::unique_ptr<MappedFile>> files_;
    std::map<std::string, TensorInfo> tensors_;
};

}  // namespace hf
}  // namespace aethermind
