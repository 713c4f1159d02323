// ref_gguf.cpp -- TEST INFRASTRUCTURE ONLY.  A C shim over NexusLLM's own
// GGUF loader (UniversalModelLoader::load_gguf, src/model_loader.cpp:416-836,
// with MemoryTierManager, src/memory_tier.cpp), compiled unmodified from the
// reference sources by `make -C oracle ref-gguf REF=<checkout>` into
// oracle/_ref/libnexus_ref_gguf.so.  The tests (and tests/golden/
// make_golden.py) use it to pin the library's GGUF parser: metadata, which
// names resolve, each tensor's dtype, dims and data pointer.
#include <cstdint>
#include <cstring>
#include <memory>

#include "memory_tier.hpp"
#include "model_loader.hpp"

struct RefGgufModel {
    char architecture[64];
    uint32_t vocab_size, hidden_size, intermediate_size, num_hidden_layers;
    uint32_t num_attention_heads, num_key_value_heads, max_position_embeddings;
    float rms_norm_eps, rope_theta;
    uint32_t is_moe, num_experts, num_experts_per_tok;
    uint64_t loaded_tensor_count;
};

struct RefGgufTensor {
    int32_t found;
    int32_t dtype;          // nexus::DataType value
    uint32_t n_dims;
    uint64_t dims[8];
    uint64_t byte_size;     // TensorView::byte_size (TensorShape::total_bytes)
    uint64_t fnv;           // FNV-1a of hash_bytes[i] bytes at the tensor's host pointer
};

static uint64_t fnv1a(const uint8_t* p, uint64_t n) {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t i = 0; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
}

// Loads `path` with the reference loader and looks up `n` names.  Returns the
// loader's NexusStatus.
extern "C" __attribute__((visibility("default"))) int32_t ref_gguf_load(const char* path, RefGgufModel* model,
                                                                         const char* const* names,
                                                                         const uint64_t* hash_bytes, uint32_t n,
                                                                         RefGgufTensor* out) {
    auto tiers = std::make_shared<nexus::MemoryTierManager>(size_t(1) << 20, size_t(1) << 20);
    nexus::UniversalModelLoader loader(tiers);
    const int32_t st = (int32_t)loader.load_gguf(path);
    const nexus::ModelMetadata& m = loader.get_metadata();
    memset(model, 0, sizeof(*model));
    strncpy(model->architecture, m.architecture.c_str(), sizeof(model->architecture) - 1);
    model->vocab_size = m.vocab_size;
    model->hidden_size = m.hidden_size;
    model->intermediate_size = m.intermediate_size;
    model->num_hidden_layers = m.num_hidden_layers;
    model->num_attention_heads = m.num_attention_heads;
    model->num_key_value_heads = m.num_key_value_heads;
    model->max_position_embeddings = m.max_position_embeddings;
    model->rms_norm_eps = m.rms_norm_eps;
    model->rope_theta = m.rope_theta;
    model->is_moe = m.is_moe;
    model->num_experts = m.num_experts;
    model->num_experts_per_tok = m.num_experts_per_tok;
    model->loaded_tensor_count = loader.get_loaded_tensor_count();
    for (uint32_t i = 0; i < n; ++i) {
        RefGgufTensor& t = out[i];
        memset(&t, 0, sizeof(t));
        nexus::TensorView* v = tiers->get_tensor_view(names[i]);
        if (!v) continue;
        t.found = 1;
        t.dtype = (int32_t)v->dtype;
        t.n_dims = (uint32_t)std::min<size_t>(8, v->shape.dims.size());
        for (uint32_t d = 0; d < t.n_dims; ++d) t.dims[d] = v->shape.dims[d];
        t.byte_size = v->byte_size;
        t.fnv = fnv1a(static_cast<const uint8_t*>(v->host_ptr), hash_bytes[i]);
    }
    return st;
}
