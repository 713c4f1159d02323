// gguf_file.cuh -- host side of the GGUF file -> device upload path
// (nexus_gpu_gguf_* in include/nexus_gpu.h).
//
// Parse: the file is memory-mapped read-only and walked with a bounds-checked
// reader: header, metadata key/values, tensor table, aligned data section
// (the layout UniversalModelLoader::load_gguf reads, src/model_loader.cpp:
// 508-720).  Model metadata follows the reference's key rules and fallbacks
// (model_loader.cpp:538-653, 793-824) so an engine sees the same numbers.
//
// Upload: the chosen tensors form one device image, each tensor on a 256-byte
// boundary.  The image goes up in 64 MiB pieces through a ring of pinned
// staging buffers: host threads copy a piece out of the mapping (page cache)
// into a staging buffer while the previous pieces' host-to-device copies run,
// one cudaMemcpyAsync per piece.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace nexus_gpu {
namespace gguf {

// ggml tensor types: (elements, bytes) per block -- the published block
// layouts -- and the NexusLLM DataType each one is (include/nexus_common.hpp:
// 244-260), -1 where NexusLLM has none.
struct TypeInfo {
    uint32_t elems, bytes;
    int32_t dtype;
};

inline bool type_info(uint32_t t, TypeInfo& ti) {
    switch (t) {
        case 0: ti = {1, 4, 0}; return true;        // F32  -> FP32
        case 1: ti = {1, 2, 1}; return true;        // F16  -> FP16
        case 2: ti = {32, 18, 7}; return true;      // Q4_0 -> GGUF_Q4_0
        case 3: ti = {32, 20, -1}; return true;     // Q4_1 (scale and min per block)
        case 6: ti = {32, 22, 10}; return true;     // Q5_0 -> GGUF_Q5_0
        case 7: ti = {32, 24, -1}; return true;     // Q5_1
        case 8: ti = {32, 34, 9}; return true;      // Q8_0 -> GGUF_Q8_0
        case 9: ti = {32, 36, -1}; return true;     // Q8_1
        case 10: ti = {256, 84, 13}; return true;   // Q2_K -> GGUF_Q2_K
        case 11: ti = {256, 110, 14}; return true;  // Q3_K -> GGUF_Q3_K
        case 12: ti = {256, 144, 8}; return true;   // Q4_K -> GGUF_Q4_K
        case 13: ti = {256, 176, 11}; return true;  // Q5_K -> GGUF_Q5_K
        case 14: ti = {256, 210, 12}; return true;  // Q6_K -> GGUF_Q6_K
        case 15: ti = {256, 292, -1}; return true;  // Q8_K
        case 24: ti = {1, 1, -1}; return true;      // I8
        case 25: ti = {1, 2, -1}; return true;      // I16
        case 26: ti = {1, 4, -1}; return true;      // I32
        case 27: ti = {1, 8, -1}; return true;      // I64
        case 28: ti = {1, 8, -1}; return true;      // F64
        case 30: ti = {1, 2, 2}; return true;       // BF16 -> BF16
        default: return false;                      // IQ* and unknown types: size not known here
    }
}

// dtypes nexus_gpu_gemv serves (NexusLLM DataType values)
inline bool served(int32_t dtype) { return dtype == 1 || dtype == 7 || dtype == 9 || dtype == 11 || dtype == 12; }

struct Tensor {
    std::string name;
    uint32_t n_dims = 0, ggml_type = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t rel_offset = 0, file_offset = 0, bytes = 0;
    int32_t dtype = -1;
};

// NexusLLM's ModelMetadata fields with its defaults (include/model_loader.hpp:10-26).
struct Model {
    std::string architecture = "llama";
    uint32_t vocab = 32000, hidden = 4096, ffn = 11008, layers = 32, heads = 32, kv_heads = 32, ctx = 4096;
    float eps = 1e-5f, rope = 10000.0f;
    bool moe = false;
    uint32_t experts = 0, experts_per_tok = 0;
};

struct Staging {
    void* host = nullptr;
    cudaEvent_t done = nullptr;
    bool busy = false;
};

struct File {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;  // general.alignment as stored (validated after the metadata)
    uint64_t data_offset = 0, skipped = 0;
    Model model;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
    std::unordered_map<std::string, size_t> by_role;  // canonical key (role_key) -> first such tensor
    int device = -1;
    std::vector<Staging> ring;  // pinned staging buffers of the upload, made on first use
};

constexpr size_t kStageBytes = size_t(64) << 20;
constexpr int kStages = 4;
constexpr uint64_t kImageAlign = 256;

// Bounds-checked little-endian reader over the mapping.
struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    template <class T>
    bool get(T& v) {
        if ((size_t)(end - p) < sizeof(T)) return false;
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return true;
    }
    bool skip(uint64_t n) {
        if ((uint64_t)(end - p) < n) return false;
        p += n;
        return true;
    }
    bool str(std::string& s) {
        uint64_t n;
        if (!get(n) || (uint64_t)(end - p) < n) return false;
        s.assign(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return true;
    }
};

// Bytes of a scalar GGUF value type (0 for string / array / unknown).
inline uint64_t scalar_bytes(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;    // u8, i8, bool
        case 2: case 3: return 2;            // u16, i16
        case 4: case 5: case 6: return 4;    // u32, i32, f32
        case 10: case 11: case 12: return 8; // u64, i64, f64
        default: return 0;
    }
}

// Skips one value of type t (arrays of arrays included, to a fixed depth).
inline bool skip_value(Reader& r, uint32_t t, int depth = 0) {
    if (t == 8) {
        std::string s;
        return r.str(s);
    }
    if (t == 9) {
        uint32_t et;
        uint64_t n;
        if (depth > 3 || !r.get(et) || !r.get(n)) return false;
        if (const uint64_t b = scalar_bytes(et)) return n <= (uint64_t)(r.end - r.p) / b && r.skip(n * b);
        for (uint64_t i = 0; i < n; ++i)
            if (!skip_value(r, et, depth + 1)) return false;
        return true;
    }
    const uint64_t b = scalar_bytes(t);
    return b != 0 && r.skip(b);
}

inline bool has(const std::string& key, const char* part) { return key.find(part) != std::string::npos; }

// A numeric metadata value, read as the reference reads it
// (model_loader.cpp:598-631): the unsigned bits of integers, floats also
// truncated to an integer.
inline void apply_number(Model& m, uint64_t& alignment, const std::string& key, uint64_t u, float f) {
    if (key == "general.alignment") alignment = u > 0 ? u : 32;
    else if (has(key, ".context_length")) m.ctx = (uint32_t)u;
    else if (has(key, ".embedding_length")) m.hidden = (uint32_t)u;
    else if (has(key, ".feed_forward_length")) m.ffn = (uint32_t)u;
    else if (has(key, ".block_count")) m.layers = (uint32_t)u;
    else if (has(key, ".attention.head_count_kv")) m.kv_heads = (uint32_t)u;
    else if (has(key, ".attention.head_count")) m.heads = (uint32_t)u;
    else if (has(key, ".rope.freq_base")) m.rope = f > 0.0f ? f : (float)u;
    else if (has(key, ".layer_norm_rms_epsilon") || has(key, ".rms_norm_eps")) m.eps = f > 0.0f ? f : 1e-5f;
    else if (has(key, ".vocab_size")) m.vocab = (uint32_t)u;
    else if (has(key, ".expert_count")) {
        m.experts = (uint32_t)u;
        m.moe = m.experts > 1;
    } else if (has(key, ".expert_used_count")) m.experts_per_tok = (uint32_t)u;
}

inline uint64_t float_to_u64(double d) { return d >= 0.0 && d < 1.8446744073709552e19 ? (uint64_t)d : 0; }

// Layer index in "blk.N.", "model.layers.N." or "layers.N." names
// (model_loader.cpp:752-788); -1 if none.
inline long layer_index(const std::string& name) {
    long best = -1;
    auto num_after = [&](size_t pos) {
        const size_t dot = name.find('.', pos);
        if (dot == std::string::npos || dot == pos) return;
        long v = 0;
        for (size_t i = pos; i < dot; ++i) {
            if (name[i] < '0' || name[i] > '9' || v > 100000000) return;
            v = v * 10 + (name[i] - '0');
        }
        best = std::max(best, v);
    };
    size_t p = name.find("blk.");
    if (p != std::string::npos) num_after(p + 4);
    p = name.find("model.layers.");
    if (p != std::string::npos) num_after(p + 13);
    p = name.find("layers.");
    if (p != std::string::npos && name.find("model.layers.") == std::string::npos) num_after(p + 7);
    return best;
}

// Canonical key of a tensor name: the equivalence classes of the reference's
// alias table (UniversalModelLoader::register_aliases, model_loader.cpp:60-
// 302) for the embeddings, the LM head, the output norm and the per-layer
// norms, projections and QKV biases.  "" for other names (MTP heads included).
inline std::string role_key(const std::string& name) {
    auto any = [&](const std::string& v, std::initializer_list<const char*> names) {
        for (const char* n : names)
            if (v == n) return true;
        return false;
    };
    if (any(name, {"token_embd", "token_embd.weight", "model.embed_tokens.weight", "tok_embeddings.weight",
                   "embeddings.weight", "embed_tokens.weight"}))
        return "token_embd";
    if (any(name, {"lm_head", "lm_head.weight", "output.weight", "output", "model.lm_head.weight"})) return "lm_head";
    if (any(name, {"output_norm", "output_norm.weight", "model.norm.weight", "norm.weight"})) return "output_norm";
    static const char* prefixes[] = {"blk.", "model.layers.", "layers.", "transformer.h."};
    for (const char* pre : prefixes) {
        const size_t n = strlen(pre);
        if (name.compare(0, n, pre) != 0) continue;
        const size_t dot = name.find('.', n);
        if (dot == std::string::npos) return "";
        const std::string layer = name.substr(n, dot - n), sfx = name.substr(dot + 1);
        const char* role = nullptr;
        if (any(sfx, {"attn_norm", "attn_norm.weight", "input_layernorm.weight", "input_layernorm",
                      "attention_norm.weight", "attention_norm", "ln_1.weight", "ln_1"}))
            role = "attn_norm";
        else if (any(sfx, {"ffn_norm", "ffn_norm.weight", "post_attention_layernorm.weight",
                           "post_attention_layernorm", "ln_2.weight", "ln_2"}))
            role = "ffn_norm";
        else if (any(sfx, {"wq", "wq.weight", "attn_q.weight", "attn_q", "self_attn.q_proj.weight", "self_attn.q_proj",
                           "q_proj.weight", "q_proj", "attention.wq.weight"}))
            role = "wq";
        else if (any(sfx, {"wk", "wk.weight", "attn_k.weight", "attn_k", "self_attn.k_proj.weight", "self_attn.k_proj",
                           "k_proj.weight", "k_proj", "attention.wk.weight"}))
            role = "wk";
        else if (any(sfx, {"wv", "wv.weight", "attn_v.weight", "attn_v", "self_attn.v_proj.weight", "self_attn.v_proj",
                           "v_proj.weight", "v_proj", "attention.wv.weight"}))
            role = "wv";
        else if (any(sfx, {"wo", "wo.weight", "attn_output.weight", "attn_output", "attn_out.weight", "attn_out",
                           "self_attn.o_proj.weight", "self_attn.o_proj", "o_proj.weight", "o_proj",
                           "attention.wo.weight"}))
            role = "wo";
        else if (any(sfx, {"ffn_gate", "ffn_gate.weight", "mlp.gate_proj.weight", "mlp.gate_proj", "gate_proj.weight",
                           "gate_proj", "feed_forward.w1.weight", "ffn_gate_exps.weight", "ffn_gate_exps"}))
            role = "ffn_gate";
        else if (any(sfx, {"ffn_up", "ffn_up.weight", "mlp.up_proj.weight", "mlp.up_proj", "up_proj.weight", "up_proj",
                           "feed_forward.w3.weight", "ffn_up_exps.weight", "ffn_up_exps"}))
            role = "ffn_up";
        else if (any(sfx, {"ffn_down", "ffn_down.weight", "mlp.down_proj.weight", "mlp.down_proj", "down_proj.weight",
                           "down_proj", "feed_forward.w2.weight", "ffn_down_exps.weight", "ffn_down_exps"}))
            role = "ffn_down";
        else if (any(sfx, {"attn_q.bias", "wq.bias", "self_attn.q_proj.bias"})) role = "bq";
        else if (any(sfx, {"attn_k.bias", "wk.bias", "self_attn.k_proj.bias"})) role = "bk";
        else if (any(sfx, {"attn_v.bias", "wv.bias", "self_attn.v_proj.bias"})) role = "bv";
        return role ? "layers." + layer + "." + role : "";
    }
    return "";
}

inline void close_file(File& f) {
    for (Staging& s : f.ring) {
        if (s.done) {
            cudaEventSynchronize(s.done);
            cudaEventDestroy(s.done);
        }
        if (s.host) cudaFreeHost(s.host);
    }
    f.ring.clear();
    if (f.base) munmap(const_cast<uint8_t*>(f.base), f.size);
    if (f.fd >= 0) close(f.fd);
    f.base = nullptr;
    f.fd = -1;
}

// Parses the file into f; on failure returns false with a message in err.
inline bool parse(const char* path, File& f, std::string& err) {
    f.fd = open(path, O_RDONLY);
    if (f.fd < 0) return err = std::string("cannot open ") + path, false;
    struct stat st;
    if (fstat(f.fd, &st) != 0 || st.st_size <= 0) return err = "cannot size the file or it is empty", false;
    f.size = (size_t)st.st_size;
    void* map = mmap(nullptr, f.size, PROT_READ, MAP_SHARED, f.fd, 0);
    if (map == MAP_FAILED) return err = "mmap failed", false;
    f.base = static_cast<const uint8_t*>(map);
    Reader r{f.base, f.base + f.size};

    uint32_t magic = 0;
    uint64_t n_tensors = 0, n_kv = 0;
    if (!r.get(magic) || magic != 0x46554747u) return err = "no GGUF magic", false;
    if (!r.get(f.version) || !r.get(n_tensors) || !r.get(n_kv)) return err = "truncated header", false;
    if (f.version < 2) return err = "GGUF v1 (32-bit counts) is not supported", false;

    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key;
        uint32_t t;
        if (!r.str(key) || !r.get(t)) return err = "truncated metadata key", false;
        if (t == 8) {
            std::string v;
            if (!r.str(v)) return err = "truncated string value of " + key, false;
            if (key == "general.architecture") f.model.architecture = v;
        } else if (t == 9) {
            const Reader at = r;
            uint32_t et;
            uint64_t n;
            if (!r.get(et) || !r.get(n)) return err = "truncated array of " + key, false;
            if ((key == "tokenizer.ggml.tokens" || has(key, ".tokens")) && n > 0) f.model.vocab = (uint32_t)n;
            r = at;
            if (!skip_value(r, 9)) return err = "truncated or malformed array " + key, false;
        } else {
            uint64_t u = 0;
            float fv = 0.0f;
            bool ok = true;
            switch (t) {
                case 0: case 1: case 7: { uint8_t v; ok = r.get(v); u = v; break; }
                case 2: case 3: { uint16_t v; ok = r.get(v); u = v; break; }
                case 4: case 5: { uint32_t v; ok = r.get(v); u = v; break; }
                case 6: { float v; ok = r.get(v); fv = v; u = float_to_u64(v); break; }
                case 10: case 11: { uint64_t v; ok = r.get(v); u = v; break; }
                case 12: { double v; ok = r.get(v); fv = (float)v; u = float_to_u64(v); break; }
                default: return err = "unknown value type " + std::to_string(t) + " of " + key, false;
            }
            if (!ok) return err = "truncated value of " + key, false;
            apply_number(f.model, f.alignment, key, u, fv);
        }
    }

    std::vector<Tensor> all;
    all.reserve((size_t)std::min<uint64_t>(n_tensors, 1u << 20));
    for (uint64_t i = 0; i < n_tensors; ++i) {
        Tensor t;
        if (!r.str(t.name) || !r.get(t.n_dims)) return err = "truncated tensor table", false;
        if (t.n_dims == 0 || t.n_dims > 4) return err = "tensor " + t.name + ": unsupported dimension count", false;
        for (uint32_t d = 0; d < t.n_dims; ++d)
            if (!r.get(t.dims[d])) return err = "truncated tensor table", false;
        if (!r.get(t.ggml_type) || !r.get(t.rel_offset)) return err = "truncated tensor table", false;
        all.push_back(std::move(t));
    }
    // The reference rounds up with a mask after casting the value to 32 bits
    // (model_loader.cpp:640,720), which is only the intended rounding for a
    // power of two below 2^32; any other value is refused here.
    if ((f.alignment & (f.alignment - 1)) != 0 || f.alignment > (uint64_t(1) << 31))
        return err = "general.alignment " + std::to_string(f.alignment) + " is not a power of two up to 2^31", false;
    const uint64_t cur = (uint64_t)(r.p - f.base);
    f.data_offset = (cur + f.alignment - 1) & ~(f.alignment - 1);

    long max_layer = -1;
    for (Tensor& t : all) {
        t.file_offset = f.data_offset + t.rel_offset;
        TypeInfo ti;
        uint64_t elems = 1;
        bool sized = type_info(t.ggml_type, ti) && t.dims[0] % ti.elems == 0;
        for (uint32_t d = 0; d < 4 && sized; ++d) {
            if (t.dims[d] != 0 && elems > UINT64_MAX / t.dims[d]) sized = false;
            else elems *= t.dims[d];
        }
        t.bytes = sized ? elems / ti.elems * ti.bytes : 0;
        t.dtype = sized ? ti.dtype : -1;
        if (t.rel_offset >= f.size || t.file_offset >= f.size || t.bytes > f.size - t.file_offset) {
            ++f.skipped;  // outside the file (the reference skips one that starts outside)
            continue;
        }
        max_layer = std::max(max_layer, layer_index(t.name));
        f.by_name.emplace(t.name, f.tensors.size());
        const std::string rk = role_key(t.name);
        if (!rk.empty()) f.by_role.emplace(rk, f.tensors.size());
        f.tensors.push_back(std::move(t));
    }

    // fallbacks for missing dimensions (model_loader.cpp:803-824)
    Model& m = f.model;
    if (max_layer >= 0 && m.layers == 0) m.layers = (uint32_t)(max_layer + 1);
    auto emb = f.by_role.find("token_embd");  // under any of its alias names
    if (emb != f.by_role.end()) {
        const Tensor& e = f.tensors[emb->second];
        if (e.n_dims >= 2) {
            if (m.hidden == 0) m.hidden = (uint32_t)std::min(e.dims[0], e.dims[1]);
            if (m.vocab == 0) m.vocab = (uint32_t)std::max(e.dims[0], e.dims[1]);
        }
    }
    if (m.heads == 0 && m.hidden > 0) m.heads = m.hidden / 64 ? m.hidden / 64 : 4;
    if (m.kv_heads == 0) m.kv_heads = m.heads;
    if (m.ffn == 0 && m.hidden > 0) m.ffn = m.hidden * 2;
    return true;
}

// Index of `name`: the tensor of that name, else the first tensor with the
// same canonical key (role_key), else -- for the LM head -- the token
// embedding (tied weights, model_loader.cpp:793-801).
inline bool find(const File& f, const std::string& name, uint64_t& idx) {
    auto it = f.by_name.find(name);
    if (it != f.by_name.end()) return idx = it->second, true;
    const std::string rk = role_key(name);
    if (rk.empty()) return false;
    it = f.by_role.find(rk);
    if (it == f.by_role.end() && rk == "lm_head") it = f.by_role.find("token_embd");
    if (it == f.by_role.end()) return false;
    idx = it->second;
    return true;
}

// Offsets of the tensors in the device image; returns the image size.
inline uint64_t image_layout(const File& f, const uint64_t* idx, uint64_t n, uint64_t* offsets) {
    uint64_t off = 0;
    for (uint64_t i = 0; i < n; ++i) {
        off = (off + kImageAlign - 1) / kImageAlign * kImageAlign;
        if (offsets) offsets[i] = off;
        off += f.tensors[idx[i]].bytes;
    }
    return off;
}

// Fills host[0, c1 - c0) with image bytes [c0, c1): the tensors' file bytes,
// zeros in the padding.  seg = the tensors in image order with their offsets.
struct Segment {
    uint64_t image_off, bytes;
    const uint8_t* src;
};

inline void fill_range(const std::vector<Segment>& seg, uint64_t c0, uint64_t c1, uint8_t* host) {
    // first segment that ends after c0
    size_t k = std::upper_bound(seg.begin(), seg.end(), c0,
                                [](uint64_t v, const Segment& s) { return v < s.image_off + s.bytes; }) -
               seg.begin();
    uint64_t pos = c0;
    for (; pos < c1 && k < seg.size(); ++k) {
        const Segment& s = seg[k];
        if (s.image_off > pos) {  // padding before this tensor
            const uint64_t z = std::min(s.image_off, c1) - pos;
            memset(host + (pos - c0), 0, z);
            pos += z;
            if (pos >= c1) break;
        }
        const uint64_t a = pos - s.image_off, b = std::min(s.bytes, c1 - s.image_off);
        if (b > a) {
            memcpy(host + (pos - c0), s.src + a, b - a);
            pos += b - a;
        }
    }
    if (pos < c1) memset(host + (pos - c0), 0, c1 - pos);
}

}  // namespace gguf
}  // namespace nexus_gpu
