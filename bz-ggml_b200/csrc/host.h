// Host-side pieces of the B200 engine that never touch the GPU: the GGUF reader, the
// `breeze.*` model configuration and the BPE tokenizer.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace bzb {

enum GgmlType : uint32_t { GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_Q4_K = 12 };

struct GgufTensor {
    std::string name;
    std::vector<int64_t> ne;  // ggml order: ne[0] is the row length
    uint32_t type = 0;
    uint64_t offset = 0;      // from the start of the file
    uint64_t nbytes = 0;
    int64_t nelem() const { int64_t n = 1; for (int64_t d : ne) n *= d; return n; }
    int64_t rows() const { return ne.empty() ? 0 : nelem() / ne[0]; }
};

// GGUF v2/v3 reader over a read-only memory map (reference: src/gguf_loader.cpp:15-197,
// which goes through ggml's gguf API; this reader parses the published container format).
class GgufFile {
public:
    ~GgufFile();
    bool open(const std::string & path, std::string & err);
    const GgufTensor * find(const std::string & name) const;
    const uint8_t * data(const GgufTensor & t) const { return base_ + t.offset; }

    int kv_u32(const std::string & key, int def) const;
    float kv_f32(const std::string & key, float def) const;
    std::string kv_str(const std::string & key, const std::string & def = "") const;
    std::vector<int> kv_i32_array(const std::string & key) const;
    std::vector<std::string> kv_str_array(const std::string & key) const;

    std::vector<GgufTensor> tensors;

private:
    struct Kv {
        uint32_t type = 0;
        uint64_t u = 0;
        int64_t i = 0;
        double f = 0;
        std::string s;
        uint32_t arr_type = 0;
        std::vector<int64_t> arr_i;
        std::vector<std::string> arr_s;
    };
    std::unordered_map<std::string, Kv> kv_;
    std::unordered_map<std::string, size_t> index_;
    uint8_t * base_ = nullptr;
    size_t size_ = 0;
};

struct TeConfig {
    int hidden, n_layer, n_head, n_kv, hd, ffn, window;
    float eps, theta_full, fscale_full, theta_sliding, qpas, embed_scale;
    std::vector<int> is_full;
};
struct BbConfig { int hidden, n_layer, n_head, n_kv, hd, ffn; float eps, theta; };
struct DdConfig {
    int hidden, n_layer, n_head, n_kv, hd, ffn, orig_ctx;
    float eps, theta, factor, high, low;
};

// codec decoder (vocoder) keys, src/config.cpp:84-99
struct VocConfig {
    int hidden, n_layer, n_head, n_kv, hd, ffn, window;
    float eps, theta;
    std::vector<int> rates, ratios;
};

// the codec encoder (src/config.cpp:68-81): SEANet filters and ratios, Mimi transformer, RVQ
struct EncConfig {
    int hidden, n_layer, n_head, hd, ffn, window, nf, dim, n_sem;
    float eps, theta;
    std::vector<int> ratios;
};

// keys and defaults of src/config.cpp:6-102 that the generation path reads
struct ModelConfig {
    int hidden, nc, vs, cb_size, bb_eos, cb_pad, cb_eos, sample_rate, samples_per_frame, max_new_tokens;
    float temperature, top_p, rep, depth_temperature, depth_top_p;
    int top_k, depth_top_k;
    TeConfig te;
    BbConfig bb;
    DdConfig dd;
    VocConfig voc;
    EncConfig enc;
};

ModelConfig parse_config(const GgufFile & g);

// SentencePiece-style BPE of src/tokenizer.cpp:19-124: the longest special token at each
// position wins, other text has ' ' mapped to U+2581 and is merged by rank with byte fallback.
class Tokenizer {
public:
    bool load(const GgufFile & g);
    std::vector<int> encode(const std::string & text, bool add_bos) const;
    int bos() const { return bos_; }

private:
    void bpe(const std::string & word, std::vector<int> & out) const;
    std::vector<std::string> id_to_token_;
    std::unordered_map<std::string, int> token_to_id_;
    std::unordered_map<std::string, int> merge_rank_;
    std::unordered_map<std::string, int> specials_;
    std::vector<size_t> special_lens_;  // distinct lengths, longest first
    std::unordered_map<int, int> byte_to_id_;
    int bos_ = 2, unk_ = 3;
};

uint16_t f32_to_f16_bits(float f);
float f16_bits_to_f32(uint16_t h);

}  // namespace bzb
