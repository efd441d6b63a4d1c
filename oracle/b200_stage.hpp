// The reference-side binding of the B200 engine: what a maintainer adds to the reference
// (as src/model_b200.hpp) so that its Model routes prefill / decode / reset through
// libtinferno_b200.so.  It compiles against the reference's own headers (src/gguf.hpp,
// src/tensor.hpp, src/common.hpp) and the engine's C ABI (include/tinferno_b200.h).
//
// In this repository it is test infrastructure: oracle/b200_stage_test.cpp builds it and
// compares it against the reference's Model on the same GGUF file (tests/test_gpu_boundary.py).
//
//   * the tensor descriptors come from GGUF::tensors() (src/gguf.hpp:26); Tensor's dtype,
//     ndim, shape[], data and nbytes (src/tensor.hpp:7-23) map one to one onto tf_tensor_desc;
//     the GGUF mmap keeps owning the bytes, the engine copies them into HBM once;
//   * the hyper-parameters are read from the GGUF keys exactly as Model::Model derives them
//     (src/model.cpp:14-41), RoPE llama3 scaling included;
//   * a non-zero status becomes std::runtime_error, the reference's error convention
//     (src/model.cpp:185,198).
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

#include "gguf.hpp"
#include "tinferno_b200.h"

namespace tinf {

// tf_hparams the way Model::Model reads them (src/model.cpp:14-41).
inline tf_hparams b200_hparams(const GGUF& g) {
    auto key = [&](const char* f) { return g.kv_arch(f); };
    tf_hparams h{};
    h.n_vocab = (int)g.u64(key("vocab_size"), 0);
    if (!h.n_vocab) h.n_vocab = (int)g.arr_str("tokenizer.ggml.tokens").size();
    h.n_embd = (int)g.u64(key("embedding_length"));
    h.n_ff = (int)g.u64(key("feed_forward_length"));
    h.n_layer = (int)g.u64(key("block_count"));
    h.n_head = (int)g.u64(key("attention.head_count"));
    h.n_kv_head = (int)g.u64(key("attention.head_count_kv"), (uint64_t)h.n_head);
    h.head_dim = h.n_head ? h.n_embd / h.n_head : 0;  // n_embd / n_head wins (src/model.cpp:22-24)
    h.rms_eps = g.f32(key("attention.layer_norm_rms_epsilon"), 1e-5f);
    h.rope_theta = g.f32(key("rope.freq_base"), 10000.0f);
    h.rope_llama3 = g.str(key("rope.scaling.type"), "") == "llama3" ? 1 : 0;
    h.rope_scale = h.rope_llama3 ? g.f32(key("rope.scaling.factor"), 32.0f) : 1.0f;
    h.rope_low_freq_f = h.rope_llama3 ? g.f32(key("rope.scaling.low_freq_factor"), 1.0f) : 1.0f;
    h.rope_high_freq_f = h.rope_llama3 ? g.f32(key("rope.scaling.high_freq_factor"), 4.0f) : 4.0f;
    h.rope_orig_ctx = h.rope_llama3 ? (float)g.u64(key("rope.scaling.original_context_length"), 8192) : 8192.0f;
    h.bos = (int)g.u64("tokenizer.ggml.bos_token_id", 1);
    h.eos = (int)g.u64("tokenizer.ggml.eos_token_id", 2);
    return h;
}

// Model's public surface (src/model.hpp:24-50) on the B200 engine, one sequence.
class ModelB200 {
public:
    ModelB200(const GGUF& g, const RunConfig& rc, int device = 0) {
        std::vector<tf_tensor_desc> d;
        d.reserve(g.tensors().size());
        for (const Tensor& t : g.tensors()) {
            tf_tensor_desc x{};
            x.name = t.name.c_str();
            x.ggml_type = ggml_from_dtype(t.dtype);
            x.ndim = t.ndim;
            for (int i = 0; i < 4; ++i) x.ne[i] = t.shape[i];
            x.data = t.data;
            x.nbytes = t.nbytes;
            d.push_back(x);
        }
        const tf_hparams h = b200_hparams(g);
        n_vocab_ = h.n_vocab;
        eos_ = h.eos;
        tf_options o{};
        o.max_seq = rc.max_seq;
        o.max_batch = 1;
        o.device = device;
        o.kv_type = TF_KV_F32;  // the reference's cache type (src/kvcache.hpp)
        o.use_graph = 1;
        o.decode_mode = 0;      // the engine's default batch-1 path
        check(tf_cuda_create(d.data(), (int)d.size(), &h, &o, &m_));
    }
    ~ModelB200() { tf_cuda_destroy(m_); }
    ModelB200(const ModelB200&) = delete;
    ModelB200& operator=(const ModelB200&) = delete;

    void prefill(const int* tokens, int n, float* logits) { check(tf_cuda_prefill(m_, 0, tokens, n, logits, nullptr)); }
    void decode(int token, float* logits) { check(tf_cuda_decode(m_, 0, token, logits, nullptr)); }
    void reset() { check(tf_cuda_reset(m_, 0)); }
    int n_pos() const { return tf_cuda_n_pos(m_, 0); }
    int n_vocab() const { return n_vocab_; }
    int eos() const { return eos_; }
    // The CLI's greedy loop (src/main.cpp:112-122) on the device: ids accepted, EOS rule kept.
    std::vector<int> generate_greedy(int first_token, int n) {
        std::vector<int> ids(n);
        int n_out = 0;
        check(tf_cuda_generate_greedy(m_, 0, first_token, n, eos_, ids.data(), &n_out));
        ids.resize(n_out);
        return ids;
    }

private:
    void check(int rc) const {
        if (rc) throw std::runtime_error(tf_cuda_last_error(m_));
    }
    tf_model* m_ = nullptr;
    int n_vocab_ = 0, eos_ = 2;
};

}  // namespace tinf
