// Test infrastructure, not product: a C-ABI shim over the UNMODIFIED reference engine
// (tinferno, compiled from its own sources by oracle/Makefile into oracle/_ref/).
// Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline / --impl reference)
// load the library this file is part of.  It is the checker for the restatement in
// tf_oracle.c and the timed CPU baseline; nothing on the CUDA product path links it.
//
// Every entry point calls the reference's public API as its own callers do:
//   Model(path, RunConfig) / prefill / decode / reset   src/model.hpp:26-50
//   stage_preset(stage, hw)                             src/common.hpp:289-322
//   matmul(C, A, Tensor, M, Exec)                        src/matmul.hpp:9
//   rmsnorm / silu_mul / softmax                         src/layers.hpp:7-10
//   rope_freqs / apply_rope_many / attn_*                src/attention.hpp:20-30
//   KVCache::init / store                                src/kvcache.hpp:9-22
//   quant_* / dequant_row / f16 conversions              src/quant.hpp:37-54
//   sample_greedy / sample_logits                        src/sampler.hpp:9-12
// Errors (std::exception) are caught here and turned into a non-zero status plus a
// message readable through ref_last_error(); nothing throws across the C boundary.
#include "model.hpp"
#include "matmul.hpp"
#include "layers.hpp"
#include "quant.hpp"
#include "sampler.hpp"
#include "attention.hpp"
#include "kvcache.hpp"

#include <cstring>
#include <random>
#include <string>

using namespace tinf;

namespace {
thread_local std::string g_err;

int fail(const std::exception& e) {
    g_err = e.what();
    return -1;
}

Tensor make_tensor(int ggml_type, const void* data, int64_t K, int64_t N) {
    Tensor t;
    t.dtype = dtype_from_ggml(ggml_type);
    t.ndim = 2;
    t.shape[0] = K;
    t.shape[1] = N;
    t.data = static_cast<const uint8_t*>(data);
    t.nbytes = tensor_nbytes(t.dtype, t.shape, 2);
    return t;
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// ---- model level -------------------------------------------------------------------
void* ref_model_create(const char* path, const char* stage, int threads, int max_seq,
                       int kv_head_major) {
    try {
        int hw = (int)std::thread::hardware_concurrency();
        RunConfig cfg = stage_preset(stage, hw > 0 ? hw : 4);
        if (threads > 0) cfg.n_threads = threads;
        cfg.max_seq = max_seq;
        if (kv_head_major == 1) cfg.kv_layout = KVLayout::HeadMajor;
        if (kv_head_major == 0) cfg.kv_layout = KVLayout::SeqMajor;
        return new Model(path, cfg);
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void ref_model_destroy(void* m) { delete static_cast<Model*>(m); }

int ref_model_prefill(void* m, const int* tokens, int n, float* logits) {
    try {
        static_cast<Model*>(m)->prefill(tokens, n, logits);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_model_decode(void* m, int token, float* logits) {
    try {
        static_cast<Model*>(m)->decode(token, logits);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

void ref_model_reset(void* m) { static_cast<Model*>(m)->reset(); }
int ref_model_n_vocab(void* m) { return static_cast<Model*>(m)->n_vocab(); }
int ref_model_n_pos(void* m) { return static_cast<Model*>(m)->n_pos(); }
int ref_model_eos(void* m) { return static_cast<Model*>(m)->eos(); }
int ref_model_n_threads(void* m) { return static_cast<Model*>(m)->cfg().n_threads; }
unsigned long long ref_model_weight_bytes(void* m) {
    return (unsigned long long)static_cast<Model*>(m)->weight_bytes();
}

// ---- op level ----------------------------------------------------------------------
int ref_matmul(float* C, const float* A, int ggml_type, const void* W, int N, int K, int M,
               int threads, int simd, int blocked) {
    try {
        Tensor t = make_tensor(ggml_type, W, K, N);
        RunConfig cfg;
        cfg.use_simd = simd != 0;
        cfg.use_blocking = blocked != 0;
        ThreadPool pool(threads > 0 ? threads : 1, false);
        Exec ex{&cfg, &pool, nullptr};
        matmul(C, A, t, M, ex);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_dequant_row(float* out, int ggml_type, const void* W, int K, long long row) {
    try {
        Tensor t = make_tensor(ggml_type, W, K, row + 1);
        dequant_row(out, t, row);
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

void ref_quant_q8_0_row(void* out, const float* x, int n) {
    quant_q8_0_row(static_cast<block_q8_0*>(out), x, n);
}
void ref_quant_q4_0_row(void* out, const float* x, int n) {
    quant_q4_0_row(static_cast<block_q4_0*>(out), x, n);
}
float ref_f16_to_f32(unsigned short h) { return f16_to_f32(h); }
unsigned short ref_f32_to_f16(float f) { return f32_to_f16(f); }

void ref_rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
    rmsnorm(out, x, w, n, eps);
}
void ref_silu_mul(float* gate, const float* up, int n) { silu_mul(gate, up, n); }
void ref_softmax(float* x, int n) { softmax(x, n); }

void ref_rope_freqs(float* out, int n_rot, float theta, int llama3, float scale, float low_f,
                    float high_f, float orig_ctx) {
    RopeParams rp;
    rp.type = llama3 ? RopeType::Llama3 : RopeType::Standard;
    rp.theta = theta;
    rp.n_rot = n_rot;
    rp.scale = scale;
    rp.low_freq_f = low_f;
    rp.high_freq_f = high_f;
    rp.orig_ctx = orig_ctx;
    std::vector<float> f;
    rope_freqs(f, rp);
    std::memcpy(out, f.data(), f.size() * sizeof(float));
}

void ref_apply_rope_many(float* x, int seq, int n_heads, int head_dim, int pos0,
                         const float* freq) {
    apply_rope_many(x, seq, n_heads, head_dim, pos0, freq, nullptr);
}

void ref_attn_prefill(float* out, const float* q, const float* k, const float* v, int seq,
                      int n_heads, int n_kv_heads, int head_dim) {
    std::vector<float> scores((size_t)seq);
    attn_prefill(out, q, k, v, seq, n_heads, n_kv_heads, head_dim, scores.data(), nullptr);
}

// Decode attention for one layer: k_all/v_all hold n_pos positions laid out
// [pos][n_kv_heads][head_dim]; they are stored through KVCache::store and then read by
// attn_decode exactly as Model::layer_decode does.
void ref_attn_decode(float* out, const float* q, const float* k_all, const float* v_all,
                     int n_pos, int n_heads, int n_kv_heads, int head_dim, int head_major) {
    KVCache kv;
    kv.init(1, n_kv_heads, head_dim, n_pos, head_major ? KVLayout::HeadMajor : KVLayout::SeqMajor);
    const size_t stride = (size_t)n_kv_heads * head_dim;
    for (int p = 0; p < n_pos; ++p) kv.store(0, p, k_all + p * stride, v_all + p * stride);
    std::vector<float> scores((size_t)n_pos);
    attn_decode(out, q, kv, 0, n_heads, n_kv_heads, head_dim, n_pos, scores.data(), nullptr);
}

int ref_sample_greedy(const float* logits, int n) { return sample_greedy(logits, n); }

// Temperature / top-p sampling with one libstdc++ mt19937 seeded like the CLI
// (src/main.cpp:111) and drawn once per step (src/main.cpp:114): step i samples from
// logits + i*n.
void ref_sample_logits_steps(const float* logits, int n, int steps, float temp, float top_p,
                             int seed, int* out) {
    std::mt19937 rng((unsigned)seed);
    for (int i = 0; i < steps; ++i)
        out[i] = sample_logits(logits + (size_t)i * n, n, temp, top_p, rng);
}

}  // extern "C"
