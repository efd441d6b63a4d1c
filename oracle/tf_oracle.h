/* Test infrastructure (the checker), not product.
 *
 * A plain-C restatement of the reference engine's hot path (tinferno, the CPU engine in
 * RohanDisa/agent-serve): the ops under src/{quant,matmul,layers,attention,kvcache,
 * sampler}.cpp and the token loop Model::prefill / Model::decode in src/model.cpp.
 * Every function names the reference file:line it restates.  The arithmetic follows the
 * reference's stage-v2 build (AVX2 + FMA, src/common.hpp:303-307): the 8-lane FMA
 * accumulation order of the SIMD dots and the horizontal-sum tree of hsum8 are kept
 * lane for lane, so the restatement reproduces the reference's v2 results bit for bit
 * wherever the compiled reference does (pinned by tests/test_oracle.py against
 * oracle/_ref and against tests/golden/).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.
 */
#ifndef TF_ORACLE_H
#define TF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids of the formats the reference reads (src/common.hpp:99). */
enum { TFO_F32 = 0, TFO_F16 = 1, TFO_Q4_0 = 2, TFO_Q4_1 = 3, TFO_Q8_0 = 8, TFO_Q6_K = 14 };

/* One weight tensor, ggml order: ne[0] = innermost (K), ne[1] = rows (N). */
typedef struct {
    const char* name;
    int ggml_type;
    int ndim;
    int64_t ne[4];
    const void* data;
    size_t nbytes;
} tfo_tensor;

typedef struct {
    int n_vocab, n_embd, n_ff, n_layer, n_head, n_kv_head, head_dim;
    float rms_eps;
    int rope_llama3; /* 0 = standard, 1 = llama3 scaling */
    float rope_theta, rope_scale, rope_low_freq_f, rope_high_freq_f, rope_orig_ctx;
    int bos, eos;
} tfo_hparams;

float tfo_f16_to_f32(uint16_t h);
uint16_t tfo_f32_to_f16(float f);
size_t tfo_row_nbytes(int ggml_type, int64_t k);

void tfo_dequant_row(float* out, int ggml_type, const void* w, int k, int64_t row);
float tfo_dot_f32(const float* a, const float* b, int n);
float tfo_dot_f16_f32(const float* x, const uint16_t* w, int n);
float tfo_dot_q8_0_f32(const float* x, const void* w, int n);
float tfo_dot_q4_0_f32(const float* x, const void* w, int n);
void tfo_matmul(float* c, const float* a, int ggml_type, const void* w, int n, int k, int m,
                int threads);

void tfo_rmsnorm(float* out, const float* x, const float* w, int n, float eps);
void tfo_silu_mul(float* gate, const float* up, int n);
void tfo_add_inplace(float* a, const float* b, int n);
void tfo_softmax(float* x, int n);
void tfo_rope_freqs(float* freq, int n_rot, float theta, int llama3, float scale, float low_f,
                    float high_f, float orig_ctx);
void tfo_rope(float* x, int seq, int n_heads, int head_dim, int pos0, const float* freq);
void tfo_attn_decode(float* out, const float* q, const float* k, const float* v, int n_pos,
                     int n_heads, int n_kv_heads, int head_dim);
void tfo_attn_prefill(float* out, const float* q, const float* k, const float* v, int seq,
                      int n_heads, int n_kv_heads, int head_dim);
int tfo_sample_greedy(const float* logits, int n);
/* sample_logits (src/sampler.cpp:15-52) with the caller's uniform draw r in [0, 1). */
int tfo_sample_logits(const float* logits, int n, float temperature, float top_p, float r);

typedef struct tfo_model tfo_model;
tfo_model* tfo_model_create(const tfo_tensor* t, int n_tensors, const tfo_hparams* hp,
                            int max_seq, int threads);
int tfo_model_prefill(tfo_model* m, const int* tokens, int n, float* logits);
int tfo_model_decode(tfo_model* m, int token, float* logits);
void tfo_model_reset(tfo_model* m);
int tfo_model_n_pos(const tfo_model* m);
void tfo_model_destroy(tfo_model* m);
const char* tfo_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
