/* tinferno-b200: B200 (sm_100a) decode/prefill engine for Llama-style GGUF models.
 *
 * C-ABI of libtinferno_b200.so.  Plain pointers and sizes only; every entry point returns
 * an int status (0 = ok) and never throws or exits.  The text of the last failure is
 * available from tf_cuda_last_error().
 *
 * The model-level calls replace the reference engine's C++ Model class
 * (RohanDisa/agent-serve src/model.hpp:24-90); the tf_op_* calls replace its op functions
 * one for one and take DEVICE pointers (they exist for the cfg3 kernel sweep and for
 * op-level parity tests).  Each declaration cites the reference interface it replaces.
 */
#ifndef TINFERNO_B200_H
#define TINFERNO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TF_ABI_VERSION 1

#if defined(__GNUC__)
#define TF_API __attribute__((visibility("default")))
#else
#define TF_API
#endif

/* ggml type ids (src/common.hpp:99 DType). */
enum { TF_F32 = 0, TF_F16 = 1, TF_Q4_0 = 2, TF_Q4_1 = 3, TF_Q8_0 = 8, TF_Q6_K = 14 };

/* KV cache element type.  F32 is the reference's own cache type (src/kvcache.hpp:26-27). */
enum { TF_KV_F32 = 0, TF_KV_F16 = 1, TF_KV_BF16 = 2 };

/* One GGUF tensor as the reference's Tensor describes it (src/tensor.hpp:7-23): ne[0] is
 * the innermost dimension (K for 2-D weights), data points at the tensor's bytes in their
 * GGUF block layout (host memory; the library copies them into HBM). */
typedef struct tf_tensor_desc {
    const char* name;
    int ggml_type;
    int ndim;
    int64_t ne[4];
    const void* data;
    size_t nbytes;
} tf_tensor_desc;

/* Hyper-parameters as the reference derives them from GGUF keys (src/model.cpp:14-41). */
typedef struct tf_hparams {
    int n_vocab, n_embd, n_ff, n_layer, n_head, n_kv_head, head_dim;
    float rms_eps;
    int rope_llama3; /* 0 = standard RoPE, 1 = llama3 frequency scaling */
    float rope_theta, rope_scale, rope_low_freq_f, rope_high_freq_f, rope_orig_ctx;
    int bos, eos;
} tf_hparams;

/* Engine options.  max_seq replaces RunConfig::max_seq (src/common.hpp:112); max_batch is
 * the number of independent sequence slots (the reference has one, src/model.hpp:29-31). */
typedef struct tf_options {
    int max_seq;
    int max_batch;
    int device;
    int kv_type;   /* TF_KV_* */
    int use_graph; /* per-kernel path: 1 = capture the decode step in a CUDA graph (default) */
    int decode_mode; /* batch-1 decode / short prefill / generate: TF_DECODE_KERNELS (default, 0)
                        launches one kernel per phase under programmatic dependent launch,
                        captured in a CUDA graph (also the path of batched decode);
                        TF_DECODE_PERSISTENT runs whole token steps in one cooperative kernel
                        (all layer matrices and the lm_head Q8_0, fp32 KV cache; tf_cuda_create
                        fails for other models) */
} tf_options;

enum { TF_DECODE_KERNELS = 0, TF_DECODE_PERSISTENT = 1 };

typedef struct tf_model tf_model;

/* Model(const std::string& path, const RunConfig&)  src/model.hpp:26, src/model.cpp:9-78.
 * Uploads every tensor once into HBM (native block layouts), sizes the KV cache and the
 * scratch, and precomputes the RoPE cos/sin table with the reference's own formula. */
TF_API int tf_cuda_create(const tf_tensor_desc* tensors, int n_tensors, const tf_hparams* hp,
                   const tf_options* opt, tf_model** out);

/* ~Model.  Releases every device allocation and the graph. */
TF_API int tf_cuda_destroy(tf_model* m);

/* Model::prefill(const int* tokens, int n, float* logits)  src/model.hpp:29, model.cpp:183-195.
 * Consumes tokens[0..n) of sequence `seq` at positions n_pos..n_pos+n-1; writes the
 * logits of the last token to `logits` (host, n_vocab floats) when non-null; when
 * `argmax_out` is non-null writes the greedy id (sample_greedy, src/sampler.cpp:8-13). */
TF_API int tf_cuda_prefill(tf_model* m, int seq, const int* tokens, int n, float* logits,
                    int* argmax_out);

/* Model::decode(int token, float* logits)  src/model.hpp:31, model.cpp:197-208. */
TF_API int tf_cuda_decode(tf_model* m, int seq, int token, float* logits, int* argmax_out);

/* The CLI's greedy loop (src/main.cpp:112-122 at --temp 0): starting from `first_token`
 * (the argmax of the prefill logits), n times { append token; stop if token == eos and
 * i > 0 (eos < 0 disables the rule); decode(token) } with the argmax fed back on the
 * device and no host round trip.  Writes the accepted ids to out_ids and their count to
 * *n_out; the sequence's position then matches the reference after the same loop. */
TF_API int tf_cuda_generate_greedy(tf_model* m, int seq, int first_token, int n, int eos, int* out_ids,
                            int* n_out);

/* Batched decode: one step for B sequences (distinct slots), token[b] appended to
 * seq_ids[b].  argmax_out[b] (host) receives each greedy id; logits (host, B*n_vocab) is
 * optional.  No reference counterpart: the reference decodes one sequence per Model. */
TF_API int tf_cuda_decode_batch(tf_model* m, const int* seq_ids, const int* tokens, int B,
                         int* argmax_out, float* logits);

/* Batched prefill: Model::prefill (src/model.cpp:183-195) for B sequences at once, each with
 * n prompt tokens (tokens[b*n + t]); attention of each sequence sees its own n tokens only,
 * as prefill does.  argmax_out[b] (host, optional) receives the greedy id after each
 * sequence's last token.  Runs n steps of B rows (the tensor-core GEMM path at B >= 16). */
TF_API int tf_cuda_prefill_batch(tf_model* m, const int* seq_ids, const int* tokens, int B, int n,
                                 int* argmax_out);

/* sample_logits(logits, n, temperature, top_p, rng)  src/sampler.cpp:15-52, on the device,
 * over the logits of row `row` of the last step (row 0 after decode / prefill).  The caller
 * draws r = uniform_real_distribution<float>(0, 1)(rng) from its own std::mt19937 (one draw
 * per sampled token, as src/main.cpp:109-114), so the random stream stays on the host.
 * temperature <= 0 is sample_greedy. */
TF_API int tf_cuda_sample(tf_model* m, int row, float temperature, float top_p, float r, int* out_id);

/* Vocab-split lm_head for batch-1 latency on several GPUs (each GPU runs the same sequence,
 * the 279 MB cfg0 lm_head is split), no reference counterpart (the reference's lm_head is one
 * matmul, src/model.cpp:205, and sample_greedy, src/sampler.cpp:8-13):
 *   tf_cuda_set_vocab_shard  this handle computes logits rows [V*rank/world, V*(rank+1)/world)
 *                            only (world == 1: the whole vocabulary again);
 *   tf_cuda_shard_key        device address of one int64: after each tf_cuda_decode_shard,
 *                            this GPU's greedy key (value, then first index on ties),
 *                            order-flipped so that a signed max all-reduce across the GPUs
 *                            (ncclAllReduce ncclInt64 ncclMax on the model's stream) leaves the
 *                            key of the whole vocabulary's argmax in every copy;
 *   tf_cuda_decode_shard     one decode step of `seq` with the split lm_head, asynchronous (no
 *                            synchronisation); token >= 0 starts a run from a host token,
 *                            token < 0 takes the argmax of the reduced key on the device;
 *   tf_cuda_shard_token      the argmax of the reduced key (host), synchronising the stream.
 * The logits of a shard step are valid for the shard's rows only. */
TF_API int tf_cuda_set_vocab_shard(tf_model* m, int rank, int world);
TF_API void* tf_cuda_shard_key(tf_model* m);
TF_API int tf_cuda_decode_shard(tf_model* m, int seq, int token);
TF_API int tf_cuda_shard_token(tf_model* m, int seq, int* token);
/* The first n greedy ids of the last device-side run (tf_cuda_generate_greedy's, or the shard
 * steps' since the last tf_cuda_decode_shard with a host token), synchronising the stream.
 * No reference counterpart (the CLI collects ids on the host, src/main.cpp:112-122). */
TF_API int tf_cuda_history(tf_model* m, int n, int* out);

/* Phase trace of the persistent decode kernel, the B200 counterpart of the reference's Timings /
 * --profile (src/common.hpp:118-134, src/main.cpp:132-141): with TFB200_PK_TRACE=1 in the
 * environment at tf_cuda_create, thread 0 of the first and of the last CTA stamp the GPU's
 * global timer at every phase boundary of the last launch.  out receives two rows of `cap`
 * entries (first CTA, last CTA), each (nanoseconds << 8 | tag); n_out[2] their counts.  Tags:
 * 10 + k phase start, 20 + k activation read, 30 + k prologue done, 40 + k rows done (k: 0 QKV,
 * 1 wo, 2 gate/up, 3 down, 5 lm_head); 50 attention start, 53 q / k / v read, 51 attention done. */
TF_API int tf_cuda_trace_read(tf_model* m, unsigned long long* out, int cap, int* n_out);

/* Launch trace of the per-kernel decode step (a model created with TFB200_GV_TRACE=1): for each
 * GEMV launch of the last step enqueued, GV_TRACE_CTAS (512) CTAs x 10 %globaltimer stamps (ns):
 * entry, after griddepcontrol.wait, prologue done (attention CTAs: q/k/v ready), rows done
 * (attention done), exit, and finer stamps inside the prologue and the fused attention; out
 * holds max_launches x 512 x 10 values, meta max_launches x 3 ints
 * {grid, attention CTAs, kind: 0 QKV, 1 wo, 2 gate/up, 3 down, 4 lm_head}.  Diagnostic only. */
TF_API int tf_cuda_launch_trace(tf_model* m, unsigned long long* out, int max_launches, int* meta, int* n_launch);

/* Model::reset()  src/model.cpp:80-83 (one slot; seq < 0 resets every slot). */
TF_API int tf_cuda_reset(tf_model* m, int seq);

/* Accessors: Model::n_pos / n_vocab / weight_bytes  src/model.hpp:35-43. */
TF_API int tf_cuda_n_pos(tf_model* m, int seq);
TF_API int tf_cuda_n_vocab(tf_model* m);
TF_API unsigned long long tf_cuda_weight_bytes(tf_model* m);
/* cudaStream_t the model runs on (for callers that time it with CUDA events). */
TF_API void* tf_cuda_stream(tf_model* m);
/* Kernels launched per decode step (for launch accounting). */
TF_API int tf_cuda_kernels_per_step(tf_model* m);

/* Page-locked host memory for output buffers, no reference counterpart (the reference's
 * logits buffer is ordinary memory, src/main.cpp:103): logits written by tf_cuda_prefill /
 * tf_cuda_decode / tf_cuda_decode_batch into a buffer from tf_host_alloc (or any page-locked
 * memory) arrive by DMA directly, without the staging copy on the host that ordinary memory
 * needs.  Free with tf_host_free. */
TF_API int tf_host_alloc(size_t bytes, void** out);
TF_API int tf_host_free(void* p);

/* Message of the last failure on this thread (m may be NULL). */
TF_API const char* tf_cuda_last_error(tf_model* m);

/* ---- op level: DEVICE pointers, launched on `stream` (NULL = default stream) ----------- */

/* matmul(float* C, const float* A, const Tensor& W, int M, const Exec&)  src/matmul.hpp:9:
 * C[M][N] = A[M][K] . W[N][K]^T, W in its GGUF block layout (row-major, ne0 = K). */
TF_API int tf_op_matmul(float* C, const float* A, int ggml_type, const void* W, int N, int K, int M,
                 void* stream);

/* Tensor-core Q8_0 GEMM in two parts, no reference counterpart (tf_op_matmul composes them
 * for M >= 16): tf_op_q8_scale finds the power-of-two scale sw of a Q8_0 matrix (one pass
 * over its block scales, synchronises the stream); tf_op_matmul_q8_tc computes C = A W^T with
 * it (M >= 16, K % 64 == 0; f16-split products, fp32 accumulation). */
TF_API int tf_op_q8_scale(const void* W, int N, int K, int* sw, void* stream);
TF_API int tf_op_matmul_q8_tc(float* C, const float* A, const void* W, int N, int K, int M, int sw,
                              void* stream);
/* The same two steps for a ggml type t of the tensor-core path (Q8_0 or Q4_0): the scale sw of
 * the matrix, then C = A W^T at M >= 16 (K % 64 == 0). */
TF_API int tf_op_weight_scale(const void* W, int t, int N, int K, int* sw, void* stream);
TF_API int tf_op_matmul_tc(float* C, const float* A, int t, const void* W, int N, int K, int M, int sw,
                           void* stream);

/* dequant_row(float* out, const Tensor& t, int64_t row)  src/quant.hpp:42: out[i][K] is
 * row rows[i] of W[N][K] (embedding lookup).  A row id outside [0, N) reads nothing: its
 * output row is zero and TF_DEV_ERR_BAD_INDEX is recorded for tf_op_device_error. */
TF_API int tf_op_dequant_rows(float* out, int ggml_type, const void* W, int N, int K, const int* rows,
                       int n_rows, void* stream);

/* rmsnorm(out, x, weight, n, eps)  src/layers.hpp:7, applied to `rows` rows of length n. */
TF_API int tf_op_rmsnorm(float* out, const float* x, const float* w, int n, int rows, float eps,
                  void* stream);

/* silu_mul(gate, up, n)  src/layers.hpp:8 */
TF_API int tf_op_silu_mul(float* gate, const float* up, int n, void* stream);

/* softmax(x, n)  src/layers.hpp:10, applied to `rows` rows of length n. */
TF_API int tf_op_softmax(float* x, int n, int rows, void* stream);

/* apply_rope_many(x, seq, n_heads, head_dim, pos0, freq)  src/attention.hpp:25. */
TF_API int tf_op_rope(float* x, int seq, int n_heads, int head_dim, int pos0, const float* freq,
               void* stream);

/* attn_decode(out, q, cache, layer, n_heads, n_kv_heads, head_dim, n_pos)
 * src/attention.hpp:27-28, over one layer's cache in the engine's layout
 * [n_kv_heads][cap][head_dim] of kv_type (TF_KV_*). */
TF_API int tf_op_attn_decode(float* out, const float* q, const void* k_cache, const void* v_cache,
                      int kv_type, int cap, int n_pos, int n_heads, int n_kv_heads, int head_dim,
                      void* stream);

/* tf_op_attn_decode with no device allocation: no reference counterpart (the reference's
 * attn_decode runs on the CPU and needs no scratch).  Same arguments and results as
 * tf_op_attn_decode; the split-K partials live in a static device array of 524288 floats
 * (n_heads * ceil(n_pos/64) * (head_dim+2) must fit, n_kv_heads <= 64, else an error).
 * For callers that cannot allocate mid-step.  Calls on one device must not overlap in time
 * (they share the scratch); the first call on a device does set-up and must precede any
 * stream capture. */
TF_API int tf_op_attn_decode_noalloc(float* out, const float* q, const void* k_cache,
                      const void* v_cache, int kv_type, int cap, int n_pos, int n_heads,
                      int n_kv_heads, int head_dim, void* stream);

/* attn_prefill(out, q, k, v, seq, n_heads, n_kv_heads, head_dim)  src/attention.hpp:29-30:
 * causal attention within the chunk; q [seq][n_heads][hd], k/v [seq][n_kv][hd]. */
TF_API int tf_op_attn_prefill(float* out, const float* q, const float* k, const float* v, int seq,
                       int n_heads, int n_kv_heads, int head_dim, void* stream);

/* sample_greedy(logits, n)  src/sampler.hpp:9: out[r] = first index of the maximum of row r. */
TF_API int tf_op_argmax(const float* logits, int n, int rows, int* out, void* stream);

/* Pipeline trace of the tensor-core GEMM, no reference counterpart (a finer-grained companion
 * of the reference's --profile timings, src/main.cpp): while `buf` (device memory, 968
 * unsigned 64-bit words, zeroed) is set, every tensor-core GEMM launch of this process has its
 * first CTA write clock64() stamps into it: [0] entry, [1] set-up done, [2] activation-copy warp
 * past its dependency wait, [3] every MMA completed, [4] epilogue done; [8 + c] weight chunk c
 * issued; [72 + 4k + i] k-stage k: dequantising warp 0 past the chunk wait (i = 0), past the
 * buffer wait (1), arrived (2), the last dequantising warp's arrival as stamp << 5 | warp (3);
 * [584 + 2k + i] the MMA thread past its wait (0), committed (1); [840 + k] activation stage k
 * issued.  nullptr switches it off. */
TF_API int tf_op_gemm_trace(unsigned long long* buf);

/* Device-side status of the op-level calls, no reference counterpart (the reference's ops
 * throw std::runtime_error on the calling thread, src/model.cpp:185,198).  Kernels cannot
 * return a status to the call that launched them, so the op-level kernels of a device record
 * the first problem they meet in one status word of that device: a bounded wait that gave up
 * (TF_DEV_ERR_WAIT_*), a position beyond the cache, a row id outside its matrix.  This call
 * waits for `stream`, stores the word in *code (0 = none) and clears it.  The tf_op_* calls
 * of the current device, tf_op_attn_decode_noalloc included, share the word. */
enum { TF_DEV_ERR_NONE = 0, TF_DEV_ERR_WAIT_FULL = 1, TF_DEV_ERR_WAIT_EMPTY = 2, TF_DEV_ERR_BAD_INDEX = 3,
       TF_DEV_ERR_POS = 4, TF_DEV_ERR_GRID_SYNC = 5 };
TF_API int tf_op_device_error(void* stream, int* code);

#ifdef __cplusplus
}
#endif
#endif
