// Dequant-GEMV: y[m][n] = sum_k x[m][k] * W[n][k] for M <= 8 activation rows, W in its
// GGUF block layout (Q8_0, Q4_0, Q4_1, Q6_K, F16, F32), with fused prologues (RMSNorm,
// embedding lookup) and epilogues (bias, residual add, SwiGLU, logits + greedy argmax,
// end-of-step bookkeeping).  Replaces matmul()/dot_weight_row() (src/matmul.cpp:5-73)
// together with the rmsnorm / apply_bias / add_inplace / silu_mul / sample_greedy calls
// that Model::layer_decode (src/model.cpp:108-142) makes around each matmul.
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace tfb {

constexpr int GV_WARPS = 8;                      // compute warps per CTA
constexpr int GV_THREADS = (GV_WARPS + 1) * 32;  // + one producer warp issuing bulk copies
constexpr int GV_STAGES = 4;                     // weight stages in flight per CTA
constexpr int GV_MAXM = 8;                       // activation rows per launch
constexpr int GV_STAGE_BUDGET = 18 * 1024;       // target bytes of weights per stage
constexpr int GV_PRE = 64;                       // epilogue operands prefetched per CTA (rows)
constexpr int GV_PRO_UNROLL = 8;                 // float4 activation loads in flight per thread

// PRO_PLANES (integer path only): the activation arrives as Q8 digit planes written by the
// previous kernel (xplanes); no activation load, norm or plane build in the prologue
enum : int { PRO_COPY = 0, PRO_RMSNORM = 1, PRO_EMBED_RMSNORM = 2, PRO_PLANES = 3 };
enum : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };
// FIN_KEY (vocab-split lm_head): the step's greedy key over this GPU's rows goes to key_out,
// order-flipped to a signed 64-bit value (key ^ 2^63) for a max all-reduce across GPUs; the
// next token comes from the reduced key (tf_key_apply_kernel)
enum : int { FIN_NONE = 0, FIN_ADVANCE = 1, FIN_ARGMAX = 2, FIN_KEY = 3 };

// Per-step control words in device memory (one set per engine).
struct StepCtl {
    unsigned int done;      // CTAs of the finishing kernel that have completed
    int gen_step;           // steps taken since the last reset of this counter
    int hist_cap;           // rows of `hist`
    int pad_;
};

struct GemvArgs {
    const uint8_t* W;   // first row of the weight block (rows contiguous, native layout)
    int wtype;
    int K;              // elements per row
    long long rb;       // bytes per row
    int n_items;        // output items: rows (P == 1) or row pairs (P == 2)
    int P;              // rows per item
    int KS;             // warps sharing one item along K
    int M;              // activation rows (<= GV_MAXM)
    int stage_bytes;    // bytes of one stage buffer (multiple of 16)
    int fast;           // 1: Q8_0 64-element-unit path
    int intq;           // 1: exact-integer path (M == 1, activation as digit planes)
    int q4;             // with intq: Q4_0 rows (natural-order planes)
    int q6;             // with intq: Q6_K rows (natural-order planes); neither: Q8_0
    // prologue
    int pro;
    const float* x;     // [M][ldx]
    int ldx;
    const float* norm_w;
    float eps;
    const uint8_t* embd; // embedding table (PRO_EMBED_RMSNORM)
    int embd_type;
    long long embd_rb;
    int n_vocab;
    const int* tokens;   // [M] token ids (device)
    float* x_out;        // CTA 0 stores the embedded rows here, [M][ldx]
    // epilogue
    int epi;
    float* y;
    int ldy;
    const float* bias;   // per row (EPI_STORE)
    float* resid;        // EPI_RESID
    int ldr;
    unsigned long long* keys;  // EPI_ARGMAX: one key per activation row
    int row_base;        // EPI_ARGMAX: vocabulary index of row 0 of W (vocab-split lm_head)
    long long* key_out;  // FIN_KEY: the step's key, order-flipped for a signed max reduction
    // end of step
    int fin;
    StepCtl* ctl;
    int* tok_next;       // FIN_ARGMAX: next input token per row
    int* pos;            // per slot
    const int* slots;    // slot of activation row m
    int* hist;           // FIN_ARGMAX: generated ids [hist_cap][M] (optional)
    int* err;
    // fused decode attention (integer path, M == 1, the QKV GEMV): the first attn_ctas ==
    // n_head * attn_nsf CTAs of the grid own one query head and one of attn_nsf position
    // splits each (RoPE, KV store, attention of `at`); they wait for the q/k/v rows through
    // sync[0] (GEMV CTAs arrive when their rows are stored) and leave through sync[1] (the
    // last one out clears both).  With attn_nsf > 1 a split leaves its partial (max, sum,
    // weighted V) in at.part and the last of the head's CTAs (aticket[head]) combines.
    int attn_ctas;
    int attn_nsf;
    unsigned* aticket;
    unsigned* sync;
    AttnArgs at;
    // digit-plane handoff between integer-path kernels (layout of q8_plane_bytes): xplanes
    // feeds PRO_PLANES; yplanes receives this kernel's output activation as planes (the
    // SwiGLU rows of EPI_SWIGLU, or the fused attention's heads), written per 32-item
    // block, so EPI_SWIGLU partitions its items in multiples of `align` = 32
    const uint8_t* xplanes;
    uint8_t* yplanes;
    int align;
    // optional launch trace (nullptr: off): thread 0 of CTA c stamps %globaltimer into
    // trace[c * GV_TRACE_SLOTS + k] at entry (0), after griddepcontrol.wait (1), prologue done
    // (2; attention CTAs: q/k/v ready), rows done (3; attention done) and exit (4); inside
    // the Q8_0 integer prologue: before griddepcontrol.wait (5), activation loaded (6), after
    // the first barrier that follows (7); attention CTAs: q/k/v loaded (5), tiles done (6),
    // the first tile's scores and softmax sums done (7), rotation and cache store done (8), the
    // first tile's scores done (9)
    unsigned long long* trace;
};

constexpr int GV_TRACE_SLOTS = 10;
constexpr int GV_TRACE_CTAS = 512;     // CTAs per launch the trace buffer holds
constexpr int GV_TRACE_LAUNCHES = 192; // launches per step the trace buffer holds

}  // namespace tfb
