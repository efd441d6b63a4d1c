// The engine behind the model-level C-ABI (include/tinferno_b200.h): weight upload, KV cache,
// scratch, the per-step kernel sequence, CUDA-graph capture and the API entry points.
//
// HBM layout (one arena, 256-byte aligned regions, 256 bytes of slack at the end):
//   per layer  attn_norm f32 | fused QKV rows [wq; wk; wv] (byte-exact concatenation of the
//              three GGUF tensors, same block layout) | fused bias [bq; bk; bv] f32 |
//              wo | ffn_norm f32 | gate/up rows interleaved (gate_i, up_i) | down
//   token_embd | output (only when not tied) | output_norm
// The concatenation / row interleave move whole rows and keep every row's bytes as they are
// in the file; bytes per token equal GGUF::weight_bytes() (src/gguf.cpp:219-223).
//
// One decode step for M rows (src/model.cpp:197-208 per row) is 5 kernels per layer + 1:
//   [embed+]rmsnorm+QKV GEMV+bias -> RoPE+KV store+flash-decode -> wo GEMV+residual ->
//   rmsnorm+gate/up GEMV+SwiGLU -> down GEMV+residual ... -> rmsnorm+lm_head GEMV+argmax
//   (+ end-of-step bookkeeping: next token, history, position), all launched with
//   programmatic dependent launch and captured once per row count into a CUDA graph.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "attention.cuh"
#include "dots.cuh"
#include "gemm.cuh"
#include "sample.cuh"
#include "persist.cuh"
#include "upload.cuh"
#include "engine.cuh"

namespace tfb {

cudaError_t launch_rmsnorm(float* out, const float* x, const float* w, int n, int rows, float eps, cudaStream_t st);
cudaError_t launch_silu_mul(float* g, const float* u, int n, cudaStream_t st);
cudaError_t launch_softmax(float* x, int n, int rows, cudaStream_t st);
cudaError_t launch_rope(float* x, int seq, int nh, int hd, int pos0, const float* freq, cudaStream_t st);
cudaError_t launch_argmax(const float* logits, int n, int rows, int* out, cudaStream_t st);

std::string& last_error_tls() {
    static thread_local std::string s;
    return s;
}
int set_error(const std::string& msg) {
    last_error_tls() = msg;
    return -1;
}

}  // namespace tfb

using namespace tfb;

namespace {

struct WeightRef {
    const uint8_t* p = nullptr;
    int type = 0;
    int K = 0;
    long long rb = 0;
    int rows = 0;
    int sw = 0;  // Q8_0 / Q4_0: power-of-two scale of the tensor-core GEMM (gemm.cuh)
};

// Whether the tensor-core GEMM takes this matrix (Q8_0, or Q4_0 on the tcgen05 kernel).
bool gemm_weight_ok(const WeightRef& w) {
    return (w.type == T_Q8_0 || (w.type == T_Q4_0 && gemm_takes_q4())) && w.K % GM_BK == 0;
}

struct LayerDev {
    const float* attn_norm;
    WeightRef qkv;          // rows = H + 2*KV
    const float* bqkv;      // nullptr when the model has no q/k/v bias
    WeightRef wo;
    const float* ffn_norm;
    WeightRef gateup;       // rows = 2*FF, interleaved
    WeightRef down;
};

const char* err_code_text(int c) {
    switch (c) {
        case ERR_WAIT_FULL: return "device wait for a weight stage timed out";
        case ERR_WAIT_EMPTY: return "device wait for a free weight stage timed out";
        case ERR_BAD_TOKEN: return "token id out of range";
        case ERR_POS: return "position out of range";
        default: return "device error";
    }
}

}  // namespace

struct tf_model {
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    tf_hparams hp{};
    tf_options opt{};
    int D = 0, H = 0, KV = 0, FF = 0, V = 0, hd = 0;
    uint8_t* arena = nullptr;
    std::vector<LayerDev> L;
    WeightRef embd, outw;
    const float* out_norm = nullptr;
    unsigned long long weight_bytes = 0;
    // KV cache
    void* kc = nullptr;
    void* vc = nullptr;
    long long layer_elems = 0, slot_elems = 0;
    float *cosb = nullptr, *sinb = nullptr;
    // scratch for up to `tile` activation rows
    int tile = 1;
    float *x = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr, *part = nullptr;
    uint8_t* xplanes = nullptr;  // digit planes handed from one integer-path GEMV step kernel to the next
    int attn_tile = 0;           // positions per tile of the fused decode attention
    unsigned* counters = nullptr;
    unsigned* d_async = nullptr;  // [n_layer][2] fused-attention arrival / departure counters,
                                  // then [n_head] tickets of the split fused attention
    bool gemm_ok = false;         // most layer weight bytes are in GEMM-able matrices
    int gtile = 0;                // rows per step on the GEMM path (0: no GEMM path)
    int ptile = 0;                // prompt tokens per prefill chunk on the GEMM path
    __half *xh = nullptr, *xl = nullptr;  // GEMM activation halves [round_up(gtile,128)][max K]
    int* d_sx = nullptr;
    SampleScratch* smp = nullptr;  // temperature / top-p sampler scratch
    float* gws = nullptr;         // split-K workspace
    unsigned* gcnt = nullptr;     // split-K tile counters
    unsigned long long* keys = nullptr;
    int *d_tokens = nullptr, *d_slots = nullptr, *d_pos = nullptr, *d_wstart = nullptr, *d_hist = nullptr;
    int *d_prompt = nullptr, *d_err = nullptr;
    StepCtl* ctl = nullptr;
    int n_split = 1;
    // host staging (pinned)
    int* hi = nullptr;      // small int staging
    int* hb = nullptr;      // batch staging: [rows] tokens in / ids out, [rows] slots
    float* hlog = nullptr;  // logits staging [tile][V]
    std::vector<int> hpos;  // host mirror of each slot's position
    std::map<long long, cudaGraphExec_t> graphs;
    int kernels_per_step = 0;
    // persistent decode kernel (batch 1)
    bool pk = false;
    PkPlan pk_plan{};
    int pk_grid = 0, pk_ctl_words = 0;
    PkMat* d_pkmats = nullptr;
    unsigned* d_pkctl = nullptr;
    unsigned long long* d_pkkeys = nullptr;
    uint2* d_pkll = nullptr;
    size_t pk_ll_pairs = 0;
    unsigned pk_ep = 1;
    float* d_pkpart = nullptr;
    unsigned* d_pktickets = nullptr;
    unsigned long long* d_pktrace = nullptr;  // phase trace (TFB200_PK_TRACE=1 at creation)
    int* d_pktrace_n = nullptr;
    int pk_trace_cap = 0;
    double upload_s = 0.0;  // seconds tf_cuda_create spent moving the weights into HBM
    // vocab-split lm_head (batch 1): this GPU's rows [vs_row0, vs_row1) of the output matrix;
    // the step's key leaves in d_keyred for a max all-reduce across the GPUs
    bool vsplit = false;
    bool split_step = false;  // set only while tf_cuda_decode_shard enqueues its step
    int vs_row0 = 0, vs_row1 = 0;
    long long* d_keyred = nullptr;
    // GEMV launch trace (TFB200_GV_TRACE=1 at creation): [GV_TRACE_LAUNCHES][GV_TRACE_CTAS]
    // [GV_TRACE_SLOTS] stamps of the last step run, and per launch {grid, attention CTAs, kind}
    // of the last step enqueued
    unsigned long long* d_gvtrace = nullptr;
    std::vector<int> gvt_meta;
    std::string err;
};

namespace {

int fail(tf_model* m, const std::string& s) {
    if (m) m->err = s;
    return set_error(s);
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) return fail(m, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// Host restatement of rope_freqs (src/attention.cpp:9-29), evaluated in float with the
// reference build's contraction of the llama3 blend.
void rope_freqs_host(std::vector<float>& f, const tf_hparams& hp) {
    const int d2 = hp.head_dim / 2;
    f.resize(d2);
    for (int i = 0; i < d2; ++i) {
        float v = 1.0f / std::pow(hp.rope_theta, (float)(2 * i) / (float)hp.head_dim);
        if (hp.rope_llama3) {
            const float wavelen = 2.0f * 3.14159265358979323846f / v;
            const float lo_wl = hp.rope_orig_ctx / hp.rope_low_freq_f;
            const float hi_wl = hp.rope_orig_ctx / hp.rope_high_freq_f;
            if (wavelen < hi_wl) {
            } else if (wavelen > lo_wl) {
                v /= hp.rope_scale;
            } else {
                const float smooth = (hp.rope_orig_ctx / wavelen - hp.rope_low_freq_f) /
                                     (hp.rope_high_freq_f - hp.rope_low_freq_f);
                v = std::fma(smooth, v, (1.0f - smooth) * v / hp.rope_scale);
            }
        }
        f[i] = v;
    }
}

const tf_tensor_desc* find_desc(const tf_tensor_desc* t, int n, const std::string& name) {
    for (int i = 0; i < n; ++i)
        if (t[i].name && name == t[i].name) return &t[i];
    return nullptr;
}

bool type_ok(int t) { return t == T_F32 || t == T_F16 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q8_0 || t == T_Q6_K; }

// Common GEMV argument skeleton for one weight block.
GemvArgs gemv_base(tf_model* m, const WeightRef& w, int n_items, int P, int M) {
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    a.W = w.p;
    a.wtype = w.type;
    a.K = w.K;
    a.rb = w.rb;
    a.n_items = n_items;
    a.P = P;
    a.M = M;
    a.err = m->d_err;
    gemv_plan(a);
    return a;
}

// Decode attention arguments of layer li (fresh step: RoPE + KV store + attention).
AttnArgs attn_args(tf_model* m, int li) {
    AttnArgs a;
    memset(&a, 0, sizeof(a));
    a.qkv = m->qkv;
    a.ld_qkv = m->H + 2 * m->KV;
    const size_t esz = m->opt.kv_type == TF_KV_F32 ? 4 : 2;
    a.kc = static_cast<uint8_t*>(m->kc) + (size_t)li * m->layer_elems * esz;
    a.vc = static_cast<uint8_t*>(m->vc) + (size_t)li * m->layer_elems * esz;
    a.slot_stride = m->slot_elems;
    a.cap = m->opt.max_seq;
    a.kv_type = m->opt.kv_type;
    a.pos = m->d_pos;
    a.wstart = m->d_wstart;
    a.slots = m->d_slots;
    a.cosb = m->cosb;
    a.sinb = m->sinb;
    a.n_head = m->hp.n_head;
    a.n_kv = m->hp.n_kv_head;
    a.hd = m->hd;
    a.n_split = m->n_split;
    a.n_rows = m->layer_elems / m->hd;
    a.part = m->part;
    a.counters = m->counters;
    a.out = m->attn;
    a.ld_out = m->H;
    a.fresh = 1;
    a.err = m->d_err;
    return a;
}

// Decode attention runs inside the QKV kernel (CTAs per query head appended to its grid) for
// batch-1 steps.  A context that fits in two of its tiles (a tile is what the QKV launch's
// shared memory holds: ~140 positions for cfg0, ~60 for cfg1) and ends at or below
// kFusedAttnMaxPos takes one CTA per head; a longer one is split over positions into nsf
// CTAs per head of at most two tiles each (the last of a head to finish combines), while
// n_head * nsf stays within half the GEMV slots; beyond that the separate split flash-decode
// kernel runs.  One CTA per head walking many tiles measured slower than the separate
// kernel (cfg1 at positions 512-640: 759 vs 962 tok/s); cfg0 at 32-96: 1872 fused vs 1523.
constexpr int kFusedAttnMaxPos = 1024;
constexpr int kFusedAttnTiles = 2;

static bool fused_attn_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_FUSED_ATTN");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

// Digit-plane handoff (gemv.cuh xplanes / yplanes) between the integer-path kernels of a
// batch-1 step: attention -> wo and gate/up -> down (TFB200_PLANES=0 turns it off).
static bool planes_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_PLANES");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

// TFB200_FUSED_SPLIT=0: no position splits in the fused attention (measurement switch)
static bool fused_split_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_FUSED_SPLIT");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

// CTAs per query head of the attention fused into batch-1 steps up to position end_pos, or 0
// when the separate attention kernel runs.
int fuse_attn_ok(const tf_model* m, int end_pos) {
    if (!fused_attn_enabled() || m->attn_tile <= 0) return 0;
    const int per = kFusedAttnTiles * m->attn_tile;
    if (end_pos <= std::min(kFusedAttnMaxPos, per)) return 1;
    if (!fused_split_enabled()) return 0;
    const int nsf = (end_pos + per - 1) / per;
    if (nsf > m->n_split || nsf * m->hp.n_head > gemv_slots(m->num_sms) / 2) return 0;
    return nsf;
}

// One step for M >= GM_MIN_M rows on the tensor-core GEMM path: per layer activation
// preparation (RMSNorm, f16 halves) before each GEMM, the split flash-decode attention over
// the M rows' slots, and a finishing kernel for the step's tokens and positions.  A matrix the
// GEMM does not take (Q4_1, Q6_K, F16, F32) runs the multi-row GEMV over row groups of up to
// `tile` rows with the same prologue and epilogue.  A prefill chunk (`chunk`) computes the
// lm_head for its last row only: Model::prefill returns that row's logits alone
// (src/model.cpp:183-195).
int enqueue_step_gemm(tf_model* m, int M, bool head, int* n_launch, bool chunk) {
    const int D = m->D, H = m->H, KV = m->KV, FF = m->FF, V = m->V;
    const int ldq = H + 2 * KV;
    int launches = 0;
    // y[M][N] (+ epilogue) = op(x)[M][K] W^T: op = RMSNorm with norm_w (embedding lookup of
    // d_tokens first when `embed`), else the rows as they are; rows [r0, r0 + rows) only
    struct Mm {
        const WeightRef* w;
        int n_items, P, epi;
        const float* x;
        int ldx;
        const float* norm_w;
        bool embed;
        float* y;
        int ldy;
        const float* bias;
        float* resid;
        unsigned long long* keys;
    };
    auto matmul = [&](const Mm& q, int r0, int rows) -> int {
        const WeightRef& w = *q.w;
        if (gemm_weight_ok(w) && rows >= GM_MIN_M) {
            XPrepArgs p;
            memset(&p, 0, sizeof(p));
            p.x = q.x + (size_t)r0 * q.ldx;
            p.ldx = q.ldx;
            p.norm_w = q.norm_w;
            p.eps = m->hp.rms_eps;
            p.K = w.K;
            p.M = rows;
            p.xh = m->xh;
            p.xl = m->xl;
            p.sx = m->d_sx;
            p.err = m->d_err;
            if (q.embed) {
                p.embd = m->embd.p;
                p.embd_type = m->embd.type;
                p.embd_rb = m->embd.rb;
                p.n_vocab = V;
                p.tokens = m->d_tokens + r0;
                p.x_out = m->x + (size_t)r0 * D;
            }
            CK(xprep_launch(p, m->stream));
            GemmArgs g;
            memset(&g, 0, sizeof(g));
            g.W = w.p;
            g.wq4 = w.type == T_Q4_0 ? 1 : 0;
            g.rb = w.rb;
            g.N = q.n_items * q.P;
            g.K = w.K;
            g.M = rows;
            g.sw = w.sw;
            g.xh = m->xh;
            g.xl = m->xl;
            g.sx = m->d_sx;
            g.epi = q.epi;
            g.ksplit = gemm_pick_split(g.N, rows, w.K, m->num_sms);
            g.ws = m->gws;
            g.tile_cnt = m->gcnt;
            g.err = m->d_err;
            g.y = q.y ? q.y + (size_t)r0 * q.ldy : nullptr;
            g.ldy = q.ldy;
            g.bias = q.bias;
            g.resid = q.resid ? q.resid + (size_t)r0 * D : nullptr;
            g.ldr = D;
            if (q.keys) {
                g.keys = q.keys + r0;
                g.store_logits = 1;
            }
            CK(gemm_launch(g, m->stream));
            launches += 2;
            return 0;
        }
        for (int b = 0; b < rows; b += m->tile) {
            const int mc = std::min(m->tile, rows - b), r = r0 + b;
            GemvArgs a = gemv_base(m, w, q.n_items, q.P, mc);
            a.pro = q.embed ? PRO_EMBED_RMSNORM : q.norm_w ? PRO_RMSNORM : PRO_COPY;
            a.x = q.x + (size_t)r * q.ldx;
            a.ldx = q.ldx;
            a.norm_w = q.norm_w;
            a.eps = m->hp.rms_eps;
            if (q.embed) {
                a.embd = m->embd.p;
                a.embd_type = m->embd.type;
                a.embd_rb = m->embd.rb;
                a.n_vocab = V;
                a.tokens = m->d_tokens + r;
                a.x_out = m->x + (size_t)r * D;
            }
            a.epi = q.epi;
            a.y = q.y ? q.y + (size_t)r * q.ldy : nullptr;
            a.ldy = q.ldy;
            a.bias = q.bias;
            a.resid = q.resid ? q.resid + (size_t)r * D : nullptr;
            a.ldr = D;
            a.keys = q.keys ? q.keys + r : nullptr;
            CK(gemv_launch(a, gemv_grid(a, m->num_sms), m->stream, true));
            ++launches;
        }
        return 0;
    };
    for (int li = 0; li < m->hp.n_layer; ++li) {
        const LayerDev& Ld = m->L[li];
        if (matmul({&Ld.qkv, ldq, 1, EPI_STORE, m->x, D, Ld.attn_norm, li == 0, m->qkv, ldq, Ld.bqkv, nullptr, nullptr},
                   0, M))
            return -1;
        {
            AttnArgs a = attn_args(m, li);
            if (chunk) {  // one sequence's prompt rows: store every row's K/V, then attend
                CK(rope_store_launch(a, M, m->stream));
                a.fresh = 2;
                ++launches;
            }
            CK(attn_decode_launch(a, M, m->stream, true));
            ++launches;
        }
        if (matmul({&Ld.wo, D, 1, EPI_RESID, m->attn, H, nullptr, false, nullptr, 0, nullptr, m->x, nullptr}, 0, M))
            return -1;
        if (matmul({&Ld.gateup, FF, 2, EPI_SWIGLU, m->x, D, Ld.ffn_norm, false, m->h, FF, nullptr, nullptr, nullptr},
                   0, M))
            return -1;
        if (matmul({&Ld.down, D, 1, EPI_RESID, m->h, FF, nullptr, false, nullptr, 0, nullptr, m->x, nullptr}, 0, M))
            return -1;
    }
    if (head) {
        const Mm q = {&m->outw, V, 1, EPI_ARGMAX, m->x, D, m->out_norm, false, m->logits, V, nullptr, nullptr, m->keys};
        // a prefill chunk needs its last row's logits only (one GEMV row); a batched step
        // needs every row's
        if (chunk ? matmul(q, M - 1, 1) : matmul(q, 0, M)) return -1;
    }
    FinishArgs f;
    memset(&f, 0, sizeof(f));
    f.M = M;
    f.keys = m->keys;
    f.tok_next = m->d_tokens;
    f.pos = m->d_pos;
    f.slots = m->d_slots;
    f.hist = m->d_hist;
    f.ctl = m->ctl;
    f.argmax = head ? 1 : 0;
    CK(finish_launch(f, m->stream));
    ++launches;
    if (n_launch) *n_launch = launches;
    return 0;
}

// fused: CTAs per query head of the attention fused into the QKV kernel (0: separate kernel)
int enqueue_step(tf_model* m, int M, bool head, bool pdl, int* n_launch, int fused, bool chunk = false,
                 bool from_key = false) {
    if (chunk) return enqueue_step_gemm(m, M, head, n_launch, true);
    if (M >= GM_MIN_M && m->gtile >= M) return enqueue_step_gemm(m, M, head, n_launch, false);
    const int D = m->D, H = m->H, KV = m->KV, FF = m->FF, V = m->V;
    const int ldq = H + 2 * KV;
    int launches = 0;
    if (from_key) {  // vocab split: this step's token is the argmax of the reduced key
        CK(key_apply_launch(m->d_keyred, m->d_tokens, m->d_hist, m->ctl, m->stream));
        ++launches;
    }
    bool fuse = false, planes_wo = false, planes_down = false;
    if (m->d_gvtrace) m->gvt_meta.clear();
    // trace slots of the next GEMV launch (kind: 0 QKV, 1 wo, 2 gate/up, 3 down, 4 lm_head)
    auto trace = [&](GemvArgs& a, int grid, int kind) {
        const int li = (int)m->gvt_meta.size() / 3;
        if (!m->d_gvtrace || li >= GV_TRACE_LAUNCHES || grid > GV_TRACE_CTAS) return;
        a.trace = m->d_gvtrace + (size_t)li * GV_TRACE_CTAS * GV_TRACE_SLOTS;
        m->gvt_meta.insert(m->gvt_meta.end(), {grid, a.attn_ctas, kind});
    };
    for (int li = 0; li < m->hp.n_layer; ++li) {
        const LayerDev& Ld = m->L[li];
        {   // [embedding +] rmsnorm + fused QKV GEMV + bias
            GemvArgs a = gemv_base(m, Ld.qkv, H + 2 * KV, 1, M);
            a.pro = li == 0 ? PRO_EMBED_RMSNORM : PRO_RMSNORM;
            a.x = m->x;
            a.ldx = D;
            a.norm_w = Ld.attn_norm;
            a.eps = m->hp.rms_eps;
            a.embd = m->embd.p;
            a.embd_type = m->embd.type;
            a.embd_rb = m->embd.rb;
            a.n_vocab = V;
            a.tokens = m->d_tokens;
            a.x_out = m->x;
            a.epi = EPI_STORE;
            a.y = m->qkv;
            a.ldy = ldq;
            a.bias = Ld.bqkv;
            fuse = fused > 0 && M == 1 && a.intq && !a.q4 && !a.q6 && m->hd % 4 == 0 && m->hd <= AT_MAX_HD;
            {   // the planes handed over are in the Q8_0 layout: the consumer must take it
                const GemvArgs wo_plan = gemv_base(m, Ld.wo, D, 1, M);
                planes_wo = fuse && planes_enabled() && m->hd % 32 == 0 && wo_plan.intq && !wo_plan.q4 && !wo_plan.q6;
            }
            int grid = gemv_grid(a, m->num_sms);
            if (fuse) {
                // the attention CTAs take slots of the GEMV grid so that all stay resident
                // one attention CTA per query head: the tail after the GEMV is then the
                // latency of one head's scores / softmax / weighted V
                a.attn_ctas = m->hp.n_head * fused;
                a.attn_nsf = fused;
                a.aticket = m->d_async + 2 * m->hp.n_layer;
                a.sync = m->d_async + 2 * li;
                a.at = attn_args(m, li);
                grid = std::max(1, std::min(grid, gemv_slots(m->num_sms) - a.attn_ctas));
                if (planes_wo) a.yplanes = m->xplanes;
            }
            trace(a, grid + a.attn_ctas, 0);
            CK(gemv_launch(a, grid + a.attn_ctas, m->stream, pdl));
            ++launches;
        }
        if (!fuse) {   // RoPE + KV store + attention
            AttnArgs a = attn_args(m, li);
            CK(attn_decode_launch(a, M, m->stream, pdl));
            ++launches;
        }
        {   // wo GEMV + residual
            GemvArgs a = gemv_base(m, Ld.wo, D, 1, M);
            a.pro = planes_wo ? PRO_PLANES : PRO_COPY;
            a.xplanes = m->xplanes;
            a.x = m->attn;
            a.ldx = H;
            a.epi = EPI_RESID;
            a.resid = m->x;
            a.ldr = D;
            trace(a, gemv_grid(a, m->num_sms), 1);
            CK(gemv_launch(a, gemv_grid(a, m->num_sms), m->stream, pdl));
            ++launches;
        }
        {   // rmsnorm + gate/up GEMV + SwiGLU
            GemvArgs a = gemv_base(m, Ld.gateup, FF, 2, M);
            a.pro = PRO_RMSNORM;
            a.x = m->x;
            a.ldx = D;
            a.norm_w = Ld.ffn_norm;
            a.eps = m->hp.rms_eps;
            a.epi = EPI_SWIGLU;
            a.y = m->h;
            a.ldy = FF;
            int grid = gemv_grid(a, m->num_sms);
            // the SwiGLU rows leave as planes when both kernels take the integer path and each
            // CTA's whole 32-row blocks fit its row buffer
            const int nblk = FF / 32;
            grid = std::min(grid, nblk);
            planes_down = planes_enabled() && a.intq && FF % 32 == 0 && grid > 0 &&
                          (nblk + grid - 1) / grid * 32 <= GV_PRE;
            {
                const GemvArgs down_plan = gemv_base(m, Ld.down, D, 1, M);
                planes_down = planes_down && down_plan.intq && !down_plan.q4 && !down_plan.q6;
            }
            if (planes_down) {
                a.align = 32;
                a.yplanes = m->xplanes;
            } else {
                grid = gemv_grid(a, m->num_sms);
            }
            trace(a, grid, 2);
            CK(gemv_launch(a, grid, m->stream, pdl));
            ++launches;
        }
        {   // down GEMV + residual
            GemvArgs a = gemv_base(m, Ld.down, D, 1, M);
            a.pro = planes_down ? PRO_PLANES : PRO_COPY;
            a.xplanes = m->xplanes;
            a.x = m->h;
            a.ldx = FF;
            a.epi = EPI_RESID;
            a.resid = m->x;
            a.ldr = D;
            if (!head && li == m->hp.n_layer - 1) {
                a.fin = FIN_ADVANCE;
                a.ctl = m->ctl;
                a.pos = m->d_pos;
                a.slots = m->d_slots;
            }
            trace(a, gemv_grid(a, m->num_sms), 3);
            CK(gemv_launch(a, gemv_grid(a, m->num_sms), m->stream, pdl));
            ++launches;
        }
    }
    if (head) {  // rmsnorm + lm_head GEMV + logits + greedy argmax + end of step
        const bool split = m->split_step && M == 1;
        const int r0 = split ? m->vs_row0 : 0, nr = split ? m->vs_row1 - m->vs_row0 : V;
        WeightRef ow = m->outw;
        ow.p += (size_t)r0 * ow.rb;
        GemvArgs a = gemv_base(m, ow, nr, 1, M);
        a.pro = PRO_RMSNORM;
        a.x = m->x;
        a.ldx = D;
        a.norm_w = m->out_norm;
        a.eps = m->hp.rms_eps;
        a.epi = EPI_ARGMAX;
        a.y = m->logits + r0;
        a.ldy = V;
        a.keys = m->keys;
        a.row_base = r0;
        a.fin = split ? FIN_KEY : FIN_ARGMAX;
        a.key_out = m->d_keyred;
        a.ctl = m->ctl;
        a.tok_next = m->d_tokens;
        a.pos = m->d_pos;
        a.slots = m->d_slots;
        a.hist = m->d_hist;
        trace(a, gemv_grid(a, m->num_sms), 4);
        CK(gemv_launch(a, gemv_grid(a, m->num_sms), m->stream, pdl));
        ++launches;
    }
    if (n_launch) *n_launch = launches;
    return 0;
}

// Run one step for M rows (tokens in d_tokens[0..M), slots in d_slots[0..M)).
int run_step(tf_model* m, int M, bool head, int fused, bool chunk = false, bool from_key = false) {
    if (!m->opt.use_graph) return enqueue_step(m, M, head, true, nullptr, fused, chunk, from_key);
    // graphs are keyed by everything that changes the launch sequence or its arguments
    const bool split = head && m->split_step && M == 1;
    const long long key = ((long long)fused << 40) + ((long long)(split ? 1 + m->vs_row0 : 0) << 20) +
                          (long long)M * 32 + (head ? 1 : 0) + (chunk ? 4 : 0) + (from_key ? 8 : 0);
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_step(m, M, head, true, nullptr, fused, chunk, from_key);
        cudaError_t e = cudaStreamEndCapture(m->stream, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return fail(m, std::string("graph capture: ") + cudaGetErrorString(e));
        cudaGraphExec_t ge = nullptr;
        e = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return fail(m, std::string("graph instantiate: ") + cudaGetErrorString(e));
        it = m->graphs.emplace(key, ge).first;
    }
    CK(cudaGraphLaunch(it->second, m->stream));
    return 0;
}

// Matrix table of the persistent kernel (batch 1): per layer QKV (rows q | k | v), wo,
// gate/up (row pairs), down, then the lm_head.  Every matrix must be Q8_0 with rows that split
// into 64-element units, at most 32 per warp lane set (16 for row pairs) for KS | PK_WARPS;
// the KV cache must be fp32.  Returns 1 (and leaves m->pk false) when the model does not fit.
int build_pk_plan(tf_model* m) {
    std::vector<PkMat> mats;
    int slot = 0, max_k = m->D;
    auto add = [&](const WeightRef& w, int n_items, int P, const float* norm_w, const float* bias) -> bool {
        if (w.type != T_Q8_0 || w.K % 64 || (reinterpret_cast<uintptr_t>(w.p) & 3) || w.K > PK_MAX_K) return false;
        int ks = 0;
        for (int k = 1; k <= PK_WARPS; k <<= 1) {
            if ((w.K / 64) % k || (w.K / 64 / k) * P > 32) continue;
            ks = k;
            if ((long long)(PK_WARPS / k) * P * w.rb <= PK_SLOT_BUDGET) break;
        }
        if (!ks) return false;
        PkMat t;
        t.W = w.p;
        t.rb = w.rb;
        t.K = w.K;
        t.n_items = n_items;
        t.P = P;
        t.KS = ks;
        t.RI = PK_WARPS / ks;
        t.norm_w = norm_w;
        t.bias = bias;
        mats.push_back(t);
        slot = std::max(slot, (int)(((long long)t.RI * P * w.rb + 32 + 15) & ~15LL));
        max_k = std::max(max_k, w.K);
        return true;
    };
    for (int li = 0; li < m->hp.n_layer; ++li) {
        const LayerDev& Ld = m->L[li];
        if (!add(Ld.qkv, m->H + 2 * m->KV, 1, Ld.attn_norm, Ld.bqkv) || !add(Ld.wo, m->D, 1, nullptr, nullptr) ||
            !add(Ld.gateup, m->FF, 2, Ld.ffn_norm, nullptr) || !add(Ld.down, m->D, 1, nullptr, nullptr))
            return 1;
    }
    if (!add(m->outw, m->V, 1, m->out_norm, nullptr)) return 1;
    // fp32 cache (the reference's type): the attention tiles arrive as bulk copies of cache rows
    if (m->opt.kv_type != TF_KV_F32 || m->hd % 4 || m->hd > 256 || m->D % 4) return 1;
    if (m->hp.n_head > m->num_sms || m->hd / 2 > PK_MAX_D2) return 1;
    // rows a CTA owns: its residual rows and QKV rows stay in shared memory
    if ((m->D + m->num_sms - 1) / m->num_sms > PK_ROWS || (m->H + 2 * m->KV + m->num_sms - 1) / m->num_sms > PK_ROWS)
        return 1;
    PkPlan plan;
    if (!pk_plan(slot, max_k, m->hd, plan) || plan.attn_tp < 16) return 1;
    if (pk_occupancy(plan.smem) < 1) {
        cudaGetLastError();
        return 1;
    }
    m->pk_plan = plan;
    m->pk_grid = m->num_sms;
    CK(cudaMalloc(&m->d_pkmats, sizeof(PkMat) * mats.size()));
    CK(cudaMemcpy(m->d_pkmats, mats.data(), sizeof(PkMat) * mats.size(), cudaMemcpyHostToDevice));
    // the step counter and the abort word; the per-step greedy keys; the LL activation pairs
    m->pk_ctl_words = 2;
    m->pk_ll_pairs = (size_t)(m->H + 2 * m->KV) + m->H + m->D + m->FF;
    CK(cudaMalloc(&m->d_pkll, sizeof(uint2) * m->pk_ll_pairs));
    CK(cudaMemset(m->d_pkll, 0, sizeof(uint2) * m->pk_ll_pairs));  // epoch 0 is never expected
    m->pk_ep = 1;
    CK(cudaMalloc(&m->d_pkctl, sizeof(unsigned) * m->pk_ctl_words));
    CK(cudaMalloc(&m->d_pkkeys, sizeof(unsigned long long) * (size_t)m->opt.max_seq));
    const int max_nsf = std::max(1, m->pk_grid / m->hp.n_head);
    CK(cudaMalloc(&m->d_pkpart, sizeof(float) * (size_t)m->hp.n_head * max_nsf * (m->hd + 2)));
    CK(cudaMalloc(&m->d_pktickets, sizeof(unsigned) * m->hp.n_head));
    CK(cudaMemset(m->d_pktickets, 0, sizeof(unsigned) * m->hp.n_head));
    if (const char* tr = getenv("TFB200_PK_TRACE"); tr && tr[0] == '1') {
        m->pk_trace_cap = 1 << 16;
        CK(cudaMalloc(&m->d_pktrace, sizeof(unsigned long long) * 2 * m->pk_trace_cap));
        CK(cudaMalloc(&m->d_pktrace_n, sizeof(int) * 2));
    }
    m->pk = true;
    return 0;
}

// Run `n_steps` batch-1 steps of slot `seq` in one persistent launch: the first n_prompt
// steps consume prompt[] (device), later ones the previous step's argmax; the lm_head runs
// from step first_head on; during prompt steps attention starts at ws_prompt.
int run_pk(tf_model* m, int seq, const int* d_prompt, int n_prompt, int n_steps, int first_head, int ws_prompt,
           int hist_cap) {
    const PkPlan& p = m->pk_plan;
    PkArgs a;
    memset(&a, 0, sizeof(a));
    a.mats = m->d_pkmats;
    a.n_layer = m->hp.n_layer;
    a.n_steps = n_steps;
    a.n_prompt = n_prompt;
    a.prompt = d_prompt;
    a.first_head = first_head;
    a.ws_prompt = ws_prompt;
    a.pos0 = m->hpos[seq];
    a.slot = seq;
    a.slot_bytes = p.slot_bytes;
    a.n_slots = p.n_slots;
    a.reg_off = p.reg_off;
    a.misc_off = p.misc_off;
    a.attn_tp = p.attn_tp;
    // position splits per query head: one tile per split while the grid has room
    const int span = m->hpos[seq] + n_steps - (n_prompt >= n_steps ? ws_prompt : 0);
    const int max_nsf = std::max(1, m->pk_grid / m->hp.n_head);
    a.nsf = std::max(1, std::min(max_nsf, (span + p.attn_tp - 1) / p.attn_tp));
    a.eps = m->hp.rms_eps;
    a.embd = m->embd.p;
    a.embd_type = m->embd.type;
    a.embd_rb = m->embd.rb;
    a.n_vocab = m->V;
    a.llq = m->d_pkll;
    a.lla = a.llq + (m->H + 2 * m->KV);
    a.llx = a.lla + m->H;
    a.llh = a.llx + m->D;
    // epochs of this launch follow the last one's, so no pair left by an earlier launch can
    // carry an epoch this launch waits for
    a.ep0 = m->pk_ep;
    m->pk_ep += (unsigned)(n_steps + 1) * (unsigned)m->hp.n_layer * PK_EPS;
    a.logits = m->logits;
    a.D = m->D;
    a.H = m->H;
    a.KVd = m->KV;
    a.FF = m->FF;
    a.kc = m->kc;
    a.vc = m->vc;
    a.layer_elems = m->layer_elems;
    a.slot_elems = m->slot_elems;
    a.cap = m->opt.max_seq;
    a.kv_type = m->opt.kv_type;
    a.cosb = m->cosb;
    a.sinb = m->sinb;
    a.n_head = m->hp.n_head;
    a.n_kv = m->hp.n_kv_head;
    a.hd = m->hd;
    a.part = m->d_pkpart;
    a.tickets = m->d_pktickets;
    a.tok = m->d_tokens;
    a.pos = m->d_pos;
    a.hist = m->d_hist;
    a.hist_cap = hist_cap;
    a.keys = m->d_pkkeys;
    a.cnt = m->d_pkctl;
    a.abort_g = reinterpret_cast<int*>(m->d_pkctl + m->pk_ctl_words - 1);
    a.err = m->d_err;
    CK(cudaMemsetAsync(m->d_pkctl, 0, sizeof(unsigned) * m->pk_ctl_words, m->stream));
    CK(cudaMemsetAsync(m->d_pkkeys, 0, sizeof(unsigned long long) * n_steps, m->stream));
    if (m->d_pktrace) {
        a.trace = m->d_pktrace;
        a.trace_cap = m->pk_trace_cap;
        a.trace_n = m->d_pktrace_n;
        CK(cudaMemsetAsync(m->d_pktrace_n, 0, sizeof(int) * 2, m->stream));
    }
    CK(pk_launch(a, m->pk_grid, p.smem, m->stream));
    return 0;
}

// Synchronise and surface any device-side error word.
int finish_call(tf_model* m) {
    CK(cudaMemcpyAsync(m->hi + 60, m->d_err, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    if (m->hi[60] != 0) {
        const int c = m->hi[60];
        cudaMemsetAsync(m->d_err, 0, sizeof(int), m->stream);
        const int T = std::max(m->tile, m->gtile);
        cudaMemsetAsync(m->counters, 0, sizeof(unsigned) * (size_t)T * m->hp.n_kv_head, m->stream);
        cudaMemsetAsync(m->ctl, 0, sizeof(unsigned), m->stream);
        cudaMemsetAsync(m->keys, 0, sizeof(unsigned long long) * T, m->stream);
        cudaMemsetAsync(m->d_async, 0, sizeof(unsigned) * (2 * m->hp.n_layer + m->hp.n_head), m->stream);
        if (m->pk) cudaMemsetAsync(m->d_pktickets, 0, sizeof(unsigned) * m->hp.n_head, m->stream);
        cudaStreamSynchronize(m->stream);
        return fail(m, err_code_text(c));
    }
    return 0;
}

int check_seq(tf_model* m, int seq) {
    if (seq < 0 || seq >= m->opt.max_batch) return fail(m, "sequence slot out of range");
    return 0;
}

int set_slot_row(tf_model* m, int row, int seq, int token) {
    m->hi[0] = token;
    m->hi[1] = seq;
    CK(cudaMemcpyAsync(m->d_tokens + row, m->hi + 0, sizeof(int), cudaMemcpyHostToDevice, m->stream));
    CK(cudaMemcpyAsync(m->d_slots + row, m->hi + 1, sizeof(int), cudaMemcpyHostToDevice, m->stream));
    return 0;
}

// Whether host memory is page-locked (tf_host_alloc, cudaMallocHost, cudaHostRegister): the
// DMA then writes the caller's buffer directly, with no staging copy on the host.
bool host_pinned(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

int read_outputs(tf_model* m, int M, float* logits, int* argmax_out) {
    const bool direct = logits && host_pinned(logits);
    if (logits)
        CK(cudaMemcpyAsync(direct ? logits : m->hlog, m->logits, sizeof(float) * (size_t)M * m->V, cudaMemcpyDeviceToHost,
                           m->stream));
    if (argmax_out) CK(cudaMemcpyAsync(m->hb, m->d_tokens, sizeof(int) * M, cudaMemcpyDeviceToHost, m->stream));
    int rc = finish_call(m);
    if (rc) return rc;
    if (logits && !direct) memcpy(logits, m->hlog, sizeof(float) * (size_t)M * m->V);
    if (argmax_out) memcpy(argmax_out, m->hb, sizeof(int) * M);
    return 0;
}

// Outputs of row `row` of the last step (a prefill chunk's last prompt token).
int read_outputs_row(tf_model* m, int row, float* logits, int* argmax_out) {
    const bool direct = logits && host_pinned(logits);
    if (logits)
        CK(cudaMemcpyAsync(direct ? logits : m->hlog, m->logits + (size_t)row * m->V, sizeof(float) * m->V,
                           cudaMemcpyDeviceToHost, m->stream));
    if (argmax_out) CK(cudaMemcpyAsync(m->hb, m->d_tokens + row, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    int rc = finish_call(m);
    if (rc) return rc;
    if (logits && !direct) memcpy(logits, m->hlog, sizeof(float) * m->V);
    if (argmax_out) *argmax_out = m->hb[0];
    return 0;
}

}  // namespace

// ============================== C-ABI ==============================================

extern "C" {

const char* tf_cuda_last_error(tf_model* m) { return m && !m->err.empty() ? m->err.c_str() : last_error_tls().c_str(); }

int tf_host_alloc(size_t bytes, void** out) {
    if (!out) return set_error("out is null");
    *out = nullptr;
    if (!bytes) return 0;
    const cudaError_t e = cudaMallocHost(out, bytes);
    if (e != cudaSuccess) return set_error(std::string("cudaMallocHost: ") + cudaGetErrorString(e));
    return 0;
}

int tf_host_free(void* p) {
    if (!p) return 0;
    const cudaError_t e = cudaFreeHost(p);
    if (e != cudaSuccess) return set_error(std::string("cudaFreeHost: ") + cudaGetErrorString(e));
    return 0;
}

int tf_cuda_destroy(tf_model* m) {
    if (!m) return 0;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
    void* dev[] = {m->arena, m->kc, m->vc, m->cosb, m->sinb, m->x, m->qkv, m->attn, m->h, m->logits, m->part,
                   m->counters, m->keys, m->d_tokens, m->d_slots, m->d_pos, m->d_wstart, m->d_hist, m->d_prompt,
                   m->d_err, m->ctl, m->d_pkmats, m->d_pkctl, m->d_pkkeys, m->d_pkll, m->d_pkpart, m->d_pktickets, m->d_keyred, m->d_pktrace, m->d_pktrace_n, m->d_async, m->xh, m->xl, m->d_sx, m->gws, m->gcnt,
                   m->xplanes, m->d_gvtrace};
    for (void* p : dev)
        if (p) cudaFree(p);
    sample_scratch_destroy(m->smp);
    if (m->hi) cudaFreeHost(m->hi);
    if (m->hb) cudaFreeHost(m->hb);
    if (m->hlog) cudaFreeHost(m->hlog);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return 0;
}

int tf_cuda_create(const tf_tensor_desc* t, int nt, const tf_hparams* hp_in, const tf_options* opt_in, tf_model** out) {
    if (!out) return set_error("out is null");
    *out = nullptr;
    if (!t || !hp_in) return set_error("null tensors or hparams");
    tf_model* m = new tf_model();
    m->hp = *hp_in;
    tf_options o;
    o.max_seq = 4096;  // RunConfig::max_seq default (src/common.hpp:112)
    o.max_batch = 1;
    o.device = 0;
    o.kv_type = TF_KV_F32;
    o.use_graph = 1;
    o.decode_mode = TF_DECODE_KERNELS;
    if (opt_in) o = *opt_in;
    if (o.max_seq <= 0 || o.max_batch <= 0) {
        delete m;
        return set_error("max_seq and max_batch must be positive");
    }
    m->opt = o;
    m->device = o.device;
    const tf_hparams& hp = m->hp;
    if (hp.n_head <= 0 || hp.n_kv_head <= 0 || hp.n_embd <= 0 || hp.n_layer <= 0 || hp.n_ff <= 0 || hp.n_vocab <= 0) {
        delete m;
        return set_error("invalid hyper-parameters");
    }
    m->hd = hp.n_embd / hp.n_head;  // head_dim = n_embd / n_head always wins (src/model.cpp:22-24)
    if (hp.head_dim != m->hd) m->hp.head_dim = m->hd;
    if (m->hd % 8 || m->hd > AT_MAX_HD || hp.n_head % hp.n_kv_head || hp.n_head / hp.n_kv_head > AT_MAX_REP) {
        delete m;
        return set_error("unsupported attention shape (head_dim must be a multiple of 8 up to 128, n_head/n_kv_head <= 8)");
    }
    if (o.max_seq > AT_CHUNK * AT_MAX_SPLIT) {
        delete m;
        return set_error("max_seq above 16384 is not supported");
    }
    m->D = hp.n_embd;
    m->H = hp.n_head * m->hd;
    m->KV = hp.n_kv_head * m->hd;
    m->FF = hp.n_ff;
    m->V = hp.n_vocab;

    cudaError_t e = cudaSetDevice(o.device);
    if (e != cudaSuccess) {
        delete m;
        return set_error(std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    }
#define CKD(call)                                                                 \
    do {                                                                          \
        cudaError_t e_ = (call);                                                  \
        if (e_ != cudaSuccess) {                                                  \
            std::string s_ = std::string(#call) + ": " + cudaGetErrorString(e_); \
            tf_cuda_destroy(m);                                                   \
            return set_error(s_);                                                 \
        }                                                                         \
    } while (0)
#define BAD(msg)                  \
    do {                          \
        std::string s_ = (msg);   \
        tf_cuda_destroy(m);       \
        return set_error(s_);     \
    } while (0)
    CKD(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    CKD(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, o.device));
    CKD(gemv_init_attrs());

    for (int i = 0; i < nt; ++i) m->weight_bytes += t[i].nbytes;

    // ---- bind tensors as the reference does (src/model.cpp:43-65) ----
    auto need = [&](const std::string& n) -> const tf_tensor_desc* { return find_desc(t, nt, n); };
    const tf_tensor_desc* te = need("token_embd.weight");
    const tf_tensor_desc* on = need("output_norm.weight");
    const tf_tensor_desc* ow = need("output.weight");
    if (!te) BAD("missing tensor token_embd.weight");
    if (!on) BAD("missing tensor output_norm.weight");
    if (!ow) ow = te;
    struct LDesc {
        const tf_tensor_desc *an, *q, *k, *v, *o, *bq, *bk, *bv, *fn, *g, *u, *d;
    };
    std::vector<LDesc> ld(hp.n_layer);
    for (int i = 0; i < hp.n_layer; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        LDesc& L = ld[i];
        const char* must[] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight",
                              "attn_output.weight", "ffn_norm.weight", "ffn_gate.weight", "ffn_up.weight",
                              "ffn_down.weight"};
        const tf_tensor_desc** dst[] = {&L.an, &L.q, &L.k, &L.v, &L.o, &L.fn, &L.g, &L.u, &L.d};
        for (int j = 0; j < 9; ++j) {
            *dst[j] = need(p + must[j]);
            if (!*dst[j]) BAD("missing tensor " + p + must[j]);
        }
        L.bq = need(p + "attn_q.bias");
        L.bk = need(p + "attn_k.bias");
        L.bv = need(p + "attn_v.bias");
    }
    // ---- shape / type validation ----
    auto check_w = [&](const tf_tensor_desc* d, int K, int N) -> std::string {
        if (!type_ok(d->ggml_type)) return std::string("unsupported ggml type in ") + d->name;
        if (d->ne[0] != K || (N > 0 && d->ne[1] != N)) return std::string("unexpected shape of ") + d->name;
        const int be = blk_elems(d->ggml_type);
        if (K % be || K % 32) return std::string("row length not divisible by block size in ") + d->name;
        if ((long long)d->nbytes != row_bytes(d->ggml_type, K) * (N > 0 ? N : d->ne[1]))
            return std::string("byte size mismatch in ") + d->name;
        return "";
    };
    std::string s;
    if (!(s = check_w(te, m->D, 0)).empty()) BAD(s);
    if (te->ne[1] < m->V) BAD("token_embd has fewer rows than n_vocab");
    if (!(s = check_w(ow, m->D, 0)).empty()) BAD(s);
    if (ow->ne[1] < m->V) BAD("output has fewer rows than n_vocab");
    if (on->ggml_type != T_F32 || on->ne[0] != m->D) BAD("output_norm.weight must be F32 [n_embd]");
    for (int i = 0; i < hp.n_layer; ++i) {
        LDesc& L = ld[i];
        if (!(s = check_w(L.q, m->D, m->H)).empty()) BAD(s);
        if (!(s = check_w(L.k, m->D, m->KV)).empty()) BAD(s);
        if (!(s = check_w(L.v, m->D, m->KV)).empty()) BAD(s);
        if (!(s = check_w(L.o, m->H, m->D)).empty()) BAD(s);
        if (!(s = check_w(L.g, m->D, m->FF)).empty()) BAD(s);
        if (!(s = check_w(L.u, m->D, m->FF)).empty()) BAD(s);
        if (!(s = check_w(L.d, m->FF, m->D)).empty()) BAD(s);
        if (L.q->ggml_type != L.k->ggml_type || L.q->ggml_type != L.v->ggml_type)
            BAD("attn_q/k/v of one layer must share a type (they are streamed as one block)");
        if (L.g->ggml_type != L.u->ggml_type) BAD("ffn_gate/ffn_up of one layer must share a type");
        if (L.an->ggml_type != T_F32 || L.fn->ggml_type != T_F32) BAD("norm weights must be F32");
        const bool any_b = L.bq || L.bk || L.bv;
        if (any_b && !(L.bq && L.bk && L.bv)) BAD("q/k/v biases must be all present or all absent");
        if (any_b && (L.bq->ggml_type != T_F32 || L.bk->ggml_type != T_F32 || L.bv->ggml_type != T_F32))
            BAD("q/k/v biases must be F32 (read as raw floats, src/model.cpp:85-89)");
    }

    // ---- arena layout ----
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o2 = off;
        off = (off + bytes + 255) & ~(size_t)255;
        return o2;
    };
    struct Place {
        size_t an, qkv, b, o, fn, gu, d;
    };
    std::vector<Place> pl(hp.n_layer);
    for (int i = 0; i < hp.n_layer; ++i) {
        LDesc& L = ld[i];
        pl[i].an = take(L.an->nbytes);
        pl[i].qkv = take(L.q->nbytes + L.k->nbytes + L.v->nbytes);
        pl[i].b = L.bq ? take((size_t)(m->H + 2 * m->KV) * 4) : 0;
        pl[i].o = take(L.o->nbytes);
        pl[i].fn = take(L.fn->nbytes);
        pl[i].gu = take(L.g->nbytes + L.u->nbytes);
        pl[i].d = take(L.d->nbytes);
    }
    const size_t p_embd = take(te->nbytes);
    const size_t p_out = (ow == te) ? p_embd : take(ow->nbytes);
    const size_t p_onorm = take(on->nbytes);
    const size_t arena_bytes = off + 256;
    CKD(cudaMalloc(&m->arena, arena_bytes));
    CKD(cudaMemset(m->arena + off, 0, 256));
    uint8_t* A = m->arena;

    auto wref = [&](const uint8_t* p, int type, int K, int rows) {
        WeightRef w;
        w.p = p;
        w.type = type;
        w.K = K;
        w.rb = row_bytes(type, K);
        w.rows = rows;
        return w;
    };
    // power-of-two scale of a matrix for the tensor-core GEMM (Q8_0 and Q4_0 rows)
    auto wscale = [](const tf_tensor_desc* t) {
        const uint8_t* b = static_cast<const uint8_t*>(t->data);
        if (t->ggml_type == T_Q8_0) return q8_scale_exponent(b, t->nbytes, 34);
        if (t->ggml_type == T_Q4_0) return q8_scale_exponent(b, t->nbytes, 18);
        return 0;
    };
    // every tensor goes through the pinned, double-buffered uploader (TFB200_UPLOAD_SYNC=1: one
    // synchronous pageable cudaMemcpy per tensor instead, for comparison)
    Uploader up;
    const char* usync = getenv("TFB200_UPLOAD_SYNC");
    const bool streamed = !(usync && usync[0] == '1');
    if (streamed) {
        // staging: TFB200_UPLOAD_CHUNK_MB per buffer (default 2: measured fastest of 2 / 8 / 32 MB
        // with the file in the page cache), 4 buffers, host copies on TFB200_UPLOAD_THREADS
        // threads (default 1: more threads measured no faster)
        const char* ce = getenv("TFB200_UPLOAD_CHUNK_MB");
        const char* te = getenv("TFB200_UPLOAD_THREADS");
        const size_t chunk = (size_t)std::max(1, ce ? atoi(ce) : 2) << 20;
        const int threads = std::max(1, std::min(32, te ? atoi(te) : 1));
        CKD(up.init(chunk, 4, threads));
    }
    auto put = [&](void* dst, const void* src, size_t n) -> cudaError_t {
        return streamed ? up.copy(dst, src, n) : cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice);
    };
    auto put_rows = [&](void* dst, size_t dpitch, const void* src, size_t width, size_t rows) -> cudaError_t {
        return streamed ? up.copy_rows(dst, dpitch, src, width, rows)
                        : cudaMemcpy2D(dst, dpitch, src, width, width, rows, cudaMemcpyHostToDevice);
    };
    const auto t_up = std::chrono::steady_clock::now();
    m->L.resize(hp.n_layer);
    for (int i = 0; i < hp.n_layer; ++i) {
        LDesc& L = ld[i];
        LayerDev& Ld = m->L[i];
        CKD(put(A + pl[i].an, L.an->data, L.an->nbytes));
        Ld.attn_norm = reinterpret_cast<const float*>(A + pl[i].an);
        CKD(put(A + pl[i].qkv, L.q->data, L.q->nbytes));
        CKD(put(A + pl[i].qkv + L.q->nbytes, L.k->data, L.k->nbytes));
        CKD(put(A + pl[i].qkv + L.q->nbytes + L.k->nbytes, L.v->data, L.v->nbytes));
        Ld.qkv = wref(A + pl[i].qkv, L.q->ggml_type, m->D, m->H + 2 * m->KV);
        Ld.qkv.sw = std::min({wscale(L.q), wscale(L.k), wscale(L.v)});
        Ld.bqkv = nullptr;
        if (L.bq) {
            float* b = reinterpret_cast<float*>(A + pl[i].b);
            CKD(put(b, L.bq->data, (size_t)m->H * 4));
            CKD(put(b + m->H, L.bk->data, (size_t)m->KV * 4));
            CKD(put(b + m->H + m->KV, L.bv->data, (size_t)m->KV * 4));
            Ld.bqkv = b;
        }
        CKD(put(A + pl[i].o, L.o->data, L.o->nbytes));
        Ld.wo = wref(A + pl[i].o, L.o->ggml_type, m->H, m->D);
        Ld.wo.sw = wscale(L.o);
        CKD(put(A + pl[i].fn, L.fn->data, L.fn->nbytes));
        Ld.ffn_norm = reinterpret_cast<const float*>(A + pl[i].fn);
        const size_t grb = (size_t)row_bytes(L.g->ggml_type, m->D);
        CKD(put_rows(A + pl[i].gu, 2 * grb, L.g->data, grb, m->FF));
        CKD(put_rows(A + pl[i].gu + grb, 2 * grb, L.u->data, grb, m->FF));
        Ld.gateup = wref(A + pl[i].gu, L.g->ggml_type, m->D, 2 * m->FF);
        Ld.gateup.sw = std::min(wscale(L.g), wscale(L.u));
        CKD(put(A + pl[i].d, L.d->data, L.d->nbytes));
        Ld.down = wref(A + pl[i].d, L.d->ggml_type, m->FF, m->D);
        Ld.down.sw = wscale(L.d);
    }
    CKD(put(A + p_embd, te->data, te->nbytes));
    m->embd = wref(A + p_embd, te->ggml_type, m->D, (int)te->ne[1]);
    if (ow != te) CKD(put(A + p_out, ow->data, ow->nbytes));
    m->outw = wref(A + p_out, ow->ggml_type, m->D, (int)ow->ne[1]);
    m->outw.sw = wscale(ow);
    {
        // steps of >= 16 rows take the tensor-core path when the matrices it can run (Q8_0,
        // Q4_0) hold most of the layer weight bytes; the others of such a step (Q4_1, Q6_K,
        // F16, F32) run the multi-row GEMV inside it
        long long tc = 0, all = 0;
        for (const LayerDev& Ld : m->L)
            for (const WeightRef* w : {&Ld.qkv, &Ld.wo, &Ld.gateup, &Ld.down}) {
                const long long b = w->rb * w->rows;
                all += b;
                if (gemm_weight_ok(*w)) tc += b;
            }
        m->gemm_ok = all > 0 && 2 * tc >= all;
    }
    CKD(put(A + p_onorm, on->data, on->nbytes));
    if (streamed) CKD(up.finish());
    m->upload_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_up).count();
    if (const char* e = getenv("TFB200_GV_TRACE"); e && e[0] == '1') {
        const size_t n = (size_t)GV_TRACE_LAUNCHES * GV_TRACE_CTAS * GV_TRACE_SLOTS;
        CKD(cudaMalloc(&m->d_gvtrace, n * sizeof(unsigned long long)));
        CKD(cudaMemset(m->d_gvtrace, 0, n * sizeof(unsigned long long)));
    }
    m->out_norm = reinterpret_cast<const float*>(A + p_onorm);

    // ---- KV cache: per layer [slot][kv_head][cap][hd] ----
    const size_t esz = o.kv_type == TF_KV_F32 ? 4 : 2;
    m->slot_elems = (long long)hp.n_kv_head * o.max_seq * m->hd;
    m->layer_elems = m->slot_elems * o.max_batch;
    const size_t kv_bytes = (size_t)m->layer_elems * hp.n_layer * esz;
    CKD(cudaMalloc(&m->kc, kv_bytes));
    CKD(cudaMalloc(&m->vc, kv_bytes));
    CKD(cudaMemset(m->kc, 0, kv_bytes));
    CKD(cudaMemset(m->vc, 0, kv_bytes));

    // ---- RoPE table: cos/sin((float)pos * freq[i]) in float, as rope_one computes them ----
    {
        std::vector<float> f;
        rope_freqs_host(f, m->hp);
        const int d2 = m->hd / 2;
        std::vector<float> c((size_t)o.max_seq * d2), sn((size_t)o.max_seq * d2);
        for (int p = 0; p < o.max_seq; ++p)
            for (int i = 0; i < d2; ++i) {
                const float ang = (float)p * f[i];
                c[(size_t)p * d2 + i] = std::cos(ang);
                sn[(size_t)p * d2 + i] = std::sin(ang);
            }
        CKD(cudaMalloc(&m->cosb, c.size() * 4));
        CKD(cudaMalloc(&m->sinb, sn.size() * 4));
        CKD(cudaMemcpy(m->cosb, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
        CKD(cudaMemcpy(m->sinb, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    }

    // ---- scratch ----
    int tile = GV_MAXM;
    for (int K : {m->D, m->H, m->FF}) tile = std::min(tile, gemv_max_rows(K));
    m->tile = std::max(1, std::min(tile, o.max_batch));
    m->gtile = (m->gemm_ok && o.max_batch >= GM_MIN_M) ? o.max_batch : 0;
    m->ptile = m->gemm_ok ? std::min(GM_BM, o.max_seq) : 0;
    if (m->ptile < GM_MIN_M) m->ptile = 0;
    m->n_split = attn_pick_split(o.max_seq);
    const int T = std::max(m->tile, std::max(m->gtile, m->ptile));
    if (m->gtile || m->ptile) {
        const int Kmax = std::max(m->D, std::max(m->H, m->FF));
        const size_t rows = (size_t)(std::max(m->gtile, m->ptile) + GM_ROW_PAD - 1) / GM_ROW_PAD * GM_ROW_PAD;
        CKD(cudaMalloc(&m->xh, rows * Kmax * sizeof(__half)));
        CKD(cudaMalloc(&m->xl, rows * Kmax * sizeof(__half)));
        CKD(cudaMemset(m->xh, 0, rows * Kmax * sizeof(__half)));
        CKD(cudaMemset(m->xl, 0, rows * Kmax * sizeof(__half)));
        CKD(cudaMalloc(&m->d_sx, rows * sizeof(int)));
        CKD(cudaMemset(m->d_sx, 0, rows * sizeof(int)));
        CKD(cudaMalloc(&m->gws, gemm_ws_floats(m->num_sms) * sizeof(float)));
        CKD(cudaMalloc(&m->gcnt, gemm_tile_counters(m->num_sms) * sizeof(unsigned)));
        CKD(cudaMemset(m->gcnt, 0, gemm_tile_counters(m->num_sms) * sizeof(unsigned)));
    }
    CKD(cudaMalloc(&m->x, sizeof(float) * T * m->D));
    CKD(cudaMalloc(&m->qkv, sizeof(float) * T * (m->H + 2 * m->KV)));
    CKD(cudaMalloc(&m->attn, sizeof(float) * T * m->H));
    CKD(cudaMalloc(&m->xplanes, (size_t)q8_plane_bytes(std::max(m->FF, m->H))));
    CKD(cudaMalloc(&m->h, sizeof(float) * T * m->FF));
    CKD(cudaMalloc(&m->logits, sizeof(float) * (size_t)T * m->V));
    CKD(cudaMalloc(&m->part, sizeof(float) * (size_t)T * hp.n_head * m->n_split * (m->hd + 2)));
    CKD(cudaMalloc(&m->counters, sizeof(unsigned) * T * hp.n_kv_head));
    CKD(cudaMemset(m->counters, 0, sizeof(unsigned) * T * hp.n_kv_head));
    CKD(cudaMalloc(&m->keys, sizeof(unsigned long long) * (T < 2 ? 2 : T)));
    CKD(cudaMemset(m->keys, 0, sizeof(unsigned long long) * (T < 2 ? 2 : T)));
    CKD(cudaMalloc(&m->d_tokens, sizeof(int) * T));
    CKD(cudaMemset(m->d_tokens, 0, sizeof(int) * T));
    CKD(cudaMalloc(&m->d_slots, sizeof(int) * T));
    CKD(cudaMemset(m->d_slots, 0, sizeof(int) * T));
    CKD(cudaMalloc(&m->d_pos, sizeof(int) * o.max_batch));
    CKD(cudaMemset(m->d_pos, 0, sizeof(int) * o.max_batch));
    CKD(cudaMalloc(&m->d_wstart, sizeof(int) * o.max_batch));
    CKD(cudaMemset(m->d_wstart, 0, sizeof(int) * o.max_batch));
    CKD(cudaMalloc(&m->d_hist, sizeof(int) * ((size_t)o.max_seq + 1) * T));
    CKD(cudaMalloc(&m->d_prompt, sizeof(int) * ((size_t)o.max_seq + 1)));
    CKD(cudaMalloc(&m->d_err, sizeof(int)));
    CKD(cudaMemset(m->d_err, 0, sizeof(int)));
    CKD(cudaMalloc(&m->d_async, sizeof(unsigned) * (2 * hp.n_layer + hp.n_head)));
    CKD(cudaMemset(m->d_async, 0, sizeof(unsigned) * (2 * hp.n_layer + hp.n_head)));
    CKD(cudaMalloc(&m->ctl, sizeof(StepCtl)));
    CKD(cudaMemset(m->ctl, 0, sizeof(StepCtl)));
    CKD(cudaMallocHost(&m->hi, sizeof(int) * 64 + sizeof(int) * ((size_t)o.max_seq + 1) * 2));
    CKD(cudaMallocHost(&m->hb, sizeof(int) * 2 * (size_t)T));
    m->smp = sample_scratch_create(m->V);
    if (!m->smp) BAD("sampler scratch allocation failed");
    CKD(cudaMallocHost(&m->hlog, sizeof(float) * (size_t)T * m->V));
    m->hpos.assign(o.max_batch, 0);
    if (o.decode_mode != TF_DECODE_KERNELS) {
        const int rc = build_pk_plan(m);
        if (rc < 0) BAD(m->err);
        if (rc > 0 && o.decode_mode == TF_DECODE_PERSISTENT) BAD("the persistent decode kernel does not take this model");
    }
    {   // positions per tile of the attention fused into the QKV kernel (same for every layer)
        const GemvArgs q = gemv_base(m, m->L[0].qkv, m->H + 2 * m->KV, 1, 1);
        m->attn_tile = (q.intq && !q.q4 && !q.q6) ? fused_attn_tile(q, m->hd) : 0;
    }
    CKD(cudaDeviceSynchronize());
    {
        int n = 0;
        // count launches of one step (no device work: enqueue into a throwaway capture)
        cudaGraph_t g = nullptr;
        CKD(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_step(m, 1, true, true, &n, fuse_attn_ok(m, 1));
        cudaStreamEndCapture(m->stream, &g);
        if (g) cudaGraphDestroy(g);
        if (rc) BAD(m->err);
        m->kernels_per_step = m->pk ? 1 : n;
    }
    *out = m;
    return 0;
#undef CKD
#undef BAD
}

int tf_cuda_reset(tf_model* m, int seq) {
    if (!m) return set_error("null model");
    CK(cudaSetDevice(m->device));
    const int s0 = seq < 0 ? 0 : seq, s1 = seq < 0 ? m->opt.max_batch : seq + 1;
    if (seq >= m->opt.max_batch) return fail(m, "sequence slot out of range");
    const size_t esz = m->opt.kv_type == TF_KV_F32 ? 4 : 2;
    for (int s = s0; s < s1; ++s) {
        m->hpos[s] = 0;
        for (int li = 0; li < m->hp.n_layer; ++li) {  // KVCache::clear (src/kvcache.cpp:16-19)
            const size_t o2 = ((size_t)li * m->layer_elems + (size_t)s * m->slot_elems) * esz;
            CK(cudaMemsetAsync(static_cast<uint8_t*>(m->kc) + o2, 0, m->slot_elems * esz, m->stream));
            CK(cudaMemsetAsync(static_cast<uint8_t*>(m->vc) + o2, 0, m->slot_elems * esz, m->stream));
        }
    }
    CK(cudaMemsetAsync(m->d_pos + s0, 0, sizeof(int) * (s1 - s0), m->stream));
    CK(cudaMemsetAsync(m->d_wstart + s0, 0, sizeof(int) * (s1 - s0), m->stream));
    return finish_call(m);
}

int tf_cuda_decode(tf_model* m, int seq, int token, float* logits, int* argmax_out) {
    if (!m) return set_error("null model");
    CK(cudaSetDevice(m->device));
    if (check_seq(m, seq)) return -1;
    if (m->hpos[seq] + 1 > m->opt.max_seq) return fail(m, "decode exceeds max_seq");
    if (token < 0 || token >= m->V) return fail(m, "token id out of range");
    if (set_slot_row(m, 0, seq, token)) return -1;
    if (m->pk) {
        if (run_pk(m, seq, m->d_tokens, 1, 1, 0, 0, 0)) return -1;
    } else if (run_step(m, 1, true, fuse_attn_ok(m, m->hpos[seq] + 1))) {
        return -1;
    }
    m->hpos[seq] += 1;
    return read_outputs(m, 1, logits, argmax_out);
}

int tf_cuda_prefill(tf_model* m, int seq, const int* tokens, int n, float* logits, int* argmax_out) {
    if (!m) return set_error("null model");
    if (n <= 0) return 0;  // Model::prefill returns immediately (src/model.cpp:184)
    CK(cudaSetDevice(m->device));
    if (check_seq(m, seq)) return -1;
    if (!tokens) return fail(m, "tokens is null");
    if (m->hpos[seq] + n > m->opt.max_seq) return fail(m, "prefill exceeds max_seq");
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->V) return fail(m, "token id out of range");
    int* stage = m->hi + 64;
    memcpy(stage, tokens, sizeof(int) * n);
    CK(cudaMemcpyAsync(m->d_prompt, stage, sizeof(int) * n, cudaMemcpyHostToDevice, m->stream));
    if (m->pk && !(m->ptile && n >= GM_MIN_M)) {
        // short prompts: all n token steps in one persistent launch; attention inside the
        // chunk sees the chunk alone, from its first position; the lm_head runs for the last
        // token only (prompts of >= 16 tokens take the tensor-core chunks below)
        if (run_pk(m, seq, m->d_prompt, n, n, n - 1, m->hpos[seq], 0)) return -1;
        m->hpos[seq] += n;
        return read_outputs(m, 1, logits, argmax_out);
    }
    // attention inside the chunk sees the chunk alone, from its first position
    m->hi[2] = m->hpos[seq];
    m->hi[3] = 0;
    CK(cudaMemcpyAsync(m->d_wstart + seq, m->hi + 2, sizeof(int), cudaMemcpyHostToDevice, m->stream));
    if (m->ptile && n >= GM_MIN_M) {
        // tensor-core path: the prompt in chunks of up to ptile rows (every chunk >= 16 rows)
        const int nc = (n + m->ptile - 1) / m->ptile;
        const int TT = std::max(m->tile, std::max(m->gtile, m->ptile));
        for (int b = 0; b < m->ptile; ++b) m->hb[TT + b] = seq;
        CK(cudaMemcpyAsync(m->d_slots, m->hb + TT, sizeof(int) * m->ptile, cudaMemcpyHostToDevice, m->stream));
        int c0 = 0, rows = 0;
        for (int c = 0; c < nc; ++c) {
            rows = (int)((long long)n * (c + 1) / nc) - c0;
            CK(cudaMemcpyAsync(m->d_tokens, m->d_prompt + c0, sizeof(int) * rows, cudaMemcpyDeviceToDevice, m->stream));
            if (run_step(m, rows, c == nc - 1, false, true)) return -1;
            c0 += rows;
        }
        CK(cudaMemcpyAsync(m->d_wstart + seq, m->hi + 3, sizeof(int), cudaMemcpyHostToDevice, m->stream));
        m->hpos[seq] += n;
        return read_outputs_row(m, rows - 1, logits, argmax_out);
    }
    if (set_slot_row(m, 0, seq, tokens[0])) return -1;
    for (int i = 0; i < n; ++i) {
        CK(cudaMemcpyAsync(m->d_tokens, m->d_prompt + i, sizeof(int), cudaMemcpyDeviceToDevice, m->stream));
        if (run_step(m, 1, i == n - 1, fuse_attn_ok(m, m->hpos[seq] + n))) return -1;
    }
    CK(cudaMemcpyAsync(m->d_wstart + seq, m->hi + 3, sizeof(int), cudaMemcpyHostToDevice, m->stream));
    m->hpos[seq] += n;
    return read_outputs(m, 1, logits, argmax_out);
}

int tf_cuda_generate_greedy(tf_model* m, int seq, int first_token, int n, int eos, int* out_ids, int* n_out) {
    if (!m) return set_error("null model");
    if (n_out) *n_out = 0;
    if (n <= 0) return 0;
    CK(cudaSetDevice(m->device));
    if (check_seq(m, seq)) return -1;
    if (!out_ids) return fail(m, "out_ids is null");
    if (m->hpos[seq] + n > m->opt.max_seq) return fail(m, "decode exceeds max_seq");
    if (first_token < 0 || first_token >= m->V) return fail(m, "token id out of range");
    if (set_slot_row(m, 0, seq, first_token)) return -1;
    if (m->pk) {
        if (run_pk(m, seq, m->d_tokens, 1, n, 0, 0, n)) return -1;
    } else {
        StepCtl c = {0u, 0, n, 0};
        memcpy(m->hi + 4, &c, sizeof(c));
        CK(cudaMemcpyAsync(m->ctl, m->hi + 4, sizeof(StepCtl), cudaMemcpyHostToDevice, m->stream));
        const int fz = fuse_attn_ok(m, m->hpos[seq] + n);
        for (int i = 0; i < n; ++i)
            if (run_step(m, 1, true, fz)) return -1;
    }
    int* hist = m->hi + 64;
    CK(cudaMemcpyAsync(hist, m->d_hist, sizeof(int) * n, cudaMemcpyDeviceToHost, m->stream));
    int rc = finish_call(m);
    if (rc) return rc;
    // accepted ids: t0 = first_token, t_i = hist[i-1]; stop before t_j == eos, j > 0
    // (src/main.cpp:113-121); j decodes were needed for the accepted tokens.
    int j = n;
    out_ids[0] = first_token;
    for (int i = 1; i < n; ++i) {
        if (eos >= 0 && hist[i - 1] == eos) {
            j = i;
            break;
        }
        out_ids[i] = hist[i - 1];
    }
    const int pos0 = m->hpos[seq];
    m->hpos[seq] = pos0 + j;
    if (j < n) {
        m->hi[2] = pos0 + j;
        CK(cudaMemcpyAsync(m->d_pos + seq, m->hi + 2, sizeof(int), cudaMemcpyHostToDevice, m->stream));
        CK(cudaStreamSynchronize(m->stream));
    }
    if (n_out) *n_out = j;
    return 0;
}

int tf_cuda_set_vocab_shard(tf_model* m, int rank, int world) {
    if (!m) return set_error("null model");
    if (world < 1 || rank < 0 || rank >= world || world > m->V) return fail(m, "bad vocab shard (rank, world)");
    CK(cudaSetDevice(m->device));
    if (!m->d_keyred) CK(cudaMalloc(&m->d_keyred, sizeof(long long)));
    const int r0 = (int)((long long)m->V * rank / world), r1 = (int)((long long)m->V * (rank + 1) / world);
    if (r0 != m->vs_row0 || r1 != m->vs_row1 || (world > 1) != m->vsplit) {
        // captured steps hold the old rows: capture again
        for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
        m->graphs.clear();
    }
    m->vs_row0 = r0;
    m->vs_row1 = r1;
    m->vsplit = world > 1;
    return 0;
}

void* tf_cuda_shard_key(tf_model* m) { return m ? static_cast<void*>(m->d_keyred) : nullptr; }

int tf_cuda_decode_shard(tf_model* m, int seq, int token) {
    if (!m) return set_error("null model");
    if (!m->d_keyred) return fail(m, "tf_cuda_set_vocab_shard was not called");
    CK(cudaSetDevice(m->device));
    if (check_seq(m, seq)) return -1;
    if (m->hpos[seq] + 1 > m->opt.max_seq) return fail(m, "decode exceeds max_seq");
    if (token >= m->V) return fail(m, "token id out of range");
    const bool from_key = token < 0;
    if (!from_key) {  // the first step of a run: host token, fresh step counter and history
        if (set_slot_row(m, 0, seq, token)) return -1;
        StepCtl c = {0u, 0, m->opt.max_seq, 0};
        memcpy(m->hi + 4, &c, sizeof(c));
        CK(cudaMemcpyAsync(m->ctl, m->hi + 4, sizeof(StepCtl), cudaMemcpyHostToDevice, m->stream));
    }
    m->split_step = m->vsplit;
    const int rc = run_step(m, 1, true, fuse_attn_ok(m, m->hpos[seq] + 1), false, from_key);
    m->split_step = false;
    if (rc) return -1;
    m->hpos[seq] += 1;
    return 0;
}

int tf_cuda_shard_token(tf_model* m, int seq, int* token) {
    if (!m) return set_error("null model");
    if (!m->d_keyred || !token) return fail(m, "no vocab shard, or token is null");
    CK(cudaSetDevice(m->device));
    if (check_seq(m, seq)) return -1;
    CK(key_apply_launch(m->d_keyred, m->d_tokens, m->d_hist, m->ctl, m->stream));
    CK(cudaMemcpyAsync(m->hb, m->d_tokens, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    const int rc = finish_call(m);
    if (rc) return rc;
    *token = m->hb[0];
    return 0;
}

int tf_cuda_trace_read(tf_model* m, unsigned long long* out, int cap, int* n_out) {
    if (!m) return set_error("null model");
    if (!m->d_pktrace) return fail(m, "no phase trace (persistent kernel created with TFB200_PK_TRACE=1)");
    if (!out || !n_out || cap < 1) return fail(m, "bad trace buffer");
    CK(cudaSetDevice(m->device));
    int n[2] = {0, 0};
    CK(cudaStreamSynchronize(m->stream));
    CK(cudaMemcpy(n, m->d_pktrace_n, sizeof(n), cudaMemcpyDeviceToHost));
    for (int w = 0; w < 2; ++w) {
        const int k = std::min(std::min(n[w], m->pk_trace_cap), cap);
        if (k) CK(cudaMemcpy(out + (size_t)w * cap, m->d_pktrace + (size_t)w * m->pk_trace_cap, sizeof(unsigned long long) * k,
                             cudaMemcpyDeviceToHost));
        n_out[w] = k;
    }
    return 0;
}

int tf_cuda_launch_trace(tf_model* m, unsigned long long* out, int max_launches, int* meta, int* n_launch) {
    if (!m) return set_error("null model");
    if (!m->d_gvtrace) return fail(m, "no launch trace (model created with TFB200_GV_TRACE=1)");
    if (!out || !meta || !n_launch || max_launches < 1) return fail(m, "bad trace buffer");
    CK(cudaSetDevice(m->device));
    const int n = std::min((int)m->gvt_meta.size() / 3, max_launches);
    CK(cudaStreamSynchronize(m->stream));
    CK(cudaMemcpy(out, m->d_gvtrace, sizeof(unsigned long long) * (size_t)n * GV_TRACE_CTAS * GV_TRACE_SLOTS,
                  cudaMemcpyDeviceToHost));
    memcpy(meta, m->gvt_meta.data(), sizeof(int) * 3 * (size_t)n);
    *n_launch = n;
    return 0;
}

int tf_cuda_history(tf_model* m, int n, int* out) {
    if (!m) return set_error("null model");
    if (n < 0 || n > m->opt.max_seq || (n && !out)) return fail(m, "bad history request");
    if (!n) return 0;
    CK(cudaSetDevice(m->device));
    CK(cudaMemcpyAsync(m->hi + 64, m->d_hist, sizeof(int) * n, cudaMemcpyDeviceToHost, m->stream));
    const int rc = finish_call(m);
    if (rc) return rc;
    memcpy(out, m->hi + 64, sizeof(int) * n);
    return 0;
}

int tf_cuda_decode_batch(tf_model* m, const int* seq_ids, const int* tokens, int B, int* argmax_out, float* logits) {
    if (!m) return set_error("null model");
    if (B <= 0) return 0;
    CK(cudaSetDevice(m->device));
    if (!seq_ids || !tokens) return fail(m, "null seq_ids or tokens");
    std::vector<char> seen(m->opt.max_batch, 0);
    for (int b = 0; b < B; ++b) {
        if (check_seq(m, seq_ids[b])) return -1;
        if (seen[seq_ids[b]]) return fail(m, "duplicate sequence slot in one batch");
        seen[seq_ids[b]] = 1;
        if (m->hpos[seq_ids[b]] + 1 > m->opt.max_seq) return fail(m, "decode exceeds max_seq");
        if (tokens[b] < 0 || tokens[b] >= m->V) return fail(m, "token id out of range");
    }
    // rows per step: the tensor-core GEMM path takes up to gtile rows, the GEMV up to tile
    const int chunk = (m->gtile && B >= GM_MIN_M) ? m->gtile : m->tile;
    for (int b0 = 0; b0 < B; b0 += chunk) {
        const int T = std::min(chunk, B - b0);
        const int TT = std::max(m->tile, m->gtile);
        memcpy(m->hb, tokens + b0, sizeof(int) * T);
        memcpy(m->hb + TT, seq_ids + b0, sizeof(int) * T);
        CK(cudaMemcpyAsync(m->d_tokens, m->hb, sizeof(int) * T, cudaMemcpyHostToDevice, m->stream));
        CK(cudaMemcpyAsync(m->d_slots, m->hb + TT, sizeof(int) * T, cudaMemcpyHostToDevice, m->stream));
        if (run_step(m, T, true, false)) return -1;
        for (int b = 0; b < T; ++b) m->hpos[seq_ids[b0 + b]] += 1;
        int rc = read_outputs(m, T, logits ? logits + (size_t)b0 * m->V : nullptr, argmax_out ? argmax_out + b0 : nullptr);
        if (rc) return rc;
    }
    return 0;
}

int tf_cuda_prefill_batch(tf_model* m, const int* seq_ids, const int* tokens, int B, int n, int* argmax_out) {
    if (!m) return set_error("null model");
    if (B <= 0 || n <= 0) return 0;
    CK(cudaSetDevice(m->device));
    if (!seq_ids || !tokens) return fail(m, "null seq_ids or tokens");
    std::vector<char> seen(m->opt.max_batch, 0);
    for (int b = 0; b < B; ++b) {
        if (check_seq(m, seq_ids[b])) return -1;
        if (seen[seq_ids[b]]) return fail(m, "duplicate sequence slot in one batch");
        seen[seq_ids[b]] = 1;
        if (m->hpos[seq_ids[b]] + n > m->opt.max_seq) return fail(m, "prefill exceeds max_seq");
        for (int t = 0; t < n; ++t)
            if (tokens[(size_t)b * n + t] < 0 || tokens[(size_t)b * n + t] >= m->V) return fail(m, "token id out of range");
    }
    const int TT = std::max(m->tile, m->gtile);
    const int chunk = (m->gtile && B >= GM_MIN_M) ? m->gtile : m->tile;
    for (int b0 = 0; b0 < B; b0 += chunk) {
        const int T = std::min(chunk, B - b0);
        // attention of each sequence starts at its prompt (src/attention.cpp:82-111)
        for (int b = 0; b < T; ++b) {
            const int sq = seq_ids[b0 + b];
            m->hb[b] = m->hpos[sq];
            CK(cudaMemcpyAsync(m->d_wstart + sq, m->hb + b, sizeof(int), cudaMemcpyHostToDevice, m->stream));
        }
        CK(cudaStreamSynchronize(m->stream));
        memcpy(m->hb + TT, seq_ids + b0, sizeof(int) * T);
        CK(cudaMemcpyAsync(m->d_slots, m->hb + TT, sizeof(int) * T, cudaMemcpyHostToDevice, m->stream));
        for (int t = 0; t < n; ++t) {
            CK(cudaStreamSynchronize(m->stream));  // the staging row is reused each step
            for (int b = 0; b < T; ++b) m->hb[b] = tokens[(size_t)(b0 + b) * n + t];
            CK(cudaMemcpyAsync(m->d_tokens, m->hb, sizeof(int) * T, cudaMemcpyHostToDevice, m->stream));
            if (run_step(m, T, t == n - 1, false)) return -1;
        }
        for (int b = 0; b < T; ++b) m->hpos[seq_ids[b0 + b]] += n;
        m->hi[3] = 0;
        for (int b = 0; b < T; ++b)
            CK(cudaMemcpyAsync(m->d_wstart + seq_ids[b0 + b], m->hi + 3, sizeof(int), cudaMemcpyHostToDevice, m->stream));
        int rc = read_outputs(m, T, nullptr, argmax_out ? argmax_out + b0 : nullptr);
        if (rc) return rc;
    }
    return 0;
}

int tf_cuda_sample(tf_model* m, int row, float temperature, float top_p, float r, int* out_id) {
    if (!m) return set_error("null model");
    if (!out_id) return fail(m, "out_id is null");
    const int T = std::max(m->tile, std::max(m->gtile, m->ptile));
    if (row < 0 || row >= T) return fail(m, "row out of range");
    CK(cudaSetDevice(m->device));
    const float* lg = m->logits + (size_t)row * m->V;
    if (temperature <= 0.0f) {  // sample_greedy (src/sampler.cpp:8-13)
        CK(launch_argmax(lg, m->V, 1, m->d_tokens + row, m->stream));
        CK(cudaMemcpyAsync(m->hb, m->d_tokens + row, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    } else {
        CK(sample_launch(m->smp, lg, m->V, temperature, top_p, r, m->stream));
        CK(cudaMemcpyAsync(m->hb, sample_result(m->smp), sizeof(int), cudaMemcpyDeviceToHost, m->stream));
    }
    int rc = finish_call(m);
    if (rc) return rc;
    *out_id = m->hb[0];
    return 0;
}

int tf_cuda_n_pos(tf_model* m, int seq) {
    if (!m || seq < 0 || seq >= m->opt.max_batch) return -1;
    return m->hpos[seq];
}
int tf_cuda_n_vocab(tf_model* m) { return m ? m->V : -1; }
unsigned long long tf_cuda_weight_bytes(tf_model* m) { return m ? m->weight_bytes : 0ull; }
void* tf_cuda_stream(tf_model* m) { return m ? (void*)m->stream : nullptr; }
int tf_cuda_kernels_per_step(tf_model* m) { return m ? m->kernels_per_step : -1; }

}  // extern "C"
