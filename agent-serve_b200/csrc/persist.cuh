// Persistent batch-1 decode kernel: one cooperative launch runs whole token steps of one
// sequence (Model::decode, src/model.cpp:197-208; the token steps of Model::prefill,
// :183-195; the CLI's greedy loop, src/main.cpp:112-122) for models whose layer matrices and
// lm_head are Q8_0.
//
// A step is, per layer, QKV GEMV -> attention -> wo GEMV -> gate/up GEMV -> down GEMV, then
// the lm_head: five all-to-all dependencies per layer.  As separate kernels every boundary
// costs a launch, a drain and a prologue while HBM idles.  Here every CTA (one per SM) owns
// the same slice of rows of every matrix for the whole launch, so its producer warp can walk
// its own weight schedule - every matrix of every layer of every step - and keep a ring of
// shared-memory stages full with 1-D bulk copies (TMA engine) without ever waiting for an
// activation.  The next phase's weights are already on chip when its activation is ready.
// Phases are separated by grid-wide arrival counters (bounded waits), not kernel launches.
#pragma once

#include "common.cuh"

namespace tfb {

constexpr int PK_WARPS = 16;                  // consumer warps per CTA
constexpr int PK_CONS = PK_WARPS * 32;        // consumer threads
constexpr int PK_THREADS = PK_CONS + 32;      // + one producer warp
constexpr int PK_MAX_SLOTS = 8;               // ring slots (weight stages) per CTA
constexpr int PK_SLOT_BUDGET = 36 * 1024;     // target weight bytes per stage
constexpr int PK_SMEM_LIMIT = 227 * 1024;     // dynamic shared memory per CTA
constexpr int PK_PRO_U = 4;                   // float4 activation chunks per consumer thread
constexpr int PK_MAX_K = PK_CONS * 4 * PK_PRO_U;  // longest row (8192 elements)
constexpr int PK_MAX_TP = PK_CONS;            // attention positions per tile (one per thread)
constexpr int PK_ROWS = 64;                   // residual rows / QKV rows a CTA may own
constexpr int PK_MAX_D2 = 128;                // head_dim / 2 of the RoPE table row kept on chip

// matrices per layer in the table: QKV (rows q | k | v), wo, gate/up (row pairs), down; the
// lm_head follows the last layer's
enum : int { PK_QKV = 0, PK_WO = 1, PK_GU = 2, PK_DOWN = 3, PK_MATS = 4, PK_HEAD = 5 };
// Inside a step, activations cross CTAs as flag-in-data pairs {value bits, epoch} written with
// one 8-byte store: a reader polls the pairs it needs until every epoch is the one it expects,
// so no fence or counter round trip sits between a phase and the next.  Epoch of buffer k
// written at (step s, layer l): ep0 + (s * n_layer + l) * PK_EPS + k.
enum : int { PE_QKV = 1, PE_ATT = 2, PE_WO = 3, PE_GU = 4, PE_DOWN = 5, PK_EPS = 8 };

// One GEMV phase: a Q8_0 matrix and its plan.  A CTA owns items [n_items*c/G,
// n_items*(c+1)/G); an item is one row (P = 1) or a gate/up row pair (P = 2); a stage holds
// RI = PK_WARPS / KS items, each warp dots one item over K / KS elements (one 64-element
// unit per lane).
struct PkMat {
    const uint8_t* W;
    long long rb;          // bytes per row
    int K, n_items, P, KS, RI;
    const float* norm_w;   // RMSNorm weights of the prologue (QKV, gate/up, lm_head)
    const float* bias;     // QKV bias (nullptr when the model has none)
};

struct PkArgs {
    const PkMat* mats;     // [PK_MATS * n_layer + 1]
    int n_layer;
    int n_steps;           // token steps in this launch
    int n_prompt;          // steps [0, n_prompt) consume prompt[], later ones the previous argmax
    const int* prompt;
    int first_head;        // first step that runs the lm_head
    int ws_prompt;         // attention window start of prompt steps (the chunk's first position)
    int pos0;              // position of step 0
    int slot;              // sequence slot
    // shared memory plan
    int slot_bytes, n_slots;
    int reg_off;           // activation planes / attention tiles region
    int misc_off;
    int attn_tp;           // attention positions per tile
    int nsf;               // attention position splits per query head (n_head * nsf <= grid)
    float eps;
    // embedding (token_embd, dequant_row)
    const uint8_t* embd;
    int embd_type;
    long long embd_rb;
    int n_vocab;
    // activations crossing CTAs: {value bits, epoch} pairs
    uint2* llq;            // q | k | v [H + 2 KV]
    uint2* lla;            // attention output [H]
    uint2* llx;            // residual stream [D] (after wo, after down)
    uint2* llh;            // SwiGLU output [FF]
    unsigned ep0;          // epoch base of this launch
    float* logits;         // [V]
    int D, H, KVd, FF;
    // fp32 KV cache and RoPE table
    void* kc;
    void* vc;
    long long layer_elems, slot_elems;
    int cap, kv_type;
    const float* cosb;
    const float* sinb;
    int n_head, n_kv, hd;
    float* part;           // [n_head][nsf][hd + 2] split partials
    unsigned* tickets;     // [n_head]
    // step state
    int* tok;              // [1] out: argmax of the last step
    int* pos;              // per slot (written once, at the end)
    int* hist;             // generated ids, hist[s - first_head]
    int hist_cap;
    unsigned long long* keys;  // [n_steps] greedy keys (zero at launch)
    unsigned* cnt;             // [1] step arrivals (zero at launch)
    int* abort_g;              // raised by any CTA that gives up (zero at launch)
    int* err;
    // optional phase trace (nullptr: off): CTA 0 and the last CTA record (globaltimer << 8 |
    // tag) at every phase boundary, trace[w * trace_cap + i], w = 0 / 1; tags in PkTrace
    unsigned long long* trace;
    int trace_cap;
    int* trace_n;              // [2] entries written
};

// trace tags: phase start 10 + kind, activation read 20 + kind, prologue done 30 + kind, rows
// done 40 + kind (kind: PK_QKV / WO / GU / DOWN / HEAD); attention start 50, q / k / v read
// 53, attention done 51
enum : int { PT_START = 10, PT_READ = 20, PT_PRO = 30, PT_LOOP = 40, PT_ATT0 = 50, PT_ATT1 = 51, PT_QKV = 53 };

// Shared-memory plan: ring slots, then the region (activation planes or attention tiles),
// then the control block.
struct PkPlan {
    int slot_bytes, n_slots, reg_off, reg_bytes, misc_off, attn_tp;
    size_t smem;
};
bool pk_plan(int slot_bytes, int max_k, int hd, PkPlan& p);
int pk_attn_fixed_floats(int hd);
cudaError_t pk_launch(const PkArgs& a, int grid, size_t smem, cudaStream_t st);
int pk_occupancy(size_t smem);

}  // namespace tfb
