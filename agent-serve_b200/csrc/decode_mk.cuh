// Persistent decode megakernel (batch 1): one cooperative launch runs whole decode steps
// (or a prefill followed by greedy generation) with grid barriers between phases.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace tfb {

constexpr int MK_WARPS = 8;                       // consumer warps per CTA (2 rows each per stage)
constexpr int MK_STAGE_BUDGET = 40 * 1024;        // target weight bytes per ring slot
constexpr int MK_THREADS = MK_WARPS * 32;         // thread 0 also drives the weight stream
constexpr int MK_MAX_SLOTS = 16;                  // ring slots (weight stages) per CTA
constexpr int MK_SMEM_LIMIT = 218 * 1024;         // dynamic shared memory per CTA
constexpr int MK_MAX_TILE = 64;                   // attention positions per tile
constexpr int MK_NW = 2;                          // float4 RMSNorm weights prefetched per thread
constexpr int AT_MAX_REP_MK = 8;                  // query heads per kv head
constexpr int AT_MAX_HD_MK = 128;

enum : int { PH_GEMV = 0, PH_ATTN = 1 };

// One phase of a decode step.  GEMV phases stream weights; the attention phase does not.
struct MkPhase {
    int kind;
    int layer;           // PH_ATTN: layer whose cache is used
    // GEMV: weight block and plan (as GemvArgs)
    const uint8_t* W;
    long long rb;
    int wtype, K, n_items, P, KS, fast;
    int ri;              // items per ring stage: (MK_WARPS / KS) * (2 / P)
    int reg;             // Q8_0 with 2048-element segments: activations held in registers
    int pro;             // PRO_COPY / PRO_RMSNORM / PRO_EMBED_RMSNORM
    const float* x;      // input activation (global), or the residual for RMSNorm prologues
    const float* norm_w;
    int epi;             // EPI_STORE / EPI_RESID / EPI_SWIGLU / EPI_ARGMAX
    float* y;
    const float* bias;
    float* resid;
};

struct MkArgs {
    const MkPhase* ph;   // phases of one step: the last one is the lm_head
    int n_ph;
    int n_steps;         // steps in this launch
    int n_prompt;        // the first n_prompt steps consume prompt[], the rest their argmax
    const int* prompt;
    int first_head;      // first step that runs the lm_head (n_prompt - 1 for prefill+gen)
    int ws_prompt;       // attention window start during prompt steps (chunk start)
    int slot;            // sequence slot
    int slot_bytes, n_slots;
    int xfloats;         // floats of the activation region (>= xpad_len of every K)
    float eps;
    // embedding
    const uint8_t* embd;
    int embd_type;
    long long embd_rb;
    int n_vocab;
    float* x_resid;      // residual stream [D]
    int D;
    // attention
    void* kc;
    void* vc;
    long long layer_elems, slot_elems;
    int cap, kv_type;
    const float* cosb;
    const float* sinb;
    int n_head, n_kv, hd;
    const float* qkv;
    float* attn_out;
    // state
    int* tok;            // [1] next input token (out: argmax of the last step)
    int* pos;            // per slot
    int* hist;           // generated ids (argmax of each head step)
    int hist_cap;
    unsigned long long* keys;  // [2] greedy keys, by step parity
    unsigned* bar;       // [0] phase arrivals, [1] exits
    int* err;
};

cudaError_t mk_launch(const MkArgs& a, int grid, cudaStream_t st);
size_t mk_smem_bytes(const MkArgs& a);
int mk_occupancy(size_t smem);

// positions per attention tile that fit the activation region
__host__ __device__ inline int mk_attn_tile(int hd, int xfloats) {
    int t = xfloats / (2 * hd + 1);
    if (t > MK_MAX_TILE) t = MK_MAX_TILE;
    return t < 1 ? 1 : t;
}

}  // namespace tfb
