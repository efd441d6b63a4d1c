// Decode / prefill attention arguments and launchers (attention.cu).
#pragma once

#include "common.cuh"

namespace tfb {

constexpr int AT_THREADS = 128;
constexpr int AT_CHUNK = 64;       // positions per CTA (decode)
constexpr int AT_MAX_SPLIT = 256;  // position splits per (row, kv head): contexts up to 16384
constexpr int AT_MAX_REP = 8;      // query heads per kv head
constexpr int AT_MAX_HD = 128;

struct AttnArgs {
    const float* qkv;       // [M][ld_qkv]: q (n_head*hd) | k (n_kv*hd) | v (n_kv*hd), bias added
    int ld_qkv;
    void* kc;               // this layer's cache base, [slot][n_kv][cap][hd]
    void* vc;
    long long slot_stride;  // elements per slot in one layer
    int cap;
    int kv_type;
    const int* pos;         // per slot: position of the token being decoded
    const int* wstart;      // per slot: first attended position (nullptr: 0)
    const int* slots;       // per row (nullptr: slot 0)
    const float* cosb;      // [cap][hd/2]
    const float* sinb;
    int n_head, n_kv, hd;
    int n_split;
    float* part;            // [M][n_head][n_split][hd + 2]
    unsigned* counters;     // [M][n_kv]
    float* out;             // [M][ld_out]
    int ld_out;
    int fresh;              // 1: decode step (rotate + store + attend over [wstart, pos])
    int n_pos_fixed;        // fresh == 0: attend over n_pos_fixed cached positions, q as given
    int* err;
};

struct PrefillAttnArgs {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    int seq, n_head, n_kv, hd;
};

int attn_pick_split(int cap);
cudaError_t attn_decode_launch(const AttnArgs& a, int M, cudaStream_t st, bool pdl);
cudaError_t attn_prefill_launch(const PrefillAttnArgs& a, cudaStream_t st);

}  // namespace tfb
