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
    int fresh;              // 1: decode step (rotate + store + attend over [wstart, pos]);
                            // 2: prefill chunk of one sequence after tf_rope_store_kernel: row m
                            //    at pos[slot] + m attends over the cache [wstart, pos] as given
    int n_pos_fixed;        // fresh == 0: attend over n_pos_fixed cached positions, q as given
    int* err;
    long long n_rows;       // hd-element rows addressable from kc / vc (0: n_kv * cap, one slot)
};

struct PrefillAttnArgs {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    int seq, n_head, n_kv, hd;
};

// ---- device helpers shared by the attention kernels ----
__device__ __forceinline__ float kv_load(const void* base, long long idx, int t) {
    if (t == KV_F32) return reinterpret_cast<const float*>(base)[idx];
    if (t == KV_F16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
}
__device__ __forceinline__ float kv_round(float v, int t) {
    if (t == KV_F32) return v;
    if (t == KV_F16) return __half2float(__float2half_rn(v));
    return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ void kv_store(void* base, long long idx, int t, float v) {
    if (t == KV_F32) reinterpret_cast<float*>(base)[idx] = v;
    else if (t == KV_F16) reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
}

// NeoX rotate-half with the reference's contraction (src/attention.cpp:31-41 built by g++:
// x0*c - x1*s -> fma(x0, c, -(x1*s)); x0*s + x1*c -> fma(x0, s, x1*c)).
__device__ __forceinline__ void rope_pair(float& a, float& b, float c, float s) {
    const float x0 = a, x1 = b;
    a = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
    b = __fmaf_rn(x0, s, __fmul_rn(x1, c));
}

// Loads `n` consecutive cache elements starting at element `e0` into dst[] as floats, all
// loads in flight before the stores (one memory round trip), 16-byte vectors.
template <int UNR = 4>
__device__ __forceinline__ void load_tile(float* dst, int dst_stride, int hd, const void* base, long long e0, int np,
                                          int kv_type, int nth) {
    const int tid = threadIdx.x;
    const int per_vec = kv_type == KV_F32 ? 4 : 8;      // elements per 16-byte vector
    const int nvec = np * hd / per_vec;
    for (int v0 = tid; v0 < nvec; v0 += nth * UNR) {  // UNR 16-byte loads in flight per thread
        uint4 r[UNR];
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
            const int v = v0 + u * nth;
            if (v < nvec) r[u] = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + (e0 * (kv_type == KV_F32 ? 4 : 2)))[v];
        }
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
            const int v = v0 + u * nth;
            if (v >= nvec) continue;
            const int e = v * per_vec;
            const int p = e / hd, d = e % hd;
            float* o = dst + (size_t)p * dst_stride + d;
            if (kv_type == KV_F32) {
                const float4 f = *reinterpret_cast<const float4*>(&r[u]);
                o[0] = f.x; o[1] = f.y; o[2] = f.z; o[3] = f.w;
            } else {
                const uint32_t w4[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t lo = w4[j] & 0xFFFFu, hi = w4[j] >> 16;
                    if (kv_type == KV_F16) {
                        o[2 * j] = __half2float(__ushort_as_half((unsigned short)lo));
                        o[2 * j + 1] = __half2float(__ushort_as_half((unsigned short)hi));
                    } else {
                        o[2 * j] = __uint_as_float(lo << 16);
                        o[2 * j + 1] = __uint_as_float(hi << 16);
                    }
                }
            }
        }
    }
}

int attn_pick_split(int cap);
cudaError_t attn_decode_launch(const AttnArgs& a, int M, cudaStream_t st, bool pdl);
cudaError_t attn_prefill_launch(const PrefillAttnArgs& a, cudaStream_t st);
cudaError_t rope_store_launch(const AttnArgs& a, int M, cudaStream_t st);

}  // namespace tfb
