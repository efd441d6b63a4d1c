// Device-side building blocks shared by every kernel: fp16 decode, mbarrier + bulk-copy
// (TMA) primitives in inline PTX for sm_100a, bounded waits, programmatic dependent launch,
// and the device error word.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace tfb {

// ggml type ids (src/common.hpp:99 of the reference)
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q8_0 = 8, T_Q6_K = 14 };
enum : int { KV_F32 = 0, KV_F16 = 1, KV_BF16 = 2 };

// Error codes written into the device error word (first writer wins).
enum : int { ERR_NONE = 0, ERR_WAIT_FULL = 1, ERR_WAIT_EMPTY = 2, ERR_BAD_TOKEN = 3, ERR_POS = 4, ERR_GRID_SYNC = 5 };

// Spin budget of every bounded wait: polls of mbarrier.try_wait with a nanosleep back-off,
// on the order of a second in total.
constexpr int kWaitPolls = 1 << 20;

__host__ __device__ constexpr int blk_elems(int t) {
    return (t == T_Q4_0 || t == T_Q4_1 || t == T_Q8_0) ? 32 : (t == T_Q6_K ? 256 : 1);
}
__host__ __device__ constexpr int blk_bytes(int t) {
    return t == T_F32 ? 4 : t == T_F16 ? 2 : t == T_Q4_0 ? 18 : t == T_Q4_1 ? 20 : t == T_Q8_0 ? 34 : t == T_Q6_K ? 210 : 0;
}
__host__ __device__ inline long long row_bytes(int t, long long k) {
    return (k / blk_elems(t)) * blk_bytes(t);
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier / bulk copy --------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (after recording `code` in *err) when
// the phase has not completed within the poll budget, or when *abort is raised by another
// warp of the block; the caller then unwinds without touching the stage.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          volatile int* abort) {
    for (int i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort && *abort) return false;
        if (i > (1 << 14)) __nanosleep(256);  // only once the wait is clearly not a stall
    }
    if (err) atomicCAS(err, 0, code);
    if (abort) *abort = 1;
    return false;
}

// Polls of a cross-CTA wait (a grid barrier or a flag another CTA of the same grid sets)
// before it gives up and reports an error.
constexpr int kGridPolls = 1 << 20;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 1-D bulk copy global -> shared (TMA engine), completion signalled on `bar` as tx bytes.
// dst, src and bytes must be multiples of 16.  No cluster multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (TMA engine; a hint, no completion to wait on).
// src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// flag-in-data pairs: {value bits, epoch}, each pair one naturally aligned 8-byte access
__device__ __forceinline__ void st_ll(uint2* p, float v, unsigned ep) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(ep) : "memory");
}
__device__ __forceinline__ uint4 ld_ll2(const uint2* p) {  // two pairs (16-byte aligned)
    uint4 r;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
__device__ __forceinline__ uint2 ld_ll1(const uint2* p) {
    uint2 r;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
    return r;
}

// ---- programmatic dependent launch -----------------------------------------------------
// Every kernel calls pdl_wait() before it reads anything an earlier kernel of the step
// wrote, and calls it unconditionally, so completion is transitive along the chain.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- reductions ------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ unsigned warp_max_u(unsigned v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

// Greedy key: the largest key is the largest logit, ties resolved to the smallest index,
// which is sample_greedy's rule (src/sampler.cpp:8-13: strict '>' keeps the first index).
// NaN logits never win, except at index 0 where the reference returns 0 (every
// comparison against a NaN logits[0] is false).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v);
    uint32_t ord;
    if (v != v) ord = (idx == 0) ? 0xFFFFFFFFu : 0u;
    else ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t key_index(unsigned long long key) {
    return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}

// Padded shared-memory layout of an activation vector: 4 floats of padding after every 64,
// so lanes reading the same element of consecutive 64-element units hit distinct banks.
__device__ __forceinline__ int xpad(int e) { return e + ((e >> 6) << 2); }
__host__ __device__ constexpr int xpad_len(int k) { return k + (k / 64) * 4 + 4; }

}  // namespace tfb
