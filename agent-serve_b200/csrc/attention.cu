// Decode attention with fused RoPE + KV-cache store, split over positions (flash-decode),
// and causal prefill attention.
//
// Replaces, per layer of Model::layer_decode (src/model.cpp:125-129): apply_rope on q and k
// (src/attention.cpp:31-47), KVCache::store (src/kvcache.cpp:31-36) and attn_decode
// (src/attention.cpp:55-80); and attn_prefill (src/attention.cpp:82-111).
//
// Cache layout (HBM): per layer [slot][kv_head][cap][head_dim] (head-major: each head's
// positions are one contiguous slab, the reference's KVLayout::HeadMajor) in fp32, fp16 or
// bf16.  One CTA handles (kv head, position split, activation row): it rotates the n_rep
// query heads of its group and the new key with the host-computed cos/sin table (the
// reference's float cos/sin of pos*freq, so the rotation itself is bit-identical: the
// products are contracted exactly as the reference's g++ build contracts them), split 0
// stores the new k/v, then it forms scores scale*dot(q,k), a max-subtracted exp partial
// and the V-weighted sum over its positions.  The last CTA of a (row, kv head) combines the
// split partials (max, sum, acc) into the normalised output.  The new position's k/v are
// taken from shared memory, never re-read from the cache slot being written.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include <atomic>

#include "attention.cuh"

namespace tfb {

// Shared memory of one CTA: the K tile (row stride hd+1, so threads reading consecutive
// positions hit distinct banks) and the V tile of its <= AT_CHUNK positions, in fp32.
static inline size_t attn_smem_bytes(int hd) { return (size_t)AT_CHUNK * (2 * hd + 1) * sizeof(float); }

// The last CTA of (row m, kv head kvh) to finish combines the nsp split partials
// (max, sum, weighted V) into the normalised output; the others return.  cw: [AT_MAX_REP]
// [AT_MAX_SPLIT] and cden: [AT_MAX_REP] shared scratch; nth threads.
__device__ __forceinline__ void attn_combine(const AttnArgs& a, int m, int kvh, int nsp, float* cwp, float* cden, int nth) {
    __shared__ int last_s;
    const int tid = threadIdx.x, hd = a.hd, n_rep = a.n_head / a.n_kv;
    float (*cw)[AT_MAX_SPLIT] = reinterpret_cast<float (*)[AT_MAX_SPLIT]>(cwp);
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned t = atomicAdd(&a.counters[(size_t)m * a.n_kv + kvh], 1u);
        last_s = (t == (unsigned)nsp - 1);
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    const float* pbase = a.part + ((size_t)m * a.n_head + (size_t)kvh * n_rep) * a.n_split * (hd + 2);
    // with few splits, one round of loads from L2: every split's maximum and sum (shared
    // memory) and this thread's partial vectors (registers); the arithmetic below runs in the
    // same order either way
    constexpr int PO = 4, PS = 4;  // outputs per thread, splits
    __shared__ float csum[AT_MAX_REP][PS];
    const bool pre = nsp <= PS && n_rep * hd <= PO * nth;
    float pv[PO][PS];
    if (pre) {
#pragma unroll
        for (int o = 0; o < PO; ++o) {
            const int i = tid + o * nth;
            if (i < n_rep * hd) {
                const float* pb = pbase + (size_t)(i / hd) * a.n_split * (hd + 2) + 2 + i % hd;
#pragma unroll
                for (int s = 0; s < PS; ++s)
                    if (s < nsp) pv[o][s] = __ldcg(pb + (size_t)s * (hd + 2));
            }
        }
    }
    for (int i = tid; i < n_rep * nsp; i += nth) {
        const int h = i / nsp, s = i % nsp;
        const float* pp = pbase + ((size_t)h * a.n_split + s) * (hd + 2);
        cw[h][s] = __ldcg(pp);
        if (pre) csum[h][s] = __ldcg(pp + 1);
    }
    __syncthreads();
    if (tid < n_rep) {
        float M = -INFINITY;
        for (int s = 0; s < nsp; ++s) M = fmaxf(M, cw[tid][s]);
        float den = 0.f;
        for (int s = 0; s < nsp; ++s) {
            const float w = expf(cw[tid][s] - M);
            den = fmaf(w, pre ? csum[tid][s] : __ldcg(pbase + ((size_t)tid * a.n_split + s) * (hd + 2) + 1), den);
            cw[tid][s] = w;
        }
        cden[tid] = den;
    }
    __syncthreads();
    if (pre) {
#pragma unroll
        for (int o = 0; o < PO; ++o) {
            const int i = tid + o * nth;
            if (i < n_rep * hd) {
                const int h = i / hd, d = i % hd;
                float num0 = 0.f, num1 = 0.f;
#pragma unroll
                for (int s = 0; s < PS; s += 2) {  // the pairs, then the odd last split, as below
                    if (s + 1 < nsp) {
                        num0 = fmaf(cw[h][s], pv[o][s], num0);
                        num1 = fmaf(cw[h][s + 1], pv[o][s + 1], num1);
                    } else if (s < nsp) {
                        num0 = fmaf(cw[h][s], pv[o][s], num0);
                    }
                }
                a.out[(size_t)m * a.ld_out + (size_t)(kvh * n_rep + h) * hd + d] = (num0 + num1) / cden[h];
            }
        }
        if (tid == 0) a.counters[(size_t)m * a.n_kv + kvh] = 0u;
        return;
    }
    for (int i = tid; i < n_rep * hd; i += nth) {
        const int h = i / hd, d = i % hd;
        const float* pb = pbase + (size_t)h * a.n_split * (hd + 2) + 2 + d;
        float num0 = 0.f, num1 = 0.f;
        int s = 0;
        for (; s + 1 < nsp; s += 2) {
            num0 = fmaf(cw[h][s], __ldcg(pb + (size_t)s * (hd + 2)), num0);
            num1 = fmaf(cw[h][s + 1], __ldcg(pb + (size_t)(s + 1) * (hd + 2)), num1);
        }
        if (s < nsp) num0 = fmaf(cw[h][s], __ldcg(pb + (size_t)s * (hd + 2)), num0);
        a.out[(size_t)m * a.ld_out + (size_t)(kvh * n_rep + h) * hd + d] = (num0 + num1) / cden[h];
    }
    if (tid == 0) a.counters[(size_t)m * a.n_kv + kvh] = 0u;
}

__global__ void __launch_bounds__(AT_THREADS) tf_attn_decode_kernel(const AttnArgs a) {
    extern __shared__ float tile[];
    __shared__ float qs[AT_MAX_REP][AT_MAX_HD];
    __shared__ float kn[AT_MAX_HD], vn[AT_MAX_HD];
    __shared__ float sc[AT_MAX_REP][AT_CHUNK];
    __shared__ float mx_s[AT_MAX_REP], l_s[AT_MAX_REP];
    __shared__ float cw[AT_MAX_REP][AT_MAX_SPLIT];
    __shared__ float cden[AT_MAX_REP];
    __shared__ __align__(8) uint64_t kvbar;

    pdl_trigger();
    pdl_wait();
    const int kvh = blockIdx.x, split = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = a.hd, d2 = hd / 2, n_rep = a.n_head / a.n_kv;
    const int slot = a.slots ? a.slots[m] : 0;
    // fresh 2 (prefill chunk of one sequence): row m is the chunk's m-th position
    const int pos = a.fresh == 2 ? a.pos[slot] + m : (a.fresh ? a.pos[slot] : a.n_pos_fixed - 1);
    if (a.fresh && (pos < 0 || pos >= a.cap)) {
        if (tid == 0 && split == 0) atomicCAS(a.err, 0, ERR_POS);
        return;
    }
    const int n_pos = pos + 1;
    // positions [ws, n_pos); ws > 0 only inside a prefill chunk, whose attention sees the
    // chunk alone (attn_prefill, src/attention.cpp:82-111)
    const int ws = (a.fresh && a.wstart) ? min(max(a.wstart[slot], 0), pos) : 0;
    const int n_att = n_pos - ws;
    const int nsp = min((int)gridDim.y, (n_att + AT_CHUNK - 1) / AT_CHUNK);  // active splits
    if (split >= nsp) return;
    const int chunk = (n_att + nsp - 1) / nsp;
    const int p0 = ws + split * chunk;
    const int p1 = min(n_pos, p0 + chunk);
    const int np = max(0, p1 - p0);
    // fp32 caches: K and V rows of the split arrive by two 1-D bulk copies (TMA), rows
    // unpadded (the score loop rotates its start per position, so the rows of one warp still
    // meet distinct banks); fp16 / bf16 caches are widened by the threads (K rows padded)
    const bool bulk = a.kv_type == KV_F32;
    const int kst = bulk ? hd : hd + 1;
    float* ks = tile;                                  // [AT_CHUNK][kst]
    float* vs = tile + (size_t)AT_CHUNK * kst;         // [AT_CHUNK][hd]

    const float* row = a.qkv + (size_t)m * a.ld_qkv;
    const float* q = row + (size_t)kvh * n_rep * hd;
    const size_t cache_off = (size_t)slot * a.slot_stride + (size_t)kvh * a.cap * hd;

    // 1) cached K/V of this split, query heads of the group, new k/v: independent loads
    const int np_cached = (a.fresh == 1 && p1 == n_pos) ? np - 1 : np;  // the new position is not read
    if (bulk) {
        if (tid == 0) {
            mbar_init(&kvbar, 1);
            mbar_fence_init();
            const uint32_t bytes = (uint32_t)np_cached * hd * 4;
            mbar_expect_tx(&kvbar, 2 * bytes);
            if (bytes) {
                const size_t e0 = cache_off + (size_t)p0 * hd;
                bulk_g2s(ks, static_cast<const float*>(a.kc) + e0, bytes, &kvbar);
                bulk_g2s(vs, static_cast<const float*>(a.vc) + e0, bytes, &kvbar);
            }
        }
    } else {
        load_tile<8>(ks, kst, hd, a.kc, (long long)(cache_off + (size_t)p0 * hd), np_cached, a.kv_type, AT_THREADS);
        load_tile<8>(vs, hd, hd, a.vc, (long long)(cache_off + (size_t)p0 * hd), np_cached, a.kv_type, AT_THREADS);
    }
    for (int i = tid; i < n_rep * hd; i += AT_THREADS) qs[i / hd][i % hd] = q[i];
    if (a.fresh == 1)
        for (int i = tid; i < hd; i += AT_THREADS) {
            kn[i] = row[(size_t)a.n_head * hd + (size_t)kvh * hd + i];
            vn[i] = row[(size_t)(a.n_head + a.n_kv) * hd + (size_t)kvh * hd + i];
        }
    __syncthreads();
    if (bulk) mbar_wait(&kvbar, 0, a.err, ERR_WAIT_FULL, nullptr);

    // 2) RoPE (fresh): the host table holds the reference's float cos/sin of pos*freq
    if (a.fresh == 1) {
        const float* cp = a.cosb + (size_t)pos * d2;
        const float* sp = a.sinb + (size_t)pos * d2;
        for (int i = tid; i < (n_rep + 1) * d2; i += AT_THREADS) {
            const int h = i / d2, j = i % d2;
            if (h < n_rep) rope_pair(qs[h][j], qs[h][j + d2], cp[j], sp[j]);
            else rope_pair(kn[j], kn[j + d2], cp[j], sp[j]);
        }
        __syncthreads();
        if (split == 0)
            for (int i = tid; i < hd; i += AT_THREADS) {
                kv_store(a.kc, (long long)(cache_off + (size_t)pos * hd + i), a.kv_type, kn[i]);
                kv_store(a.vc, (long long)(cache_off + (size_t)pos * hd + i), a.kv_type, vn[i]);
            }
        if (p1 == n_pos)
            for (int i = tid; i < hd; i += AT_THREADS) {
                // the new key/value enter at the stored precision, as later steps read them
                ks[(size_t)(np - 1) * kst + i] = kv_round(kn[i], a.kv_type);
                vs[(size_t)(np - 1) * hd + i] = kv_round(vn[i], a.kv_type);
            }
        __syncthreads();
    }

    // 3) scores: thread per (head, position), scale * dot(q, k) (attn_decode, src/attention.cpp:63-64)
    const float scale = 1.0f / sqrtf((float)hd);
    for (int i = tid; i < n_rep * np; i += AT_THREADS) {
        const int h = i / np, p = i % np;
        const float* kp = ks + (size_t)p * kst;
        const int rot = p % hd;  // start of this position's walk over the dims
        float s0 = 0.f, s1 = 0.f;
        for (int d = 0; d < hd; d += 2) {
            int e0 = d + rot, e1 = d + 1 + rot;
            e0 -= e0 >= hd ? hd : 0;
            e1 -= e1 >= hd ? hd : 0;
            s0 = fmaf(qs[h][e0], kp[e0], s0);
            s1 = fmaf(qs[h][e1], kp[e1], s1);
        }
        sc[h][p] = scale * (s0 + s1);
    }
    __syncthreads();
    // 4) max-subtracted exponentials per head (softmax, src/layers.cpp:25-35)
    for (int h = warp; h < n_rep; h += AT_THREADS / 32) {
        float mx = -INFINITY;
        for (int i = lane; i < np; i += 32) mx = fmaxf(mx, sc[h][i]);
        mx = warp_max(mx);
        float l = 0.f;
        for (int i = lane; i < np; i += 32) {
            const float e = expf(sc[h][i] - mx);
            sc[h][i] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            mx_s[h] = mx;
            l_s[h] = l;
        }
    }
    __syncthreads();
    // 5) weighted V: thread per (head, dim)
    for (int i = tid; i < n_rep * hd; i += AT_THREADS) {
        const int h = i / hd, d = i % hd;
        float acc0 = 0.f, acc1 = 0.f;
        int p = 0;
        for (; p + 1 < np; p += 2) {
            acc0 = fmaf(sc[h][p], vs[(size_t)p * hd + d], acc0);
            acc1 = fmaf(sc[h][p + 1], vs[(size_t)(p + 1) * hd + d], acc1);
        }
        if (p < np) acc0 = fmaf(sc[h][p], vs[(size_t)p * hd + d], acc0);
        const float acc = acc0 + acc1;
        const int head = kvh * n_rep + h;
        if (nsp == 1) {
            a.out[(size_t)m * a.ld_out + (size_t)head * hd + d] = acc / l_s[h];
        } else {
            float* pp = a.part + (((size_t)m * a.n_head + head) * a.n_split + split) * (hd + 2);
            pp[2 + d] = acc;
            if (d == 0) {
                pp[0] = mx_s[h];
                pp[1] = l_s[h];
            }
        }
    }
    if (nsp == 1) return;

    attn_combine(a, m, kvh, nsp, &cw[0][0], cden, AT_THREADS);
}

// ---- streaming decode attention (fp32 caches, many rows) -------------------------------------
// One CTA per (row, kv head, position split) walks its positions in tiles of AS_TILE held in
// a ring of AS_NB shared-memory buffers filled by the TMA engine: the K rows as hd/32 boxes of
// 32 positions x 32 floats through a 2-D tensor map with the 128-byte swizzle (16-byte chunk c
// of row r stored at chunk c ^ (r % 8) of its 128-byte line), the V rows by one 1-D bulk copy.
// Per tile, with the whole group of query heads of the kv head (GQA) sharing the tile:
//   scores   lane = position, warp = a slice of hd/8 dims: float4 K reads at the swizzled
//            chunk (the 8 lanes of a quarter-warp meet 8 distinct chunks: no bank conflicts),
//            q read as warp-wide broadcasts, the 8 slices' partial dots summed in a fixed
//            order through shared memory;
//   softmax  warp = query head, lane = position: running max / sum (attn_decode's softmax,
//            src/attention.cpp:63-72, as an online softmax over tiles);
//   P.V      warp = positions p = warp (mod 8), lane = 4 dims, every head of the group held
//            in registers; the 8 warps' sums meet once per split at the end.
// Two CTA barriers per tile; the buffer of tile t - 1 is refilled with tile t + 2 after the
// first one.  Splits of one row combine through attn_combine.
constexpr int AS_THREADS = 256;
constexpr int AS_TILE = 32;
constexpr int AS_NB = 3;
static inline size_t attn_stream_smem_bytes(int hd) {
    // + 1 KB: the swizzled K boxes start on 1024-byte boundaries
    const size_t tiles = (size_t)AS_NB * AS_TILE * 2 * hd * sizeof(float) + 1024;
    const size_t fin = (size_t)(AS_THREADS / 32) * AT_MAX_REP * hd * sizeof(float);  // final sums
    const size_t comb = (size_t)(AT_MAX_REP * AT_MAX_SPLIT + AT_MAX_SPLIT) * sizeof(float);
    size_t m = tiles > fin ? tiles : fin;
    return m > comb ? m : comb;
}

// byte offset of element d of position r in a tile of swizzled K boxes (box d / 32, line r,
// chunk (d % 32) / 4 at chunk ^ (r % 8))
__device__ __forceinline__ uint32_t as_koff(int r, int d) {
    return (uint32_t)((d >> 5) * (AS_TILE * 128) + r * 128 + ((((d >> 2) & 7) ^ (r & 7)) << 4) + (d & 3) * 4);
}

template <int R>  // query heads per kv head
__global__ void __launch_bounds__(AS_THREADS, 2) tf_attn_stream_kernel(const AttnArgs a,
                                                                        const __grid_constant__ CUtensorMap kmap) {
    extern __shared__ __align__(16) float kvt_raw[];
    // the swizzled K boxes need 1024-byte aligned buffers
    float* kvt = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(kvt_raw) +
                                          ((1024u - (smem_u32(kvt_raw) & 1023u)) & 1023u));
    __shared__ __align__(16) float qs[R][AT_MAX_HD];
    __shared__ float red[AS_THREADS / 32][R][AS_TILE];  // partial scores per dim slice
    __shared__ __align__(16) float ep[AS_TILE][8];       // exp(score - max), [position][head]
    __shared__ float kn[AT_MAX_HD], vn[AT_MAX_HD];
    __shared__ __align__(16) float al_s[8];
    __shared__ float mx_s[R], l_s[R];
    __shared__ __align__(8) uint64_t full[AS_NB];

    const int kvh = blockIdx.x, split = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // set-up that depends on no earlier kernel
    if (tid == 0) {
        for (int b = 0; b < AS_NB; ++b) mbar_init(&full[b], 1);
        mbar_fence_init();
    }
    if (tid < R) {
        mx_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    if (tid < 8) al_s[tid] = 0.f;
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    const int hd = a.hd, d2 = hd / 2, cpw = hd / 32;
    const int slot = a.slots ? a.slots[m] : 0;
    const int pos = a.fresh == 2 ? a.pos[slot] + m : (a.fresh ? a.pos[slot] : a.n_pos_fixed - 1);
    if (a.fresh && (pos < 0 || pos >= a.cap)) {
        if (tid == 0 && split == 0) atomicCAS(a.err, 0, ERR_POS);
        return;
    }
    const int n_pos = pos + 1;
    const int ws = (a.fresh && a.wstart) ? min(max(a.wstart[slot], 0), pos) : 0;
    const int n_att = n_pos - ws;
    const int nsp = min((int)gridDim.y, (n_att + 4 * AS_TILE - 1) / (4 * AS_TILE));  // >= 4 tiles a split
    if (split >= nsp) return;
    const int span = (n_att + nsp - 1) / nsp;
    const int p0 = ws + split * span, p1 = min(n_pos, p0 + span);
    const int n_tiles = (p1 - p0 + AS_TILE - 1) / AS_TILE;
    const float* row = a.qkv + (size_t)m * a.ld_qkv;
    const size_t cache_off = (size_t)slot * a.slot_stride + (size_t)kvh * a.cap * hd;
    const float* vc = static_cast<const float*>(a.vc) + cache_off;
    const int krow0 = (int)(cache_off / hd);                // the pair's first row in the K tensor map
    const bool fresh_last = a.fresh == 1 && p1 == n_pos;  // this split holds the new position
    float* kbuf = kvt;                                     // [AS_NB][hd / 32 boxes][AS_TILE][32], swizzled
    float* vbuf = kvt + (size_t)AS_NB * AS_TILE * hd;      // [AS_NB][AS_TILE][hd]

    // tile t into buffer t % AS_NB, issued by lane 0 of the last warp: the K boxes always carry
    // 32 positions (rows past the cache read as zeros, rows past the split are not used), the
    // V copy the tile's cached rows
    constexpr int IW = AS_THREADS / 32 - 1;
    auto issue = [&](int t) {
        if (lane != 0) return;
        const int b = t % AS_NB, q0 = p0 + t * AS_TILE, qn = min(AS_TILE, p1 - q0);
        const int qc = (fresh_last && q0 + qn == n_pos) ? qn - 1 : qn;  // cached rows of the tile
        mbar_expect_tx(&full[b], (uint32_t)(AS_TILE * hd * 4 + qc * hd * 4));
        uint8_t* kb = reinterpret_cast<uint8_t*>(kbuf + (size_t)b * AS_TILE * hd);
        for (int bx = 0; bx < cpw; ++bx)
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                    smem_u32(kb + bx * AS_TILE * 128)),
                "l"(reinterpret_cast<uint64_t>(&kmap)), "r"(32 * bx), "r"(krow0 + q0), "r"(smem_u32(&full[b]))
                : "memory");
        if (qc) bulk_g2s(vbuf + (size_t)b * AS_TILE * hd, vc + (size_t)q0 * hd, (uint32_t)(qc * hd * 4), &full[b]);
    };
    if (warp == IW) {
        issue(0);
        if (n_tiles > 1) issue(1);
    }
    // the group's query heads and the new key, rotated for a decode step (q, k, cos, sin in one
    // round of loads), and the new value
    {
        const float* cp = a.cosb + (size_t)pos * d2;
        const float* sp = a.sinb + (size_t)pos * d2;
        for (int i = tid; i < (R + 1) * d2; i += AS_THREADS) {
            const int h = i / d2, j = i % d2;
            const float* src = h < R ? row + (size_t)(kvh * R + h) * hd : row + (size_t)a.n_head * hd + (size_t)kvh * hd;
            float x0 = src[j], x1 = src[j + d2];
            if (a.fresh == 1) rope_pair(x0, x1, cp[j], sp[j]);
            if (h < R) {
                qs[h][j] = x0;
                qs[h][j + d2] = x1;
            } else {
                kn[j] = x0;
                kn[j + d2] = x1;
            }
        }
        if (a.fresh == 1)
            for (int i = tid; i < hd; i += AS_THREADS) vn[i] = row[(size_t)(a.n_head + a.n_kv) * hd + (size_t)kvh * hd + i];
    }
    __syncthreads();
    if (a.fresh == 1 && split == 0)
        for (int i = tid; i < hd; i += AS_THREADS) {
            kv_store(a.kc, (long long)(cache_off + (size_t)pos * hd + i), a.kv_type, kn[i]);
            kv_store(a.vc, (long long)(cache_off + (size_t)pos * hd + i), a.kv_type, vn[i]);
        }
    const float scale = 1.0f / sqrtf((float)hd);
    // P.V accumulators: head pairs (2hp, 2hp + 1) packed per dim, RP pairs x 4 dims
    constexpr int RP = (R + 1) / 2;
    float2 acc[RP][4];
#pragma unroll
    for (int h = 0; h < RP; ++h) acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = make_float2(0.f, 0.f);
    const bool pv_lane = lane < hd / 4;
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
        const int b = t % AS_NB, q0 = p0 + t * AS_TILE, qn = min(AS_TILE, p1 - q0);
        uint8_t* ks = reinterpret_cast<uint8_t*>(kbuf + (size_t)b * AS_TILE * hd);
        float* vs = vbuf + (size_t)b * AS_TILE * hd;
        if (!mbar_wait(&full[b], (t / AS_NB) & 1, a.err, ERR_WAIT_FULL, nullptr)) ok = false;
        if (fresh_last && q0 + qn == n_pos) {  // uniform: the new key / value enter the tile
            for (int i = tid; i < hd; i += AS_THREADS) {
                *reinterpret_cast<float*>(ks + as_koff(qn - 1, i)) = kn[i];  // fp32 cache: stored exactly
                vs[(size_t)(qn - 1) * hd + i] = vn[i];
            }
            __syncthreads();
        }
        {   // partial scores of this warp's dim slice (attn_decode, src/attention.cpp:63-64)
            // packed fp32 pairs (even, odd dims), summed at the end
            float2 sp[R];
#pragma unroll
            for (int h = 0; h < R; ++h) sp[h] = make_float2(0.f, 0.f);
            if (lane < qn) {
                for (int c = 0; c < cpw; ++c) {
                    const float4 k4 = *reinterpret_cast<const float4*>(ks + as_koff(lane, 4 * (warp * cpw + c)));
                    const float2 k01 = make_float2(k4.x, k4.y), k23 = make_float2(k4.z, k4.w);
#pragma unroll
                    for (int h = 0; h < R; ++h) {
                        const float4 q4 = reinterpret_cast<const float4*>(qs[h])[warp * cpw + c];
                        sp[h] = __ffma2_rn(make_float2(q4.x, q4.y), k01, sp[h]);
                        sp[h] = __ffma2_rn(make_float2(q4.z, q4.w), k23, sp[h]);
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < R; ++h) red[warp][h][lane] = sp[h].x + sp[h].y;
        }
        __syncthreads();
        // every thread has finished tile t - 1's P.V: its buffer takes tile t + 2
        if (warp == IW && t + 2 < n_tiles) issue(t + 2);
        if (warp < R) {  // running max and sum of head `warp`
            const int h = warp;
            float sv = -INFINITY;
            if (lane < qn) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < AS_THREADS / 32; ++w) v += red[w][h][lane];
                sv = scale * v;
            }
            const float tm = warp_max(sv);
            const float mold = mx_s[h];
            const float mnew = fmaxf(mold, tm);
            const float e = lane < qn ? expf(sv - mnew) : 0.f;
            ep[lane][h] = e;
            const float lt = warp_sum(e);
            if (lane == 0) {
                const float alpha = expf(mold - mnew);  // 0 on the first tile
                al_s[h] = alpha;
                l_s[h] = fmaf(l_s[h], alpha, lt);
                mx_s[h] = mnew;
            }
        }
        __syncthreads();
        if (pv_lane) {  // weighted V over positions warp, warp + 8, ...
            const float4 a0 = reinterpret_cast<const float4*>(al_s)[0], a1 = reinterpret_cast<const float4*>(al_s)[1];
            const float2 alp[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w), make_float2(a1.x, a1.y),
                                   make_float2(a1.z, a1.w)};
#pragma unroll
            for (int h = 0; h < RP; ++h) {
                acc[h][0] = __fmul2_rn(acc[h][0], alp[h]);
                acc[h][1] = __fmul2_rn(acc[h][1], alp[h]);
                acc[h][2] = __fmul2_rn(acc[h][2], alp[h]);
                acc[h][3] = __fmul2_rn(acc[h][3], alp[h]);
            }
            for (int p = warp; p < qn; p += AS_THREADS / 32) {
                const float4 v4 = reinterpret_cast<const float4*>(vs + (size_t)p * hd)[lane];
                const float4 e0 = reinterpret_cast<const float4*>(ep[p])[0];
                const float4 e1 = R > 4 ? reinterpret_cast<const float4*>(ep[p])[1] : e0;
                const float2 ep2[4] = {make_float2(e0.x, e0.y), make_float2(e0.z, e0.w), make_float2(e1.x, e1.y),
                                       make_float2(e1.z, e1.w)};
                const float2 vx = make_float2(v4.x, v4.x), vy = make_float2(v4.y, v4.y);
                const float2 vz = make_float2(v4.z, v4.z), vw = make_float2(v4.w, v4.w);
#pragma unroll
                for (int h = 0; h < RP; ++h) {
                    acc[h][0] = __ffma2_rn(ep2[h], vx, acc[h][0]);
                    acc[h][1] = __ffma2_rn(ep2[h], vy, acc[h][1]);
                    acc[h][2] = __ffma2_rn(ep2[h], vz, acc[h][2]);
                    acc[h][3] = __ffma2_rn(ep2[h], vw, acc[h][3]);
                }
            }
        }
    }
    // the 8 warps' P.V sums (tile buffers are free: every issued copy was waited for)
    __syncthreads();
    float* fin = kvt;  // [warp][head][hd]
    if (pv_lane)
#pragma unroll
        for (int h = 0; h < R; ++h) {
            const int hp = h >> 1;
            const bool odd = h & 1;
            reinterpret_cast<float4*>(fin + ((size_t)warp * R + h) * hd)[lane] =
                odd ? make_float4(acc[hp][0].y, acc[hp][1].y, acc[hp][2].y, acc[hp][3].y)
                    : make_float4(acc[hp][0].x, acc[hp][1].x, acc[hp][2].x, acc[hp][3].x);
        }
    __syncthreads();
    if (ok)
        for (int i = tid; i < R * hd; i += AS_THREADS) {
            const int h = i / hd, d = i % hd;
            float o = 0.f;
#pragma unroll
            for (int w = 0; w < AS_THREADS / 32; ++w) o += fin[((size_t)w * R + h) * hd + d];
            const int head = kvh * R + h;
            if (nsp == 1) {
                a.out[(size_t)m * a.ld_out + (size_t)head * hd + d] = o / l_s[h];
            } else {
                float* pp = a.part + (((size_t)m * a.n_head + head) * a.n_split + split) * (hd + 2);
                pp[2 + d] = o;
                if (d == 0) {
                    pp[0] = mx_s[h];
                    pp[1] = l_s[h];
                }
            }
        }
    // a CTA whose tile wait gave up (ERR_WAIT_FULL is recorded) still arrives at its head's
    // counter, so the counter returns to zero; the call's output is then not valid
    if (!ok && nsp == 1) return;
    // the combine's scratch reuses the tile buffers
    if (nsp > 1) {
        __syncthreads();
        attn_combine(a, m, kvh, nsp, kvt, kvt + AT_MAX_REP * AT_MAX_SPLIT, AS_THREADS);
    }
}

// ---- prefill attention (attn_prefill): one CTA per (query row i, head h) -----------------
__global__ void __launch_bounds__(AT_THREADS) tf_attn_prefill_kernel(const PrefillAttnArgs a) {
    extern __shared__ float sbuf[];  // [seq] scores
    __shared__ float qs[AT_MAX_HD];
    __shared__ float red[AT_THREADS / 32];
    __shared__ float stat[2];
    const int i = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = a.hd, n_rep = a.n_head / a.n_kv, hv = h / n_rep;
    const float* qi = a.q + ((size_t)i * a.n_head + h) * hd;
    for (int d = tid; d < hd; d += AT_THREADS) qs[d] = qi[d];
    __syncthreads();
    const float scale = 1.0f / sqrtf((float)hd);
    for (int j = warp; j <= i; j += AT_THREADS / 32) {
        const float* kj = a.k + ((size_t)j * a.n_kv + hv) * hd;
        float s = 0.f;
        for (int d = lane; d < hd; d += 32) s = fmaf(qs[d], kj[d], s);
        s = warp_sum(s);
        if (lane == 0) sbuf[j] = scale * s;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = tid; j <= i; j += AT_THREADS) mx = fmaxf(mx, sbuf[j]);
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float v = red[0];
        for (int w = 1; w < AT_THREADS / 32; ++w) v = fmaxf(v, red[w]);
        stat[0] = v;
    }
    __syncthreads();
    mx = stat[0];
    float l = 0.f;
    for (int j = tid; j <= i; j += AT_THREADS) {
        const float e = expf(sbuf[j] - mx);
        sbuf[j] = e;
        l += e;
    }
    l = warp_sum(l);
    __syncthreads();
    if (lane == 0) red[warp] = l;
    __syncthreads();
    if (tid == 0) {
        float v = 0.f;
        for (int w = 0; w < AT_THREADS / 32; ++w) v += red[w];
        stat[1] = v;
    }
    __syncthreads();
    const float inv = 1.0f / stat[1];
    for (int d = tid; d < hd; d += AT_THREADS) {
        float acc = 0.f;
        for (int j = 0; j <= i; ++j) acc = fmaf(sbuf[j] * inv, a.v[((size_t)j * a.n_kv + hv) * hd + d], acc);
        a.out[((size_t)i * a.n_head + h) * hd + d] = acc;
    }
}

// ---- prefill chunk, first half: RoPE of q (in place) and k, K/V store -------------------------
// One CTA per (row, head), a thread per rotation pair; row m is position pos[slot] + m.  The
// attention of the chunk then runs over the cache alone (fresh == 2), so that every row sees
// the keys of the rows before it (attn_prefill's causal mask, src/attention.cpp:82-111).
__global__ void tf_rope_store_kernel(const AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
    const int hd = a.hd, d2 = hd / 2;
    const int slot = a.slots ? a.slots[m] : 0;
    const int pos = a.pos[slot] + m;
    if (pos < 0 || pos >= a.cap) {
        if (j == 0) atomicCAS(a.err, 0, ERR_POS);
        return;
    }
    float* row = const_cast<float*>(a.qkv) + (size_t)m * a.ld_qkv;
    const float c = a.cosb[(size_t)pos * d2 + j], sn = a.sinb[(size_t)pos * d2 + j];
    if (h < a.n_head) {
        float* q = row + (size_t)h * hd;
        float x0 = q[j], x1 = q[j + d2];
        rope_pair(x0, x1, c, sn);
        q[j] = x0;
        q[j + d2] = x1;
    } else {
        const int kvh = h - a.n_head;
        const float* k = row + (size_t)a.n_head * hd + (size_t)kvh * hd;
        const float* v = row + (size_t)(a.n_head + a.n_kv) * hd + (size_t)kvh * hd;
        float x0 = k[j], x1 = k[j + d2];
        rope_pair(x0, x1, c, sn);
        const size_t off = (size_t)slot * a.slot_stride + (size_t)kvh * a.cap * hd + (size_t)pos * hd;
        kv_store(a.kc, (long long)(off + j), a.kv_type, x0);
        kv_store(a.kc, (long long)(off + j + d2), a.kv_type, x1);
        kv_store(a.vc, (long long)(off + j), a.kv_type, v[j]);
        kv_store(a.vc, (long long)(off + j + d2), a.kv_type, v[j + d2]);
    }
}

// ---- host ------------------------------------------------------------------------------
int attn_pick_split(int cap) {
    const int s = (cap + AT_CHUNK - 1) / AT_CHUNK;
    return s < 1 ? 1 : (s > AT_MAX_SPLIT ? AT_MAX_SPLIT : s);
}

// rows x kv heads that fill the GPU without position splits for the streaming kernel
static int attn_stream_splits(const AttnArgs& a, int M) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // one wave of the two resident CTAs per SM (TFB200_ATTN_WAVES): a CTA's set-up and
    // combine cost a few microseconds, so fewer, longer splits measured faster (cfg4 at 256
    // rows x 512 positions: 9.95 ms per step at one wave, 10.9 at four); the kernel itself
    // keeps at least four tiles per split
    static int waves = -1;
    if (waves < 0) {
        const char* e = getenv("TFB200_ATTN_WAVES");
        waves = e ? atoi(e) : 1;
        if (waves < 1) waves = 1;
    }
    // rounded down: a split count that leaves a partial second wave doubles the kernel's time
    // (cfg4 at 32 rows x 1026 positions: 5 splits = 320 CTAs for 296 slots)
    const int pairs = M * a.n_kv;
    int s = waves * 2 * sms / pairs;
    return s < 1 ? 1 : (s > a.n_split ? a.n_split : s);
}

// The K cache of one layer as a 2-D tensor map: n_rows rows of hd floats, boxes of 32 rows x 32
// floats (128 bytes: the 128-byte swizzle's line), rows past n_rows read as zeros.
static bool attn_k_map(CUtensorMap* m, const AttnArgs& a) {
    static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    static std::atomic<bool> tried{false};
    if (!tried.load()) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        tried.store(true);
    }
    if (!enc || (reinterpret_cast<uintptr_t>(a.kc) & 15)) return false;
    const long long rows = a.n_rows > 0 ? a.n_rows : (long long)a.n_kv * a.cap;
    const cuuint64_t dims[2] = {(cuuint64_t)a.hd, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)a.hd * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)AS_TILE};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.kc, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t attn_decode_launch(const AttnArgs& a, int M, cudaStream_t st, bool pdl) {
    if (a.hd > AT_MAX_HD || a.hd % 8 || a.n_head / a.n_kv > AT_MAX_REP) return cudaErrorInvalidValue;
    alignas(64) CUtensorMap kmap;
    memset(&kmap, 0, sizeof(kmap));
    // many rows: the streaming kernel (fp32 cache, K boxes through the tensor map)
    if (a.kv_type == KV_F32 && M * a.n_kv >= 16 && a.hd % 32 == 0 && attn_k_map(&kmap, a)) {
        static const void* const fns[AT_MAX_REP] = {
            (const void*)tf_attn_stream_kernel<1>, (const void*)tf_attn_stream_kernel<2>, (const void*)tf_attn_stream_kernel<3>,
            (const void*)tf_attn_stream_kernel<4>, (const void*)tf_attn_stream_kernel<5>, (const void*)tf_attn_stream_kernel<6>,
            (const void*)tf_attn_stream_kernel<7>, (const void*)tf_attn_stream_kernel<8>};
        const int R = a.n_head / a.n_kv;
        const void* fn = fns[R - 1];
        // set once per device; setting an attribute twice is harmless, so concurrent first
        // calls only need the flag itself to be race-free
        static std::atomic<bool> sattr[64][AT_MAX_REP] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) dev = 0;
        if (!sattr[dev][R - 1]) {
            cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)attn_stream_smem_bytes(AT_MAX_HD));
            if (e != cudaSuccess) return e;
            // two CTAs per SM need the whole shared-memory carve-out
            e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
            if (e != cudaSuccess) return e;
            sattr[dev][R - 1].store(true);
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(a.n_kv, attn_stream_splits(a, M), M);
        cfg.blockDim = dim3(AS_THREADS);
        cfg.dynamicSmemBytes = attn_stream_smem_bytes(a.hd);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        AttnArgs aa = a;
        void* args[] = {&aa, &kmap};
        return cudaLaunchKernelExC(&cfg, fn, args);
    }
    const int max_pos = a.fresh ? a.cap : a.n_pos_fixed;
    if ((max_pos + a.n_split - 1) / a.n_split > AT_CHUNK || a.n_split > AT_MAX_SPLIT) return cudaErrorInvalidValue;
    const size_t smem = attn_smem_bytes(a.hd);
    static std::atomic<bool> attrs[64] = {};  // set once per device (see sattr above)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attrs[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tf_attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)attn_smem_bytes(AT_MAX_HD));
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(tf_attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        attrs[dev].store(true);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_kv, a.n_split, M);
    cfg.blockDim = dim3(AT_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tf_attn_decode_kernel, a);
}

cudaError_t rope_store_launch(const AttnArgs& a, int M, cudaStream_t st) {
    if (a.hd > AT_MAX_HD || a.hd % 2) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M, a.n_head + a.n_kv);
    cfg.blockDim = dim3(a.hd / 2);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tf_rope_store_kernel, a);
}

cudaError_t attn_prefill_launch(const PrefillAttnArgs& a, cudaStream_t st) {
    if (a.hd > AT_MAX_HD) return cudaErrorInvalidValue;
    const size_t smem = (size_t)a.seq * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(tf_attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    tf_attn_prefill_kernel<<<dim3(a.seq, a.n_head), AT_THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace tfb
