// Q8_0 / Q4_0 GEMM for M >= 16 activation rows (see gemm.cuh).
//
// Default path, tf_gemm_q8_tc_kernel (5th-gen tensor cores): a CTA owns 128 weight rows x NT
// (32, 64, 128 or 256) activation rows, k in stages of 64, in 128-byte swizzled K-major shared
// memory, with its warps in three roles synchronised by mbarriers (no CTA-wide barrier per
// stage).  Sixteen dequantising warps, four threads per weight row, turn 16-weight pieces into
// exact f16 halves Wh, Wl of q*d*2^sw in one of two weight buffers; their quantised words come
// either (WT: K a multiple of 256, tiles up to 128 rows) from a ring of chunks of four stages,
// each one 2-D tensor-map copy of the tile's 128 rows, or from global memory into registers
// four stages ahead.  One warp issues those copies and the bulk copies of the activation halves
// Xh, Xl (prepared once per matmul by tf_xprep_kernel in the operand layout); one thread
// issues tcgen05.mma (kind::f16, fp32 accumulator in TMEM) three times per k step: Wh*Xh,
// Wh*Xl, Wl*Xh, and commits each stage to the barriers that free its buffers.  The epilogue
// reads TMEM, scales back by 2^-(sw+sx[m]) (per-column factors computed once), stages the tile
// in shared memory and, when the k range is split, sums the splits of the tile through
// distributed shared memory of their thread-block cluster in split order;
// then the fused epilogue (bias, residual add, SwiGLU on interleaved gate/up rows, logits +
// greedy argmax keys).

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include "dots.cuh"
#include "gemm.cuh"

namespace tfb {

// byte offset of element (row, k) of a [rows][64] f16 operand tile in the 128-byte swizzled
// K-major layout: 8-row atoms of 1024 B, the 16-byte chunk c of line r stored at chunk c ^ r
__host__ __device__ __forceinline__ uint32_t gm_kint_off(int row, int k) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

// ---- activation preparation ----------------------------------------------------------------
// One CTA per activation row: [embedding lookup ->] [RMSNorm (src/layers.cpp:7-12) ->]
// power-of-two scale to |x| < 2^14 -> f16 halves.
constexpr int XP_THREADS = 256;
constexpr int XP_REG_CHUNKS = 12;  // float4 chunks a thread holds in registers: rows of K <= 12288

// tf_xprep_kernel with the row in registers (rows read from memory, K <= XP_THREADS * 4 *
// XP_REG_CHUNKS; xprep_launch picks it): thread t
// holds float4 chunks t, t + 256, ... of the row, so the RMSNorm's double sum runs in the
// shared-memory path's order (per thread over its chunks, then warps in order) and every output
// bit is the same; two CTA barriers instead of four, and no pass through shared memory.  An
// 8-element chunk of the operand layout is the float4 chunks 2i (even lane) and 2i + 1 (the
// next lane): the even lane stores its Xh 16 bytes, the odd lane its Xl 16 bytes, each with
// the other lane's half exchanged by one shuffle pair.
__global__ void __launch_bounds__(XP_THREADS) tf_xprep_rows_kernel(const XPrepArgs a) {
    __shared__ double redd[XP_THREADS / 32];
    __shared__ float redf[XP_THREADS / 32];
    const int m = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.K, nq = K >> 2;
    // as tf_xprep_kernel: the GEMM may start its set-up now, the reads wait for the writer
    pdl_trigger();
    pdl_wait();
    const float4* xg = reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx);
    float4 v[XP_REG_CHUNKS];
#pragma unroll
    for (int j = 0; j < XP_REG_CHUNKS; ++j) {
        const int c = tid + j * XP_THREADS;
        v[j] = c < nq ? xg[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (a.norm_w) {
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < XP_REG_CHUNKS; ++j) {
            if (tid + j * XP_THREADS < nq) {
                ss = fma((double)v[j].x, (double)v[j].x, ss);
                ss = fma((double)v[j].y, (double)v[j].y, ss);
                ss = fma((double)v[j].z, (double)v[j].z, ss);
                ss = fma((double)v[j].w, (double)v[j].w, ss);
            }
        }
        ss = warp_sum_d(ss);
        if (lane == 0) redd[warp] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < XP_THREADS / 32; ++w) tot += redd[w];
        const float inv = 1.0f / sqrtf((float)(tot / K) + a.eps);
#pragma unroll
        for (int j = 0; j < XP_REG_CHUNKS; ++j) {
            const int c = tid + j * XP_THREADS;
            if (c < nq) {
                const float4 w = reinterpret_cast<const float4*>(a.norm_w)[c];
                v[j].x = __fmul_rn(__fmul_rn(v[j].x, inv), w.x);
                v[j].y = __fmul_rn(__fmul_rn(v[j].y, inv), w.y);
                v[j].z = __fmul_rn(__fmul_rn(v[j].z, inv), w.z);
                v[j].w = __fmul_rn(__fmul_rn(v[j].w, inv), w.w);
            }
        }
    }
    float am = 0.f;
#pragma unroll
    for (int j = 0; j < XP_REG_CHUNKS; ++j)  // chunks past the row are zeros
        am = fmaxf(fmaxf(am, fmaxf(fabsf(v[j].x), fabsf(v[j].y))), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
    am = warp_max(am);
    if (lane == 0) redf[warp] = am;
    __syncthreads();
    am = 0.f;
    for (int w = 0; w < XP_THREADS / 32; ++w) am = fmaxf(am, redf[w]);
    const int be = (int)((__float_as_uint(am) >> 23) & 0xFFu);  // as below
    int sx = 140 - be;
    sx = sx > 100 ? 100 : (sx < -100 ? -100 : sx);
    const float S = ldexpf(1.0f, sx);
    const bool odd = lane & 1;
#pragma unroll
    for (int j = 0; j < XP_REG_CHUNKS; ++j) {
        if (j * XP_THREADS >= nq) break;  // uniform over the CTA
        const int c = tid + j * XP_THREADS;
        const float e[4] = {v[j].x * S, v[j].y * S, v[j].z * S, v[j].w * S};  // exact scaling
        uint32_t hw[2], lw[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const __half h0 = __float2half_rn(e[2 * i]), h1 = __float2half_rn(e[2 * i + 1]);
            const __half l0 = __float2half_rn(e[2 * i] - __half2float(h0));
            const __half l1 = __float2half_rn(e[2 * i + 1] - __half2float(h1));
            hw[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            lw[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        // the even lane takes the odd lane's Xh words, the odd lane the even lane's Xl words
        const uint32_t s0 = __shfl_xor_sync(0xffffffffu, odd ? hw[0] : lw[0], 1);
        const uint32_t s1 = __shfl_xor_sync(0xffffffffu, odd ? hw[1] : lw[1], 1);
        if (c < nq) {
            const int e0 = 4 * (c & ~1);  // first element of the 8-element chunk
            const size_t off = (size_t)(e0 >> 6) * a.mp * (GM_BK * 2) + gm_kint_off(m, e0 & 63);
            if (!odd)
                *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.xh) + off) = make_uint4(hw[0], hw[1], s0, s1);
            else
                *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.xl) + off) = make_uint4(s0, s1, lw[0], lw[1]);
        }
    }
    if (tid == 0) a.sx[m] = sx;
}

__global__ void __launch_bounds__(XP_THREADS) tf_xprep_kernel(const XPrepArgs a) {
    extern __shared__ __align__(16) float xrow[];  // xpad layout
    __shared__ double redd[8];
    __shared__ float redf[8];
    const int m = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nth = blockDim.x;
    const int K = a.K, nq = K >> 2;
    // the GEMM that reads these operands may start its set-up and weight prefetch now; every
    // read below waits for the kernel that wrote the input row
    pdl_trigger();
    pdl_wait();
    if (a.embd) {
        int tok = a.tokens[m];
        if (tok < 0 || tok >= a.n_vocab) {
            if (tid == 0) atomicCAS(a.err, 0, ERR_BAD_TOKEN);
            tok = 0;
        }
        embed_row(xrow, a.embd, a.embd_type, a.embd_rb, K, tok, nth);
        __syncthreads();
        for (int e = tid; e < K; e += nth) a.x_out[(size_t)m * a.ldx + e] = xrow[xpad(e)];
    } else {
        const float4* xg = reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx);
        for (int c = tid; c < nq; c += nth) *reinterpret_cast<float4*>(xrow + xpad(4 * c)) = xg[c];
    }
    __syncthreads();
    if (a.norm_w) {
        double ss = 0.0;
        for (int c = tid; c < nq; c += nth) {
            const float4 v = *reinterpret_cast<const float4*>(xrow + xpad(4 * c));
            ss = fma((double)v.x, (double)v.x, ss);
            ss = fma((double)v.y, (double)v.y, ss);
            ss = fma((double)v.z, (double)v.z, ss);
            ss = fma((double)v.w, (double)v.w, ss);
        }
        ss = warp_sum_d(ss);
        if (lane == 0) redd[warp] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < nth / 32; ++w) tot += redd[w];
        const float inv = 1.0f / sqrtf((float)(tot / K) + a.eps);
        for (int c = tid; c < nq; c += nth) {
            float4* p = reinterpret_cast<float4*>(xrow + xpad(4 * c));
            const float4 w = reinterpret_cast<const float4*>(a.norm_w)[c];
            float4 v = *p;
            v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
            *p = v;
        }
        __syncthreads();
    }
    float am = 0.f;
    for (int e = tid; e < K; e += nth) am = fmaxf(am, fabsf(xrow[xpad(e)]));
    am = warp_max(am);
    if (lane == 0) redf[warp] = am;
    __syncthreads();
    am = 0.f;
    for (int w = 0; w < nth / 32; ++w) am = fmaxf(am, redf[w]);
    // am < 2^(be-126) for a normal am with biased exponent be: 2^sx = 2^(140-be) keeps the
    // scaled row below 2^14; zero / subnormal rows take the largest shift
    const int be = (int)((__float_as_uint(am) >> 23) & 0xFFu);
    int sx = 140 - be;
    sx = sx > 100 ? 100 : (sx < -100 ? -100 : sx);
    const float S = ldexpf(1.0f, sx);
    // 8-element chunks into the GEMM's operand layout (gemm.cuh, XPrepArgs::mp)
    for (int c = tid; c < K / 8; c += nth) {
        const int e0 = 8 * c;
        uint32_t hv[4], lv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float v0 = xrow[xpad(e0 + 2 * i)] * S, v1 = xrow[xpad(e0 + 2 * i + 1)] * S;  // exact scaling
            const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
            const __half l0 = __float2half_rn(v0 - __half2float(h0)), l1 = __float2half_rn(v1 - __half2float(h1));
            hv[i] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            lv[i] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        const size_t off = (size_t)(e0 >> 6) * a.mp * (GM_BK * 2) + gm_kint_off(m, e0 & 63);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.xh) + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.xl) + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
    if (tid == 0) a.sx[m] = sx;
}

// ---- the GEMM ------------------------------------------------------------------------------

constexpr int GM_EPI_LD = GM_BN + 4;         // epilogue tile row stride (floats)

// The weight words a dequantising thread of the tcgen05 kernel needs for weight row r, k-stage
// kc, 16-weight piece jh = 2 * block + half: w[0] holds the block's fp16 scale (word 0 or 8 of
// the stage's 68-byte unit), w[1..5] the five words 4*jh .. 4*jh + 4 (bytes 16*jh .. 16*jh +
// 19), whose bytes 2 * block + 2 .. + 17 are the piece's 16 quants.
// Q4_0 (Q4): the stage's 36-byte unit holds two 18-byte blocks; both halves of block j read
// the five words 4j .. 4j + 4, whose first word carries the block's scale (low half for block
// 0, high half for block 1) and whose bytes 2j + 2 .. + 17 are its 16 quant bytes (weight i
// in the low nibble of byte i, weight 16 + i in the high nibble).
template <bool Q4>
__device__ __forceinline__ void gm_load_w16(uint32_t (&w)[6], const GemmArgs& a, int n, int kc, int jh) {
    if (n < a.N) {
        const uint32_t* p = reinterpret_cast<const uint32_t*>(a.W + (long long)n * a.rb + (long long)kc * (Q4 ? 36 : 68));
        const int w0 = Q4 ? 4 * (jh >> 1) : 4 * jh;
        w[0] = __ldg(p + (Q4 ? w0 : 8 * (jh >> 1)));
#pragma unroll
        for (int i = 0; i < 5; ++i) w[1 + i] = __ldg(p + w0 + i);
    } else {
#pragma unroll
        for (int i = 0; i < 6; ++i) w[i] = 0u;
    }
}


// One 16-weight piece of gm_load_w16's words into the exact f16 split, with packed half2
// arithmetic and no per-element conversion: q is made exact in f16 from its byte (0x6400 |
// (q + 128) is 1024 + q + 128; Q4_0: (0x6400 | nibble) - 1032 is nibble - 8), Wh = q * dh rounds
// the exact product once (dh = d * 2^sw, an f16 value; at most 19 significant bits for Q8_0, 15
// for Q4_0), and Wl = fma(q, dh, -Wh) is the exact remainder.  One instruction stream for every
// lane of a warp (the lanes hold pieces of either block of a stage, and of either nibble half
// for Q4_0): the pieces of block 1 start two bytes later in their five window words, so a
// funnel shift by 16 bits (0 for block 0) aligns both, and the nibble half is a shift by
// 4 * half.  hv / lv: the piece's 16 halves in k order, two per word (even k in the low half).
template <bool Q4>
__device__ __forceinline__ void gm_dequant16_r(const uint32_t (&w)[6], uint32_t blk, uint32_t half, float wscale,
                                               uint32_t (&hv)[8], uint32_t (&lv)[8]) {
    const uint32_t sh = blk << 4;
    const uint32_t dbits = (w[0] >> sh) & 0xFFFFu;
    const __half dsc = __float2half_rn(__half2float(__ushort_as_half((unsigned short)dbits)) * wscale);
    const __half2 d2 = __halves2half2(dsc, dsc);
    const unsigned short kb = Q4 ? 0x6408u : 0x6480u;  // 1032 (nibble - 8) or 1152 (byte ^ 0x80 - 128)
    const __half2 kq = __halves2half2(__ushort_as_half(kb), __ushort_as_half(kb));
    uint32_t q[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) q[i] = __funnelshift_r(w[1 + i], i < 4 ? w[2 + i] : 0u, sh);
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
        const int b = 2 + e;  // the piece's bytes are 2 .. 17 of the aligned window
        const uint32_t wd = Q4 ? ((q[b >> 2] >> (half << 2)) & 0x0F0F0F0Fu) : (q[b >> 2] ^ 0x80808080u);
        const uint32_t sel = (uint32_t)(b & 3) | (4u << 4) | ((uint32_t)((b & 3) + 1) << 8) | (4u << 12);
        const uint32_t qb = __byte_perm(wd, 0x64646464u, sel);
        const __half2 q2 = __hsub2(*reinterpret_cast<const __half2*>(&qb), kq);
        const __half2 hi = __hmul2(q2, d2);
        const __half2 lo = __hfma2(q2, d2, __hneg2(hi));
        hv[e >> 1] = *reinterpret_cast<const uint32_t*>(&hi);
        lv[e >> 1] = *reinterpret_cast<const uint32_t*>(&lo);
    }
}

// eight consecutive 32-bit tensor-memory columns of this thread's lane (the warp's lane quarter)
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// Split-K reduction and the fused epilogue over a CTA tile staged in shared memory as
// tile[m - m0][n - n0] (BMT activation rows x GM_BN weight rows, row stride GM_EPI_LD).
// With split-K (grid.z = ks > 1, every CTA of the grid resident: ks x tiles <= SMs) each split
// publishes its partial tile, waits (bounded) for the other splits of its tile, then sums all
// partials, in split order, for its own 1/ks of the tile's activation rows and applies the
// epilogue to those rows: the reduction is spread over the splits and deterministic.
// ---- thread-block cluster helpers (split-K reduction through distributed shared memory) ----
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float4 ld_cluster_v4(uint32_t local_addr, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(r)
                 : "memory");
    return v;
}

// CLUSTER: the k splits of a tile are one thread-block cluster (grid.z = cluster size = ks), so
// each split reduces its slice of rows by reading the other splits' tiles straight from their
// shared memory; otherwise the splits meet through the global workspace and tile counters.
// Either way the splits are summed in split order (deterministic).
template <int BMT, bool CLUSTER, int NTH>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs& a, float* tile, int m0, int n0, bool ok_in = true) {
    const int tid = threadIdx.x;
    const int rv = min(BMT, a.M - m0);  // valid activation rows of the tile
    int mlo = 0, mhi = rv;
    if (CLUSTER && gridDim.z > 1) {
        const int ks = (int)gridDim.z, z = (int)blockIdx.z;  // cluster rank z holds split z
        cluster_sync_all();  // every split's tile is in its shared memory
        mlo = rv * z / ks;
        mhi = rv * (z + 1) / ks;
        // this CTA's rows of the tile are read by no other split: the sums overwrite them
        for (int i = tid; i < (mhi - mlo) * (GM_BN / 4); i += NTH) {
            const int mm = mlo + i / (GM_BN / 4), n4 = i % (GM_BN / 4);
            float* t = tile + mm * GM_EPI_LD + 4 * n4;
            const uint32_t la = smem_u32(t);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < ks; ++q) {
                const float4 u = ld_cluster_v4(la, q);
                v.x += u.x;
                v.y += u.y;
                v.z += u.z;
                v.w += u.w;
            }
            *reinterpret_cast<float4*>(t) = v;
        }
        cluster_sync_all();  // no split leaves while another still reads its tile
        if (!ok_in) return;  // the error word holds the failure (the barriers were still kept)
    } else if (gridDim.z > 1) {
        __shared__ int ok_s;
        const int ks = (int)gridDim.z, z = (int)blockIdx.z;
        float* wz = a.ws + (size_t)z * a.M * a.N;
        for (int i = tid; i < rv * GM_BN; i += NTH) {
            const int mm = i / GM_BN, nn = i % GM_BN, n = n0 + nn;
            if (n < a.N) wz[(size_t)(m0 + mm) * a.N + n] = tile[mm * GM_EPI_LD + nn];
        }
        __threadfence();
        __syncthreads();
        unsigned* cnt = a.tile_cnt + 2 * (blockIdx.y * gridDim.x + blockIdx.x);
        if (tid == 0) {
            red_release_gpu_add(cnt, 1u);
            int i = 0;
            for (; i < kGridPolls; ++i) {
                if (ld_acquire_gpu(cnt) >= (unsigned)ks) break;
                if (i > 64) __nanosleep(i > 65536 ? 1024 : 64);
            }
            ok_s = i < kGridPolls;
            if (!ok_s && a.err) atomicCAS(a.err, 0, ERR_GRID_SYNC);
        }
        __syncthreads();
        const bool ok = ok_s != 0;
        mlo = rv * z / ks;
        mhi = rv * (z + 1) / ks;
        if (ok)
            for (int i = tid; i < (mhi - mlo) * GM_BN; i += NTH) {
                const int mm = mlo + i / GM_BN, nn = i % GM_BN, n = n0 + nn;
                if (n >= a.N) continue;
                float v = 0.f;
                for (int q = 0; q < ks; ++q) v += __ldcg(a.ws + ((size_t)q * a.M + m0 + mm) * a.N + n);
                tile[mm * GM_EPI_LD + nn] = v;
            }
        __syncthreads();
        if (tid == 0) {  // the last split out clears the tile's counters for the next launch
            const unsigned d = atomicAdd(cnt + 1, 1u);
            if (d == (unsigned)ks - 1) {
                cnt[0] = 0u;
                cnt[1] = 0u;
            }
        }
        if (!ok) return;
    }
    if (a.epi == EPI_ARGMAX) {
        if (tid < mhi - mlo) {
            const int mm = mlo + tid, m = m0 + mm;
            unsigned long long best = 0ull;
            for (int nn = 0; nn < GM_BN && n0 + nn < a.N; ++nn) {
                const float v = tile[mm * GM_EPI_LD + nn];
                const unsigned long long k = argmax_key(v, (uint32_t)(n0 + nn));
                best = k > best ? k : best;
            }
            if (best) atomicMax(&a.keys[m], best);
        }
        if (a.store_logits)
            for (int i = tid; i < (mhi - mlo) * GM_BN; i += NTH) {
                const int mm = mlo + i / GM_BN, nn = i % GM_BN, m = m0 + mm, n = n0 + nn;
                if (n < a.N) a.y[(size_t)m * a.ldy + n] = tile[mm * GM_EPI_LD + nn];
            }
        return;
    }
    if (a.epi == EPI_SWIGLU) {  // one (gate, up) row pair per iteration: rows 2j and 2j + 1
        for (int i = tid; i < (mhi - mlo) * (GM_BN / 2); i += NTH) {
            const int mm = mlo + i / (GM_BN / 2), j = i % (GM_BN / 2), m = m0 + mm, n = n0 + 2 * j;
            if (n >= a.N) continue;  // N is even: the up row n + 1 exists with its gate row
            const float2 gu = *reinterpret_cast<const float2*>(tile + mm * GM_EPI_LD + 2 * j);
            a.y[(size_t)m * a.ldy + (n >> 1)] = __fmul_rn(__fdiv_rn(gu.x, 1.0f + expf(-gu.x)), gu.y);
        }
        return;
    }
    for (int i = tid; i < (mhi - mlo) * GM_BN; i += NTH) {
        const int mm = mlo + i / GM_BN, nn = i % GM_BN, m = m0 + mm, n = n0 + nn;
        if (n >= a.N) continue;
        const float v = tile[mm * GM_EPI_LD + nn];
        if (a.epi == EPI_STORE) {
            a.y[(size_t)m * a.ldy + n] = v + (a.bias ? a.bias[n] : 0.f);
        } else {  // EPI_RESID
            a.resid[(size_t)m * a.ldr + n] += v;
        }
    }
}

// ---- the GEMM on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) ---------------
// The products run as tcgen05.mma
// (kind::f16, M = 128 weight rows, N = NT activation rows, K = 16) issued by one thread, with the
// fp32 accumulator in tensor memory.  Operands sit in shared memory in the canonical K-major
// 128-byte-swizzled layout: a row's 64 k values (128 B) form one line of an 8-line, 1024-byte
// atom, and the 16-byte chunk c of line r is stored at chunk c ^ r, so that the tensor cores'
// reads of eight lines spread over all banks; atoms of 8 rows are SBO = 1024 B apart, and the
// 16-element k steps of the stage are 32 B apart within the lines.
// A tcgen05.commit per stage arrives on the barriers of the buffers it read once its MMAs
// have completed.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr) {
    // start >> 4 [0,14), LBO [16,30) (1: unused by swizzled K-major), SBO >> 4 [32,46),
    // version 1 [46,48), base offset 0, layout 2 = 128-byte swizzle [61,64)
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// the same with the A operand (the weights) in tensor memory: lane r holds row r, column c the
// k pair (2c, 2c + 1) of the instruction's 16 k values
__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
        :
        : "r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Shared memory of the tcgen05 GEMM: a ring of gemm_x_stages activation stages (Xh, Xl), whose
// bulk copies run that many stages ahead of the MMAs, and (WT) the ring of quantised weight
// chunks.  The dequantised weights (Wh, Wl of two k stages: the tensor cores read one while the
// dequantising warps write the next) live in tensor memory beside the accumulator, so the
// tensor cores' reads of the A operand and the dequantising warps' writes take no
// shared-memory bandwidth.
// Accumulators: for tiles up to 128 rows one per product of the split, Wh*Xh, Wh*Xl and Wl*Xh,
// side by side, so that the first two come from one MMA whose B operand is the stage's Xh and Xl
// halves together (2 NT rows, contiguous in shared memory): two MMAs per k step instead of three
// (at a few rows an MMA's cost barely depends on its N).  The 256-row tile keeps one
// accumulator and three MMAs (N is at its limit).  The epilogue sums the accumulators.
template <int NT>
constexpr int gemm_n_acc() {
    return NT <= 128 ? 3 : 1;
}
// tensor-memory columns: the accumulators' NT columns each, then per weight buffer Wh (32
// columns: 128 rows x 64 halves) and Wl (32); allocated as a power of two.  Weight buffers: as
// many as the 512 columns hold (up to four), so that the dequantising warps run that many stages
// ahead of the MMAs (an MMA batch completes ~1000 cycles after it is issued)
template <int NT>
constexpr uint32_t gemm_acc_cols() {
    return (uint32_t)(gemm_n_acc<NT>() * NT);
}
template <int NT>
constexpr int gemm_w_bufs() {
    return (512 - (int)gemm_acc_cols<NT>()) / 64 > 4 ? 4 : (512 - (int)gemm_acc_cols<NT>()) / 64;
}
template <int NT>
constexpr uint32_t gemm_tmem_cols() {
    return gemm_acc_cols<NT>() + 64u * gemm_w_bufs<NT>() <= 256 ? 256u : 512u;
}
template <int NT>
constexpr size_t gemm_x_stage_bytes() {
    return (size_t)2 * NT * GM_BK * 2;
}
// WT (weights by tensor-map copy, K % 256 == 0): the quantised rows arrive in chunks of GM_WCH
// stages (4 x 68 = 272 bytes of a Q8_0 row, 4 x 36 = 144 of a Q4_0 row: 16-byte multiples), one
// 2-D copy of 128 rows per chunk, into a ring of gemm_raw_chunks chunks; without WT every
// dequantising thread loads its words from global memory into registers.
constexpr int GM_WCH = 4;
template <bool Q4>
constexpr uint32_t gemm_chunk_bytes() {
    return (uint32_t)GM_BN * GM_WCH * (Q4 ? 36 : 68);
}
template <int NT, bool WT>
constexpr int gemm_x_stages() {
    // deep enough to cover a bulk copy's latency under the weight stream (~2000 cycles, two stages)
    return NT <= 32 ? 8 : NT <= 64 ? 6 : NT <= 128 ? 4 : 3;
}
template <int NT, bool Q4, bool WT>
constexpr int gemm_raw_chunks() {
    return !WT ? 0 : Q4 ? (NT <= 64 ? 4 : 3) : (NT <= 32 ? 4 : NT <= 64 ? 3 : 2);
}
template <int NT, bool Q4, bool WT>
constexpr size_t gemm_tc_smem_bytes() {
    const size_t pipe = (size_t)gemm_x_stages<NT, WT>() * gemm_x_stage_bytes<NT>() +
                        (size_t)gemm_raw_chunks<NT, Q4, WT>() * gemm_chunk_bytes<Q4>();
    const size_t epi = (size_t)NT * GM_EPI_LD * 4 + (size_t)NT * 4;  // tile + column scales
    // at least enough to keep a third CTA (a second with 512 columns) off the SM: tcgen05.alloc
    // waits while the SM's 512 columns are taken, and a waiting CTA must not hold up the other
    // k splits of its cluster
    const size_t floor = gemm_tmem_cols<NT>() > 256 ? (size_t)120 * 1024 : (size_t)80 * 1024;
    const size_t need = (pipe > epi ? pipe : epi) + GM_TC_TAIL + 1024;  // + mbarriers, TMEM address, alignment
    return need > floor ? need : floor;
}

template <int NT, bool Q4, bool WT>
__global__ void __launch_bounds__(GM_TC_THREADS, 1) tf_gemm_q8_tc_kernel(const GemmArgs a,
                                                                         const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // the swizzle atoms need 1024-byte aligned stage buffers
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * GM_BN, m0 = blockIdx.y * NT;
    const int nk_all = a.K / GM_BK;
    // the k range of this split (whole chunks with WT)
    const int ku = WT ? GM_WCH : 1, nu = nk_all / ku;
    const int kb = ku * (int)((long long)nu * blockIdx.z / gridDim.z);
    const int nk = ku * (int)((long long)nu * (blockIdx.z + 1) / gridDim.z) - kb;
    const float wscale = ldexpf(1.0f, a.sw);
    constexpr int XS = gemm_x_stages<NT, WT>();
    constexpr int WB = gemm_w_bufs<NT>();
    constexpr int RC = gemm_raw_chunks<NT, Q4, WT>();
    constexpr int RCd = RC > 0 ? RC : 1;  // (divisor in code only the WT instantiations run)
    constexpr int UB = Q4 ? 36 : 68;               // bytes of a row's 64-weight stage
    constexpr uint32_t RB = GM_WCH * UB;           // bytes of a row's chunk
    constexpr uint32_t XH = NT * GM_BK * 2;  // bytes of one activation half of a stage
    uint8_t* tail = smem + gemm_tc_smem_bytes<NT, Q4, WT>() - GM_TC_TAIL - 1024;
    // [WB] weight stage written (dequant warps; warp 0 arrives only once it has also seen the
    // stage's activations land, so this one barrier is all the MMA thread waits on)
    uint64_t* wready = reinterpret_cast<uint64_t*>(tail);
    uint64_t* wfree = wready + WB;                         // [WB] its MMAs completed
    uint64_t* xfull = wfree + WB;                          // [XS] activation stage landed
    uint64_t* xempty = xfull + XS;                         // [XS] its MMAs completed
    uint64_t* mma_done = xempty + XS;                      // every MMA completed
    uint64_t* rfull = mma_done + 1;                        // [RC] weight chunk landed (WT)
    uint64_t* rempty = rfull + RC;                         // [RC] chunk read by the dequantising warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rempty + RC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const bool trc = a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
    auto stamp = [&](int i) {
        if (trc) a.trace[i] = (unsigned long long)clock64();
    };
    if (tid == 0) stamp(0);
    auto xh = [&](int b) { return smem + (size_t)b * 2 * XH; };
    auto raw = [&](int c) { return smem + (size_t)XS * 2 * XH + (size_t)c * gemm_chunk_bytes<Q4>(); };
    constexpr uint32_t TCOLS = gemm_tmem_cols<NT>();

    if (warp == 0) {  // TMEM: the NT x 128 fp32 accumulator (NT columns) and the two weight buffers
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    if (tid == GM_DQ_THREADS) {
        for (int i = 0; i < WB; ++i) {
            mbar_init(&wready[i], GM_DQ_THREADS / 32);
            mbar_init(&wfree[i], 1);
        }
        for (int i = 0; i < XS; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], 1);
        }
        mbar_init(mma_done, 1);
        for (int i = 0; i < RC; ++i) {
            mbar_init(&rfull[i], 1);
            mbar_init(&rempty[i], GM_DQ_THREADS / 32);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) stamp(1);

    // dequantising warp w: weight rows 32 (w % 4) + lane (its tensor-memory lane quarter), the
    // stage's 16-weight piece w / 4 (block, half: the MMA k step it feeds); its Wh / Wl words go to
    // tensor-memory columns AC + 64 s + (0 | 32) + 8 * piece of weight buffer s
    constexpr uint32_t AC = gemm_acc_cols<NT>();  // first column of the weight buffers
    const uint32_t tq = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + AC + 8u * (uint32_t)(warp >> 2);
    if (WT && warp < GM_DQ_THREADS / 32) {
        // ---- dequantising warps (WT): stage kc's words from the chunk ring ----
        const int wr = 32 * (warp & 3) + lane, wjh = warp >> 2;  // weight row, 16-weight piece (block, half)
        const int sw0 = Q4 ? 4 * (wjh >> 1) : 8 * (wjh >> 1);  // word of the block's scale
        const int ww0 = Q4 ? 4 * (wjh >> 1) : 4 * wjh;         // first of the piece's five words
        pdl_trigger();
        pdl_wait();
        bool ok = true;
        for (int kc = 0; kc < nk && ok; ++kc) {
            const int s = kc % WB, ci = kc / GM_WCH, j = kc % GM_WCH, slot = ci % RCd;
            if (j == 0) ok = mbar_wait(&rfull[slot], (ci / RCd) & 1, a.err, ERR_WAIT_FULL, abort_flag);
            const bool tk = tid == 0 && kc < GM_TR_MAXK;
            if (tk) stamp(GM_TR_DQ + 4 * kc);
            // buffer s was last read by the MMAs of stage kc - WB
            if (ok && kc >= WB) ok = mbar_wait(&wfree[s], ((kc / WB) - 1) & 1, a.err, ERR_WAIT_EMPTY, abort_flag);
            if (ok && warp == 0) ok = mbar_wait(&xfull[kc % XS], (kc / XS) & 1, a.err, ERR_WAIT_FULL, abort_flag);
            if (tk) stamp(GM_TR_DQ + 4 * kc + 1);
            ok = __all_sync(0xffffffffu, ok);  // the tensor-memory stores below are warp-wide
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t* rw = reinterpret_cast<const uint32_t*>(raw(slot) + wr * RB + j * UB);
            uint32_t w[6], hv[8], lv[8];
            w[0] = rw[sw0];
#pragma unroll
            for (int i = 0; i < 5; ++i) w[1 + i] = rw[ww0 + i];
            gm_dequant16_r<Q4>(w, (uint32_t)(wjh >> 1), (uint32_t)(wjh & 1), wscale, hv, lv);
            tmem_st8(tq + 64u * (uint32_t)s, hv);
            tmem_st8(tq + 64u * (uint32_t)s + 32u, lv);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&wready[s]);
                if (j == GM_WCH - 1) mbar_arrive(&rempty[slot]);  // the chunk's last stage is read
                if (trc && kc < GM_TR_MAXK) {  // warp 0's arrival; the last arrival and its warp
                    const unsigned long long t = (unsigned long long)clock64();
                    if (warp == 0) a.trace[GM_TR_DQ + 4 * kc + 2] = t;
                    atomicMax(&a.trace[GM_TR_DQ + 4 * kc + 3], (t << 5) | (unsigned long long)warp);
                }
            }
        }
    } else if (warp < GM_DQ_THREADS / 32) {
        // ---- dequantising warps: stage kc's weights into weight buffer kc % WB ----
        // The weight words of the next GM_WPF stages are in flight in registers (a stage's
        // 68-byte row pieces come from HBM); the first ones are requested before the PDL wait.
        constexpr int PF = GM_WPF;
        const int wr = 32 * (warp & 3) + lane, wjh = warp >> 2;  // weight row, 16-weight piece (block, half)
        uint32_t wbuf[PF][6];                    // weight words of stage kc in slot kc % PF
#pragma unroll
        for (int u = 0; u < PF; ++u)
            if (u < nk) gm_load_w16<Q4>(wbuf[u], a, n0 + wr, kb + u, wjh);
        pdl_trigger();
        pdl_wait();
        bool ok = true;
        // unrolled by PF so that every register slot index is static
        for (int kc0 = 0; kc0 < nk && ok; kc0 += PF) {
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int kc = kc0 + u;
                if (kc < nk && ok) {
                    const int s = kc % WB;
                    const bool tk = tid == 0 && kc < GM_TR_MAXK;
                    if (tk) stamp(GM_TR_DQ + 4 * kc);
                    // buffer s was last read by the MMAs of stage kc - WB
                    if (kc >= WB) ok = mbar_wait(&wfree[s], ((kc / WB) - 1) & 1, a.err, ERR_WAIT_EMPTY, abort_flag);
                    if (ok && warp == 0)
                        ok = mbar_wait(&xfull[kc % XS], (kc / XS) & 1, a.err, ERR_WAIT_FULL, abort_flag);
                    if (tk) stamp(GM_TR_DQ + 4 * kc + 1);
                    ok = __all_sync(0xffffffffu, ok);  // the tensor-memory stores below are warp-wide
                    if (ok) {
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        uint32_t hv[8], lv[8];
                        gm_dequant16_r<Q4>(wbuf[u], (uint32_t)(wjh >> 1), (uint32_t)(wjh & 1), wscale, hv, lv);
                        if (kc + PF < nk) gm_load_w16<Q4>(wbuf[u], a, n0 + wr, kb + kc + PF, wjh);
                        tmem_st8(tq + 64u * (uint32_t)s, hv);
                        tmem_st8(tq + 64u * (uint32_t)s + 32u, lv);
                        // the stores complete before the tensor cores read them, then the warp arrives
                        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&wready[s]);
                            if (trc && kc < GM_TR_MAXK) {  // warp 0's arrival; the last arrival and its warp
                                const unsigned long long t = (unsigned long long)clock64();
                                if (warp == 0) a.trace[GM_TR_DQ + 4 * kc + 2] = t;
                                atomicMax(&a.trace[GM_TR_DQ + 4 * kc + 3], (t << 5) | (unsigned long long)warp);
                            }
                        }
                    }
                }
            }
        }
    } else if (warp == GM_X_WARP) {
        // ---- activation copies: stage kc into ring slot kc % XS (two bulk copies) ----
        pdl_trigger();
        pdl_wait();
        if (lane == 0) {
            stamp(2);
            const size_t xstride = (size_t)a.mp * (GM_BK * 2);
            const uint8_t* xhs = reinterpret_cast<const uint8_t*>(a.xh) + (size_t)kb * xstride + (size_t)m0 * (GM_BK * 2);
            const uint8_t* xls = reinterpret_cast<const uint8_t*>(a.xl) + (size_t)kb * xstride + (size_t)m0 * (GM_BK * 2);
            int issued = 0;
            for (int kc = 0; kc < nk; ++kc) {
                const int b = kc % XS;
                if (kc >= XS && !mbar_wait(&xempty[b], ((kc / XS) - 1) & 1, a.err, ERR_WAIT_EMPTY, abort_flag)) break;
                if (kc < GM_TR_MAXK) stamp(GM_TR_X + kc);
                mbar_expect_tx(&xfull[b], 2 * XH);
                bulk_g2s(xh(b), xhs + (size_t)kc * xstride, XH, &xfull[b]);
                bulk_g2s(xh(b) + XH, xls + (size_t)kc * xstride, XH, &xfull[b]);
                ++issued;
            }
            // copies in flight land before the buffers are reused (only pending after an abort)
            for (int kc = issued > XS ? issued - XS : 0; kc < issued; ++kc)
                mbar_wait(&xfull[kc % XS], (kc / XS) & 1, nullptr, 0, nullptr);
        }
        __syncwarp();  // the other lanes wait here without issuing, not in a polling loop
    } else if (warp == GM_W_WARP) {
        // ---- weight chunks (WT): one 2-D tensor copy of the tile's 128 rows x RB bytes per chunk
        // (rows past N filled with zeros) into ring slot c % RC, the first RC before the PDL wait;
        // chunk c takes the slot once the dequantising warps have read chunk c - RC ----
        if (WT && lane == 0) {
            const int nch = nk / GM_WCH;
            auto issue_chunk = [&](int c) {
                const int slot = c % RCd;
                if (c < GM_TR_DQ - GM_TR_CHUNK) stamp(GM_TR_CHUNK + c);
                mbar_expect_tx(&rfull[slot], gemm_chunk_bytes<Q4>());
                // x: the chunk's first 16-bit element of the row (a multiple of 8: 16-byte aligned)
                const int x = (kb + c * GM_WCH) * UB / 2;
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                        smem_u32(raw(slot))),
                    "l"(reinterpret_cast<uint64_t>(&wmap)), "r"(x), "r"(n0), "r"(smem_u32(&rfull[slot]))
                    : "memory");
            };
            const int pre = nch < RC ? nch : RC;
            for (int c = 0; c < pre; ++c) issue_chunk(c);
            int issued = pre;
            pdl_trigger();
            pdl_wait();
            for (int c = pre; c < nch; ++c) {
                if (!mbar_wait(&rempty[c % RCd], ((c / RCd) - 1) & 1, a.err, ERR_WAIT_EMPTY, abort_flag)) break;
                issue_chunk(c);
                ++issued;
            }
            // copies in flight land before the buffers are reused (only pending after an abort)
            for (int c = issued > RC ? issued - RC : 0; c < issued; ++c)
                mbar_wait(&rfull[c % RCd], (c / RCd) & 1, nullptr, 0, nullptr);
        } else {
            pdl_trigger();
            pdl_wait();
        }
        __syncwarp();
    } else {  // warp == GM_MMA_WARP
        // ---- MMA issue: one thread ----
        pdl_trigger();
        pdl_wait();
        if (lane == 0) {
            // instruction descriptors: D f32, A/B f16, both K-major, M = 128, N = NT (and 2 NT)
            const uint32_t idesc = (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(GM_BN >> 4) << 24);
            const uint32_t idesc2 = (1u << 4) | ((uint32_t)((2 * NT) >> 3) << 17) | ((uint32_t)(GM_BN >> 4) << 24);
            for (int kc = 0; kc < nk; ++kc) {
                const int s = kc % WB, b = kc % XS;
                // the weights of stage kc are in buffer s, and (dequantising warp 0 saw it before
                // it arrived) its activations in ring slot b
                if (!mbar_wait(&wready[s], (kc / WB) & 1, a.err, ERR_WAIT_FULL, abort_flag)) break;
                if (kc < GM_TR_MAXK) stamp(GM_TR_MMA + 2 * kc);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                // Wh / Wl of buffer s in tensor memory (8 columns per k step), Xh / Xl in shared memory
                // (a k step is 32 bytes along the lines: 2 in the descriptor's start-address field,
                // which holds address >> 4 < 2^14 with room for the steps)
                const uint32_t ah = tmem + AC + 64u * (uint32_t)s, al = ah + 32u;
                const uint64_t dh = umma_desc_k_sw128(smem_u32(xh(b))), dl = umma_desc_k_sw128(smem_u32(xh(b)) + XH);
#pragma unroll
                for (int j = 0; j < GM_BK / 16; ++j) {  // 16-element k steps
                    const uint32_t c = 8u * j;
                    const uint32_t first = (kc > 0 || j > 0) ? 1u : 0u;
                    if constexpr (gemm_n_acc<NT>() > 1) {
                        // Wh * [Xh; Xl] into columns [0, 2 NT), Wl * Xh into [2 NT, 3 NT)
                        umma_f16_ta(tmem, ah + c, dh + 2u * j, idesc2, first);
                        umma_f16_ta(tmem + 2u * NT, al + c, dh + 2u * j, idesc, first);
                    } else {
                        umma_f16_ta(tmem, ah + c, dh + 2u * j, idesc, first);
                        umma_f16_ta(tmem, ah + c, dl + 2u * j, idesc, 1u);
                        umma_f16_ta(tmem, al + c, dh + 2u * j, idesc, 1u);
                    }
                }
                umma_commit(&wfree[s]);
                umma_commit(&xempty[b]);
                if (kc < GM_TR_MAXK) stamp(GM_TR_MMA + 2 * kc + 1);
            }
            umma_commit(mma_done);  // arrives once every MMA issued above has completed
        }
        __syncwarp();
    }
    // (not cut short by an abort: TMEM stays allocated until every issued MMA has completed)
    if (!mbar_wait(mma_done, 0, a.err, ERR_WAIT_FULL, nullptr)) *abort_flag = 1;
    if (tid == 0) stamp(3);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    __syncthreads();
    const bool ok = *abort_flag == 0 && nk > 0;

    // ---- epilogue: TMEM -> registers -> scaled tile[m][n] in shared memory ----
    float* tile = reinterpret_cast<float*>(smem);  // [NT][GM_EPI_LD], the pipeline buffers are free
    // 2^-(sw + sx[m]) of every activation row of the tile (0 for rows past M or after an error),
    // kept beside the tile
    float* colsc = tile + (size_t)NT * GM_EPI_LD;
    if (tid < NT) {
        const int m = m0 + tid;
        colsc[tid] = (ok && m < a.M) ? ldexpf(1.0f, -(a.sw + a.sx[m])) : 0.f;
    }
    __syncthreads();
    if (warp < 16) {  // sixteen warps: four TMEM lane quarters x four column groups
        const int row = 32 * (warp & 3) + lane;  // weight row of this thread's TMEM lane
        const int c0 = (warp >> 2) * (NT / 4);
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        if constexpr (gemm_n_acc<NT>() == 1) {
            for (int c = c0; c < c0 + NT / 4; c += 16) {
                uint32_t r[16];
                tmem_ld16(tl + (uint32_t)c, r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int u = 0; u < 16; ++u) tile[(c + u) * GM_EPI_LD + row] = __uint_as_float(r[u]) * colsc[c + u];
            }
        } else {  // the three accumulators: main product plus the sum of the two corrections
            for (int c = c0; c < c0 + NT / 4; c += 8) {
                uint32_t r0[8], r1[8], r2[8];
                tmem_ld8(tl + (uint32_t)c, r0);
                tmem_ld8(tl + (uint32_t)(NT + c), r1);
                tmem_ld8(tl + (uint32_t)(2 * NT + c), r2);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    tile[(c + u) * GM_EPI_LD + row] =
                        (__uint_as_float(r0[u]) + (__uint_as_float(r1[u]) + __uint_as_float(r2[u]))) * colsc[c + u];
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
    // with k splits the cluster's barriers are kept even after an error (gemm_epilogue returns
    // after them); without, the error word holds the failure
    if (!ok && gridDim.z == 1) return;
    gemm_epilogue<NT, true, GM_TC_THREADS>(a, tile, m0, n0, ok);
    if (trc) {
        __syncthreads();
        if (tid == 0) stamp(4);
    }
}

// ---- end of a step at M rows ------------------------------------------------------------------
__global__ void tf_finish_kernel(const FinishArgs a) {
    __shared__ int gs_s;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) gs_s = a.ctl->gen_step;
    __syncthreads();
    const int gs = gs_s;
    for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
        if (a.argmax) {
            const unsigned long long k = a.keys[m];
            a.keys[m] = 0ull;
            const int tok = (int)key_index(k);
            a.tok_next[m] = tok;
            if (a.hist && gs < a.ctl->hist_cap) a.hist[(size_t)gs * a.M + m] = tok;
        }
        atomicAdd(&a.pos[a.slots[m]], 1);  // rows of one prefill chunk share a slot
    }
    __syncthreads();
    if (threadIdx.x == 0 && a.argmax) a.ctl->gen_step = gs + 1;
}

// ---- host ----------------------------------------------------------------------------------------
static cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t xprep_launch(const XPrepArgs& a, cudaStream_t st) {
    if (a.K % GM_BK) return cudaErrorInvalidValue;
    // rows read from memory (no embedding lookup) that fit the registers: the register kernel
    const bool regs = !a.embd && a.K / 4 <= XP_THREADS * XP_REG_CHUNKS;
    const size_t smem = regs ? 0 : (size_t)xpad_len(a.K) * 4;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(tf_xprep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    XPrepArgs aa = a;
    aa.mp = gemm_x_rows(a.M);
    // programmatic dependent launch: the CTAs become resident while the previous kernel drains
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.M);
    cfg.blockDim = dim3(XP_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, regs ? tf_xprep_rows_kernel : tf_xprep_kernel, aa);
}

int gemm_x_rows(int M) {
    const int nt = gemm_tile_rows(M);
    return (M + nt - 1) / nt * nt;
}

int gemm_tile_rows(int M) {
    // the MMA's N is the tile's activation rows: a tile no wider than the rows present keeps
    // the tensor-core time of a few-row step down (TFB200_GEMM_NT=128: at least 128 rows, at
    // most 128; =256: at least 128 rows)
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_GEMM_NT");
        v = e ? atoi(e) : 0;
    }
    if (v == 128) return 128;
    if (M > 128) return 256;
    if (v == 256 || M > 64) return 128;
    return M > 32 ? 64 : 32;
}

bool gemm_takes_q4() { return true; }


// The tensor map of a weight matrix for the WT path: 16-bit elements, rows of rb / 2 elements
// rb bytes apart, boxes of one chunk (GM_WCH stages) x 128 rows; rows past N read as zeros.
static bool gemm_weight_map(CUtensorMap* m, const GemmArgs& a) {
    static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    if (!enc) return false;
    const int ub = a.wq4 ? 36 : 68;
    const cuuint64_t dims[2] = {(cuuint64_t)(a.rb / 2), (cuuint64_t)a.N};
    const cuuint64_t strides[1] = {(cuuint64_t)a.rb};
    const cuuint32_t box[2] = {(cuuint32_t)(GM_WCH * ub / 2), (cuuint32_t)GM_BN};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(a.W), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool gemm_wt_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_GEMM_WT");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

static unsigned long long* g_gemm_trace = nullptr;
void gemm_set_trace(unsigned long long* buf) { g_gemm_trace = buf; }

cudaError_t gemm_launch(const GemmArgs& a, cudaStream_t st) {
    if (a.K % GM_BK || a.M <= 0 || a.N <= 0) return cudaErrorInvalidValue;
    int ks = a.ksplit > 1 ? a.ksplit : 1;
    if (ks > 1 && (!a.ws || !a.tile_cnt || ks > GM_MAX_SPLIT)) return cudaErrorInvalidValue;
    GemmArgs aa = a;
    if (!aa.trace) aa.trace = g_gemm_trace;
    aa.mp = gemm_x_rows(a.M);
    alignas(64) CUtensorMap wmap;
    memset(&wmap, 0, sizeof(wmap));
    void* args[] = {&aa, &wmap};
    const int nt = gemm_tile_rows(a.M);
    const int wi = nt == 256 ? 3 : nt == 128 ? 2 : nt == 64 ? 1 : 0;
    const bool q4 = a.wq4 != 0;
    // weights by bulk copy: rows 16-byte aligned, whole chunks per split (tiles up to 128 rows:
    // the 256-row tile's activation stages leave no room for the chunk ring)
    const int nch = a.K / (GM_BK * GM_WCH);
    const bool wt = gemm_wt_enabled() && nt <= 128 && a.K % (GM_BK * GM_WCH) == 0 && a.rb % 16 == 0 &&
                    (reinterpret_cast<uintptr_t>(a.W) & 15) == 0 && nch > 0 && gemm_weight_map(&wmap, a);
    if (wt && ks > nch) ks = nch;
    static const size_t sms[4][2][2] = {
        {{gemm_tc_smem_bytes<32, false, false>(), gemm_tc_smem_bytes<32, false, true>()},
         {gemm_tc_smem_bytes<32, true, false>(), gemm_tc_smem_bytes<32, true, true>()}},
        {{gemm_tc_smem_bytes<64, false, false>(), gemm_tc_smem_bytes<64, false, true>()},
         {gemm_tc_smem_bytes<64, true, false>(), gemm_tc_smem_bytes<64, true, true>()}},
        {{gemm_tc_smem_bytes<128, false, false>(), gemm_tc_smem_bytes<128, false, true>()},
         {gemm_tc_smem_bytes<128, true, false>(), gemm_tc_smem_bytes<128, true, true>()}},
        {{gemm_tc_smem_bytes<256, false, false>(), 0}, {gemm_tc_smem_bytes<256, true, false>(), 0}}};
    static const void* fns[4][2][2] = {
        {{(const void*)tf_gemm_q8_tc_kernel<32, false, false>, (const void*)tf_gemm_q8_tc_kernel<32, false, true>},
         {(const void*)tf_gemm_q8_tc_kernel<32, true, false>, (const void*)tf_gemm_q8_tc_kernel<32, true, true>}},
        {{(const void*)tf_gemm_q8_tc_kernel<64, false, false>, (const void*)tf_gemm_q8_tc_kernel<64, false, true>},
         {(const void*)tf_gemm_q8_tc_kernel<64, true, false>, (const void*)tf_gemm_q8_tc_kernel<64, true, true>}},
        {{(const void*)tf_gemm_q8_tc_kernel<128, false, false>, (const void*)tf_gemm_q8_tc_kernel<128, false, true>},
         {(const void*)tf_gemm_q8_tc_kernel<128, true, false>, (const void*)tf_gemm_q8_tc_kernel<128, true, true>}},
        {{(const void*)tf_gemm_q8_tc_kernel<256, false, false>, nullptr},
         {(const void*)tf_gemm_q8_tc_kernel<256, true, false>, nullptr}}};
    const size_t sm = sms[wi][q4][wt];
    const void* fn = fns[wi][q4][wt];
    static bool tc_attr[64][4][2][2] = {};
    int dv = 0;
    cudaGetDevice(&dv);
    if (dv < 0 || dv >= 64) dv = 0;
    if (!tc_attr[dv][wi][q4][wt]) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        tc_attr[dv][wi][q4][wt] = true;
    }
    // the k splits of a tile form one cluster (their reduction goes through distributed
    // shared memory)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.N + GM_BN - 1) / GM_BN, (a.M + nt - 1) / nt, ks);
    cfg.blockDim = dim3(GM_TC_THREADS);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = (unsigned)ks;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t finish_launch(const FinishArgs& a, cudaStream_t st) {
    FinishArgs aa = a;
    void* args[] = {&aa};
    return launch_pdl((const void*)tf_finish_kernel, dim3(1), dim3(256), 0, st, args);
}

// Device version of q8_scale_exponent for weights that live only on the device: the largest
// |d| bits over all blocks (one pass over the scale bytes).
__global__ void tf_q8_dmax_kernel(const uint8_t* W, long long n_blocks, int block_bytes, unsigned* out) {
    unsigned mx = 0;
    for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks; b += (long long)gridDim.x * blockDim.x) {
        const unsigned d = ((unsigned)W[b * block_bytes] | ((unsigned)W[b * block_bytes + 1] << 8)) & 0x7FFFu;
        mx = d > mx ? d : mx;
    }
    mx = warp_max_u(mx);
    if ((threadIdx.x & 31) == 0) atomicMax(out, mx);
}

int q8_exponent_from_dbits(unsigned mx) {
    if (mx == 0 || mx >= 0x7C00u) return 0;
    const int E = (mx >> 10) > 0 ? (int)(mx >> 10) : 1;
    return 21 - E;
}

cudaError_t q8_scale_exponent_device(const uint8_t* W, long long n_blocks, unsigned* scratch, int* sw, cudaStream_t st,
                                     int block_bytes) {
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(unsigned), st);
    if (e != cudaSuccess) return e;
    tf_q8_dmax_kernel<<<296, 256, 0, st>>>(W, n_blocks, block_bytes, scratch);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    unsigned h = 0;
    if ((e = cudaMemcpyAsync(&h, scratch, sizeof(unsigned), cudaMemcpyDeviceToHost, st)) != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return e;
    *sw = q8_exponent_from_dbits(h);
    return cudaSuccess;
}

// 2^sw with |q * d| * 2^sw < 2^14 for every block of the matrix (|q| <= 128; Q4_0 blocks,
// |q| <= 8, take the same bound).  The fp16 d leads every Q8_0 and Q4_0 block.
int q8_scale_exponent(const uint8_t* blocks, size_t nbytes, int block_bytes) {
    unsigned mx = 0;
    for (size_t o = 0; o + block_bytes <= nbytes; o += block_bytes) {
        const unsigned d = ((unsigned)blocks[o] | ((unsigned)blocks[o + 1] << 8)) & 0x7FFFu;
        mx = d > mx ? d : mx;
    }
    // |d| < 2^(E-14) for the f16 biased exponent E (subnormals: E = 1), so |q*d| < 2^(E-7)
    // and 2^(21-E) maps the matrix below 2^14
    return q8_exponent_from_dbits(mx);
}

}  // namespace tfb
