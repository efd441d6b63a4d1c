// Dequant-GEMV kernel (see gemv.cuh).
//
// Data movement: each CTA owns a contiguous range of output items; its weight bytes are a
// contiguous byte range of the tensor, streamed global -> shared in stages by a producer
// warp with 1-D bulk copies (TMA engine, mbarrier completion), GV_STAGES deep.  The copies
// are issued before griddepcontrol.wait, so under programmatic dependent launch a kernel
// streams its weights while the previous kernel of the step is still finishing.  The
// activation rows sit in shared memory in a padded layout (xpad) after the prologue.
//
// Arithmetic: fp32 activations times dequantised weights with fp32 accumulation, the
// reference's own arithmetic (src/quant.cpp:266-363): for Q8_0/Q4_0 the block sum
// sum_j x_j*q_j is formed first and scaled by the block's fp16 d; Q4_1/Q6_K/F16/F32 rows
// are dequantised exactly as dequant_row does and dotted (src/matmul.cpp:5-20).  The
// summation order differs from the CPU's 8-lane order; results agree to fp32 rounding.
//
// Q8_0 fast path: a lane owns 64-element units (two 34-byte blocks = 17 aligned words,
// conflict-free shared loads at a 17-word lane stride); int8 -> fp32 conversion uses the
// exact magic-number construction 0x4B0000xx - (2^23 + 128) (one PRMT + one FADD), which
// keeps the conversion off the 16/clk conversion pipe.
//
// Exact-integer paths (one activation row; dots.cuh): the prologue turns the row into three
// signed-byte digit planes per 32-element block, each lane keeps its unit's plane words in
// registers, and the block sums are exact dp4a sums scaled by the block's d (and 2^-sh):
// Q8_0 rows (INTQ 1; INTQ 4 is the same kernel with the split fused attention), Q4_0 rows of
// matrices of 32 MB and more (INTQ 2) and Q6_K rows with K % 512 == 0 (INTQ 3).  Each is its
// own instantiation, so the Q8_0 kernel that a Q8_0 step launches for every GEMV carries no
// other path's code or registers.
#include <algorithm>
#include <cstdlib>

#include "dots.cuh"
#include "gemv.cuh"

namespace tfb {

// floats of the cross-warp reduction buffer: two parities x warps x (2 rows x max(M, 2))
__host__ __device__ constexpr int gv_red_floats(int maxm) { return 2 * GV_WARPS * 2 * (maxm < 2 ? 2 : maxm); }

// launch trace: this CTA's stamp k (see GemvArgs::trace)
__device__ __noinline__ void gv_stamp(unsigned long long* trace, int k) {
    trace[(size_t)blockIdx.x * GV_TRACE_SLOTS + k] = global_ns();
}
// the same, taken once `dep` has been computed
__device__ __noinline__ void gv_stamp_after(unsigned long long* trace, int k, double dep) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "d"(dep));
    trace[(size_t)blockIdx.x * GV_TRACE_SLOTS + k] = t;
}

__device__ __forceinline__ void named_bar_compute() {
    asm volatile("bar.sync 1, %0;" ::"n"(GV_WARPS * 32) : "memory");
}

// Split fused attention, after the tile loop: this split's partial (max, sum, weighted V;
// every split CTA leaves one, an empty or failed one with max -inf and sum 0, so the head's
// ticket count stays whole) goes to part[qh][sp]; the last of the head's CTAs combines the
// nsf partials in split order (deterministic) into out and the wo digit planes.  pacc holds
// the ng groups' weighted V sums; scratch (3 * nsf floats) and flag[1] are shared memory.
// Out of line, with plain arguments, so that the QKV GEMV's register allocation does not
// carry it.
__device__ __noinline__ void fused_attn_split_out(float* part, int n_split, unsigned* ticket, float* out,
                                                  uint8_t* yplanes, int n_head, int qh, int sp, int nsf, int hd,
                                                  int ng, const float* pacc, float* scratch, int* flag, float m_run,
                                                  float l_run) {
    const int tid = threadIdx.x, nth = blockDim.x;
    float* pp = part + ((size_t)qh * n_split + sp) * (hd + 2);
    for (int d = tid; d < hd; d += nth) {
        float o = 0.f;
        for (int g = 0; g < ng; ++g) o += pacc[g * hd + d];
        pp[2 + d] = o;
    }
    if (tid == 0) {
        pp[0] = m_run;
        pp[1] = l_run;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) flag[1] = atomicAdd(ticket + qh, 1u) == (unsigned)nsf - 1;
    __syncthreads();
    if (!flag[1]) return;
    __threadfence();
    float* cm = scratch;  // [nsf] maxima, [nsf] sums, [nsf] weights
    const float* pb = part + (size_t)qh * n_split * (hd + 2);
    for (int q = tid; q < nsf; q += nth) {
        cm[q] = __ldcg(pb + (size_t)q * (hd + 2));
        cm[nsf + q] = __ldcg(pb + (size_t)q * (hd + 2) + 1);
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int q = 0; q < nsf; ++q) mx = fmaxf(mx, cm[q]);
    for (int q = tid; q < nsf; q += nth) cm[2 * nsf + q] = expf(cm[q] - mx);
    __syncthreads();
    float den = 0.f;
    for (int q = 0; q < nsf; ++q) den = fmaf(cm[2 * nsf + q], cm[nsf + q], den);
    for (int d = tid; d < hd; d += nth) {  // whole warps (hd is a multiple of 32)
        float num = 0.f;
        for (int q = 0; q < nsf; ++q) num = fmaf(cm[2 * nsf + q], __ldcg(pb + (size_t)q * (hd + 2) + 2 + d), num);
        const float o = num / den;
        out[(size_t)qh * hd + d] = o;
        if (yplanes) {
            const int pstride = q8_plane_stride(n_head * hd);
            q8_block_planes_warp(o, (qh * hd + d) >> 5, yplanes, pstride, reinterpret_cast<float*>(yplanes + 3 * pstride));
        }
    }
    if (tid == 0) ticket[qh] = 0u;
}

// ---- fused decode attention (one query head per CTA, appended to the QKV GEMV grid) -------
// Model::layer_decode's apply_rope on q and k, KVCache::store and attn_decode for query head
// `cta` (src/model.cpp:125-129, src/attention.cpp:31-80), M == 1.  The cached K/V rows and the
// position's cos/sin are loaded into shared memory before the q/k/v of this step exist (they
// do not depend on them), so the loads overlap the GEMV CTAs' work; then the CTA waits
// (bounded) until every GEMV CTA has stored its rows, rotates, stores the new k/v (the first
// query head of each kv group) and attends over [ws, pos] in tiles of `tp` positions with an
// online softmax.  Every phase uses the whole CTA: one position per thread for the scores
// (float4 reads of q and of K rows padded to hd + 4 floats), CTA-wide max / sum, and ng
// groups of hd threads for the weighted V sum (group g takes positions g, g + ng, ...).
// SPLIT (its own kernel instantiation, launched only when a head's positions are split):
// CTA cta owns query head cta % n_head and position split cta / n_head of attn_nsf.
template <bool SPLIT, bool TR>
__device__ __forceinline__ void fused_attention(const GemvArgs& a, uint8_t* smem, size_t avail, int cta, int G) {
    const AttnArgs& t = a.at;
    const int tid = threadIdx.x, nth = blockDim.x, warp = tid >> 5, lane = tid & 31, nw = nth >> 5;
    const int hd = t.hd, d2 = hd / 2, n_rep = t.n_head / t.n_kv;
    const int nsf = SPLIT ? (a.attn_nsf > 1 ? a.attn_nsf : 1) : 1;  // position splits per query head
    const int qh = SPLIT ? cta % t.n_head : cta, sp = SPLIT ? cta / t.n_head : 0, kvh = qh / n_rep;
    const bool storer = qh % n_rep == 0 && sp == 0;
    const int kst = hd + 4;
    const int ng = min(8, nth / hd);
    float* f = reinterpret_cast<float*>(smem);
    float* qs = f;                   // [hd]
    float* kn = qs + hd;             // [hd]
    float* vn = kn + hd;             // [hd]
    float* cs = vn + hd;             // [d2] cos / sin of pos
    float* sn = cs + d2;             // [d2]
    float* red = sn + d2;            // [2][32] per-warp maxima / sums
    int* flag = reinterpret_cast<int*>(red + 64);
    float* pacc = red + 68;          // [ng][hd]
    float* sc = pacc + ng * hd;      // [tp] exp(score - max)
    const int fixed = 4 * hd + 68 + ng * hd;
    int tp = (int)((avail / 4 - fixed) / (1 + kst + hd));
    tp = (tp > 256 ? 256 : tp) & ~3;  // <= one position per thread; keeps ks 16-byte aligned
    float* ks = sc + tp;             // [tp][kst]
    float* vs = ks + (size_t)tp * kst;  // [tp][hd]

    pdl_trigger();
    pdl_wait();
    if (TR && tid == 0) gv_stamp(a.trace, 1);
    const int slot = t.slots ? t.slots[0] : 0;
    const int pos = t.pos[slot];
    const bool pos_ok = pos >= 0 && pos < t.cap && tp >= 4;
    const int ws = pos_ok ? ((t.wstart) ? min(max(t.wstart[slot], 0), pos) : 0) : 0;
    const size_t cache_off = (size_t)slot * t.slot_stride + (size_t)kvh * t.cap * hd;
    // this split's positions [s0, s1) of [ws, pos] (split 0 is never empty)
    int s0 = ws, s1 = pos + 1;
    if constexpr (SPLIT) {
        const int span = pos_ok ? (pos + 1 - ws + nsf - 1) / nsf : 0;
        s0 = ws + sp * span;
        s1 = pos_ok ? min(pos + 1, s0 + span) : s0;
    }
    // the first tile's cached rows and the rotation of pos, before q/k/v are ready
    if (pos_ok) {
        if (!SPLIT || s0 < s1) {
            const int np = min(s1, s0 + tp) - s0;
            const int npc = (s0 + np == pos + 1) ? np - 1 : np;
            load_tile(ks, kst, hd, t.kc, (long long)(cache_off + (size_t)s0 * hd), npc, t.kv_type, nth);
            load_tile(vs, hd, hd, t.vc, (long long)(cache_off + (size_t)s0 * hd), npc, t.kv_type, nth);
        }
        for (int i = tid; i < d2; i += nth) {
            cs[i] = t.cosb[(size_t)pos * d2 + i];
            sn[i] = t.sinb[(size_t)pos * d2 + i];
        }
    }
    if (tid == 0) {
        int ok = 1;
        if (!pos_ok) {
            atomicCAS(t.err, 0, ERR_POS);
            ok = 0;
        } else {
            int i = 0;
            for (; i < kGridPolls; ++i) {
                if (ld_acquire_gpu(a.sync) >= (unsigned)G) break;
                if (i > 64) __nanosleep(i > 65536 ? 1024 : 32);
            }
            if (i == kGridPolls) {
                atomicCAS(t.err, 0, ERR_GRID_SYNC);
                ok = 0;
            }
        }
        *flag = ok;
        if (TR) gv_stamp(a.trace, 2);
    }
    __syncthreads();
    float m_run = -INFINITY, l_run = 0.f, acc = 0.f;
    const bool pv_thread = tid < ng * hd;
    if (*flag) {
        const float* row = t.qkv;
        for (int i = tid; i < hd; i += nth) {
            qs[i] = __ldcg(row + (size_t)qh * hd + i);
            kn[i] = __ldcg(row + (size_t)t.n_head * hd + (size_t)kvh * hd + i);
            vn[i] = __ldcg(row + (size_t)(t.n_head + t.n_kv) * hd + (size_t)kvh * hd + i);
        }
        __syncthreads();
        if (TR && tid == 0) gv_stamp(a.trace, 5);
        for (int i = tid; i < hd; i += nth) {
            const int j = i % d2;
            if (i < d2) rope_pair(qs[j], qs[j + d2], cs[j], sn[j]);
            else rope_pair(kn[j], kn[j + d2], cs[j], sn[j]);
        }
        __syncthreads();
        if (storer)
            for (int i = tid; i < hd; i += nth) {
                kv_store(t.kc, (long long)(cache_off + (size_t)pos * hd + i), t.kv_type, kn[i]);
                kv_store(t.vc, (long long)(cache_off + (size_t)pos * hd + i), t.kv_type, vn[i]);
            }
        if (TR && tid == 0) gv_stamp(a.trace, 8);
        const float scale = 1.0f / sqrtf((float)hd);
        const int pg = tid / hd, pd = tid % hd;
        for (int t0 = s0; t0 < s1; t0 += tp) {
            const int np = min(s1, t0 + tp) - t0;
            const bool last = t0 + np == pos + 1;
            if (t0 != s0) {
                load_tile(ks, kst, hd, t.kc, (long long)(cache_off + (size_t)t0 * hd), last ? np - 1 : np, t.kv_type,
                          nth);
                load_tile(vs, hd, hd, t.vc, (long long)(cache_off + (size_t)t0 * hd), last ? np - 1 : np, t.kv_type,
                          nth);
            }
            if (last)
                for (int i = tid; i < hd; i += nth) {
                    // the new key/value enter at the stored precision, as later steps read them
                    ks[(size_t)(np - 1) * kst + i] = kv_round(kn[i], t.kv_type);
                    vs[(size_t)(np - 1) * hd + i] = kv_round(vn[i], t.kv_type);
                }
            __syncthreads();
            // scores: scale * q.k, one position per thread
            float sv = -INFINITY;
            if (tid < np) {
                const float4* kp = reinterpret_cast<const float4*>(ks + (size_t)tid * kst);
                const float4* q4 = reinterpret_cast<const float4*>(qs);
                float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
                for (int d = 0; d < hd / 4; ++d) {
                    const float4 k = kp[d], q = q4[d];
                    s0 = fmaf(q.x, k.x, s0);
                    s1 = fmaf(q.y, k.y, s1);
                    s2 = fmaf(q.z, k.z, s2);
                    s3 = fmaf(q.w, k.w, s3);
                }
                sv = scale * ((s0 + s1) + (s2 + s3));
            }
            if (TR && tid == 0 && t0 == s0) gv_stamp(a.trace, 9);
            float tm = warp_max(sv);
            if (lane == 0) red[warp] = tm;
            __syncthreads();
            tm = red[0];
            for (int w = 1; w < nw; ++w) tm = fmaxf(tm, red[w]);
            const float mnew = fmaxf(m_run, tm);
            float e = 0.f;
            if (tid < np) {
                e = expf(sv - mnew);
                sc[tid] = e;
            }
            e = warp_sum(e);
            if (lane == 0) red[32 + warp] = e;
            __syncthreads();
            float lt = 0.f;
            for (int w = 0; w < nw; ++w) lt += red[32 + w];
            if (TR && tid == 0 && t0 == s0) gv_stamp(a.trace, 7);
            const float alpha = expf(m_run - mnew);  // 0 on the first tile
            l_run = fmaf(l_run, alpha, lt);
            m_run = mnew;
            if (pv_thread) {
                float a0 = 0.f, a1 = 0.f;
                int p = pg;
                for (; p + ng < np; p += 2 * ng) {
                    a0 = fmaf(sc[p], vs[(size_t)p * hd + pd], a0);
                    a1 = fmaf(sc[p + ng], vs[(size_t)(p + ng) * hd + pd], a1);
                }
                if (p < np) a0 = fmaf(sc[p], vs[(size_t)p * hd + pd], a0);
                acc = fmaf(acc, alpha, a0 + a1);
            }
            __syncthreads();
        }
        if (TR && tid == 0) gv_stamp(a.trace, 6);
        if constexpr (!SPLIT) {
            if (pv_thread) pacc[tid] = acc;
            __syncthreads();
            for (int d = tid; d < hd; d += nth) {  // whole warps (hd is a multiple of 32)
                float o = 0.f;
                for (int g = 0; g < ng; ++g) o += pacc[g * hd + d];
                o = o / l_run;
                t.out[(size_t)qh * hd + d] = o;
                if (a.yplanes) {
                    const int pstride = q8_plane_stride(t.n_head * hd);
                    q8_block_planes_warp(o, (qh * hd + d) >> 5, a.yplanes, pstride,
                                         reinterpret_cast<float*>(a.yplanes + 3 * pstride));
                }
            }
        }
    }
    if constexpr (SPLIT) {
        if (pv_thread) pacc[tid] = acc;
        __syncthreads();
        fused_attn_split_out(t.part, t.n_split, a.aticket, t.out, a.yplanes, t.n_head, qh, sp, nsf, hd, ng, pacc, ks,
                             flag, m_run, l_run);
    }
    // leave; the last attention CTA out clears the counters for this layer's next step
    __syncthreads();
    if (tid == 0) {
        if (TR) gv_stamp(a.trace, 3);
        const unsigned d = atomicAdd(a.sync + 1, 1u);
        if (d == (unsigned)a.attn_ctas - 1) {
            a.sync[0] = 0u;
            a.sync[1] = 0u;
        }
        if (TR) gv_stamp(a.trace, 4);
    }
}

// INTQ: 0 fp32 dots, 1 Q8_0 integer path, 2 Q4_0 integer path, 3 Q6_K integer path, 4 the Q8_0
// integer path whose fused attention splits each head's positions over several CTAs (each its
// own function, so the Q8_0 kernel that every GEMV of a Q8_0 step runs carries no other code)
// TR: the launch-trace instantiation (stamps into a.trace; see GemvArgs::trace)
template <int MAXM, int INTQ, bool TR>
__global__ void __launch_bounds__(GV_THREADS, 2) tf_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int xl = xpad_len(a.K);
    const int xbytes = ((a.M * xl * 4) + 127) & ~127;
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* stages = smem + xbytes;
    float* red = reinterpret_cast<float*>(stages + (size_t)GV_STAGES * a.stage_bytes);  // [2][W][2][max(MAXM, 2)]
    double* redd = reinterpret_cast<double*>(red + gv_red_floats(MAXM));                   // [W][MAXM]
    float* pre = reinterpret_cast<float*>(redd + GV_WARPS * MAXM);                        // [MAXM][GV_PRE]
    uint64_t* full = reinterpret_cast<uint64_t*>(pre + MAXM * GV_PRE);
    uint64_t* empty = full + GV_STAGES;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + GV_STAGES);
    unsigned long long* ckey = reinterpret_cast<unsigned long long*>(empty + GV_STAGES + 1);

    // CTAs [0, attn_ctas) are the fused attention CTAs (first, so they are resident and load
    // their K/V rows while the GEMV CTAs work); GEMV CTA gb = blockIdx.x - attn_ctas
    const int G = (int)gridDim.x - a.attn_ctas;
    const int gb = (int)blockIdx.x - a.attn_ctas;
    if (TR && tid == 0) gv_stamp(a.trace, 0);
    if constexpr (INTQ == 1 || INTQ == 4) {  // the attention fuses into Q8_0 QKV launches only
        if (gb < 0) {
            fused_attention<INTQ == 4, TR>(a, smem, (size_t)xbytes + (size_t)GV_STAGES * a.stage_bytes, (int)blockIdx.x, G);
            return;
        }
    }
    const int al = a.align > 1 ? a.align : 1;  // n_items is a multiple of al
    const int i0 = al * (int)((long long)(a.n_items / al) * gb / G);
    const int i1 = al * (int)((long long)(a.n_items / al) * (gb + 1) / G);
    const int RI = GV_WARPS / a.KS;
    const int n_stages = (i1 - i0 + RI - 1) / RI;
    const bool prefetched = (i1 - i0) <= GV_PRE && (a.epi == EPI_RESID || (a.epi == EPI_STORE && a.bias));

    if (tid == 0) {
        for (int s = 0; s < GV_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GV_WARPS);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (tid < MAXM) ckey[tid] = 0ull;
    __syncthreads();
    pdl_trigger();

    if (warp == GV_WARPS) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int issued = 0;
            for (int s = 0; s < n_stages; ++s) {
                const int slot = s % GV_STAGES;
                if (s >= GV_STAGES &&
                    !mbar_wait(&empty[slot], ((s / GV_STAGES) - 1) & 1, a.err, ERR_WAIT_EMPTY, abort_flag))
                    break;
                const int si0 = i0 + s * RI, si1 = min(si0 + RI, i1);
                const long long r0 = (long long)si0 * a.P, r1 = (long long)si1 * a.P;
                // [ga, gb) is the 16-byte aligned body, moved by the bulk copy; the last
                // (end - gb) < 16 bytes are copied here with plain loads, so nothing outside
                // the stage's rows (beyond the aligned-down start) is ever read.
                const uintptr_t g = reinterpret_cast<uintptr_t>(a.W + r0 * a.rb);
                const uintptr_t end = g + (uintptr_t)((r1 - r0) * a.rb);
                const uintptr_t ga = g & ~(uintptr_t)15;
                const uintptr_t gb = end & ~(uintptr_t)15;
                uint8_t* dst = stages + (size_t)slot * a.stage_bytes;
                for (uintptr_t p = (gb > ga ? gb : ga); p < end; ++p) dst[p - ga] = *reinterpret_cast<const uint8_t*>(p);
                const uint32_t bytes = gb > ga ? (uint32_t)(gb - ga) : 0u;
                mbar_expect_tx(&full[slot], bytes);
                if (bytes) bulk_g2s(dst, reinterpret_cast<const void*>(ga), bytes, &full[slot]);
                ++issued;
            }
            // Copies in flight must land before the block exits (only pending on an abort).
            const int first = issued > GV_STAGES ? issued - GV_STAGES : 0;
            for (int s = first; s < issued; ++s) mbar_wait(&full[s % GV_STAGES], (s / GV_STAGES) & 1, nullptr, 0, nullptr);
        }
        return;
    }

    // ---------------- consumers: prologue ----------------
    const int nth = GV_WARPS * 32;
    // static operands first (they do not depend on the previous kernel): bias of this
    // CTA's rows and the RMSNorm weights of this thread's activation chunks
    if (prefetched && a.epi == EPI_STORE)
        for (int i = tid; i < i1 - i0; i += nth) pre[i] = a.bias[i0 + i];
    const int nq = a.K >> 2;  // float4 chunks per activation row
    float4 wn[GV_PRO_UNROLL];
    const bool norm_regs = (a.pro == PRO_RMSNORM || a.pro == PRO_EMBED_RMSNORM) && nq <= nth * GV_PRO_UNROLL;
    if (norm_regs) {
#pragma unroll
        for (int u = 0; u < GV_PRO_UNROLL; ++u) {
            const int c = tid + u * nth;
            wn[u] = c < nq ? reinterpret_cast<const float4*>(a.norm_w)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    if (TR && tid == 0) gv_stamp(a.trace, 5);
    pdl_wait();
    if (TR && tid == 0) gv_stamp(a.trace, 1);
    if (prefetched && a.epi == EPI_RESID)
        for (int i = tid; i < (i1 - i0) * a.M; i += nth) {
            const int m = i / (i1 - i0), r = i % (i1 - i0);
            pre[m * GV_PRE + r] = a.resid[(size_t)m * a.ldr + i0 + r];
        }
    // Q8_0 integer path (M == 1): the activation row stays in registers through the RMSNorm
    // and leaves as digit planes in the activation region (dots.cuh).
    constexpr bool use_int = INTQ != 0;
    constexpr bool q4 = INTQ == 2;
    constexpr bool q6 = INTQ == 3;  // Q6_K rows: the Q4_0 planes, 64-element units of super-blocks
    static_assert(!INTQ || MAXM == 1, "integer path is for one activation row");
    const int U = a.K / a.KS / 64;               // 64-element units per row segment
    const int prow = a.P == 2 ? lane >> 4 : 0;   // row of the item this lane works on
    const int pu = a.P == 2 ? lane & 15 : lane;  // unit within the segment
    const bool pact = pu < U;
    uint32_t pl[INTQ ? (q6 ? 48 : 51) : 1];
    float invA = 0.f, invB = 0.f;
    const uint32_t* q6sum = nullptr;  // Q6_K: this lane's 16-element digit sums (shared memory)
    if constexpr (INTQ) {
        if ((INTQ == 1 || INTQ == 4) && a.pro == PRO_PLANES) {
            // the previous kernel left the activation as planes: one coalesced copy into the
            // activation region (all loads in flight before the stores), then the lanes read
            // their units from shared memory as below
            const int pstride = q8_plane_stride(a.K);
            const int nw4 = q8_plane_bytes(a.K) / 4;
            const int n16 = nw4 / 4;
            const uint4* src = reinterpret_cast<const uint4*>(a.xplanes);
            uint4* dst = reinterpret_cast<uint4*>(xs);
            for (int base = tid; base < n16; base += nth * GV_PRO_UNROLL) {
                uint4 r[GV_PRO_UNROLL];
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u)
                    if (base + u * nth < n16) r[u] = __ldcg(src + base + u * nth);
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u)
                    if (base + u * nth < n16) dst[base + u * nth] = r[u];
            }
            for (int i = 4 * n16 + tid; i < nw4; i += nth)
                reinterpret_cast<uint32_t*>(xs)[i] = __ldcg(reinterpret_cast<const uint32_t*>(a.xplanes) + i);
            if (TR && tid == 0) gv_stamp(a.trace, 6);
            named_bar_compute();
            if (TR && tid == 0) gv_stamp(a.trace, 7);
            const uint8_t* planes = reinterpret_cast<const uint8_t*>(xs);
            const float* pinv = reinterpret_cast<const float*>(planes + 3 * pstride);
            const int unit = (warp % a.KS) * U + pu;
#pragma unroll
            for (int i = 0; i < 51; ++i) pl[i] = 0u;
            if (pact) {
                const uint32_t* pw = reinterpret_cast<const uint32_t*>(planes + (size_t)unit * 68);
#pragma unroll
                for (int i = 0; i < 17; ++i) {
                    pl[i] = pw[i];
                    pl[17 + i] = pw[pstride / 4 + i];
                    pl[34 + i] = pw[pstride / 2 + i];
                }
                invA = pinv[2 * unit];
                invB = pinv[2 * unit + 1];
            }
        } else {
            float4 v[GV_PRO_UNROLL];
            if (a.pro == PRO_EMBED_RMSNORM) {
                int tok = a.tokens[0];
                if (tok < 0 || tok >= a.n_vocab) {
                    if (tid == 0) atomicCAS(a.err, 0, ERR_BAD_TOKEN);
                    tok = 0;
                }
                embed_row(xs, a.embd, a.embd_type, a.embd_rb, a.K, tok, nth);
                named_bar_compute();
                if (gb == 0)
                    for (int e = tid; e < a.K; e += nth) a.x_out[e] = xs[xpad(e)];
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                    const int c = tid + u * nth;
                    v[u] = c < nq ? *reinterpret_cast<const float4*>(xs + xpad(4 * c)) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            } else {
                const float4* xg = reinterpret_cast<const float4*>(a.x);
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                    const int c = tid + u * nth;
                    v[u] = c < nq ? xg[c] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            if (a.pro != PRO_COPY) {
                // rmsnorm (src/layers.cpp:7-12), in the same order as the fp32 path below
                double ss = 0.0;
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                    if (tid + u * nth < nq) {
                        ss = fma((double)v[u].x, (double)v[u].x, ss);
                        ss = fma((double)v[u].y, (double)v[u].y, ss);
                        ss = fma((double)v[u].z, (double)v[u].z, ss);
                        ss = fma((double)v[u].w, (double)v[u].w, ss);
                    }
                }
                if (TR && tid == 0) gv_stamp_after(a.trace, 6, ss);
                ss = warp_sum_d(ss);
                if (lane == 0) redd[warp] = ss;
                named_bar_compute();
                if (TR && tid == 0) gv_stamp(a.trace, 7);
                double tot = 0.0;
                for (int w = 0; w < GV_WARPS; ++w) tot += redd[w];
                const float inv = 1.0f / sqrtf((float)(tot / a.K) + a.eps);
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                    const float4 wv = wn[u];
                    v[u].x = __fmul_rn(__fmul_rn(v[u].x, inv), wv.x);
                    v[u].y = __fmul_rn(__fmul_rn(v[u].y, inv), wv.y);
                    v[u].z = __fmul_rn(__fmul_rn(v[u].z, inv), wv.z);
                    v[u].w = __fmul_rn(__fmul_rn(v[u].w, inv), wv.w);
                }
            }
            // the planes overwrite the activation region, which only the embedding path read
            if (a.pro == PRO_EMBED_RMSNORM) named_bar_compute();
            uint8_t* planes = reinterpret_cast<uint8_t*>(xs);
            const int unit = (warp % a.KS) * U + pu;
            if constexpr (q6) {
                float* pinv = reinterpret_cast<float*>(planes + 3 * a.K);
                int* psum = reinterpret_cast<int*>(pinv + a.K / 32);
                q4_build_planes<GV_PRO_UNROLL, true>(v, a.K, nth, tid, planes, a.K, pinv, psum);
                named_bar_compute();
#pragma unroll
                for (int i = 0; i < 48; ++i) pl[i] = 0u;
                // unit (h, j) of super-block sbg: activation blocks A = 8 sbg + 4h + j, B = A + 2
                const int sbg = (warp % a.KS) * (a.K / a.KS / 256) + (pact ? pu >> 2 : 0);
                const int blkA = 8 * sbg + 4 * ((pu >> 1) & 1) + (pu & 1), blkB = blkA + 2;
                q6sum = reinterpret_cast<const uint32_t*>(psum) + 4 * blkA;
                if (pact) {
                    const uint32_t* pw = reinterpret_cast<const uint32_t*>(planes);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
#pragma unroll
                        for (int p = 0; p < 3; ++p) {
                            pl[16 * p + i] = pw[p * (a.K / 4) + 8 * blkA + i];
                            pl[16 * p + 8 + i] = pw[p * (a.K / 4) + 8 * blkB + i];
                        }
                    invA = pinv[blkA];
                    invB = pinv[blkB];
                }
            } else if constexpr (q4) {
                float* pinv = reinterpret_cast<float*>(planes + 3 * a.K);
                int* psum = reinterpret_cast<int*>(pinv + a.K / 32);
                q4_build_planes<GV_PRO_UNROLL>(v, a.K, nth, tid, planes, a.K, pinv, psum);
                named_bar_compute();
#pragma unroll
                for (int i = 0; i < 51; ++i) pl[i] = 0u;
                if (pact) {
                    const uint32_t* pw = reinterpret_cast<const uint32_t*>(planes) + 16 * unit;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        pl[i] = pw[i];
                        pl[16 + i] = pw[a.K / 4 + i];
                        pl[32 + i] = pw[a.K / 2 + i];
                    }
#pragma unroll
                    for (int p = 0; p < 3; ++p)
                        pl[48 + p] = ((uint32_t)psum[4 * (2 * unit) + p] & 0xFFFFu) |
                                     ((uint32_t)psum[4 * (2 * unit + 1) + p] << 16);
                    invA = pinv[2 * unit];
                    invB = pinv[2 * unit + 1];
                }
            } else {
            const int pstride = (int)((a.rb + 15) & ~15LL);
            float* pinv = reinterpret_cast<float*>(planes + 3 * pstride);
            q8_build_planes<GV_PRO_UNROLL>(v, a.K, nth, tid, planes, pstride, pinv);
            named_bar_compute();
#pragma unroll
            for (int i = 0; i < 51; ++i) pl[i] = 0u;
            if (pact) {
                const uint32_t* pw = reinterpret_cast<const uint32_t*>(planes + (size_t)unit * 68);
#pragma unroll
                for (int i = 0; i < 17; ++i) {
                    pl[i] = pw[i];
                    pl[17 + i] = pw[pstride / 4 + i];
                    pl[34 + i] = pw[pstride / 2 + i];
                }
                invA = pinv[2 * unit];
                invB = pinv[2 * unit + 1];
            }
            }
        }
    }
    for (int m = 0; m < a.M && !use_int; ++m) {
        float* xm = xs + m * xl;
        if (a.pro == PRO_EMBED_RMSNORM) {
            int tok = a.tokens[m];
            if (tok < 0 || tok >= a.n_vocab) {
                if (tid == 0) atomicCAS(a.err, 0, ERR_BAD_TOKEN);
                tok = 0;
            }
            embed_row(xm, a.embd, a.embd_type, a.embd_rb, a.K, tok, GV_WARPS * 32);
        } else {
            // all loads of a row issued before any store: one memory round trip
            const float4* xg = reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx);
            for (int base = tid; base < nq; base += nth * GV_PRO_UNROLL) {
                float4 v[GV_PRO_UNROLL];
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                    const int c = base + u * nth;
                    if (c < nq) v[u] = xg[c];
                }
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                    const int c = base + u * nth;
                    if (c < nq) *reinterpret_cast<float4*>(xm + xpad(4 * c)) = v[u];
                }
            }
        }
    }
    if (!use_int) named_bar_compute();
    if (!use_int && a.pro == PRO_EMBED_RMSNORM && gb == 0)
        for (int m = 0; m < a.M; ++m)
            for (int e = tid; e < a.K; e += nth) a.x_out[(size_t)m * a.ldx + e] = xs[m * xl + xpad(e)];
    if (!use_int && a.pro != PRO_COPY) {
        // rmsnorm (src/layers.cpp:7-12): sum of squares in double, inv in float,
        // out = (x * inv) * w.
        for (int m = 0; m < a.M; ++m) {
            const float* xm = xs + m * xl;
            double ss = 0.0;
            for (int c = tid; c < nq; c += nth) {
                const float4 v = *reinterpret_cast<const float4*>(xm + xpad(4 * c));
                ss = fma((double)v.x, (double)v.x, ss);
                ss = fma((double)v.y, (double)v.y, ss);
                ss = fma((double)v.z, (double)v.z, ss);
                ss = fma((double)v.w, (double)v.w, ss);
            }
            ss = warp_sum_d(ss);
            if (lane == 0) redd[warp * MAXM + m] = ss;
        }
        named_bar_compute();
        for (int m = 0; m < a.M; ++m) {
            double ss = 0.0;
            for (int w = 0; w < GV_WARPS; ++w) ss += redd[w * MAXM + m];
            const float inv = 1.0f / sqrtf((float)(ss / a.K) + a.eps);
            float* xm = xs + m * xl;
            if (norm_regs) {
#pragma unroll
                for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                    const int c = tid + u * nth;
                    if (c < nq) {
                        float4* p = reinterpret_cast<float4*>(xm + xpad(4 * c));
                        float4 v = *p;
                        v.x = __fmul_rn(__fmul_rn(v.x, inv), wn[u].x);
                        v.y = __fmul_rn(__fmul_rn(v.y, inv), wn[u].y);
                        v.z = __fmul_rn(__fmul_rn(v.z, inv), wn[u].z);
                        v.w = __fmul_rn(__fmul_rn(v.w, inv), wn[u].w);
                        *p = v;
                    }
                }
            } else {
                for (int e = tid; e < a.K; e += nth) xm[xpad(e)] = __fmul_rn(__fmul_rn(xm[xpad(e)], inv), a.norm_w[e]);
            }
        }
    }
    if (!use_int) named_bar_compute();

    // ---------------- consumers: main loop ----------------
    if (TR && tid == 0) gv_stamp(a.trace, 2);
    const int kseg = a.K / a.KS;
    const int my_item = warp / a.KS, my_ks = warp % a.KS;
    unsigned long long best[MAXM];
#pragma unroll
    for (int m = 0; m < MAXM; ++m) best[m] = 0ull;

    if constexpr (INTQ) {
        // Two stages per iteration: each warp dots its item of stage s and of stage s + 1 (two
        // independent dp4a chains), one shuffle tree reduces both, KS > 1 partials meet after
        // one named barrier, and the two items' epilogues run in parallel in two lanes.
        const int P = a.P, KS = a.KS;
        constexpr int ubytes = q4 ? 36 : 68;  // bytes of a 64-element unit (Q4_0 / Q8_0)
        // Q6_K: the lane's unit is (h, j) of super-block my_ks * U / 4 + pu / 4 of its row
        const int lane_off = (my_item * P + prow) * (int)a.rb +
                             (q6 ? (my_ks * (U / 4) + (pact ? pu >> 2 : 0)) * 210
                                 : (my_ks * U + (pact ? pu : 0)) * ubytes);
        const int q6h = (pu >> 1) & 1, q6j = pu & 1;
        const uint32_t q6sel = (lane_off & 2) ? 0x5432u : 0x3210u;
        const bool lane_ok = pact && prow < P;
        // after the reduction: lanes [0, 16) hold item 0 and [16, 32) item 1 (P == 1); for
        // P == 2 lanes [0, 8) / [8, 16) the first row (gate) of items 0 / 1, [16, 24) / [24, 32)
        // the second row (up)
        const int rsel = P == 1 ? (lane >> 4) & 1 : (lane >> 3) & 1;
        const bool leader = (lane & (P == 1 ? 15 : 7)) == 0;
        const bool first_row = P == 1 || lane < 16;
        const long long step_bytes = (long long)RI * P * a.rb;
        for (int s = 0, it = 0; s < n_stages; s += 2, ++it) {
            const bool two = s + 1 < n_stages;
            const int slot0 = s % GV_STAGES, slot1 = (s + 1) % GV_STAGES;
            bool ok = mbar_wait(&full[slot0], (s / GV_STAGES) & 1, a.err, ERR_WAIT_FULL, abort_flag);
            if (two && ok) ok = mbar_wait(&full[slot1], ((s + 1) / GV_STAGES) & 1, a.err, ERR_WAIT_FULL, abort_flag);
            const int item0 = i0 + s * RI + my_item, item1 = item0 + RI;
            const uintptr_t g0 = reinterpret_cast<uintptr_t>(a.W) + (uintptr_t)((long long)s * step_bytes +
                                                                               (long long)i0 * P * a.rb);
            const uintptr_t g1 = g0 + (uintptr_t)step_bytes;
            // both dots run unconditionally (a stale or partly filled slot is still inside the
            // stage buffer); invalid results are selected away, never multiplied
            const uint32_t* wp0 =
                reinterpret_cast<const uint32_t*>(stages + (size_t)slot0 * a.stage_bytes + (g0 & 15) + lane_off);
            const uint32_t* wp1 =
                reinterpret_cast<const uint32_t*>(stages + (size_t)slot1 * a.stage_bytes + (g1 & 15) + lane_off);
            float d0, d1;
            if constexpr (q6) {
                d0 = unit_dot_q6k_int(reinterpret_cast<const uint8_t*>(wp0), q6h, q6j, q6sel, pl, q6sum, invA, invB);
                d1 = unit_dot_q6k_int(reinterpret_cast<const uint8_t*>(wp1), q6h, q6j, q6sel, pl, q6sum, invA, invB);
            } else if constexpr (q4) {
                d0 = unit_dot_q4_int(wp0, pl, invA, invB);
                d1 = unit_dot_q4_int(wp1, pl, invA, invB);
            } else {
                d0 = unit_dot_q8_int(wp0, pl, invA, invB);
                d1 = unit_dot_q8_int(wp1, pl, invA, invB);
            }
            const bool ok0 = ok && item0 < i1, ok1 = ok && two && item1 < i1;
            const float v0 = (ok0 && lane_ok) ? d0 : 0.f;
            const float v1 = (ok1 && lane_ok) ? d1 : 0.f;
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[slot0]);
                if (two) mbar_arrive(&empty[slot1]);
            }
            const int hx = P == 1 ? 16 : 8;
            const bool hi = (lane & hx) != 0;
            float keep = hi ? v1 : v0;
            keep += __shfl_xor_sync(0xffffffffu, hi ? v0 : v1, hx);
            if (P == 1) keep += __shfl_xor_sync(0xffffffffu, keep, 8);
            keep += __shfl_xor_sync(0xffffffffu, keep, 4);
            keep += __shfl_xor_sync(0xffffffffu, keep, 2);
            keep += __shfl_xor_sync(0xffffffffu, keep, 1);
            bool mine = true;
            if (KS > 1) {
                float* rb = red + ((it & 1) * GV_WARPS + warp) * 4;
                if (leader) rb[rsel * 2 + (first_row ? 0 : 1)] = keep;
                named_bar_compute();
                mine = my_ks == 0;
                if (mine && leader) {
                    float v = 0.f;
                    for (int k = 0; k < KS; ++k) v += red[((it & 1) * GV_WARPS + warp + k) * 4 + rsel * 2 + (first_row ? 0 : 1)];
                    keep = v;
                }
            }
            const float other = __shfl_xor_sync(0xffffffffu, keep, 16);  // P == 2: the up row's sum
            const bool okr = rsel ? ok1 : ok0;
            if (mine && leader && first_row && okr) {
                const int row = rsel ? item1 : item0;
                if (a.epi == EPI_STORE) {
                    const float b = a.bias ? (prefetched ? pre[row - i0] : a.bias[row]) : 0.f;
                    a.y[row] = keep + b;
                } else if (a.epi == EPI_RESID) {
                    const float r = prefetched ? pre[row - i0] : a.resid[row];
                    a.resid[row] = r + keep;
                } else if (a.epi == EPI_SWIGLU) {
                    const float hv = __fmul_rn(__fdiv_rn(keep, 1.0f + expf(-keep)), other);
                    a.y[row] = hv;
                    if (a.yplanes) pre[row - i0] = hv;
                } else {  // EPI_ARGMAX
                    a.y[row] = keep;
                    const unsigned long long k = argmax_key(keep, (uint32_t)(row + a.row_base));
                    best[0] = k > best[0] ? k : best[0];
                }
            }
        }
    }
    for (int s = 0; s < n_stages && !INTQ; ++s) {
        const int slot = s % GV_STAGES;
        const bool ok = mbar_wait(&full[slot], (s / GV_STAGES) & 1, a.err, ERR_WAIT_FULL, abort_flag);
        const int si0 = i0 + s * RI, si1 = min(si0 + RI, i1);
        const int item = si0 + my_item;
        float acc0[MAXM], acc1[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc0[m] = acc1[m] = 0.f;
        if (ok && item < si1) {
            const uintptr_t g = reinterpret_cast<uintptr_t>(a.W + (long long)si0 * a.P * a.rb);
            const uint8_t* sb = stages + (size_t)slot * a.stage_bytes + (g & 15);
            const uint8_t* ib = sb + (long long)my_item * a.P * a.rb;
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                if (p < a.P) {
                    const uint8_t* rowp = ib + (long long)p * a.rb;
                    float part[MAXM];
#pragma unroll
                    for (int m = 0; m < MAXM; ++m) part[m] = 0.f;
                    if (a.fast) {
                        const uint8_t* seg = rowp + (long long)my_ks * (kseg / 64) * 68;
                        dot_q8_fast<MAXM>(seg, kseg / 64, xs + (size_t)(my_ks * kseg / 64) * 68, xl, a.M, lane, part);
                    } else {
                        const long long seg_off = row_bytes(a.wtype, (long long)my_ks * kseg);
                        dot_generic<MAXM>(a.wtype, rowp + seg_off, my_ks * kseg, kseg, xs, xl, a.M, lane, part);
                    }
#pragma unroll
                    for (int m = 0; m < MAXM; ++m) {
                        const float v = warp_sum(part[m]);
                        if (p == 0) acc0[m] = v;
                        else acc1[m] = v;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        bool have = ok && item < si1;
        if (a.KS > 1) {
            float* rb = red + ((s & 1) * GV_WARPS + warp) * 2 * MAXM;
            if (lane == 0 && have)
#pragma unroll
                for (int m = 0; m < MAXM; ++m) {
                    rb[m] = acc0[m];
                    rb[MAXM + m] = acc1[m];
                }
            named_bar_compute();
            have = have && my_ks == 0;
            if (have && lane == 0) {
#pragma unroll
                for (int m = 0; m < MAXM; ++m) {
                    float v0 = 0.f, v1 = 0.f;
                    for (int k = 0; k < a.KS; ++k) {
                        const float* q = red + ((s & 1) * GV_WARPS + warp + k) * 2 * MAXM;
                        v0 += q[m];
                        v1 += q[MAXM + m];
                    }
                    acc0[m] = v0;
                    acc1[m] = v1;
                }
            }
        }
        if (have && lane == 0) {
            const int row = item;
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m >= a.M) break;
                if (a.epi == EPI_STORE) {
                    const float b = a.bias ? (prefetched ? pre[row - i0] : a.bias[row]) : 0.f;
                    a.y[(size_t)m * a.ldy + row] = acc0[m] + b;
                } else if (a.epi == EPI_RESID) {
                    const float r = prefetched ? pre[m * GV_PRE + row - i0] : a.resid[(size_t)m * a.ldr + row];
                    a.resid[(size_t)m * a.ldr + row] = r + acc0[m];
                } else if (a.epi == EPI_SWIGLU) {
                    const float g = acc0[m], u = acc1[m];
                    a.y[(size_t)m * a.ldy + row] = __fmul_rn(__fdiv_rn(g, 1.0f + expf(-g)), u);
                } else {  // EPI_ARGMAX
                    const float v = acc0[m];
                    a.y[(size_t)m * a.ldy + row] = v;
                    const unsigned long long k = argmax_key(v, (uint32_t)(row + a.row_base));
                    best[m] = k > best[m] ? k : best[m];
                }
            }
        }
    }

    if (TR && tid == 0) gv_stamp(a.trace, 3);
    if (a.epi == EPI_ARGMAX)  // the lanes that ran argmax epilogues
        for (int m = 0; m < a.M; ++m)
            if (best[m]) atomicMax(&ckey[m], best[m]);
    // with fused attention the attention CTAs read this CTA's rows: publish them
    if (a.attn_ctas && lane == 0) __threadfence();
    named_bar_compute();
    if (tid == 0 && a.attn_ctas) red_release_gpu_add(a.sync, 1u);
    if (INTQ && a.epi == EPI_SWIGLU && a.yplanes) {
        // this CTA's SwiGLU rows (whole 32-row blocks, in `pre`) as planes for the next kernel
        const int pstride = q8_plane_stride(a.n_items);
        float* inv = reinterpret_cast<float*>(a.yplanes + 3 * pstride);
        for (int b = warp; b < (i1 - i0) / 32; b += GV_WARPS)
            q8_block_planes_warp(pre[b * 32 + lane], i0 / 32 + b, a.yplanes, pstride, inv);
    }
    if (tid == 0) {
        if (a.epi == EPI_ARGMAX)
            for (int m = 0; m < a.M; ++m) atomicMax(&a.keys[m], ckey[m]);
        if (a.fin != FIN_NONE) {
            __threadfence();
            const unsigned t = atomicAdd(&a.ctl->done, 1u);
            if (t == (unsigned)G - 1) {
                __threadfence();
                const int gs = atomicAdd(&a.ctl->gen_step, 0);
                for (int m = 0; m < a.M; ++m) {
                    if (a.fin == FIN_ARGMAX) {
                        const unsigned long long k = atomicExch(&a.keys[m], 0ull);
                        const int tok = (int)key_index(k);
                        a.tok_next[m] = tok;
                        if (a.hist && gs < a.ctl->hist_cap) a.hist[(size_t)gs * a.M + m] = tok;
                    } else if (a.fin == FIN_KEY) {
                        const unsigned long long k = atomicExch(&a.keys[m], 0ull);
                        a.key_out[m] = (long long)(k ^ 0x8000000000000000ull);
                    }
                    a.pos[a.slots[m]] += 1;
                }
                a.ctl->gen_step = gs + 1;
                atomicExch(&a.ctl->done, 0u);
                __threadfence();
            }
        }
        if (TR) gv_stamp(a.trace, 4);
    }
}

// Vocab-split lm_head: the token of the next step from the key reduced across GPUs (max of
// the flipped keys; the reference's first-index tie rule survives the reduction because the
// key orders equal logits by descending 0xFFFFFFFF - index), and its history entry.
__global__ void tf_key_apply_kernel(const long long* key, int* tok, int* hist, const StepCtl* ctl) {
    const unsigned long long k = (unsigned long long)key[0] ^ 0x8000000000000000ull;
    const int t = (int)key_index(k);
    tok[0] = t;
    const int gs = ctl->gen_step - 1;
    if (hist && gs >= 0 && gs < ctl->hist_cap) hist[gs] = t;
}

cudaError_t key_apply_launch(const long long* key, int* tok, int* hist, const StepCtl* ctl, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tf_key_apply_kernel, key, tok, hist, ctl);
}

// ---- host side --------------------------------------------------------------------------

// Positions per tile of the attention fused into an integer-path QKV launch `a` (M == 1): the
// same arithmetic as fused_attention's tile size over the shared memory it is given.
int fused_attn_tile(const GemvArgs& a, int hd) {
    const size_t xbytes = ((size_t)xpad_len(a.K) * 4 + 127) & ~(size_t)127;
    const size_t avail = xbytes + (size_t)GV_STAGES * a.stage_bytes;
    const int ng = std::min(8, GV_THREADS / hd);
    const int fixed = 4 * hd + 68 + ng * hd;
    int tp = (int)((avail / 4 - fixed) / (size_t)(1 + (hd + 4) + hd));
    tp = (tp > 256 ? 256 : tp) & ~3;
    return tp > 0 ? tp : 0;
}

size_t gemv_smem_bytes(int M, int K, int stage_bytes, int maxm) {
    const size_t xbytes = ((size_t)M * xpad_len(K) * 4 + 127) & ~(size_t)127;
    return xbytes + (size_t)GV_STAGES * stage_bytes + (size_t)gv_red_floats(maxm) * 4 + GV_WARPS * maxm * 8 +
           (size_t)maxm * GV_PRE * 4 + 2 * GV_STAGES * 8 + 8 + maxm * 8;
}

static int pick_maxm(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

// Choose the k-split and stage size for a weight shape (see GemvArgs).
// k-split and stage size for a weight shape and `warps` consumer warps: the smallest split
// whose stage (warps/KS items) fits `budget` bytes.
// The exact-integer Q8_0 path is the default; TFB200_Q8_INT=0 selects the fp32 path (both
// are exact-product paths of the same sums; the switch exists for measurement).
static bool q8_int_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_Q8_INT");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

// Smallest Q4_0 matrix on the integer path (TFB200_Q4_INT_MIN_MB overrides the 32 MB default).
static long long q4_int_min_bytes() {
    static long long v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_Q4_INT_MIN_MB");
        v = e ? (long long)atoi(e) << 20 : 32ll << 20;
        if (v < 0) v = 0;
    }
    return v;
}

// TFB200_Q6_INT=0 keeps Q6_K rows on the fp32 dequant path (for measurement)
static bool q6_int_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_Q6_INT");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

void gemv_plan_w(GemvArgs& a, int warps, int budget) {
    const int be = blk_elems(a.wtype) == 1 ? 32 : blk_elems(a.wtype);
    const bool q8fast = (a.wtype == T_Q8_0) && (a.K % 64 == 0);
    // Q4_0 takes the integer path only for large matrices: its plane build (with block digit
    // sums) lengthens the prologue, which the small matrices of a decode step cannot hide
    // (cfg2 decode 476 tok/s with it on every layer, 509 without; the 128256 x 2048 lm_head
    // shape 3263 GB/s with it, 840 without)
    const bool q4int = (a.wtype == T_Q4_0) && (a.K % 64 == 0) && a.M == 1 &&
                       (long long)a.n_items * a.P * a.rb >= q4_int_min_bytes();
    // Q6_K rows (cfg2's 215 MB lm_head) take the integer path at any size: the fp32 dequant
    // of a 256-element super-block is several times the plane build's cost.  K % 512 keeps the
    // rows (210 bytes per super-block) 4-byte aligned; single-row items only (Q6_K gate/up
    // pairs stay on the fp32 path).
    const bool q6int = (a.wtype == T_Q6_K) && (a.K % 512 == 0) && a.M == 1 && a.P == 1;
    int best = -1;
    for (int ks = 1; ks <= warps; ks <<= 1) {
        if (a.K % ks) continue;
        const int seg = a.K / ks;
        if (seg % be) continue;
        if ((q8fast || q4int) && seg % 64) continue;
        best = ks;
        const long long payload = (long long)(warps / ks) * a.P * a.rb;
        if (payload <= budget) break;
    }
    if (best < 0) best = 1;
    a.KS = best;
    // the fast path reads 4-byte words: rows must start 4-byte aligned
    a.fast = q8fast && ((a.K / best) % 64 == 0) && ((reinterpret_cast<uintptr_t>(a.W) & 3) == 0);
    // integer path: one activation row, every lane of a warp on one 64-element unit of one of
    // the item's P rows, the whole row prologue held in registers (K <= 8192)
    const int units = a.K / best / 64;
    const bool w4 = (reinterpret_cast<uintptr_t>(a.W) & 3) == 0;
    const bool q4ok = q4int && (a.K / best) % 64 == 0 && w4;
    const bool q6ok = q6int && (a.K / best) % 256 == 0 && w4 && q6_int_enabled();
    a.intq = (a.fast || q4ok || q6ok) && a.M == 1 && units * a.P <= 32 &&
             a.K <= GV_WARPS * 32 * 4 * GV_PRO_UNROLL && q8_int_enabled();
    a.q4 = a.intq && a.wtype == T_Q4_0;
    a.q6 = a.intq && a.wtype == T_Q6_K;
    const long long payload = (long long)(warps / best) * a.P * a.rb;
    a.stage_bytes = (int)((payload + 32 + 15) & ~15LL);
}
void gemv_plan(GemvArgs& a) { gemv_plan_w(a, GV_WARPS, GV_STAGE_BUDGET); }

int gemv_max_rows(int K) {
    // activation rows whose padded copies fit next to the stages
    const size_t per = (size_t)xpad_len(K) * 4;
    int m = (int)((96 * 1024) / per);
    return m < 1 ? 1 : (m > GV_MAXM ? GV_MAXM : m);
}

template <int MAXM, int INTQ, bool TR = false>
static cudaError_t init_one() {
    cudaError_t e =
        cudaFuncSetAttribute(tf_gemv_kernel<MAXM, INTQ, TR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    // every kernel of the step asks for the same (maximal) shared-memory carve-out, so the
    // SMs never have to drain to re-partition L1 / shared memory between kernels
    return cudaFuncSetAttribute(tf_gemv_kernel<MAXM, INTQ, TR>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
}

cudaError_t gemv_init_attrs() {
    cudaError_t e;
    if ((e = init_one<1, 0>())) return e;
    if ((e = init_one<1, 1>())) return e;
    if ((e = init_one<1, 2>())) return e;
    if ((e = init_one<1, 3>())) return e;
    if ((e = init_one<1, 4>())) return e;
    if ((e = init_one<1, 1, true>())) return e;
    if ((e = init_one<1, 4, true>())) return e;
    if ((e = init_one<2, 0>())) return e;
    if ((e = init_one<4, 0>())) return e;
    return init_one<8, 0>();
}

template <int MAXM, int INTQ, bool TR = false>
static cudaError_t launch_t(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
    const size_t smem = gemv_smem_bytes(a.M, a.K, a.stage_bytes, MAXM);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tf_gemv_kernel<MAXM, INTQ, TR>, a);
}

cudaError_t gemv_launch(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
    switch (pick_maxm(a.M)) {
        case 1:
            if (!a.intq) return launch_t<1, 0>(a, grid, st, pdl);
            if (a.q6) return launch_t<1, 3>(a, grid, st, pdl);
            if (a.q4) return launch_t<1, 2>(a, grid, st, pdl);
            if (a.trace)  // the launch-trace instantiations (Q8_0 integer path only)
                return a.attn_nsf > 1 ? launch_t<1, 4, true>(a, grid, st, pdl) : launch_t<1, 1, true>(a, grid, st, pdl);
            return a.attn_nsf > 1 ? launch_t<1, 4>(a, grid, st, pdl) : launch_t<1, 1>(a, grid, st, pdl);
        case 2: return launch_t<2, 0>(a, grid, st, pdl);
        case 4: return launch_t<4, 0>(a, grid, st, pdl);
        default: return launch_t<8, 0>(a, grid, st, pdl);
    }
}

// CTAs per SM for the GEMV grids (TFB200_GEMV_CPS, 1 or 2, default 2).  Two half-size CTAs
// per SM measured faster for batch-1 decode (1137 vs 814 tok/s on cfg0): while one CTA of a
// kernel drains its last stages, the other slot takes the next kernel's CTA, which starts
// its weight prefetch under programmatic dependent launch.
static int gemv_ctas_per_sm() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("TFB200_GEMV_CPS");
        v = e ? atoi(e) : 2;
        if (v < 1) v = 1;
        if (v > 2) v = 2;
    }
    return v;
}

int gemv_slots(int num_sms) { return num_sms * gemv_ctas_per_sm(); }

int gemv_grid(const GemvArgs& a, int num_sms) {
    const int RI = GV_WARPS / a.KS;
    const int stages = (a.n_items + RI - 1) / RI;
    const int cap = num_sms * gemv_ctas_per_sm();
    return stages < cap ? (stages > 0 ? stages : 1) : cap;
}

}  // namespace tfb
