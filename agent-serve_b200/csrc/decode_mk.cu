// Persistent decode megakernel for batch-1 decode / prefill / greedy generation.
//
// Why: a decode step is ~5 dependent phases per layer (QKV, attention, wo, gate/up, down)
// plus the lm_head, each an all-to-all dependency on the previous phase's output.  As
// separate kernels every boundary costs launch + drain + a memory round trip while HBM
// idles.  Here one cooperative launch (one CTA per SM, all co-resident) runs every phase of
// every step; phases are separated by a grid barrier, and the weight stream never stops:
//
//   weight stream   thread 0 walks the whole schedule (all steps, all GEMV phases, this
//                   CTA's rows) and keeps a ring of shared-memory slots full with 1-D bulk
//                   copies (TMA engine).  It issues without ever blocking: whenever it waits
//                   (for a slot it consumes, at a grid barrier, between attention sub-steps)
//                   it tops the ring up, so the next phase's weights are already in shared
//                   memory when the barrier resolves.  There is no separate producer warp, so
//                   the 8 warps of a CTA (two per scheduler) may hold up to 255 registers,
//                   which the register-resident activations of the row dot need.
//   consumer warps  per phase: wait at the barrier, stage the input activation (RMSNorm /
//                   embedding fused), consume this CTA's ring slots (2 rows per warp per
//                   slot), apply the epilogue, arrive at the barrier.
//   attention       on CTAs 0..n_kv-1 (one kv head each): RoPE with the host cos/sin table,
//                   KV store, online-softmax attention over [window start, pos].
//
// Every wait is bounded (mbarrier waits and the grid barrier); on a timeout the CTA records
// an error code, raises its abort flag, lets its in-flight copies land and exits.
// Cross-CTA data (residual, q/k/v, attention output, FFN activations, greedy keys) is read
// with ld.global.cg so no stale L1 line is ever used.
#include "decode_mk.cuh"
#include "dots.cuh"

namespace tfb {


__device__ __forceinline__ void cbar() { asm volatile("bar.sync 2, %0;" ::"n"(MK_THREADS) : "memory"); }
__device__ __forceinline__ void kbar() { asm volatile("bar.sync 1, %0;" ::"n"(MK_THREADS) : "memory"); }

// Non-blocking test of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// ---- the weight stream (thread 0 only) --------------------------------------------------
// Cursor over this CTA's stages of every GEMV phase of every step, in consumption order.
struct MkProd {
    int s, p, si0, i1;  // current stage: step, phase, first item, end item of the phase
    int issued;         // stages issued so far (ring position)
    int done;           // the whole schedule is issued
};

struct MkCtx {
    const MkArgs* a;
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    volatile int* abort_flag;
    MkProd* pr;
    int cta, G;
};

// Move the cursor to the first stage at or after (s, p) that has work for this CTA.
__device__ void prod_seek(const MkCtx& c, int s, int p) {
    const MkArgs& a = *c.a;
    MkProd* pr = c.pr;
    for (; s < a.n_steps; ++s, p = 0) {
        const int nph = s >= a.first_head ? a.n_ph : a.n_ph - 1;
        for (; p < nph; ++p) {
            const MkPhase& P = a.ph[p];
            if (P.kind != PH_GEMV) continue;
            const int i0 = (int)((long long)P.n_items * c.cta / c.G), i1 = (int)((long long)P.n_items * (c.cta + 1) / c.G);
            if (i0 >= i1) continue;
            pr->s = s;
            pr->p = p;
            pr->si0 = i0;
            pr->i1 = i1;
            return;
        }
    }
    pr->done = 1;
}

// Issue as many stages as there are free slots; never blocks.
__device__ void produce(const MkCtx& c) {
    MkProd* pr = c.pr;
    const MkArgs& a = *c.a;
    while (!pr->done && !*c.abort_flag) {
        const int slot = pr->issued % a.n_slots;
        if (pr->issued >= a.n_slots && !mbar_test(&c.empty[slot], ((pr->issued / a.n_slots) - 1) & 1)) return;
        const MkPhase& P = a.ph[pr->p];
        const int si1 = min(pr->si0 + P.ri, pr->i1);
        // [ga, gb) is the 16-byte aligned body, moved by the bulk copy; the last (end - gb)
        // < 16 bytes are copied here with plain loads, so nothing beyond the stage's rows (or
        // before its aligned-down start) is read.
        const uintptr_t g = reinterpret_cast<uintptr_t>(P.W + (long long)pr->si0 * P.P * P.rb);
        const uintptr_t end = g + (uintptr_t)((long long)(si1 - pr->si0) * P.P * P.rb);
        const uintptr_t ga = g & ~(uintptr_t)15, gb = end & ~(uintptr_t)15;
        uint8_t* dst = c.ring + (size_t)slot * a.slot_bytes;
        for (uintptr_t q = (gb > ga ? gb : ga); q < end; ++q) dst[q - ga] = *reinterpret_cast<const uint8_t*>(q);
        const uint32_t bytes = gb > ga ? (uint32_t)(gb - ga) : 0u;
        mbar_expect_tx(&c.full[slot], bytes);
        if (bytes) bulk_g2s(dst, reinterpret_cast<const void*>(ga), bytes, &c.full[slot]);
        ++pr->issued;
        pr->si0 = si1;
        if (pr->si0 >= pr->i1) prod_seek(c, pr->s, pr->p + 1);
    }
}

// Wait for ring slot `consumed` (all threads); thread 0 keeps the stream going meanwhile.
__device__ __forceinline__ bool wait_slot(const MkCtx& c, int consumed, int* err) {
    const int n = c.a->n_slots;
    uint64_t* bar = &c.full[consumed % n];
    const uint32_t par = (consumed / n) & 1;
    if (threadIdx.x == 0) {
        int i = 0;
        for (; i < kWaitPolls; ++i) {
            produce(c);
            if (mbar_test(bar, par) || *c.abort_flag) break;
            if (i > (1 << 14)) __nanosleep(256);
        }
        if (i == kWaitPolls) {
            atomicCAS(err, 0, ERR_WAIT_FULL);
            *c.abort_flag = 1;
        }
    }
    __syncwarp();
    return mbar_wait(bar, par, err, ERR_WAIT_FULL, c.abort_flag);
}

// Grid barrier among all CTAs: arrive, then wait (bounded) until `target` arrivals are
// counted; thread 0 keeps the weight stream going while it spins.  Returns false on a
// timeout or an earlier abort.
__device__ bool grid_sync(const MkCtx& c, unsigned target, int* err, volatile int* sh_ok) {
    cbar();
    if (threadIdx.x == 0) {
        int ok = 1;
        if (*c.abort_flag) {
            ok = 0;
        } else {
            // release: this CTA's phase results are visible before its arrival is counted
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(c.a->bar) : "memory");
            int i = 0;
            for (; i < kGridPolls; ++i) {
                if (ld_acquire_gpu(c.a->bar) >= target) break;
                produce(c);
                if (i > 4096) __nanosleep(i > 65536 ? 1024 : 32);
            }
            if (i == kGridPolls) {
                atomicCAS(err, 0, ERR_GRID_SYNC);
                *c.abort_flag = 1;
                ok = 0;
            }
            __threadfence();
        }
        *sh_ok = ok;
    }
    cbar();
    return *sh_ok != 0;
}

// ---- attention ---------------------------------------------------------------------------

// NeoX rotate-half with the reference build's contraction (src/attention.cpp:31-41).
__device__ __forceinline__ void mk_rope_pair(float& a, float& b, float c, float s) {
    const float x0 = a, x1 = b;
    a = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
    b = __fmaf_rn(x0, s, __fmul_rn(x1, c));
}
__device__ __forceinline__ float mk_kv_round(float v, int t) {
    if (t == KV_F32) return v;
    if (t == KV_F16) return __half2float(__float2half_rn(v));
    return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ void mk_kv_store(void* base, size_t idx, int t, float v) {
    if (t == KV_F32) reinterpret_cast<float*>(base)[idx] = v;
    else if (t == KV_F16) reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
}

// Cached K or V rows [p0, p0+np) of one head into dst (row stride `stride` floats).
__device__ void mk_load_rows(float* dst, int stride, int hd, const void* base, size_t e0, int np, int kv_type) {
    const int tid = threadIdx.x;
    const int per_vec = kv_type == KV_F32 ? 4 : 8;
    const int nvec = np * hd / per_vec;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + e0 * (kv_type == KV_F32 ? 4 : 2));
    for (int v0 = tid; v0 < nvec; v0 += MK_THREADS * 4) {
        uint4 r[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int v = v0 + u * MK_THREADS;
            if (v < nvec) r[u] = __ldcg(src + v);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int v = v0 + u * MK_THREADS;
            if (v >= nvec) continue;
            const int e = v * per_vec;
            float* o = dst + (size_t)(e / hd) * stride + (e % hd);
            if (kv_type == KV_F32) {
                o[0] = __uint_as_float(r[u].x);
                o[1] = __uint_as_float(r[u].y);
                o[2] = __uint_as_float(r[u].z);
                o[3] = __uint_as_float(r[u].w);
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

struct MkShared {
    float qs[AT_MAX_REP_MK][AT_MAX_HD_MK];
    float kn[AT_MAX_HD_MK], vn[AT_MAX_HD_MK];
    float sc[AT_MAX_REP_MK][MK_MAX_TILE];
    float mx[AT_MAX_REP_MK], l[AT_MAX_REP_MK], alpha[AT_MAX_REP_MK];
    MkProd prod;
};

// Attention of kv head `kvh` for the token at `pos` (src/attention.cpp:55-80 with the RoPE
// and KV store of src/model.cpp:125-127), positions [ws, pos], online softmax over tiles.
__device__ __noinline__ void mk_attention(const MkCtx& c, int layer, int kvh, int pos, int ws, float* tile, int tp,
                                          MkShared& S) {
    const MkArgs& a = *c.a;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nth = MK_THREADS;
    const int hd = a.hd, d2 = hd / 2, n_rep = a.n_head / a.n_kv;
    const size_t esz = a.kv_type == KV_F32 ? 4 : 2;
    void* kc = static_cast<uint8_t*>(a.kc) + (size_t)layer * a.layer_elems * esz;
    void* vc = static_cast<uint8_t*>(a.vc) + (size_t)layer * a.layer_elems * esz;
    const size_t head_off = (size_t)a.slot * a.slot_elems + (size_t)kvh * a.cap * hd;
    const float* q = a.qkv + (size_t)kvh * n_rep * hd;
    for (int i = tid; i < n_rep * hd; i += nth) S.qs[i / hd][i % hd] = __ldcg(q + i);
    for (int i = tid; i < hd; i += nth) {
        S.kn[i] = __ldcg(a.qkv + (size_t)a.n_head * hd + (size_t)kvh * hd + i);
        S.vn[i] = __ldcg(a.qkv + (size_t)(a.n_head + a.n_kv) * hd + (size_t)kvh * hd + i);
    }
    if (tid == 0) produce(c);
    cbar();
    const float* cp = a.cosb + (size_t)pos * d2;
    const float* sp = a.sinb + (size_t)pos * d2;
    for (int i = tid; i < (n_rep + 1) * d2; i += nth) {
        const int h = i / d2, j = i % d2;
        if (h < n_rep) mk_rope_pair(S.qs[h][j], S.qs[h][j + d2], cp[j], sp[j]);
        else mk_rope_pair(S.kn[j], S.kn[j + d2], cp[j], sp[j]);
    }
    cbar();
    for (int i = tid; i < hd; i += nth) {
        mk_kv_store(kc, head_off + (size_t)pos * hd + i, a.kv_type, S.kn[i]);
        mk_kv_store(vc, head_off + (size_t)pos * hd + i, a.kv_type, S.vn[i]);
    }
    const float scale = 1.0f / sqrtf((float)hd);
    float* ks = tile;                           // [tp][hd + 1]
    float* vs = tile + (size_t)tp * (hd + 1);   // [tp][hd]
    constexpr int PER = (AT_MAX_REP_MK * AT_MAX_HD_MK + MK_THREADS - 1) / MK_THREADS;
    float acc[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) acc[k] = 0.f;
    if (tid < n_rep) {
        S.mx[tid] = -INFINITY;
        S.l[tid] = 0.f;
    }
    for (int t0 = ws; t0 <= pos; t0 += tp) {
        const int np = min(tp, pos + 1 - t0);
        const int np_cached = (t0 + np == pos + 1) ? np - 1 : np;
        mk_load_rows(ks, hd + 1, hd, kc, head_off + (size_t)t0 * hd, np_cached, a.kv_type);
        mk_load_rows(vs, hd, hd, vc, head_off + (size_t)t0 * hd, np_cached, a.kv_type);
        if (np_cached < np)
            for (int i = tid; i < hd; i += nth) {
                ks[(size_t)(np - 1) * (hd + 1) + i] = mk_kv_round(S.kn[i], a.kv_type);
                vs[(size_t)(np - 1) * hd + i] = mk_kv_round(S.vn[i], a.kv_type);
            }
        if (tid == 0) produce(c);
        cbar();
        for (int i = tid; i < n_rep * np; i += nth) {
            const int h = i / np, p = i % np;
            const float* kp = ks + (size_t)p * (hd + 1);
            float s0 = 0.f, s1 = 0.f;
            for (int d = 0; d < hd; d += 2) {
                s0 = fmaf(S.qs[h][d], kp[d], s0);
                s1 = fmaf(S.qs[h][d + 1], kp[d + 1], s1);
            }
            S.sc[h][p] = scale * (s0 + s1);
        }
        cbar();
        for (int h = warp; h < n_rep; h += MK_WARPS) {
            float mt = -INFINITY;
            for (int i = lane; i < np; i += 32) mt = fmaxf(mt, S.sc[h][i]);
            mt = warp_max(mt);
            const float mnew = fmaxf(S.mx[h], mt);
            float lt = 0.f;
            for (int i = lane; i < np; i += 32) {
                const float e = expf(S.sc[h][i] - mnew);
                S.sc[h][i] = e;
                lt += e;
            }
            lt = warp_sum(lt);
            if (lane == 0) {
                const float al = expf(S.mx[h] - mnew);  // 0 on the first tile
                S.alpha[h] = al;
                S.l[h] = fmaf(S.l[h], al, lt);
                S.mx[h] = mnew;
            }
        }
        cbar();
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int i = tid + k * nth;
            if (i < n_rep * hd) {
                const int h = i / hd, d = i % hd;
                float a0 = acc[k] * S.alpha[h], a1 = 0.f;
                int p = 0;
                for (; p + 1 < np; p += 2) {
                    a0 = fmaf(S.sc[h][p], vs[(size_t)p * hd + d], a0);
                    a1 = fmaf(S.sc[h][p + 1], vs[(size_t)(p + 1) * hd + d], a1);
                }
                if (p < np) a0 = fmaf(S.sc[h][p], vs[(size_t)p * hd + d], a0);
                acc[k] = a0 + a1;
            }
        }
        if (tid == 0) produce(c);
        cbar();
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int i = tid + k * nth;
        if (i < n_rep * hd) {
            const int h = i / hd, d = i % hd;
            a.attn_out[(size_t)(kvh * n_rep + h) * hd + d] = acc[k] / S.l[h];
        }
    }
}

// ---- one GEMV phase's ring stages ---------------------------------------------------------
// This CTA's items [i0, i1): the row dots, the k-split combine and the epilogue.  Warp w takes
// segment ks = w % KS of the 2 rows of item group w / KS (two items when P == 1, one gate/up
// pair when P == 2).  Out of line so the hot loop gets the whole register budget (with REG
// the lane's 64 activations live in registers for the phase).
template <bool REG>
__device__ __noinline__ unsigned long long mk_gemv_stages(const MkCtx& c, const MkPhase& Pg, float* red,
                                                          const float* pre, const float* xs, int i0, int i1,
                                                          bool prefetched, int& consumed) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const MkArgs& a = *c.a;
    const int K = Pg.K, KS = Pg.KS, PP = Pg.P, ri = Pg.ri, epi = Pg.epi, wtype = Pg.wtype;
    const int fast = Pg.fast;
    const long long rb = Pg.rb;
    const uint8_t* W = Pg.W;
    float* const y = Pg.y;
    const float* const bias = Pg.bias;
    float* const resid = Pg.resid;
    const int n_slots = a.n_slots, slot_bytes = a.slot_bytes;
    int* const err = a.err;
    uint8_t* const ring = c.ring;
    uint64_t* const empty = c.empty;

    const int kseg = K / KS;
    const int ipw = 2 / PP;  // items per warp
    const int my_grp = warp / KS, my_ks = warp % KS;
    const int xl = xpad_len(K);
    float xr[REG ? 64 : 1];
    if constexpr (REG) {
        const float* xsrc = xs + (size_t)(my_ks * 32 + lane) * 68;
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(xsrc + j);
            xr[j] = v.x;
            xr[j + 1] = v.y;
            xr[j + 2] = v.z;
            xr[j + 3] = v.w;
        }
    }
    unsigned long long best = 0ull;
    int sidx = 0;
    for (int si0 = i0; si0 < i1; si0 += ri, ++sidx) {
        const int slot = consumed % n_slots;
        const bool ok = wait_slot(c, consumed, err);
        ++consumed;
        const int si1 = min(si0 + ri, i1);
        const int item0 = si0 + my_grp * ipw;            // first item of this warp
        const int nrows = min(2, (si1 - item0) * PP);    // valid rows of the group
        float v0 = 0.f, v1 = 0.f;
        if (ok && nrows > 0) {
            const uintptr_t g = reinterpret_cast<uintptr_t>(W + (long long)si0 * PP * rb);
            const uint8_t* r0 = ring + (size_t)slot * slot_bytes + (g & 15) + (long long)(my_grp * 2) * rb;
            const uint8_t* r1 = nrows > 1 ? r0 + rb : r0;  // a missing second row re-reads the first
            float p0 = 0.f, p1 = 0.f;
            if constexpr (REG) {
                const size_t off = (size_t)my_ks * 2176 + (size_t)lane * 68;
                unit_dot_q8_reg(reinterpret_cast<const uint32_t*>(r0 + off), xr, p0);
                unit_dot_q8_reg(reinterpret_cast<const uint32_t*>(r1 + off), xr, p1);
            } else {
                float a0[1] = {0.f}, a1[1] = {0.f};
                if (fast) {
                    const long long off = (long long)my_ks * (kseg / 64) * 68;
                    const float* xseg = xs + (size_t)(my_ks * kseg / 64) * 68;
                    dot_q8_fast<1>(r0 + off, kseg / 64, xseg, xl, 1, lane, a0);
                    dot_q8_fast<1>(r1 + off, kseg / 64, xseg, xl, 1, lane, a1);
                } else {
                    const long long off = row_bytes(wtype, (long long)my_ks * kseg);
                    dot_generic<1>(wtype, r0 + off, my_ks * kseg, kseg, xs, xl, 1, lane, a0);
                    dot_generic<1>(wtype, r1 + off, my_ks * kseg, kseg, xs, xl, 1, lane, a1);
                }
                p0 = a0[0];
                p1 = a1[0];
            }
            v0 = warp_sum(p0);
            v1 = warp_sum(p1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        bool have = ok && nrows > 0;
        if (KS > 1) {
            float* rbuf = red + ((sidx & 1) * MK_WARPS + warp) * 2;
            if (lane == 0 && have) {
                rbuf[0] = v0;
                rbuf[1] = v1;
            }
            kbar();
            have = have && my_ks == 0;
            if (have && lane == 0) {
                float s0 = 0.f, s1 = 0.f;
                for (int k = 0; k < KS; ++k) {
                    s0 += red[((sidx & 1) * MK_WARPS + warp + k) * 2];
                    s1 += red[((sidx & 1) * MK_WARPS + warp + k) * 2 + 1];
                }
                v0 = s0;
                v1 = s1;
            }
        }
        if (have && lane == 0) {
            if (epi == EPI_SWIGLU) {
                y[item0] = __fmul_rn(__fdiv_rn(v0, 1.0f + expf(-v0)), v1);
            } else {
                for (int r = 0; r < nrows; ++r) {
                    const int row = item0 + r;
                    const float v = r == 0 ? v0 : v1;
                    if (epi == EPI_STORE) {
                        const float b = bias ? (prefetched ? pre[row - i0] : bias[row]) : 0.f;
                        y[row] = v + b;
                    } else if (epi == EPI_RESID) {
                        const float rr = prefetched ? pre[row - i0] : __ldcg(resid + row);
                        resid[row] = rr + v;
                    } else {
                        y[row] = v;
                        const unsigned long long k = argmax_key(v, (uint32_t)row);
                        best = k > best ? k : best;
                    }
                }
            }
        }
    }
    return best;
}

// All 8 warps are consumers (two per scheduler: up to 255 registers a thread).
__global__ void __launch_bounds__(MK_THREADS, 1) tf_decode_mk_kernel(const MkArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ MkShared S;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nth = MK_THREADS;
    const int G = gridDim.x, cta = blockIdx.x;
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* ring = smem + (((size_t)a.xfloats * 4 + 127) & ~(size_t)127);
    float* red = reinterpret_cast<float*>(ring + (size_t)a.n_slots * a.slot_bytes);  // [2][W][2]
    double* redd = reinterpret_cast<double*>(red + 2 * MK_WARPS * 2);                 // [W]
    float* pre = reinterpret_cast<float*>(redd + MK_WARPS);                           // [GV_PRE]
    uint64_t* full = reinterpret_cast<uint64_t*>(pre + GV_PRE);
    uint64_t* empty = full + MK_MAX_SLOTS;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + MK_MAX_SLOTS);
    volatile int* sh_ok = abort_flag + 1;
    unsigned long long* ckey = reinterpret_cast<unsigned long long*>(empty + MK_MAX_SLOTS + 1);

    MkCtx c;
    c.a = &a;
    c.ring = ring;
    c.full = full;
    c.empty = empty;
    c.abort_flag = abort_flag;
    c.pr = &S.prod;
    c.cta = cta;
    c.G = G;

    if (tid == 0) {
        for (int s = 0; s < a.n_slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MK_WARPS);
        }
        *abort_flag = 0;
        *ckey = 0ull;
        mbar_fence_init();
        S.prod.issued = 0;
        S.prod.done = 0;
        prod_seek(c, 0, 0);
        produce(c);  // fill the ring before anything else
    }
    __syncthreads();

    int pos = __ldcg(a.pos + a.slot);
    int tok = a.n_prompt > 0 ? a.prompt[0] : __ldcg(a.tok);
    unsigned phases_done = 0;
    int consumed = 0;
    bool alive = true;
    const int tp = mk_attn_tile(a.hd, a.xfloats);
    float4 nw[MK_NW];  // RMSNorm weights of phase nw_phase, this thread's chunks
    int nw_phase = -1;

    for (int s = 0; s < a.n_steps && alive; ++s) {
        const bool head = s >= a.first_head;
        const int nph = head ? a.n_ph : a.n_ph - 1;
        const int ws = s < a.n_prompt ? a.ws_prompt : 0;
        if (tok < 0 || tok >= a.n_vocab) {
            if (tid == 0) atomicCAS(a.err, 0, ERR_BAD_TOKEN);
            tok = 0;
        }
        for (int p = 0; p < nph && alive; ++p) {
            const MkPhase& P = a.ph[p];
            if (tid == 0) produce(c);
            if (P.kind == PH_ATTN) {
                if (cta < a.n_kv) mk_attention(c, P.layer, cta, pos, ws, xs, tp, S);
            } else {
                // ---- prologue: the input activation, RMSNorm, epilogue operands ----
                const int K = P.K;
                const int i0 = (int)((long long)P.n_items * cta / G), i1 = (int)((long long)P.n_items * (cta + 1) / G);
                const bool prefetched = (i1 - i0) <= GV_PRE && (P.epi == EPI_RESID || (P.epi == EPI_STORE && P.bias));
                if (prefetched)
                    for (int i = tid; i < i1 - i0; i += nth)
                        pre[i] = P.epi == EPI_RESID ? __ldcg(P.resid + i0 + i) : P.bias[i0 + i];
                const int nq = K >> 2;
                if (P.pro == PRO_EMBED_RMSNORM) {
                    embed_row(xs, a.embd, a.embd_type, a.embd_rb, K, tok, nth);
                    cbar();
                    if (cta == 0)
                        for (int e = tid; e < K; e += nth) a.x_resid[e] = xs[xpad(e)];
                } else {
                    const float4* xg = reinterpret_cast<const float4*>(P.x);
                    for (int base = tid; base < nq; base += nth * GV_PRO_UNROLL) {
                        float4 v[GV_PRO_UNROLL];
#pragma unroll
                        for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                            const int cc = base + u * nth;
                            if (cc < nq) v[u] = __ldcg(xg + cc);
                        }
#pragma unroll
                        for (int u = 0; u < GV_PRO_UNROLL; ++u) {
                            const int cc = base + u * nth;
                            if (cc < nq) *reinterpret_cast<float4*>(xs + xpad(4 * cc)) = v[u];
                        }
                    }
                }
                if (P.pro != PRO_COPY) {
                    // rmsnorm (src/layers.cpp:7-12): double sum of squares, out = (x * inv) * w
                    cbar();
                    double ss = 0.0;
                    for (int cc = tid; cc < nq; cc += nth) {
                        const float4 v = *reinterpret_cast<const float4*>(xs + xpad(4 * cc));
                        ss = fma((double)v.x, (double)v.x, ss);
                        ss = fma((double)v.y, (double)v.y, ss);
                        ss = fma((double)v.z, (double)v.z, ss);
                        ss = fma((double)v.w, (double)v.w, ss);
                    }
                    ss = warp_sum_d(ss);
                    if (lane == 0) redd[warp] = ss;
                    cbar();
                    double tot = 0.0;
                    for (int w = 0; w < MK_WARPS; ++w) tot += redd[w];
                    const float inv = 1.0f / sqrtf((float)(tot / K) + a.eps);
                    for (int cc = tid; cc < nq; cc += nth) {
                        float4* px = reinterpret_cast<float4*>(xs + xpad(4 * cc));
                        const int u = (cc - tid) / nth;  // fetched before the barrier when u < MK_NW
                        const float4 wv = (nw_phase == p && u < MK_NW) ? nw[u < MK_NW ? u : 0]
                                                                       : reinterpret_cast<const float4*>(P.norm_w)[cc];
                        float4 v = *px;
                        v.x = __fmul_rn(__fmul_rn(v.x, inv), wv.x);
                        v.y = __fmul_rn(__fmul_rn(v.y, inv), wv.y);
                        v.z = __fmul_rn(__fmul_rn(v.z, inv), wv.z);
                        v.w = __fmul_rn(__fmul_rn(v.w, inv), wv.w);
                        *px = v;
                    }
                }
                cbar();
                // ---- this CTA's stages of the ring ----
                const unsigned long long best =
                    P.reg ? mk_gemv_stages<true>(c, P, red, pre, xs, i0, i1, prefetched, consumed)
                          : mk_gemv_stages<false>(c, P, red, pre, xs, i0, i1, prefetched, consumed);
                if (P.epi == EPI_ARGMAX) {
                    if (lane == 0 && best) atomicMax(ckey, best);
                    cbar();
                    if (tid == 0) {
                        atomicMax(&a.keys[s & 1], *ckey);
                        *ckey = 0ull;
                    }
                }
            }
            ++phases_done;
            {   // the next phase's RMSNorm weights are static: fetch them before the barrier
                const int pn = p + 1 < nph ? p + 1 : 0;
                const MkPhase& N = a.ph[pn];
                nw_phase = -1;
                if (N.kind == PH_GEMV && N.pro != PRO_COPY) {
#pragma unroll
                    for (int u = 0; u < MK_NW; ++u) {
                        const int cc = tid + u * nth;
                        if (cc < (N.K >> 2)) nw[u] = reinterpret_cast<const float4*>(N.norm_w)[cc];
                    }
                    nw_phase = pn;
                }
            }
            if (!grid_sync(c, phases_done * (unsigned)G, a.err, sh_ok)) {
                alive = false;
                break;
            }
            // after the first barrier of step s every CTA has read step s-1's key: the
            // key of parity (s+1) can be cleared for step s+1
            if (p == 0 && cta == 0 && tid == 0) a.keys[(s + 1) & 1] = 0ull;
        }
        if (!alive) break;
        pos += 1;
        if (head) {
            const int t = (int)key_index(__ldcg(a.keys + (s & 1)));
            if (cta == 0 && tid == 0) {
                const int gi = s - a.first_head;
                if (a.hist && gi < a.hist_cap) a.hist[gi] = t;
                *a.tok = t;
            }
            tok = t;
        }
        if (s + 1 < a.n_prompt) tok = a.prompt[s + 1];
    }
    if (cta == 0 && tid == 0 && alive) a.pos[a.slot] = pos;
    // copies still in flight (only after an abort) land before the block exits
    if (tid == 0) {
        const int issued = S.prod.issued;
        const int first = issued > a.n_slots ? issued - a.n_slots : 0;
        for (int q = first; q < issued; ++q) mbar_wait(&full[q % a.n_slots], (q / a.n_slots) & 1, nullptr, 0, nullptr);
    }
    // the last CTA out resets the barrier counters and keys for the next launch
    cbar();
    if (tid == 0) {
        __threadfence();
        const unsigned t = atomicAdd(a.bar + 1, 1u);
        if (t == (unsigned)G - 1) {
            a.bar[0] = 0u;
            a.keys[0] = 0ull;
            a.keys[1] = 0ull;
            __threadfence();
            atomicExch(a.bar + 1, 0u);
        }
    }
}

size_t mk_smem_bytes(const MkArgs& a) {
    return (((size_t)a.xfloats * 4 + 127) & ~(size_t)127) + (size_t)a.n_slots * a.slot_bytes + 2 * MK_WARPS * 2 * 4 +
           MK_WARPS * 8 + GV_PRE * 4 + 2 * MK_MAX_SLOTS * 8 + 8 + 8;
}

// Resident CTAs per SM for a given dynamic shared-memory size (the cooperative launch needs
// one per SM); -1 on an error.
int mk_occupancy(size_t smem) {
    if (cudaFuncSetAttribute(tf_decode_mk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return -1;
    if (cudaFuncSetAttribute(tf_decode_mk_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
        return -1;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, tf_decode_mk_kernel, MK_THREADS, smem) != cudaSuccess) return -1;
    return n;
}

cudaError_t mk_launch(const MkArgs& a, int grid, cudaStream_t st) {
    const size_t smem = mk_smem_bytes(a);
    cudaError_t e = cudaFuncSetAttribute(tf_decode_mk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tf_decode_mk_kernel, a);
}

}  // namespace tfb
