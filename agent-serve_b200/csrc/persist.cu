// Persistent batch-1 decode kernel (see persist.cuh).
//
// CTA layout: 16 consumer warps and one producer warp, one CTA per SM (cooperative launch,
// so all CTAs are co-resident and may wait for one another).
//
//   producer   lane 0 of the last warp walks this CTA's stages of every GEMV phase of every
//              step in consumption order and issues them as 1-D bulk copies into a ring of
//              shared-memory slots (mbarrier full / empty pairs).  It only ever waits for a
//              free slot, never for an activation, so the weights of the next phases stream
//              in while the consumers wait at a phase boundary.
//   consumers  per phase: wait (bounded) until every CTA has arrived at the phase this one
//              depends on, build the activation's digit planes in shared memory (RMSNorm or
//              embedding fused), dot this CTA's rows on the exact-integer Q8_0 path (dots.cuh),
//              apply the epilogue, arrive.  The attention phase runs on CTAs
//              [0, n_head * nsf): RoPE + KV store + online-softmax attention of one query head
//              (and one position split), its first K/V tile requested (bulk copies) before
//              the q/k/v exist.
//
// Inside a step the phases hand their outputs over as flag-in-data pairs {value, epoch}
// (one 8-byte store per value, persist.cuh): a consumer polls exactly the pairs it needs, so
// a phase boundary costs the store's propagation and one poll, with no fence and no counter.
// Every phase needs all of the previous phase's outputs (directly, or for the attention
// through the heads that cover every QKV row), so no CTA can overwrite a buffer that another
// CTA has still to read.  Between steps the CTAs meet at one counter (fence, release add,
// acquire), which also orders each step's KV-cache stores before the next step's reads.  A
// CTA keeps on chip what only it updates (its rows of the residual stream) and what it reads
// at every layer (its QKV bias rows, the step's RoPE row).  Every wait is bounded; a CTA that
// gives up records the error code, raises the launch's abort word (every other wait checks
// it) and leaves after its copies in flight have landed.
#include <algorithm>
#include <cstdlib>

#include "attention.cuh"
#include "dots.cuh"
#include "persist.cuh"

namespace tfb {

struct PkMisc {
    uint64_t full[PK_MAX_SLOTS];
    uint64_t empty[PK_MAX_SLOTS];
    uint64_t abar;  // attention K / V tile copies
    double redd[PK_WARPS];
    float red[2][PK_WARPS][4];
    float xo[PK_ROWS];        // this CTA's rows of the residual stream (it alone updates them)
    float pre[PK_ROWS];       // this CTA's QKV bias rows
    float cs[PK_MAX_D2];      // RoPE cos / sin of this step's position (attention CTAs)
    float sn[PK_MAX_D2];
    unsigned long long ckey;
    int ok;
    int abort;  // this CTA gave up: its producer stops, its waits return at once
    int flag;
    int trace_i;  // phase-trace entries written by this CTA
};

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(PK_CONS) : "memory"); }
__device__ __forceinline__ int ld_vol(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

struct PkRing {
    uint8_t* base;
    int slot_bytes, n_slots;
    uint64_t* full;
    uint64_t* empty;
};

struct PkCtx {
    const PkArgs* a;
    PkRing rg;
    PkMisc* S;
    uint8_t* reg;
    int cta, G;
    int cs;     // ring stages consumed so far
    int tiles;  // attention tiles loaded so far (phase of abar)
};

__device__ __forceinline__ int item_begin(int n, int c, int G) { return (int)((long long)n * c / G); }

// Phase trace (PkArgs::trace): thread 0 of CTA 0 and of the last CTA stamp the global timer.
__device__ __forceinline__ void pk_trace(const PkCtx& c, int tag) {
    const PkArgs& a = *c.a;
    if (!a.trace || threadIdx.x != 0) return;
    const int w = c.cta == 0 ? 0 : (c.cta == c.G - 1 ? 1 : -1);
    if (w < 0) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const int i = c.S->trace_i++;
    if (i < a.trace_cap) a.trace[(size_t)w * a.trace_cap + i] = (t << 8) | (unsigned)tag;
    a.trace_n[w] = i + 1;
}

// ---- producer -----------------------------------------------------------------------------
__device__ void pk_produce(const PkArgs& a, const PkRing& rg, PkMisc* S, int cta, int G) {
    int issued = 0;
    bool stop = false;
    auto issue_mat = [&](const PkMat& mt) {
        const int i0 = item_begin(mt.n_items, cta, G), i1 = item_begin(mt.n_items, cta + 1, G);
        for (int si0 = i0; si0 < i1; si0 += mt.RI) {
            const int slot = issued % rg.n_slots;
            if (issued >= rg.n_slots &&
                !mbar_wait(&rg.empty[slot], ((issued / rg.n_slots) - 1) & 1, a.err, ERR_WAIT_EMPTY, &S->abort)) {
                stop = true;
                return;
            }
            const int si1 = min(si0 + mt.RI, i1);
            // [ga, gb) is the 16-byte aligned body, moved by the bulk copy; the last (end - gb)
            // < 16 bytes are copied here with plain loads, so nothing beyond the stage's rows
            // (or before its aligned-down start) is read.
            const uintptr_t g = reinterpret_cast<uintptr_t>(mt.W + (long long)si0 * mt.P * mt.rb);
            const uintptr_t end = g + (uintptr_t)((long long)(si1 - si0) * mt.P * mt.rb);
            const uintptr_t ga = g & ~(uintptr_t)15, gb = end & ~(uintptr_t)15;
            uint8_t* dst = rg.base + (size_t)slot * rg.slot_bytes;
            for (uintptr_t p = (gb > ga ? gb : ga); p < end; ++p) dst[p - ga] = *reinterpret_cast<const uint8_t*>(p);
            const uint32_t bytes = gb > ga ? (uint32_t)(gb - ga) : 0u;
            mbar_expect_tx(&rg.full[slot], bytes);
            if (bytes) bulk_g2s(dst, reinterpret_cast<const void*>(ga), bytes, &rg.full[slot]);
            ++issued;
        }
    };
    for (int s = 0; s < a.n_steps && !stop; ++s) {
        for (int l = 0; l < a.n_layer && !stop; ++l)
            for (int k = 0; k < PK_MATS && !stop; ++k) issue_mat(a.mats[PK_MATS * l + k]);
        if (s >= a.first_head && !stop) issue_mat(a.mats[PK_MATS * a.n_layer]);
    }
    // copies in flight land before the CTA exits
    const int first = issued > rg.n_slots ? issued - rg.n_slots : 0;
    for (int q = first; q < issued; ++q) mbar_wait(&rg.full[q % rg.n_slots], (q / rg.n_slots) & 1, nullptr, 0, nullptr);
}

// ---- phase boundaries -----------------------------------------------------------------------
// Bounded wait (thread 0) until *cnt >= target; every consumer thread gets the verdict.
__device__ bool pk_wait(PkCtx& c, const unsigned* cnt, unsigned target) {
    if (threadIdx.x == 0) {
        int ok = ld_vol(c.a->abort_g) == 0;
        if (ok && cnt) {
            int i = 0;
            for (; i < kGridPolls; ++i) {
                if (ld_acquire_gpu(cnt) >= target) break;
                if ((i & 31) == 31 && ld_vol(c.a->abort_g)) {
                    ok = 0;
                    break;
                }
                if (i > 32) __nanosleep(i > 65536 ? 1024 : 20);
            }
            if (i == kGridPolls) {
                atomicCAS(c.a->err, 0, ERR_GRID_SYNC);
                ok = 0;
            }
        }
        if (!ok) {
            atomicExch(c.a->abort_g, 1);
            *reinterpret_cast<volatile int*>(&c.S->abort) = 1;
        }
        c.S->ok = ok;
    }
    cbar();
    return *reinterpret_cast<volatile int*>(&c.S->ok) != 0;
}

// One verdict for the whole CTA: false when any thread saw a failure (ok false), when this
// CTA's producer gave up, or when another CTA raised the abort word.
__device__ bool pk_verdict(PkCtx& c, bool ok) {
    if (!ok) *reinterpret_cast<volatile int*>(&c.S->abort) = 1;
    cbar();
    if (threadIdx.x == 0) {
        const int v = *reinterpret_cast<volatile int*>(&c.S->abort) == 0 && ld_vol(c.a->abort_g) == 0;
        if (!v) atomicExch(c.a->abort_g, 1);
        c.S->ok = v;
    }
    cbar();
    return *reinterpret_cast<volatile int*>(&c.S->ok) != 0;
}

// Poll this thread's float4 chunks q = tid + u * PK_CONS (< nq) of an LL vector until every
// pair carries epoch ep; the values land in v.  Bounded; false on a timeout or an abort.
__device__ bool ll_read(PkCtx& c, const uint2* src, int nq, unsigned ep, float4 (&v)[PK_PRO_U]) {
    unsigned todo = 0;
#pragma unroll
    for (int u = 0; u < PK_PRO_U; ++u) {
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if ((int)threadIdx.x + u * PK_CONS < nq) todo |= 1u << u;
    }
    for (int i = 0; i < kGridPolls && todo; ++i) {
#pragma unroll
        for (int u = 0; u < PK_PRO_U; ++u) {
            if (!(todo >> u & 1u)) continue;
            const int q = (int)threadIdx.x + u * PK_CONS;
            const uint4 lo = ld_ll2(src + 4 * q), hi = ld_ll2(src + 4 * q + 2);
            if (lo.y == ep && lo.w == ep && hi.y == ep && hi.w == ep) {
                v[u] = make_float4(__uint_as_float(lo.x), __uint_as_float(lo.z), __uint_as_float(hi.x),
                                   __uint_as_float(hi.z));
                todo &= ~(1u << u);
            }
        }
        if (!todo) break;
        if ((i & 15) == 15 && (ld_vol(&c.S->abort) || ld_vol(c.a->abort_g))) return false;
        if (i > 8) __nanosleep(i > 65536 ? 1024 : 64);
    }
    if (todo) {
        atomicCAS(c.a->err, 0, ERR_GRID_SYNC);
        return false;
    }
    return true;
}

// Attention tile: cached K rows [p0, p0 + n) of one head into ks (row stride kst floats,
// one bulk copy per row; the padding keeps the one-position-per-thread score reads
// conflict-free) and the V rows into vs (one bulk copy), fp32 cache.  Issued by warp 0;
// completion on abar.
__device__ __forceinline__ void pk_issue_tile(PkCtx& c, float* ks, float* vs, int kst, int hd, const float* kc,
                                              const float* vc, int n) {
    const int lane = threadIdx.x & 31;
    if (threadIdx.x < 32) {
        if (lane == 0) mbar_expect_tx(&c.S->abar, (uint32_t)(2 * n * hd * 4));
        __syncwarp();
        for (int r = lane; r < n; r += 32) bulk_g2s(ks + (size_t)r * kst, kc + (size_t)r * hd, (uint32_t)hd * 4, &c.S->abar);
        if (lane == 0 && n) bulk_g2s(vs, vc, (uint32_t)(n * hd * 4), &c.S->abar);
    }
}

// ---- GEMV phase ------------------------------------------------------------------------------
// kind PK_QKV: RMSNorm(x) (layer 0: of the embedded token) -> q | k | v (+ bias)
//      PK_WO:  attention output -> x += W o
//      PK_GU:  RMSNorm(x) -> h = silu(gate) * up
//      PK_DOWN: h -> x += W h
//      PK_HEAD: RMSNorm(x) -> logits, greedy key of the step
// token >= 0: embed that token (layer-0 QKV); token == -2: embed the argmax of step - 1.
// src / ep_in: the LL vector the activation is read from and its epoch (unused when
// embedding); ep_out: the epoch of this phase's outputs.
// One copy of this code serves every GEMV phase (kind is a run-time value and the kernel calls
// it from one place): the phases run one after another, so a single copy stays in the
// instruction cache where five specialised ones would evict each other at every layer.
__device__ __forceinline__ bool pk_gemv(PkCtx& c, const PkMat& mat, int kind, const uint2* src, unsigned ep_in,
                                        unsigned ep_out, int token, int step) {
    const PkArgs& a = *c.a;
    const PkMat mt = mat;  // the plan in registers (the table is in global memory)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = mt.K, nq = K >> 2;
    const bool norm = kind == PK_QKV || kind == PK_GU || kind == PK_HEAD;
    const bool embed = kind == PK_QKV && token != -1;
    const int i0 = item_begin(mt.n_items, c.cta, c.G), i1 = item_begin(mt.n_items, c.cta + 1, c.G);
    if (kind == PK_QKV)  // static operands first: this CTA's bias rows (zero without bias)
        for (int r = tid; r < i1 - i0; r += PK_CONS) c.S->pre[r] = mt.bias ? __ldg(mt.bias + i0 + r) : 0.f;
    float4 wn[PK_PRO_U];
    if (norm) {  // and the RMSNorm weights of this thread's chunks
#pragma unroll
        for (int u = 0; u < PK_PRO_U; ++u) {
            const int q = tid + u * PK_CONS;
            wn[u] = q < nq ? __ldg(reinterpret_cast<const float4*>(mt.norm_w) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }

    pk_trace(c, PT_START + kind);
    // ---- prologue: the activation as digit planes in the region, the lane's unit in registers
    float4 v[PK_PRO_U];
    float* xs = reinterpret_cast<float*>(c.reg);
    if (embed) {
        int tok = token;
        if (token == -2) {
            const unsigned long long key = __ldcg(a.keys + step - 1);
            tok = (int)key_index(key);
            const int hi = step - 1 - a.first_head;
            if (c.cta == 0 && tid == 0 && hi >= 0 && hi < a.hist_cap) a.hist[hi] = tok;
        }
        if (tok < 0 || tok >= a.n_vocab) {
            if (tid == 0) atomicCAS(a.err, 0, ERR_BAD_TOKEN);
            tok = 0;
        }
        embed_row(xs, a.embd, a.embd_type, a.embd_rb, K, tok, PK_CONS);
        cbar();
        // this CTA's rows of the residual stream: the rows its wo / down epilogues update
        const int r0 = item_begin(a.D, c.cta, c.G), r1 = item_begin(a.D, c.cta + 1, c.G);
        for (int e = r0 + tid; e < r1; e += PK_CONS) c.S->xo[e - r0] = xs[xpad(e)];
#pragma unroll
        for (int u = 0; u < PK_PRO_U; ++u) {
            const int q = tid + u * PK_CONS;
            v[u] = q < nq ? *reinterpret_cast<const float4*>(xs + xpad(4 * q)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    } else {
        const bool got = ll_read(c, src, nq, ep_in, v);
        if (!pk_verdict(c, got)) return false;
        pk_trace(c, PT_READ + kind);
    }
    if (norm) {
        // rmsnorm (src/layers.cpp:7-12): sum of squares in double, inv in float, (x * inv) * w
        double ss = 0.0;
#pragma unroll
        for (int u = 0; u < PK_PRO_U; ++u) {
            if (tid + u * PK_CONS < nq) {
                ss = fma((double)v[u].x, (double)v[u].x, ss);
                ss = fma((double)v[u].y, (double)v[u].y, ss);
                ss = fma((double)v[u].z, (double)v[u].z, ss);
                ss = fma((double)v[u].w, (double)v[u].w, ss);
            }
        }
        ss = warp_sum_d(ss);
        if (lane == 0) c.S->redd[warp] = ss;
        cbar();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < PK_WARPS; ++w) tot += c.S->redd[w];
        const float inv = 1.0f / sqrtf((float)(tot / K) + a.eps);
#pragma unroll
        for (int u = 0; u < PK_PRO_U; ++u) {
            v[u].x = __fmul_rn(__fmul_rn(v[u].x, inv), wn[u].x);
            v[u].y = __fmul_rn(__fmul_rn(v[u].y, inv), wn[u].y);
            v[u].z = __fmul_rn(__fmul_rn(v[u].z, inv), wn[u].z);
            v[u].w = __fmul_rn(__fmul_rn(v[u].w, inv), wn[u].w);
        }
    }
    if (embed) cbar();  // the planes overwrite the embedded row
    const int pstride = q8_plane_stride(K);
    float* pinv = reinterpret_cast<float*>(c.reg + 3 * pstride);
    q8_build_planes<PK_PRO_U>(v, K, PK_CONS, tid, c.reg, pstride, pinv);
    cbar();
    const int P = mt.P, KS = mt.KS, RI = mt.RI;
    const int U = K / KS / 64;
    const int my_item = warp / KS, my_ks = warp % KS;
    const int prow = P == 2 ? lane >> 4 : 0;
    const int pu = P == 2 ? lane & 15 : lane;
    const bool pact = pu < U;
    uint32_t pl[51];
    float invA = 0.f, invB = 0.f;
#pragma unroll
    for (int i = 0; i < 51; ++i) pl[i] = 0u;
    if (pact) {
        const int unit = my_ks * U + pu;
        const uint32_t* pw = reinterpret_cast<const uint32_t*>(c.reg + (size_t)unit * 68);
#pragma unroll
        for (int i = 0; i < 17; ++i) {
            pl[i] = pw[i];
            pl[17 + i] = pw[pstride / 4 + i];
            pl[34 + i] = pw[pstride / 2 + i];
        }
        invA = pinv[2 * unit];
        invB = pinv[2 * unit + 1];
    }

    pk_trace(c, PT_PRO + kind);
    // ---- main loop: two stages per iteration (two independent dp4a chains per warp)
    const int n_stages = (i1 - i0 + RI - 1) / RI;
    const long long rb = mt.rb;
    const int lane_off = (my_item * P + prow) * (int)rb + (my_ks * U + (pact ? pu : 0)) * 68;
    const bool lane_ok = pact && prow < P;
    const int rsel = P == 1 ? (lane >> 4) & 1 : (lane >> 3) & 1;
    const bool leader = (lane & (P == 1 ? 15 : 7)) == 0;
    const bool first_row = P == 1 || lane < 16;
    const long long step_bytes = (long long)RI * P * rb;
    unsigned long long best = 0ull;
    bool ok = true;
    const PkRing& rg = c.rg;
    for (int s = 0, it = 0; s < n_stages; s += 2, ++it) {
        const bool two = s + 1 < n_stages;
        const int q0 = c.cs + s, q1 = q0 + 1;
        const int slot0 = q0 % rg.n_slots, slot1 = q1 % rg.n_slots;
        ok = mbar_wait(&rg.full[slot0], (q0 / rg.n_slots) & 1, a.err, ERR_WAIT_FULL, &c.S->abort) && ok;
        if (two && ok) ok = mbar_wait(&rg.full[slot1], (q1 / rg.n_slots) & 1, a.err, ERR_WAIT_FULL, &c.S->abort);
        const int item0 = i0 + s * RI + my_item, item1 = item0 + RI;
        const uintptr_t g0 = reinterpret_cast<uintptr_t>(mt.W) + (uintptr_t)((long long)s * step_bytes +
                                                                            (long long)i0 * P * rb);
        const uintptr_t g1 = g0 + (uintptr_t)step_bytes;
        // both dots run unconditionally (a stale or partly filled slot is still inside the
        // ring); invalid results are selected away, never used
        const uint32_t* wp0 = reinterpret_cast<const uint32_t*>(rg.base + (size_t)slot0 * rg.slot_bytes + (g0 & 15) +
                                                                lane_off);
        const uint32_t* wp1 = reinterpret_cast<const uint32_t*>(rg.base + (size_t)slot1 * rg.slot_bytes + (g1 & 15) +
                                                                lane_off);
        const float d0 = unit_dot_q8_int(wp0, pl, invA, invB);
        const float d1 = unit_dot_q8_int(wp1, pl, invA, invB);
        const bool ok0 = ok && item0 < i1, ok1 = ok && two && item1 < i1;
        const float v0 = (ok0 && lane_ok) ? d0 : 0.f;
        const float v1 = (ok1 && lane_ok) ? d1 : 0.f;
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&rg.empty[slot0]);
            if (two) mbar_arrive(&rg.empty[slot1]);
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
            float* rbuf = &c.S->red[it & 1][warp][0];
            if (leader) rbuf[rsel * 2 + (first_row ? 0 : 1)] = keep;
            cbar();
            mine = my_ks == 0;
            if (mine && leader) {
                float acc = 0.f;
                for (int k = 0; k < KS; ++k) acc += c.S->red[it & 1][warp + k][rsel * 2 + (first_row ? 0 : 1)];
                keep = acc;
            }
        }
        const float other = __shfl_xor_sync(0xffffffffu, keep, 16);  // P == 2: the up row's sum
        const bool okr = rsel ? ok1 : ok0;
        if (mine && leader && first_row && okr) {
            const int row = rsel ? item1 : item0;
            if (kind == PK_QKV) {
                st_ll(a.llq + row, keep + c.S->pre[row - i0], ep_out);
            } else if (kind == PK_WO || kind == PK_DOWN) {
                // wo / down rows are the CTA's residual rows (both partition D the same way)
                const float xv = c.S->xo[row - i0] + keep;
                c.S->xo[row - i0] = xv;
                st_ll(a.llx + row, xv, ep_out);
            } else if (kind == PK_GU) {
                st_ll(a.llh + row, __fmul_rn(__fdiv_rn(keep, 1.0f + expf(-keep)), other), ep_out);
            } else {
                a.logits[row] = keep;
                const unsigned long long k = argmax_key(keep, (uint32_t)row);
                best = k > best ? k : best;
            }
        }
        // a failed wait does not leave the loop: every warp takes the same barriers; once the
        // abort flag is up the remaining waits return at once
    }
    pk_trace(c, PT_LOOP + kind);
    c.cs += n_stages;
    if (kind == PK_HEAD && best) atomicMax(&c.S->ckey, best);
    if (!ok) *reinterpret_cast<volatile int*>(&c.S->abort) = 1;
    cbar();
    if (tid == 0) {  // one verdict for the whole CTA
        const bool cta_ok = *reinterpret_cast<volatile int*>(&c.S->abort) == 0 && ld_vol(a.abort_g) == 0;
        if (kind == PK_HEAD) {
            const unsigned long long k = c.S->ckey;
            c.S->ckey = 0ull;
            if (k && cta_ok) atomicMax(a.keys + step, k);
        }
        if (!cta_ok) {
            atomicExch(a.abort_g, 1);
            *reinterpret_cast<volatile int*>(&c.S->abort) = 1;
        }
        c.S->ok = cta_ok;
    }
    cbar();
    return *reinterpret_cast<volatile int*>(&c.S->ok) != 0;
}

// ---- attention phase ---------------------------------------------------------------------------
// Model::layer_decode's apply_rope on q and k, KVCache::store and attn_decode for query head
// item % n_head over position split item / n_head (src/model.cpp:125-129,
// src/attention.cpp:31-80).  One position per thread for the scores (K rows padded to
// hd + 4 floats), CTA-wide max / sum, ng groups of hd threads for the weighted V sum; with
// nsf > 1 each split leaves (max, sum, weighted V) and the last of the head's CTAs combines
// the splits in split order.
__device__ bool pk_attention(PkCtx& c, int layer, int item, int pos, int ws, unsigned ep_qkv, unsigned ep_att) {
    const PkArgs& a = *c.a;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hd = a.hd, d2 = hd / 2, n_rep = a.n_head / a.n_kv;
    const int nsf = a.nsf, qh = item % a.n_head, sp = item / a.n_head, kvh = qh / n_rep;
    const bool storer = qh % n_rep == 0 && sp == 0;
    const int kst = hd + 4, ng = min(8, PK_CONS / hd), tp = a.attn_tp;
    float* f = reinterpret_cast<float*>(c.reg);
    float* qs = f;                   // [hd]
    float* kn = qs + hd;             // [hd]
    float* vn = kn + hd;             // [hd]
    const float* cs = c.S->cs;       // [d2], loaded at the start of the step
    const float* sn = c.S->sn;
    float* red = vn + 2 * hd;        // [2][32] (after a gap of hd floats: the layout of pk_plan)
    float* pacc = red + 64;          // [ng][hd]
    float* sc = pacc + ng * hd;      // [tp]
    float* ks = sc + tp;             // [tp][kst]
    float* vs = ks + (size_t)tp * kst;  // [tp][hd]
    float* kc = static_cast<float*>(a.kc) + (size_t)layer * a.layer_elems;
    float* vc = static_cast<float*>(a.vc) + (size_t)layer * a.layer_elems;
    const size_t cache_off = (size_t)a.slot * a.slot_elems + (size_t)kvh * a.cap * hd;
    const int span = (pos + 1 - ws + nsf - 1) / nsf;
    const int s0 = ws + sp * span, s1 = min(pos + 1, s0 + span);  // split 0 is never empty
    const float* kcf = kc + cache_off;
    const float* vcf = vc + cache_off;
    // the first tile's cached rows (bulk copies) and the rotation of pos, before q / k / v exist
    if (s0 < s1) {
        const int np = min(s1, s0 + tp) - s0;
        const int npc = (s0 + np == pos + 1) ? np - 1 : np;
        pk_issue_tile(c, ks, vs, kst, hd, kcf + (size_t)s0 * hd, vcf + (size_t)s0 * hd, npc);
    }
    pk_trace(c, PT_ATT0);
    {   // this head's q and its kv head's k, v: one LL pair per thread, polled
        bool got = true;
        if (tid < 3 * hd) {
            const int part = tid / hd, i = tid % hd;
            const size_t off = part == 0 ? (size_t)qh * hd : (size_t)a.H + (part == 2 ? a.KVd : 0) + (size_t)kvh * hd;
            int n = 0;
            uint2 pr = ld_ll1(a.llq + off + i);
            for (; pr.y != ep_qkv && n < kGridPolls; ++n) {
                if ((n & 15) == 15 && (ld_vol(&c.S->abort) || ld_vol(a.abort_g))) break;
                if (n > 8) __nanosleep(n > 65536 ? 1024 : 64);
                pr = ld_ll1(a.llq + off + i);
            }
            got = pr.y == ep_qkv;
            if (!got && n == kGridPolls) atomicCAS(a.err, 0, ERR_GRID_SYNC);
            (part == 0 ? qs : part == 1 ? kn : vn)[i] = __uint_as_float(pr.x);
        }
        if (!pk_verdict(c, got)) {
            if (s0 < s1) {  // the tile's copies land before the CTA unwinds
                mbar_wait(&c.S->abar, c.tiles & 1, nullptr, 0, nullptr);
                ++c.tiles;
            }
            return false;
        }
    }
    cbar();
    for (int i = tid; i < hd; i += PK_CONS) {
        const int j = i % d2;
        if (i < d2) rope_pair(qs[j], qs[j + d2], cs[j], sn[j]);
        else rope_pair(kn[j], kn[j + d2], cs[j], sn[j]);
    }
    cbar();
    if (storer)
        for (int i = tid; i < hd; i += PK_CONS) {
            kc[cache_off + (size_t)pos * hd + i] = kn[i];
            vc[cache_off + (size_t)pos * hd + i] = vn[i];
        }
    pk_trace(c, PT_QKV);
    const float scale = 1.0f / sqrtf((float)hd);
    const int pg = tid / hd, pd = tid % hd;
    const bool pv_thread = tid < ng * hd;
    float m_run = -INFINITY, l_run = 0.f, acc = 0.f;
    bool tile_ok = true;
    for (int t0 = s0; t0 < s1; t0 += tp) {
        const int np = min(s1, t0 + tp) - t0;
        const bool last = t0 + np == pos + 1;
        if (t0 != s0) pk_issue_tile(c, ks, vs, kst, hd, kcf + (size_t)t0 * hd, vcf + (size_t)t0 * hd, last ? np - 1 : np);
        // every thread waits for the tile's copies (bounded); a failed wait leaves the CTA
        // unwinding with the others (the error is recorded, the abort word raised)
        if (!mbar_wait(&c.S->abar, c.tiles & 1, a.err, ERR_WAIT_FULL, &c.S->abort)) tile_ok = false;
        ++c.tiles;
        if (last)
            for (int i = tid; i < hd; i += PK_CONS) {  // the new key / value (fp32: stored exactly)
                ks[(size_t)(np - 1) * kst + i] = kn[i];
                vs[(size_t)(np - 1) * hd + i] = vn[i];
            }
        cbar();
        float sv = -INFINITY;
        if (tid < np) {
            const float4* kp = reinterpret_cast<const float4*>(ks + (size_t)tid * kst);
            const float4* q4 = reinterpret_cast<const float4*>(qs);
            float e0 = 0.f, e1 = 0.f, e2 = 0.f, e3 = 0.f;
            for (int d = 0; d < hd / 4; ++d) {
                const float4 k = kp[d], q = q4[d];
                e0 = fmaf(q.x, k.x, e0);
                e1 = fmaf(q.y, k.y, e1);
                e2 = fmaf(q.z, k.z, e2);
                e3 = fmaf(q.w, k.w, e3);
            }
            sv = scale * ((e0 + e1) + (e2 + e3));
        }
        float tm = warp_max(sv);
        if (lane == 0) red[warp] = tm;
        cbar();
        tm = red[0];
        for (int w = 1; w < PK_WARPS; ++w) tm = fmaxf(tm, red[w]);
        const float mnew = fmaxf(m_run, tm);
        float e = 0.f;
        if (tid < np) {
            e = expf(sv - mnew);
            sc[tid] = e;
        }
        e = warp_sum(e);
        if (lane == 0) red[32 + warp] = e;
        cbar();
        float lt = 0.f;
        for (int w = 0; w < PK_WARPS; ++w) lt += red[32 + w];
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
        cbar();
    }
    pk_trace(c, PT_ATT1);
    if (!pk_verdict(c, tile_ok)) return false;
    if (pv_thread) pacc[tid] = acc;
    cbar();
    if (nsf == 1) {
        for (int d = tid; d < hd; d += PK_CONS) {
            float o = 0.f;
            for (int g = 0; g < ng; ++g) o += pacc[g * hd + d];
            st_ll(a.lla + (size_t)qh * hd + d, o / l_run, ep_att);
        }
        return true;
    }
    // split: this split's partial, then the last of the head's splits combines in split order
    float* pp = a.part + ((size_t)qh * nsf + sp) * (hd + 2);
    for (int d = tid; d < hd; d += PK_CONS) {
        float o = 0.f;
        for (int g = 0; g < ng; ++g) o += pacc[g * hd + d];
        pp[2 + d] = o;
    }
    if (tid == 0) {
        pp[0] = m_run;
        pp[1] = l_run;
    }
    __threadfence();
    cbar();
    if (tid == 0) c.S->flag = atomicAdd(a.tickets + qh, 1u) == (unsigned)nsf - 1;
    cbar();
    if (!*reinterpret_cast<volatile int*>(&c.S->flag)) return true;
    __threadfence();
    float* cm = ks;  // [nsf] maxima, [nsf] sums, [nsf] weights
    const float* pb = a.part + (size_t)qh * nsf * (hd + 2);
    for (int q = tid; q < nsf; q += PK_CONS) {
        cm[q] = __ldcg(pb + (size_t)q * (hd + 2));
        cm[nsf + q] = __ldcg(pb + (size_t)q * (hd + 2) + 1);
    }
    cbar();
    float mx = -INFINITY;
    for (int q = 0; q < nsf; ++q) mx = fmaxf(mx, cm[q]);
    for (int q = tid; q < nsf; q += PK_CONS) cm[2 * nsf + q] = expf(cm[q] - mx);
    cbar();
    float den = 0.f;
    for (int q = 0; q < nsf; ++q) den = fmaf(cm[2 * nsf + q], cm[nsf + q], den);
    for (int d = tid; d < hd; d += PK_CONS) {
        float num = 0.f;
        for (int q = 0; q < nsf; ++q) num = fmaf(cm[2 * nsf + q], __ldcg(pb + (size_t)q * (hd + 2) + 2 + d), num);
        st_ll(a.lla + (size_t)qh * hd + d, num / den, ep_att);
    }
    if (tid == 0) a.tickets[qh] = 0u;
    return true;
}

// ---- the kernel ----------------------------------------------------------------------------
__global__ void __launch_bounds__(PK_THREADS, 1) tf_decode_persistent_kernel(const __grid_constant__ PkArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    PkMisc* S = reinterpret_cast<PkMisc*>(smem + a.misc_off);
    const PkRing rg{smem, a.slot_bytes, a.n_slots, S->full, S->empty};
    const int tid = threadIdx.x, warp = tid >> 5;
    const int cta = (int)blockIdx.x, G = (int)gridDim.x;
    if (tid == 0) {
        for (int s = 0; s < a.n_slots; ++s) {
            mbar_init(&S->full[s], 1);
            mbar_init(&S->empty[s], PK_WARPS);
        }
        mbar_init(&S->abar, 1);
        S->trace_i = 0;
        S->abort = 0;
        S->ckey = 0ull;
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == PK_WARPS) {
        if ((tid & 31) == 0) pk_produce(a, rg, S, cta, G);
        return;
    }
    PkCtx c{&a, rg, S, smem + a.reg_off, cta, G, 0, 0};
    const int L = a.n_layer;
    const unsigned uG = (unsigned)G;
    const int n_att = a.n_head * a.nsf;
    bool ok = true;
    for (int s = 0; s < a.n_steps && ok; ++s) {
        const int pos = a.pos0 + s;
        if (pos < 0 || pos >= a.cap) {
            if (tid == 0) {
                atomicCAS(a.err, 0, ERR_POS);
                atomicExch(a.abort_g, 1);
                *reinterpret_cast<volatile int*>(&S->abort) = 1;
            }
            ok = false;
            break;
        }
        // every CTA has finished the previous step: its KV-cache stores and greedy key are out
        if (s > 0 && !pk_wait(c, a.cnt, (unsigned)s * uG)) {
            ok = false;
            break;
        }
        // the cache rows other CTAs stored (generic proxy) are read by bulk copies (async proxy)
        if (tid < 32 && cta < n_att) asm volatile("fence.proxy.async;" ::: "memory");
        const int ws = s < a.n_prompt ? min(max(a.ws_prompt, 0), pos) : 0;
        const int token = s < a.n_prompt ? a.prompt[s] : -2;
        if (cta < n_att)  // the step's RoPE row, read at every layer's attention
            for (int i = tid; i < a.hd / 2; i += PK_CONS) {
                S->cs[i] = __ldg(a.cosb + (size_t)pos * (a.hd / 2) + i);
                S->sn[i] = __ldg(a.sinb + (size_t)pos * (a.hd / 2) + i);
            }
        const unsigned eb = a.ep0 + (unsigned)s * (unsigned)L * PK_EPS;  // epochs of this step
        // phases of the step in order: per layer QKV, attention, wo, gate/up, down; then the
        // lm_head (one call site for every GEMV phase)
        const int n_ph = L * 5 + (s >= a.first_head ? 1 : 0);
        for (int ph = 0; ph < n_ph && ok; ++ph) {
            const int l = ph / 5, k = ph % 5;
            const unsigned e = eb + (unsigned)l * PK_EPS;
            if (k == 1) {
                if (cta < n_att) ok = pk_attention(c, l, cta, pos, ws, e + PE_QKV, e + PE_ATT);
                continue;
            }
            const int kind = l == L ? PK_HEAD : k == 0 ? PK_QKV : k == 2 ? PK_WO : k == 3 ? PK_GU : PK_DOWN;
            const PkMat& mt = l == L ? a.mats[PK_MATS * L] : a.mats[PK_MATS * l + (k == 0 ? 0 : k - 1)];
            const uint2* src = k == 2 ? a.lla : k == 4 ? a.llh : a.llx;
            const unsigned ep_in = l == L || k == 0 ? e - PK_EPS + PE_DOWN : k == 2 ? e + PE_ATT : k == 3 ? e + PE_WO
                                                                                                   : e + PE_GU;
            const unsigned ep_out = k == 0 ? e + PE_QKV : k == 2 ? e + PE_WO : k == 3 ? e + PE_GU : e + PE_DOWN;
            ok = pk_gemv(c, mt, kind, src, ep_in, ep_out, (l == 0 && k == 0) ? token : -1, s);
        }
        if (ok) {  // step done: fence (cumulative over the CTA's stores), then count the arrival
            cbar();
            if (tid == 0) {
                __threadfence();
                red_release_gpu_add(a.cnt, 1u);
            }
        }
    }
    if (!ok || cta != 0) return;
    // CTA 0 publishes the last step's argmax and the new position once every CTA is done
    if (!pk_wait(c, a.cnt, (unsigned)a.n_steps * uG)) return;
    if (tid == 0) {
        const int sl = a.n_steps - 1;
        if (sl >= a.first_head) {
            const int tok = (int)key_index(__ldcg(a.keys + sl));
            a.tok[0] = tok;
            if (sl - a.first_head < a.hist_cap) a.hist[sl - a.first_head] = tok;
        }
        a.pos[a.slot] = a.pos0 + a.n_steps;
    }
}

// ---- host side ---------------------------------------------------------------------------------
int pk_attn_fixed_floats(int hd) { return 4 * hd + 64 + std::min(8, PK_CONS / hd) * hd; }

bool pk_plan(int slot_bytes, int max_k, int hd, PkPlan& p) {
    const int misc = (int)((sizeof(PkMisc) + 127) & ~(size_t)127);
    const int act = (std::max(q8_plane_bytes(max_k), xpad_len(max_k) * 4) + 127) & ~127;
    const int kst = hd + 4;
    const int per_pos = 4 * (1 + kst + hd);
    const int fixed = 4 * pk_attn_fixed_floats(hd);
    const int att_min = fixed + 64 * per_pos;
    int want = 5;
    if (const char* e = getenv("TFB200_PK_SLOTS")) want = std::max(2, std::min(PK_MAX_SLOTS, atoi(e)));
    for (int n = want; n >= 2; --n) {
        const int reg = PK_SMEM_LIMIT - n * slot_bytes - misc;
        if (reg < act || reg < att_min) continue;
        int tp = (reg - fixed) / per_pos;
        tp = std::min(tp, PK_MAX_TP) & ~3;
        p.slot_bytes = slot_bytes;
        p.n_slots = n;
        p.reg_off = n * slot_bytes;
        p.reg_bytes = reg;
        p.misc_off = p.reg_off + reg;
        p.attn_tp = tp;
        p.smem = (size_t)p.misc_off + misc;
        return true;
    }
    return false;
}

int pk_occupancy(size_t smem) {
    cudaError_t e = cudaFuncSetAttribute(tf_decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return 0;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, tf_decode_persistent_kernel, PK_THREADS, smem) !=
        cudaSuccess)
        return 0;
    return occ;
}

cudaError_t pk_launch(const PkArgs& a, int grid, size_t smem, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(PK_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tf_decode_persistent_kernel, a);
}

}  // namespace tfb
