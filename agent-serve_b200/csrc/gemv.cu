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
#include "gemv.cuh"

namespace tfb {

__device__ __forceinline__ void named_bar_compute() {
    asm volatile("bar.sync 1, %0;" ::"n"(GV_WARPS * 32) : "memory");
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

__device__ __forceinline__ float q8_magic(uint32_t wbiased, int byte) {
    // wbiased holds four (q + 128) bytes; returns q of byte `byte` exactly.
    return __int_as_float((int)__byte_perm(wbiased, 0x4B000000u, 0x7650u | (uint32_t)byte)) - 8388736.0f;
}

// ---- Q8_0 fast path: one row segment of `units` 64-element units -----------------------
template <int MAXM>
__device__ __forceinline__ void dot_q8_fast(const uint8_t* seg, int units, const float* xseg, int xl, int M,
                                            int lane, float (&acc)[MAXM]) {
    for (int u = lane; u < units; u += 32) {
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(seg + (size_t)u * 68);
        uint32_t w[17];
#pragma unroll
        for (int i = 0; i < 17; ++i) w[i] = wp[i];
        const float dA = h2f(w[0]);
        const float dB = h2f(w[8] >> 16);
#pragma unroll
        for (int i = 0; i < 17; ++i) w[i] ^= 0x80808080u;
        const float* xu = xseg + (size_t)u * 68;
        float sA[MAXM], sB[MAXM];
#pragma unroll
        for (int m = 0; m < MAXM; ++m) sA[m] = sB[m] = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            float qa[4], qb[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int ja = 2 + 4 * g + e;        // byte of block A within the unit
                qa[e] = q8_magic(w[ja >> 2], ja & 3);
                const int jb = 36 + 4 * g + e;       // byte of block B
                qb[e] = q8_magic(w[jb >> 2], jb & 3);
            }
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < M) {
                    const float4 xa = *reinterpret_cast<const float4*>(xu + m * xl + 4 * g);
                    const float4 xb = *reinterpret_cast<const float4*>(xu + m * xl + 32 + 4 * g);
                    sA[m] = fmaf(xa.x, qa[0], sA[m]);
                    sA[m] = fmaf(xa.y, qa[1], sA[m]);
                    sA[m] = fmaf(xa.z, qa[2], sA[m]);
                    sA[m] = fmaf(xa.w, qa[3], sA[m]);
                    sB[m] = fmaf(xb.x, qb[0], sB[m]);
                    sB[m] = fmaf(xb.y, qb[1], sB[m]);
                    sB[m] = fmaf(xb.z, qb[2], sB[m]);
                    sB[m] = fmaf(xb.w, qb[3], sB[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            acc[m] = fmaf(dA, sA[m], acc[m]);
            acc[m] = fmaf(dB, sB[m], acc[m]);
        }
    }
}

// ---- generic path: one lane per block (32 elements; 256 for Q6_K) ----------------------
// Produces either (scale, q[32]) with the block scale applied to the block sum (Q8_0, Q4_0,
// as src/quant.cpp:266-363 do) or dequantised w[32] (Q4_1, Q6_K, F16, F32, as
// dequant_row + dot_f32 do).
template <int MAXM>
__device__ __forceinline__ void dot_generic(int t, const uint8_t* seg, int e0, int nelem, const float* xs, int xl,
                                            int M, int lane, float (&acc)[MAXM]) {
    const int be = (t == T_Q6_K) ? 256 : 32;
    const int bb = (t == T_F32) ? 128 : (t == T_F16) ? 64 : blk_bytes(t);
    const int nblk = nelem / be;
    for (int b = lane; b < nblk; b += 32) {
        const uint8_t* p = seg + (size_t)b * bb;
        const int groups = be / 32;
        for (int g = 0; g < groups; ++g) {
            float w[32];
            float scale = 1.f;
            bool scaled = false;
            if (t == T_Q8_0) {
                scale = h2f(ld_u16(p));
                scaled = true;
#pragma unroll
                for (int j = 0; j < 32; ++j) w[j] = (float)(int8_t)p[2 + j];
            } else if (t == T_Q4_0) {
                scale = h2f(ld_u16(p));
                scaled = true;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const uint32_t q = p[2 + j];
                    w[j] = (float)((int)(q & 15u) - 8);
                    w[j + 16] = (float)((int)(q >> 4) - 8);
                }
            } else if (t == T_Q4_1) {
                const float d = h2f(ld_u16(p)), mn = h2f(ld_u16(p + 2));
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const uint32_t q = p[4 + j];
                    w[j] = __fmaf_rn((float)(q & 15u), d, mn);
                    w[j + 16] = __fmaf_rn((float)(q >> 4), d, mn);
                }
            } else if (t == T_Q6_K) {
                const int h = g >> 2, tq = g & 3;
                const float d = h2f(ld_u16(p + 208));
                const uint8_t* ql = p + 64 * h + ((tq & 1) ? 32 : 0);
                const uint8_t* qh = p + 128 + 32 * h;
                const int8_t* sc = reinterpret_cast<const int8_t*>(p + 192 + 8 * h + 2 * tq);
                const float ds0 = __fmul_rn(d, (float)sc[0]);
                const float ds1 = __fmul_rn(d, (float)sc[1]);
#pragma unroll
                for (int l = 0; l < 32; ++l) {
                    const uint32_t lo = (tq >= 2) ? (ql[l] >> 4) : (ql[l] & 15u);
                    const uint32_t hi = (qh[l] >> (2 * tq)) & 3u;
                    const int q = (int)(lo | (hi << 4)) - 32;
                    w[l] = __fmul_rn(l < 16 ? ds0 : ds1, (float)q);
                }
            } else if (t == T_F16) {
#pragma unroll
                for (int j = 0; j < 32; ++j) w[j] = h2f(ld_u16(p + 2 * j));
            } else {  // F32: rows are 4-byte aligned
                const float* fp = reinterpret_cast<const float*>(p);
#pragma unroll
                for (int j = 0; j < 32; ++j) w[j] = fp[j];
            }
            const int ebase = e0 + b * be + 32 * g;
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < M) {
                    const float* xm = xs + m * xl;
                    float s = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j) s = fmaf(xm[xpad(ebase + j)], w[j], s);
                    acc[m] = scaled ? fmaf(scale, s, acc[m]) : acc[m] + s;
                }
            }
        }
    }
}

// ---- embedding row dequantisation into shared memory (dequant_row, src/quant.cpp:133) ---
__device__ void embed_row(float* xm, const uint8_t* E, int t, long long rb, int K, long long tok) {
    const uint8_t* row = E + tok * rb;
    const int be = (t == T_Q6_K) ? 256 : 32;
    const int bb = (t == T_F32) ? 128 : (t == T_F16) ? 64 : blk_bytes(t);
    const int tid = threadIdx.x;
    const int nb = K / be;
    for (int b = tid; b < nb; b += GV_WARPS * 32) {
        const uint8_t* p = row + (size_t)b * bb;
        for (int g = 0; g < be / 32; ++g) {
            const int e = b * be + 32 * g;
            for (int j = 0; j < 32; ++j) {
                float v;
                if (t == T_Q8_0) {
                    v = __fmul_rn(h2f(ld_u16(p)), (float)(int8_t)p[2 + j]);
                } else if (t == T_Q4_0) {
                    const uint32_t q = p[2 + (j & 15)];
                    v = __fmul_rn(h2f(ld_u16(p)), (float)((int)((j < 16) ? (q & 15u) : (q >> 4)) - 8));
                } else if (t == T_Q4_1) {
                    const uint32_t q = p[4 + (j & 15)];
                    v = __fmaf_rn((float)((j < 16) ? (q & 15u) : (q >> 4)), h2f(ld_u16(p)), h2f(ld_u16(p + 2)));
                } else if (t == T_Q6_K) {
                    const int h = g >> 2, tq = g & 3;
                    const uint8_t* ql = p + 64 * h + ((tq & 1) ? 32 : 0);
                    const uint8_t* qh = p + 128 + 32 * h;
                    const int8_t sc = reinterpret_cast<const int8_t*>(p + 192 + 8 * h + 2 * tq)[j >> 4];
                    const uint32_t lo = (tq >= 2) ? (ql[j] >> 4) : (ql[j] & 15u);
                    const uint32_t hi = (qh[j] >> (2 * tq)) & 3u;
                    v = __fmul_rn(__fmul_rn(h2f(ld_u16(p + 208)), (float)sc), (float)((int)(lo | (hi << 4)) - 32));
                } else if (t == T_F16) {
                    v = h2f(ld_u16(p + 2 * (32 * g + j)));
                } else {
                    v = reinterpret_cast<const float*>(p)[32 * g + j];
                }
                xm[xpad(e + j)] = v;
            }
        }
    }
}

template <int MAXM>
__global__ void __launch_bounds__(GV_THREADS, 2) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int xl = xpad_len(a.K);
    const int xbytes = ((a.M * xl * 4) + 127) & ~127;
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* stages = smem + xbytes;
    float* red = reinterpret_cast<float*>(stages + (size_t)GV_STAGES * a.stage_bytes);  // [2][W][2][MAXM]
    double* redd = reinterpret_cast<double*>(red + 2 * GV_WARPS * 2 * MAXM);              // [W][MAXM]
    uint64_t* full = reinterpret_cast<uint64_t*>(redd + GV_WARPS * MAXM);
    uint64_t* empty = full + GV_STAGES;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + GV_STAGES);
    unsigned long long* ckey = reinterpret_cast<unsigned long long*>(empty + GV_STAGES + 1);

    const int i0 = (int)((long long)a.n_items * blockIdx.x / gridDim.x);
    const int i1 = (int)((long long)a.n_items * (blockIdx.x + 1) / gridDim.x);
    const int RI = GV_WARPS / a.KS;
    const int n_stages = (i1 - i0 + RI - 1) / RI;

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
    pdl_wait();
    const int nth = GV_WARPS * 32;
    for (int m = 0; m < a.M; ++m) {
        float* xm = xs + m * xl;
        if (a.pro == PRO_EMBED_RMSNORM) {
            int tok = a.tokens[m];
            if (tok < 0 || tok >= a.n_vocab) {
                if (tid == 0) atomicCAS(a.err, 0, ERR_BAD_TOKEN);
                tok = 0;
            }
            embed_row(xm, a.embd, a.embd_type, a.embd_rb, a.K, tok);
            named_bar_compute();
            if (blockIdx.x == 0)
                for (int e = tid; e < a.K; e += nth) a.x_out[(size_t)m * a.ldx + e] = xm[xpad(e)];
        } else {
            const float* xg = a.x + (size_t)m * a.ldx;
            for (int e = tid; e < a.K; e += nth) xm[xpad(e)] = xg[e];
        }
    }
    if (a.pro != PRO_COPY) {
        // rmsnorm (src/layers.cpp:7-12): sum of squares in double, inv in float,
        // out = (x * inv) * w.
        named_bar_compute();
        for (int m = 0; m < a.M; ++m) {
            const float* xm = xs + m * xl;
            double ss = 0.0;
            for (int e = tid; e < a.K; e += nth) {
                const double v = (double)xm[xpad(e)];
                ss = fma(v, v, ss);
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
            for (int e = tid; e < a.K; e += nth) xm[xpad(e)] = __fmul_rn(__fmul_rn(xm[xpad(e)], inv), a.norm_w[e]);
        }
    }
    named_bar_compute();

    // ---------------- consumers: main loop ----------------
    const int kseg = a.K / a.KS;
    const int my_item = warp / a.KS, my_ks = warp % a.KS;
    unsigned long long best[MAXM];
#pragma unroll
    for (int m = 0; m < MAXM; ++m) best[m] = 0ull;

    for (int s = 0; s < n_stages; ++s) {
        const int slot = s % GV_STAGES;
        const bool ok = mbar_wait(&full[slot], (s / GV_STAGES) & 1, a.err, ERR_WAIT_FULL, abort_flag);
        const int si0 = i0 + s * RI, si1 = min(si0 + RI, i1);
        const int item = si0 + my_item;
        float acc[2][MAXM];
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
            for (int m = 0; m < MAXM; ++m) acc[p][m] = 0.f;
        if (ok && item < si1) {
            const uintptr_t g = reinterpret_cast<uintptr_t>(a.W + (long long)si0 * a.P * a.rb);
            const uint8_t* sb = stages + (size_t)slot * a.stage_bytes + (g & 15);
            const uint8_t* ib = sb + (long long)my_item * a.P * a.rb;
            for (int p = 0; p < a.P; ++p) {
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
                for (int m = 0; m < MAXM; ++m) acc[p][m] = warp_sum(part[m]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        bool have = ok && item < si1;
        if (a.KS > 1) {
            float* rb = red + ((s & 1) * GV_WARPS + warp) * 2 * MAXM;
            if (lane == 0 && have)
                for (int p = 0; p < 2; ++p)
                    for (int m = 0; m < MAXM; ++m) rb[p * MAXM + m] = acc[p][m];
            named_bar_compute();
            have = have && my_ks == 0;
            if (have && lane == 0) {
                for (int p = 0; p < 2; ++p)
                    for (int m = 0; m < MAXM; ++m) {
                        float v = 0.f;
                        for (int k = 0; k < a.KS; ++k) v += red[((s & 1) * GV_WARPS + warp + k) * 2 * MAXM + p * MAXM + m];
                        acc[p][m] = v;
                    }
            }
        }
        if (have && lane == 0) {
            const int row = item;
            for (int m = 0; m < a.M; ++m) {
                if (a.epi == EPI_STORE) {
                    const float v = acc[0][m] + (a.bias ? a.bias[row] : 0.f);
                    a.y[(size_t)m * a.ldy + row] = v;
                } else if (a.epi == EPI_RESID) {
                    a.resid[(size_t)m * a.ldr + row] += acc[0][m];
                } else if (a.epi == EPI_SWIGLU) {
                    const float g = acc[0][m], u = acc[1][m];
                    a.y[(size_t)m * a.ldy + row] = __fmul_rn(__fdiv_rn(g, 1.0f + expf(-g)), u);
                } else {  // EPI_ARGMAX
                    const float v = acc[0][m];
                    a.y[(size_t)m * a.ldy + row] = v;
                    const unsigned long long k = argmax_key(v, (uint32_t)row);
                    best[m] = k > best[m] ? k : best[m];
                }
            }
        }
    }

    if (a.epi == EPI_ARGMAX && lane == 0)
        for (int m = 0; m < a.M; ++m)
            if (best[m]) atomicMax(&ckey[m], best[m]);
    named_bar_compute();
    if (tid == 0) {
        if (a.epi == EPI_ARGMAX)
            for (int m = 0; m < a.M; ++m) atomicMax(&a.keys[m], ckey[m]);
        if (a.fin != FIN_NONE) {
            __threadfence();
            const unsigned t = atomicAdd(&a.ctl->done, 1u);
            if (t == gridDim.x - 1) {
                __threadfence();
                const int gs = atomicAdd(&a.ctl->gen_step, 0);
                for (int m = 0; m < a.M; ++m) {
                    if (a.fin == FIN_ARGMAX) {
                        const unsigned long long k = atomicExch(&a.keys[m], 0ull);
                        const int tok = (int)key_index(k);
                        a.tok_next[m] = tok;
                        if (a.hist && gs < a.ctl->hist_cap) a.hist[(size_t)gs * a.M + m] = tok;
                    }
                    a.pos[a.slots[m]] += 1;
                }
                a.ctl->gen_step = gs + 1;
                atomicExch(&a.ctl->done, 0u);
                __threadfence();
            }
        }
    }
}

// ---- host side --------------------------------------------------------------------------

size_t gemv_smem_bytes(int M, int K, int stage_bytes, int maxm) {
    const size_t xbytes = ((size_t)M * xpad_len(K) * 4 + 127) & ~(size_t)127;
    return xbytes + (size_t)GV_STAGES * stage_bytes + 2 * GV_WARPS * 2 * maxm * 4 + GV_WARPS * maxm * 8 +
           2 * GV_STAGES * 8 + 8 + maxm * 8;
}

static int pick_maxm(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

// Choose the k-split and stage size for a weight shape (see GemvArgs).
void gemv_plan(GemvArgs& a) {
    const int be = blk_elems(a.wtype) == 1 ? 32 : blk_elems(a.wtype);
    const bool q8fast = (a.wtype == T_Q8_0) && (a.K % 64 == 0);
    int best = -1;
    for (int ks = 1; ks <= GV_WARPS; ks <<= 1) {
        if (a.K % ks) continue;
        const int seg = a.K / ks;
        if (seg % be) continue;
        if (q8fast && seg % 64) continue;
        best = ks;
        const long long payload = (long long)(GV_WARPS / ks) * a.P * a.rb;
        if (payload <= GV_STAGE_BUDGET) break;
    }
    if (best < 0) best = 1;
    a.KS = best;
    // the fast path reads 4-byte words: rows must start 4-byte aligned
    a.fast = q8fast && ((a.K / best) % 64 == 0) && ((reinterpret_cast<uintptr_t>(a.W) & 3) == 0);
    const long long payload = (long long)(GV_WARPS / best) * a.P * a.rb;
    a.stage_bytes = (int)((payload + 32 + 15) & ~15LL);
}

int gemv_max_rows(int K) {
    // activation rows whose padded copies fit next to the stages
    const size_t per = (size_t)xpad_len(K) * 4;
    int m = (int)((96 * 1024) / per);
    return m < 1 ? 1 : (m > GV_MAXM ? GV_MAXM : m);
}

cudaError_t gemv_init_attrs() {
    cudaError_t e;
    const int lim = 200 * 1024;
    if ((e = cudaFuncSetAttribute(gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim))) return e;
    return cudaFuncSetAttribute(gemv_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
}

template <int MAXM>
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
    return cudaLaunchKernelEx(&cfg, gemv_kernel<MAXM>, a);
}

cudaError_t gemv_launch(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
    switch (pick_maxm(a.M)) {
        case 1: return launch_t<1>(a, grid, st, pdl);
        case 2: return launch_t<2>(a, grid, st, pdl);
        case 4: return launch_t<4>(a, grid, st, pdl);
        default: return launch_t<8>(a, grid, st, pdl);
    }
}

int gemv_grid(const GemvArgs& a, int num_sms) {
    const int RI = GV_WARPS / a.KS;
    const int stages = (a.n_items + RI - 1) / RI;
    return stages < num_sms ? (stages > 0 ? stages : 1) : num_sms;
}

}  // namespace tfb
