/* Test infrastructure (the checker), not product -- see tf_oracle.h.
 *
 * Plain-C restatement of the reference engine's hot path.  Arithmetic notes:
 *  - The reference is built by g++ with -std=c++17 -O3 -mavx2 -mfma -mf16c
 *    (CMakeLists.txt:12-18).  g++ contracts a*b+c into one FMA in C++ code, so every
 *    scalar "acc += a*b" of the reference is an fmaf() here, and every _mm256_fmadd_ps
 *    lane is an fmaf() on that lane.  This file is compiled with -ffp-contract=off so
 *    that no other fusion happens.
 *  - hsum8 (src/quant.cpp:186-196) adds lanes as ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)).
 */
#define _GNU_SOURCE
#include "tf_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[256];

const char* tfo_last_error(void) { return g_err; }

/* ---- fp16 ---------------------------------------------------------------------------- */

/* src/quant.cpp:16-45.  The v2 build converts with F16C (_mm_cvtph_ps), which is exact for
 * every half including subnormals; the bit construction below is the same exact mapping. */
float tfo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            exp = 127 - 14;
            while ((mant & 0x400) == 0) {
                mant <<= 1;
                --exp;
            }
            mant &= 0x3FF;
            bits = sign | (exp << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp + (127 - 15)) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* src/quant.cpp:47-49: the v2 build uses _mm_cvtps_ph(x, 0), i.e. IEEE round to nearest
 * even with overflow to infinity and gradual underflow. */
uint16_t tfo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u | ((ax >> 13) & 0x3FFu) : 0));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 */
    if (ax < 0x38800000u) {                                  /* below the smallest normal */
        if (ax < 0x33000000u) return (uint16_t)sign;         /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e; /* value = m * 2^(e-150); half subnormal unit 2^-24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

/* src/tensor.cpp:42-70 */
static int blck_size(int t) {
    switch (t) {
        case TFO_Q4_0: case TFO_Q4_1: case TFO_Q8_0: return 32;
        case TFO_Q6_K: return 256;
        default: return 1;
    }
}
static size_t blck_nbytes(int t) {
    switch (t) {
        case TFO_F32: return 4;
        case TFO_F16: return 2;
        case TFO_Q4_0: return 18;
        case TFO_Q4_1: return 20;
        case TFO_Q8_0: return 34;
        case TFO_Q6_K: return 210;
        default: return 0;
    }
}
size_t tfo_row_nbytes(int t, int64_t k) { return (size_t)(k / blck_size(t)) * blck_nbytes(t); }

static float ld_f16(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return tfo_f16_to_f32(h);
}

/* ---- dequantisation ------------------------------------------------------------------ */

/* src/quant.cpp:66-72  block_q8_0 = {fp16 d; int8 qs[32]} (34 B, src/quant.hpp:13-16) */
static void dequant_q8_0(float* out, const uint8_t* x, int n) {
    for (int i = 0; i < n / 32; ++i) {
        const uint8_t* b = x + 34 * (size_t)i;
        float d = ld_f16(b);
        for (int j = 0; j < 32; ++j) out[i * 32 + j] = d * (float)(int8_t)b[2 + j];
    }
}

/* src/quant.cpp:74-85  block_q4_0 = {fp16 d; u8 qs[16]} (18 B): low nibble -> j, high -> j+16 */
static void dequant_q4_0(float* out, const uint8_t* x, int n) {
    for (int i = 0; i < n / 32; ++i) {
        const uint8_t* b = x + 18 * (size_t)i;
        float d = ld_f16(b);
        for (int j = 0; j < 16; ++j) {
            out[i * 32 + j] = d * (float)((b[2 + j] & 0x0F) - 8);
            out[i * 32 + j + 16] = d * (float)((b[2 + j] >> 4) - 8);
        }
    }
}

/* src/quant.cpp:87-99  block_q4_1 = {fp16 d; fp16 m; u8 qs[16]} (20 B); y = q*d + m, which
 * the reference's g++ build contracts to one FMA. */
static void dequant_q4_1(float* out, const uint8_t* x, int n) {
    for (int i = 0; i < n / 32; ++i) {
        const uint8_t* b = x + 20 * (size_t)i;
        float d = ld_f16(b), m = ld_f16(b + 2);
        for (int j = 0; j < 16; ++j) {
            out[i * 32 + j] = fmaf((float)(b[4 + j] & 0x0F), d, m);
            out[i * 32 + j + 16] = fmaf((float)(b[4 + j] >> 4), d, m);
        }
    }
}

/* src/quant.cpp:101-127  block_q6_K = {u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d} (210 B).
 * Each 128-element half: element l (0..31) of quarter t takes 4 low bits from ql (low or
 * high nibble) and 2 high bits from qh at shift 2t, minus 32; scale index l/16 + 2t. */
static void dequant_q6_K(float* out, const uint8_t* x, int n) {
    for (int i = 0; i < n / 256; ++i) {
        const uint8_t* b = x + 210 * (size_t)i;
        const uint8_t* ql = b;
        const uint8_t* qh = b + 128;
        const int8_t* sc = (const int8_t*)(b + 192);
        const float d = ld_f16(b + 208);
        float* y = out + i * 256;
        for (int n0 = 0; n0 < 256; n0 += 128) {
            for (int l = 0; l < 32; ++l) {
                int is = l / 16;
                int q1 = (int)(int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = (int)(int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)(int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = (int)(int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l] = d * (float)sc[is] * (float)q1;
                y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                y[l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
            y += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

/* src/quant.cpp:133-145 */
void tfo_dequant_row(float* out, int t, const void* w, int k, int64_t row) {
    const uint8_t* src = (const uint8_t*)w + (size_t)row * tfo_row_nbytes(t, k);
    switch (t) {
        case TFO_F32: memcpy(out, src, (size_t)k * 4); break;
        case TFO_F16:
            for (int i = 0; i < k; ++i) out[i] = ld_f16(src + 2 * i);
            break;
        case TFO_Q8_0: dequant_q8_0(out, src, k); break;
        case TFO_Q4_0: dequant_q4_0(out, src, k); break;
        case TFO_Q4_1: dequant_q4_1(out, src, k); break;
        case TFO_Q6_K: dequant_q6_K(out, src, k); break;
        default: break;
    }
}

/* ---- dots (stage-v2 arithmetic) ------------------------------------------------------ */

/* src/quant.cpp:186-196 */
static float hsum8(const float v[8]) {
    float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
    return (a0 + a1) + (a2 + a3);
}

/* src/quant.cpp:198-214 (AVX2 branch): 8 lane accumulators, four FMAs per 32 elements,
 * then 8-element steps, hsum8, then a scalar (contracted) tail. */
float tfo_dot_f32(const float* a, const float* b, int n) {
    float acc[8] = {0};
    int i = 0;
    for (; i + 32 <= n; i += 32)
        for (int u = 0; u < 32; u += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + u + l], b[i + u + l], acc[l]);
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = hsum8(acc);
    for (; i < n; ++i) s = fmaf(a[i], b[i], s);
    return s;
}

/* src/quant.cpp:245-258 (AVX2 branch) */
float tfo_dot_f16_f32(const float* x, const uint16_t* w, int n) {
    float acc[8] = {0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(x[i + l], tfo_f16_to_f32(w[i + l]), acc[l]);
    float s = hsum8(acc);
    for (; i < n; ++i) s = fmaf(x[i], tfo_f16_to_f32(w[i]), s);
    return s;
}

/* src/quant.cpp:266-283 (AVX2 branch): per block, 8 lanes x 4 FMAs of x * float(q), hsum8,
 * then sum += d * blocksum (contracted). */
float tfo_dot_q8_0_f32(const float* x, const void* wv, int n) {
    const uint8_t* w = (const uint8_t*)wv;
    float sum = 0;
    for (int i = 0; i < n / 32; ++i) {
        const uint8_t* b = w + 34 * (size_t)i;
        const float d = ld_f16(b);
        const float* xi = x + 32 * i;
        float acc[8] = {0};
        for (int j = 0; j < 32; j += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(xi[j + l], (float)(int8_t)b[2 + j + l], acc[l]);
        sum = fmaf(d, hsum8(acc), sum);
    }
    return sum;
}

/* src/quant.cpp:323-347 (AVX2 branch): nibbles expanded so element j < 16 is the low nibble
 * of qs[j] and element j >= 16 the high nibble of qs[j-16], minus 8; same FMA order. */
float tfo_dot_q4_0_f32(const float* x, const void* wv, int n) {
    const uint8_t* w = (const uint8_t*)wv;
    float sum = 0;
    for (int i = 0; i < n / 32; ++i) {
        const uint8_t* b = w + 18 * (size_t)i;
        const float d = ld_f16(b);
        const float* xi = x + 32 * i;
        float q[32];
        for (int j = 0; j < 16; ++j) {
            q[j] = (float)((b[2 + j] & 0x0F) - 8);
            q[j + 16] = (float)((b[2 + j] >> 4) - 8);
        }
        float acc[8] = {0};
        for (int j = 0; j < 32; j += 8)
            for (int l = 0; l < 8; ++l) acc[l] = fmaf(xi[j + l], q[j + l], acc[l]);
        sum = fmaf(d, hsum8(acc), sum);
    }
    return sum;
}

/* src/matmul.cpp:5-20: per-dtype row dot; Q4_1 / Q6_K rows are dequantised first and then
 * go through dot_f32. */
static float dot_weight_row(const float* x, int t, const uint8_t* w, int64_t row, int k,
                            float* tmp) {
    const uint8_t* src = w + (size_t)row * tfo_row_nbytes(t, k);
    switch (t) {
        case TFO_F32: return tfo_dot_f32(x, (const float*)src, k);
        case TFO_F16: return tfo_dot_f16_f32(x, (const uint16_t*)src, k);
        case TFO_Q8_0: return tfo_dot_q8_0_f32(x, src, k);
        case TFO_Q4_0: return tfo_dot_q4_0_f32(x, src, k);
        default:
            tfo_dequant_row(tmp, t, w, k, row);
            return tfo_dot_f32(x, tmp, k);
    }
}

typedef struct {
    float* c;
    const float* a;
    int t;
    const uint8_t* w;
    int n, k, m, n0, n1;
} mm_job;

static void* mm_worker(void* p) {
    mm_job* j = (mm_job*)p;
    float* tmp = (float*)malloc((size_t)j->k * sizeof(float));
    for (int n = j->n0; n < j->n1; ++n)
        for (int m = 0; m < j->m; ++m)
            j->c[(size_t)m * j->n + n] = dot_weight_row(j->a + (size_t)m * j->k, j->t, j->w, n, j->k, tmp);
    free(tmp);
    return NULL;
}

/* src/matmul.cpp:22-32 and :64-73 (gemm_naive, the stage-v2 path): C[m,n] = dot(A[m,:], W[n,:]).
 * Rows n are split over threads; the split does not change any result. */
void tfo_matmul(float* c, const float* a, int t, const void* w, int n, int k, int m, int threads) {
    if (threads < 1) threads = 1;
    if ((long long)n * k * m < (1LL << 20)) threads = 1;
    if (threads > 64) threads = 64;
    pthread_t tid[64];
    int live[64] = {0};
    mm_job jobs[64];
    int chunk = (n + threads - 1) / threads;
    for (int i = 0; i < threads; ++i) {
        int n0 = i * chunk, n1 = n0 + chunk < n ? n0 + chunk : n;
        mm_job jb = {c, a, t, (const uint8_t*)w, n, k, m, n0, n0 < n1 ? n1 : n0};
        jobs[i] = jb;
    }
    for (int i = 1; i < threads; ++i) {
        if (jobs[i].n0 >= jobs[i].n1) continue;
        if (pthread_create(&tid[i], NULL, mm_worker, &jobs[i]) == 0) live[i] = 1;
        else mm_worker(&jobs[i]);
    }
    mm_worker(&jobs[0]);
    for (int i = 1; i < threads; ++i)
        if (live[i]) pthread_join(tid[i], NULL);
}

/* ---- elementwise --------------------------------------------------------------------- */

/* src/layers.cpp:7-12: sum of squares in double (contracted: ss = fma(x, x, ss)). */
void tfo_rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
    double ss = 0;
    for (int i = 0; i < n; ++i) ss = fma((double)x[i], (double)x[i], ss);
    float inv = 1.0f / sqrtf((float)(ss / n) + eps);
    for (int i = 0; i < n; ++i) out[i] = x[i] * inv * w[i];
}

/* src/layers.cpp:14-19 */
void tfo_silu_mul(float* gate, const float* up, int n) {
    for (int i = 0; i < n; ++i) {
        float v = gate[i];
        gate[i] = (v / (1.0f + expf(-v))) * up[i];
    }
}

/* src/layers.cpp:21-23 */
void tfo_add_inplace(float* a, const float* b, int n) {
    for (int i = 0; i < n; ++i) a[i] += b[i];
}

/* src/layers.cpp:25-35 */
void tfo_softmax(float* x, int n) {
    float m = x[0];
    for (int i = 1; i < n; ++i) m = x[i] > m ? x[i] : m;
    float s = 0;
    for (int i = 0; i < n; ++i) {
        x[i] = expf(x[i] - m);
        s += x[i];
    }
    float inv = 1.0f / s;
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* ---- RoPE ---------------------------------------------------------------------------- */

/* src/attention.cpp:9-29 */
void tfo_rope_freqs(float* freq, int n_rot, float theta, int llama3, float scale, float low_f,
                    float high_f, float orig_ctx) {
    int d2 = n_rot / 2;
    for (int i = 0; i < d2; ++i) {
        float f = 1.0f / powf(theta, (float)(2 * i) / (float)n_rot);
        if (llama3) {
            float wavelen = 2.0f * 3.14159265358979323846f / f;
            float lo_wl = orig_ctx / low_f;
            float hi_wl = orig_ctx / high_f;
            if (wavelen < hi_wl) {
            } else if (wavelen > lo_wl) {
                f /= scale;
            } else {
                float smooth = (orig_ctx / wavelen - low_f) / (high_f - low_f);
                /* (1-smooth)*f/scale + smooth*f, the final multiply-add contracted */
                f = fmaf(smooth, f, (1.0f - smooth) * f / scale);
            }
        }
        freq[i] = f;
    }
}

/* src/attention.cpp:31-41 and :49-53: NeoX rotate-half on pairs (x[i], x[i + hd/2]) by angle
 * pos * freq[i]; cos/sin in float.  The g++ build evaluates x0*c - x1*s as
 * fma(x0, c, -(x1*s)) and x0*s + x1*c as fma(x0, s, x1*c). */
void tfo_rope(float* x, int seq, int n_heads, int head_dim, int pos0, const float* freq) {
    int d2 = head_dim / 2;
    for (int t = 0; t < seq; ++t)
        for (int h = 0; h < n_heads; ++h) {
            float* v = x + ((size_t)t * n_heads + h) * head_dim;
            for (int i = 0; i < d2; ++i) {
                float ang = (float)(pos0 + t) * freq[i];
                float c = cosf(ang), s = sinf(ang);
                float x0 = v[i], x1 = v[i + d2];
                v[i] = fmaf(x0, c, -(x1 * s));
                v[i + d2] = fmaf(x0, s, x1 * c);
            }
        }
}

/* ---- attention ----------------------------------------------------------------------- */

/* src/attention.cpp:55-80.  k, v are [n_pos][n_kv_heads][head_dim] (the SeqMajor cache of
 * src/kvcache.cpp:21-29; the layout does not change any result). */
void tfo_attn_decode(float* out, const float* q, const float* k, const float* v, int n_pos,
                     int n_heads, int n_kv_heads, int head_dim) {
    const int n_rep = n_heads / n_kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float* sc = (float*)malloc((size_t)n_pos * sizeof(float));
    for (int h = 0; h < n_heads; ++h) {
        const int hv = h / n_rep;
        const float* qh = q + (size_t)h * head_dim;
        for (int p = 0; p < n_pos; ++p)
            sc[p] = scale * tfo_dot_f32(qh, k + ((size_t)p * n_kv_heads + hv) * head_dim, head_dim);
        tfo_softmax(sc, n_pos);
        float* oh = out + (size_t)h * head_dim;
        memset(oh, 0, (size_t)head_dim * sizeof(float));
        for (int p = 0; p < n_pos; ++p) {
            const float* vp = v + ((size_t)p * n_kv_heads + hv) * head_dim;
            for (int d = 0; d < head_dim; ++d) oh[d] = fmaf(sc[p], vp[d], oh[d]);
        }
    }
    free(sc);
}

/* src/attention.cpp:82-111: causal attention within the prompt chunk. */
void tfo_attn_prefill(float* out, const float* q, const float* k, const float* v, int seq,
                      int n_heads, int n_kv_heads, int head_dim) {
    const int n_rep = n_heads / n_kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float* sc = (float*)malloc((size_t)seq * sizeof(float));
    for (int h = 0; h < n_heads; ++h) {
        const int hv = h / n_rep;
        for (int i = 0; i < seq; ++i) {
            const float* qi = q + ((size_t)i * n_heads + h) * head_dim;
            for (int j = 0; j <= i; ++j)
                sc[j] = scale * tfo_dot_f32(qi, k + ((size_t)j * n_kv_heads + hv) * head_dim, head_dim);
            tfo_softmax(sc, i + 1);
            float* oi = out + ((size_t)i * n_heads + h) * head_dim;
            memset(oi, 0, (size_t)head_dim * sizeof(float));
            for (int j = 0; j <= i; ++j) {
                const float* vj = v + ((size_t)j * n_kv_heads + hv) * head_dim;
                for (int d = 0; d < head_dim; ++d) oi[d] = fmaf(sc[j], vj[d], oi[d]);
            }
        }
    }
    free(sc);
}

/* src/sampler.cpp:8-13: first index wins ties (strict >). */
int tfo_sample_greedy(const float* logits, int n) {
    int b = 0;
    for (int i = 1; i < n; ++i)
        if (logits[i] > logits[b]) b = i;
    return b;
}

/* src/sampler.cpp:15-52 with the caller's uniform draw r in [0, 1) (the reference draws it
 * inside, uniform_real_distribution<float>(0, 1) over its std::mt19937): the candidates in
 * descending-logit order, p = exp((l - l_max) / temperature) normalised by the running float
 * sum, the top-p prefix up to and including the first index where the running sum reaches
 * top_p (renormalised over that prefix), then the first prefix entry whose running sum is at
 * least r (the last entry if none).  Logits that tie exactly are ordered by index here; the
 * reference's std::sort leaves their order unspecified.  temperature <= 0 is greedy. */
static const float* tfo_sort_keys;
static int tfo_desc_logit(const void* a, const void* b) {
    const int i = *(const int*)a, j = *(const int*)b;
    const float x = tfo_sort_keys[i], y = tfo_sort_keys[j];
    if (x > y) return -1;
    if (x < y) return 1;
    return (i > j) - (i < j);
}

int tfo_sample_logits(const float* logits, int n, float temperature, float top_p, float r) {
    if (temperature <= 0.0f) return tfo_sample_greedy(logits, n);
    int* order = (int*)malloc(sizeof(int) * (size_t)n);
    float* p = (float*)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < n; ++i) order[i] = i;
    tfo_sort_keys = logits;
    qsort(order, (size_t)n, sizeof(int), tfo_desc_logit);
    const float top = logits[order[0]];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        p[i] = expf((logits[order[i]] - top) / temperature);
        sum += p[i];
    }
    for (int i = 0; i < n; ++i) p[i] /= sum;
    int keep = n;
    if (top_p < 1.0f) {
        float run = 0.0f;
        keep = 0;
        while (keep < n) {
            run += p[keep];
            ++keep;
            if (run >= top_p) break;
        }
        float z = 0.0f;
        for (int i = 0; i < keep; ++i) z += p[i];
        for (int i = 0; i < keep; ++i) p[i] /= z;
    }
    int pick = order[keep - 1];
    float run = 0.0f;
    for (int i = 0; i < keep; ++i) {
        run += p[i];
        if (r <= run) {
            pick = order[i];
            break;
        }
    }
    free(order);
    free(p);
    return pick;
}

/* ---- the token loop ------------------------------------------------------------------ */

typedef struct {
    const tfo_tensor *attn_norm, *wq, *wk, *wv, *wo, *bq, *bk, *bv, *ffn_norm, *gate, *up, *down;
} layer_w;

struct tfo_model {
    tfo_hparams hp;
    int max_seq, threads, n_pos;
    const tfo_tensor *tok_embd, *output_norm, *output;
    layer_w* layers;
    float* freq;
    float *kc, *vc; /* [layer][pos][kv_head][head_dim] */
    float *x, *xb, *q, *k, *v, *hb, *hb2, *logits;
};

static const tfo_tensor* find_t(const tfo_tensor* t, int n, const char* name) {
    for (int i = 0; i < n; ++i)
        if (strcmp(t[i].name, name) == 0) return &t[i];
    return NULL;
}

/* Tensor binding and scratch sizing follow src/model.cpp:43-77 (output.weight falls back to
 * token_embd.weight when absent, biases are optional). */
tfo_model* tfo_model_create(const tfo_tensor* t, int nt, const tfo_hparams* hp, int max_seq,
                            int threads) {
    tfo_model* m = (tfo_model*)calloc(1, sizeof(tfo_model));
    m->hp = *hp;
    m->max_seq = max_seq;
    m->threads = threads;
    char nm[128];
#define MUST(dst, name)                                                   \
    do {                                                                  \
        dst = find_t(t, nt, name);                                        \
        if (!dst) {                                                       \
            snprintf(g_err, sizeof g_err, "missing tensor %s", name);     \
            tfo_model_destroy(m);                                         \
            return NULL;                                                  \
        }                                                                 \
    } while (0)
    MUST(m->tok_embd, "token_embd.weight");
    MUST(m->output_norm, "output_norm.weight");
    m->output = find_t(t, nt, "output.weight");
    if (!m->output) m->output = m->tok_embd;
    m->layers = (layer_w*)calloc((size_t)hp->n_layer, sizeof(layer_w));
    for (int i = 0; i < hp->n_layer; ++i) {
        layer_w* L = &m->layers[i];
#define LW(dst, suffix)                                   \
    do {                                                  \
        snprintf(nm, sizeof nm, "blk.%d.%s", i, suffix);  \
        MUST(dst, nm);                                    \
    } while (0)
#define LO(dst, suffix)                                   \
    do {                                                  \
        snprintf(nm, sizeof nm, "blk.%d.%s", i, suffix);  \
        dst = find_t(t, nt, nm);                          \
    } while (0)
        LW(L->attn_norm, "attn_norm.weight");
        LW(L->wq, "attn_q.weight");
        LW(L->wk, "attn_k.weight");
        LW(L->wv, "attn_v.weight");
        LW(L->wo, "attn_output.weight");
        LO(L->bq, "attn_q.bias");
        LO(L->bk, "attn_k.bias");
        LO(L->bv, "attn_v.bias");
        LW(L->ffn_norm, "ffn_norm.weight");
        LW(L->gate, "ffn_gate.weight");
        LW(L->up, "ffn_up.weight");
        LW(L->down, "ffn_down.weight");
    }
#undef MUST
    const int D = hp->n_embd, H = hp->n_head * hp->head_dim, KV = hp->n_kv_head * hp->head_dim;
    m->freq = (float*)calloc((size_t)hp->head_dim / 2, sizeof(float));
    tfo_rope_freqs(m->freq, hp->head_dim, hp->rope_theta, hp->rope_llama3, hp->rope_scale,
                   hp->rope_low_freq_f, hp->rope_high_freq_f, hp->rope_orig_ctx);
    size_t kvn = (size_t)hp->n_layer * max_seq * KV;
    m->kc = (float*)calloc(kvn, sizeof(float));
    m->vc = (float*)calloc(kvn, sizeof(float));
    m->x = (float*)calloc((size_t)max_seq * D, sizeof(float));
    m->xb = (float*)calloc((size_t)max_seq * (D > H ? D : H), sizeof(float));
    m->q = (float*)calloc((size_t)max_seq * (H > D ? H : D), sizeof(float));
    m->k = (float*)calloc((size_t)max_seq * KV, sizeof(float));
    m->v = (float*)calloc((size_t)max_seq * KV, sizeof(float));
    m->hb = (float*)calloc((size_t)max_seq * hp->n_ff, sizeof(float));
    m->hb2 = (float*)calloc((size_t)max_seq * hp->n_ff, sizeof(float));
    m->logits = (float*)calloc((size_t)hp->n_vocab, sizeof(float));
    if (!m->kc || !m->vc || !m->x || !m->xb || !m->q || !m->k || !m->v || !m->hb || !m->hb2) {
        snprintf(g_err, sizeof g_err, "out of memory");
        tfo_model_destroy(m);
        return NULL;
    }
    return m;
}

static void mm(tfo_model* m, float* c, const float* a, const tfo_tensor* w, int rows) {
    tfo_matmul(c, a, w->ggml_type, w->data, (int)w->ne[1], (int)w->ne[0], rows, m->threads);
}

/* src/model.cpp:85-89 */
static void bias(float* x, const tfo_tensor* b, int n) {
    if (!b) return;
    const float* bp = (const float*)b->data;
    for (int i = 0; i < n; ++i) x[i] += bp[i];
}

/* src/model.cpp:108-142 (seq == 1) and :144-181 (seq rows at positions n_pos..). For seq == 1
 * attention runs over the cache (attn_decode), otherwise over the fresh chunk (attn_prefill). */
static void layer(tfo_model* m, int li, float* x, int seq) {
    const tfo_hparams* hp = &m->hp;
    const layer_w* L = &m->layers[li];
    const int D = hp->n_embd, H = hp->n_head * hp->head_dim, KV = hp->n_kv_head * hp->head_dim;
    for (int i = 0; i < seq; ++i)
        tfo_rmsnorm(m->xb + (size_t)i * D, x + (size_t)i * D, (const float*)L->attn_norm->data, D, hp->rms_eps);
    mm(m, m->q, m->xb, L->wq, seq);
    mm(m, m->k, m->xb, L->wk, seq);
    mm(m, m->v, m->xb, L->wv, seq);
    for (int i = 0; i < seq; ++i) {
        bias(m->q + (size_t)i * H, L->bq, H);
        bias(m->k + (size_t)i * KV, L->bk, KV);
        bias(m->v + (size_t)i * KV, L->bv, KV);
    }
    tfo_rope(m->q, seq, hp->n_head, hp->head_dim, m->n_pos, m->freq);
    tfo_rope(m->k, seq, hp->n_kv_head, hp->head_dim, m->n_pos, m->freq);
    float* kl = m->kc + (size_t)li * m->max_seq * KV;
    float* vl = m->vc + (size_t)li * m->max_seq * KV;
    memcpy(kl + (size_t)m->n_pos * KV, m->k, (size_t)seq * KV * sizeof(float));
    memcpy(vl + (size_t)m->n_pos * KV, m->v, (size_t)seq * KV * sizeof(float));
    if (seq == 1)
        tfo_attn_decode(m->xb, m->q, kl, vl, m->n_pos + 1, hp->n_head, hp->n_kv_head, hp->head_dim);
    else
        tfo_attn_prefill(m->xb, m->q, m->k, m->v, seq, hp->n_head, hp->n_kv_head, hp->head_dim);
    mm(m, m->q, m->xb, L->wo, seq);
    for (int i = 0; i < seq; ++i) tfo_add_inplace(x + (size_t)i * D, m->q + (size_t)i * D, D);
    for (int i = 0; i < seq; ++i)
        tfo_rmsnorm(m->xb + (size_t)i * D, x + (size_t)i * D, (const float*)L->ffn_norm->data, D, hp->rms_eps);
    mm(m, m->hb, m->xb, L->gate, seq);
    mm(m, m->hb2, m->xb, L->up, seq);
    tfo_silu_mul(m->hb, m->hb2, seq * hp->n_ff);
    mm(m, m->xb, m->hb, L->down, seq);
    for (int i = 0; i < seq; ++i) tfo_add_inplace(x + (size_t)i * D, m->xb + (size_t)i * D, D);
}

static void head(tfo_model* m, const float* xlast, float* logits) {
    tfo_rmsnorm(m->xb, xlast, (const float*)m->output_norm->data, m->hp.n_embd, m->hp.rms_eps);
    mm(m, logits ? logits : m->logits, m->xb, m->output, 1);
}

/* src/model.cpp:183-195 */
int tfo_model_prefill(tfo_model* m, const int* tokens, int n, float* logits) {
    if (n <= 0) return 0;
    if (m->n_pos + n > m->max_seq) {
        snprintf(g_err, sizeof g_err, "prefill exceeds max_seq");
        return -1;
    }
    const int D = m->hp.n_embd;
    for (int i = 0; i < n; ++i)
        tfo_dequant_row(m->x + (size_t)i * D, m->tok_embd->ggml_type, m->tok_embd->data, D, tokens[i]);
    for (int li = 0; li < m->hp.n_layer; ++li) layer(m, li, m->x, n);
    head(m, m->x + (size_t)(n - 1) * D, logits);
    m->n_pos += n;
    return 0;
}

/* src/model.cpp:197-208 */
int tfo_model_decode(tfo_model* m, int token, float* logits) {
    if (m->n_pos + 1 > m->max_seq) {
        snprintf(g_err, sizeof g_err, "decode exceeds max_seq");
        return -1;
    }
    tfo_dequant_row(m->x, m->tok_embd->ggml_type, m->tok_embd->data, m->hp.n_embd, token);
    for (int li = 0; li < m->hp.n_layer; ++li) layer(m, li, m->x, 1);
    head(m, m->x, logits);
    m->n_pos += 1;
    return 0;
}

/* src/model.cpp:80-83 */
void tfo_model_reset(tfo_model* m) {
    m->n_pos = 0;
    const size_t kvn = (size_t)m->hp.n_layer * m->max_seq * m->hp.n_kv_head * m->hp.head_dim;
    memset(m->kc, 0, kvn * sizeof(float));
    memset(m->vc, 0, kvn * sizeof(float));
}

int tfo_model_n_pos(const tfo_model* m) { return m->n_pos; }

void tfo_model_destroy(tfo_model* m) {
    if (!m) return;
    free(m->layers);
    free(m->freq);
    free(m->kc);
    free(m->vc);
    free(m->x);
    free(m->xb);
    free(m->q);
    free(m->k);
    free(m->v);
    free(m->hb);
    free(m->hb2);
    free(m->logits);
    free(m);
}
