// Standalone elementwise kernels behind the op-level C-ABI (tf_op_*): the fused engine path
// does this work inside the GEMV / attention kernels; these exist so every reference op
// has a device implementation that can be checked against it one for one.
#include "common.cuh"

namespace tfb {

// rmsnorm  src/layers.cpp:7-12 (sum of squares in double; out = (x * inv) * w)
__global__ void tf_rmsnorm_kernel(float* out, const float* x, const float* w, int n, float eps) {
    __shared__ double red[32];
    const float* xr = x + (size_t)blockIdx.x * n;
    float* o = out + (size_t)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fma((double)xr[i], (double)xr[i], ss);
    ss = warp_sum_d(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    const float inv = 1.0f / sqrtf((float)(tot / n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// silu_mul  src/layers.cpp:14-19
__global__ void tf_silu_mul_kernel(float* g, const float* u, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = g[i];
        g[i] = __fmul_rn(__fdiv_rn(v, 1.0f + expf(-v)), u[i]);
    }
}

// softmax  src/layers.cpp:25-35 (one block per row)
__global__ void tf_softmax_kernel(float* x, int n) {
    __shared__ float red[32];
    __shared__ float stat;
    float* r = x + (size_t)blockIdx.x * n;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, r[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = red[0];
        for (int i = 1; i < (int)(blockDim.x >> 5); ++i) v = fmaxf(v, red[i]);
        stat = v;
    }
    __syncthreads();
    m = stat;
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(r[i] - m);
        r[i] = e;
        s += e;
    }
    s = warp_sum(s);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) v += red[i];
        stat = 1.0f / v;
    }
    __syncthreads();
    const float inv = stat;
    for (int i = threadIdx.x; i < n; i += blockDim.x) r[i] *= inv;
}

// apply_rope_many  src/attention.cpp:31-53 with the reference build's contraction
__global__ void tf_rope_kernel(float* x, int seq, int n_heads, int hd, int pos0, const float* freq) {
    const int d2 = hd / 2;
    const long long total = (long long)seq * n_heads * d2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int j = (int)(i % d2);
        const long long th = i / d2;
        const int t = (int)(th / n_heads);
        float* v = x + th * hd;
        const float ang = __fmul_rn((float)(pos0 + t), freq[j]);
        const float c = cosf(ang), s = sinf(ang);
        const float x0 = v[j], x1 = v[j + d2];
        v[j] = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
        v[j + d2] = __fmaf_rn(x0, s, __fmul_rn(x1, c));
    }
}

// sample_greedy  src/sampler.cpp:8-13: single pass, one block per row, u64 key max
__global__ void tf_argmax_kernel(const float* logits, int n, int* out) {
    __shared__ unsigned long long best;
    if (threadIdx.x == 0) best = 0ull;
    __syncthreads();
    const float* r = logits + (size_t)blockIdx.x * n;
    unsigned long long k = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long c = argmax_key(r[i], (uint32_t)i);
        k = c > k ? c : k;
    }
    atomicMax(&best, k);
    __syncthreads();
    if (threadIdx.x == 0) out[blockIdx.x] = (int)key_index(best);
}

// dequant_row  src/quant.cpp:133-145 for a list of rows
__device__ void embed_row_global(float* out, const uint8_t* E, int t, long long rb, int K, long long tok);

// Row ids outside [0, N) read nothing: the output row is zero and ERR_BAD_TOKEN is recorded.
__global__ void tf_dequant_rows_kernel(float* out, const uint8_t* W, int t, long long rb, int N, int K, const int* rows,
                                       int* err) {
    const int r = rows[blockIdx.x];
    float* o = out + (size_t)blockIdx.x * K;
    if (r < 0 || r >= N) {
        for (int e = threadIdx.x; e < K; e += blockDim.x) o[e] = 0.f;
        if (threadIdx.x == 0) atomicCAS(err, 0, ERR_BAD_TOKEN);
        return;
    }
    embed_row_global(o, W, t, rb, K, r);
}

__device__ void embed_row_global(float* out, const uint8_t* E, int t, long long rb, int K, long long tok) {
    const uint8_t* p0 = E + tok * rb;
    for (int e = threadIdx.x; e < K; e += blockDim.x) {
        float v;
        if (t == T_F32) {
            v = reinterpret_cast<const float*>(p0)[e];
        } else if (t == T_F16) {
            v = h2f((uint32_t)p0[2 * e] | ((uint32_t)p0[2 * e + 1] << 8));
        } else if (t == T_Q8_0) {
            const uint8_t* p = p0 + (e / 32) * 34;
            v = __fmul_rn(h2f((uint32_t)p[0] | ((uint32_t)p[1] << 8)), (float)(int8_t)p[2 + e % 32]);
        } else if (t == T_Q4_0) {
            const uint8_t* p = p0 + (e / 32) * 18;
            const int j = e % 32;
            const uint32_t q = p[2 + (j & 15)];
            v = __fmul_rn(h2f((uint32_t)p[0] | ((uint32_t)p[1] << 8)), (float)((int)(j < 16 ? (q & 15u) : (q >> 4)) - 8));
        } else if (t == T_Q4_1) {
            const uint8_t* p = p0 + (e / 32) * 20;
            const int j = e % 32;
            const uint32_t q = p[4 + (j & 15)];
            v = __fmaf_rn((float)(j < 16 ? (q & 15u) : (q >> 4)), h2f((uint32_t)p[0] | ((uint32_t)p[1] << 8)),
                          h2f((uint32_t)p[2] | ((uint32_t)p[3] << 8)));
        } else {  // Q6_K
            const uint8_t* p = p0 + (e / 256) * 210;
            const int w = e % 256, h = w / 128, r = w % 128, tq = r / 32, l = r % 32;
            const uint8_t* ql = p + 64 * h + ((tq & 1) ? 32 : 0);
            const uint8_t* qh = p + 128 + 32 * h;
            const int8_t sc = reinterpret_cast<const int8_t*>(p + 192 + 8 * h + 2 * tq)[l >> 4];
            const uint32_t lo = (tq >= 2) ? (ql[l] >> 4) : (ql[l] & 15u);
            const uint32_t hi = (qh[l] >> (2 * tq)) & 3u;
            v = __fmul_rn(__fmul_rn(h2f((uint32_t)p[208] | ((uint32_t)p[209] << 8)), (float)sc),
                          (float)((int)(lo | (hi << 4)) - 32));
        }
        out[e] = v;
    }
}

cudaError_t launch_rmsnorm(float* out, const float* x, const float* w, int n, int rows, float eps, cudaStream_t st) {
    tf_rmsnorm_kernel<<<rows, 256, 0, st>>>(out, x, w, n, eps);
    return cudaGetLastError();
}
cudaError_t launch_silu_mul(float* g, const float* u, int n, cudaStream_t st) {
    tf_silu_mul_kernel<<<(n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096, 256, 0, st>>>(g, u, n);
    return cudaGetLastError();
}
cudaError_t launch_softmax(float* x, int n, int rows, cudaStream_t st) {
    tf_softmax_kernel<<<rows, 256, 0, st>>>(x, n);
    return cudaGetLastError();
}
cudaError_t launch_rope(float* x, int seq, int nh, int hd, int pos0, const float* freq, cudaStream_t st) {
    const long long total = (long long)seq * nh * (hd / 2);
    int blocks = (int)((total + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    tf_rope_kernel<<<blocks, 256, 0, st>>>(x, seq, nh, hd, pos0, freq);
    return cudaGetLastError();
}
cudaError_t launch_argmax(const float* logits, int n, int rows, int* out, cudaStream_t st) {
    tf_argmax_kernel<<<rows, 1024, 0, st>>>(logits, n, out);
    return cudaGetLastError();
}
cudaError_t launch_dequant_rows(float* out, int t, const void* W, int N, int K, const int* rows, int n_rows, int* err,
                                cudaStream_t st) {
    tf_dequant_rows_kernel<<<n_rows, 256, 0, st>>>(out, static_cast<const uint8_t*>(W), t, row_bytes(t, K), N, K, rows,
                                                   err);
    return cudaGetLastError();
}

}  // namespace tfb
