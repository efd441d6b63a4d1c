// Op-level C-ABI (tf_op_*): each reference op on device pointers, for the cfg3 kernel sweep
// and for op-by-op parity against the reference.
#include <mutex>
#include <string>

#include "attention.cuh"
#include "engine.cuh"
#include "gemm.cuh"

namespace tfb {
cudaError_t launch_rmsnorm(float* out, const float* x, const float* w, int n, int rows, float eps, cudaStream_t st);
cudaError_t launch_silu_mul(float* g, const float* u, int n, cudaStream_t st);
cudaError_t launch_softmax(float* x, int n, int rows, cudaStream_t st);
cudaError_t launch_rope(float* x, int seq, int nh, int hd, int pos0, const float* freq, cudaStream_t st);
cudaError_t launch_argmax(const float* logits, int n, int rows, int* out, cudaStream_t st);
cudaError_t launch_dequant_rows(float* out, int t, const void* W, int N, int K, const int* rows, int n_rows, int* err,
                                cudaStream_t st);
}  // namespace tfb

namespace tfb {

// Status word of the op-level kernels: a __device__ variable has its own instance on every
// device that loads the module, so each device has one word, and nothing is allocated.
// Kernels record the first ERR_* code with atomicCAS; tf_op_device_error reads and clears it.
static __device__ int op_dev_err;

int op_err_word(int** out) {
    static std::mutex mu;
    static int* words[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return set_error("device ordinal out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!words[dev]) {
        e = cudaGetSymbolAddress((void**)&words[dev], op_dev_err);
        if (e != cudaSuccess) {
            words[dev] = nullptr;
            return set_error(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        }
    }
    *out = words[dev];
    return 0;
}

}  // namespace tfb

using namespace tfb;

namespace {
int op_status(cudaError_t e, const char* what) {
    if (e != cudaSuccess) return set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return 0;
}
bool type_ok(int t) { return t == T_F32 || t == T_F16 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q8_0 || t == T_Q6_K; }
int err_word(int** out) { return op_err_word(out); }
}  // namespace

extern "C" {

int tf_op_q8_scale(const void* W, int N, int K, int* sw, void* stream) {
    if (!W || !sw || N <= 0 || K <= 0 || K % 32) return set_error("bad Q8_0 matrix");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned* scratch = nullptr;
    if (op_status(cudaMallocAsync((void**)&scratch, sizeof(unsigned), st), "alloc")) return -1;
    const int rc = op_status(q8_scale_exponent_device(static_cast<const uint8_t*>(W), (long long)N * (K / 32), scratch,
                                                      sw, st),
                             "q8_scale");
    cudaFreeAsync(scratch, st);
    return rc;
}

}  // extern "C"

namespace {
// C = A W^T on the tcgen05 GEMM for Q8_0 or Q4_0 weights (t), with the matrix scale sw.
int matmul_tc(float* C, const float* A, int t, const void* W, int N, int K, int M, int sw, void* stream) {
    if (N <= 0 || K <= 0 || M < GM_MIN_M || K % GM_BK) return set_error("tensor-core GEMM needs M >= 16 and K % 64 == 0");
    if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(W) & 3))
        return set_error("A must be 16-byte and W 4-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* err = nullptr;
    if (err_word(&err)) return -1;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t rows = (size_t)(M + GM_ROW_PAD - 1) / GM_ROW_PAD * GM_ROW_PAD;
    __half *xh = nullptr, *xl = nullptr;
    int* sx = nullptr;
    float* ws = nullptr;
    unsigned* cnt = nullptr;
    const int ks = gemm_pick_split(N, M, K, sms);
    int rc = op_status(cudaMallocAsync((void**)&xh, rows * K * sizeof(__half), st), "alloc");
    if (!rc) rc = op_status(cudaMallocAsync((void**)&xl, rows * K * sizeof(__half), st), "alloc");
    if (!rc) rc = op_status(cudaMallocAsync((void**)&sx, rows * sizeof(int), st), "alloc");
    if (!rc && ks > 1) rc = op_status(cudaMallocAsync((void**)&ws, (size_t)ks * M * N * sizeof(float), st), "alloc");
    if (!rc && ks > 1)
        rc = op_status(cudaMallocAsync((void**)&cnt, (size_t)gemm_tile_counters(sms) * sizeof(unsigned), st), "alloc");
    if (!rc && ks > 1) rc = op_status(cudaMemsetAsync(cnt, 0, (size_t)gemm_tile_counters(sms) * sizeof(unsigned), st), "memset");
    if (!rc) rc = op_status(cudaMemsetAsync(xh, 0, rows * K * sizeof(__half), st), "memset");
    if (!rc) rc = op_status(cudaMemsetAsync(xl, 0, rows * K * sizeof(__half), st), "memset");
    if (!rc) {
        XPrepArgs p;
        memset(&p, 0, sizeof(p));
        p.x = A;
        p.ldx = K;
        p.K = K;
        p.M = M;
        p.xh = xh;
        p.xl = xl;
        p.sx = sx;
        p.err = err;
        rc = op_status(xprep_launch(p, st), "xprep");
    }
    if (!rc) {
        GemmArgs g;
        memset(&g, 0, sizeof(g));
        g.W = static_cast<const uint8_t*>(W);
        g.rb = row_bytes(t, K);
        g.wq4 = t == T_Q4_0 ? 1 : 0;
        g.N = N;
        g.K = K;
        g.M = M;
        g.sw = sw;
        g.xh = xh;
        g.xl = xl;
        g.sx = sx;
        g.epi = EPI_STORE;
        g.y = C;
        g.ldy = N;
        g.ksplit = ks;
        g.ws = ws;
        g.tile_cnt = cnt;
        g.err = err;
        rc = op_status(gemm_launch(g, st), "gemm");
    }
    void* bufs[] = {xh, xl, sx, ws, cnt};
    for (void* b : bufs)
        if (b) cudaFreeAsync(b, st);
    return rc;
}

}  // namespace

extern "C" {

int tf_op_matmul_q8_tc(float* C, const float* A, const void* W, int N, int K, int M, int sw, void* stream) {
    return matmul_tc(C, A, T_Q8_0, W, N, K, M, sw, stream);
}

int tf_op_weight_scale(const void* W, int t, int N, int K, int* sw, void* stream) {
    if (t != T_Q8_0 && t != T_Q4_0) return set_error("tensor-core path takes Q8_0 or Q4_0 weights");
    if (!W || !sw || N <= 0 || K <= 0 || K % 32) return set_error("bad weight matrix");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned* scratch = nullptr;
    if (op_status(cudaMallocAsync((void**)&scratch, sizeof(unsigned), st), "alloc")) return -1;
    const int rc = op_status(q8_scale_exponent_device(static_cast<const uint8_t*>(W), (long long)N * (K / 32), scratch,
                                                      sw, st, t == T_Q8_0 ? 34 : 18),
                             "weight_scale");
    cudaFreeAsync(scratch, st);
    return rc;
}

int tf_op_matmul_tc(float* C, const float* A, int t, const void* W, int N, int K, int M, int sw, void* stream) {
    if (t != T_Q8_0 && t != T_Q4_0) return set_error("tensor-core path takes Q8_0 or Q4_0 weights");
    return matmul_tc(C, A, t, W, N, K, M, sw, stream);
}

int tf_op_matmul(float* C, const float* A, int t, const void* W, int N, int K, int M, void* stream) {
    if (!type_ok(t)) return set_error("unsupported ggml type");
    if (N <= 0 || K <= 0 || M < 0) return set_error("bad matmul shape");
    if (K % 32 || K % blk_elems(t)) return set_error("row length not divisible by block size");
    if (M == 0) return 0;
    if (t == T_F32 && (reinterpret_cast<uintptr_t>(W) & 3)) return set_error("F32 weights must be 4-byte aligned");
    if (reinterpret_cast<uintptr_t>(A) & 15) return set_error("A must be 16-byte aligned");
    if ((t == T_Q8_0 || t == T_Q4_0) && M >= GM_MIN_M && K % GM_BK == 0 && !(reinterpret_cast<uintptr_t>(W) & 3)) {
        // M >= 16: the tensor-core GEMM (scale of the matrix, then the GEMM)
        int sw = 0;
        if (tf_op_weight_scale(W, t, N, K, &sw, stream)) return -1;
        return matmul_tc(C, A, t, W, N, K, M, sw, stream);
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int* err = nullptr;
    if (err_word(&err)) return -1;
    if (op_status(gemv_init_attrs(), "cudaFuncSetAttribute")) return -1;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tile = gemv_max_rows(K);
    for (int m0 = 0; m0 < M; m0 += tile) {
        GemvArgs a;
        memset(&a, 0, sizeof(a));
        a.W = static_cast<const uint8_t*>(W);
        a.wtype = t;
        a.K = K;
        a.rb = row_bytes(t, K);
        a.n_items = N;
        a.P = 1;
        a.M = M - m0 < tile ? M - m0 : tile;
        a.err = err;
        gemv_plan(a);
        a.pro = PRO_COPY;
        a.x = A + (size_t)m0 * K;
        a.ldx = K;
        a.epi = EPI_STORE;
        a.y = C + (size_t)m0 * N;
        a.ldy = N;
        if (op_status(gemv_launch(a, gemv_grid(a, sms), st, false), "gemv")) return -1;
    }
    return 0;
}

int tf_op_dequant_rows(float* out, int t, const void* W, int N, int K, const int* rows, int n_rows, void* stream) {
    if (!type_ok(t)) return set_error("unsupported ggml type");
    if (N <= 0 || K <= 0 || K % blk_elems(t)) return set_error("bad matrix shape");
    if (n_rows <= 0) return 0;
    int* err = nullptr;
    if (err_word(&err)) return -1;
    return op_status(launch_dequant_rows(out, t, W, N, K, rows, n_rows, err, static_cast<cudaStream_t>(stream)),
                     "dequant_rows");
}

int tf_op_gemm_trace(unsigned long long* buf) {
    gemm_set_trace(buf);
    return 0;
}

int tf_op_device_error(void* stream, int* code) {
    if (!code) return set_error("code must not be null");
    *code = 0;
    int* err = nullptr;
    if (err_word(&err)) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int h = 0;
    if (op_status(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync")) return -1;
    if (op_status(cudaStreamSynchronize(st), "cudaStreamSynchronize")) return -1;
    if (h && op_status(cudaMemsetAsync(err, 0, sizeof(int), st), "cudaMemsetAsync")) return -1;
    *code = h;
    return 0;
}

int tf_op_rmsnorm(float* out, const float* x, const float* w, int n, int rows, float eps, void* stream) {
    if (rows <= 0) return 0;
    return op_status(launch_rmsnorm(out, x, w, n, rows, eps, static_cast<cudaStream_t>(stream)), "rmsnorm");
}

int tf_op_silu_mul(float* gate, const float* up, int n, void* stream) {
    if (n <= 0) return 0;
    return op_status(launch_silu_mul(gate, up, n, static_cast<cudaStream_t>(stream)), "silu_mul");
}

int tf_op_softmax(float* x, int n, int rows, void* stream) {
    if (rows <= 0 || n <= 0) return 0;
    return op_status(launch_softmax(x, n, rows, static_cast<cudaStream_t>(stream)), "softmax");
}

int tf_op_rope(float* x, int seq, int n_heads, int head_dim, int pos0, const float* freq, void* stream) {
    if (seq <= 0) return 0;
    return op_status(launch_rope(x, seq, n_heads, head_dim, pos0, freq, static_cast<cudaStream_t>(stream)), "rope");
}

int tf_op_attn_decode(float* out, const float* q, const void* k_cache, const void* v_cache, int kv_type, int cap,
                      int n_pos, int n_heads, int n_kv_heads, int head_dim, void* stream) {
    if (n_pos <= 0 || n_pos > cap) return set_error("n_pos must be in [1, cap]");
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return set_error("n_heads must be a positive multiple of n_kv_heads");
    if (head_dim <= 0 || head_dim % 8) return set_error("head_dim must be a positive multiple of 8");
    int* err = nullptr;
    if (err_word(&err)) return -1;
    const int n_split = attn_pick_split(n_pos);
    float* part = nullptr;
    unsigned* counters = nullptr;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_split > 1) {
        if (op_status(cudaMallocAsync((void**)&part, sizeof(float) * n_heads * n_split * (head_dim + 2), st), "alloc")) return -1;
        if (op_status(cudaMallocAsync((void**)&counters, sizeof(unsigned) * n_kv_heads, st), "alloc")) return -1;
        cudaMemsetAsync(counters, 0, sizeof(unsigned) * n_kv_heads, st);
    }
    AttnArgs a;
    memset(&a, 0, sizeof(a));
    a.qkv = q;
    a.ld_qkv = n_heads * head_dim;
    a.kc = const_cast<void*>(k_cache);
    a.vc = const_cast<void*>(v_cache);
    a.slot_stride = 0;
    a.cap = cap;
    a.kv_type = kv_type;
    a.n_head = n_heads;
    a.n_kv = n_kv_heads;
    a.hd = head_dim;
    a.n_split = n_split;
    a.part = part;
    a.counters = counters;
    a.out = out;
    a.ld_out = n_heads * head_dim;
    a.fresh = 0;
    a.n_pos_fixed = n_pos;
    a.err = err;
    int rc = op_status(attn_decode_launch(a, 1, st, false), "attn_decode");
    if (part) cudaFreeAsync(part, st);
    if (counters) cudaFreeAsync(counters, st);
    return rc;
}

int tf_op_attn_prefill(float* out, const float* q, const float* k, const float* v, int seq, int n_heads, int n_kv_heads,
                       int head_dim, void* stream) {
    if (seq <= 0) return 0;
    if (n_heads % n_kv_heads) return set_error("n_heads must be a multiple of n_kv_heads");
    PrefillAttnArgs a{q, k, v, out, seq, n_heads, n_kv_heads, head_dim};
    return op_status(attn_prefill_launch(a, static_cast<cudaStream_t>(stream)), "attn_prefill");
}

int tf_op_argmax(const float* logits, int n, int rows, int* out, void* stream) {
    if (rows <= 0 || n <= 0) return 0;
    return op_status(launch_argmax(logits, n, rows, out, static_cast<cudaStream_t>(stream)), "argmax");
}

}  // extern "C"
