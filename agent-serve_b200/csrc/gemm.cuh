// Q8_0 (and, at op level, Q4_0) GEMM on the tensor cores for M >= 16 activation rows
// (batched decode, prefill): Y[m][n] = sum_k X[m][k] * W[n][k], W in its GGUF block layout.  Replaces matmul()
// (src/matmul.cpp:22-73) at M >= 16 together with the rmsnorm / apply_bias / add_inplace /
// silu_mul / sample_greedy calls around each matmul of Model::layer_decode/layer_prefill.
//
// Arithmetic: fp32-equivalent on the f16 tensor pipe.  Every weight q*d (at most 19
// significant bits for Q8_0, 15 for Q4_0)
// is split exactly into two f16 halves Wh + Wl after a per-matrix power-of-two scale 2^sw,
// and every activation into Xh + Xl after a per-row scale 2^sx; the products Wh*Xh, Wh*Xl and
// Wl*Xh are accumulated in fp32 (the dropped Wl*Xl term is 2^-22 relative).  The result is
// scaled back by 2^-(sw+sx) exactly.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace tfb {

constexpr int GM_BN = 128;      // weight rows per CTA
constexpr int GM_BM = 128;      // activation rows per CTA
constexpr int GM_BK = 64;       // k per pipeline stage (two Q8_0 blocks)
constexpr int GM_DQ_THREADS = 512;  // tcgen05 kernel: dequantising threads, 4 per weight row
constexpr int GM_TC_THREADS = GM_DQ_THREADS + 96;  // + an activation-copy warp, an MMA warp, a weight-copy warp
constexpr int GM_X_WARP = GM_DQ_THREADS / 32;      // warp roles after the dequantising warps
constexpr int GM_MMA_WARP = GM_X_WARP + 1;
constexpr int GM_W_WARP = GM_X_WARP + 2;
constexpr int GM_TC_TAIL = 512;     // tcgen05 kernel: shared bytes of barriers and flags
constexpr int GM_MIN_M = 16;    // below this the GEMV kernel runs
constexpr int GM_WPF = 4;       // tcgen05 GEMM: weight stages in flight per thread (registers)

// Activation preparation: optional embedding lookup, optional RMSNorm, then the f16 split.
struct XPrepArgs {
    const float* x;       // [M][ldx] input (or the residual stream for RMSNorm)
    int ldx;
    const float* norm_w;  // RMSNorm weights or nullptr (no norm)
    float eps;
    const uint8_t* embd;  // embedding table: rows are looked up from tokens[] (then x_out)
    int embd_type;
    long long embd_rb;
    int n_vocab;
    const int* tokens;
    float* x_out;         // [M][ldx]: the embedded rows (the residual stream)
    int K, M;
    // xh / xl: the halves in the GEMM's operand layout: k-stage kc (64 columns) of rows
    // [0, mp) is one block of mp * 128 bytes at kc * mp * 128, row r of it at the 128-byte
    // swizzled K-major offsets of an 8-row atom (r / 8) * 1024 (gm_kint_off), so the NT rows
    // of a tile are one contiguous NT * 128-byte block per stage; mp = gemm_x_rows(M) (set
    // by xprep_launch)
    __half* xh;
    __half* xl;
    int* sx;              // [M] scale exponents
    int* err;
    int mp;
};

struct GemmArgs {
    const uint8_t* W;     // Q8_0 rows (Q4_0 rows when wq4)
    int wq4;              // 1: Q4_0 weights (18-byte blocks) on the tcgen05 path
    long long rb;
    int N, K, M;
    int sw;               // weight scale exponent
    const __half* xh;     // XPrepArgs' operand layout (mp = gemm_x_rows(M), set by gemm_launch)
    const __half* xl;
    const int* sx;        // [M]
    int mp;
    // epilogue (GemvArgs conventions)
    int epi;              // EPI_STORE / EPI_RESID / EPI_SWIGLU (interleaved gate/up rows) / EPI_ARGMAX
    float* y;
    int ldy;
    const float* bias;
    float* resid;
    int ldr;
    unsigned long long* keys;  // EPI_ARGMAX: one key per activation row
    int store_logits;          // EPI_ARGMAX: also store the logits in y
    // split-K (grid.z = ksplit > 1): the splits of a tile are one thread-block cluster and sum
    // through distributed shared memory; ws / tile_cnt serve the non-cluster reduction of
    // gemm_epilogue (global workspace, tile arrivals)
    int ksplit;
    float* ws;
    unsigned* tile_cnt;
    int* err;
    // optional pipeline trace of CTA (0, 0, 0) of the tcgen05 kernel (nullptr: off): clock64()
    // stamps at the GM_TR_* slots below (gemm_set_trace)
    unsigned long long* trace;
};

// trace slots: kernel entry, set-up done, copy warp past its wait, every MMA completed, epilogue
// done; per weight chunk c its copy issue; per k stage kc: dequantising warp 0 past the chunk wait,
// past its waits and arrived, the last dequantising warp's arrival (stamp << 5 | warp); the MMA
// thread past its wait and committed; the activation stage's copy issue
constexpr int GM_TR_CHUNK = 8, GM_TR_DQ = 72, GM_TR_MMA = 584, GM_TR_X = 840, GM_TR_SLOTS = 968, GM_TR_MAXK = 128;
// every later gemm_launch of this process traces into buf (device memory, GM_TR_SLOTS words; nullptr: off)
void gemm_set_trace(unsigned long long* buf);

constexpr int GM_ROW_PAD = 256;  // activation buffers hold a multiple of this many rows

constexpr int GM_MAX_SPLIT = 8;
// workspace floats / tile counters the split-K path needs for `num_sms` SMs
inline size_t gemm_ws_floats(int num_sms) { return (size_t)GM_MAX_SPLIT * num_sms * GM_BN * GM_ROW_PAD; }
inline int gemm_tile_counters(int num_sms) { return 2 * num_sms; }  // arrivals, departures per tile
// activation rows per tcgen05 CTA tile for an M-row GEMM (32, 64, 128 or 256: the smallest
// that holds M up to 128 rows, 256 above; TFB200_GEMM_NT=128 keeps 128-row tiles at every M)
int gemm_tile_rows(int M);
// rows per k-stage block of the activation operand layout for an M-row GEMM
int gemm_x_rows(int M);
// k splits for an N x M GEMM: enough CTAs to cover the SMs once when the tiles alone do not
inline int gemm_pick_split(int N, int M, int K, int num_sms) {
    const int mt = gemm_tile_rows(M);  // activation rows per CTA tile
    const int tiles = ((N + GM_BN - 1) / GM_BN) * ((M + mt - 1) / mt);
    if (tiles >= num_sms) return 1;
    int s = num_sms / tiles;
    const int nk = K / GM_BK;
    s = s > GM_MAX_SPLIT ? GM_MAX_SPLIT : s;
    s = s > nk / 2 ? nk / 2 : s;
    return s < 1 ? 1 : s;
}

// End of a step at M rows: next tokens from the greedy keys, positions, generated ids.
struct FinishArgs {
    int M;
    unsigned long long* keys;  // reset to 0
    int* tok_next;
    int* pos;
    const int* slots;
    int* hist;                 // [hist_cap][M] or nullptr
    StepCtl* ctl;
    int argmax;                // 0: positions only (a step without lm_head)
};

cudaError_t xprep_launch(const XPrepArgs& a, cudaStream_t st);

cudaError_t gemm_launch(const GemmArgs& a, cudaStream_t st);
cudaError_t finish_launch(const FinishArgs& a, cudaStream_t st);
// per-matrix sw of host-resident blocks (block_bytes 34 for Q8_0, 18 for Q4_0)
int q8_scale_exponent(const uint8_t* host_blocks, size_t nbytes, int block_bytes = 34);
// whether gemm_launch takes Q4_0 weights (the tcgen05 kernel does)
bool gemm_takes_q4();
int q8_exponent_from_dbits(unsigned max_abs_d_bits);
// sw of device-resident Q8_0 blocks (synchronises `st`); scratch: one device unsigned
cudaError_t q8_scale_exponent_device(const uint8_t* W, long long n_blocks, unsigned* scratch, int* sw, cudaStream_t st,
                                     int block_bytes = 34);  // 18 for Q4_0 blocks

}  // namespace tfb
