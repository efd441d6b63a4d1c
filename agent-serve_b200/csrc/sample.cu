// Temperature / top-p sampling of one row of logits on the device: sample_logits
// (src/sampler.cpp:15-52).  The caller draws the uniform r in [0, 1) with its own generator
// (the reference's std::mt19937 + uniform_real_distribution<float>, one draw per sampled
// token, src/main.cpp:109-114), so the random stream stays on the host.
//
// Order of work, as the reference: indices sorted by logit, descending (a stable radix sort:
// equal logits keep index order); p_i = exp((l_i - max) / T); normalise by the sum; with
// top_p < 1 keep the shortest prefix whose mass reaches top_p and renormalise it; return the
// first index whose running mass reaches r (else the last kept one).  The sums and running
// masses are formed in double and rounded to float where the reference holds floats; they
// differ from the reference's sequential float sums by rounding only.
#include <cub/device/device_radix_sort.cuh>

#include "sample.cuh"

namespace tfb {

constexpr int SM_THREADS = 1024;

// descending-order radix keys of the logits (monotone map of the float bits, inverted)
__global__ void tf_sample_keys_kernel(const float* logits, int n, uint32_t* keys, int* vals) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t u = __float_as_uint(logits[i]);
    const uint32_t asc = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    keys[i] = ~asc;
    vals[i] = i;
}

// Block-wide exclusive scan of one double per thread (SM_THREADS threads).
__device__ double block_exclusive_scan(double v, double* sh, double& total) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    double x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        double w = lane < SM_THREADS / 32 ? sh[lane] : 0.0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        sh[lane] = w;  // inclusive prefix of warp sums
    }
    __syncthreads();
    total = sh[SM_THREADS / 32 - 1];
    const double before = (warp > 0 ? sh[warp - 1] : 0.0) + (x - v);
    __syncthreads();
    return before;
}

// One CTA: softmax over the sorted logits, top-p cut, pick with r.
__global__ void __launch_bounds__(SM_THREADS) tf_sample_pick_kernel(const float* logits, const int* order, int n,
                                                                 float temperature, float top_p, float r, int* out) {
    __shared__ double sh[SM_THREADS / 32];
    __shared__ int found;
    const int tid = threadIdx.x;
    const int per = (n + SM_THREADS - 1) / SM_THREADS;
    const int b = tid * per, e = min(n, b + per);  // this thread's contiguous slice of the order
    const float mx = logits[order[0]];
    // p_i = exp((l - max) / T) and their sum
    double part = 0.0;
    for (int i = b; i < e; ++i) part += (double)expf((logits[order[i]] - mx) / temperature);
    double s_tot;
    block_exclusive_scan(part, sh, s_tot);
    const float s = (float)s_tot;
    // top-p: the shortest prefix with mass >= top_p
    int last = n;
    double z = 1.0;
    if (top_p < 1.0f) {
        double run = 0.0;
        for (int i = b; i < e; ++i) run += (double)(expf((logits[order[i]] - mx) / temperature) / s);
        double tot;
        const double before = block_exclusive_scan(run, sh, tot);
        if (tid == 0) found = n;
        __syncthreads();
        double acc = before;
        if (acc < (double)top_p || tid == 0) {
            for (int i = b; i < e; ++i) {
                acc += (double)(expf((logits[order[i]] - mx) / temperature) / s);
                if (acc >= (double)top_p) {
                    atomicMin(&found, i + 1);
                    break;
                }
            }
        }
        __syncthreads();
        last = found;
        // z: mass of the kept prefix
        double zp = 0.0;
        for (int i = b; i < min(e, last); ++i) zp += (double)(expf((logits[order[i]] - mx) / temperature) / s);
        block_exclusive_scan(zp, sh, z);
    }
    const float zf = (float)z;
    // pick: the first kept index whose running (renormalised) mass reaches r
    double run = 0.0;
    for (int i = b; i < min(e, last); ++i) {
        float p = expf((logits[order[i]] - mx) / temperature) / s;
        if (top_p < 1.0f) p /= zf;
        run += (double)p;
    }
    double tot;
    const double before = block_exclusive_scan(run, sh, tot);
    if (tid == 0) found = last;  // none reached: the last kept index
    __syncthreads();
    double acc = before;
    if (acc < (double)r || tid == 0) {  // earlier slices already reached r otherwise
        for (int i = b; i < min(e, last); ++i) {
            float p = expf((logits[order[i]] - mx) / temperature) / s;
            if (top_p < 1.0f) p /= zf;
            acc += (double)p;
            if ((double)r <= acc) {
                atomicMin(&found, i);
                break;
            }
        }
    }
    __syncthreads();
    if (tid == 0) *out = order[found < last ? found : last - 1];
}

// Scratch for one sampler (sizes for n logits).
struct SampleScratch {
    uint32_t* keys_in = nullptr;
    uint32_t* keys_out = nullptr;
    int* vals_in = nullptr;
    int* vals_out = nullptr;
    void* temp = nullptr;
    size_t temp_bytes = 0;
    int* out = nullptr;
    int n = 0;
};

SampleScratch* sample_scratch_create(int n) {
    SampleScratch* s = new SampleScratch();
    s->n = n;
    cudaError_t e = cudaSuccess;
    if (cub::DeviceRadixSort::SortPairs(nullptr, s->temp_bytes, s->keys_in, s->keys_out, s->vals_in, s->vals_out, n) !=
        cudaSuccess)
        e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaMalloc(&s->keys_in, sizeof(uint32_t) * n);
    if (e == cudaSuccess) e = cudaMalloc(&s->keys_out, sizeof(uint32_t) * n);
    if (e == cudaSuccess) e = cudaMalloc(&s->vals_in, sizeof(int) * n);
    if (e == cudaSuccess) e = cudaMalloc(&s->vals_out, sizeof(int) * n);
    if (e == cudaSuccess) e = cudaMalloc(&s->temp, s->temp_bytes > 0 ? s->temp_bytes : 16);
    if (e == cudaSuccess) e = cudaMalloc(&s->out, sizeof(int));
    if (e != cudaSuccess) {
        sample_scratch_destroy(s);
        return nullptr;
    }
    return s;
}

void sample_scratch_destroy(SampleScratch* s) {
    if (!s) return;
    void* p[] = {s->keys_in, s->keys_out, s->vals_in, s->vals_out, s->temp, s->out};
    for (void* q : p)
        if (q) cudaFree(q);
    delete s;
}

cudaError_t sample_launch(SampleScratch* s, const float* logits, int n, float temperature, float top_p, float r,
                          cudaStream_t st) {
    if (!s || n > s->n || n <= 0) return cudaErrorInvalidValue;
    tf_sample_keys_kernel<<<(n + 255) / 256, 256, 0, st>>>(logits, n, s->keys_in, s->vals_in);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    size_t tb = s->temp_bytes;
    e = cub::DeviceRadixSort::SortPairs(s->temp, tb, s->keys_in, s->keys_out, s->vals_in, s->vals_out, n, 0, 32, st);
    if (e != cudaSuccess) return e;
    tf_sample_pick_kernel<<<1, SM_THREADS, 0, st>>>(logits, s->vals_out, n, temperature, top_p, r, s->out);
    return cudaGetLastError();
}

int* sample_result(SampleScratch* s) { return s ? s->out : nullptr; }

}  // namespace tfb
