// tf_op_attn_decode_noalloc: decode attention over a cache with its split-K scratch in a
// fixed, statically allocated device array instead of cudaMallocAsync.
//
// Who needs it: callers that cannot allocate device memory while they run a step.  The
// engine sizes its KV cache to fill the HBM it is given, so an embedder that has handed the
// rest of the device to its own arena has no room left for a per-call allocation, and
// cudaMallocAsync / cudaFreeAsync on such a device can fail mid-step.  This entry point
// allocates nothing: the partial results and the per-head arrival counters live in the
// file-scope arrays below, whose device addresses are looked up once per device.
//
// Limits and rules:
//  * scratch holds at most NA_PART_FLOATS floats of partials: n_heads * n_split * (head_dim+2)
//    with n_split = ceil(n_pos / 64); larger calls are rejected with an error, nothing runs.
//  * n_kv_heads <= NA_MAX_KV.
//  * the per-head arrival counters must be zero when a launch starts; every call clears the
//    ones it uses with cudaMemsetAsync on its stream before the launch (a memset allocates
//    nothing), so a call that an earlier call's failed wait left non-zero still starts
//    clean.  The partials need no initial value (each is written before it is read).
//  * device-side problems (a bounded wait that gave up) go to the op-level status word of
//    the device, which tf_op_device_error reads and clears: the kernel cannot return them
//    to this call.
//  * the scratch is shared by every call on a device: two calls that overlap in time (on
//    two streams, or from two host threads) race on it and give wrong results.  Serialise
//    them (one stream, or an event between them).
//  * the first call on a device does the set-up (symbol lookup, kernel attributes), which
//    is not a stream operation: make that first call before any stream capture.  The set-up
//    is guarded by a mutex, so first calls from several host threads are safe; later calls
//    still must not overlap in time.
#include <mutex>
#include <string>

#include "attention.cuh"
#include "engine.cuh"

namespace {

constexpr long long NA_PART_FLOATS = 1 << 19;  // 2 MiB of partials
constexpr int NA_MAX_KV = 64;
constexpr int NA_MAX_DEV = 64;

static __device__ __align__(256) float na_part[NA_PART_FLOATS];
static __device__ __align__(256) unsigned na_counters[NA_MAX_KV];

struct NaScratch {
    bool ready;
    float* part;
    unsigned* counters;
    int* err;
};
NaScratch g_na[NA_MAX_DEV];
std::mutex g_na_mu;

int na_status(cudaError_t e, const char* what) {
    if (e != cudaSuccess) return tfb::set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return 0;
}

// Device addresses of the scratch arrays on the current device (looked up once per device).
int na_setup(NaScratch** out) {
    int dev = 0;
    if (na_status(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
    if (dev < 0 || dev >= NA_MAX_DEV) return tfb::set_error("device ordinal out of range for the static scratch");
    std::lock_guard<std::mutex> lock(g_na_mu);
    NaScratch& s = g_na[dev];
    if (!s.ready) {
        if (na_status(cudaGetSymbolAddress((void**)&s.part, na_part), "cudaGetSymbolAddress")) return -1;
        if (na_status(cudaGetSymbolAddress((void**)&s.counters, na_counters), "cudaGetSymbolAddress")) return -1;
        if (tfb::op_err_word(&s.err)) return -1;
        s.ready = true;
    }
    *out = &s;
    return 0;
}

}  // namespace

extern "C" {

int tf_op_attn_decode_noalloc(float* out, const float* q, const void* k_cache, const void* v_cache, int kv_type,
                              int cap, int n_pos, int n_heads, int n_kv_heads, int head_dim, void* stream) {
    using namespace tfb;
    if (n_pos <= 0 || n_pos > cap) return set_error("n_pos must be in [1, cap]");
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads)
        return set_error("n_heads must be a positive multiple of n_kv_heads");
    if (n_kv_heads > NA_MAX_KV) return set_error("n_kv_heads exceeds the static scratch limit (64)");
    if (head_dim <= 0 || head_dim % 8) return set_error("head_dim must be a positive multiple of 8");
    const int n_split = attn_pick_split(n_pos);
    if (n_split > 1 && (long long)n_heads * n_split * (head_dim + 2) > NA_PART_FLOATS)
        return set_error("attention scratch exceeds the static limit of 524288 floats "
                         "(n_heads * ceil(n_pos/64) * (head_dim+2))");
    NaScratch* s = nullptr;
    if (na_setup(&s)) return -1;
    AttnArgs a = {};
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
    a.part = n_split > 1 ? s->part : nullptr;
    a.counters = n_split > 1 ? s->counters : nullptr;
    a.out = out;
    a.ld_out = n_heads * head_dim;
    a.fresh = 0;
    a.n_pos_fixed = n_pos;
    a.err = s->err;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_split > 1 && na_status(cudaMemsetAsync(s->counters, 0, sizeof(unsigned) * n_kv_heads, st), "cudaMemsetAsync"))
        return -1;
    return na_status(attn_decode_launch(a, 1, st, false), "attn_decode");
}

}  // extern "C"
