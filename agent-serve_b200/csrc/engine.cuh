// Host-side engine internals shared by model.cu and ops.cu.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <string>
#include <vector>

#include "tinferno_b200.h"
#include "gemv.cuh"

namespace tfb {

// kernels (gemv.cu, attention.cu, misc.cu)
void gemv_plan(GemvArgs& a);
void gemv_plan_w(GemvArgs& a, int warps, int budget);
int gemv_grid(const GemvArgs& a, int num_sms);
int gemv_slots(int num_sms);  // resident GEMV CTAs the device holds (SMs x CTAs per SM)
int gemv_max_rows(int K);
int fused_attn_tile(const GemvArgs& a, int hd);  // positions per fused-attention tile of a QKV launch
cudaError_t gemv_launch(const GemvArgs& a, int grid, cudaStream_t st, bool pdl);
cudaError_t key_apply_launch(const long long* key, int* tok, int* hist, const StepCtl* ctl, cudaStream_t st);
cudaError_t gemv_init_attrs();

struct AttnArgs;
struct PrefillAttnArgs;
int attn_pick_split(int cap);

std::string& last_error_tls();
int set_error(const std::string& msg);

constexpr int kMaxDevices = 64;
// The current device's op-level status word (ops.cu): a static device variable, no allocation.
int op_err_word(int** out);

}  // namespace tfb
