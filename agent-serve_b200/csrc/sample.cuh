// Device temperature / top-p sampler (sample.cu).
#pragma once

#include "common.cuh"

namespace tfb {

struct SampleScratch;
SampleScratch* sample_scratch_create(int n);
void sample_scratch_destroy(SampleScratch* s);
// Samples one id from logits[0..n) with the caller's uniform draw r; the id lands in
// sample_result(s) (device).
cudaError_t sample_launch(SampleScratch* s, const float* logits, int n, float temperature, float top_p, float r,
                          cudaStream_t st);
int* sample_result(SampleScratch* s);

}  // namespace tfb
