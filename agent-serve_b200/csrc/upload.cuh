// Weight upload: host tensor bytes (the caller's GGUF mapping) streamed into HBM through
// pinned staging buffers on a copy stream of their own.  The host copies chunk i + 1 into one
// staging buffer (several threads) while the DMA engine moves chunk i out of another, so
// reading the file and crossing PCIe overlap; a pageable cudaMemcpy does both in turn.
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

namespace tfb {

class Uploader {
public:
    ~Uploader();
    // nbuf staging buffers of `chunk` bytes each; host copies split over `threads` threads
    cudaError_t init(size_t chunk, int nbuf, int threads);
    // dst[0, bytes) = src[0, bytes)
    cudaError_t copy(void* dst, const void* src, size_t bytes);
    // rows of `width` bytes: dst row r at dst + r * dpitch, src rows contiguous
    cudaError_t copy_rows(void* dst, size_t dpitch, const void* src, size_t width, size_t rows);
    // waits for every copy; the first error of any of them
    cudaError_t finish();
    size_t bytes() const { return bytes_; }

private:
    cudaError_t stage(size_t n, const void* src, int* buf, void** ptr);
    std::vector<void*> buf_;
    std::vector<cudaEvent_t> ev_;
    std::vector<bool> used_;
    cudaStream_t st_ = nullptr;
    size_t chunk_ = 0, fill_ = 0;
    int next_ = 0, threads_ = 1;
    bool started_ = false;
    size_t bytes_ = 0;
};

}  // namespace tfb
