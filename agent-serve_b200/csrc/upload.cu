// Pinned, double-buffered weight upload (see upload.cuh).
#include "upload.cuh"

#include <algorithm>
#include <cstring>
#include <thread>

namespace tfb {

Uploader::~Uploader() {
    if (st_) cudaStreamSynchronize(st_);
    for (cudaEvent_t e : ev_)
        if (e) cudaEventDestroy(e);
    for (void* b : buf_)
        if (b) cudaFreeHost(b);
    if (st_) cudaStreamDestroy(st_);
}

cudaError_t Uploader::init(size_t chunk, int nbuf, int threads) {
    chunk_ = chunk;
    threads_ = std::max(1, threads);
    cudaError_t e = cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking);
    if (e != cudaSuccess) return e;
    buf_.assign(nbuf, nullptr);
    ev_.assign(nbuf, nullptr);
    used_.assign(nbuf, false);
    for (int i = 0; i < nbuf; ++i) {
        if ((e = cudaMallocHost(&buf_[i], chunk)) != cudaSuccess) return e;
        if ((e = cudaEventCreateWithFlags(&ev_[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Copy n <= chunk bytes of src into staging memory: the rest of the current buffer, or the
// next buffer once the DMA that last read it has finished.  *ptr receives the staged bytes.
cudaError_t Uploader::stage(size_t n, const void* src, int* buf, void** ptr) {
    if (fill_ + n > chunk_ || !started_) {
        next_ = started_ ? (next_ + 1) % (int)buf_.size() : 0;
        started_ = true;
        fill_ = 0;
        if (used_[next_]) {
            cudaError_t e = cudaEventSynchronize(ev_[next_]);
            if (e != cudaSuccess) return e;
        }
    }
    const int b = next_;
    uint8_t* d = static_cast<uint8_t*>(buf_[b]) + fill_;
    const uint8_t* s = static_cast<const uint8_t*>(src);
    const int nt = n >= ((size_t)4 << 20) ? threads_ : 1;
    if (nt == 1) {
        std::memcpy(d, s, n);
    } else {
        std::vector<std::thread> th;
        const size_t part = (n + nt - 1) / nt;
        for (int t = 0; t < nt; ++t) {
            const size_t o = (size_t)t * part;
            if (o >= n) break;
            th.emplace_back([=] { std::memcpy(d + o, s + o, std::min(part, n - o)); });
        }
        for (auto& x : th) x.join();
    }
    fill_ += (n + 255) & ~(size_t)255;
    used_[b] = true;
    *buf = b;
    *ptr = d;
    bytes_ += n;
    return cudaSuccess;
}

cudaError_t Uploader::copy(void* dst, const void* src, size_t bytes) {
    for (size_t o = 0; o < bytes; o += chunk_) {
        const size_t n = std::min(chunk_, bytes - o);
        int b = 0;
        void* p = nullptr;
        cudaError_t e = stage(n, static_cast<const uint8_t*>(src) + o, &b, &p);
        if (e != cudaSuccess) return e;
        e = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + o, p, n, cudaMemcpyHostToDevice, st_);
        if (e != cudaSuccess) return e;
        if ((e = cudaEventRecord(ev_[b], st_)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t Uploader::copy_rows(void* dst, size_t dpitch, const void* src, size_t width, size_t rows) {
    if (width == 0 || rows == 0) return cudaSuccess;
    // one row is staged whole: a row wider than a staging buffer goes row by row through copy()
    if (width > chunk_) {
        for (size_t r = 0; r < rows; ++r) {
            cudaError_t e = copy(static_cast<uint8_t*>(dst) + r * dpitch, static_cast<const uint8_t*>(src) + r * width,
                                 width);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    const size_t per = std::max<size_t>(1, chunk_ / width);
    for (size_t r = 0; r < rows; r += per) {
        const size_t n = std::min(per, rows - r);
        int b = 0;
        void* p = nullptr;
        cudaError_t e = stage(n * width, static_cast<const uint8_t*>(src) + r * width, &b, &p);
        if (e != cudaSuccess) return e;
        e = cudaMemcpy2DAsync(static_cast<uint8_t*>(dst) + r * dpitch, dpitch, p, width, width, n,
                              cudaMemcpyHostToDevice, st_);
        if (e != cudaSuccess) return e;
        if ((e = cudaEventRecord(ev_[b], st_)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t Uploader::finish() {
    cudaError_t e = cudaStreamSynchronize(st_);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace tfb
