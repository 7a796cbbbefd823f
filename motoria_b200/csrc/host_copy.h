// host_copy.h -- host-side pieces of miag_moe's transfer pipeline: the
// threads that copy between a caller's pageable buffer and the pinned
// staging buffer, and the split of a batch into pieces.  Plain C++ (no CUDA),
// so the CPU tests compile it on its own.
#pragma once

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace miag {

// Host threads that split one memcpy between them: miag_moe's copies between
// the caller's pageable buffer and the context's pinned staging buffer.  The
// calling thread copies the first part and returns when every part is done,
// so a worker never misses a generation.  A worker spins for a while after
// its part (one call issues its copies a few microseconds apart) and then
// sleeps until the next one.
class CopyPool {
  public:
    explicit CopyPool(int workers) {
        for (int i = 0; i < workers; i++) threads_.emplace_back([this, i] { run(i + 1); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> g(m_);
            stop_ = true;
        }
        wake_.notify_all();
        for (std::thread &t : threads_) t.join();
    }
    int workers() const { return (int)threads_.size(); }
    void copy(void *dst, const void *src, size_t bytes) {
        const int parts = workers() + 1;
        if (parts == 1 || bytes < ((size_t)256 << 10)) {
            memcpy(dst, src, bytes);
            return;
        }
        dst_ = (char *)dst;
        src_ = (const char *)src;
        bytes_ = bytes;
        parts_ = parts;
        left_.store(parts - 1, std::memory_order_relaxed);
        gen_.fetch_add(1, std::memory_order_release);
        { std::lock_guard<std::mutex> g(m_); }  // a worker going to sleep sees the new generation
        wake_.notify_all();
        part(0);
        while (left_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
    }

  private:
    void part(int i) const {
        const size_t per = ((bytes_ + parts_ - 1) / parts_ + 63) & ~(size_t)63;
        const size_t b = std::min(bytes_, (size_t)i * per), e = std::min(bytes_, b + per);
        if (e > b) memcpy(dst_ + b, src_ + b, e - b);
    }
    void run(int i) {
        uint64_t seen = 0;
        for (;;) {
            const auto t0 = std::chrono::steady_clock::now();
            for (int n = 0; gen_.load(std::memory_order_acquire) == seen; n++) {
                if ((n & 255) == 255 &&
                    std::chrono::steady_clock::now() - t0 > std::chrono::microseconds(200)) {
                    std::unique_lock<std::mutex> l(m_);
                    wake_.wait(l, [&] {
                        return stop_ || gen_.load(std::memory_order_acquire) != seen;
                    });
                    if (stop_) return;
                    break;
                }
            }
            seen = gen_.load(std::memory_order_acquire);
            part(i);
            left_.fetch_sub(1, std::memory_order_acq_rel);
        }
    }
    std::vector<std::thread> threads_;
    std::mutex m_;
    std::condition_variable wake_;
    bool stop_ = false;
    std::atomic<uint64_t> gen_{0};
    std::atomic<int> left_{0};
    int parts_ = 1;
    char *dst_ = nullptr;
    const char *src_ = nullptr;
    size_t bytes_ = 0;
};

// Piece boundaries: with three or more pieces, a first and a last piece of
// n / (2 chunks) tokens and equal pieces between them, else equal pieces
// (multiples of 32 tokens).  Only the first piece's copy in and the last
// piece's copy out are exposed, while every piece costs one stream of the
// layer's expert weights: at config 5 (4096 tokens, 4 pieces) edges of 512
// tokens took 2.55 ms a pinned call against 2.66 with equal pieces.
inline std::vector<int> piece_bounds(int n, int chunks) {
    int edge = (n / (2 * chunks) + 31) & ~31;
    if (chunks < 3 || 2 * edge >= n) edge = 0;
    const int m = edge ? chunks - 2 : chunks, mid = n - 2 * edge;  // m equal pieces over mid
    std::vector<int> b{0};
    if (edge) b.push_back(edge);
    for (int i = 1; i < m; i++) {
        const int t = edge + ((int)((long long)mid * i / m) & ~31);
        if (t > b.back()) b.push_back(t);
    }
    if (edge) b.push_back(n - edge);
    b.push_back(n);
    return b;
}

}  // namespace miag
