// fs_hoststage.h -- host-side staging of pageable host memory for the
// host-slice sorts (sort_u32(&mut [u32]) and kin).
//
// A copy between pageable host memory and the device is done by the driver
// through its own page-locked bounce buffer with one CPU thread: about
// 13 GB/s each way on a B200 box, which made a 16M-key host-slice sort spend
// 9 of its 10 ms in copies.  Here the copy is cut into chunks that cycle
// through a small ring of page-locked buffers owned by the sorter: several
// host threads fill (or drain) one chunk while the DMA engine moves the
// previous one, so the transfer runs at the bus rate instead of one core's
// memcpy rate.  The reference's unified memory needed no copy at all
// (forge-sort src/lib.rs:791-998 memcpys into a shared Metal buffer).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace fs {

// A fixed set of worker threads running one function over thread ids
// 0..n-1 per call; the caller blocks until all have returned.
class CopyPool {
 public:
  explicit CopyPool(int threads) : n_(threads < 1 ? 1 : threads) {
    for (int i = 1; i < n_; ++i) workers_.emplace_back([this, i] { loop(i); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return n_; }
  // fn(i) for i in [0, size()); thread 0 is the caller
  void run(const std::function<void(int)>& fn) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn_ = &fn;
      pending_ = n_ - 1;
      ++gen_;
    }
    cv_.notify_all();
    fn(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [this] { return pending_ == 0; });
    fn_ = nullptr;
  }

 private:
  void loop(int i) {
    unsigned long long seen = 0;
    for (;;) {
      const std::function<void(int)>* f;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
        f = fn_;
      }
      (*f)(i);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_.notify_one();
    }
  }
  int n_;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  const std::function<void(int)>* fn_ = nullptr;
  int pending_ = 0;
  unsigned long long gen_ = 0;
  bool stop_ = false;
};

// Ring of page-locked chunk buffers + the events that say when the DMA of
// each has finished.  All copies are enqueued on the caller's stream.
struct HostStage {
  static constexpr int NB = 3;                  // chunks in flight
  static constexpr size_t CHUNK = 8u << 20;     // bytes per chunk
  void* buf[NB] = {};
  cudaEvent_t ev[NB] = {};
  bool used[NB] = {};
  CopyPool* pool = nullptr;

  ~HostStage() { release(); }
  void release() {
    for (int i = 0; i < NB; ++i) {
      if (ev[i]) cudaEventSynchronize(ev[i]), cudaEventDestroy(ev[i]);
      if (buf[i]) cudaFreeHost(buf[i]);
      buf[i] = nullptr;
      ev[i] = nullptr;
      used[i] = false;
    }
    delete pool;
    pool = nullptr;
  }
  cudaError_t ensure() {
    if (buf[0]) return cudaSuccess;
    for (int i = 0; i < NB; ++i) {
      cudaError_t e = cudaHostAlloc(&buf[i], CHUNK, cudaHostAllocPortable);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
      if (e != cudaSuccess) {
        release();
        return e;
      }
    }
    const unsigned hw = std::thread::hardware_concurrency();
    pool = new CopyPool((int)std::min(8u, std::max(1u, hw / 2)));
    return cudaSuccess;
  }
  // memcpy of `bytes` split over the pool's threads
  void par_copy(void* dst, const void* src, size_t bytes) {
    const int t = pool->size();
    const size_t per = ((bytes + t - 1) / t + 63) & ~size_t(63);
    pool->run([&](int i) {
      const size_t lo = std::min(bytes, per * (size_t)i), hi = std::min(bytes, lo + per);
      if (hi > lo) std::memcpy(static_cast<char*>(dst) + lo, static_cast<const char*>(src) + lo, hi - lo);
    });
  }
  // pageable host -> device, in stream order on `st`; returns once the last
  // chunk is handed to the DMA engine (the copies complete in stream order)
  cudaError_t to_device(void* dev, const void* host, size_t bytes, cudaStream_t st) {
    cudaError_t e = ensure();
    if (e != cudaSuccess) return e;
    for (size_t off = 0, k = 0; off < bytes; off += CHUNK, ++k) {
      const int b = (int)(k % NB);
      const size_t len = std::min(CHUNK, bytes - off);
      if (used[b] && (e = cudaEventSynchronize(ev[b])) != cudaSuccess) return e;
      par_copy(buf[b], static_cast<const char*>(host) + off, len);
      if ((e = cudaMemcpyAsync(static_cast<char*>(dev) + off, buf[b], len, cudaMemcpyHostToDevice, st)) !=
          cudaSuccess)
        return e;
      if ((e = cudaEventRecord(ev[b], st)) != cudaSuccess) return e;
      used[b] = true;
    }
    return cudaSuccess;
  }
  // device -> pageable host, after the work already enqueued on `st`;
  // returns when every byte has landed in host memory
  cudaError_t to_host(void* host, const void* dev, size_t bytes, cudaStream_t st) {
    cudaError_t e = ensure();
    if (e != cudaSuccess) return e;
    const size_t nk = (bytes + CHUNK - 1) / CHUNK;
    auto issue = [&](size_t k) -> cudaError_t {
      const int b = (int)(k % NB);
      const size_t off = k * CHUNK, len = std::min(CHUNK, bytes - off);
      cudaError_t r;
      if (used[b] && (r = cudaEventSynchronize(ev[b])) != cudaSuccess) return r;
      if ((r = cudaMemcpyAsync(buf[b], static_cast<const char*>(dev) + off, len, cudaMemcpyDeviceToHost, st)) !=
          cudaSuccess)
        return r;
      used[b] = true;
      return cudaEventRecord(ev[b], st);
    };
    for (size_t k = 0; k < nk && k < (size_t)NB; ++k)
      if ((e = issue(k)) != cudaSuccess) return e;
    for (size_t k = 0; k < nk; ++k) {
      const int b = (int)(k % NB);
      const size_t off = k * CHUNK, len = std::min(CHUNK, bytes - off);
      if ((e = cudaEventSynchronize(ev[b])) != cudaSuccess) return e;
      par_copy(static_cast<char*>(host) + off, buf[b], len);
      used[b] = false;  // drained: free for the next chunk
      if (k + NB < nk && (e = issue(k + NB)) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
};

}  // namespace fs
