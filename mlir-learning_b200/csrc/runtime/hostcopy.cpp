// hostcopy.cpp -- logits from HBM into caller-owned host memory (hostcopy.h).
#include "hostcopy.h"

#include <sched.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>

#include <algorithm>
#include <condition_variable>
#include <mutex>
#include <thread>

#include "../../../include/gpt2_b200.h"

namespace gpt2 {
void set_error(const char *fmt, ...);

namespace {
constexpr size_t kHugePage = size_t(2) << 20;
constexpr size_t kChunkBytes = size_t(32) << 20;  // one pinned staging buffer
constexpr int kStages = 3;                        // DMA of two chunks in flight while one is copied out

// memcpy split over a fixed set of threads that live for the rest of the
// process.  The pool is never destroyed (threads detached, object leaked), so
// nothing at library unload or process exit waits on it.
class CopyPool {
 public:
  explicit CopyPool(int n) : n_(n) {
    for (int i = 1; i < n_; ++i) std::thread([this, i] { worker(i); }).detach();
  }

  // Copies [src, src + bytes) to dst with every thread of the pool (the caller
  // takes the first slice); returns when all slices are done.
  void copy(void *dst, const void *src, size_t bytes) {
    std::lock_guard<std::mutex> one(call_mu_);
    {
      std::lock_guard<std::mutex> lk(mu_);
      dst_ = static_cast<char *>(dst);
      src_ = static_cast<const char *>(src);
      bytes_ = bytes;
      pending_ = n_ - 1;
      ++gen_;
    }
    cv_.notify_all();
    part(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [this] { return pending_ == 0; });
  }

 private:
  // Slice i, in whole 4 KiB pages so that two threads never fault the same page.
  void part(int i) const {
    const size_t per = ((bytes_ + n_ - 1) / n_ + 4095) & ~size_t(4095);
    const size_t lo = std::min(bytes_, per * i), hi = std::min(bytes_, lo + per);
    if (hi > lo) memcpy(dst_ + lo, src_ + lo, hi - lo);
  }

  void worker(int i) {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
      }
      part(i);  // the job's fields were published under mu_ and stay fixed until pending_ reaches 0
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_.notify_one();
    }
  }

  const int n_;
  std::mutex call_mu_, mu_;
  std::condition_variable cv_, done_;
  char *dst_ = nullptr;
  const char *src_ = nullptr;
  size_t bytes_ = 0;
  int pending_ = 0;
  uint64_t gen_ = 0;
};

CopyPool &pool() {
  static CopyPool *p = [] {
    int n = 8;
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof set, &set) == 0) n = CPU_COUNT(&set);
    if (const char *e = getenv("GPT2_COPY_THREADS")) n = atoi(e);
    return new CopyPool(std::max(1, std::min(n, 16)));
  }();
  return *p;
}

struct Staging {
  float *buf[kStages] = {};
  cudaEvent_t ev[kStages] = {};
  size_t bytes = 0;
  int device = -1;
};
Staging g_stage;
std::mutex g_stage_mu;

void free_staging_locked() {
  for (int i = 0; i < kStages; ++i) {
    if (g_stage.buf[i]) cudaFreeHost(g_stage.buf[i]);
    if (g_stage.ev[i]) cudaEventDestroy(g_stage.ev[i]);
  }
  g_stage = Staging();
}

int fail(cudaError_t e, const char *what) {
  set_error("copy of logits to host memory: %s: %s", what, cudaGetErrorString(e));
  return GPT2_ECUDA;
}
}  // namespace

void *alloc_host_output(size_t bytes) {
  if (bytes < 2 * kHugePage) return malloc(bytes);
  void *p = nullptr;
  if (posix_memalign(&p, kHugePage, bytes) != 0) return nullptr;
  madvise(p, bytes, MADV_HUGEPAGE);  // advice only: ignored where huge pages are off
  return p;
}

void release_host_staging() {
  std::lock_guard<std::mutex> lk(g_stage_mu);
  free_staging_locked();
}

int copy_rows_to_host(const float *d_src, int64_t ld, int64_t rows, int64_t cols, float *dst, cudaStream_t st) {
  const size_t row_bytes = sizeof(float) * cols;
  cudaPointerAttributes at{};
  const bool pinned = cudaPointerGetAttributes(&at, dst) == cudaSuccess && at.type == cudaMemoryTypeHost;
  cudaGetLastError();  // a pageable pointer may leave an error behind on older drivers
  if (pinned || (size_t)rows * row_bytes <= kChunkBytes) {
    cudaError_t e = cudaMemcpy2DAsync(dst, row_bytes, d_src, sizeof(float) * ld, row_bytes, rows,
                                      cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? 0 : fail(e, "cudaMemcpy2DAsync");
  }
  std::lock_guard<std::mutex> lk(g_stage_mu);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "cudaGetDevice");
  const int64_t rpc = std::max<int64_t>(1, (int64_t)(kChunkBytes / row_bytes));  // rows per chunk
  const size_t need = (size_t)rpc * row_bytes;
  if (g_stage.bytes < need || g_stage.device != dev) {
    free_staging_locked();
    for (int i = 0; i < kStages; ++i) {
      e = cudaHostAlloc(reinterpret_cast<void **>(&g_stage.buf[i]), need, cudaHostAllocPortable);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&g_stage.ev[i], cudaEventDisableTiming);
      if (e != cudaSuccess) {
        free_staging_locked();
        return fail(e, "pinned staging allocation");
      }
    }
    g_stage.bytes = need;
    g_stage.device = dev;
  }
  const int64_t n = (rows + rpc - 1) / rpc;
  auto issue = [&](int64_t i) {
    const int64_t r = std::min(rpc, rows - i * rpc);
    cudaError_t ei = cudaMemcpy2DAsync(g_stage.buf[i % kStages], row_bytes, d_src + i * rpc * ld,
                                       sizeof(float) * ld, row_bytes, r, cudaMemcpyDeviceToHost, st);
    if (ei == cudaSuccess) ei = cudaEventRecord(g_stage.ev[i % kStages], st);
    return ei;
  };
  // On a failure, copies already issued into the staging buffers finish before returning.
  auto fail_drain = [&](cudaError_t ef, const char *what) {
    cudaStreamSynchronize(st);
    return fail(ef, what);
  };
  for (int64_t i = 0; i < std::min<int64_t>(n, kStages - 1); ++i)
    if ((e = issue(i)) != cudaSuccess) return fail_drain(e, "cudaMemcpy2DAsync");
  for (int64_t i = 0; i < n; ++i) {
    if ((e = cudaEventSynchronize(g_stage.ev[i % kStages])) != cudaSuccess)
      return fail_drain(e, "cudaEventSynchronize");
    // The buffer of chunk i + kStages - 1 held chunk i - 1, copied out in the previous iteration.
    if (i + kStages - 1 < n && (e = issue(i + kStages - 1)) != cudaSuccess)
      return fail_drain(e, "cudaMemcpy2DAsync");
    const int64_t r = std::min(rpc, rows - i * rpc);
    pool().copy(dst + i * rpc * cols, g_stage.buf[i % kStages], (size_t)r * row_bytes);
  }
  return 0;
}

}  // namespace gpt2
