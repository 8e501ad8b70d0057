// hostcopy.cpp -- logits from HBM into caller-owned host memory (hostcopy.h).
#include "hostcopy.h"

#include <sched.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <mutex>
#include <thread>

#include "../../../include/gpt2_b200.h"

namespace gpt2 {
void set_error(const char *fmt, ...);

namespace {
constexpr size_t kHugePage = size_t(2) << 20;
constexpr int kStages = 4;  // pinned staging buffers: DMA of the next chunks runs while earlier ones are copied out

size_t chunk_bytes() {
  static const size_t b = [] {
    size_t mb = 32;
    if (const char *e = getenv("GPT2_COPY_CHUNK_MB")) mb = std::max(1, atoi(e));
    return mb << 20;
  }();
  return b;
}

// Spins briefly, then yields the CPU, so that a worker waiting for the next
// chunk never starves the thread that issues the copies.
inline void cpu_relax(uint32_t &spins) {
  if (++spins < 1024) __builtin_ia32_pause();
  else std::this_thread::yield();
}

// The copy-out of one call, run by a fixed set of host threads that live for
// the rest of the process (never destroyed: threads detached, object leaked,
// so nothing at library unload or process exit waits on them).  The calling
// thread enqueues the DMA of chunk c into staging slot c % kStages once every
// worker is done with the slot's previous chunk; worker i copies slice i of
// every chunk, waiting for each chunk's DMA on its own, so no worker waits
// for another between chunks.
class CopyPipeline {
 public:
  explicit CopyPipeline(int n) : n_(n) {
    for (int i = 0; i < n_; ++i) std::thread([this, i] { worker(i); }).detach();
  }
  int threads() const { return n_; }

  // Runs the copy of `chunks` chunks; issue(c) enqueues chunk c's DMA and
  // records its slot's event (false on a CUDA error).  Returns the first CUDA
  // error seen (cudaSuccess if none).
  template <typename Issue>
  cudaError_t run(char *dst, float *const *stage, cudaEvent_t *ev, int64_t chunks, int64_t rows_per_chunk,
                  int64_t rows, size_t row_bytes, int device, Issue issue) {
    std::lock_guard<std::mutex> one(call_mu_);
    dst_ = dst;
    for (int s = 0; s < kStages; ++s) {
      stage_[s] = stage[s];
      ev_[s] = ev[s];
      slot_done_[s].store(0, std::memory_order_relaxed);
    }
    chunks_ = chunks;
    rpc_ = rows_per_chunk;
    rows_ = rows;
    row_bytes_ = row_bytes;
    device_ = device;
    err_.store(cudaSuccess, std::memory_order_relaxed);
    issued_.store(0, std::memory_order_relaxed);
    {
      std::lock_guard<std::mutex> lk(mu_);
      pending_ = n_;
      ++gen_;
    }
    cv_.notify_all();
    cudaError_t first = cudaSuccess;
    for (int64_t c = 0; c < chunks; ++c) {
      const int s = static_cast<int>(c % kStages);
      // The slot's previous chunk, c - kStages, is copied out by every worker.
      const int64_t need = static_cast<int64_t>(n_) * (c / kStages);
      while (slot_done_[s].load(std::memory_order_acquire) < need) std::this_thread::yield();
      if (first == cudaSuccess) first = issue(c);
      if (first != cudaSuccess) err_.store(first, std::memory_order_relaxed);  // the workers skip the copies
      issued_.store(c + 1, std::memory_order_release);
    }
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [this] { return pending_ == 0; });
    const cudaError_t e = err_.load();
    return first != cudaSuccess ? first : e;
  }

 private:
  void worker(int i) {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
      }
      cudaSetDevice(device_);
      for (int64_t c = 0; c < chunks_; ++c) {
        uint32_t spins = 0;
        while (issued_.load(std::memory_order_acquire) <= c) cpu_relax(spins);
        const int s = static_cast<int>(c % kStages);
        if (err_.load(std::memory_order_relaxed) == cudaSuccess) {
          const cudaError_t e = cudaEventSynchronize(ev_[s]);
          if (e != cudaSuccess) {
            cudaError_t expect = cudaSuccess;
            err_.compare_exchange_strong(expect, e);
          } else {
            // Slice i of the chunk, cut at absolute 2 MiB boundaries of the destination so that no two
            // threads fault the same (huge) page.
            const uintptr_t start = reinterpret_cast<uintptr_t>(dst_) + static_cast<size_t>(c * rpc_) * row_bytes_;
            const uintptr_t end = start + static_cast<size_t>(std::min(rpc_, rows_ - c * rpc_)) * row_bytes_;
            const uintptr_t per = (end - start + n_ - 1) / n_;
            auto cut = [&](int k) {
              const uintptr_t x = (start + per * k + kHugePage / 2) & ~(uintptr_t)(kHugePage - 1);
              return k == 0 ? start : k == n_ ? end : std::min(end, std::max(start, x));
            };
            const uintptr_t lo = cut(i), hi = cut(i + 1);
            if (hi > lo)
              memcpy(reinterpret_cast<void *>(lo), reinterpret_cast<const char *>(stage_[s]) + (lo - start), hi - lo);
          }
        }
        slot_done_[s].fetch_add(1, std::memory_order_release);
      }
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_.notify_one();
    }
  }

  const int n_;
  std::mutex call_mu_, mu_;
  std::condition_variable cv_, done_;
  int pending_ = 0;
  uint64_t gen_ = 0;
  // the current call (written before gen_ advances, fixed until every worker is done)
  char *dst_ = nullptr;
  float *stage_[kStages] = {};
  cudaEvent_t ev_[kStages] = {};
  int64_t chunks_ = 0, rpc_ = 0, rows_ = 0;
  size_t row_bytes_ = 0;
  int device_ = 0;
  std::atomic<int64_t> issued_{0};
  std::atomic<int64_t> slot_done_[kStages];
  std::atomic<cudaError_t> err_{cudaSuccess};
};

CopyPipeline &pipeline() {
  static CopyPipeline *p = [] {
    // Three quarters of the CPUs this process may run on (measured best on a
    // 16-CPU host: 12 workers; the copy is bound by host memory bandwidth).
    int n = 8;
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof set, &set) == 0) n = CPU_COUNT(&set) - CPU_COUNT(&set) / 4;
    if (const char *e = getenv("GPT2_COPY_THREADS")) n = atoi(e);
    return new CopyPipeline(std::max(1, std::min(n, 32)));
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
  if (pinned || (size_t)rows * row_bytes <= chunk_bytes()) {
    cudaError_t e = cudaMemcpy2DAsync(dst, row_bytes, d_src, sizeof(float) * ld, row_bytes, rows,
                                      cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? 0 : fail(e, "cudaMemcpy2DAsync");
  }
  std::lock_guard<std::mutex> lk(g_stage_mu);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(e, "cudaGetDevice");
  const int64_t rpc = std::max<int64_t>(1, (int64_t)(chunk_bytes() / row_bytes));  // rows per chunk
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
  auto issue = [&](int64_t c) {
    const int64_t r = std::min(rpc, rows - c * rpc);
    const int s = static_cast<int>(c % kStages);
    cudaError_t ei = cudaMemcpy2DAsync(g_stage.buf[s], row_bytes, d_src + c * rpc * ld, sizeof(float) * ld,
                                       row_bytes, r, cudaMemcpyDeviceToHost, st);
    if (ei == cudaSuccess) ei = cudaEventRecord(g_stage.ev[s], st);
    return ei;
  };
  e = pipeline().run(reinterpret_cast<char *>(dst), g_stage.buf, g_stage.ev, n, rpc, rows, row_bytes, dev, issue);
  if (e != cudaSuccess) {
    cudaStreamSynchronize(st);  // copies already issued into the staging buffers finish first
    return fail(e, "staged copy");
  }
  return 0;
}

}  // namespace gpt2
