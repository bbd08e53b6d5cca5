// Pipelined copies between pageable host memory and the device.
//
// The drop-in call `kernel[grid, block](numpy arrays)` copies every array in
// and every written array back (reference: src/thork/runtime.py:656-700),
// and NumPy arrays live in pageable memory.  A plain cudaMemcpy from pageable
// memory moves one bounce buffer at a time with a single-threaded host copy.
// Here large pageable copies go through a ring of pinned slots instead: a
// pool of host threads fills (or drains) one slot while the copy engine
// moves the previous one, so host copies and DMA overlap and the host side
// runs at multi-core memcpy speed.  Semantics match cudaMemcpyAsync on
// pageable memory: an HtoD copy returns once the source has been read (the
// device side completes in stream order); a DtoH copy returns complete.

#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "thork_internal.h"
#include "thork_rt.h"

namespace {

constexpr size_t kSlotBytes = 8u << 20;  // one pinned slot
constexpr int kSlots = 4;
constexpr size_t kStagedMin = 1u << 20;  // smaller copies go straight to cudaMemcpy
constexpr size_t kPieceMin = 256u << 10;  // smallest share of a slot one thread copies
constexpr int kMaxDevices = 64;

// Host threads that split one memcpy between them.  The pool is created on
// first use and never destroyed (its threads are detached and idle at exit);
// in a forked child the workers do not exist, so copies run on the caller.
class CopyPool {
 public:
  static CopyPool &get() {
    static CopyPool *pool = new CopyPool();
    return *pool;
  }

  void copy(void *dst, const void *src, size_t len) {
    const int parts = static_cast<int>(std::min<size_t>(workers_ + 1, len / kPieceMin));
    if (parts <= 1 || getpid() != pid_) {
      memcpy(dst, src, len);
      return;
    }
    std::unique_lock<std::mutex> job(job_mu_);  // one split copy at a time
    {
      std::lock_guard<std::mutex> lk(mu_);
      dst_ = static_cast<char *>(dst);
      src_ = static_cast<const char *>(src);
      len_ = len;
      parts_ = parts;
      next_ = 0;
      remaining_ = parts;
      ++gen_;
    }
    cv_.notify_all();
    work();  // the caller takes parts too
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return remaining_ == 0; });
  }

 private:
  CopyPool() : pid_(getpid()) {
    const unsigned hc = std::thread::hardware_concurrency();
    workers_ = static_cast<int>(std::min(7u, hc > 2 ? hc / 2 - 1 : 0u));
    for (int i = 0; i < workers_; ++i) std::thread([this] { loop(); }).detach();
  }

  // Copy parts of the current job until none are left.
  void work() {
    for (;;) {
      int part;
      char *dst;
      const char *src;
      size_t lo, hi;
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (next_ >= parts_) return;
        part = next_++;
        const size_t piece = (len_ / parts_ + 63) & ~size_t(63);
        lo = std::min(len_, piece * part);
        hi = part == parts_ - 1 ? len_ : std::min(len_, lo + piece);
        dst = dst_;
        src = src_;
      }
      if (hi > lo) memcpy(dst + lo, src + lo, hi - lo);
      std::lock_guard<std::mutex> lk(mu_);
      if (--remaining_ == 0) done_cv_.notify_all();
    }
  }

  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
      }
      work();
    }
  }

  pid_t pid_;
  int workers_ = 0;
  std::mutex job_mu_, mu_;
  std::condition_variable cv_, done_cv_;
  char *dst_ = nullptr;
  const char *src_ = nullptr;
  size_t len_ = 0;
  int parts_ = 0, next_ = 0, remaining_ = 0;
  uint64_t gen_ = 0;
};

// Per-device ring of pinned slots; an event per slot marks the last DMA
// that read or wrote it.
struct Ring {
  std::mutex mu;
  char *slot[kSlots] = {};
  cudaEvent_t ev[kSlots] = {};
  bool ready = false;
};
Ring g_ring[kMaxDevices];

int ring_for_device(Ring **out) {
  int dev;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return thork_set_error(THORK_ERR_INVALID, "device index %d too large", dev);
  *out = &g_ring[dev];
  return THORK_OK;
}

// Called with ring.mu held.
int ring_init(Ring &r) {
  if (r.ready) return THORK_OK;
  void *base = nullptr;
  cudaError_t e = cudaHostAlloc(&base, kSlotBytes * kSlots, cudaHostAllocDefault);
  if (e != cudaSuccess) return thork_cuda_error(e, "cudaHostAlloc(staging ring)");
  for (int k = 0; k < kSlots; ++k) {
    r.slot[k] = static_cast<char *>(base) + k * kSlotBytes;
    e = cudaEventCreateWithFlags(&r.ev[k], cudaEventDisableTiming);
    if (e != cudaSuccess) return thork_cuda_error(e, "cudaEventCreate(staging ring)");
  }
  r.ready = true;
  return THORK_OK;
}

}  // namespace

bool thork_is_pageable(const void *host_ptr) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, host_ptr) != cudaSuccess) {
    cudaGetLastError();  // clear the (non-sticky) error an unknown pointer leaves
    return true;
  }
  return a.type == cudaMemoryTypeUnregistered;
}

size_t thork_staged_min_bytes() { return kStagedMin; }

namespace {
// Chunk size of one copy: a quarter of it, so that even a 4 MiB copy
// overlaps host copies with DMA, within [1 MiB, one slot].
size_t chunk_bytes(size_t n) {
  const size_t c = ((n / 4) + 4095) & ~size_t(4095);
  return std::max<size_t>(kStagedMin, std::min(kSlotBytes, c));
}
}  // namespace

int thork_staged_htod(void *d_dst, const void *h_src, size_t n, cudaStream_t s) {
  Ring *r;
  int rc;
  if ((rc = ring_for_device(&r))) return rc;
  std::lock_guard<std::mutex> lk(r->mu);
  if ((rc = ring_init(*r))) return rc;
  const char *src = static_cast<const char *>(h_src);
  char *dst = static_cast<char *>(d_dst);
  const size_t chunk = chunk_bytes(n);
  int k = 0;
  for (size_t off = 0; off < n; off += chunk, k = (k + 1) % kSlots) {
    const size_t len = std::min(chunk, n - off);
    cudaError_t e = cudaEventSynchronize(r->ev[k]);  // the slot's last DMA is done
    if (e != cudaSuccess) return thork_cuda_error(e, "staged HtoD: slot wait");
    CopyPool::get().copy(r->slot[k], src + off, len);
    e = cudaMemcpyAsync(dst + off, r->slot[k], len, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return thork_cuda_error(e, "staged HtoD: cudaMemcpyAsync");
    e = cudaEventRecord(r->ev[k], s);
    if (e != cudaSuccess) return thork_cuda_error(e, "staged HtoD: cudaEventRecord");
  }
  return THORK_OK;
}

int thork_staged_dtoh(void *h_dst, const void *d_src, size_t n, cudaStream_t s) {
  Ring *r;
  int rc;
  if ((rc = ring_for_device(&r))) return rc;
  std::lock_guard<std::mutex> lk(r->mu);
  if ((rc = ring_init(*r))) return rc;
  const char *src = static_cast<const char *>(d_src);
  char *dst = static_cast<char *>(h_dst);
  const size_t chunk = chunk_bytes(n);
  const size_t chunks = (n + chunk - 1) / chunk;
  auto issue = [&](size_t i) -> int {
    const int k = static_cast<int>(i % kSlots);
    const size_t off = i * chunk, len = std::min(chunk, n - off);
    cudaError_t e = cudaEventSynchronize(r->ev[k]);  // e.g. an HtoD still reading the slot
    if (e != cudaSuccess) return thork_cuda_error(e, "staged DtoH: slot wait");
    e = cudaMemcpyAsync(r->slot[k], src + off, len, cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return thork_cuda_error(e, "staged DtoH: cudaMemcpyAsync");
    e = cudaEventRecord(r->ev[k], s);
    if (e != cudaSuccess) return thork_cuda_error(e, "staged DtoH: cudaEventRecord");
    return THORK_OK;
  };
  for (size_t i = 0; i < chunks && i < static_cast<size_t>(kSlots); ++i)
    if ((rc = issue(i))) return rc;
  for (size_t i = 0; i < chunks; ++i) {
    const int k = static_cast<int>(i % kSlots);
    const size_t off = i * chunk, len = std::min(chunk, n - off);
    cudaError_t e = cudaEventSynchronize(r->ev[k]);
    if (e != cudaSuccess) return thork_cuda_error(e, "staged DtoH: chunk wait");
    CopyPool::get().copy(dst + off, r->slot[k], len);
    if (i + kSlots < chunks && (rc = issue(i + kSlots))) return rc;
  }
  return THORK_OK;
}
