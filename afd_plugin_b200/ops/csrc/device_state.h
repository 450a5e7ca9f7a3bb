// Per-device host state of the launchers.  One process may drive several
// GPUs (a test harness, a multi-GPU server thread pool), so kernel attribute
// opt-ins and cached device properties are kept per device, never in one
// process-wide static.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

namespace afd {

constexpr int kMaxDevices = 64;

// The calling thread's current device, or -1 if the runtime cannot say.
int current_device();

// Multiprocessor count of the current device (cached per device; 148 on B200).
int device_sm_count();

// Runs a set-up function once per device and remembers success.  A failure is
// returned to the caller and retried on the next call.
class PerDeviceOnce {
 public:
  template <typename F>
  cudaError_t run(F&& fn) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fn();
    if (done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mutex_);
    if (done_[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    const cudaError_t e = fn();
    if (e == cudaSuccess) done_[dev].store(true, std::memory_order_release);
    return e;
  }

 private:
  std::atomic<bool> done_[kMaxDevices] = {};
  std::mutex mutex_;
};

// L2 eviction hints of the streaming loads (bit 0: grouped GEMM weight
// tiles, bit 1: MLA decode KV rows).  AFD_L2_HINTS=0 / gemm / mla / all
// (default all) selects them, for A/B measurements on one machine.
constexpr int kL2HintGemm = 1, kL2HintMla = 2;
int l2_hint_mask();

}  // namespace afd
