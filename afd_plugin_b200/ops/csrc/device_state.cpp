#include "device_state.h"

#include <cstdlib>
#include <string>

namespace afd {

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int device_sm_count() {
  static std::atomic<int> cache[kMaxDevices] = {};
  const int dev = current_device();
  if (dev >= 0 && dev < kMaxDevices) {
    const int v = cache[dev].load(std::memory_order_relaxed);
    if (v > 0) return v;
  }
  int sms = 0;
  if (dev < 0 || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 1;  // the query failed: launches still cover all work, just with a small grid
  if (dev >= 0 && dev < kMaxDevices) cache[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

int l2_hint_mask() {
  static const int mask = [] {
    const char* v = std::getenv("AFD_L2_HINTS");
    if (v == nullptr) return kL2HintGemm | kL2HintMla;
    const std::string s(v);
    if (s == "0" || s == "off") return 0;
    if (s == "gemm") return kL2HintGemm;
    if (s == "mla") return kL2HintMla;
    return kL2HintGemm | kL2HintMla;
  }();
  return mask;
}

}  // namespace afd
