// device_once.h — run a host-side set-up step once per CUDA device.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

namespace uocr {

// Kernel attribute set-up (shared-memory opt-in, carve-out) once per device
// ordinal, safe from several host threads.  Ordinals of 64 and above, which
// the bit set cannot hold, run the step on every call (setting an attribute
// again is harmless).
class PerDeviceOnce {
 public:
  template <class Fn>
  void run(Fn&& fn) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) {
      fn();
      return;
    }
    const uint64_t bit = uint64_t{1} << dev;
    if (done_.load(std::memory_order_acquire) & bit) return;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_.load(std::memory_order_relaxed) & bit) return;
    fn();
    done_.fetch_or(bit, std::memory_order_release);
  }

 private:
  std::atomic<uint64_t> done_{0};
  std::mutex mu_;
};

}  // namespace uocr
