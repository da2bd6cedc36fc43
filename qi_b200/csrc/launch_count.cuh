// Process-wide count of the kernels this library has launched (or recorded
// into a CUDA graph under capture).  Every launch site adds its launches;
// qi_b200_launch_count reads the total.
#pragma once
#include <atomic>

namespace qib {

inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> n{0};
  return n;
}

inline void count_launches(int n) { launch_counter().fetch_add(static_cast<unsigned long long>(n), std::memory_order_relaxed); }

}  // namespace qib
