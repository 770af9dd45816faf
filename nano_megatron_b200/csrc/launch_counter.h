// Host-side count of kernel launches issued by this library (all devices).
#pragma once

#include <atomic>

namespace nmb {
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> counter{0};
  return counter;
}
}  // namespace nmb

#define NMB_LAUNCHED(n) ::nmb::launch_counter().fetch_add((n), std::memory_order_relaxed)
