// Bounded host waits on the device. Every wait of the device on itself is
// bounded (an mbarrier wait gives up after 1 s and records MS_E_TIMEOUT), so
// a stream that is still busy after host_wait_limit_s() seconds is stuck,
// not slow: the entry point returns MS_E_TIMEOUT instead of blocking its
// caller forever.
#pragma once
#include <chrono>
#include <cstdlib>
#include <thread>

#include <cuda_runtime.h>

namespace ms {

// MS_HOST_WAIT_S from the environment (seconds, > 0), default 60.
inline double host_wait_limit_s() {
  static const double v = [] {
    const char* e = std::getenv("MS_HOST_WAIT_S");
    const double d = e ? std::atof(e) : 0.0;
    return d > 0.0 ? d : 60.0;
  }();
  return v;
}

// Polls query() (cudaStreamQuery / cudaEventQuery) until it stops answering
// cudaErrorNotReady or the limit passes. Yields for the first 2 ms, then
// sleeps 20 us between polls. Returns the query's answer, or
// cudaErrorTimeout.
template <class Q>
inline cudaError_t poll_bounded(Q query) {
  const auto t0 = std::chrono::steady_clock::now();
  const double limit = host_wait_limit_s();
  for (unsigned it = 0;; ++it) {
    const cudaError_t e = query();
    if (e != cudaErrorNotReady) return e;
    if ((it & 31) == 31) {
      const double el =
          std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if (el > limit) return cudaErrorTimeout;
      if (el > 2e-3) {
        std::this_thread::sleep_for(std::chrono::microseconds(20));
        continue;
      }
    }
    std::this_thread::yield();
  }
}

inline cudaError_t stream_wait_bounded(cudaStream_t s) {
  return poll_bounded([s] { return cudaStreamQuery(s); });
}
inline cudaError_t event_wait_bounded(cudaEvent_t ev) {
  return poll_bounded([ev] { return cudaEventQuery(ev); });
}

}  // namespace ms
