#pragma once

// Per-op timing records (API of the reference's
// include/cutriton/runtime/profiler.h:10-36). CUDA ops are timed with events
// around each plan op; CPU/mock kernels use ScopedCpuTimer.

#include <chrono>
#include <string>
#include <vector>

namespace cutriton {

struct ProfileEvent {
  std::string name;
  std::string backend;
  double duration_ms{0.0};
};

class Profiler {
 public:
  void Record(std::string name, std::string backend, double duration_ms);
  const std::vector<ProfileEvent>& events() const { return events_; }
  void Clear() { events_.clear(); }

 private:
  std::vector<ProfileEvent> events_;
};

class ScopedCpuTimer {
 public:
  ScopedCpuTimer(Profiler* profiler, std::string name, std::string backend);
  ~ScopedCpuTimer();

 private:
  Profiler* profiler_{nullptr};
  std::string name_;
  std::string backend_;
  std::chrono::steady_clock::time_point start_;
};

}  // namespace cutriton
