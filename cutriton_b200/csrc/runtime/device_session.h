#pragma once

// Per-context CUDA resources of an ExecutionContext.
//
//   DeviceSession  the retained primary context, the context's own stream,
//                  one start/end event pair per plan op (profiling), and the
//                  error block: a pinned, device-mapped host word that
//                  kernels with bounded waits write when a wait expires
//                  (layout shared with kernels/common.cuh).
//   GraphCache     instantiated CUDA Graphs keyed by the launch fingerprint
//                  (bound addresses, shapes, workspace, selected candidates),
//                  least recently used first out; O(1) lookup by hash with the
//                  full fingerprint compared on a hit.

#include <cstdint>
#include <functional>
#include <list>
#include <memory>
#include <unordered_map>
#include <vector>

#include "../cuda_driver.h"
#include "cutriton/core/status.h"

namespace cutriton {
namespace runtime {

struct DeviceErrorWord {
  std::uint32_t code;   // 0 = no error
  std::uint32_t site;   // kernel-defined location of the expired wait
  std::uint32_t block;  // linear CTA index that gave up
  std::uint32_t reserved[13];
};

class DeviceSession {
 public:
  // Retains device `device_id`'s primary context and creates the stream,
  // the error word and `op_count` event pairs (only when `profiling`).
  static Status Open(int device_id, std::size_t op_count, bool profiling, std::unique_ptr<DeviceSession>* out);
  ~DeviceSession();
  DeviceSession(const DeviceSession&) = delete;
  DeviceSession& operator=(const DeviceSession&) = delete;

  Status MakeCurrent() const;
  CUstream own_stream() const { return own_stream_; }
  void* error_word_device() const { return reinterpret_cast<void*>(error_device_); }
  // Reads and clears the error word; a non-OK status describes the expired wait.
  Status TakeDeviceError();
  CUevent op_start(std::size_t op) const { return events_[op].first; }
  CUevent op_end(std::size_t op) const { return events_[op].second; }
  bool has_events() const { return !events_.empty(); }

 private:
  DeviceSession() = default;

  CUdevice device_{};
  CUcontext context_{nullptr};
  CUstream own_stream_{nullptr};
  DeviceErrorWord* error_host_{nullptr};
  CUdeviceptr error_device_{0};
  std::vector<std::pair<CUevent, CUevent>> events_;
};

// 64-bit hash of a launch fingerprint (a sequence of 64-bit words).
std::uint64_t HashWords(const std::vector<std::uint64_t>& words);

class GraphCache {
 public:
  explicit GraphCache(std::size_t capacity) : capacity_(capacity == 0 ? 1 : capacity) {}
  ~GraphCache() { Clear(); }
  GraphCache(const GraphCache&) = delete;
  GraphCache& operator=(const GraphCache&) = delete;

  // The executable graph for `fingerprint`, capturing it with `record` (which
  // enqueues the work on `stream`) on a miss and evicting the least recently
  // used entry when full.
  Status Acquire(const std::vector<std::uint64_t>& fingerprint, CUstream stream,
                 const std::function<Status()>& record, CUgraphExec* exec);
  void Clear();
  std::size_t size() const { return order_.size(); }

 private:
  struct Entry {
    std::vector<std::uint64_t> fingerprint;
    std::uint64_t hash{0};
    CUgraph graph{nullptr};
    CUgraphExec exec{nullptr};
  };
  static void Release(Entry* entry);

  std::size_t capacity_;
  std::list<Entry> order_;  // most recently used first
  std::unordered_multimap<std::uint64_t, std::list<Entry>::iterator> by_hash_;
};

}  // namespace runtime
}  // namespace cutriton
