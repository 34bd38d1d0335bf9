#pragma once

// Candidate selection for one plan op (TuningMode kTuneOnMiss /
// kForceRetune), and the on-disk cache of the choices.
//
// The cache key is a SHA-256 digest of a canonical description of the op:
// op type, each tensor's role, name, dtype, layout and shape, the sorted
// attributes, every candidate's kernel identity (pack, kernel, variant,
// ABI, binary digest) and the device (compute capability, UUID) and driver.
// A choice is one small JSON file per key, written to a temporary file and
// renamed into place, so readers never see a partial file.
//
// Measurement: every candidate is launched `warmup` times, its output is
// compared with the default candidate's (a candidate that computes
// something else is never eligible), then the eligible candidates are timed
// in interleaved rounds (A B C A B C ...) with CUDA events so clock and
// thermal drift hit them alike; the median decides. Another candidate
// replaces the default only when it is faster by more than the noise margin.

#include <functional>
#include <memory>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

#include "cutriton/backend/backend.h"
#include "cutriton/ir/graph.h"
#include "cutriton/runtime/executable_plan.h"
#include "cutriton/runtime/tuning.h"

namespace cutriton {
namespace runtime {

std::string TuningFingerprint(const PlanOp& op, const Node& node, const Graph& graph, int device_id);

// The candidate id stored for `key`, if any (unreadable files count as misses).
std::optional<std::string> LoadTuningChoice(const std::string& cache_dir, const std::string& key);
Status StoreTuningChoice(const std::string& cache_dir, const std::string& key, const PlanOp& op,
                         std::size_t chosen, const std::vector<double>& median_ms);

struct TuningTarget {
  const PlanOp* op{nullptr};
  const Node* node{nullptr};
  int device_id{0};
  std::unordered_map<std::string, Tensor>* tensors{nullptr};
  void* error_word{nullptr};
  // Reads and clears the device error word (after a synchronize); a non-OK
  // status means a kernel of the candidate just run reported an error.
  std::function<Status()> take_device_error;
  std::shared_ptr<CudaModuleCache> modules;
};

// Picks the candidate of `target.op` to run; `median_ms` gets one entry per
// candidate (infinity for the ineligible ones).
Status TuneCandidates(const TuningTarget& target, const TuningConfig& config, std::size_t* chosen,
                      std::vector<double>* median_ms);

}  // namespace runtime
}  // namespace cutriton
