#pragma once

// Declarative execution candidates produced by Backend::Lower (API of the
// reference's include/cutriton/backend/kernel_invocation.h:11-35).

#include <string>
#include <variant>
#include <vector>

#include "cutriton/backend/kernel_artifact.h"

namespace cutriton {

struct KernelInvocation {
  KernelArtifact artifact;
  std::vector<std::string> inputs;
  std::vector<std::string> outputs;
};

// Zero-copy alias (Flatten): output views the input's bytes.
struct ViewInvocation {
  std::string input;
  std::string output;
};

// Scratch tensor of an unfused candidate; shaped like `like_value`, placed in
// a shared workspace slot.
struct CandidateTemporary {
  std::string name;
  std::string like_value;
  std::size_t slot{0};
};

using PlanStep = std::variant<KernelInvocation, ViewInvocation>;

struct ExecutionCandidate {
  std::string candidate_id;
  std::vector<PlanStep> steps;
  std::vector<CandidateTemporary> temporaries;
  bool is_default{false};
};

}  // namespace cutriton
