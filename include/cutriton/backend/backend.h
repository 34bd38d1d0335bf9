#pragma once

// Backend plugin interface and registry (API of the reference's
// include/cutriton/backend/backend.h:18-104). The only production backend in
// this library is "cuda_sm100": artifact-backed sm_100a cubins launched by the
// generic driver-API launcher. "cuda_triton" is accepted as a target alias.

#include <memory>
#include <shared_mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "cutriton/backend/kernel_artifact.h"
#include "cutriton/backend/kernel_invocation.h"
#include "cutriton/core/device.h"
#include "cutriton/core/status.h"
#include "cutriton/core/tensor.h"
#include "cutriton/ir/graph.h"

namespace cutriton {

class Profiler;
class CudaModuleCache;

struct BackendOptions {
  Device device{};
  std::vector<std::string> kernel_artifact_paths;
  // Single-pack spelling kept for source compatibility.
  std::string kernel_artifact_dir;
};

struct LoweringContext {
  const Graph* graph{nullptr};
  const BackendOptions* options{nullptr};
  const ArtifactRepository* artifacts{nullptr};
  const KernelCatalog* catalog{nullptr};
};

// Per-call runtime objects; valid only during OpKernel::Compute.
struct KernelContext {
  const Node* node{nullptr};
  std::unordered_map<std::string, Tensor>* tensors{nullptr};
  void* stream{nullptr};  // CUstream for CUDA backends
  Profiler* profiler{nullptr};
  // Device address bound to a kernel's first runtime_reserved parameter: the
  // context's error block (kernels record expired bounded waits there).
  void* runtime_scratch{nullptr};
};

class OpKernel {
 public:
  virtual ~OpKernel() = default;
  virtual const char* backend_name() const = 0;
  virtual const char* op_type() const = 0;
  virtual Status Compute(KernelContext* context) = 0;
};

class Backend {
 public:
  virtual ~Backend() = default;
  virtual const char* name() const = 0;
  virtual Status CheckSupport(const Node& node, const Graph& graph,
                              const BackendOptions& options) const = 0;
  // Default: one legacy candidate whose kernel comes from CreateKernel.
  virtual Status Lower(const Node& node, const LoweringContext& context,
                       std::vector<ExecutionCandidate>* candidates) const;
  virtual Status CreateKernel(const Node& node, const Graph& graph,
                              const BackendOptions& options,
                              std::unique_ptr<OpKernel>* kernel) const = 0;
};

class KernelRegistry {
 public:
  static KernelRegistry& Global();
  Status RegisterBackend(std::shared_ptr<Backend> backend);
  std::shared_ptr<Backend> GetBackend(const std::string& name) const;
  std::vector<std::string> AvailableBackends() const;
  void ClearForTests();

 private:
  mutable std::shared_mutex mutex_;
  std::unordered_map<std::string, std::shared_ptr<Backend>> backends_;
};

std::shared_ptr<Backend> CreateCpuReferenceBackend();
std::shared_ptr<Backend> CreateCudaSm100Backend();
// Source-compatibility spelling: returns the cuda_sm100 backend.
std::shared_ptr<Backend> CreateCudaTritonBackend();
Status RegisterBuiltinBackends();

// True for target names served by the artifact-backed CUDA backend.
bool IsCudaArtifactTarget(const std::string& target);
// Maps a user-facing target ("cuda_triton" alias included) to a backend name.
std::string CanonicalTargetName(const std::string& target);

Status CreateCudaModuleCache(int device_id, std::shared_ptr<CudaModuleCache>* cache);
Status CreateInvocationKernel(const KernelInvocation& invocation, int device_id,
                              std::shared_ptr<CudaModuleCache> cache,
                              std::unique_ptr<OpKernel>* kernel);
std::size_t LoadedModuleCount(const std::shared_ptr<CudaModuleCache>& cache);

}  // namespace cutriton
