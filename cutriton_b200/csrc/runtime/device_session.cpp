#include "device_session.h"

#include <cstring>
#include <sstream>

namespace cutriton {
namespace runtime {

Status DeviceSession::Open(int device_id, std::size_t op_count, bool profiling, std::unique_ptr<DeviceSession>* out) {
  std::unique_ptr<DeviceSession> session(new DeviceSession());
  CUTRITON_RETURN_IF_ERROR(drv::RetainPrimaryContext(device_id, &session->device_, &session->context_));
  const auto& api = drv::Get();
  CUTRITON_RETURN_IF_ERROR(
      drv::Check(api.cuStreamCreate(&session->own_stream_, CU_STREAM_NON_BLOCKING), "cuStreamCreate"));
  void* host = nullptr;
  CUTRITON_RETURN_IF_ERROR(drv::Check(
      api.cuMemHostAlloc(&host, sizeof(DeviceErrorWord), CU_MEMHOSTALLOC_DEVICEMAP | CU_MEMHOSTALLOC_PORTABLE),
      "cuMemHostAlloc"));
  session->error_host_ = static_cast<DeviceErrorWord*>(host);
  std::memset(host, 0, sizeof(DeviceErrorWord));
  CUTRITON_RETURN_IF_ERROR(
      drv::Check(api.cuMemHostGetDevicePointer(&session->error_device_, host, 0), "cuMemHostGetDevicePointer"));
  if (profiling) {
    session->events_.assign(op_count, {nullptr, nullptr});
    for (auto& pair : session->events_) {
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&pair.first, CU_EVENT_DEFAULT), "cuEventCreate"));
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&pair.second, CU_EVENT_DEFAULT), "cuEventCreate"));
    }
  }
  *out = std::move(session);
  return Status::OK();
}

DeviceSession::~DeviceSession() {
  const auto& api = drv::Get();
  if (context_ != nullptr) api.cuCtxSetCurrent(context_);
  for (auto& pair : events_) {
    if (pair.first != nullptr) api.cuEventDestroy(pair.first);
    if (pair.second != nullptr) api.cuEventDestroy(pair.second);
  }
  if (own_stream_ != nullptr) api.cuStreamDestroy(own_stream_);
  if (error_host_ != nullptr) api.cuMemFreeHost(error_host_);
  if (context_ != nullptr) api.cuDevicePrimaryCtxRelease(device_);
}

Status DeviceSession::MakeCurrent() const { return drv::Check(drv::Get().cuCtxSetCurrent(context_), "cuCtxSetCurrent"); }

Status DeviceSession::TakeDeviceError() {
  if (error_host_ == nullptr || error_host_->code == 0) return Status::OK();
  std::ostringstream what;
  what << "a kernel abandoned a bounded wait (code " << error_host_->code << ", site " << error_host_->site
       << ", block " << error_host_->block << ")";
  std::memset(error_host_, 0, sizeof(DeviceErrorWord));
  return Status::RuntimeError(what.str());
}

std::uint64_t HashWords(const std::vector<std::uint64_t>& words) {
  // splitmix64 finaliser folded over the words.
  std::uint64_t h = 0x9E3779B97F4A7C15ull ^ words.size();
  for (std::uint64_t w : words) {
    std::uint64_t z = w + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    h ^= z ^ (z >> 31);
  }
  return h;
}

void GraphCache::Release(Entry* entry) {
  const auto& api = drv::Get();
  if (entry->exec != nullptr) api.cuGraphExecDestroy(entry->exec);
  if (entry->graph != nullptr) api.cuGraphDestroy(entry->graph);
  entry->exec = nullptr;
  entry->graph = nullptr;
}

void GraphCache::Clear() {
  for (Entry& entry : order_) Release(&entry);
  order_.clear();
  by_hash_.clear();
}

Status GraphCache::Acquire(const std::vector<std::uint64_t>& fingerprint, CUstream stream,
                           const std::function<Status()>& record, CUgraphExec* exec) {
  const std::uint64_t hash = HashWords(fingerprint);
  const auto range = by_hash_.equal_range(hash);
  for (auto it = range.first; it != range.second; ++it) {
    if (it->second->fingerprint != fingerprint) continue;
    order_.splice(order_.begin(), order_, it->second);  // now most recent
    *exec = order_.front().exec;
    return Status::OK();
  }

  const auto& api = drv::Get();
  Entry fresh;
  fresh.fingerprint = fingerprint;
  fresh.hash = hash;
  CUTRITON_RETURN_IF_ERROR(
      drv::Check(api.cuStreamBeginCapture(stream, CU_STREAM_CAPTURE_MODE_GLOBAL), "cuStreamBeginCapture"));
  const Status recorded = record();
  // Capture must end whatever happened while recording.
  const Status ended = drv::Check(api.cuStreamEndCapture(stream, &fresh.graph), "cuStreamEndCapture");
  Status status = !recorded.ok() ? recorded : ended;
  if (status.ok()) {
    status = drv::Check(api.cuGraphInstantiateWithFlags(&fresh.exec, fresh.graph, 0), "cuGraphInstantiateWithFlags");
  }
  if (!status.ok()) {
    Release(&fresh);
    return status;
  }
  while (order_.size() >= capacity_) {
    Entry& victim = order_.back();
    const auto victims = by_hash_.equal_range(victim.hash);
    for (auto it = victims.first; it != victims.second; ++it) {
      if (&*it->second == &victim) {
        by_hash_.erase(it);
        break;
      }
    }
    Release(&victim);
    order_.pop_back();
  }
  order_.push_front(std::move(fresh));
  by_hash_.emplace(hash, order_.begin());
  *exec = order_.front().exec;
  return Status::OK();
}

}  // namespace runtime
}  // namespace cutriton
