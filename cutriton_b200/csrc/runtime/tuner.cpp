#include "tuner.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <limits>
#include <sstream>
#include <type_traits>
#include <variant>

#include "../backend/json.h"
#include "../cuda_driver.h"
#include "cutriton/backend/kernel_artifact.h"
#include "cutriton/core/buffer.h"

namespace cutriton {
namespace runtime {
namespace {

// A challenger must beat the default's median by more than this fraction.
constexpr double kNoiseMargin = 0.02;

// IEEE binary16 -> double, from the definition of the format.
double HalfValue(std::uint16_t bits) {
  const int sign = (bits >> 15) != 0 ? -1 : 1;
  const int exponent = (bits >> 10) & 0x1F;
  const int fraction = bits & 0x3FF;
  if (exponent == 0x1F) {
    return fraction == 0 ? sign * std::numeric_limits<double>::infinity() : std::numeric_limits<double>::quiet_NaN();
  }
  if (exponent == 0) return sign * std::ldexp(static_cast<double>(fraction), -24);
  return sign * std::ldexp(static_cast<double>(1024 + fraction), exponent - 25);
}

// Host copy of a tensor's elements as doubles (FP32 / FP16 outputs).
Status ReadBack(const Tensor& tensor, std::vector<double>* values) {
  const std::size_t count = static_cast<std::size_t>(tensor.desc().NumElements());
  const std::size_t bytes = tensor.desc().ByteSize();
  std::vector<unsigned char> raw(bytes);
  CUTRITON_RETURN_IF_ERROR(tensor.buffer()->CopyToHost(raw.data(), bytes, tensor.byte_offset()));
  values->resize(count);
  switch (tensor.desc().dtype) {
    case DataType::kFloat32:
      for (std::size_t i = 0; i < count; ++i) {
        float f;
        std::memcpy(&f, raw.data() + 4 * i, 4);
        (*values)[i] = f;
      }
      return Status::OK();
    case DataType::kFloat16:
      for (std::size_t i = 0; i < count; ++i) {
        std::uint16_t h;
        std::memcpy(&h, raw.data() + 2 * i, 2);
        (*values)[i] = HalfValue(h);
      }
      return Status::OK();
    default:
      return Status::Unsupported("the tuner compares float32 / float16 outputs only");
  }
}

// True when `got` matches `want` wherever `want` is finite (intermediate
// inputs hold arbitrary data while tuning, so non-finite reference elements
// carry no information).
bool SameResult(const std::vector<double>& want, const std::vector<double>& got, double tolerance) {
  if (want.size() != got.size()) return false;
  for (std::size_t i = 0; i < want.size(); ++i) {
    if (!std::isfinite(want[i])) continue;
    if (!std::isfinite(got[i]) || std::fabs(got[i] - want[i]) > tolerance * (1.0 + std::fabs(want[i]))) return false;
  }
  return true;
}

template <typename T>
void PutAttribute(std::ostringstream& out, const T& value) {
  if constexpr (std::is_same_v<T, std::vector<int64_t>> || std::is_same_v<T, std::vector<double>>) {
    out << '[';
    for (std::size_t i = 0; i < value.size(); ++i) out << (i ? "," : "") << value[i];
    out << ']';
  } else if constexpr (std::is_same_v<T, double>) {
    out.precision(17);
    out << value;
  } else {
    out << value;
  }
}

std::filesystem::path ChoicePath(const std::string& cache_dir, const std::string& key) {
  return std::filesystem::path(cache_dir) / (key + ".json");
}

struct Timer {
  CUstream stream{nullptr};
  CUevent start{nullptr};
  CUevent stop{nullptr};
  ~Timer() {
    const auto& api = drv::Get();
    if (start != nullptr) api.cuEventDestroy(start);
    if (stop != nullptr) api.cuEventDestroy(stop);
    if (stream != nullptr) api.cuStreamDestroy(stream);
  }
};

}  // namespace

std::string TuningFingerprint(const PlanOp& op, const Node& node, const Graph& graph, int device_id) {
  std::ostringstream text;
  text << "op=" << op.op_type << ";device=" << device_id << ';';
  const auto describe = [&](const char* role, const std::vector<std::string>& names) {
    for (std::size_t i = 0; i < names.size(); ++i) {
      text << role << i << '=' << names[i];
      if (const ValueDesc* value = graph.FindValue(names[i])) {
        text << '/' << DataTypeName(value->tensor.dtype) << '/' << value->tensor.layout << '/';
        for (int64_t d : value->tensor.shape) text << d << 'x';
      }
      text << ';';
    }
  };
  describe("in", op.inputs);
  describe("out", op.outputs);
  std::vector<const std::pair<const std::string, Attribute>*> attributes;
  for (const auto& entry : node.attributes()) attributes.push_back(&entry);
  std::sort(attributes.begin(), attributes.end(), [](const auto* a, const auto* b) { return a->first < b->first; });
  for (const auto* entry : attributes) {
    text << "attr:" << entry->first << '=';
    std::visit([&](const auto& v) { PutAttribute(text, v); }, entry->second);
    text << ';';
  }
  for (const ExecutionCandidate& candidate : op.candidates) {
    text << "candidate=" << candidate.candidate_id;
    for (const PlanStep& step : candidate.steps) {
      if (const auto* kernel = std::get_if<KernelInvocation>(&step)) {
        const KernelArtifact& a = kernel->artifact;
        text << '{' << a.pack_name << '@' << a.pack_version << ':' << a.kernel_id << '@' << a.kernel_version << ':'
             << a.variant_id << ":abi" << a.abi_schema_version << ':' << a.generator_version << ':' << a.sha256 << '}';
      } else {
        text << "{view}";
      }
    }
    text << ';';
  }
  const auto& api = drv::Get();
  CUdevice device{};
  if (api.available && api.cuDeviceGet(&device, device_id) == CUDA_SUCCESS) {
    int major = 0, minor = 0;
    CUuuid uuid{};
    api.cuDeviceGetAttribute(&major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, device);
    api.cuDeviceGetAttribute(&minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, device);
    api.cuDeviceGetUuid(&uuid, device);
    text << "sm=" << major << '.' << minor << ";uuid=";
    for (unsigned char b : uuid.bytes) text << static_cast<int>(b) << '.';
    int driver = 0;
    api.cuDriverGetVersion(&driver);
    text << ";driver=" << driver << ';';
  }
  return Sha256Hex(text.str()).substr(0, 32);
}

std::optional<std::string> LoadTuningChoice(const std::string& cache_dir, const std::string& key) {
  std::ifstream in(ChoicePath(cache_dir, key));
  if (!in) return std::nullopt;
  std::stringstream text;
  text << in.rdbuf();
  try {
    const json::Value doc = json::Parse(text.str());
    if (doc.at("key").str() != key) return std::nullopt;
    return doc.at("choice").str();
  } catch (const std::exception&) {
    return std::nullopt;
  }
}

Status StoreTuningChoice(const std::string& cache_dir, const std::string& key, const PlanOp& op,
                         std::size_t chosen, const std::vector<double>& median_ms) {
  std::error_code error;
  std::filesystem::create_directories(cache_dir, error);
  if (error) return Status::RuntimeError("tuning cache: cannot create " + cache_dir + ": " + error.message());
  const auto escape = [](const std::string& s) {
    std::string out;
    for (char c : s) {
      if (c == '"' || c == '\\') out += '\\';
      out += c;
    }
    return out;
  };
  std::ostringstream doc;
  doc << "{\n  \"format\": \"cutriton_b200.tuning.v1\",\n  \"key\": \"" << key << "\",\n  \"op\": \""
      << escape(op.node_name) << "\",\n  \"choice\": \"" << escape(op.candidates.at(chosen).candidate_id)
      << "\",\n  \"median_ms\": {";
  for (std::size_t c = 0; c < op.candidates.size(); ++c) {
    doc << (c ? ", " : "") << '"' << escape(op.candidates[c].candidate_id) << "\": ";
    if (std::isfinite(median_ms[c])) {
      doc << median_ms[c];
    } else {
      doc << "null";
    }
  }
  doc << "}\n}\n";
  const std::filesystem::path target = ChoicePath(cache_dir, key);
  const std::filesystem::path staging = target.string() + ".partial";
  {
    std::ofstream out(staging, std::ios::trunc);
    out << doc.str();
    if (!out) return Status::RuntimeError("tuning cache: cannot write " + staging.string());
  }
  std::filesystem::rename(staging, target, error);
  if (error) {
    std::filesystem::remove(staging);
    return Status::RuntimeError("tuning cache: cannot publish " + target.string() + ": " + error.message());
  }
  return Status::OK();
}

Status TuneCandidates(const TuningTarget& target, const TuningConfig& config, std::size_t* chosen,
                      std::vector<double>* median_ms) {
  const PlanOp& op = *target.op;
  const auto& api = drv::Get();
  Timer timer;
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuStreamCreate(&timer.stream, CU_STREAM_NON_BLOCKING), "cuStreamCreate"));
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&timer.start, CU_EVENT_DEFAULT), "cuEventCreate"));
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&timer.stop, CU_EVENT_DEFAULT), "cuEventCreate"));

  // Kernels of every candidate (views launch nothing and are not timed).
  std::vector<std::vector<std::unique_ptr<OpKernel>>> kernels(op.candidates.size());
  for (std::size_t c = 0; c < op.candidates.size(); ++c) {
    for (const PlanStep& step : op.candidates[c].steps) {
      if (const auto* invocation = std::get_if<KernelInvocation>(&step)) {
        std::unique_ptr<OpKernel> kernel;
        CUTRITON_RETURN_IF_ERROR(CreateInvocationKernel(*invocation, target.device_id, target.modules, &kernel));
        kernels[c].push_back(std::move(kernel));
      }
    }
  }
  KernelContext context{target.node, target.tensors, timer.stream, nullptr, target.error_word};
  const auto launch = [&](std::size_t c) -> Status {
    for (auto& kernel : kernels[c]) CUTRITON_RETURN_IF_ERROR(kernel->Compute(&context));
    return Status::OK();
  };
  const Tensor& output = target.tensors->at(op.outputs.front());
  const double tolerance = output.desc().dtype == DataType::kFloat16 ? 1e-2 : 1e-4;

  // Warm-up and eligibility, default candidate first (it is the reference).
  const std::size_t fallback = op.selected_candidate;
  std::vector<std::size_t> eligible;
  std::vector<double> reference;
  std::vector<std::size_t> order{fallback};
  for (std::size_t c = 0; c < op.candidates.size(); ++c) {
    if (c != fallback) order.push_back(c);
  }
  for (std::size_t c : order) {
    if (kernels[c].empty()) continue;
    for (int w = 0; w < std::max(1, config.warmup_iterations); ++w) CUTRITON_RETURN_IF_ERROR(launch(c));
    CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuStreamSynchronize(timer.stream), "cuStreamSynchronize"));
    // A candidate whose kernel reported an error (a shape or alignment
    // outside its contract, an abandoned wait) is not eligible; the default
    // candidate's error is the op's error.
    if (target.take_device_error) {
      const Status device = target.take_device_error();
      if (!device.ok()) {
        if (c == fallback) return device;
        continue;
      }
    }
    std::vector<double> produced;
    CUTRITON_RETURN_IF_ERROR(ReadBack(output, &produced));
    if (c == fallback) {
      reference = std::move(produced);
    } else if (!SameResult(reference, produced, tolerance)) {
      continue;
    }
    eligible.push_back(c);
  }
  if (eligible.empty()) return Status::RuntimeError("tuner: no candidate of " + op.node_name + " could run");

  // Interleaved timing rounds. Each timed launch queues behind an untimed
  // one of the same candidate, so its host-side preparation (argument
  // binding, tensor-map encoding) runs while the GPU is busy and the events
  // bracket device time only; a candidate with more tensor maps is not
  // charged for them, as it is not inside a captured graph.
  std::vector<std::vector<double>> samples(op.candidates.size());
  for (int round = 0; round < std::max(1, config.measurement_iterations); ++round) {
    for (std::size_t c : eligible) {
      CUTRITON_RETURN_IF_ERROR(launch(c));
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventRecord(timer.start, timer.stream), "cuEventRecord"));
      CUTRITON_RETURN_IF_ERROR(launch(c));
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventRecord(timer.stop, timer.stream), "cuEventRecord"));
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventSynchronize(timer.stop), "cuEventSynchronize"));
      float ms = 0.0f;
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventElapsedTime(&ms, timer.start, timer.stop), "cuEventElapsedTime"));
      samples[c].push_back(ms);
    }
  }
  if (target.take_device_error) CUTRITON_RETURN_IF_ERROR(target.take_device_error());
  median_ms->assign(op.candidates.size(), std::numeric_limits<double>::infinity());
  for (std::size_t c : eligible) {
    auto& s = samples[c];
    std::nth_element(s.begin(), s.begin() + s.size() / 2, s.end());
    (*median_ms)[c] = s[s.size() / 2];
  }
  std::size_t best = eligible.front();
  for (std::size_t c : eligible) {
    if ((*median_ms)[c] < (*median_ms)[best]) best = c;
  }
  // Keep the default unless the winner clearly beats it.
  if (best != fallback && std::isfinite((*median_ms)[fallback]) &&
      (*median_ms)[best] > (1.0 - kNoiseMargin) * (*median_ms)[fallback]) {
    best = fallback;
  }
  *chosen = best;
  return Status::OK();
}

}  // namespace runtime
}  // namespace cutriton
