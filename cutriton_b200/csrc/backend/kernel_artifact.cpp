// Kernel Pack loader (pack.json schema v2, ABI v1/v2) and catalog.
//
// Validation rules follow the reference loader
// (src/backend/kernel_artifact.cpp:342-532): required keys, safe relative
// binary paths, SHA-256 of every binary, two trailing runtime_reserved
// arguments, grid AST depth <= 8 with a closed node set, a closed constraint
// set, and exactly one default variant per op type being present. Extensions:
// binary_format "cubin", argument source "tensor_map" / "input_numel",
// argument field "prepack", and the constraints listed in kernel_artifact.h.

#include "cutriton/backend/kernel_artifact.h"

#include <array>
#include <fstream>
#include <iomanip>
#include <sstream>
#include <stdexcept>
#include <unordered_set>

#include "json.h"

namespace cutriton {
namespace {

// ---- SHA-256 (FIPS 180-4) ---------------------------------------------------

constexpr std::array<std::uint32_t, 64> kRoundConstants = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u,
    0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu,
    0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu,
    0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau, 0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u,
    0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu,
    0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
    0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u, 0x19a4c116u,
    0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u,
    0xc67178f2u};

inline std::uint32_t Rotr(std::uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void CompressBlock(std::array<std::uint32_t, 8>& state, const unsigned char* block) {
  std::uint32_t w[64];
  for (int t = 0; t < 16; ++t) {
    w[t] = (std::uint32_t(block[4 * t]) << 24) | (std::uint32_t(block[4 * t + 1]) << 16) |
           (std::uint32_t(block[4 * t + 2]) << 8) | std::uint32_t(block[4 * t + 3]);
  }
  for (int t = 16; t < 64; ++t) {
    const std::uint32_t sigma0 = Rotr(w[t - 15], 7) ^ Rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
    const std::uint32_t sigma1 = Rotr(w[t - 2], 17) ^ Rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
    w[t] = w[t - 16] + sigma0 + w[t - 7] + sigma1;
  }
  std::array<std::uint32_t, 8> v = state;  // a..h
  for (int t = 0; t < 64; ++t) {
    const std::uint32_t big_sigma1 = Rotr(v[4], 6) ^ Rotr(v[4], 11) ^ Rotr(v[4], 25);
    const std::uint32_t choose = (v[4] & v[5]) ^ (~v[4] & v[6]);
    const std::uint32_t t1 = v[7] + big_sigma1 + choose + kRoundConstants[t] + w[t];
    const std::uint32_t big_sigma0 = Rotr(v[0], 2) ^ Rotr(v[0], 13) ^ Rotr(v[0], 22);
    const std::uint32_t majority = (v[0] & v[1]) ^ (v[0] & v[2]) ^ (v[1] & v[2]);
    const std::uint32_t t2 = big_sigma0 + majority;
    for (int i = 7; i > 0; --i) v[i] = v[i - 1];
    v[4] += t1;
    v[0] = t1 + t2;
  }
  for (int i = 0; i < 8; ++i) state[i] += v[i];
}

// ---- manifest field helpers -------------------------------------------------

int AsInt(const json::Value& v) { return static_cast<int>(v.num()); }

int IntOr(const json::Value& object, const char* key, int fallback) {
  const json::Value* v = object.find(key);
  return v == nullptr ? fallback : AsInt(*v);
}

double DoubleOr(const json::Value& object, const char* key, double fallback) {
  const json::Value* v = object.find(key);
  return v == nullptr ? fallback : v->num();
}

std::vector<int64_t> IntList(const json::Value& v) {
  std::vector<int64_t> out;
  for (const auto& item : v.list()) out.push_back(static_cast<int64_t>(item.num()));
  return out;
}

void OnlyKeys(const json::Value& v, std::initializer_list<const char*> allowed, const char* what) {
  std::unordered_set<std::string> ok(allowed.begin(), allowed.end());
  for (const auto& member : v.object()) {
    if (ok.count(member.first) == 0) {
      throw std::runtime_error(std::string("unknown ") + what + " field: " + member.first);
    }
  }
}

KernelArgumentSourceKind SourceKindOf(const std::string& kind) {
  static const std::pair<const char*, KernelArgumentSourceKind> table[] = {
      {"input", KernelArgumentSourceKind::kInput},
      {"output", KernelArgumentSourceKind::kOutput},
      {"input_dim", KernelArgumentSourceKind::kInputDim},
      {"input_dim_product", KernelArgumentSourceKind::kInputDimProduct},
      {"output_dim", KernelArgumentSourceKind::kOutputDim},
      {"output_numel", KernelArgumentSourceKind::kOutputNumElements},
      {"input_numel", KernelArgumentSourceKind::kInputNumElements},
      {"attribute_i64", KernelArgumentSourceKind::kAttributeInt64},
      {"attribute_f64", KernelArgumentSourceKind::kAttributeFloat64},
      {"literal_i32", KernelArgumentSourceKind::kLiteralInt32},
      {"runtime_reserved", KernelArgumentSourceKind::kRuntimeReserved},
      {"tensor_map", KernelArgumentSourceKind::kTensorMap},
  };
  for (const auto& entry : table) {
    if (kind == entry.first) return entry.second;
  }
  throw std::runtime_error("unsupported argument source: " + kind);
}

GridExpression GridNode(const json::Value& v, int depth) {
  if (depth > 8) throw std::runtime_error("grid expression is too deep");
  GridExpression e;
  const std::string& kind = v.at("kind").str();
  if (kind == "literal") {
    OnlyKeys(v, {"kind", "value"}, "grid expression");
    e.kind = GridExpressionKind::kLiteral;
    e.literal = AsInt(v.at("value"));
    if (e.literal <= 0) throw std::runtime_error("grid literal must be positive");
  } else if (kind == "input_dim" || kind == "output_dim") {
    OnlyKeys(v, {"kind", "index", "axis"}, "grid expression");
    e.kind = kind == "input_dim" ? GridExpressionKind::kInputDim : GridExpressionKind::kOutputDim;
    e.tensor_index = AsInt(v.at("index"));
    e.axis = AsInt(v.at("axis"));
  } else if (kind == "input_numel" || kind == "output_numel") {
    OnlyKeys(v, {"kind", "index"}, "grid expression");
    e.kind = kind == "input_numel" ? GridExpressionKind::kInputNumElements
                                   : GridExpressionKind::kOutputNumElements;
    e.tensor_index = AsInt(v.at("index"));
  } else if (kind == "meta") {
    OnlyKeys(v, {"kind", "name"}, "grid expression");
    e.kind = GridExpressionKind::kVariantMeta;
    e.meta_name = v.at("name").str();
    if (e.meta_name.empty()) throw std::runtime_error("grid meta name is empty");
  } else if (kind == "sm_count") {
    OnlyKeys(v, {"kind"}, "grid expression");
    e.kind = GridExpressionKind::kDeviceSmCount;
  } else if (kind == "ceil_div" || kind == "mul" || kind == "min") {
    OnlyKeys(v, {"kind", "args"}, "grid expression");
    const auto& args = v.at("args").list();
    if (args.size() != 2) throw std::runtime_error(kind + " grid expression needs two operands");
    e.kind = kind == "ceil_div" ? GridExpressionKind::kCeilDiv
             : kind == "mul"    ? GridExpressionKind::kMultiply
                                : GridExpressionKind::kMinimum;
    for (const auto& arg : args) e.operands.push_back(GridNode(arg, depth + 1));
  } else {
    throw std::runtime_error("unsupported grid expression kind: " + kind);
  }
  return e;
}

// ABI v1: {"op":"ceil_div","value":{"kind":"output_numel","index":i},"divisor":d}
GridExpression LegacyGrid(const json::Value& v) {
  if (v.at("op").str() != "ceil_div" || v.at("value").at("kind").str() != "output_numel") {
    throw std::runtime_error("unsupported ABI v1 grid expression");
  }
  GridExpression numel;
  numel.kind = GridExpressionKind::kOutputNumElements;
  numel.tensor_index = IntOr(v.at("value"), "index", 0);
  GridExpression divisor;
  divisor.literal = AsInt(v.at("divisor"));
  if (divisor.literal <= 0) throw std::runtime_error("grid divisor must be positive");
  GridExpression e;
  e.kind = GridExpressionKind::kCeilDiv;
  e.operands = {numel, divisor};
  return e;
}

KernelArgumentSpec ParseArgument(const json::Value& v) {
  KernelArgumentSpec arg;
  arg.name = v.at("name").str();
  arg.type = v.at("type").str();
  const json::Value& src = v.at("source");
  KernelArgumentSource& s = arg.source;
  s.kind = SourceKindOf(src.at("kind").str());
  s.index = IntOr(src, "index", 0);
  s.axis = IntOr(src, "axis", 0);
  s.begin_axis = IntOr(src, "begin_axis", 0);
  if (const auto* name = src.find("name")) s.attribute_name = name->str();
  if (const auto* alt = src.find("alternate_name")) s.alternate_attribute_name = alt->str();
  s.attribute_index = IntOr(src, "index", 0);
  s.default_int = IntOr(src, "default", 0);
  s.default_float = DoubleOr(src, "default", 0.0);
  if (const auto* prepack = src.find("prepack")) s.prepack = prepack->str();
  if (s.kind == KernelArgumentSourceKind::kTensorMap) {
    const std::string& tensor = src.at("tensor").str();
    if (tensor != "input" && tensor != "output") {
      throw std::runtime_error("tensor_map source must name an input or output");
    }
    s.map_output = tensor == "output";
    s.box = IntList(src.at("box"));
    s.swizzle_bytes = IntOr(src, "swizzle", 0);
    s.swizzle_atom_bytes = static_cast<int>(IntOr(src, "swizzle_atom", 0));
    s.merge_inner = static_cast<int>(IntOr(src, "merge_inner", 1));
    s.optional = IntOr(src, "optional", 0) != 0;
    if (s.merge_inner < 1 || s.merge_inner > 4) throw std::runtime_error("tensor_map merge_inner must be 1..4");
    if (s.box.empty() || s.box.size() > 5) throw std::runtime_error("tensor_map box rank must be 1..5");
    for (int64_t extent : s.box) {
      if (extent <= 0 || extent > 256) throw std::runtime_error("tensor_map box extent must be 1..256");
    }
    if (s.swizzle_bytes != 0 && s.swizzle_bytes != 32 && s.swizzle_bytes != 64 &&
        s.swizzle_bytes != 128) {
      throw std::runtime_error("tensor_map swizzle must be 0, 32, 64 or 128");
    }
    if (s.swizzle_atom_bytes != 0 && (s.swizzle_atom_bytes != 32 || s.swizzle_bytes != 128)) {
      throw std::runtime_error("tensor_map swizzle_atom must be 32 with a 128-byte swizzle");
    }
  }
  return arg;
}

KernelConstraint ParseConstraint(const json::Value& v) {
  KernelConstraint c;
  const std::string& kind = v.at("kind").str();
  auto tensor_ref = [&]() {
    const std::string& source = v.at("source").str();
    if (source != "input" && source != "output") {
      throw std::runtime_error(kind + " source must be input or output");
    }
    c.tensor_is_output = source == "output";
    c.tensor_index = IntOr(v, "index", 0);
  };
  if (kind == "attribute_i64_eq") {
    c.kind = KernelConstraintKind::kAttributeInt64Equals;
    c.attribute_name = v.at("name").str();
    c.expected = AsInt(v.at("value"));
    c.default_value = IntOr(v, "default", 0);
  } else if (kind == "input_count_eq") {
    c.kind = KernelConstraintKind::kInputCountEquals;
    c.expected = AsInt(v.at("value"));
  } else if (kind == "tensor_rank_eq") {
    c.kind = KernelConstraintKind::kTensorRankEquals;
    tensor_ref();
    c.expected = AsInt(v.at("value"));
  } else if (kind == "attribute_list_eq") {
    c.kind = KernelConstraintKind::kAttributeListEquals;
    c.attribute_name = v.at("name").str();
    c.expected_list = IntList(v.at("value"));
    if (const auto* d = v.find("default")) c.default_list = IntList(*d);
  } else if (kind == "dim_multiple_of" || kind == "dim_le") {
    c.kind = kind == "dim_le" ? KernelConstraintKind::kDimLessEqual
                              : KernelConstraintKind::kDimMultipleOf;
    tensor_ref();
    c.axis = AsInt(v.at("axis"));
    c.expected = AsInt(v.at("value"));
    if (c.expected <= 0) throw std::runtime_error(kind + " value must be positive");
  } else if (kind == "input_is_constant") {
    c.kind = KernelConstraintKind::kInputIsConstant;
    c.tensor_index = AsInt(v.at("index"));
  } else {
    throw std::runtime_error("unsupported kernel constraint: " + kind);
  }
  return c;
}

std::string ReadFile(const std::filesystem::path& path, bool* ok) {
  std::ifstream in(path, std::ios::binary);
  *ok = static_cast<bool>(in);
  std::ostringstream data;
  if (*ok) data << in.rdbuf();
  return data.str();
}

}  // namespace

std::string Sha256Hex(const std::string& bytes) {
  std::array<std::uint32_t, 8> state = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                        0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  const auto* data = reinterpret_cast<const unsigned char*>(bytes.data());
  const std::size_t full = bytes.size() / 64;
  for (std::size_t b = 0; b < full; ++b) CompressBlock(state, data + 64 * b);
  // Final one or two blocks: remaining bytes, 0x80, zero pad, 64-bit length.
  unsigned char tail[128] = {0};
  const std::size_t rest = bytes.size() - 64 * full;
  for (std::size_t i = 0; i < rest; ++i) tail[i] = data[64 * full + i];
  tail[rest] = 0x80;
  const std::size_t tail_len = rest + 1 + 8 <= 64 ? 64 : 128;
  const std::uint64_t bit_length = static_cast<std::uint64_t>(bytes.size()) * 8u;
  for (int i = 0; i < 8; ++i) tail[tail_len - 1 - i] = static_cast<unsigned char>(bit_length >> (8 * i));
  CompressBlock(state, tail);
  if (tail_len == 128) CompressBlock(state, tail + 64);
  std::ostringstream hex;
  hex << std::hex << std::setfill('0');
  for (std::uint32_t word : state) hex << std::setw(8) << word;
  return hex.str();
}

Status ArtifactRepository::Load(const std::vector<std::string>& paths) {
  artifacts_.clear();
  by_op_type_.clear();
  repository_hash_.clear();
  if (paths.empty()) return Status::InvalidArgument("kernel artifact paths are empty");
  std::string digest_material;
  std::vector<KernelArtifact> loaded;
  try {
    for (const auto& item : paths) {
      std::filesystem::path manifest(item);
      if (std::filesystem::is_directory(manifest)) manifest /= "pack.json";
      if (!std::filesystem::exists(manifest)) {
        return Status::NotFound("Kernel Pack not found: " + manifest.string());
      }
      const std::filesystem::path root = manifest.parent_path();
      bool readable = false;
      const std::string text = ReadFile(manifest, &readable);
      if (!readable) return Status::NotFound("Kernel Pack is unreadable: " + manifest.string());
      const json::Value pack = json::Parse(text);
      if (AsInt(pack.at("schema_version")) != 2) {
        return Status::InvalidArgument("Kernel Pack schema v2 is required; regenerate artifacts");
      }
      const int abi = AsInt(pack.at("abi_schema_version"));
      if (abi != 1 && abi != 2) return Status::InvalidArgument("unsupported Kernel Pack ABI schema");
      const std::string pack_name = pack.at("pack_name").str();
      const int pack_version = AsInt(pack.at("pack_version"));
      const std::string generator = pack.at("generator_version").str();
      const std::string triton_version = pack.at("triton_version").str();
      digest_material += Sha256Hex(text);
      for (const auto& entry : pack.at("kernels").list()) {
        KernelArtifact a;
        a.pack_name = pack_name;
        a.pack_version = pack_version;
        a.generator_version = generator;
        a.triton_version = triton_version;
        a.abi_schema_version = abi;
        a.kernel_id = entry.at("kernel_id").str();
        a.op_type = entry.at("op_type").str();
        a.kernel_version = AsInt(entry.at("kernel_version"));
        a.variant_id = entry.at("variant_id").str();
        a.is_default = entry.at("default").flag();
        a.symbol = entry.at("symbol").str();
        a.binary_format = entry.at("binary_format").str();
        a.sha256 = entry.at("sha256").str();
        a.dtype = entry.at("dtype").str();
        a.layout = entry.at("layout").str();
        a.min_compute_capability = AsInt(entry.at("min_compute_capability"));
        a.num_warps = AsInt(entry.at("num_warps"));
        a.num_stages = AsInt(entry.at("num_stages"));
        a.shared_memory_bytes = AsInt(entry.at("shared_memory_bytes"));
        a.programmatic_launch = a.binary_format == "cubin" && IntOr(entry, "programmatic_launch", 0) != 0;
        if (a.num_warps <= 0 || a.num_warps > 32) throw std::runtime_error("num_warps must be 1..32");
        if (a.shared_memory_bytes < 0 || a.shared_memory_bytes > 232448) {
          throw std::runtime_error("shared_memory_bytes exceeds the sm_100 limit");
        }
        if (abi == 1) {
          a.launch_grid[0] = LegacyGrid(entry.at("grid"));
          a.grid_divisor = AsInt(entry.at("grid").at("divisor"));
        } else {
          const auto& axes = entry.at("grid").list();
          if (axes.empty() || axes.size() > 3) throw std::runtime_error("ABI v2 grid must have one to three axes");
          for (std::size_t i = 0; i < axes.size(); ++i) a.launch_grid[i] = GridNode(axes[i], 0);
          for (const auto& meta : entry.at("tuning").object()) {
            const int value = AsInt(meta.second);
            if (meta.first.empty() || value <= 0) throw std::runtime_error("variant launch metadata is invalid");
            a.launch_meta.emplace(meta.first, value);
          }
        }
        const std::filesystem::path relative(entry.at("binary").str());
        if (relative.is_absolute() || relative.string().find("..") != std::string::npos) {
          throw std::runtime_error("unsafe Kernel Pack binary path");
        }
        a.binary_path = root / relative;
        bool found = false;
        const std::string binary = ReadFile(a.binary_path, &found);
        if (!found) return Status::NotFound("kernel binary not found: " + a.binary_path.string());
        if (Sha256Hex(binary) != a.sha256) {
          return Status::InvalidArgument("kernel binary SHA-256 mismatch: " + a.binary_path.string());
        }
        for (const auto& arg : entry.at("arguments").list()) a.arguments.push_back(ParseArgument(arg));
        std::unordered_set<std::string> names;
        int reserved = 0;
        for (std::size_t i = 0; i < a.arguments.size(); ++i) {
          if (!names.insert(a.arguments[i].name).second) throw std::runtime_error("duplicate kernel argument name");
          if (a.arguments[i].source.kind == KernelArgumentSourceKind::kRuntimeReserved) {
            ++reserved;
            if (i + 2 < a.arguments.size()) {
              throw std::runtime_error("runtime reserved arguments must be at the ABI tail");
            }
          }
        }
        if (reserved != 2) throw std::runtime_error("kernel ABI requires two runtime reserved arguments");
        for (const auto& c : entry.at("constraints").list()) a.constraints.push_back(ParseConstraint(c));
        if (a.kernel_id.empty() || a.variant_id.empty() || a.symbol.empty() ||
            (a.binary_format != "ptx" && a.binary_format != "cubin")) {
          throw std::runtime_error("incomplete kernel artifact entry");
        }
        digest_material += a.sha256;
        loaded.push_back(std::move(a));
      }
    }
  } catch (const std::exception& error) {
    return Status::InvalidArgument(std::string("invalid Kernel Pack: ") + error.what());
  }
  std::unordered_map<std::string, std::vector<KernelArtifact>> by_op;
  for (const auto& a : loaded) by_op[a.op_type].push_back(a);
  for (const auto& entry : by_op) {
    int defaults = 0;
    for (const auto& a : entry.second) defaults += a.is_default ? 1 : 0;
    if (defaults == 0) return Status::InvalidArgument("no default kernel variant for " + entry.first);
  }
  artifacts_ = std::move(loaded);
  by_op_type_ = std::move(by_op);
  repository_hash_ = Sha256Hex(digest_material);
  return Status::OK();
}

const std::vector<KernelArtifact>* ArtifactRepository::Find(const std::string& op_type) const {
  const auto it = by_op_type_.find(op_type);
  return it == by_op_type_.end() ? nullptr : &it->second;
}

std::vector<const KernelArtifact*> KernelCatalog::Query(const std::string& op_type,
                                                        const std::string& dtype,
                                                        const std::string& layout,
                                                        int compute_capability) const {
  std::vector<const KernelArtifact*> matches;
  if (repository_ == nullptr) return matches;
  const auto* list = repository_->Find(op_type);
  if (list == nullptr) return matches;
  for (const auto& a : *list) {
    const bool layout_ok = layout.empty() || a.layout.empty() || a.layout == layout;
    if (a.dtype == dtype && layout_ok && compute_capability >= a.min_compute_capability) {
      matches.push_back(&a);
    }
  }
  return matches;
}

}  // namespace cutriton
