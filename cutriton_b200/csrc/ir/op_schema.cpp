#include "cutriton/ir/op_schema.h"

#include <algorithm>
#include <mutex>

namespace cutriton {

OpSchemaRegistry& OpSchemaRegistry::Global() {
  static OpSchemaRegistry registry;
  return registry;
}

Status OpSchemaRegistry::Register(OpSchema schema) {
  if (schema.op_type.empty() || !schema.infer || schema.min_inputs > schema.max_inputs ||
      schema.outputs == 0) {
    return Status::InvalidArgument("op schema is incomplete");
  }
  std::unique_lock<std::shared_mutex> lock(mutex_);
  const std::string key = schema.op_type;
  if (schemas_.count(key) != 0) return Status::AlreadyExists("op schema already registered: " + key);
  schemas_.emplace(key, std::make_shared<const OpSchema>(std::move(schema)));
  return Status::OK();
}

std::shared_ptr<const OpSchema> OpSchemaRegistry::Find(const std::string& op_type) const {
  std::shared_lock<std::shared_mutex> lock(mutex_);
  const auto it = schemas_.find(op_type);
  return it == schemas_.end() ? nullptr : it->second;
}

std::vector<std::string> OpSchemaRegistry::AvailableOps() const {
  std::shared_lock<std::shared_mutex> lock(mutex_);
  std::vector<std::string> names;
  names.reserve(schemas_.size());
  for (const auto& entry : schemas_) names.push_back(entry.first);
  std::sort(names.begin(), names.end());
  return names;
}

void OpSchemaRegistry::ClearForTests() {
  std::unique_lock<std::shared_mutex> lock(mutex_);
  schemas_.clear();
}

}  // namespace cutriton
