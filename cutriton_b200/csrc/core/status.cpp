#include "cutriton/core/status.h"

namespace cutriton {

const char* ErrorCodeName(ErrorCode code) {
  switch (code) {
    case ErrorCode::kOk: return "OK";
    case ErrorCode::kInvalidArgument: return "InvalidArgument";
    case ErrorCode::kNotFound: return "NotFound";
    case ErrorCode::kAlreadyExists: return "AlreadyExists";
    case ErrorCode::kUnsupported: return "Unsupported";
    case ErrorCode::kShapeError: return "ShapeError";
    case ErrorCode::kRuntimeError: return "RuntimeError";
    case ErrorCode::kInternal: return "Internal";
  }
  return "Unknown";
}

std::string Status::ToString() const {
  return ok() ? std::string("OK") : std::string(ErrorCodeName(code_)) + ": " + message_;
}

}  // namespace cutriton
