#pragma once

// Typed error reporting for every public call. No exception crosses the API:
// each fallible call returns a Status (same contract as the reference engine's
// include/cutriton/core/status.h:9-74).

#include <string>
#include <utility>

namespace cutriton {

enum class ErrorCode {
  kOk = 0,
  kInvalidArgument,
  kNotFound,
  kAlreadyExists,
  kUnsupported,
  kShapeError,
  kRuntimeError,
  kInternal,
};

class Status {
 public:
  Status() = default;
  Status(ErrorCode code, std::string message)
      : code_(code), message_(std::move(message)) {}

  static Status OK() { return Status(); }
  static Status InvalidArgument(std::string m) { return {ErrorCode::kInvalidArgument, std::move(m)}; }
  static Status NotFound(std::string m) { return {ErrorCode::kNotFound, std::move(m)}; }
  static Status AlreadyExists(std::string m) { return {ErrorCode::kAlreadyExists, std::move(m)}; }
  static Status Unsupported(std::string m) { return {ErrorCode::kUnsupported, std::move(m)}; }
  static Status ShapeError(std::string m) { return {ErrorCode::kShapeError, std::move(m)}; }
  static Status RuntimeError(std::string m) { return {ErrorCode::kRuntimeError, std::move(m)}; }
  static Status Internal(std::string m) { return {ErrorCode::kInternal, std::move(m)}; }

  bool ok() const { return code_ == ErrorCode::kOk; }
  ErrorCode code() const { return code_; }
  const std::string& message() const { return message_; }
  // "<category>: <message>", or "OK".
  std::string ToString() const;

 private:
  ErrorCode code_{ErrorCode::kOk};
  std::string message_;
};

// Stable category name for an error code.
const char* ErrorCodeName(ErrorCode code);

}  // namespace cutriton

// Propagates the first failing Status out of the enclosing function.
#define CUTRITON_RETURN_IF_ERROR(expr)                \
  do {                                                \
    ::cutriton::Status _cutriton_status = (expr);     \
    if (!_cutriton_status.ok()) return _cutriton_status; \
  } while (false)
