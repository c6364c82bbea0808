// Status codes shared by the host runtime and the device kernels.
//
// Parity: include/hcp_ringattn/core/status.h:7-45 of the reference (Status with kOk /
// kInvalidArgument / kUnimplemented / kInternal). Extended with the device-side failure codes
// that a bounded wait or a bounds check writes into the runtime's status word instead of
// trapping, so that a broken peer or a bad argument never hangs or faults a shared GPU.
#pragma once

#include <cstdint>
#include <string>

namespace hcp {

enum class StatusCode : int32_t {
  kOk = 0,
  kInvalidArgument = 1,
  kUnimplemented = 2,
  kInternal = 3,
  // device-reported
  kMbarTimeout = 16,      // an intra-CTA pipeline wait ran out of its time budget
  kPeerTimeout = 17,      // a wait on another rank's flag ran out of its time budget
  kOutOfBounds = 18,      // a device bounds check rejected an index (access skipped)
  kCudaError = 19,
};

// Layout of the int32 device status word array every kernel receives.
//   [0] code (first error wins, atomicCAS from 0)
//   [1] site id (kernel-specific), [2] info a, [3] info b
constexpr int kStatusWords = 8;

class Status {
 public:
  Status() = default;
  Status(StatusCode code, std::string msg) : code_(code), msg_(std::move(msg)) {}
  static Status Ok() { return Status(); }
  static Status InvalidArgument(std::string m) { return {StatusCode::kInvalidArgument, std::move(m)}; }
  static Status Unimplemented(std::string m) { return {StatusCode::kUnimplemented, std::move(m)}; }
  static Status Internal(std::string m) { return {StatusCode::kInternal, std::move(m)}; }
  bool ok() const { return code_ == StatusCode::kOk; }
  StatusCode code() const { return code_; }
  const std::string& message() const { return msg_; }
  std::string ToString() const {
    return ok() ? std::string("OK") : ("code=" + std::to_string(int(code_)) + ": " + msg_);
  }

 private:
  StatusCode code_ = StatusCode::kOk;
  std::string msg_;
};

}  // namespace hcp
