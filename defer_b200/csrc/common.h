// Shared host-side definitions: status codes (mirroring the reference's
// DeferError, src/error.rs:5-14), the thread-local error message, and CUDA
// error plumbing.
#pragma once
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace defer {

// Status codes of the C ABI. 1-7 mirror DeferError (error.rs:5-14).
enum Status : int {
  kOk = 0,
  kIo = 1,
  kParse = 2,
  kModel = 3,
  kCheckpoint = 4,
  kWal = 5,
  kTokenizer = 6,
  kDivergence = 7,
  kCuda = 8,
  kDeviceTimeout = 9,
  kInvalidArgument = 10,
};

struct Error : std::runtime_error {
  Status status;
  Error(Status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void fail(Status s, const std::string& m) { throw Error(s, m); }

void set_last_error(const std::string& m);
const char* last_error();

}  // namespace defer

#define DEFER_CUDA(call)                                                                               \
  do {                                                                                                 \
    cudaError_t e_ = (call);                                                                           \
    if (e_ != cudaSuccess)                                                                             \
      ::defer::fail(::defer::kCuda, std::string(#call) + ": " + cudaGetErrorString(e_));               \
  } while (0)
