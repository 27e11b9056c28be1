// Host-side status helpers shared by the C ABI translation units.
#pragma once

#include <cuda_runtime.h>

#include <string>

namespace vx {

// Status codes of the C ABI (include/voxcpm_b200.h).
enum Status : int {
  kOk = 0,
  kUnsupported = 1,   // shape or layout the kernels do not serve; nothing launched
  kInvalid = 2,       // bad argument (null pointer, misalignment, size)
  kCudaError = 3,     // a CUDA runtime call failed
  kDeviceTimeout = 4, // a bounded device wait gave up (see vx_device_error)
};


/// Records `message` as the calling thread's last error; returns `status`.
int Fail(int status, const std::string& message);
/// kOk, or kCudaError with the CUDA error text.
int FromCuda(cudaError_t error, const char* what);
/// Adds a message for a non-kOk status of an internal launcher.
int Checked(int status, const char* what);
const char* LastError();

}  // namespace vx
