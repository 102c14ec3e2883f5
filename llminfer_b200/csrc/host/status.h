// Error reporting shared by the C ABI: a status code is returned and a
// message is kept per thread for llmi_cuda_last_error().  Errors are values,
// never exceptions (the reference builds with -fno-exceptions and returns
// Error / Result<T>, include/llminfer/Support/Result.h:12-61).
#pragma once

#include "llmi_cuda.h"

#include <cuda_runtime.h>

namespace llmi {

// Records a printf-style message for the calling thread and returns status.
int fail(int status, const char *format, ...) __attribute__((format(printf, 2, 3)));
void clear_error();
const char *last_error();

// LLMI_OK for cudaSuccess, else LLMI_CUDA_ERROR with "<what>: <cuda message>".
int check_cuda(cudaError_t error, const char *what);

// Devices the library serves (current_device rejects higher indices).
constexpr int kMaxDevices = 64;

// Device attributes of the current device, cached per device.
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  size_t max_smem_optin = 0;
};
int current_device(DeviceInfo &info);

}  // namespace llmi
