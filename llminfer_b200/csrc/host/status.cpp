#include "status.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

namespace llmi {
namespace {
thread_local std::string g_message;

std::mutex g_info_mutex;
DeviceInfo g_info[kMaxDevices];
}  // namespace

int fail(int status, const char *format, ...) {
  char buffer[512];
  va_list args;
  va_start(args, format);
  std::vsnprintf(buffer, sizeof buffer, format, args);
  va_end(args);
  g_message = buffer;
  return status;
}

void clear_error() { g_message.clear(); }
const char *last_error() { return g_message.c_str(); }

int check_cuda(cudaError_t error, const char *what) {
  if (error == cudaSuccess)
    return LLMI_OK;
  return fail(LLMI_CUDA_ERROR, "%s: %s", what, cudaGetErrorString(error));
}

int current_device(DeviceInfo &info) {
  int device = 0;
  if (int s = check_cuda(cudaGetDevice(&device), "cudaGetDevice"))
    return s;
  if (device < 0 || device >= kMaxDevices)
    return fail(LLMI_UNSUPPORTED, "device index %d out of range", device);
  std::lock_guard<std::mutex> lock(g_info_mutex);
  DeviceInfo &slot = g_info[device];
  if (slot.device != device) {
    int sms = 0, smem = 0;
    if (int s = check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device),
                           "cudaDeviceGetAttribute(SM count)"))
      return s;
    if (int s = check_cuda(
            cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device),
            "cudaDeviceGetAttribute(shared memory)"))
      return s;
    slot.sm_count = sms;
    slot.max_smem_optin = size_t(smem);
    slot.device = device;
  }
  info = slot;
  return LLMI_OK;
}

}  // namespace llmi

extern "C" const char *llmi_cuda_last_error(void) { return llmi::last_error(); }

extern "C" const char *llmi_cuda_status_name(int status) {
  switch (status) {
  case LLMI_OK: return "LLMI_OK";
  case LLMI_INVALID_ARGUMENT: return "LLMI_INVALID_ARGUMENT";
  case LLMI_UNSUPPORTED: return "LLMI_UNSUPPORTED";
  case LLMI_CUDA_ERROR: return "LLMI_CUDA_ERROR";
  case LLMI_DEVICE_TIMEOUT: return "LLMI_DEVICE_TIMEOUT";
  case LLMI_WORKSPACE_TOO_SMALL: return "LLMI_WORKSPACE_TOO_SMALL";
  case LLMI_SESSION_INVALID: return "LLMI_SESSION_INVALID";
  case LLMI_CAPACITY_EXCEEDED: return "LLMI_CAPACITY_EXCEEDED";
  default: return "LLMI_UNKNOWN_STATUS";
  }
}
