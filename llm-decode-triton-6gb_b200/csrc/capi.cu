// C-ABI plumbing: status strings, last CUDA error text, per-device property cache.
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace b2d {

namespace {
thread_local char g_last_error[256] = {0};
constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
bool g_have[kMaxDevices] = {false};
}  // namespace

void set_cuda_error(cudaError_t e) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
}

void set_error_text(const char* text) { std::snprintf(g_last_error, sizeof(g_last_error), "%s", text); }

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return B2D_OK;
  set_cuda_error(e);
  return B2D_ERR_LAUNCH;
}

int device_info(DeviceInfo* out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    if (e != cudaSuccess) set_cuda_error(e);
    return B2D_ERR_DEVICE;
  }
  if (!g_have[dev]) {
    DeviceInfo d;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, dev) != cudaSuccess) {
      set_cuda_error(cudaGetLastError());
      return B2D_ERR_DEVICE;
    }
    if (d.cc_major != 10) {
      std::snprintf(g_last_error, sizeof(g_last_error), "device %d has compute capability %d.x; built for sm_100a",
                    dev, d.cc_major);
      return B2D_ERR_DEVICE;
    }
    g_info[dev] = d;
    g_have[dev] = true;
  }
  *out = g_info[dev];
  return B2D_OK;
}

}  // namespace b2d

extern "C" const char* b2d_strerror(int status) {
  switch (status) {
    case B2D_OK: return "ok";
    case B2D_ERR_ARG: return "invalid argument (null pointer or negative size)";
    case B2D_ERR_SHAPE: return "unsupported shape";
    case B2D_ERR_DTYPE: return "unsupported dtype";
    case B2D_ERR_ALIGN: return "pointer or leading dimension not aligned for vector loads";
    case B2D_ERR_WORKSPACE: return "workspace missing or too small";
    case B2D_ERR_LAUNCH: return "CUDA launch failed";
    case B2D_ERR_DEVICE: return "no usable sm_100 CUDA device";
    default: return "unknown status";
  }
}

extern "C" const char* b2d_last_cuda_error(void) { return b2d::g_last_error; }

extern "C" int b2d_version(void) { return (1 << 16) | 0; }
