// abi.cu -- library-wide C ABI entry points (version, status strings, last
// CUDA error) and the host helpers shared by the kernels' launchers.
#include <mutex>
#include <vector>

#include "common.cuh"

namespace pa {

static thread_local int t_last_cuda_error = 0;

void set_last_cuda_error(cudaError_t e) { t_last_cuda_error = (int)e; }

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return PA_OK;
  set_last_cuda_error(e);
  return PA_ERR_CUDA;
}

// SM count of the current device, cached per device.  Also rejects devices
// that are not sm_100 (the kernels are built for sm_100a only).
int device_sm_count(int* sms) {
  static std::mutex mu;
  static std::vector<std::pair<int, int>> cache;  // (device, sms or -1)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return PA_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lk(mu);
  for (auto& c : cache)
    if (c.first == dev) {
      if (c.second < 0) return PA_ERR_NO_DEVICE;
      *sms = c.second;
      return PA_OK;
    }
  int n = 0, major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    cache.push_back({dev, -1});
    return PA_ERR_NO_DEVICE;
  }
  const bool ok = (major == 10 && minor == 0);
  cache.push_back({dev, ok ? n : -1});
  if (!ok) return PA_ERR_NO_DEVICE;
  *sms = n;
  return PA_OK;
}

}  // namespace pa

extern "C" int pa_abi_version(void) { return PA_B200_ABI_VERSION; }

extern "C" int pa_last_cuda_error(void) { return pa::t_last_cuda_error; }

extern "C" const char* pa_strerror(int status) {
  switch (status) {
    case PA_OK: return "ok";
    case PA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PA_ERR_NUM_HEADS: return "n_head must be divisible by n_kv_head";
    case PA_ERR_HEAD_DIM: return "unsupported head_dim";
    case PA_ERR_DTYPE: return "unsupported KV cache dtype";
    case PA_ERR_BLOCK_SIZE: return "unsupported block_size";
    case PA_ERR_ALIGNMENT: return "pointer is not 16-byte aligned";
    case PA_ERR_WORKSPACE: return "workspace missing or too small";
    case PA_ERR_CUDA: return "CUDA error";
    case PA_ERR_TOO_LARGE: return "size exceeds a supported limit";
    case PA_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
    default: return "unknown status";
  }
}
