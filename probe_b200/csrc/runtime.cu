// Host runtime: device cache, error word, status strings, driver entry points.
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "runtime.h"

namespace lora {

namespace {
constexpr int kMaxDevices = 64;
std::once_flag g_dev_once[kMaxDevices];
DeviceInfo g_dev[kMaxDevices];
}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LORA_B200_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return (dev >= 0 && dev < kMaxDevices) ? dev : -1;
}

const DeviceInfo& device_info(int dev) {
  std::call_once(g_dev_once[dev], [dev] {
    DeviceInfo& d = g_dev[dev];
    int major = 0, minor = 0, sms = 0, optin = 0, per_sm = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    d.num_sms = sms;
    d.is_sm100 = (major == 10 && minor == 0);
    d.max_smem_optin = static_cast<size_t>(optin);
    d.smem_per_sm = per_sm;
    int* word = nullptr;
    if (cudaMalloc(&word, sizeof(int)) == cudaSuccess) {
      cudaMemset(word, 0, sizeof(int));
      cudaDeviceSynchronize();
      d.err_word = word;
    } else {
      cudaGetLastError();
    }
  });
  return g_dev[dev];
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

}  // namespace lora

extern "C" int lora_b200_abi_version(void) { return 1; }

extern "C" const char* lora_b200_status_string(int status) {
  switch (status) {
    case LORA_OK: return "ok";
    case LORA_ERR_SHAPE: return "shape";
    case LORA_ERR_ALIGN: return "alignment";
    case LORA_ERR_DTYPE: return "dtype";
    case LORA_ERR_DEVICE: return "device";
    case LORA_ERR_INDEX: return "index out of range";
    case LORA_ERR_CUDA: return "cuda error";
    case LORA_ERR_TIMEOUT: return "device wait timed out";
    case LORA_ERR_WORKSPACE: return "workspace";
    case LORA_ERR_UNSUPPORTED: return "unsupported";
    case LORA_ERR_ARG: return "invalid argument";
    default: return "unknown";
  }
}

extern "C" int lora_b200_device_error(int device, int* code) {
  if (code == nullptr) return LORA_ERR_ARG;
  *code = 0;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return LORA_ERR_DEVICE;
  if (device < 0 || device >= 64) return LORA_ERR_DEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return LORA_ERR_DEVICE;
  const lora::DeviceInfo& info = lora::device_info(device);
  int rc = LORA_OK;
  if (info.err_word == nullptr) {
    rc = LORA_ERR_CUDA;
  } else if (cudaDeviceSynchronize() != cudaSuccess ||
             cudaMemcpy(code, info.err_word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
             cudaMemset(info.err_word, 0, sizeof(int)) != cudaSuccess) {
    rc = LORA_ERR_CUDA;
  }
  cudaSetDevice(prev);
  return rc;
}
