// Host-side runtime shared by the entry points: per-device properties, the
// device error word, and the driver's tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace lora {

struct DeviceInfo {
  int num_sms = 0;
  bool is_sm100 = false;
  int* err_word = nullptr;  // device int, first recorded error code (0 = none)
  size_t max_smem_optin = 0;
  int smem_per_sm = 0;  // shared memory of one SM (all resident CTAs together)
};

// Current CUDA device, or -1 if none is usable.
int current_device();

// Properties of `dev`, initialised on first use (allocates the 4-byte error
// word on that device once; never freed).
const DeviceInfo& device_info(int dev);

// cuTensorMapEncodeTiled from the driver (resolved once through the runtime's
// driver entry-point query, so the library does not link libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

int gemm_pick_bn(int64_t M, int64_t N, int num_sms);

// Programmatic dependent launch for the kernels that support it (default on).
// Such a kernel may start while the kernel launched just before it on the
// stream is still running: it reads weights (W, lora_A, lora_B, the adapter
// tables) before griddepcontrol.wait and activations, z, the tile table and
// every global write after it.  LORA_B200_PDL=0 launches every kernel in plain
// stream order (read once per process).
bool pdl_enabled();

}  // namespace lora
