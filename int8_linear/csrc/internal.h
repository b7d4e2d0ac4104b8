// Host-side helpers shared by the translation units of the library.
#pragma once

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <utility>
#include <cuda_runtime.h>

#include "../../include/int8_linear_b200.h"

namespace i8l {

// Records a one-line message for i8l_last_error() and returns `code`.
int set_error(int code, const char *fmt, ...);

// Maps a CUDA runtime error to I8L_ECUDA with its name and the failing step.
int cuda_error(cudaError_t e, const char *what);

// SM count and opt-in shared memory of the current device (cached per device).
struct DeviceInfo {
  int device;
  int sms;
  int max_smem_optin;
  int cc_major, cc_minor;
};
int device_info(DeviceInfo *out);

// Device pointer of the status word kernels set when a bounded wait gives up.
int *status_ptr();

// Whether kernels are launched with programmatic stream serialisation (PDL).
bool pdl_enabled();

// Launches `kernel` with the PDL attribute when pdl_enabled(), in thread-block
// clusters of `cluster` CTAs along x when cluster > 1.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, int cluster, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace i8l
