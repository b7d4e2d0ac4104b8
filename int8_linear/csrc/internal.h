// Host-side helpers shared by the translation units of the library.
#pragma once

#include <cstdarg>
#include <cstddef>
#include <cstdint>
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

}  // namespace i8l
