// Shared C-ABI plumbing: per-thread error messages, the cached device query and
// the device status word that kernels with bounded waits write to.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace i8l {

// Status word: kernels atomicOr a bit here when one of their bounded waits ran
// out.  Host code reaches it through status_ptr(), which resolves the symbol's
// device address once per device.
__device__ int g_status;

static thread_local char t_err[512] = "no error";
static std::atomic<int> g_pdl{0};

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_error(cudaError_t e, const char *what) {
  return set_error(I8L_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceInfo g_info[kMaxDevices];
bool g_have[kMaxDevices];
int *g_status_addr[kMaxDevices];
}  // namespace

int device_info(DeviceInfo *out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(I8L_EINVAL, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_have[dev]) {
    DeviceInfo d{};
    d.device = dev;
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
            cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return cuda_error(e, "cudaDeviceGetAttribute");
    if (d.cc_major != 10 || d.cc_minor != 0)
      return set_error(I8L_ENOTSUP, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev,
                       d.cc_major, d.cc_minor);
    g_info[dev] = d;
    g_have[dev] = true;
  }
  *out = g_info[dev];
  return I8L_OK;
}

int *status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_status_addr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
    g_status_addr[dev] = static_cast<int *>(p);
  }
  return g_status_addr[dev];
}

}  // namespace i8l

using namespace i8l;

extern "C" const char *i8l_last_error(void) { return t_err; }

extern "C" int i8l_read_status(int32_t *status_out) {
  if (!status_out) return set_error(I8L_EINVAL, "status_out is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_error(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_status, sizeof(int));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyFromSymbol(status)");
  *status_out = v;
  return I8L_OK;
}

extern "C" int i8l_clear_status(void) {
  const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyToSymbol(status)");
  return I8L_OK;
}

extern "C" const char *i8l_version(void) { return "0.1.0 sm_100a"; }

extern "C" int i8l_set_pdl(int32_t enable) {
  g_pdl.store(enable ? 1 : 0, std::memory_order_relaxed);
  return I8L_OK;
}

extern "C" int32_t i8l_get_pdl(void) { return g_pdl.load(std::memory_order_relaxed); }
