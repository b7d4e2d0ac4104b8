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

// The CUDA-core GEMM for decode batches of <= 8 tokens (split mode 5, gemv_sm100.cu).
struct GemvPlan {
  int mt;          // tokens the kernel variant holds (1, 2, 4, 8)
  int ctas;        // CTAs, each owning a contiguous range of output columns
  int max_rows;    // most columns one CTA owns
  int stage_rows;  // weight rows per shared-memory stage
  int stages;      // ring depth
  size_t smem;     // dynamic shared memory per CTA
};
// The activation prologue of a CUDA-core GEMM: the kernel quantises its own bf16/fp16
// input (mode 1 per-token, 2 add + RMSNorm, 3 SiLU-and-mul) instead of reading int8.
struct GemvPro {
  int mode;
  const void *x;
  int64_t ldx;  // elements
  int x_dtype;
  const void *res;  // mode 2: residual or NULL
  int64_t ldr;
  void *rout;       // mode 2: residual output (with res)
  int64_t ldro;
  const void *nw;   // mode 2: norm weight [K]
  int nw_dtype;
  float eps;
  int precise, round_silu;
};
int gemv_plan(int M, int N, int K, const i8l_tile *tile, GemvPlan *p);
int gemv_run(const int8_t *A, int64_t lda, const int8_t *W, int64_t ldw, const float *sa,
             int32_t sa_per_row, const float *sb, int32_t sb_per_col, const void *bias,
             int32_t bias_dtype, void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N,
             int32_t K, const i8l_tile *tile, void *stream, const GemvPro *pro = nullptr);

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
