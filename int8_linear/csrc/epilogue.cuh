// Epilogue arithmetic shared by the GEMM kernels: scale/bias loads, the dequantisation
// in the reference kernel's order and the stores of one output value.
#pragma once

#include "common.cuh"

namespace i8l {

__device__ __forceinline__ float load_scalar_f(const void *p, int dtype, long long i) {
  switch (dtype) {
    case I8L_BF16:
      return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    case I8L_F16:
      return __half2float(static_cast<const __half *>(p)[i]);
    default:
      return static_cast<const float *>(p)[i];
  }
}

// The reference's epilogue order: float(acc) * sa, then * sb, then + bias, each
// rounded in fp32 (no contraction into an FMA), then one rounding to the output.
__device__ __forceinline__ float dequant(int acc, float sa, float sb, float bias,
                                         bool has_bias) {
  float v = __int2float_rn(acc);
  v = __fmul_rn(v, sa);
  v = __fmul_rn(v, sb);
  if (has_bias) v = __fadd_rn(v, bias);
  return v;
}

// Two 16-bit outputs (v0 in the low half), each rounded as out_bits16 rounds it.
__device__ __forceinline__ uint32_t pack16x2(int dtype, float v0, float v1) {
  uint32_t p;
  if (dtype == I8L_BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(v1), "f"(v0));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(v1), "f"(v0));
  return p;
}

// Storage bits of one output value.
__device__ __forceinline__ uint32_t out_bits16(int dtype, float v) {
  if (dtype == I8L_BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t *>(&h);
  }
  __half h = __float2half_rn(v);
  return *reinterpret_cast<uint16_t *>(&h);
}

__device__ __forceinline__ uint32_t out_bits32(int dtype, int acc, float v) {
  return dtype == I8L_I32 ? static_cast<uint32_t>(acc) : __float_as_uint(v);
}

__device__ __forceinline__ void store_elem(void *out, int dtype, long long idx,
                                           int acc, float v) {
  switch (dtype) {
    case I8L_BF16:
      static_cast<__nv_bfloat16 *>(out)[idx] = __float2bfloat16_rn(v);
      break;
    case I8L_F16:
      static_cast<__half *>(out)[idx] = __float2half_rn(v);
      break;
    case I8L_F32:
      static_cast<float *>(out)[idx] = v;
      break;
    default:
      static_cast<int *>(out)[idx] = acc;
      break;
  }
}

}  // namespace i8l
