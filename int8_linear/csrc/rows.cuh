// Row helpers shared by the per-token quantisers (quant.cu) and the tensor-parallel
// exchange kernels (peer.cu): block reductions, the vectorised row layout, the
// reference's row quantiser and the launch shape of a one-row-per-CTA kernel.
#pragma once

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace i8l {

// Both reductions leave the result in every thread.  `red` holds 32 floats that no
// thread reads or writes between the previous barrier and this call (each reduction of
// a row gets its own array; a loop over rows ends each row with a barrier).
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < nw ? red[l] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < nw ? red[l] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// block_sum / block_max of R rows at once (one barrier each), every row's value through
// exactly the one-row reduction's steps.  `red` holds R x 32 floats, as `red` above.
template <int R, bool kMax>
__device__ __forceinline__ void block_reduce_n(float (&v)[R], float (*red)[32]) {
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, v[r], o);
      v[r] = kMax ? fmaxf(v[r], t) : __fadd_rn(v[r], t);
    }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0)
#pragma unroll
    for (int r = 0; r < R; ++r) red[r][w] = v[r];
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    v[r] = l < nw ? red[r][l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, v[r], o);
      v[r] = kMax ? fmaxf(v[r], t) : __fadd_rn(v[r], t);
    }
  }
}

// Which row elements thread t owns: vector v (0..NV-1) covers columns
// [(v*blockDim + t)*VW, +VW).  VW is 8 (16-byte vectors of 16-bit values) or 1.
template <int VW>
__device__ __forceinline__ int col_of(int v) {
  return (v * blockDim.x + threadIdx.x) * VW;
}

template <int DT, int VW>
__device__ __forceinline__ void load_vec(const void *row, int col, float (&out)[VW]) {
  using T = typename ActType<DT>::T;
  const T *p = static_cast<const T *>(row) + col;
  if constexpr (VW == 8 && sizeof(T) == 2) {
    const uint4 raw = *reinterpret_cast<const uint4 *>(p);
    const T *h = reinterpret_cast<const T *>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = ActType<DT>::to_f32(h[i]);
  } else {
#pragma unroll
    for (int i = 0; i < VW; ++i) out[i] = ActType<DT>::to_f32(p[i]);
  }
}

template <int DT, int VW>
__device__ __forceinline__ void store_vec(void *row, int col, const float (&in)[VW]) {
  using T = typename ActType<DT>::T;
  T *p = static_cast<T *>(row) + col;
  if constexpr (VW == 8 && sizeof(T) == 2) {
    uint4 raw;
    T *h = reinterpret_cast<T *>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = ActType<DT>::from_f32(in[i]);
    *reinterpret_cast<uint4 *>(p) = raw;
  } else {
#pragma unroll
    for (int i = 0; i < VW; ++i) p[i] = ActType<DT>::from_f32(in[i]);
  }
}

__device__ __forceinline__ float load_weight(const void *w, int dtype, int col);

// VW consecutive weight values from column col: one 16-byte load (two for fp32) when
// `vec` (the weight pointer is 16-byte aligned and VW == 8), else scalar loads.
template <int VW>
__device__ __forceinline__ void load_weight_vec(const void *w, int dtype, int col, bool vec,
                                                float (&out)[VW]) {
  if constexpr (VW == 8) {
    if (vec && (dtype == I8L_BF16 || dtype == I8L_F16)) {
      const uint4 raw = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(w) + col);
      if (dtype == I8L_BF16) {
        const __nv_bfloat16 *h = reinterpret_cast<const __nv_bfloat16 *>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = __bfloat162float(h[i]);
      } else {
        const __half *h = reinterpret_cast<const __half *>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = __half2float(h[i]);
      }
      return;
    }
    if (vec && dtype == I8L_F32) {
      const float4 a = *reinterpret_cast<const float4 *>(static_cast<const float *>(w) + col);
      const float4 b = *reinterpret_cast<const float4 *>(static_cast<const float *>(w) + col + 4);
      out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
      out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < VW; ++i) out[i] = load_weight(w, dtype, col + i);
}

__device__ __forceinline__ float load_weight(const void *w, int dtype, int col) {
  switch (dtype) {
    case I8L_BF16:
      return __bfloat162float(static_cast<const __nv_bfloat16 *>(w)[col]);
    case I8L_F16:
      return __half2float(static_cast<const __half *>(w)[col]);
    default:
      return static_cast<const float *>(w)[col];
  }
}

// Rounds an fp32 value to the weight dtype and back (the reference's
// xn.to(w.dtype)); fp32 weights leave it unchanged.
__device__ __forceinline__ float round_to_weight(float v, int dtype) {
  switch (dtype) {
    case I8L_BF16:
      return round_through<I8L_BF16>(v);
    case I8L_F16:
      return round_through<I8L_F16>(v);
    default:
      return v;
  }
}

// q = rint(y * inv) saturated to [-128, 127] for this thread's values in columns < K
// of `qrow` (the quantising half of quantize_row, for an absmax found elsewhere).
template <int NV, int VW>
__device__ __forceinline__ void quantize_vals(const float (&y)[NV][VW], int K, int8_t *qrow, float inv) {
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int col = col_of<VW>(v);
    if (col >= K) continue;
    float p[VW];
    if constexpr (VW % 2 == 0) {
#pragma unroll
      for (int i = 0; i < VW; i += 2) mul2_rn(p[i], p[i + 1], y[v][i], y[v][i + 1], inv, inv);
    } else {
#pragma unroll
      for (int i = 0; i < VW; ++i) p[i] = __fmul_rn(y[v][i], inv);
    }
    if constexpr (VW == 8) {
      // cvt.pack.sat: two int32 saturated to [-128, 127] and packed per instruction
      // (the clamp and the byte packing in one step).
      uint32_t w[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r0 = __float2int_rn(p[4 * h]), r1 = __float2int_rn(p[4 * h + 1]);
        const int r2 = __float2int_rn(p[4 * h + 2]), r3 = __float2int_rn(p[4 * h + 3]);
        uint32_t t;
        asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(t) : "r"(r3), "r"(r2));
        asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w[h]) : "r"(r1), "r"(r0), "r"(t));
      }
      *reinterpret_cast<uint2 *>(qrow + col) = make_uint2(w[0], w[1]);
    } else {
      int8_t q[VW];
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        int r = __float2int_rn(p[i]);
        r = r < -128 ? -128 : (r > 127 ? 127 : r);
        q[i] = static_cast<int8_t>(r);
      }
#pragma unroll
      for (int i = 0; i < VW; ++i) qrow[col + i] = q[i];
    }
  }
}

// The row quantiser of the reference (_quantize_row, fused_quant.py:41-53):
// scale = absmax/127, inv = 127/absmax (0 for a zero row), q = rint(y*inv)
// saturated to [-128, 127].  `y` holds this thread's values (0 where the thread
// owns no column), `valid` marks the real ones.
//
// For rows split across GPUs: with amax_out the row's local absmax is written there and
// nothing is quantised; with amax_in (e.g. the MAX over GPUs) that absmax is used in
// place of the row's own, so every GPU quantises exactly as one GPU would.
template <int NV, int VW>
__device__ __forceinline__ void quantize_row(const float (&y)[NV][VW], int K, int8_t *qrow,
                                             float *scale_out, int precise, float *red,
                                             const float *amax_in = nullptr,
                                             float *amax_out = nullptr) {
  float amax = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int i = 0; i < VW; ++i) amax = fmaxf(amax, fabsf(y[v][i]));
  amax = block_max(amax, red);
  if (amax_out) {
    if (threadIdx.x == 0) *amax_out = amax;
    return;
  }
  if (amax_in) amax = *amax_in;
  if (threadIdx.x == 0) *scale_out = precise ? div_rn(amax, 127.f) : div_full(amax, 127.f);
  const float inv = amax == 0.f ? 0.f : (precise ? div_rn(127.f, amax) : div_full(127.f, amax));
  quantize_vals<NV, VW>(y, K, qrow, inv);
}

// Most threads a one-row CTA may have with NV vectors of VW values per thread (the
// kernels' launch bounds): 1024 for one or two vectors per thread or scalar rows,
// else 256.
constexpr __host__ __device__ int row_max_threads(int nv, int vw) {
  return (vw == 1 || nv <= 2) ? 1024 : 256;
}

// Threads and values per thread for a row of `cols` values: vectors of VW
// values, the fewest vectors per thread that keep the CTA at <= 256 threads
// (the scalar path may grow to 1024 threads of 16 values).
struct RowShape {
  int nv;
  int threads;
};

// `max_threads` above 256 spreads a row thinner (fewer values per thread, shorter
// chains of loads and math per thread), which pays for batches with fewer rows than
// SMs; with many rows per SM, 256 threads with more values each keep more work in
// flight.  Only kernels whose row reduction is a maximum may pick the shape per call
// (row_threads); a sum of squares keeps one shape, so that a row's result does not
// depend on the batch it came in.
inline bool row_shape(int cols, int vw, RowShape *s, int max_threads = 256) {
  const int vecs = (cols + vw - 1) / vw;
  static const int kNv[] = {1, 2, 3, 4, 6, 8, 12, 16};
  for (int nv : kNv) {
    int threads = (vecs + nv - 1) / nv;
    threads = ((threads + 31) / 32) * 32;
    const int base = max_threads == 256 ? (vw == 1 && nv == 16 ? 1024 : 256) : max_threads;
    const int cap = std::min(base, row_max_threads(nv, vw));
    if (max_threads < 256 && nv > 4) break;  // long rows keep the default shapes (registers)
    if (threads <= cap) {
      s->nv = nv;
      s->threads = std::max(32, threads);
      return true;
    }
  }
  // A cap below 256 that no shape of at most 4 vectors meets falls back to the defaults.
  return max_threads < 256 && row_shape(cols, vw, s, 256);
}

// Row-shape thread cap for a max-reduction row kernel over a batch of M rows: up to
// 1024 threads while there are fewer rows than SMs, 256 beyond, and 128 from 8 rows per
// SM (more vectors in flight per thread and twice the resident rows; measured on the
// plain quantiser at M=4096, K=2048: 256 threads per row left it latency-bound at 38 %
// of HBM).
inline int row_threads(int M) {
  DeviceInfo di;
  const int sms = device_info(&di) == I8L_OK ? di.sms : 148;
  return M < sms ? 1024 : (M < 8 * sms ? 256 : 128);
}

inline bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

#define I8L_DISPATCH_NV(NVVAL, ...)                                                \
  switch (NVVAL) {                                                                 \
    case 1: { constexpr int NV = 1; __VA_ARGS__; } break;                          \
    case 2: { constexpr int NV = 2; __VA_ARGS__; } break;                          \
    case 3: { constexpr int NV = 3; __VA_ARGS__; } break;                          \
    case 4: { constexpr int NV = 4; __VA_ARGS__; } break;                          \
    case 6: { constexpr int NV = 6; __VA_ARGS__; } break;                          \
    case 8: { constexpr int NV = 8; __VA_ARGS__; } break;                          \
    case 12: { constexpr int NV = 12; __VA_ARGS__; } break;                        \
    default: { constexpr int NV = 16; __VA_ARGS__; } break;                        \
  }

}  // namespace i8l
