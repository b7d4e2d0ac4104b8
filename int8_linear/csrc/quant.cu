// Per-token int8 quantisers fused into the op before them, for sm_100a:
//   add + RMSNorm + quantise   (reference: int8_linear/fused_quant.py:56-73)
//   SiLU-and-mul + quantise    (reference: int8_linear/fused_quant.py:76-88)
//   plain per-token quantise   (the step the reference leaves to vLLM's
//                               scaled_int8_quant; arithmetic of the reference's
//                               torch `quant`, tests/test_fused_quant.py:26-31)
// One CTA per token row.  Each thread holds its slice of the row in registers
// (16-byte vector loads when the row allows, else scalar loads), so the row is
// read from HBM once; the sum of squares and the absolute maximum are reduced with
// warp shuffles and one shared-memory exchange.
//
// Arithmetic follows the reference kernels step by step (fused_quant.py:41-88):
// fp32 math, rounding through the activation/weight dtypes where the reference
// rounds, CUDA's rsqrtf/expf where the reference calls libdevice rsqrt/exp,
// Triton's approximate `/` (div.full.f32) where the reference uses a plain
// divide, IEEE division for the quantiser when precise_div is set, and
// round-half-to-even with saturation to [-128, 127].
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "rows.cuh"

namespace i8l {

// Batches from which add_rmsnorm_quant runs several rows per CTA (measured on B200 at
// K=2048, µs per call: M=2048 6.47 with one row per CTA against 6.88 with two; M=4096
// 11.4-11.7 with two or four rows against 11.6-12.1 with one; eight rows per CTA took
// twice as long).
constexpr int kNormTwoRowsMin = 4096;
constexpr int kNormFourRowsMin = 4096;

struct NormArgs {
  const void *x;
  long long ldx;
  const void *res;
  long long ldr;
  const void *w;
  int w_dtype;
  int8_t *q;
  long long ldq;
  float *scale;
  void *rout;
  long long ldro;
  int K;
  float eps;
  int precise;
  int w_vec;  // the weight pointer allows 16-byte loads
};

// WDT: the weight dtype fixed at compile time (vector rows), or -1 to read it from the
// arguments (scalar rows).
template <int DT, int NV, int VW, int WDT>
__global__ void __launch_bounds__(row_max_threads(NV, VW)) add_rmsnorm_quant_kernel(const NormArgs a) {
  const int wdt = WDT >= 0 ? WDT : a.w_dtype;
  // Let the next kernel in the stream start its prologue now (in a decode chain, the
  // next GEMM prefetches its weights while this row is normalised).
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32], red2[32];
  using T = typename ActType<DT>::T;
  const long long row = blockIdx.x;
  const T *xrow = static_cast<const T *>(a.x) + row * a.ldx;
  float x[NV][VW], wv[NV][VW];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int col = col_of<VW>(v);
    if (col < a.K) {
      load_vec<DT, VW>(xrow, col, x[v]);
      load_weight_vec<VW>(a.w, wdt, col, a.w_vec != 0, wv[v]);
      if (a.res) {
        float r[VW];
        load_vec<DT, VW>(static_cast<const T *>(a.res) + row * a.ldr, col, r);
        if constexpr (VW % 2 == 0) {
#pragma unroll
          for (int i = 0; i < VW; i += 2)
            add2_rn(x[v][i], x[v][i + 1], x[v][i], x[v][i + 1], r[i], r[i + 1]);
        } else {
#pragma unroll
          for (int i = 0; i < VW; ++i) x[v][i] = __fadd_rn(x[v][i], r[i]);
        }
        store_vec<DT, VW>(static_cast<T *>(a.rout) + row * a.ldro, col, x[v]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < VW; ++i) x[v][i] = 0.f;
    }
  }
  // Squares two at a time; their sum stays in column order (the bits depend on it).
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float sq[VW];
    if constexpr (VW % 2 == 0) {
#pragma unroll
      for (int i = 0; i < VW; i += 2) mul2_rn(sq[i], sq[i + 1], x[v][i], x[v][i + 1], x[v][i], x[v][i + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < VW; ++i) sq[i] = __fmul_rn(x[v][i], x[v][i]);
    }
#pragma unroll
    for (int i = 0; i < VW; ++i) ss = __fadd_rn(ss, sq[i]);
  }
  ss = block_sum(ss, red);
  // var = sum(x^2) / K with Triton's plain `/`, then xn = x * rsqrt(var + eps).
  const float var = div_full(ss, static_cast<float>(a.K));
  const float rs = rsqrtf(__fadd_rn(var, a.eps));
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int col = col_of<VW>(v);
    if (col >= a.K) continue;
    if constexpr (VW % 2 == 0 && WDT >= 0) {
      // y = round(round_w(x * rs) * w), two columns per instruction
#pragma unroll
      for (int i = 0; i < VW; i += 2) {
        float n0, n1;
        mul2_rn(n0, n1, x[v][i], x[v][i + 1], rs, rs);
        round2_through<WDT>(n0, n1);
        mul2_rn(x[v][i], x[v][i + 1], n0, n1, wv[v][i], wv[v][i + 1]);
        round2_through<DT>(x[v][i], x[v][i + 1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        const float xn = round_to_weight(__fmul_rn(x[v][i], rs), wdt);
        x[v][i] = round_through<DT>(__fmul_rn(xn, wv[v][i]));
      }
    }
  }
  quantize_row<NV, VW>(x, a.K, a.q + row * a.ldq, a.scale + row, a.precise, red2);
}

// add_rmsnorm_quant_kernel for R rows per CTA (large batches, 16-byte vectors): every
// thread owns the same columns in each row as the one-row kernel gives it, and each
// row's sums, maxima and roundings take exactly that kernel's steps, so the bits are the
// same.  Every load (weights, then x and residual of every row) is issued before any
// arithmetic or store, so all of them are in flight together (a residual store between
// two rows' loads would hold the second row's loads back, as the compiler cannot tell
// the store from the loads).  The last CTA may have fewer rows.
template <int DT, int NV, int WDT, int R>
__global__ void __launch_bounds__(256) add_rmsnorm_quant_rows_kernel(const NormArgs a, int M) {
  constexpr int VW = 8;
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[R][32], red2[R][32];
  using T = typename ActType<DT>::T;
  const long long row0 = static_cast<long long>(R) * blockIdx.x;
  const int nrows = static_cast<int>(min(static_cast<long long>(R), M - row0));
  float wv[NV][VW];
  uint4 xr[R][NV], rr[R][NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int col = col_of<VW>(v);
#pragma unroll
    for (int r = 0; r < R; ++r) xr[r][v] = rr[r][v] = make_uint4(0u, 0u, 0u, 0u);
    if (col >= a.K) continue;
    load_weight_vec<VW>(a.w, WDT, col, a.w_vec != 0, wv[v]);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r >= nrows) break;
      const long long row = row0 + r;
      xr[r][v] = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.x) + row * a.ldx + col);
      if (a.res) rr[r][v] = *reinterpret_cast<const uint4 *>(static_cast<const T *>(a.res) + row * a.ldr + col);
    }
  }
  float x[R][NV][VW];
  float ss[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    ss[r] = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const T *h = reinterpret_cast<const T *>(&xr[r][v]);
#pragma unroll
      for (int i = 0; i < VW; ++i) x[r][v][i] = ActType<DT>::to_f32(h[i]);
      const int col = col_of<VW>(v);
      if (a.res && r < nrows && col < a.K) {
        const T *g = reinterpret_cast<const T *>(&rr[r][v]);
        float rv[VW];
#pragma unroll
        for (int i = 0; i < VW; ++i) rv[i] = ActType<DT>::to_f32(g[i]);
#pragma unroll
        for (int i = 0; i < VW; i += 2)
          add2_rn(x[r][v][i], x[r][v][i + 1], x[r][v][i], x[r][v][i + 1], rv[i], rv[i + 1]);
        store_vec<DT, VW>(static_cast<T *>(a.rout) + (row0 + r) * a.ldro, col, x[r][v]);
      }
      float sq[VW];
#pragma unroll
      for (int i = 0; i < VW; i += 2)
        mul2_rn(sq[i], sq[i + 1], x[r][v][i], x[r][v][i + 1], x[r][v][i], x[r][v][i + 1]);
#pragma unroll
      for (int i = 0; i < VW; ++i) ss[r] = __fadd_rn(ss[r], sq[i]);
    }
  }
  block_reduce_n<R, false>(ss, red);
  float amax[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    amax[r] = 0.f;
    const float var = div_full(ss[r], static_cast<float>(a.K));
    const float rs = rsqrtf(__fadd_rn(var, a.eps));
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      if (col_of<VW>(v) >= a.K) continue;
#pragma unroll
      for (int i = 0; i < VW; i += 2) {
        float n0, n1;
        mul2_rn(n0, n1, x[r][v][i], x[r][v][i + 1], rs, rs);
        round2_through<WDT>(n0, n1);
        mul2_rn(x[r][v][i], x[r][v][i + 1], n0, n1, wv[v][i], wv[v][i + 1]);
        round2_through<DT>(x[r][v][i], x[r][v][i + 1]);
      }
#pragma unroll
      for (int i = 0; i < VW; ++i) amax[r] = fmaxf(amax[r], fabsf(x[r][v][i]));
    }
  }
  block_reduce_n<R, true>(amax, red2);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r >= nrows) break;
    const long long row = row0 + r;
    if (threadIdx.x == 0)
      a.scale[row] = a.precise ? div_rn(amax[r], 127.f) : div_full(amax[r], 127.f);
    const float inv = amax[r] == 0.f ? 0.f : (a.precise ? div_rn(127.f, amax[r]) : div_full(127.f, amax[r]));
    quantize_vals<NV, VW>(x[r], a.K, a.q + row * a.ldq, inv);
  }
}

struct SiluArgs {
  const float *amax_in;  // per row, or NULL
  float *amax_out;       // per row, or NULL
  const void *gu;
  long long ld;
  int8_t *q;
  long long ldq;
  float *scale;
  int I;
  int precise;
  int round_silu;
};

template <int DT, int NV, int VW>
__global__ void __launch_bounds__(row_max_threads(NV, VW)) silu_mul_quant_kernel(const SiluArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  using T = typename ActType<DT>::T;
  const long long row = blockIdx.x;
  const T *grow = static_cast<const T *>(a.gu) + row * a.ld;
  const T *urow = grow + a.I;
  float y[NV][VW];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int col = col_of<VW>(v);
    if (col < a.I) {
      float g[VW], u[VW];
      load_vec<DT, VW>(grow, col, g);
      load_vec<DT, VW>(urow, col, u);
      if constexpr (VW % 2 == 0) {
        // silu(g) = g / (1 + exp(-g)) with Triton's plain `/`; the sums, products and
        // roundings two columns per instruction.
#pragma unroll
        for (int i = 0; i < VW; i += 2) {
          float d0, d1, s0, s1;
          add2_rn(d0, d1, 1.0f, 1.0f, expf(-g[i]), expf(-g[i + 1]));
          s0 = div_full(g[i], d0);
          s1 = div_full(g[i + 1], d1);
          if (a.round_silu) round2_through<DT>(s0, s1);
          mul2_rn(y[v][i], y[v][i + 1], s0, s1, u[i], u[i + 1]);
          round2_through<DT>(y[v][i], y[v][i + 1]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < VW; ++i) {
          // silu(g) = g / (1 + exp(-g)) with Triton's plain `/`.
          float s = div_full(g[i], __fadd_rn(1.0f, expf(-g[i])));
          if (a.round_silu) s = round_through<DT>(s);
          y[v][i] = round_through<DT>(__fmul_rn(s, u[i]));
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < VW; ++i) y[v][i] = 0.f;
    }
  }
  quantize_row<NV, VW>(y, a.I, a.q + row * a.ldq, a.scale + row, a.precise, red,
                       a.amax_in ? a.amax_in + row : nullptr, a.amax_out ? a.amax_out + row : nullptr);
}

struct QuantArgs {
  const float *amax_in;  // per row, or NULL
  float *amax_out;       // per row, or NULL
  const void *x;
  long long ldx;
  int8_t *q;
  long long ldq;
  float *scale;
  int K;
  int precise;
};

template <int DT, int NV, int VW>
__global__ void __launch_bounds__(row_max_threads(NV, VW)) quant_rows_kernel(const QuantArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  using T = typename ActType<DT>::T;
  const long long row = blockIdx.x;
  const T *xrow = static_cast<const T *>(a.x) + row * a.ldx;
  float y[NV][VW];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int col = col_of<VW>(v);
    if (col < a.K) {
      load_vec<DT, VW>(xrow, col, y[v]);
    } else {
#pragma unroll
      for (int i = 0; i < VW; ++i) y[v][i] = 0.f;
    }
  }
  quantize_row<NV, VW>(y, a.K, a.q + row * a.ldq, a.scale + row, a.precise, red,
                       a.amax_in ? a.amax_in + row : nullptr, a.amax_out ? a.amax_out + row : nullptr);
}

// Dequantisation of an int32 product computed elsewhere (e.g. summed over the GPUs of
// a row-parallel layer): out = cast(((float(acc) * sa[m]) * sb[n]) + bias[n]), the same
// fp32 steps as the GEMM epilogue, so the result matches a one-GPU GEMM bit for bit.
struct DequantArgs {
  const int *acc;
  long long lda;
  const float *sa;
  int sa_per_row;
  const float *sb;
  int sb_per_col;
  const void *bias;
  int bias_dtype;
  void *out;
  int out_dtype;
  long long ldo;
  int M, N;
};

__global__ void __launch_bounds__(256) dequant_i32_kernel(const DequantArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const long long total = static_cast<long long>(a.M) * a.N;
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
    const int m = static_cast<int>(i / a.N), n = static_cast<int>(i - static_cast<long long>(m) * a.N);
    float v = __int2float_rn(a.acc[m * a.lda + n]);
    v = __fmul_rn(v, a.sa_per_row ? a.sa[m] : a.sa[0]);
    v = __fmul_rn(v, a.sb_per_col ? a.sb[n] : a.sb[0]);
    if (a.bias) {
      float b;
      if (a.bias_dtype == I8L_BF16)
        b = __bfloat162float(static_cast<const __nv_bfloat16 *>(a.bias)[n]);
      else if (a.bias_dtype == I8L_F16)
        b = __half2float(static_cast<const __half *>(a.bias)[n]);
      else
        b = static_cast<const float *>(a.bias)[n];
      v = __fadd_rn(v, b);
    }
    const long long o = m * a.ldo + n;
    if (a.out_dtype == I8L_BF16)
      static_cast<__nv_bfloat16 *>(a.out)[o] = __float2bfloat16_rn(v);
    else if (a.out_dtype == I8L_F16)
      static_cast<__half *>(a.out)[o] = __float2half_rn(v);
    else
      static_cast<float *>(a.out)[o] = v;
  }
}

// The same arithmetic, 8 consecutive outputs per thread: two 16-byte int32 loads and one
// 16-byte store of 16-bit outputs (two of fp32), one row/column computation per 8 values.
// Rows must hold a multiple of 8 values with 16-byte aligned starts.
__global__ void __launch_bounds__(256) dequant_i32_vec8_kernel(const DequantArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int per_row = a.N / 8;
  const long long total = static_cast<long long>(a.M) * per_row;
  for (long long gi = blockIdx.x * 256LL + threadIdx.x; gi < total; gi += 256LL * gridDim.x) {
    const int m = static_cast<int>(gi / per_row);
    const int n0 = static_cast<int>(gi - static_cast<long long>(m) * per_row) * 8;
    const int4 *src = reinterpret_cast<const int4 *>(a.acc + m * a.lda + n0);
    const int4 p0 = src[0], p1 = src[1];
    const int acc[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    const float sa = a.sa_per_row ? a.sa[m] : a.sa[0];
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + j;
      v[j] = __fmul_rn(__fmul_rn(__int2float_rn(acc[j]), sa), a.sb_per_col ? a.sb[n] : a.sb[0]);
      if (a.bias) {
        float b;
        if (a.bias_dtype == I8L_BF16)
          b = __bfloat162float(static_cast<const __nv_bfloat16 *>(a.bias)[n]);
        else if (a.bias_dtype == I8L_F16)
          b = __half2float(static_cast<const __half *>(a.bias)[n]);
        else
          b = static_cast<const float *>(a.bias)[n];
        v[j] = __fadd_rn(v[j], b);
      }
    }
    const long long o = m * a.ldo + n0;
    if (a.out_dtype == I8L_F32) {
      float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(a.out) + o);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t lo, hi;
        if (a.out_dtype == I8L_BF16) {
          lo = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * j]));
          hi = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * j + 1]));
        } else {
          lo = __half_as_ushort(__float2half_rn(v[2 * j]));
          hi = __half_as_ushort(__float2half_rn(v[2 * j + 1]));
        }
        w[j] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.out) + o) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// ------------------------------------------------------------------ launch

}  // namespace i8l

using namespace i8l;

namespace {

int check_act(int act) {
  if (act != I8L_BF16 && act != I8L_F16)
    return set_error(I8L_ENOTSUP, "activation dtype code %d not supported (bf16 or fp16)", act);
  return I8L_OK;
}

int finish_launch(cudaError_t err, const char *what) {
  if (err != cudaSuccess) return cuda_error(err, what);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  return I8L_OK;
}

}  // namespace

extern "C" int i8l_add_rmsnorm_quant(const void *x, int64_t ldx, const void *residual,
                                     int64_t ldr, const void *weight, int32_t act_dtype,
                                     int32_t w_dtype, int8_t *q, int64_t ldq, float *scale,
                                     void *rout, int64_t ldro, int32_t M, int32_t K, float eps,
                                     int32_t precise_div, void *stream) {
  int e = check_act(act_dtype);
  if (e) return e;
  if (w_dtype < I8L_BF16 || w_dtype > I8L_F32)
    return set_error(I8L_ENOTSUP, "weight dtype code %d not supported", w_dtype);
  if (M < 0 || K <= 0) return set_error(I8L_EINVAL, "bad size M=%d K=%d", M, K);
  if (M == 0) return I8L_OK;
  if (!x || !weight || !q || !scale) return set_error(I8L_EINVAL, "NULL pointer argument");
  if ((residual == nullptr) != (rout == nullptr))
    return set_error(I8L_EINVAL, "residual and residual_out must be given together");
  if (ldx < K || ldq < K || (residual && (ldr < K || ldro < K)))
    return set_error(I8L_EINVAL, "row stride smaller than K");
  NormArgs a{x, ldx, residual, ldr, weight, w_dtype, q, ldq, scale, rout, ldro, K, eps, precise_div,
             aligned16(weight) ? 1 : 0};
  const bool vec = K % 8 == 0 && ldx % 8 == 0 && ldq % 8 == 0 && aligned16(x) && aligned16(q) &&
                   (!residual || (ldr % 8 == 0 && ldro % 8 == 0 && aligned16(residual) &&
                                  aligned16(rout)));
  RowShape rs;
  if (!row_shape(K, vec ? 8 : 1, &rs)) return set_error(I8L_ENOTSUP, "row of %d values is too long", K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nv = rs.nv, th = rs.threads;
  cudaError_t err = cudaSuccess;
  // Several rows per CTA for large batches of short rows (same bits, see the kernel):
  // 2 from kNormTwoRowsMin rows, 4 from kNormFourRowsMin when a row is one vector per thread.
  const bool two_rows = vec && nv <= 4 && th <= 256 && M >= kNormTwoRowsMin;
  const bool four_rows = two_rows && nv == 1 && M >= kNormFourRowsMin;
#define I8L_NORM_VEC(ADT, WDTV)                                                                     \
  if (four_rows) {                                                                                  \
    err = launch(add_rmsnorm_quant_rows_kernel<ADT, 1, WDTV, 4>, dim3((M + 3) / 4), dim3(th), 0, s, 1, a, M); \
  } else if (two_rows) {                                                                            \
    switch (nv) {                                                                                   \
      case 1: err = launch(add_rmsnorm_quant_rows_kernel<ADT, 1, WDTV, 2>, dim3((M + 1) / 2), dim3(th), 0, s, 1, a, M); break; \
      case 2: err = launch(add_rmsnorm_quant_rows_kernel<ADT, 2, WDTV, 2>, dim3((M + 1) / 2), dim3(th), 0, s, 1, a, M); break; \
      case 3: err = launch(add_rmsnorm_quant_rows_kernel<ADT, 3, WDTV, 2>, dim3((M + 1) / 2), dim3(th), 0, s, 1, a, M); break; \
      default: err = launch(add_rmsnorm_quant_rows_kernel<ADT, 4, WDTV, 2>, dim3((M + 1) / 2), dim3(th), 0, s, 1, a, M); break; \
    }                                                                                               \
  } else {                                                                                          \
    I8L_DISPATCH_NV(nv, (err = launch(add_rmsnorm_quant_kernel<ADT, NV, 8, WDTV>, dim3(M), dim3(th), 0, s, 1, a))) \
  }
  if (act_dtype == I8L_BF16) {
    if (vec) {
      if (w_dtype == I8L_BF16) { I8L_NORM_VEC(I8L_BF16, I8L_BF16) }
      else if (w_dtype == I8L_F16) { I8L_NORM_VEC(I8L_BF16, I8L_F16) }
      else { I8L_NORM_VEC(I8L_BF16, I8L_F32) }
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(add_rmsnorm_quant_kernel<I8L_BF16, NV, 1, -1>, dim3(M), dim3(th), 0, s, 1, a)))
    }
  } else {
    if (vec) {
      if (w_dtype == I8L_BF16) { I8L_NORM_VEC(I8L_F16, I8L_BF16) }
      else if (w_dtype == I8L_F16) { I8L_NORM_VEC(I8L_F16, I8L_F16) }
      else { I8L_NORM_VEC(I8L_F16, I8L_F32) }
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(add_rmsnorm_quant_kernel<I8L_F16, NV, 1, -1>, dim3(M), dim3(th), 0, s, 1, a)))
    }
  }
#undef I8L_NORM_VEC
  return finish_launch(err, "add_rmsnorm_quant launch");
}

extern "C" int i8l_silu_mul_quant(const void *gate_up, int64_t ld, int32_t act_dtype, int8_t *q,
                                  int64_t ldq, float *scale, int32_t M, int32_t I,
                                  int32_t precise_div, int32_t round_silu, void *stream) {
  return i8l_silu_mul_quant_ex(gate_up, ld, act_dtype, q, ldq, scale, M, I, precise_div,
                               round_silu, nullptr, nullptr, stream);
}

extern "C" int i8l_silu_mul_quant_ex(const void *gate_up, int64_t ld, int32_t act_dtype,
                                     int8_t *q, int64_t ldq, float *scale, int32_t M, int32_t I,
                                     int32_t precise_div, int32_t round_silu,
                                     const float *absmax_in, float *absmax_out, void *stream) {
  int e = check_act(act_dtype);
  if (e) return e;
  if (M < 0 || I <= 0) return set_error(I8L_EINVAL, "bad size M=%d I=%d", M, I);
  if (M == 0) return I8L_OK;
  if (!gate_up || (!absmax_out && (!q || !scale)))
    return set_error(I8L_EINVAL, "NULL pointer argument");
  if (absmax_in && absmax_out) return set_error(I8L_EINVAL, "absmax_in and absmax_out are exclusive");
  if (ld < 2LL * I || (!absmax_out && ldq < I)) return set_error(I8L_EINVAL, "row stride too small");
  SiluArgs a{absmax_in, absmax_out, gate_up, ld, q, ldq, scale, I, precise_div, round_silu};
  const bool vec = I % 8 == 0 && ld % 8 == 0 && aligned16(gate_up) &&
                   (absmax_out || (ldq % 8 == 0 && aligned16(q)));
  RowShape rs;
  if (!row_shape(I, vec ? 8 : 1, &rs, row_threads(M))) return set_error(I8L_ENOTSUP, "row of %d values is too long", I);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nv = rs.nv, th = rs.threads;
  cudaError_t err = cudaSuccess;
  if (act_dtype == I8L_BF16) {
    if (vec) {
      I8L_DISPATCH_NV(nv, (err = launch(silu_mul_quant_kernel<I8L_BF16, NV, 8>, dim3(M), dim3(th), 0, s, 1, a)))
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(silu_mul_quant_kernel<I8L_BF16, NV, 1>, dim3(M), dim3(th), 0, s, 1, a)))
    }
  } else {
    if (vec) {
      I8L_DISPATCH_NV(nv, (err = launch(silu_mul_quant_kernel<I8L_F16, NV, 8>, dim3(M), dim3(th), 0, s, 1, a)))
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(silu_mul_quant_kernel<I8L_F16, NV, 1>, dim3(M), dim3(th), 0, s, 1, a)))
    }
  }
  return finish_launch(err, "silu_mul_quant launch");
}

extern "C" int i8l_quant_rows(const void *x, int64_t ldx, int32_t act_dtype, int8_t *q,
                              int64_t ldq, float *scale, int32_t M, int32_t K,
                              int32_t precise_div, void *stream) {
  return i8l_quant_rows_ex(x, ldx, act_dtype, q, ldq, scale, M, K, precise_div, nullptr, nullptr,
                           stream);
}

extern "C" int i8l_quant_rows_ex(const void *x, int64_t ldx, int32_t act_dtype, int8_t *q,
                                 int64_t ldq, float *scale, int32_t M, int32_t K,
                                 int32_t precise_div, const float *absmax_in, float *absmax_out,
                                 void *stream) {
  int e = check_act(act_dtype);
  if (e) return e;
  if (M < 0 || K <= 0) return set_error(I8L_EINVAL, "bad size M=%d K=%d", M, K);
  if (M == 0) return I8L_OK;
  if (!x || (!absmax_out && (!q || !scale))) return set_error(I8L_EINVAL, "NULL pointer argument");
  if (absmax_in && absmax_out) return set_error(I8L_EINVAL, "absmax_in and absmax_out are exclusive");
  if (ldx < K || (!absmax_out && ldq < K)) return set_error(I8L_EINVAL, "row stride smaller than K");
  QuantArgs a{absmax_in, absmax_out, x, ldx, q, ldq, scale, K, precise_div};
  const bool vec = K % 8 == 0 && ldx % 8 == 0 && aligned16(x) &&
                   (absmax_out || (ldq % 8 == 0 && aligned16(q)));
  RowShape rs;
  if (!row_shape(K, vec ? 8 : 1, &rs, row_threads(M))) return set_error(I8L_ENOTSUP, "row of %d values is too long", K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nv = rs.nv, th = rs.threads;
  cudaError_t err = cudaSuccess;
  if (act_dtype == I8L_BF16) {
    if (vec) {
      I8L_DISPATCH_NV(nv, (err = launch(quant_rows_kernel<I8L_BF16, NV, 8>, dim3(M), dim3(th), 0, s, 1, a)))
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(quant_rows_kernel<I8L_BF16, NV, 1>, dim3(M), dim3(th), 0, s, 1, a)))
    }
  } else {
    if (vec) {
      I8L_DISPATCH_NV(nv, (err = launch(quant_rows_kernel<I8L_F16, NV, 8>, dim3(M), dim3(th), 0, s, 1, a)))
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(quant_rows_kernel<I8L_F16, NV, 1>, dim3(M), dim3(th), 0, s, 1, a)))
    }
  }
  return finish_launch(err, "quant_rows launch");
}

extern "C" int i8l_dequant_i32(const int32_t *acc, int64_t lda, const float *sa, int32_t sa_per_row,
                               const float *sb, int32_t sb_per_col, const void *bias,
                               int32_t bias_dtype, void *out, int32_t out_dtype, int64_t ldo,
                               int32_t M, int32_t N, void *stream) {
  if (M < 0 || N < 0) return set_error(I8L_EINVAL, "bad size M=%d N=%d", M, N);
  if (M == 0 || N == 0) return I8L_OK;
  if (!acc || !sa || !sb || !out) return set_error(I8L_EINVAL, "NULL pointer argument");
  if (out_dtype < I8L_BF16 || out_dtype > I8L_F32)
    return set_error(I8L_ENOTSUP, "output dtype code %d not supported", out_dtype);
  if (bias && (bias_dtype < I8L_BF16 || bias_dtype > I8L_F32))
    return set_error(I8L_ENOTSUP, "bias dtype code %d not supported", bias_dtype);
  if (lda < N || ldo < N) return set_error(I8L_EINVAL, "row stride smaller than N");
  DequantArgs a{reinterpret_cast<const int *>(acc), lda, sa, sa_per_row, sb, sb_per_col, bias,
                bias_dtype, out, out_dtype, ldo, M, N};
  const long long total = static_cast<long long>(M) * N;
  const int esize = out_dtype == I8L_F32 ? 4 : 2;
  const bool vec = N % 8 == 0 && lda % 4 == 0 && (ldo * esize) % 16 == 0 && aligned16(acc) &&
                   aligned16(out);
  const long long units = vec ? total / 8 : total;
  const int blocks = static_cast<int>(std::min<long long>((units + 255) / 256, 148LL * 16));
  cudaError_t err = launch(vec ? dequant_i32_vec8_kernel : dequant_i32_kernel, dim3(blocks), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), 1, a);
  return finish_launch(err, "dequant_i32 launch");
}
