// W8A8 GEMM for decode batches of at most 8 tokens, on the CUDA cores (split mode 5).
//
// Computes what the reference's Triton kernel _w8a8_mm computes
// (int8_linear/kernel.py:63-124 in AshrithaG/int8-linear), with the same epilogue
// order as the tensor-core kernel (epilogue.cuh):
//     out[m,n] = cast( ((float(acc[m,n]) * sa[m]) * sb[n]) + float(bias[n]) )
//
// Why a CUDA-core path: with 1-8 tokens a tcgen05 MMA does 1-8 useful columns of 128,
// and spreading a weight of a few MB over all SMs forces split-K, whose cross-CTA
// reduction (cluster DSMEM round trips, or L2 partial sums) costs microseconds after
// the dependency wait.  Here every CTA owns complete output columns: the weight's N rows
// are dealt out in contiguous ranges, one per CTA, so no CTA ever needs another's sums.
//
// Per CTA (9 warps):
//   warp 0 lane 0  producer: streams the CTA's weight rows through a ring of shared-
//                  memory stages with 1-D bulk copies (cp.async.bulk, completion counted
//                  on an mbarrier).  Weights never depend on the previous kernel, so the
//                  producer starts at once: under programmatic dependent launch the first
//                  `stages` stages (often the CTA's whole share) arrive while the kernel
//                  before is still running.
//   warps 1-8      wait for the previous kernel (griddepcontrol.wait), copy the M x K
//                  activation into shared memory, then take (row group, 512-byte K
//                  segment) tasks: each lane keeps its 16 activation bytes of the segment
//                  per token in registers, multiplies them into RG weight rows with dp4a
//                  (exact int32), the warp sums the lanes with shuffles and lane 0 adds the
//                  result into the row's shared int32 accumulator (integer adds: order-
//                  free, exact).  Last, the accumulators are dequantised and stored with
//                  consecutive threads on consecutive output columns.
#include <algorithm>

#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"
#include "rows.cuh"

namespace i8l {

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvConsumers = 32 * kGemvConsumerWarps;
constexpr int kGemvThreads = kGemvConsumers + 32;
constexpr int kGemvSeg = 512;  // K bytes of one task: 32 lanes x 16 bytes

struct GemvArgs {
  int M, N, K;
  const int8_t *A;
  long long lda;
  const int8_t *W;
  long long ldw;
  const float *sa;
  const float *sb;
  int sa_per_row, sb_per_col;
  const void *bias;
  int bias_dtype;
  void *out;
  int out_dtype;
  long long ldc;
  int stage_rows;  // weight rows per ring stage
  int stages;      // ring depth
  int max_rows;    // most rows one CTA owns (sizes the accumulators)
  int *status;
  // Activation prologue (pro != 0): every CTA makes the int8 activation and its per-token
  // scales itself from a bf16/fp16 input, as the standalone quantiser kernel would, instead
  // of reading them: 1 per-token quantisation of X, 2 add + RMSNorm + quantisation of X
  // (+ residual; CTA 0 writes the residual output), 3 SiLU-and-mul + quantisation of
  // X = [gate | up].
  int pro;
  const void *x;
  long long ldx;
  int x_dtype;
  const void *res;
  long long ldr;
  void *rout;
  long long ldro;
  const void *nw;
  int nw_dtype;
  float eps;
  int precise, round_silu;
  int pro_threads;  // threads per row of the standalone kernel (its reduction order)
};

// Shared memory: barriers | accumulators [max_rows][MT] int32 | activation [M][K] |
// ring [stages][stage_rows][K].  Every part starts on a 16-byte boundary (bulk copies
// and 16-byte vector loads need it).
struct GemvLayout {
  size_t bars, acc, act, ring, total;
  __host__ __device__ GemvLayout(int stages, int max_rows, int mt, int m, int k, int stage_rows) {
    bars = 0;
    acc = ((2 * static_cast<size_t>(stages) * 8 + 16) + 15) & ~static_cast<size_t>(15);
    act = acc + ((static_cast<size_t>(max_rows) * mt * 4 + 15) & ~static_cast<size_t>(15));
    ring = act + static_cast<size_t>(m) * k;
    total = ring + static_cast<size_t>(stages) * stage_rows * k;
  }
};

// 1-D bulk copy global -> shared, completion counted in bytes on `bar`.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes,
                                          uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 16 bytes through L2 only: the activation was written by the kernel before this one.
__device__ __forceinline__ uint4 ld_cg_v4(const int8_t *p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ int dot16(const uint4 &w, const uint4 &x, int c) {
  c = __dp4a(static_cast<int>(w.x), static_cast<int>(x.x), c);
  c = __dp4a(static_cast<int>(w.y), static_cast<int>(x.y), c);
  c = __dp4a(static_cast<int>(w.z), static_cast<int>(x.z), c);
  return __dp4a(static_cast<int>(w.w), static_cast<int>(x.w), c);
}

// Sums V per-lane values (V a power of two, at most 32) over the 32 lanes of a warp,
// transposing as it goes: at each of log2(V) steps a lane keeps half of its values and
// adds the partner lane's copy of that half (one shuffle per kept value), so after the
// steps every lane holds one value index; plain butterfly steps then finish the sum.
// 31 shuffles for 32 values instead of 5 per value.  Lane l ends with the total of
// value (l >> (5 - log2 V)) & (V - 1).
template <int V>
__device__ __forceinline__ int warp_sum_transposed(int (&v)[V], int lane) {
  constexpr int P = V == 1 ? 0 : V == 2 ? 1 : V == 4 ? 2 : V == 8 ? 3 : V == 16 ? 4 : 5;
  static_assert((1 << P) == V, "V must be a power of two <= 32");
#pragma unroll
  for (int step = 0; step < P; ++step) {
    const int o = 16 >> step;
    const int half = V >> (step + 1);
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const int send = upper ? v[i] : v[i + half];
      const int keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  int r = v[0];
#pragma unroll
  for (int o = 16 >> P; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

// ---------------------------------------------------------------- activation prologue
__device__ __forceinline__ float half_bits_to_f32(uint32_t h, bool f16) {
  return f16 ? __half2float(__ushort_as_half(static_cast<unsigned short>(h))) : __uint_as_float(h << 16);
}

__device__ __forceinline__ void unpack8(const uint4 &r, bool f16, float (&o)[8]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    o[2 * j] = half_bits_to_f32(w[j] & 0xffffu, f16);
    o[2 * j + 1] = half_bits_to_f32(w[j] >> 16, f16);
  }
}

__device__ __forceinline__ uint32_t f32_to_half_bits(float v, bool f16) {
  if (f16) return __half_as_ushort(__float2half_rn(v));
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float round_act(float v, bool f16) {
  return f16 ? round_through<I8L_F16>(v) : round_through<I8L_BF16>(v);
}

__device__ __forceinline__ float round_weight_dtype(float v, int dtype) {
  return dtype == I8L_BF16 ? round_through<I8L_BF16>(v)
                           : (dtype == I8L_F16 ? round_through<I8L_F16>(v) : v);
}

__device__ __forceinline__ float weight_at(const void *w, int dtype, int i) {
  return dtype == I8L_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(w)[i])
                           : (dtype == I8L_F16 ? __half2float(static_cast<const __half *>(w)[i])
                                               : static_cast<const float *>(w)[i]);
}

// Sums (or maxima) of MT per-row values over the consumer threads, each row in exactly
// the steps of the standalone kernels' block reduction over `nw` warps: a butterfly in
// the warp, the warp results in shared memory, then every warp reads them (lanes past nw
// read 0) and butterflies again.  All MT rows share the two barriers.
template <int MT, bool kMax>
__device__ __forceinline__ void rows_reduce(float (&v)[MT], float (*red)[8], int ctid, int nw) {
  const int lane = ctid & 31, w = ctid >> 5;
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, v[m], o);
      v[m] = kMax ? fmaxf(v[m], t) : __fadd_rn(v[m], t);
    }
  if (lane == 0)
#pragma unroll
    for (int m = 0; m < MT; ++m) red[m][w] = v[m];
  named_bar_sync(1, kGemvConsumers);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    v[m] = lane < nw ? red[m][lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, v[m], o);
      v[m] = kMax ? fmaxf(v[m], t) : __fadd_rn(v[m], t);
    }
  }
  named_bar_sync(1, kGemvConsumers);
}

// The M x K int8 activation (into `act`, rows K bytes apart) and its per-token scales
// (into scale_s) from the prologue's input, with the standalone kernels' arithmetic:
//   pro 1  quant_rows_kernel        y = x
//   pro 2  add_rmsnorm_quant_kernel x += res (stored rounded as the residual output);
//          var = sum(x^2)/K (same per-thread order and reduction tree), xn = x*rsqrt(var+eps),
//          y = act(weight_dtype(xn) * w)
//   pro 3  silu_mul_quant_kernel    y = act(act?(g / (1 + exp(-g))) * u)
// then the row quantiser: scale = absmax/127, q = rint(y * 127/absmax) saturated.  Thread
// ctid < pro_threads owns vectors (v * pro_threads + ctid) * 8 of every row, as the
// standalone kernel's thread ctid does.  NVP: vectors per thread.
template <int MT, int NVP>
__device__ __forceinline__ void gemv_prologue(const GemvArgs &a, int8_t *act, float *scale_s,
                                              float (*red)[8], int ctid) {
  const int K = a.K, th = a.pro_threads, nw = th >> 5;
  const bool f16 = a.x_dtype == I8L_F16;
  const auto *xb = static_cast<const uint8_t *>(a.x);
  float y[MT][NVP][8];
  float ss[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    ss[m] = 0.f;
#pragma unroll
    for (int v = 0; v < NVP; ++v) {
      const int col = (v * th + ctid) * 8;
      const bool live = m < a.M && ctid < th && col < K;
#pragma unroll
      for (int i = 0; i < 8; ++i) y[m][v][i] = 0.f;
      if (!live) continue;
      const uint4 xr = __ldcg(reinterpret_cast<const uint4 *>(xb + (m * a.ldx + col) * 2));
      if (a.pro == 3) {
        const uint4 ur = __ldcg(reinterpret_cast<const uint4 *>(xb + (m * a.ldx + K + col) * 2));
        float g[8], u[8];
        unpack8(xr, f16, g);
        unpack8(ur, f16, u);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float sl = div_full(g[i], __fadd_rn(1.0f, expf(-g[i])));
          if (a.round_silu) sl = round_act(sl, f16);
          y[m][v][i] = round_act(__fmul_rn(sl, u[i]), f16);
        }
      } else {
        unpack8(xr, f16, y[m][v]);
        if (a.pro == 2 && a.res) {
          const uint4 rr = __ldcg(reinterpret_cast<const uint4 *>(
              static_cast<const uint8_t *>(a.res) + (m * a.ldr + col) * 2));
          float r[8];
          unpack8(rr, f16, r);
          uint32_t packed[4];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[m][v][i] = __fadd_rn(y[m][v][i], r[i]);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            packed[j] = f32_to_half_bits(y[m][v][2 * j], f16) | (f32_to_half_bits(y[m][v][2 * j + 1], f16) << 16);
          if (blockIdx.x == 0)
            *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(a.rout) + (m * a.ldro + col) * 2) =
                make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
        if (a.pro == 2)
#pragma unroll
          for (int i = 0; i < 8; ++i) ss[m] = __fadd_rn(ss[m], __fmul_rn(y[m][v][i], y[m][v][i]));
      }
    }
  }
  if (a.pro == 2) {
    rows_reduce<MT, false>(ss, red, ctid, nw);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float var = div_full(ss[m], static_cast<float>(K));
      const float rs = rsqrtf(__fadd_rn(var, a.eps));
#pragma unroll
      for (int v = 0; v < NVP; ++v) {
        const int col = (v * th + ctid) * 8;
        if (!(m < a.M && ctid < th && col < K)) continue;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xn = round_weight_dtype(__fmul_rn(y[m][v][i], rs), a.nw_dtype);
          y[m][v][i] = round_act(__fmul_rn(xn, weight_at(a.nw, a.nw_dtype, col + i)), f16);
        }
      }
    }
  }
  float mx[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    mx[m] = 0.f;
#pragma unroll
    for (int v = 0; v < NVP; ++v)
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[m] = fmaxf(mx[m], fabsf(y[m][v][i]));
  }
  rows_reduce<MT, true>(mx, red, ctid, nw);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m >= a.M) continue;
    const float amax = mx[m];
    if (ctid == 0) scale_s[m] = a.precise ? div_rn(amax, 127.f) : div_full(amax, 127.f);
    const float inv = amax == 0.f ? 0.f : (a.precise ? div_rn(127.f, amax) : div_full(127.f, amax));
#pragma unroll
    for (int v = 0; v < NVP; ++v) {
      const int col = (v * th + ctid) * 8;
      if (!(ctid < th && col < K)) continue;
      uint32_t w[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r0 = __float2int_rn(__fmul_rn(y[m][v][4 * h], inv));
        const int r1 = __float2int_rn(__fmul_rn(y[m][v][4 * h + 1], inv));
        const int r2 = __float2int_rn(__fmul_rn(y[m][v][4 * h + 2], inv));
        const int r3 = __float2int_rn(__fmul_rn(y[m][v][4 * h + 3], inv));
        uint32_t t;
        asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(t) : "r"(r3), "r"(r2));
        asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w[h]) : "r"(r1), "r"(r0), "r"(t));
      }
      *reinterpret_cast<uint2 *>(act + static_cast<size_t>(m) * K + col) = make_uint2(w[0], w[1]);
    }
  }
}

// MT: most tokens (1, 2, 4 or 8); RG: weight rows per task (activation reuse).
// NVP: vectors per thread of the activation prologue, 0 for an int8 activation.  Up to 8
// tokens two CTAs share an SM (the next kernel's beside this one); 16 tokens hold more
// registers (one CTA per SM).
template <int MT, int RG, int NVP>
__global__ void __launch_bounds__(kGemvThreads, MT <= 8 ? 2 : 1) w8a8_gemv_sm100(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float pro_red[8][8];
  __shared__ float pro_scale[8];
  const GemvLayout L(a.stages, a.max_rows, MT, a.M, a.K, a.stage_rows);
  const int S = a.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem);
  uint64_t *empty = full + S;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + S);
  int *acc = reinterpret_cast<int *>(smem + L.acc);
  int8_t *act = reinterpret_cast<int8_t *>(smem + L.act);
  uint8_t *ring = smem + L.ring;
  const int K = a.K;
  const size_t stage_bytes = static_cast<size_t>(a.stage_rows) * K;

  const int n0 = static_cast<int>(static_cast<long long>(blockIdx.x) * a.N / gridDim.x);
  const int n1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * a.N / gridDim.x);
  const int rows = n1 - n0;
  const int nst = (rows + a.stage_rows - 1) / a.stage_rows;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGemvConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();  // each weight byte is read once
      int issued = 0;
      for (int it = 0; it < nst; ++it) {
        const int s = it % S;
        const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
        if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag, a.status, kStatusProducerWait)) break;
        const int r0 = n0 + it * a.stage_rows;
        const int rc = min(a.stage_rows, n1 - r0);
        uint8_t *dst = ring + s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rc) * K);
        if (a.ldw == K) {
          bulk_load(dst, a.W + static_cast<long long>(r0) * K, static_cast<uint32_t>(rc) * K, &full[s], pol);
        } else {
          for (int r = 0; r < rc; ++r)
            bulk_load(dst + static_cast<size_t>(r) * K, a.W + static_cast<long long>(r0 + r) * a.ldw,
                      static_cast<uint32_t>(K), &full[s], pol);
        }
        ++issued;
      }
      if (issued < nst) {
        // Gave up: let the copies in flight land before the CTA's memory goes away.
        // They are the last min(issued, S) stages issued; each completes its phase.
        for (int it = max(0, issued - S); it < issued; ++it) {
          volatile int no_abort = 0;
          mbar_wait_bounded(&full[it % S], static_cast<uint32_t>(it / S) & 1u, &no_abort, a.status,
                            kStatusDrainWait);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int ctid = threadIdx.x - 32;
  const int cw = warp - 1;
  pdl_wait();  // the activation, scales and output belong to the stream's order
  for (int i = ctid; i < rows * MT; i += kGemvConsumers) acc[i] = 0;
  if constexpr (NVP > 0) {
    gemv_prologue<MT, NVP>(a, act, pro_scale, pro_red, ctid);
  } else {
    const int chunks = K / 16;
    const int n = a.M * chunks;
    for (int i = ctid; i < n; i += kGemvConsumers) {
      const int m = i / chunks, c = i - m * chunks;
      *reinterpret_cast<uint4 *>(act + static_cast<size_t>(m) * K + c * 16) =
          ld_cg_v4(a.A + m * a.lda + c * 16);
    }
  }
  named_bar_sync(1, kGemvConsumers);

  const int nseg = (K + kGemvSeg - 1) / kGemvSeg;
  bool ok = true;
  for (int it = 0; it < nst && ok; ++it) {
    const int s = it % S;
    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(it / S) & 1u, abort_flag, a.status,
                           kStatusMmaWait)) {
      ok = false;
      break;
    }
    const int rc = min(a.stage_rows, rows - it * a.stage_rows);
    const int8_t *st = reinterpret_cast<const int8_t *>(ring + s * stage_bytes);
    const int ngroups = (rc + RG - 1) / RG;
    for (int task = cw; task < ngroups * nseg; task += kGemvConsumerWarps) {
      const int g = task / nseg, j = task - g * nseg;
      const int kb = j * kGemvSeg + lane * 16;
      const bool live = kb < K;
      uint4 x[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m)
        x[m] = (live && m < a.M) ? *reinterpret_cast<const uint4 *>(act + static_cast<size_t>(m) * K + kb)
                                 : make_uint4(0u, 0u, 0u, 0u);
      int sum[RG * MT];   // value rr * MT + m: row g*RG + rr, token m
#pragma unroll
      for (int rr = 0; rr < RG; ++rr) {
        const int r = g * RG + rr;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (live && r < rc) w = *reinterpret_cast<const uint4 *>(st + static_cast<size_t>(r) * K + kb);
#pragma unroll
        for (int m = 0; m < MT; ++m) sum[rr * MT + m] = dot16(w, x[m], 0);
      }
      constexpr int kV = RG * MT;
      constexpr int kShift = kV == 1 ? 5 : kV == 2 ? 4 : kV == 4 ? 3 : kV == 8 ? 2 : kV == 16 ? 1 : 0;
      const int total = warp_sum_transposed<kV>(sum, lane);
      if ((lane & ((1 << kShift) - 1)) == 0) {
        const int idx = (lane >> kShift) & (kV - 1);
        const int r = g * RG + idx / MT, m = idx % MT;
        if (r < rc && m < a.M) atomicAdd(&acc[(it * a.stage_rows + r) * MT + m], total);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!named_bar_and(1, kGemvConsumers, ok)) return;

  // -------------------------------------------------------------- epilogue
  const bool raw = a.out_dtype == I8L_I32;
  const bool has_bias = a.bias != nullptr;
  for (int i = ctid; i < rows * a.M; i += kGemvConsumers) {
    const int m = i / rows, r = i - m * rows;
    const int n = n0 + r;
    const int v = acc[r * MT + m];
    float f = 0.f;
    if (!raw) {
      const float sa = NVP > 0 ? pro_scale[m] : (a.sa_per_row ? a.sa[m] : a.sa[0]);
      const float sb = a.sb_per_col ? a.sb[n] : a.sb[0];
      f = dequant(v, sa, sb, has_bias ? load_scalar_f(a.bias, a.bias_dtype, n) : 0.f, has_bias);
    }
    store_elem(a.out, a.out_dtype, static_cast<long long>(m) * a.ldc + n, v, f);
  }
}

template <int MT, int RG, int NVP>
static int launch_gemv(const GemvArgs &a, int ctas, size_t smem, cudaStream_t stream) {
  static size_t configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64 || smem > configured[dev]) {
    e = cudaFuncSetAttribute(w8a8_gemv_sm100<MT, RG, NVP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemv smem)");
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  e = launch(w8a8_gemv_sm100<MT, RG, NVP>, dim3(ctas), dim3(kGemvThreads), smem, stream, 1, a);
  if (e != cudaSuccess) return cuda_error(e, "gemv launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "gemv launch");
  return I8L_OK;
}

// Shared memory of one of two CTAs that share an SM (228 KB minus 1 KB reserved per CTA).
constexpr int kGemvHalfSmem = 233472 / 2 - 1024;

int gemv_plan(int M, int N, int K, const i8l_tile *t, GemvPlan *p) {
  DeviceInfo di;
  int e = device_info(&di);
  if (e) return e;
  const int mt = t->tok_tile;
  if (mt != 1 && mt != 2 && mt != 4 && mt != 8 && mt != 16)
    return set_error(I8L_ENOTSUP, "CUDA-core tiles (split 5) take tok_tile 1, 2, 4, 8 or 16, got %d", mt);
  if (M > mt)
    return set_error(I8L_ENOTSUP, "CUDA-core tile for %d tokens given M=%d", mt, M);
  p->mt = mt;
  p->ctas = t->ctas > 0 ? std::min(t->ctas, N) : std::min(di.sms, N);
  p->max_rows = (N + p->ctas - 1) / p->ctas;
  // Stages of about 32 KB of whole rows (bulk copies that size reach the SM's full ingest
  // rate), rounded up to whole row groups of the kernel's tasks when that stays <= 48 KB,
  // at most one CTA's rows.
  const int rg = mt == 16 ? 2 : (mt == 8 ? 4 : 8);
  int sr = std::max(1, 32768 / K);
  const int sr_groups = (sr + rg - 1) / rg * rg;
  if (static_cast<long long>(sr_groups) * K <= 49152) sr = sr_groups;
  p->stage_rows = std::max(1, std::min(p->max_rows, sr));
  const int needed = (p->max_rows + p->stage_rows - 1) / p->stage_rows;
  const size_t fixed = GemvLayout(0, p->max_rows, mt, M, K, p->stage_rows).ring + 2 * 8 * 16;
  const size_t stage = static_cast<size_t>(p->stage_rows) * K;
  // stages = 0: as many as fit beside a second CTA on the SM (the next kernel's, under
  // programmatic dependent launch); a given depth is capped by what one CTA can hold.
  const long long budget = (t->stages > 0 || mt == 16) ? di.max_smem_optin : kGemvHalfSmem;
  const long long fit = (budget - static_cast<long long>(fixed)) / static_cast<long long>(stage);
  long long st = t->stages > 0 ? std::min<long long>(t->stages, fit) : fit;
  st = std::max(1LL, std::min<long long>(st, std::max(needed, 1)));
  p->stages = static_cast<int>(st);
  p->smem = GemvLayout(p->stages, p->max_rows, mt, M, K, p->stage_rows).total;
  if (p->smem > static_cast<size_t>(di.max_smem_optin))
    return set_error(I8L_ENOTSUP,
                     "CUDA-core tile needs %zu bytes of shared memory (M=%d, K=%d, %d stages of %d rows); "
                     "%d available",
                     p->smem, M, K, p->stages, p->stage_rows, di.max_smem_optin);
  return I8L_OK;
}

int gemv_run(const int8_t *A, int64_t lda, const int8_t *W, int64_t ldw, const float *sa,
             int32_t sa_per_row, const float *sb, int32_t sb_per_col, const void *bias,
             int32_t bias_dtype, void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N,
             int32_t K, const i8l_tile *tile, void *stream, const GemvPro *pro) {
  GemvPlan p;
  int e = gemv_plan(M, N, K, tile, &p);
  if (e) return e;
  GemvArgs a{};
  int nvp = 0;
  if (pro) {
    if (pro->x_dtype != I8L_BF16 && pro->x_dtype != I8L_F16)
      return set_error(I8L_ENOTSUP, "activation dtype code %d not supported (bf16 or fp16)", pro->x_dtype);
    if (!pro->x) return set_error(I8L_EINVAL, "NULL activation pointer");
    if (pro->ldx < (pro->mode == 3 ? 2LL * K : static_cast<long long>(K)))
      return set_error(I8L_EINVAL, "activation row stride %lld too small for K=%d",
                       static_cast<long long>(pro->ldx), K);
    if (K % 8 || pro->ldx % 8 || !aligned16(pro->x))
      return set_error(I8L_ENOTSUP, "the fused quantiser needs 16-byte aligned activation rows");
    if (pro->mode == 2) {
      if (!pro->nw) return set_error(I8L_EINVAL, "NULL norm weight");
      if (pro->nw_dtype < I8L_BF16 || pro->nw_dtype > I8L_F32)
        return set_error(I8L_ENOTSUP, "norm weight dtype code %d not supported", pro->nw_dtype);
      if ((pro->res == nullptr) != (pro->rout == nullptr))
        return set_error(I8L_EINVAL, "residual and residual_out must be given together");
      if (pro->res) {
        if (pro->ldr < K || pro->ldro < K) return set_error(I8L_EINVAL, "residual row stride smaller than K");
        if (pro->ldr % 8 || pro->ldro % 8 || !aligned16(pro->res) || !aligned16(pro->rout))
          return set_error(I8L_ENOTSUP, "the fused norm needs 16-byte aligned residual rows");
      }
    }
    RowShape rs;
    if (!row_shape(K, 8, &rs)) return set_error(I8L_ENOTSUP, "row of %d values is too long", K);
    nvp = rs.nv;
    if (rs.threads > kGemvConsumers || nvp > 3 || p.mt * nvp > 8)
      return set_error(I8L_ENOTSUP,
                       "the fused quantiser holds at most 8 row vectors of 8 values per thread "
                       "(%d tokens x %d vectors for K=%d)", p.mt, nvp, K);
    a.pro = pro->mode;
    a.x = pro->x;
    a.ldx = pro->ldx;
    a.x_dtype = pro->x_dtype;
    a.res = pro->res;
    a.ldr = pro->ldr;
    a.rout = pro->rout;
    a.ldro = pro->ldro;
    a.nw = pro->nw;
    a.nw_dtype = pro->nw_dtype;
    a.eps = pro->eps;
    a.precise = pro->precise ? 1 : 0;
    a.round_silu = pro->round_silu ? 1 : 0;
    a.pro_threads = rs.threads;
  }
  a.M = M;
  a.N = N;
  a.K = K;
  a.A = A;
  a.lda = lda;
  a.W = W;
  a.ldw = ldw;
  a.sa = sa;
  a.sb = sb;
  a.sa_per_row = sa_per_row ? 1 : 0;
  a.sb_per_col = sb_per_col ? 1 : 0;
  a.bias = out_dtype == I8L_I32 ? nullptr : bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  a.ldc = ldc;
  a.stage_rows = p.stage_rows;
  a.stages = p.stages;
  a.max_rows = p.max_rows;
  a.status = status_ptr();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define I8L_GEMV(MT, RG)                                                      \
  switch (nvp) {                                                              \
    case 0: return launch_gemv<MT, RG, 0>(a, p.ctas, p.smem, s);              \
    case 1: return launch_gemv<MT, RG, (MT <= 8 ? 1 : 0)>(a, p.ctas, p.smem, s); \
    case 2: return launch_gemv<MT, RG, (MT <= 4 ? 2 : 0)>(a, p.ctas, p.smem, s); \
    default: return launch_gemv<MT, RG, (MT <= 2 ? 3 : 0)>(a, p.ctas, p.smem, s); \
  }
  if (p.mt == 16) {
    if (nvp) return set_error(I8L_ENOTSUP, "the fused quantiser takes batches of at most 8 tokens");
    return launch_gemv<16, 2, 0>(a, p.ctas, p.smem, s);
  }
  switch (p.mt) {
    case 1:
      I8L_GEMV(1, 8)
    case 2:
      I8L_GEMV(2, 8)
    case 4:
      I8L_GEMV(4, 8)
    default:
      I8L_GEMV(8, 4)
  }
#undef I8L_GEMV
}

// Arguments every CUDA-core entry point checks before planning.
static int gemv_check(const int8_t *W, int64_t ldw, const float *sb, const void *bias, int32_t bias_dtype,
                      void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N, int32_t K) {
  if (M < 0 || N < 0 || K < 0) return set_error(I8L_EINVAL, "negative size M=%d N=%d K=%d", M, N, K);
  if (out_dtype < I8L_BF16 || out_dtype > I8L_I32)
    return set_error(I8L_ENOTSUP, "output dtype code %d not supported", out_dtype);
  if (K == 0) return set_error(I8L_ENOTSUP, "K=0 is not supported");
  if (K % 16) return set_error(I8L_ENOTSUP, "K=%d must be a multiple of 16", K);
  if (!W || !out) return set_error(I8L_EINVAL, "NULL operand pointer");
  if (ldw < K || ldc < N) return set_error(I8L_EINVAL, "leading dimensions ldw=%lld ldc=%lld too small",
                                           static_cast<long long>(ldw), static_cast<long long>(ldc));
  if (reinterpret_cast<uintptr_t>(W) % 16 || ldw % 16)
    return set_error(I8L_ENOTSUP, "the int8 weight and its row stride must be 16-byte aligned");
  if (out_dtype != I8L_I32) {
    if (!sb) return set_error(I8L_EINVAL, "NULL scale pointer");
    if (bias && (bias_dtype < I8L_BF16 || bias_dtype > I8L_F32))
      return set_error(I8L_ENOTSUP, "bias dtype code %d not supported", bias_dtype);
  }
  return I8L_OK;
}

// The tile of a fused-quantiser call: the caller's (a CUDA-core tile), or the CUDA-core
// tile for the fewest tokens that hold M.
static int gemv_tile(int32_t M, const i8l_tile *tile, i8l_tile *t) {
  if (tile && (tile->tok_tile || tile->w_tile || tile->split)) {
    if (tile->split != 5)
      return set_error(I8L_ENOTSUP, "the fused quantiser runs on CUDA-core tiles (split 5), got split %d",
                       tile->split);
    *t = *tile;
    return I8L_OK;
  }
  if (M > 8) return set_error(I8L_ENOTSUP, "the fused quantiser takes batches of at most 8 tokens, got %d", M);
  *t = i8l_tile{};
  t->tok_tile = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  t->split = 5;
  if (tile) {
    t->stages = tile->stages;
    t->ctas = tile->ctas;
  }
  return I8L_OK;
}

}  // namespace i8l

using namespace i8l;

extern "C" int i8l_rmsnorm_w8a8_mm(const void *x, int64_t ldx, const void *residual, int64_t ldr,
                                   const void *norm_weight, int32_t act_dtype, int32_t w_dtype,
                                   float eps, int32_t precise_div, void *residual_out, int64_t ldro,
                                   const int8_t *W, int64_t ldw, const float *sb, int32_t sb_per_col,
                                   const void *bias, int32_t bias_dtype, void *out, int32_t out_dtype,
                                   int64_t ldc, int32_t M, int32_t N, int32_t K, const i8l_tile *tile,
                                   void *stream) {
  int e = gemv_check(W, ldw, sb, bias, bias_dtype, out, out_dtype, ldc, M, N, K);
  if (e || M == 0 || N == 0) return e;
  i8l_tile t;
  if ((e = gemv_tile(M, tile, &t))) return e;
  const GemvPro pro{2, x, ldx, act_dtype, residual, ldr, residual_out, ldro, norm_weight, w_dtype, eps,
                    precise_div, 0};
  return gemv_run(nullptr, 0, W, ldw, nullptr, 0, sb, sb_per_col, bias, bias_dtype, out, out_dtype, ldc,
                  M, N, K, &t, stream, &pro);
}

extern "C" int i8l_silu_mul_w8a8_mm(const void *gate_up, int64_t ld, int32_t act_dtype,
                                    int32_t precise_div, int32_t round_silu, const int8_t *W,
                                    int64_t ldw, const float *sb, int32_t sb_per_col, const void *bias,
                                    int32_t bias_dtype, void *out, int32_t out_dtype, int64_t ldc,
                                    int32_t M, int32_t N, int32_t K, const i8l_tile *tile, void *stream) {
  int e = gemv_check(W, ldw, sb, bias, bias_dtype, out, out_dtype, ldc, M, N, K);
  if (e || M == 0 || N == 0) return e;
  i8l_tile t;
  if ((e = gemv_tile(M, tile, &t))) return e;
  const GemvPro pro{3, gate_up, ld, act_dtype, nullptr, 0, nullptr, 0, nullptr, 0, 0.f, precise_div,
                    round_silu};
  return gemv_run(nullptr, 0, W, ldw, nullptr, 0, sb, sb_per_col, bias, bias_dtype, out, out_dtype, ldc,
                  M, N, K, &t, stream, &pro);
}
