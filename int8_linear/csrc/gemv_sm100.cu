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

// MT: most tokens (1, 2, 4 or 8); RG: weight rows per task (activation reuse).
template <int MT, int RG>
__global__ void __launch_bounds__(kGemvThreads, 2) w8a8_gemv_sm100(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
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
  {
    const int chunks = K / 16;
    const int n = a.M * chunks;
    for (int i = ctid; i < n; i += kGemvConsumers) {
      const int m = i / chunks, c = i - m * chunks;
      *reinterpret_cast<uint4 *>(act + static_cast<size_t>(m) * K + c * 16) =
          ld_cg_v4(a.A + m * a.lda + c * 16);
    }
    for (int i = ctid; i < rows * MT; i += kGemvConsumers) acc[i] = 0;
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
      const float sa = a.sa_per_row ? a.sa[m] : a.sa[0];
      const float sb = a.sb_per_col ? a.sb[n] : a.sb[0];
      f = dequant(v, sa, sb, has_bias ? load_scalar_f(a.bias, a.bias_dtype, n) : 0.f, has_bias);
    }
    store_elem(a.out, a.out_dtype, static_cast<long long>(m) * a.ldc + n, v, f);
  }
}

template <int MT, int RG>
static int launch_gemv(const GemvArgs &a, int ctas, size_t smem, cudaStream_t stream) {
  static size_t configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64 || smem > configured[dev]) {
    e = cudaFuncSetAttribute(w8a8_gemv_sm100<MT, RG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemv smem)");
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  e = launch(w8a8_gemv_sm100<MT, RG>, dim3(ctas), dim3(kGemvThreads), smem, stream, 1, a);
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
  if (mt != 1 && mt != 2 && mt != 4 && mt != 8)
    return set_error(I8L_ENOTSUP, "CUDA-core tiles (split 5) take tok_tile 1, 2, 4 or 8, got %d", mt);
  if (M > mt)
    return set_error(I8L_ENOTSUP, "CUDA-core tile for %d tokens given M=%d", mt, M);
  p->mt = mt;
  p->ctas = t->ctas > 0 ? std::min(t->ctas, N) : std::min(di.sms, N);
  p->max_rows = (N + p->ctas - 1) / p->ctas;
  // Stages of about 32 KB of whole rows (bulk copies that size reach the SM's full ingest
  // rate), rounded up to whole row groups of the kernel's tasks when that stays <= 48 KB,
  // at most one CTA's rows.
  const int rg = mt == 8 ? 4 : 8;
  int sr = std::max(1, 32768 / K);
  const int sr_groups = (sr + rg - 1) / rg * rg;
  if (static_cast<long long>(sr_groups) * K <= 49152) sr = sr_groups;
  p->stage_rows = std::max(1, std::min(p->max_rows, sr));
  const int needed = (p->max_rows + p->stage_rows - 1) / p->stage_rows;
  const size_t fixed = GemvLayout(0, p->max_rows, mt, M, K, p->stage_rows).ring + 2 * 8 * 16;
  const size_t stage = static_cast<size_t>(p->stage_rows) * K;
  // stages = 0: as many as fit beside a second CTA on the SM (the next kernel's, under
  // programmatic dependent launch); a given depth is capped by what one CTA can hold.
  const long long budget = t->stages > 0 ? di.max_smem_optin : kGemvHalfSmem;
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
             int32_t K, const i8l_tile *tile, void *stream) {
  GemvPlan p;
  int e = gemv_plan(M, N, K, tile, &p);
  if (e) return e;
  GemvArgs a{};
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
  switch (p.mt) {
    case 1:
      return launch_gemv<1, 8>(a, p.ctas, p.smem, s);
    case 2:
      return launch_gemv<2, 8>(a, p.ctas, p.smem, s);
    case 4:
      return launch_gemv<4, 8>(a, p.ctas, p.smem, s);
    default:
      return launch_gemv<8, 4>(a, p.ctas, p.smem, s);
  }
}

}  // namespace i8l
