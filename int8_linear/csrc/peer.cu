// Tensor-parallel exchange kernels over NVLink peer memory, for sm_100a.
//
// A row-parallel W8A8 layer (o_proj, down) leaves each GPU an int32 partial product
// over its K/g slice; a row-split activation (the q slice of qkv, gate||up) needs the
// GLOBAL per-token absmax before it is quantised.  Instead of an NCCL collective
// followed by a separate kernel, each kernel here moves its data to the peer GPUs
// itself and computes on what arrives:
//
//   tp_allreduce_dequant      partial int32 rows -> sum over GPUs -> dequant -> bf16
//   tp_allreduce_add_rmsnorm_quant
//                             the same sum and dequant, then residual add + RMSNorm +
//                             per-token int8 of the result, in one pass per row
//   tp_quant_rows             local row absmax -> MAX over GPUs -> quantise the slice
//   tp_silu_mul_quant         silu(gate)*up absmax -> MAX over GPUs -> quantise
//
// Each GPU owns one exchange buffer (cudaMalloc'd, opened by every peer through a
// CUDA IPC handle): an inbox of 2 parities x world sources x slot bytes.
//
// One CTA handles rows r = blockIdx.x, blockIdx.x + gridDim.x, ... (the grid never
// exceeds the SM count, so all CTAs of every GPU are resident together and no wait
// depends on scheduling order).  Per call, CTA c takes epoch e = ++epochs[c] (its own
// counter in local memory; all GPUs run the same calls in the same order, so the
// counters agree).  Data moves in a low-latency format: every 8-byte word holds a
// 4-byte value and the 4-byte epoch and is written with one store to the peer's
// inbox[e & 1][rank], so a word arrives whole (aligned 8-byte stores are single-copy
// atomic).  The receiver polls its own inbox words until their epoch reads e (bounded
// in time): no fence, no separate flag, no CTA barrier, one NVLink trip.  Two parities
// suffice: a GPU can be at most one call ahead of a peer for a given CTA, because
// finishing call e needed the peer's call-e data, which the peer sends only after its
// call e-1 kernel completed (and with it every read of the other parity).
//
// Integer sums and maxima are exact and order-free, so every GPU computes exactly the
// result one GPU computes on the whole row.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "internal.h"
#include "rows.cuh"

namespace i8l {

constexpr int kMaxRanks = I8L_MAX_RANKS;

struct PeerArgs {
  uint8_t *base[kMaxRanks];  // every GPU's exchange buffer (this GPU's at base[rank])
  unsigned *epochs;          // this GPU's per-CTA call counters
  int *status;
  int rank, world;
  long long slot_bytes;      // bytes of one (parity, source) inbox slot
  int max_rows;
  unsigned long long timeout_ns;
  int two_shot;              // row-parallel sums: reduce-scatter + all-gather (see exchange_groups)
};

// inbox[parity][src] of GPU `dst`.
__device__ __forceinline__ uint8_t *inbox(const PeerArgs &p, int dst, unsigned parity, int src) {
  return p.base[dst] + (static_cast<size_t>(parity) * p.world + src) * static_cast<size_t>(p.slot_bytes);
}

// One 16-byte store of two values, each paired with the epoch: {v0, e, v1, e}.
__device__ __forceinline__ void st_ll(void *p, unsigned v0, unsigned v1, unsigned e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v0), "r"(e), "r"(v1),
               "r"(e)
               : "memory");
}

__device__ __forceinline__ uint4 ld_volatile_v4(const void *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Waits until both halves of the 16-byte word at p carry epoch e and returns the two
// values.  A wait past the time limit sets the status bit and clears `ok`; a thread
// whose `ok` is clear no longer waits (its results are invalid and the host reports
// the status), so a dead peer costs each thread one time limit at most.
__device__ __forceinline__ uint2 wait_ll(const PeerArgs &p, const void *addr, unsigned e, bool &ok) {
  uint4 w = ld_volatile_v4(addr);
  if ((w.y == e && w.w == e) || !ok) return make_uint2(w.x, w.z);
  const unsigned long long t0 = globaltimer_ns();
  for (unsigned it = 1;; ++it) {
    w = ld_volatile_v4(addr);
    if (w.y == e && w.w == e) break;
    if ((it & 15u) == 0 && globaltimer_ns() - t0 > p.timeout_ns) {
      atomicOr(p.status, kStatusPeerWait);
      ok = false;
      break;
    }
  }
  return make_uint2(w.x, w.z);
}

__device__ __forceinline__ int4 ld_cg_i4(const void *p) {
  int4 v;
  asm volatile("ld.global.cg.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// The CTA's epoch for this call (after the dependency wait: the previous call's
// kernel has completed and stored its counter).
__device__ __forceinline__ unsigned peer_begin(const PeerArgs &p, unsigned *smem_e) {
  if (threadIdx.x == 0) *smem_e = p.epochs[blockIdx.x] + 1u;
  __syncthreads();
  return *smem_e;
}

__device__ __forceinline__ void peer_end(const PeerArgs &p, unsigned e) {
  if (threadIdx.x == 0) p.epochs[blockIdx.x] = e;
}

// Sends four int32 values (one 4-column group) of a row to every peer's inbox, in the
// low-latency format (32 bytes per group).
__device__ __forceinline__ void send_group(const PeerArgs &p, size_t off, int4 v, unsigned e) {
  const unsigned par = e & 1u;
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    uint8_t *dst = inbox(p, r, par, p.rank) + off;
    st_ll(dst, static_cast<unsigned>(v.x), static_cast<unsigned>(v.y), e);
    st_ll(dst + 16, static_cast<unsigned>(v.z), static_cast<unsigned>(v.w), e);
  }
}

// Adds every peer's four int32 values of the group at `off` into v.
__device__ __forceinline__ void receive_group(const PeerArgs &p, size_t off, int4 &v, unsigned e, bool &ok) {
  const unsigned par = e & 1u;
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    const uint8_t *src = inbox(p, p.rank, par, r) + off;
    const uint2 a = wait_ll(p, src, e, ok);
    const uint2 b = wait_ll(p, src + 16, e, ok);
    v.x += static_cast<int>(a.x);
    v.y += static_cast<int>(a.y);
    v.z += static_cast<int>(b.x);
    v.w += static_cast<int>(b.y);
  }
}

// Sums G 4-column groups of one row over the GPUs: group g (columns cols[g]..+3, skipped
// when cols[g] >= N) of this GPU's partials is v[g] on entry and the sum on return.
// One-shot: every GPU sends its groups to every other GPU and adds what arrives.
// Two-shot: the row's columns are split into `world` equal slices; the GPU that owns a
// group's slice receives that group from every other GPU and adds it (reduce-scatter),
// then sends the sum to every other GPU, which takes it as is (all-gather).  A group
// travels into inbox[parity][src] at its column offset in both phases: in the first
// only into the owner's slice columns, in the second only from the owner into its own
// slice columns, so the two never write the same words of a call.
template <int G>
__device__ __forceinline__ void exchange_groups(const PeerArgs &p, size_t row_off, const int (&cols)[G],
                                                int4 (&v)[G], int N, unsigned e, bool &ok) {
  if (!p.two_shot) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      if (cols[g] < N) send_group(p, row_off + static_cast<size_t>(cols[g]) * 8, v[g], e);
#pragma unroll
    for (int g = 0; g < G; ++g)
      if (cols[g] < N) receive_group(p, row_off + static_cast<size_t>(cols[g]) * 8, v[g], e, ok);
    return;
  }
  const unsigned par = e & 1u;
  const int slice = N / p.world;
  // phase 1: each group not in this GPU's slice to its owner
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (cols[g] >= N) continue;
    const int o = cols[g] / slice;
    if (o == p.rank) continue;
    uint8_t *dst = inbox(p, o, par, p.rank) + row_off + static_cast<size_t>(cols[g]) * 8;
    st_ll(dst, static_cast<unsigned>(v[g].x), static_cast<unsigned>(v[g].y), e);
    st_ll(dst + 16, static_cast<unsigned>(v[g].z), static_cast<unsigned>(v[g].w), e);
  }
  // this GPU's slice: add every other GPU's group, then send the sum to each of them
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (cols[g] >= N || cols[g] / slice != p.rank) continue;
    const size_t off = row_off + static_cast<size_t>(cols[g]) * 8;
    receive_group(p, off, v[g], e, ok);
    send_group(p, off, v[g], e);
  }
  // phase 2: the other slices' sums from their owners
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (cols[g] >= N) continue;
    const int o = cols[g] / slice;
    if (o == p.rank) continue;
    const uint8_t *src = inbox(p, p.rank, par, o) + row_off + static_cast<size_t>(cols[g]) * 8;
    const uint2 lo = wait_ll(p, src, e, ok);
    const uint2 hi = wait_ll(p, src + 16, e, ok);
    v[g] = make_int4(static_cast<int>(lo.x), static_cast<int>(lo.y), static_cast<int>(hi.x),
                     static_cast<int>(hi.y));
  }
}

// ------------------------------------------------------------------ all-reduce + dequant

struct ReduceArgs {
  PeerArgs p;
  const int *partial;  // this GPU's int32 partial product, row m at partial + m*ldp
  long long ldp;
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

__device__ __forceinline__ float bias_at(const void *bias, int dtype, int n) {
  if (dtype == I8L_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(bias)[n]);
  if (dtype == I8L_F16) return __half2float(static_cast<const __half *>(bias)[n]);
  return static_cast<const float *>(bias)[n];
}

// The GEMM epilogue's arithmetic: ((float(acc) * sa) * sb) + bias, fp32, no FMA.
__device__ __forceinline__ float dequant_one(int acc, float sa, const ReduceArgs &a, int n) {
  float v = __fmul_rn(__int2float_rn(acc), sa);
  v = __fmul_rn(v, a.sb_per_col ? a.sb[n] : a.sb[0]);
  if (a.bias) v = __fadd_rn(v, bias_at(a.bias, a.bias_dtype, n));
  return v;
}

// Sums row `row` of the int32 partials over the GPUs into `acc` (this thread's
// 4-column groups c = (v*blockDim + tid)*4, v < NV); a group occupies 32 bytes of the
// inbox (low-latency format).
template <int NV>
__device__ __forceinline__ void reduce_row(const ReduceArgs &a, int row, unsigned e, bool &ok,
                                           int4 (&acc)[NV]) {
  const size_t off = static_cast<size_t>(row) * a.N * 8;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int c = (v * blockDim.x + threadIdx.x) * 4;
    acc[v] = make_int4(0, 0, 0, 0);
    if (c < a.N) acc[v] = ld_cg_i4(a.partial + static_cast<long long>(row) * a.ldp + c);
  }
  int cols[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) cols[v] = (v * blockDim.x + threadIdx.x) * 4;
  exchange_groups<NV>(a.p, off, cols, acc, a.N, e, ok);
}

template <int NV>
__global__ void __launch_bounds__(256) tp_allreduce_dequant_kernel(const ReduceArgs a) {
  __shared__ unsigned s_e;
  pdl_launch_dependents();
  pdl_wait();
  const unsigned e = peer_begin(a.p, &s_e);
  bool ok = true;
  for (int row = blockIdx.x; row < a.M; row += gridDim.x) {
    int4 acc[NV];
    reduce_row<NV>(a, row, e, ok, acc);
    const float sa = a.sa_per_row ? a.sa[row] : a.sa[0];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int c = (v * blockDim.x + threadIdx.x) * 4;
      if (c >= a.N) continue;
      const int q[4] = {acc[v].x, acc[v].y, acc[v].z, acc[v].w};
      for (int i = 0; i < 4; ++i) {
        const float val = dequant_one(q[i], sa, a, c + i);
        const long long o = static_cast<long long>(row) * a.ldo + c + i;
        if (a.out_dtype == I8L_BF16)
          static_cast<__nv_bfloat16 *>(a.out)[o] = __float2bfloat16_rn(val);
        else if (a.out_dtype == I8L_F16)
          static_cast<__half *>(a.out)[o] = __float2half_rn(val);
        else
          static_cast<float *>(a.out)[o] = val;
      }
    }
  }
  peer_end(a.p, e);
}

// ------------------------------------------------------------------ all-reduce + norm

struct ReduceNormArgs {
  ReduceArgs r;         // out_dtype = activation dtype; out unused
  const void *res;      // residual [M, N], may be NULL
  long long ldr;
  const void *w;        // norm weight [N]
  int w_dtype;
  int8_t *q;
  long long ldq;
  float *scale;
  void *rout;           // residual out [M, N] (with res)
  long long ldro;
  void *h_out;          // optional: the dequantised layer output [M, N]
  long long ldh;
  float eps;
  int precise;
  int w_vec;  // the norm weight pointer allows 16-byte loads
};

// Row thread layout of the norm kernel (add_rmsnorm_quant_kernel with VW = 8): thread t
// owns 8-column vectors (v*blockDim + t)*8.  The all-reduce works on 4-column groups,
// so a thread owns groups 2*(v*blockDim + t) and 2*(v*blockDim + t) + 1.  With the same
// blockDim and NV as the norm kernel, the sum of squares is accumulated in the same
// order, so the result equals dequant followed by add_rmsnorm_quant bit for bit.
template <int DT, int NV>
__global__ void __launch_bounds__(row_max_threads(NV, 8)) tp_allreduce_norm_kernel(const ReduceNormArgs a) {
  using T = typename ActType<DT>::T;
  __shared__ unsigned s_e;
  __shared__ float red[32], red2[32];
  pdl_launch_dependents();
  pdl_wait();
  const ReduceArgs &ra = a.r;
  const PeerArgs &p = ra.p;
  const unsigned e = peer_begin(p, &s_e);
  const int N = ra.N;
  bool ok = true;
  for (int row = blockIdx.x; row < ra.M; row += gridDim.x) {
    // 1. exchange: this thread's 8-column vectors as pairs of 4-column groups
    const size_t off = static_cast<size_t>(row) * N * 8;
    int4 acc[NV][2];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int c = col_of<8>(v);
      acc[v][0] = acc[v][1] = make_int4(0, 0, 0, 0);
      if (c < N) {
        const int *src = ra.partial + static_cast<long long>(row) * ra.ldp + c;
        acc[v][0] = ld_cg_i4(src);
        acc[v][1] = ld_cg_i4(src + 4);
      }
    }
    {
      int cols[2 * NV];
      int4 grp[2 * NV];
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int c = col_of<8>(v);
        cols[2 * v] = c < N ? c : N;
        cols[2 * v + 1] = c < N ? c + 4 : N;
        grp[2 * v] = acc[v][0];
        grp[2 * v + 1] = acc[v][1];
      }
      exchange_groups<2 * NV>(p, off, cols, grp, N, e, ok);
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        acc[v][0] = grp[2 * v];
        acc[v][1] = grp[2 * v + 1];
      }
    }
    // 2. dequant to the activation dtype (the layer output h), + residual, RMSNorm
    const float sa = ra.sa_per_row ? ra.sa[row] : ra.sa[0];
    float x[NV][8], wv[NV][8];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int c = col_of<8>(v);
      if (c < N) {
        load_weight_vec<8>(a.w, a.w_dtype, c, a.w_vec != 0, wv[v]);
        const int q[8] = {acc[v][0].x, acc[v][0].y, acc[v][0].z, acc[v][0].w,
                          acc[v][1].x, acc[v][1].y, acc[v][1].z, acc[v][1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) x[v][i] = round_through<DT>(dequant_one(q[i], sa, ra, c + i));
        if (a.h_out) store_vec<DT, 8>(static_cast<T *>(a.h_out) + row * a.ldh, c, x[v]);
        if (a.res) {
          float rr[8];
          load_vec<DT, 8>(static_cast<const T *>(a.res) + row * a.ldr, c, rr);
#pragma unroll
          for (int i = 0; i < 8; ++i) x[v][i] = __fadd_rn(x[v][i], rr[i]);
          store_vec<DT, 8>(static_cast<T *>(a.rout) + row * a.ldro, c, x[v]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[v][i] = 0.f;
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(x[v][i], x[v][i]));
    ss = block_sum(ss, red);
    const float var = div_full(ss, static_cast<float>(N));
    const float rs = rsqrtf(__fadd_rn(var, a.eps));
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int c = col_of<8>(v);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (c < N) {
          const float xn = round_to_weight(__fmul_rn(x[v][i], rs), a.w_dtype);
          x[v][i] = round_through<DT>(__fmul_rn(xn, wv[v][i]));
        }
      }
    }
    quantize_row<NV, 8>(x, N, a.q + row * a.ldq, a.scale + row, a.precise, red2);
    __syncthreads();  // `red` and `red2` are reused by the next row
  }
  peer_end(p, e);
}

// ------------------------------------------------------------------ split-row quantisers

// Exchange this row's local absmax for the global one (MAX over the GPUs): thread 0
// sends one 16-byte word {amax, e, amax, e} to every peer, thread r < world reads peer
// r's word; the result lands in *smem_amax for the whole CTA.
__device__ __forceinline__ float global_absmax(const PeerArgs &p, int row, unsigned e, float local,
                                               bool &ok, float *smem_amax, float *smem_part) {
  const unsigned par = e & 1u;
  const size_t off = static_cast<size_t>(row) * 16;
  const unsigned bits = __float_as_uint(local);
  if (threadIdx.x == 0)
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank) st_ll(inbox(p, r, par, p.rank) + off, bits, bits, e);
  const int src = threadIdx.x;
  if (src < p.world) {
    float v = local;
    if (src != p.rank) v = __uint_as_float(wait_ll(p, inbox(p, p.rank, par, src) + off, e, ok).x);
    smem_part[src] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = smem_part[0];
    for (int r = 1; r < p.world; ++r) m = fmaxf(m, smem_part[r]);
    *smem_amax = m;
  }
  __syncthreads();
  return *smem_amax;
}

struct SplitQuantArgs {
  PeerArgs p;
  const void *x;   // plain: x [M, K]; silu: gate||up [M, 2K] (this GPU's gate and up slices)
  long long ldx;
  int8_t *q;
  long long ldq;
  float *scale;
  int M, K;
  int precise;
  int round_silu;
};

template <int DT, int NV, int VW, bool kSilu>
__global__ void __launch_bounds__(row_max_threads(NV, VW)) tp_split_quant_kernel(const SplitQuantArgs a) {
  using T = typename ActType<DT>::T;
  __shared__ unsigned s_e;
  __shared__ float s_amax;
  __shared__ float s_part[kMaxRanks];
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const unsigned e = peer_begin(a.p, &s_e);
  bool ok = true;
  for (int row = blockIdx.x; row < a.M; row += gridDim.x) {
    const T *xrow = static_cast<const T *>(a.x) + row * a.ldx;
    float y[NV][VW];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int col = col_of<VW>(v);
      if (col < a.K) {
        if constexpr (kSilu) {
          float g[VW], u[VW];
          load_vec<DT, VW>(xrow, col, g);
          load_vec<DT, VW>(xrow + a.K, col, u);
#pragma unroll
          for (int i = 0; i < VW; ++i) {
            float s = div_full(g[i], __fadd_rn(1.0f, expf(-g[i])));
            if (a.round_silu) s = round_through<DT>(s);
            y[v][i] = round_through<DT>(__fmul_rn(s, u[i]));
          }
        } else {
          load_vec<DT, VW>(xrow, col, y[v]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < VW; ++i) y[v][i] = 0.f;
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int i = 0; i < VW; ++i) amax = fmaxf(amax, fabsf(y[v][i]));
    amax = block_max(amax, red);
    const float m = global_absmax(a.p, row, e, amax, ok, &s_amax, s_part);
    if (threadIdx.x == 0) a.scale[row] = a.precise ? div_rn(m, 127.f) : div_full(m, 127.f);
    const float inv = m == 0.f ? 0.f : (a.precise ? div_rn(127.f, m) : div_full(127.f, m));
    quantize_vals<NV, VW>(y, a.K, a.q + row * a.ldq, inv);
    __syncthreads();  // `red`, `s_part` and `s_amax` are reused by the next row
  }
  peer_end(a.p, e);
}

// ------------------------------------------------------------------ host side

static int peer_args(const i8l_peer_comm *c, PeerArgs *p, int rows, long long row_bytes) {
  if (!c) return set_error(I8L_EINVAL, "NULL peer communicator");
  if (c->world < 1 || c->world > kMaxRanks || c->rank < 0 || c->rank >= c->world)
    return set_error(I8L_EINVAL, "rank %d / world %d outside [0, %d)", c->rank, c->world, kMaxRanks);
  if (!c->epochs) return set_error(I8L_EINVAL, "peer communicator without epoch counters");
  for (int r = 0; r < c->world; ++r)
    if (!c->bases[r]) return set_error(I8L_EINVAL, "peer communicator: buffer of rank %d missing", r);
  if (rows > c->max_rows)
    return set_error(I8L_ENOTSUP, "%d rows exceed the exchange buffer's %d", rows, c->max_rows);
  if (static_cast<long long>(rows) * row_bytes > c->slot_bytes)
    return set_error(I8L_ENOTSUP, "%lld bytes per source exceed the exchange slot of %lld",
                     static_cast<long long>(rows) * row_bytes, static_cast<long long>(c->slot_bytes));
  *p = PeerArgs{};
  for (int r = 0; r < c->world; ++r) p->base[r] = static_cast<uint8_t *>(c->bases[r]);
  p->epochs = c->epochs;
  p->status = status_ptr();
  if (!p->status) return set_error(I8L_ECUDA, "device status word unavailable");
  p->rank = c->rank;
  p->world = c->world;
  p->slot_bytes = c->slot_bytes;
  p->max_rows = c->max_rows;
  p->timeout_ns = c->timeout_ns ? c->timeout_ns : kWaitLimitNs;
  return I8L_OK;
}

// Whether a row-parallel exchange of M rows of N int32 runs two-shot (the comm's
// two_shot_rows; 0 = from 16 rows with 4 or more GPUs: on 4 B200s the TP stand-in took
// 41.8 / 59.3 / 98.0 / 146.9 µs per layer one-shot and 45.2 / 56.6 / 72.5 / 94.7 two-shot
// at 1 / 16 / 64 / 128 rows).
static void set_two_shot(const i8l_peer_comm *c, PeerArgs *p, int M, int N) {
  const int rows = c->two_shot_rows == 0 ? (c->world >= 4 ? 16 : -1) : c->two_shot_rows;
  p->two_shot = (rows > 0 && M >= rows && c->world > 1 && N % (4 * c->world) == 0) ? 1 : 0;
}

// CTAs: one per row up to the SM count (all resident at once; see the file comment),
// and never more than the epoch counters the communicator holds.
static int peer_grid(const i8l_peer_comm *c, int M) {
  DeviceInfo di;
  const int sms = device_info(&di) == I8L_OK ? di.sms : 148;
  return std::max(1, std::min({M, sms, c->max_rows}));
}

static int finish(cudaError_t err, const char *what) {
  if (err != cudaSuccess) return cuda_error(err, what);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  return I8L_OK;
}

}  // namespace i8l

using namespace i8l;

extern "C" size_t i8l_peer_buffer_bytes(int64_t slot_bytes, int32_t world) {
  if (slot_bytes <= 0 || slot_bytes % 16 || world < 1 || world > kMaxRanks) return 0;
  return 2ull * static_cast<size_t>(world) * static_cast<size_t>(slot_bytes);
}

extern "C" int i8l_peer_alloc(size_t bytes, void **ptr, void *handle_out) {
  if (!ptr || !handle_out || bytes == 0) return set_error(I8L_EINVAL, "bad i8l_peer_alloc arguments");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(exchange buffer)");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_error(e, "exchange buffer set-up");
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return I8L_OK;
}

extern "C" int i8l_peer_open(const void *handle, void **ptr) {
  if (!handle || !ptr) return set_error(I8L_EINVAL, "bad i8l_peer_open arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_error(e, "cudaIpcOpenMemHandle(peer exchange buffer)");
  *ptr = p;
  return I8L_OK;
}

extern "C" int i8l_peer_close(void *ptr) {
  if (!ptr) return I8L_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? I8L_OK : cuda_error(e, "cudaIpcCloseMemHandle");
}

extern "C" int i8l_peer_free(void *ptr) {
  if (!ptr) return I8L_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? I8L_OK : cuda_error(e, "cudaFree(exchange buffer)");
}

extern "C" int i8l_tp_allreduce_dequant(const i8l_peer_comm *comm, const int32_t *partial,
                                        int64_t ldp, const float *sa, int32_t sa_per_row,
                                        const float *sb, int32_t sb_per_col, const void *bias,
                                        int32_t bias_dtype, void *out, int32_t out_dtype,
                                        int64_t ldo, int32_t M, int32_t N, void *stream) {
  if (M < 0 || N < 0) return set_error(I8L_EINVAL, "bad size M=%d N=%d", M, N);
  if (M == 0 || N == 0) return I8L_OK;
  if (!partial || !sa || !sb || !out) return set_error(I8L_EINVAL, "NULL pointer argument");
  if (out_dtype < I8L_BF16 || out_dtype > I8L_F32)
    return set_error(I8L_ENOTSUP, "output dtype code %d not supported", out_dtype);
  if (bias && (bias_dtype < I8L_BF16 || bias_dtype > I8L_F32))
    return set_error(I8L_ENOTSUP, "bias dtype code %d not supported", bias_dtype);
  if (ldp < N || ldo < N) return set_error(I8L_EINVAL, "row stride smaller than N");
  if (N % 4 || ldp % 4 || reinterpret_cast<uintptr_t>(partial) % 16)
    return set_error(I8L_ENOTSUP, "the exchange moves 16-byte groups: N and ldp must be multiples of 4");
  ReduceArgs a{};
  int e = peer_args(comm, &a.p, M, static_cast<long long>(N) * 8);
  if (e) return e;
  set_two_shot(comm, &a.p, M, N);
  a.partial = partial;
  a.ldp = ldp;
  a.sa = sa;
  a.sa_per_row = sa_per_row;
  a.sb = sb;
  a.sb_per_col = sb_per_col;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  a.ldo = ldo;
  a.M = M;
  a.N = N;
  const int groups = (N + 3) / 4;
  const int nv = (groups + 255) / 256;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(peer_grid(comm, M));
  cudaError_t err;
  switch (nv) {
    case 1: err = launch(tp_allreduce_dequant_kernel<1>, grid, dim3(256), 0, s, 1, a); break;
    case 2: err = launch(tp_allreduce_dequant_kernel<2>, grid, dim3(256), 0, s, 1, a); break;
    case 3: err = launch(tp_allreduce_dequant_kernel<3>, grid, dim3(256), 0, s, 1, a); break;
    case 4: err = launch(tp_allreduce_dequant_kernel<4>, grid, dim3(256), 0, s, 1, a); break;
    case 5: case 6: case 7: case 8:
      err = launch(tp_allreduce_dequant_kernel<8>, grid, dim3(256), 0, s, 1, a); break;
    default:
      return set_error(I8L_ENOTSUP, "rows of %d values exceed the exchange kernel's 8192", N);
  }
  return finish(err, "tp_allreduce_dequant launch");
}

extern "C" int i8l_tp_allreduce_add_rmsnorm_quant(
    const i8l_peer_comm *comm, const int32_t *partial, int64_t ldp, const float *sa,
    int32_t sa_per_row, const float *sb, int32_t sb_per_col, const void *bias, int32_t bias_dtype,
    const void *residual, int64_t ldr, const void *weight, int32_t act_dtype, int32_t w_dtype,
    int8_t *q, int64_t ldq, float *scale, void *rout, int64_t ldro, void *h_out, int64_t ldh,
    int32_t M, int32_t N, float eps, int32_t precise_div, void *stream) {
  if (M < 0 || N <= 0) return set_error(I8L_EINVAL, "bad size M=%d N=%d", M, N);
  if (M == 0) return I8L_OK;
  if (act_dtype != I8L_BF16 && act_dtype != I8L_F16)
    return set_error(I8L_ENOTSUP, "activation dtype code %d not supported (bf16 or fp16)", act_dtype);
  if (w_dtype < I8L_BF16 || w_dtype > I8L_F32)
    return set_error(I8L_ENOTSUP, "weight dtype code %d not supported", w_dtype);
  if (bias && (bias_dtype < I8L_BF16 || bias_dtype > I8L_F32))
    return set_error(I8L_ENOTSUP, "bias dtype code %d not supported", bias_dtype);
  if (!partial || !sa || !sb || !weight || !q || !scale)
    return set_error(I8L_EINVAL, "NULL pointer argument");
  if ((residual == nullptr) != (rout == nullptr))
    return set_error(I8L_EINVAL, "residual and residual_out must be given together");
  if (ldp < N || ldq < N || (residual && (ldr < N || ldro < N)) || (h_out && ldh < N))
    return set_error(I8L_EINVAL, "row stride smaller than N");
  // The fused kernel takes the norm kernel's vector layout (8 values per thread-vector).
  const bool vec = N % 8 == 0 && ldp % 4 == 0 && ldq % 8 == 0 && aligned16(partial) && aligned16(q) &&
                   (!residual || (ldr % 8 == 0 && ldro % 8 == 0 && aligned16(residual) && aligned16(rout))) &&
                   (!h_out || (ldh % 8 == 0 && aligned16(h_out)));
  RowShape rs;
  if (!vec || !row_shape(N, 8, &rs))
    return set_error(I8L_ENOTSUP, "fused exchange + norm needs N %% 8 == 0, 16-byte aligned rows, N <= 32768");
  ReduceNormArgs a{};
  int e = peer_args(comm, &a.r.p, M, static_cast<long long>(N) * 8);
  if (e) return e;
  set_two_shot(comm, &a.r.p, M, N);
  a.r.partial = partial;
  a.r.ldp = ldp;
  a.r.sa = sa;
  a.r.sa_per_row = sa_per_row;
  a.r.sb = sb;
  a.r.sb_per_col = sb_per_col;
  a.r.bias = bias;
  a.r.bias_dtype = bias_dtype;
  a.r.out_dtype = act_dtype;
  a.r.M = M;
  a.r.N = N;
  a.res = residual;
  a.ldr = ldr;
  a.w = weight;
  a.w_dtype = w_dtype;
  a.q = q;
  a.ldq = ldq;
  a.scale = scale;
  a.rout = rout;
  a.ldro = ldro;
  a.h_out = h_out;
  a.ldh = ldh;
  a.eps = eps;
  a.precise = precise_div;
  a.w_vec = aligned16(weight) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(peer_grid(comm, M));
  const int nv = rs.nv, th = rs.threads;
  cudaError_t err = cudaSuccess;
  if (act_dtype == I8L_BF16) {
    I8L_DISPATCH_NV(nv, (err = launch(tp_allreduce_norm_kernel<I8L_BF16, NV>, grid, dim3(th), 0, s, 1, a)))
  } else {
    I8L_DISPATCH_NV(nv, (err = launch(tp_allreduce_norm_kernel<I8L_F16, NV>, grid, dim3(th), 0, s, 1, a)))
  }
  return finish(err, "tp_allreduce_add_rmsnorm_quant launch");
}

template <bool kSilu>
static int split_quant(const i8l_peer_comm *comm, const void *x, int64_t ldx, int32_t act_dtype,
                       int8_t *q, int64_t ldq, float *scale, int32_t M, int32_t K, int32_t precise_div,
                       int32_t round_silu, void *stream) {
  if (act_dtype != I8L_BF16 && act_dtype != I8L_F16)
    return set_error(I8L_ENOTSUP, "activation dtype code %d not supported (bf16 or fp16)", act_dtype);
  if (M < 0 || K <= 0) return set_error(I8L_EINVAL, "bad size M=%d K=%d", M, K);
  if (M == 0) return I8L_OK;
  if (!x || !q || !scale) return set_error(I8L_EINVAL, "NULL pointer argument");
  if (ldx < (kSilu ? 2LL * K : K) || ldq < K) return set_error(I8L_EINVAL, "row stride too small");
  SplitQuantArgs a{};
  int e = peer_args(comm, &a.p, M, 16);
  if (e) return e;
  a.x = x;
  a.ldx = ldx;
  a.q = q;
  a.ldq = ldq;
  a.scale = scale;
  a.M = M;
  a.K = K;
  a.precise = precise_div;
  a.round_silu = round_silu;
  // The same thread layout as the one-GPU quantisers (so the code paths agree).
  const bool vec = K % 8 == 0 && ldx % 8 == 0 && ldq % 8 == 0 && aligned16(x) && aligned16(q);
  RowShape rs;
  if (!row_shape(K, vec ? 8 : 1, &rs, row_threads(M)))
    return set_error(I8L_ENOTSUP, "row of %d values is too long", K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(peer_grid(comm, M));
  const int nv = rs.nv, th = rs.threads;
  cudaError_t err = cudaSuccess;
  if (act_dtype == I8L_BF16) {
    if (vec) {
      I8L_DISPATCH_NV(nv, (err = launch(tp_split_quant_kernel<I8L_BF16, NV, 8, kSilu>, grid, dim3(th), 0, s, 1, a)))
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(tp_split_quant_kernel<I8L_BF16, NV, 1, kSilu>, grid, dim3(th), 0, s, 1, a)))
    }
  } else {
    if (vec) {
      I8L_DISPATCH_NV(nv, (err = launch(tp_split_quant_kernel<I8L_F16, NV, 8, kSilu>, grid, dim3(th), 0, s, 1, a)))
    } else {
      I8L_DISPATCH_NV(nv, (err = launch(tp_split_quant_kernel<I8L_F16, NV, 1, kSilu>, grid, dim3(th), 0, s, 1, a)))
    }
  }
  return finish(err, kSilu ? "tp_silu_mul_quant launch" : "tp_quant_rows launch");
}

extern "C" int i8l_tp_quant_rows(const i8l_peer_comm *comm, const void *x, int64_t ldx,
                                 int32_t act_dtype, int8_t *q, int64_t ldq, float *scale, int32_t M,
                                 int32_t K, int32_t precise_div, void *stream) {
  return split_quant<false>(comm, x, ldx, act_dtype, q, ldq, scale, M, K, precise_div, 0, stream);
}

extern "C" int i8l_tp_silu_mul_quant(const i8l_peer_comm *comm, const void *gate_up, int64_t ld,
                                     int32_t act_dtype, int8_t *q, int64_t ldq, float *scale,
                                     int32_t M, int32_t I, int32_t precise_div, int32_t round_silu,
                                     void *stream) {
  return split_quant<true>(comm, gate_up, ld, act_dtype, q, ldq, scale, M, I, precise_div,
                           round_silu, stream);
}
