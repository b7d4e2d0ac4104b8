// W8A8 GEMM for sm_100a: int8 x int8 -> int32 on the tcgen05 tensor cores with
// the accumulator in TMEM, operands streamed by TMA through a shared-memory
// ring, and the dequantisation (x scale_a x scale_b + bias, rounded once to the
// output type) fused into the epilogue.
//
// Computes what the reference's Triton kernel _w8a8_mm computes
// (int8_linear/kernel.py:63-124 in AshrithaG/int8-linear):
//     out[m,n] = cast( ((float(acc[m,n]) * sa[m]) * sb[n]) + float(bias[n]) )
// with acc the exact int32 product, or acc itself when the output is int32.
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0  TMA producer  - one thread fills the stage ring (X tile 128x128 B,
//                           Y tile TNx128 B per stage, 128-byte swizzle);
//   warp 1  MMA issuer    - one thread issues tcgen05.mma.kind::i8 (M=128, N=TN,
//                           K=32) into one of two TMEM accumulators;
//   warps 2-5 epilogue    - tcgen05.ld the accumulator, dequantise and store, or
//                           add a partial sum into the int32 workspace.
// X is the operand on the 128-row MMA side, Y the TN-row side.  For decode
// shapes the weight is X (swap_ab: each tile is 128 output columns by TN
// tokens); for prefill shapes the activation is X.
//
// Work split: the (tile, k-block) iteration space is divided among the CTAs.
// Whole tiles go round-robin (the library's choice for prefill and for decode tiles
// that fill the SMs); cluster split-K shares one tile's k-blocks among the CTAs of a
// thread-block cluster (decode tiles on few tiles, reduced over distributed shared
// memory, see the epilogue).  On request (split 2, stream-K) the tail (the last
// partial wave plus one full wave) is divided into equal contiguous k-block ranges,
// so some tiles are computed in pieces by several CTAs.  Each piece adds its int32
// partial sums into a workspace slot with red.add and counts its k-blocks on the
// slot's counter; the CTA whose count completes the tile reads the slot, runs
// the epilogue and zeroes the slot again.  Integer addition is exact and
// order-free, so the result does not depend on which CTA finishes last, and no
// CTA ever waits on another.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"

namespace i8l {

constexpr int kBK = 128;        // K bytes per stage: one 128-byte swizzle row
constexpr int kXRows = 128;     // MMA M
constexpr int kThreads = 192;   // 6 warps
constexpr int kEpiWarps = 4;

struct GemmArgs {
  int M, N, K;
  int tiles_x, tiles_y, kblocks;
  int total_tiles, dp_tiles;
  long long sk_iters;
  int group;
  int stages;
  int swap;
  const float *sa;
  const float *sb;
  int sa_per_row, sb_per_col;
  const void *bias;
  int bias_dtype;
  void *out;
  int out_dtype;
  long long ldc;
  int vec_store;  // direct-store fallback: 16-byte vector stores allowed
  int tma_out;    // output written through shared memory by TMA stores
  int *ws;        // workspace slots, 128*TN int32 each ([TN][128] per slot)
  int *counters;  // one k-block counter per slot
  int *status;
  int cluster;    // >1: the CTAs of each cluster split K of one tile (reduced over DSMEM)
  // Partial sums are received in the staging area (free from the start with plain
  // stores), so senders push as soon as their own MMAs are done; else in the
  // receiver's operand ring once its MMAs are done and it has said so.
  int cluster_early;
  // Direct activation loads (swap tiles holding every token, one segment per CTA whose
  // k-blocks all fit in the ring): the epilogue warps copy A's k-blocks into the ring's
  // Y slots with plain loads after the dependency wait, so the activation never queues
  // in the SM's TMA unit behind weight prefetches; the producer loads only weights.
  int act_direct;
  const int8_t *act;
  long long lda;
  // Per-token quantisation fused into the direct activation loads: act_src holds the
  // bf16/fp16 activation (act_src_dtype, rows act_ld elements apart); the loader finds
  // each token's absmax over all K, quantises its k-blocks as the row quantiser does
  // (scale = absmax/127, q = rint(x * 127/absmax)), and the epilogue uses those scales.
  int act_quant;
  int act_src_dtype;
  int act_precise;
  const void *act_src;
  long long act_ld;
  // CTA pairs (cta_group::2): the two CTAs of each 2-CTA cluster compute one tile of
  // 256 X rows (tiles_x counts 256-row tiles) x TN Y rows; each loads 128 X rows and
  // TN/2 Y rows per k-block, the even CTA issues the 256-row MMAs.  Whole tiles only.
  int pair;
};

struct Segment {
  int tile;
  int kb0, kb1;
};

// The deterministic sequence of (tile, k-range) segments one CTA processes.
// Producer, MMA issuer and epilogue each walk their own copy.
struct Schedule {
  int dp_next;
  long long it, it_end;

  // Each role initialises its copy before the dependency wait: the divisions here
  // (64-bit ones for stream-K) then overlap the previous kernel instead of delaying
  // the first load after the wait.
  __device__ __forceinline__ void init(const GemmArgs &a) {
    if (a.pair) {  // both CTAs of a pair walk the same tiles
      dp_next = static_cast<int>(blockIdx.x) >> 1;
      it = it_end = 0;
      return;
    }
    if (a.cluster > 1) {
      // One tile per cluster; CTA rank r takes the r-th of `cluster` equal k ranges.
      const int r = static_cast<int>(blockIdx.x) % a.cluster;
      dp_next = static_cast<int>(blockIdx.x) / a.cluster;
      it = a.kblocks * r / a.cluster;
      it_end = a.kblocks * (r + 1) / a.cluster;
      return;
    }
    dp_next = blockIdx.x;
    if (a.sk_iters == 0) {
      it = it_end = 0;
      return;
    }
    const long long g = gridDim.x;
    it = a.sk_iters * static_cast<long long>(blockIdx.x) / g;
    it_end = a.sk_iters * static_cast<long long>(blockIdx.x + 1) / g;
  }

  __device__ __forceinline__ bool next(const GemmArgs &a, Segment &s) {
    if (a.pair) {
      if (dp_next >= a.total_tiles) return false;
      s.tile = dp_next;
      s.kb0 = 0;
      s.kb1 = a.kblocks;
      dp_next += static_cast<int>(gridDim.x) >> 1;
      return true;
    }
    if (a.cluster > 1) {
      if (dp_next < 0) return false;
      s.tile = dp_next;
      s.kb0 = static_cast<int>(it);
      s.kb1 = static_cast<int>(it_end);
      dp_next = -1;
      return true;
    }
    if (dp_next < a.dp_tiles) {
      s.tile = dp_next;
      s.kb0 = 0;
      s.kb1 = a.kblocks;
      dp_next += gridDim.x;
      return true;
    }
    if (it < it_end) {
      const long long t = it / a.kblocks;
      const int kb0 = static_cast<int>(it - t * a.kblocks);
      const long long left = it_end - it;
      const int kb1 = static_cast<int>(
          left < static_cast<long long>(a.kblocks - kb0) ? kb0 + left : a.kblocks);
      s.tile = a.dp_tiles + static_cast<int>(t);
      s.kb0 = kb0;
      s.kb1 = kb1;
      it += kb1 - kb0;
      return true;
    }
    return false;
  }
};

// Workspace slot of a stream-K tile that is split: one less than the first CTA
// whose range starts strictly inside the tile.  Distinct split tiles get
// distinct slots in [0, gridDim.x - 1).
__device__ __forceinline__ int split_slot(const GemmArgs &a, int tile) {
  const long long s = tile - a.dp_tiles;
  const long long g = gridDim.x;
  const long long num = (s * a.kblocks + 1) * g;
  const long long b = (num + a.sk_iters - 1) / a.sk_iters;
  return static_cast<int>(b - 1);
}

// Tile index -> (x tile, y tile), walking `group` x tiles together so CTAs that
// run at the same time share Y tiles in L2.
__device__ __forceinline__ void tile_coords(const GemmArgs &a, int t, int &tx,
                                            int &ty) {
  if (a.tiles_y == 1) {  // one Y tile (a decode batch): no divisions
    tx = t;
    ty = 0;
    return;
  }
  const int per_group = a.group * a.tiles_y;
  const int g = t / per_group;
  const int first = g * a.group;
  const int gsz = min(a.tiles_x - first, a.group);
  const int r = t - g * per_group;
  tx = first + r % gsz;
  ty = r / gsz;
}

// This CTA's (x tile, y tile): with CTA pairs the 256-row x tile of the pair is split
// into the two CTAs' 128-row halves.
__device__ __forceinline__ void cta_tile(const GemmArgs &a, int t, int &tx, int &ty) {
  tile_coords(a, t, tx, ty);
  if (a.pair) tx = 2 * tx + static_cast<int>(blockIdx.x & 1u);
}

// Everything one epilogue thread needs about the current tile.
struct TileCtx {
  int tx, ty, ncols;
  uint32_t taddr;     // TMEM address of this warp's lanes in the accumulator
  const float *s_col; // per accumulator column: sb (normal) or sa (swap), smem
  const float *b_col; // per accumulator column: bias (normal), smem
  float s_row, b_row; // per TMEM lane: sa (normal) or sb, bias (swap)
};

// 16 consecutive per-column floats of the tile context (shared memory, 16-byte
// aligned) into registers.  Loaded before any output is written: the compiler cannot
// tell the output stores from these loads, so loads left between the stores would wait
// for each one in turn (measured: ~1100 cycles per 16 values, against ~100).
__device__ __forceinline__ void load16(const float *p, float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 f = reinterpret_cast<const float4 *>(p)[q];
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
}

// Storage bits (16-bit outputs in the low half) of the 16 values of this thread's TMEM
// lane, columns c0..c0+15 of a swap_ab tile: token scales per column, weight scale and
// bias per lane.
__device__ __forceinline__ void out_bits16x(const GemmArgs &a, const TileCtx &t, int c0, const uint32_t (&r)[16],
                                            uint32_t (&bits)[16]) {
  const bool has_bias = a.bias != nullptr;
  float sa[16];
  load16(t.s_col + c0, sa);
  const bool wide = a.out_dtype == I8L_BF16 || a.out_dtype == I8L_F16;
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const int a0 = static_cast<int>(r[j]), a1 = static_cast<int>(r[j + 1]);
    const float v0 = dequant(a0, sa[j], t.s_row, t.b_row, has_bias);
    const float v1 = dequant(a1, sa[j + 1], t.s_row, t.b_row, has_bias);
    if (wide) {
      const uint32_t p = pack16x2(a.out_dtype, v0, v1);
      bits[j] = p & 0xffffu;
      bits[j + 1] = p >> 16;
    } else {
      bits[j] = out_bits32(a.out_dtype, a0, v0);
      bits[j + 1] = out_bits32(a.out_dtype, a1, v1);
    }
  }
}

// Plain stores of the 16 values of this thread's TMEM lane, columns c0..c0+15 (output
// not TMA-addressable, or few output rows).  The scales and bias come from the tile
// context, fetched before the accumulator was ready; every value is computed before the
// first store.
template <int TN>
__device__ __forceinline__ void epilogue_direct(const GemmArgs &a, const TileCtx &t, int row,
                                                int c0, const uint32_t (&r)[16]) {
  uint32_t bits[16];
  const bool wide = a.out_dtype == I8L_BF16 || a.out_dtype == I8L_F16;
  if (a.swap) {
    const int n = t.tx * kXRows + row;
    if (n >= a.N) return;
    const int m0 = t.ty * TN + c0;
    out_bits16x(a, t, c0, r, bits);
    const long long ldc = a.ldc;
    const long long base = static_cast<long long>(m0) * ldc + n;
    const int live = min(16, a.M - m0);
    if (wide) {
      uint16_t *o = static_cast<uint16_t *>(a.out) + base;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < live) o[j * ldc] = static_cast<uint16_t>(bits[j]);
    } else {
      uint32_t *o = static_cast<uint32_t *>(a.out) + base;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < live) o[j * ldc] = bits[j];
    }
  } else {
    const int m = t.tx * kXRows + row;
    if (m >= a.M) return;
    const int n0 = t.ty * TN + c0;
    const bool has_bias = a.bias != nullptr;
    float sb[16], bias[16];
    load16(t.s_col + c0, sb);
    load16(t.b_col + c0, bias);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const int a0 = static_cast<int>(r[j]), a1 = static_cast<int>(r[j + 1]);
      const float v0 = dequant(a0, t.s_row, sb[j], bias[j], has_bias);
      const float v1 = dequant(a1, t.s_row, sb[j + 1], bias[j + 1], has_bias);
      if (wide) {
        const uint32_t p = pack16x2(a.out_dtype, v0, v1);
        bits[j] = p & 0xffffu;
        bits[j + 1] = p >> 16;
      } else {
        bits[j] = out_bits32(a.out_dtype, a0, v0);
        bits[j + 1] = out_bits32(a.out_dtype, a1, v1);
      }
    }
    const long long base = static_cast<long long>(m) * a.ldc + n0;
    const int live = min(16, a.N - n0);
    if (wide) {
      uint16_t *o = static_cast<uint16_t *>(a.out) + base;
      if (a.vec_store && live == 16) {  // 32 bytes of one row: two 16-byte stores
        uint4 *v = reinterpret_cast<uint4 *>(o);
        v[0] = make_uint4(bits[0] | (bits[1] << 16), bits[2] | (bits[3] << 16), bits[4] | (bits[5] << 16),
                          bits[6] | (bits[7] << 16));
        v[1] = make_uint4(bits[8] | (bits[9] << 16), bits[10] | (bits[11] << 16),
                          bits[12] | (bits[13] << 16), bits[14] | (bits[15] << 16));
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < live) o[j] = static_cast<uint16_t>(bits[j]);
      }
    } else {
      uint32_t *o = static_cast<uint32_t *>(a.out) + base;
      if (a.vec_store && live == 16) {
        uint4 *v = reinterpret_cast<uint4 *>(o);
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = make_uint4(bits[4 * q], bits[4 * q + 1], bits[4 * q + 2], bits[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < live) o[j] = bits[j];
      }
    }
  }
}

// Narrow tiles: 8 consecutive outputs of token row m (tile columns c0..c0+7), dequantised
// (sa: the row's scale) and stored with one 16-byte store (32 bytes for 32-bit outputs)
// where the row allows.
template <int TN>
__device__ __forceinline__ void store_row8(const GemmArgs &a, const TileCtx &t, int m, int c0,
                                           float sa, const uint32_t (&r)[8]) {
  const bool raw = a.out_dtype == I8L_I32;
  const bool has_bias = a.bias != nullptr;
  const bool narrow16 = a.out_dtype == I8L_BF16 || a.out_dtype == I8L_F16;
  const int n0 = t.ty * TN + c0;
  const int nv = min(8, a.N - n0);
  uint32_t bits[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int acc = static_cast<int>(r[j]);
    const float v = raw ? 0.f : dequant(acc, sa, t.s_col[c0 + j], t.b_col[c0 + j], has_bias);
    bits[j] = narrow16 ? out_bits16(a.out_dtype, v) : out_bits32(a.out_dtype, acc, v);
  }
  const long long idx = static_cast<long long>(m) * a.ldc + n0;
  if (a.vec_store && nv == 8) {
    if (narrow16) {
      *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.out) + idx) =
          make_uint4(bits[0] | (bits[1] << 16), bits[2] | (bits[3] << 16), bits[4] | (bits[5] << 16),
                     bits[6] | (bits[7] << 16));
    } else {
      uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint32_t *>(a.out) + idx);
      p[0] = make_uint4(bits[0], bits[1], bits[2], bits[3]);
      p[1] = make_uint4(bits[4], bits[5], bits[6], bits[7]);
    }
    return;
  }
  for (int j = 0; j < nv; ++j) {
    if (narrow16)
      static_cast<uint16_t *>(a.out)[idx + j] = static_cast<uint16_t>(bits[j]);
    else
      static_cast<uint32_t *>(a.out)[idx + j] = bits[j];
  }
}

// Number of accumulator columns of a tile that hold real (in-range) Y rows.
template <int TN>
__device__ __forceinline__ int live_cols(const GemmArgs &a, int ty) {
  const int rows_y = a.swap ? a.M : a.N;
  return min(TN, rows_y - ty * TN);
}

__device__ __forceinline__ int ld_cg_s32(const int *p) {
  int v;
  asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 16 bytes from global memory through L2 only (never a stale L1 line).
__device__ __forceinline__ uint4 ld_cg_v4(const int8_t *p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_cg_s32(int *p, int v) {
  asm volatile("st.global.cg.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

constexpr int kStageBufBytes = 2048;                            // one staging buffer
constexpr int kStagingBytes = kEpiWarps * 2 * kStageBufBytes;   // 16 KB
constexpr int kScalFloats = 256;                                // per array per buffer
constexpr int kScalBytes = 2 * 2 * kScalFloats * 4;             // [2 arrays][2 acc][256]

// Kernel variants: 0 one CTA per tile; 1 CTA pairs (cta_group::2, 256-row tiles);
// 2 narrow (decode batches of <= 16 tokens with the weight on the N side: 64-row
// token tile, 256 weight rows per MMA, one accumulator so two CTAs share an SM).
constexpr int kVarOne = 0, kVarPair = 1, kVarNarrow = 2;

template <int TN, int kVar = kVarOne>
struct SmemLayout {
  static constexpr int kXRowsV = kVar == kVarNarrow ? 64 : kXRows;  // X rows per stage
  static constexpr int kXBytes = kXRowsV * kBK;
  static constexpr int kYRows = kVar == kVarPair ? TN / 2 : TN;     // Y rows this CTA holds
  static constexpr int kYBytes = kYRows * kBK;
  static constexpr int kStageBytes = kXBytes + kYBytes;
  // Decode tiles rotate their k-steps over several accumulators: a chain of
  // accumulating MMAs into the same columns runs one MMA at a time, and an N=16 MMA
  // is far too short to hide that latency.  The epilogue adds the chains (int32
  // addition is exact and order-free).  Two accumulators (double buffer) x chains.
  static constexpr int kChains = TN <= 16 ? 4 : (TN <= 64 ? 2 : 1);
  static constexpr int kAccCols = kChains * TN;
  // Narrow tiles keep one accumulator (one tile per CTA), so two CTAs fit an SM's TMEM.
  static constexpr int kAccBufs = kVar == kVarNarrow ? 1 : 2;
  static constexpr int kTmemCols = (kAccBufs * kAccCols < 32) ? 32 : kAccBufs * kAccCols;
  // stages | staging | scales | barriers: full[S], empty[S], acc_full[2],
  // acc_empty[2], drain, peer, done, act | tmem slot, flags
  static size_t bytes(int stages) {
    return 1024 /* alignment slack */ + static_cast<size_t>(stages) * kStageBytes +
           kStagingBytes + kScalBytes + static_cast<size_t>(2 * stages + 8) * 8 + 64;
  }
};

// Accumulator columns c..c+15 of this warp's TMEM lanes, summed over the k-step
// chains (chain j at taddr + j*TN).
template <int TN>
__device__ __forceinline__ void tmem_acc16(uint32_t taddr, int c, uint32_t (&r)[16]) {
  constexpr int kChains = SmemLayout<TN>::kChains;
  tmem_ld16(taddr + c, r);
  if constexpr (kChains > 1) {
    uint32_t q[kChains - 1][16];
#pragma unroll
    for (int j = 1; j < kChains; ++j) tmem_ld16(taddr + j * TN + c, q[j - 1]);
    tmem_ld_wait();
#pragma unroll
    for (int j = 1; j < kChains; ++j)
#pragma unroll
      for (int i = 0; i < 16; ++i) r[i] += q[j - 1][i];
  } else {
    tmem_ld_wait();
  }
}

// A warp's two 2 KB staging buffers for TMA stores / reduces; lane 0 owns the
// bulk groups.  acquire() returns a buffer no bulk operation still reads.
struct Staging {
  uint8_t *base;
  uint32_t count;

  __device__ __forceinline__ uint8_t *acquire(int lane) {
    if (count >= 2 && lane == 0) bulk_wait_read<1>();
    __syncwarp();
    uint8_t *b = base + (count & 1u) * kStageBufBytes;
    ++count;
    return b;
  }

  __device__ __forceinline__ void drain(int lane) {
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }
};

// Writes 16 values (columns c0..c0+15 of this thread's TMEM lane) through the
// staging buffer and a TMA store.  Swap: box {32 n, 16 m}.
template <int TN>
__device__ __forceinline__ void emit_swap16(const GemmArgs &a, const CUtensorMap *map_out,
                                            const TileCtx &t, int quarter, int lane, int c0,
                                            const uint32_t (&r)[16], Staging &st) {
  uint32_t bits[16];
  out_bits16x(a, t, c0, r, bits);
  uint8_t *buf = st.acquire(lane);
  if (a.out_dtype == I8L_BF16 || a.out_dtype == I8L_F16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) reinterpret_cast<uint16_t *>(buf)[j * 32 + lane] = static_cast<uint16_t>(bits[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) reinterpret_cast<uint32_t *>(buf)[j * 32 + lane] = bits[j];
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const int n0 = t.tx * kXRows + quarter * 32, m0 = t.ty * TN + c0;
    if (n0 < a.N && m0 < a.M) tma_store_2d(map_out, buf, n0, m0);  // skip boxes wholly outside
    bulk_commit();
  }
}

// Normal orientation: one 64-byte-per-row subtile (32 columns of a 16-bit
// output from r0 and r1, or 16 columns of a 32-bit output from r0), written
// with the 64-byte swizzle the output tensor map uses.  Box {cols, 32 m}.
template <int TN>
__device__ __forceinline__ void emit_normal(const GemmArgs &a, const CUtensorMap *map_out,
                                            const TileCtx &t, int quarter, int lane, int c0,
                                            const uint32_t (&r0)[16], const uint32_t (&r1)[16],
                                            Staging &st) {
  uint8_t *buf = st.acquire(lane);
  const bool raw = a.out_dtype == I8L_I32;
  const bool has_bias = a.bias != nullptr;
  uint32_t p[16];
  if (a.out_dtype == I8L_BF16 || a.out_dtype == I8L_F16) {
    // Column scales and bias by 16-byte loads; two outputs per conversion.
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float sb[16], bias[16];
      load16(t.s_col + c0 + 16 * h, sb);
      if (has_bias) load16(t.b_col + c0 + 16 * h, bias);
      const uint32_t (&r)[16] = h ? r1 : r0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v0 = dequant(static_cast<int>(r[2 * j]), t.s_row, sb[2 * j], has_bias ? bias[2 * j] : 0.f, has_bias);
        const float v1 =
            dequant(static_cast<int>(r[2 * j + 1]), t.s_row, sb[2 * j + 1], has_bias ? bias[2 * j + 1] : 0.f, has_bias);
        p[8 * h + j] = pack16x2(a.out_dtype, v0, v1);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int acc = static_cast<int>(r0[j]);
      const float v = raw ? 0.f : dequant(acc, t.s_row, t.s_col[c0 + j], t.b_col[c0 + j], has_bias);
      p[j] = out_bits32(a.out_dtype, acc, v);
    }
  }
  uint8_t *rowp = buf + lane * 64;
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4 *>(rowp + ((c ^ sw) << 4)) =
        make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const int n0 = t.ty * TN + c0, m0 = t.tx * kXRows + quarter * 32;
    if (n0 < a.N && m0 < a.M) tma_store_2d(map_out, buf, n0, m0);  // skip boxes wholly outside
    bulk_commit();
  }
}

// Direct activation loads: k-blocks kb0..kb1-1 of A (all TN token rows; rows past M
// and columns past K read as zero, as the TMA zero fill gives) into Y slots 0.. of
// the ring, each [TN rows][128 B] with the 128-byte swizzle of the TMA operand map
// (16-byte chunk c of row r at chunk c ^ (r & 7)).  Each thread issues up to eight
// 16-byte L2 loads before its first shared store, so their latencies overlap.
template <int TN>
__device__ __forceinline__ void load_act_direct(const GemmArgs &a, uint8_t *sy, int kb0, int kb1,
                                                int tid) {
  constexpr int kChunks = TN * (kBK / 16);
  constexpr int kThr = kEpiWarps * 32;
  const int n = (kb1 - kb0) * kChunks;
  for (int base = tid; base < n; base += 8 * kThr) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int id = base + u * kThr;
      v[u] = make_uint4(0u, 0u, 0u, 0u);
      if (id < n) {
        const int j = id / kChunks, r = (id % kChunks) >> 3, c = id & 7;
        const long long col = static_cast<long long>(kb0 + j) * kBK + c * 16;
        if (r < a.M && col < a.K) v[u] = ld_cg_v4(a.act + static_cast<long long>(r) * a.lda + col);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int id = base + u * kThr;
      if (id < n) {
        const int j = id / kChunks, r = (id % kChunks) >> 3, c = id & 7;
        *reinterpret_cast<uint4 *>(sy + static_cast<size_t>(j) * (TN * kBK) + r * kBK +
                                   ((c ^ (r & 7)) << 4)) = v[u];
      }
    }
  }
}

// Value j (0..7) of 8 bf16 or fp16 values packed in a uint4, as float (exact).
__device__ __forceinline__ float act_val(const uint4 &v, int j, int f16) {
  const uint32_t w = (&v.x)[j >> 1];
  const uint32_t h = (j & 1) ? (w >> 16) : (w & 0xffffu);
  return f16 ? __half2float(__ushort_as_half(static_cast<unsigned short>(h))) : __uint_as_float(h << 16);
}

// Direct activation loads with per-token quantisation (a.act_quant): first each token
// row's absmax over all K (all epilogue threads, 32-byte units), giving its scale and
// reciprocal exactly as the row quantiser computes them (scale = absmax/127, inv =
// 127/absmax or 0, by IEEE or Triton's full-range division); then k-blocks kb0..kb1-1
// quantised, q = rint(x * inv) saturated to [-128, 127], into the Y slots in the
// layout load_act_direct writes.  Rows past M are zero.  All epilogue warps take part
// (named barrier 3 between the steps).
template <int TN>
__device__ __forceinline__ void load_act_quant(const GemmArgs &a, uint8_t *sy, int kb0, int kb1,
                                               int tid, float *act_scale, float *act_inv) {
  constexpr int kChunks = TN * (kBK / 16);
  constexpr int kThr = kEpiWarps * 32;
  const int f16 = a.act_src_dtype == I8L_F16;
  const uint8_t *src = static_cast<const uint8_t *>(a.act_src);
  const long long ld_bytes = a.act_ld * 2;
  // Row absmax: units of 16 values (32 bytes) over all rows, 8 per thread in flight;
  // each unit's max (fmaxf from 0, so NaN is ignored as the row quantiser ignores it)
  // goes into the row's slot with an integer atomicMax, exact for non-negative floats.
  int *amax_bits = reinterpret_cast<int *>(act_inv);
  for (int r = tid; r < TN; r += kThr) amax_bits[r] = 0;
  named_bar_sync(3, kThr);
  const int cpr = a.K / 16;  // units per row (K is a multiple of 16)
  const int units = min(a.M, TN) * cpr;
  for (int u0 = tid; u0 < units; u0 += 8 * kThr) {
    uint4 q[8][2];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int id = u0 + u * kThr;
      q[u][0] = q[u][1] = make_uint4(0u, 0u, 0u, 0u);
      if (id < units) {
        const int8_t *p = reinterpret_cast<const int8_t *>(src + (id / cpr) * ld_bytes + (id % cpr) * 32);
        q[u][0] = ld_cg_v4(p);
        q[u][1] = ld_cg_v4(p + 16);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int id = u0 + u * kThr;
      if (id < units) {
        float mx = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) mx = fmaxf(mx, fabsf(act_val(q[u][e >> 3], e & 7, f16)));
        atomicMax(&amax_bits[id / cpr], __float_as_int(mx));
      }
    }
  }
  named_bar_sync(3, kThr);
  for (int r = tid; r < a.M && r < TN; r += kThr) {
    const float amax = __int_as_float(amax_bits[r]);
    act_scale[r] = a.act_precise ? div_rn(amax, 127.f) : div_full(amax, 127.f);
    act_inv[r] = amax == 0.f ? 0.f : (a.act_precise ? div_rn(127.f, amax) : div_full(127.f, amax));
  }
  named_bar_sync(3, kThr);
  const int n = (kb1 - kb0) * kChunks;
  for (int base = tid; base < n; base += 4 * kThr) {
    uint4 v[4][2];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int id = base + u * kThr;
      v[u][0] = v[u][1] = make_uint4(0u, 0u, 0u, 0u);
      if (id < n) {
        const int j = id / kChunks, r = (id % kChunks) >> 3, c = id & 7;
        const long long col = static_cast<long long>(kb0 + j) * kBK + c * 16;
        if (r < a.M && col < a.K) {
          const int8_t *p = reinterpret_cast<const int8_t *>(src + r * ld_bytes + col * 2);
          v[u][0] = ld_cg_v4(p);
          v[u][1] = ld_cg_v4(p + 16);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int id = base + u * kThr;
      if (id < n) {
        const int j = id / kChunks, r = (id % kChunks) >> 3, c = id & 7;
        uint32_t packed[4] = {0u, 0u, 0u, 0u};
        if (r < a.M) {
          const float inv = act_inv[r];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            int q = __float2int_rn(__fmul_rn(act_val(v[u][e >> 3], e & 7, f16), inv));
            q = q < -128 ? -128 : (q > 127 ? 127 : q);
            packed[e >> 2] |= (static_cast<uint32_t>(q) & 0xffu) << ((e & 3) * 8);
          }
        }
        *reinterpret_cast<uint4 *>(sy + static_cast<size_t>(j) * (TN * kBK) + r * kBK +
                                   ((c ^ (r & 7)) << 4)) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
      }
    }
  }
}

// Decode tiles (TN <= 64) cap registers so two CTAs fit on an SM: with programmatic
// dependent launch the next GEMM's CTA streams its weights beside this one.
template <int TN, int kVar>
__global__ void __launch_bounds__(kThreads, (TN <= 64 || kVar == kVarNarrow) ? 2 : 1)
    w8a8_gemm_sm100(const __grid_constant__ CUtensorMap map_x,
                    const __grid_constant__ CUtensorMap map_y,
                    const __grid_constant__ CUtensorMap map_out,
                    const __grid_constant__ CUtensorMap map_ws, const GemmArgs a) {
  constexpr bool kPair = kVar == kVarPair;
  constexpr bool kNarrow = kVar == kVarNarrow;
  using L = SmemLayout<TN, kVar>;
  // CTA pairs: rank 1 loads its halves and runs its epilogue; rank 0 also issues the MMAs.
  const int rank = kPair ? static_cast<int>(blockIdx.x & 1u) : 0;
  const bool leader = rank == 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = a.stages;
  uint8_t *sx = smem;
  uint8_t *sy = smem + static_cast<size_t>(S) * L::kXBytes;
  uint8_t *staging = smem + static_cast<size_t>(S) * L::kStageBytes;
  float *scal = reinterpret_cast<float *>(staging + kStagingBytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(scal) + kScalBytes);
  uint64_t *empty = full + S;
  uint64_t *acc_full = empty + S;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint64_t *peer_bar = drain + 1;  // cluster leader: contributors' partial sums have landed
  uint64_t *done_bar = drain + 2;  // cluster sender: the receivers' rings are free for it
  uint64_t *act_bar = drain + 3;   // direct activation loads have landed in the Y slots
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *last_flag = abort_flag + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kPair ? 2 * kEpiWarps : kEpiWarps);  // both CTAs' epilogues
    }
    mbar_init(drain, 1);
    mbar_init(peer_bar, 1);
    // Narrow tiles: the leader's go; swap_ab tiles: one arrival from each other CTA.
    mbar_init(done_bar, (!kNarrow && !kPair && a.cluster > 1) ? a.cluster - 1 : 1);
    mbar_init(act_bar, kEpiWarps);
    if (kNarrow && a.cluster_early && cluster_ctarank() == 0) {
      // One tile per cluster: its partial sums arrive as (cluster-1) slots of the
      // live column chunks of the M token rows.  Armed before the cluster sync, so
      // before any byte lands.
      int tx, ty;
      tile_coords(a, static_cast<int>(blockIdx.x) / a.cluster, tx, ty);
      const int nch = (live_cols<TN>(a, ty) + 15) / 16;
      mbar_arrive_expect_tx(peer_bar, static_cast<uint32_t>((a.cluster - 1) * nch * 16 * a.M * 4));
    }
    if constexpr (!kNarrow && !kPair) {
      if (a.cluster > 1) {
        // Spread reduction (swap_ab tiles): 16-column chunk c of the tile belongs to CTA
        // rank c % cluster, which receives it from the other (cluster-1) CTAs.  Armed
        // before the cluster sync, so before any byte lands.
        int tx, ty;
        tile_coords(a, static_cast<int>(blockIdx.x) / a.cluster, tx, ty);
        const int nch = (live_cols<TN>(a, ty) + 15) / 16;
        const int r = static_cast<int>(cluster_ctarank());
        const int owned = nch > r ? (nch - r + a.cluster - 1) / a.cluster : 0;
        mbar_arrive_expect_tx(peer_bar, static_cast<uint32_t>((a.cluster - 1) * owned * 16 * kXRows * 4));
      }
    }
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_y);
  }
  if (warp == 2 && lane == 0) {
    if (a.tma_out) tma_prefetch_desc(&map_out);
    if (a.sk_iters > 0) tma_prefetch_desc(&map_ws);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_slot, L::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, L::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Every CTA's barriers (and a pair's TMEM) are set up before any CTA of the cluster
  // signals them.
  if (a.cluster > 1 || kPair) cluster_sync();
  // The next kernel in the stream may start its own prologue now; it waits for this
  // grid before touching anything this grid writes.
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_x = a.swap ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_y = policy_evict_last();
      // One X / Y tile of a stage.  CTA pairs: this CTA's 128 X rows and its half of the
      // TN Y rows, counted on the even CTA's `full` barrier.
      auto load_x = [&](int st, int kb, int tx) {
        if constexpr (kPair)
          tma_load_2d_pair(sx + static_cast<size_t>(st) * L::kXBytes, &map_x,
                           map_to_rank(smem_u32(&full[st]), 0), kb * kBK, tx * kXRows, pol_x);
        else
          tma_load_2d(sx + static_cast<size_t>(st) * L::kXBytes, &map_x, &full[st], kb * kBK,
                      tx * kXRows, pol_x);
      };
      auto load_y = [&](int st, int kb, int ty) {
        if constexpr (kPair)
          tma_load_2d_pair(sy + static_cast<size_t>(st) * L::kYBytes, &map_y,
                           map_to_rank(smem_u32(&full[st]), 0), kb * kBK,
                           ty * TN + rank * L::kYRows, pol_y);
        else
          tma_load_2d(sy + static_cast<size_t>(st) * L::kYBytes, &map_y, &full[st], kb * kBK,
                      ty * TN, pol_y);
      };
      // Bytes one stage's `full` barrier waits for (both CTAs' with pairs; armed by the
      // even CTA only).
      const uint32_t stage_tx = kPair ? 2u * L::kStageBytes
                                      : (a.act_direct ? static_cast<uint32_t>(L::kXBytes) : L::kStageBytes);
      // Weight tiles of the first stages are loaded before waiting for the previous
      // kernel: inference weights are never written by the kernel just before.  The
      // weight is X with swap_ab, else Y.  Activations wait for pdl_wait().
      int pre = 0;
      {
        Schedule ps;
        ps.init(a);
        Segment sg;
        while (pre < S && ps.next(a, sg)) {
          int tx, ty;
          cta_tile(a, sg.tile, tx, ty);
          for (int kb = sg.kb0; kb < sg.kb1 && pre < S; ++kb, ++pre) {
            if (leader) mbar_arrive_expect_tx(&full[pre], stage_tx);
            if (a.swap)
              load_x(pre, kb, tx);
            else
              load_y(pre, kb, ty);
          }
        }
      }
      Schedule sch;
      sch.init(a);
      pdl_wait();
      Segment seg;
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      while (ok && sch.next(a, seg)) {
        int tx, ty;
        cta_tile(a, seg.tile, tx, ty);
        for (int kb = seg.kb0; kb < seg.kb1; ++kb) {
          if (issued < pre) {
            // Stage already claimed above with its weight tile: add the activation
            // (with direct activation loads the epilogue warps fill the Y slot).
            if (a.act_direct) {
            } else if (a.swap)
              load_y(stage, kb, ty);
            else
              load_x(stage, kb, tx);
          } else {
            if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, a.status,
                                   kStatusProducerWait)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(&full[stage], kPair ? stage_tx : L::kStageBytes);
            load_x(stage, kb, tx);
            load_y(stage, kb, ty);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // Let the loads already issued land before the CTA exits (a pair's loads are
        // all counted on the even CTA's barriers; the odd CTA stays alive until the
        // even one leaves, at the cluster barrier at the end).
        int st = stage;
        uint32_t ph = phase;
        const long long n = issued < S ? issued : S;
        for (long long i = 0; i < n; ++i) {
          if (--st < 0) {
            st = S - 1;
            ph ^= 1u;
          }
          volatile int no_abort = 0;
          mbar_wait_bounded(&full[st], ph, &no_abort, a.status, kStatusDrainWait);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (CTA pairs: the even CTA issues the 256-row MMAs for both.)
    if (lane == 0 && leader) {
      constexpr uint32_t kIdesc = idesc_i8(kPair ? 2 * kXRows : L::kXRowsV, TN);
      Schedule sch;
      sch.init(a);
      Segment seg;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      while (ok && sch.next(a, seg)) {
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u, abort_flag, a.status,
                               kStatusMmaWait)) {
          ok = false;
          break;
        }
        if (a.act_direct && !issued_any &&
            !mbar_wait_bounded(act_bar, 0, abort_flag, a.status, kStatusMmaWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * L::kAccCols);
        int kstep = 0;
        for (int kb = seg.kb0; kb < seg.kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, a.status,
                                 kStatusMmaWait)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_u32(sx + static_cast<size_t>(stage) * L::kXBytes));
          const uint64_t bd = sw128_kmajor_desc(smem_u32(sy + static_cast<size_t>(stage) * L::kYBytes));
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k, ++kstep) {
            const int ch = kstep % L::kChains;
            if constexpr (kPair)
              mma_i8_pair(d + static_cast<uint32_t>(ch * TN), ad + 2 * k, bd + 2 * k, kIdesc,
                          kstep >= L::kChains ? 1u : 0u);
            else
              mma_i8(d + static_cast<uint32_t>(ch * TN), ad + 2 * k, bd + 2 * k, kIdesc,
                     kstep >= L::kChains ? 1u : 0u);
          }
          issued_any = true;
          if constexpr (kPair)
            mma_commit_pair_mc(&empty[stage], 0x3);  // frees the stage in both CTAs
          else
            mma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (kPair)
          mma_commit_pair_mc(&acc_full[acc], 0x3);  // both CTAs' epilogues may read
        else
          mma_commit(&acc_full[acc]);
        if (++acc == L::kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // Let the MMAs in flight finish before TMEM and shared memory go away.
        if constexpr (kPair)
          mma_commit_pair(drain);
        else
          mma_commit(drain);
        volatile int no_abort = 0;
        mbar_wait_bounded(drain, 0, &no_abort, a.status, kStatusDrainWait);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;
    const int epi_tid = threadIdx.x - 64;
    // This warp is done reading an accumulator (CTA pairs: the even CTA's barrier
    // counts both CTAs' epilogue warps).
    auto release_acc = [&](uint64_t *bar) {
      if constexpr (kPair) {
        if (leader)
          mbar_arrive(bar);
        else
          mbar_arrive_remote(map_to_rank(smem_u32(bar), 0));
      } else {
        mbar_arrive(bar);
      }
    };
    Schedule sch;
    sch.init(a);
    Segment seg;
    pdl_wait();  // scales, outputs and the workspace belong to the stream's order
    if (a.act_direct) {
      Schedule s0 = sch;
      Segment g0;
      if (s0.next(a, g0)) {
        if (a.act_quant)
          load_act_quant<TN>(a, sy, g0.kb0, g0.kb1, epi_tid, scal + 2 * kScalFloats,
                             scal + 3 * kScalFloats);
        else
          load_act_direct<TN>(a, sy, g0.kb0, g0.kb1, epi_tid);
      }
      fence_proxy_async_smem();  // generic-proxy stores -> operands of tcgen05.mma
      __syncwarp();
      if (lane == 0) mbar_arrive(act_bar);
    }
    const bool raw = a.out_dtype == I8L_I32;
    const bool has_bias = a.bias != nullptr;
    const bool wide = a.out_dtype == I8L_BF16 || a.out_dtype == I8L_F16;
    Staging st{staging + static_cast<size_t>(quarter) * 2 * kStageBufBytes, 0u};
    int acc = 0;
    uint32_t acc_phase = 0;
    while (sch.next(a, seg)) {
      TileCtx t;
      cta_tile(a, seg.tile, t.tx, t.ty);
      t.ncols = live_cols<TN>(a, t.ty);
      t.taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                static_cast<uint32_t>(acc * L::kAccCols);
      // Scales and bias for this tile, fetched before the accumulator is ready.
      float *s_col = scal + acc * kScalFloats;
      float *b_col = scal + 2 * kScalFloats + acc * kScalFloats;
      t.s_col = s_col;
      t.b_col = b_col;
      t.s_row = 0.f;
      t.b_row = 0.f;
      if (!raw) {
        if (a.swap) {
          const int n = t.tx * kXRows + row;
          if (n < a.N) {
            t.s_row = a.sb_per_col ? a.sb[n] : a.sb[0];
            t.b_row = has_bias ? load_scalar_f(a.bias, a.bias_dtype, n) : 0.f;
          }
          // (fused activation quantisation: the loader's scales, in the b_col area,
          // which swap tiles do not use)
          for (int c = epi_tid; c < TN; c += kEpiWarps * 32) {
            const int m = t.ty * TN + c;
            s_col[c] = m < a.M ? (a.act_quant ? scal[2 * kScalFloats + m]
                                              : (a.sa_per_row ? a.sa[m] : a.sa[0]))
                               : 0.f;
          }
        } else {
          const int m = t.tx * kXRows + row;
          if (m < a.M) t.s_row = a.sa_per_row ? a.sa[m] : a.sa[0];
          if constexpr (kNarrow) {
            // Token-row scales in the second accumulator's (unused) scale slot.
            if (epi_tid < a.M) scal[kScalFloats + epi_tid] = a.sa_per_row ? a.sa[epi_tid] : a.sa[0];
          }
          for (int c = epi_tid; c < TN; c += kEpiWarps * 32) {
            const int n = t.ty * TN + c;
            s_col[c] = n < a.N ? (a.sb_per_col ? a.sb[n] : a.sb[0]) : 0.f;
            b_col[c] = (has_bias && n < a.N) ? load_scalar_f(a.bias, a.bias_dtype, n) : 0.f;
          }
        }
      }
      const bool ok = mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, a.status,
                                        kStatusEpilogueWait);
      // All four epilogue warps continue or all stop: they meet at named barriers
      // below.  The barrier also publishes the scale arrays written above.
      if (!named_bar_and(2, kEpiWarps * 32, ok)) break;
      tc_fence_after();
      const bool whole = seg.kb0 == 0 && seg.kb1 == a.kblocks;
      if constexpr (kNarrow) {
        // Narrow tiles: the M <= 16 token rows are TMEM lanes 0..M-1, which only warp
        // quarter 0 can read.  That warp copies its rows' 256 int32 sums into `rows`
        // (shared memory); then all four epilogue warps work on 8-column groups: a
        // contributor pushes the groups into its slot of the leader (partial sums of
        // [M rows][TN] int32 per contributor: in the leader's staging area when early,
        // else in its idle operand ring after the go signal); the leader adds the slots
        // to its own rows, dequantises and stores.
        const int nch = (t.ncols + 15) / 16;
        const int ngroups = a.M * (TN / 8);
        const uint32_t rank = a.cluster > 1 ? cluster_ctarank() : 0u;
        uint32_t *slots = reinterpret_cast<uint32_t *>(a.cluster_early ? staging : sx);
        uint32_t *rows = reinterpret_cast<uint32_t *>(a.cluster_early ? sx : staging);
        // `rows` holds token row m's 16-byte units at u ^ (m & 7): the quarter-0 lanes
        // store whole rows at a 1 KB stride, which would otherwise all hit one bank.
        if (quarter == 0) {
          for (int c = 0; c < nch; c += 4) {
            uint32_t r[4][16];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (c + j < nch) tmem_ld16(t.taddr + (c + j) * 16, r[j]);
            tmem_ld_wait();
            if (lane < a.M) {
              uint4 *dst = reinterpret_cast<uint4 *>(rows + lane * TN);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (c + j < nch)
#pragma unroll
                  for (int v = 0; v < 4; ++v)
                    dst[((c + j) * 4 + v) ^ (lane & 7)] =
                        make_uint4(r[j][4 * v], r[j][4 * v + 1], r[j][4 * v + 2], r[j][4 * v + 3]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(&acc_empty[acc]);
        named_bar_sync(1, kEpiWarps * 32);  // `rows` complete
        if (a.cluster > 1 && rank != 0) {
          const bool go = a.cluster_early ||
                          __all_sync(0xffffffffu, mbar_wait_cluster_bounded(
                                                      done_bar, 0, abort_flag, a.status,
                                                      kStatusClusterWait));
          if (go) {
            const uint32_t bar0 = map_to_rank(smem_u32(peer_bar), 0);
            for (int gidx = epi_tid; gidx < ngroups; gidx += kEpiWarps * 32) {
              const int m = gidx / (TN / 8), c = (gidx % (TN / 8)) * 8;
              if (c >= nch * 16) continue;
              const uint4 *src = reinterpret_cast<const uint4 *>(rows + m * TN);
              const int u = c / 4;
              const uint32_t dst = map_to_rank(
                  smem_u32(slots + ((static_cast<size_t>(rank) - 1) * a.M + m) * TN + c), 0);
              st_async_v4(dst, src[u ^ (m & 7)], bar0);
              st_async_v4(dst + 16, src[(u + 1) ^ (m & 7)], bar0);
            }
          }
        } else {
          bool got = true;
          if (a.cluster > 1) {
            if (epi_tid == 0 && !a.cluster_early) {
              mbar_arrive_expect_tx(peer_bar, static_cast<uint32_t>((a.cluster - 1) * nch * 16 * a.M * 4));
              for (int p = 1; p < a.cluster; ++p)
                mbar_arrive_remote(map_to_rank(smem_u32(done_bar), static_cast<uint32_t>(p)));
            }
            got = __all_sync(0xffffffffu, mbar_wait_bounded(peer_bar, 0, abort_flag, a.status,
                                                             kStatusClusterWait));
          }
          if (got) {
            const float *sa_rows = scal + kScalFloats;  // the second accumulator's scale slot
            for (int gidx = epi_tid; gidx < ngroups; gidx += kEpiWarps * 32) {
              const int m = gidx / (TN / 8), c = (gidx % (TN / 8)) * 8;
              if (c >= t.ncols) continue;
              uint32_t r[8];
              {
                const uint4 *src = reinterpret_cast<const uint4 *>(rows + m * TN);
                const uint4 q0 = src[(c / 4) ^ (m & 7)], q1 = src[(c / 4 + 1) ^ (m & 7)];
                r[0] = q0.x; r[1] = q0.y; r[2] = q0.z; r[3] = q0.w;
                r[4] = q1.x; r[5] = q1.y; r[6] = q1.z; r[7] = q1.w;
              }
              for (int p = 1; p < a.cluster; ++p) {
                const uint4 *src = reinterpret_cast<const uint4 *>(
                    slots + ((static_cast<size_t>(p) - 1) * a.M + m) * TN + c);
                const uint4 q0 = src[0], q1 = src[1];
                r[0] += q0.x; r[1] += q0.y; r[2] += q0.z; r[3] += q0.w;
                r[4] += q1.x; r[5] += q1.y; r[6] += q1.z; r[7] += q1.w;
              }
              store_row8<TN>(a, t, m, c, sa_rows[m], r);
            }
          }
        }
      } else if (a.cluster > 1) {
        // Cluster split-K, spread reduction.  Each CTA holds the partial sums of its k
        // range for the whole tile; 16-column chunk c is finished by CTA rank
        // c % cluster.  Every CTA sends the chunks it does not own into slot (sender)
        // of the owner's receive area, completing the owner's barrier by bytes, then
        // adds the (cluster-1) received slots to its own chunks, dequantises and stores
        // them.  Each SM thus takes in (cluster-1)/cluster of one tile's partial sums
        // and stores 1/cluster of the tile, where a single leader would take in
        // (cluster-1) tiles' worth and store it all.  Integer sums: the order of the
        // additions does not change the result.  A chunk slot is 128 rows x 64 bytes,
        // the four 16-byte units of a row XOR-swizzled by (row >> 1) & 3.
        //   Early mode (the receive slots fit the staging area, free from the start
        //   with plain stores): each thread pushes its rows with st.async.
        //   Ring mode: the receive slots lie at the start of the operand ring, idle
        //   once this CTA's MMAs are done (acc_full); each CTA tells the others so,
        //   writes its outgoing chunks, grouped by owner, at the end of its own ring,
        //   and one thread sends each owner's group with one bulk copy once every
        //   other CTA has said its ring is free.
        const int C = a.cluster;
        const uint32_t rank = cluster_ctarank();
        const int nch = (t.ncols + 15) / 16;
        const int sw = (row >> 1) & 3;  // 64-byte rows: 16-byte units swizzled over the banks
        constexpr int kChunkWords = kXRows * 16;  // one chunk slot: 8 KB
        // Live chunks rank o owns; o's receive area holds slot (sender, j) at sender * that + j.
        auto owned_by = [&](int o) { return nch > o ? (nch - o + C - 1) / C : 0; };
        const int mine = owned_by(static_cast<int>(rank));
        uint32_t *slots = reinterpret_cast<uint32_t *>(a.cluster_early ? staging : sx);
        if (a.cluster_early) {
          for (int c = 0; c < nch; ++c) {
            const uint32_t owner = static_cast<uint32_t>(c % C);
            if (owner == rank) continue;
            uint32_t r[16];
            tmem_acc16<TN>(t.taddr, c * 16, r);
            const int sender = static_cast<int>(rank < owner ? rank : rank - 1);
            const uint32_t bar = map_to_rank(smem_u32(peer_bar), owner);
            const uint32_t dst = map_to_rank(
                smem_u32(slots + (static_cast<size_t>(sender) * owned_by(static_cast<int>(owner)) + c / C) *
                                     kChunkWords + row * 16),
                owner);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              st_async_v4(dst + ((v ^ sw) << 4),
                          make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]), bar);
          }
        } else {
          if (epi_tid == 0)
            for (int p = 1; p < C; ++p)
              mbar_arrive_remote(map_to_rank(smem_u32(done_bar), (rank + static_cast<uint32_t>(p)) % C));
          const int out_chunks = nch - mine;
          uint32_t *out = reinterpret_cast<uint32_t *>(staging) - static_cast<size_t>(out_chunks) * kChunkWords;
          int group = 0;  // first outgoing slot of the current owner's group
          for (int o = 0; o < C; ++o) {
            if (o == static_cast<int>(rank)) continue;
            for (int j = 0, c = o; c < nch; ++j, c += C) {
              uint32_t r[16];
              tmem_acc16<TN>(t.taddr, c * 16, r);
              uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<size_t>(group + j) * kChunkWords + row * 16);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v ^ sw] = make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
            }
            group += owned_by(o);
          }
          fence_proxy_async_smem();  // generic-proxy stores -> source of the bulk copies
          named_bar_sync(1, kEpiWarps * 32);
          if (epi_tid == 0 && mbar_wait_cluster_bounded(done_bar, 0, abort_flag, a.status, kStatusClusterWait)) {
            group = 0;
            for (int o = 0; o < C; ++o) {
              if (o == static_cast<int>(rank)) continue;
              const int n_o = owned_by(o);
              if (n_o > 0) {
                const int sender = static_cast<int>(rank) < o ? static_cast<int>(rank) : static_cast<int>(rank) - 1;
                bulk_copy_to_rank(
                    map_to_rank(smem_u32(slots + static_cast<size_t>(sender) * n_o * kChunkWords),
                                static_cast<uint32_t>(o)),
                    smem_u32(out + static_cast<size_t>(group) * kChunkWords),
                    static_cast<uint32_t>(n_o) * kChunkWords * 4,
                    map_to_rank(smem_u32(peer_bar), static_cast<uint32_t>(o)));
              }
              group += n_o;
            }
          }
        }
        const bool got = __all_sync(0xffffffffu, mbar_wait_bounded(peer_bar, 0, abort_flag, a.status,
                                                                    kStatusClusterWait));
        for (int c = static_cast<int>(rank); c < nch; c += C) {
          uint32_t r[16];
          tmem_acc16<TN>(t.taddr, c * 16, r);
          if (!got) continue;
          for (int p = 0; p < C - 1; ++p) {
            const uint4 *src = reinterpret_cast<const uint4 *>(
                slots + (static_cast<size_t>(p) * mine + c / C) * kChunkWords + row * 16);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const uint4 q = src[v ^ sw];
              r[4 * v] += q.x;
              r[4 * v + 1] += q.y;
              r[4 * v + 2] += q.z;
              r[4 * v + 3] += q.w;
            }
          }
          if (a.tma_out)
            emit_swap16<TN>(a, &map_out, t, quarter, lane, c * 16, r, st);
          else
            epilogue_direct<TN>(a, t, row, c * 16, r);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(&acc_empty[acc]);
      } else if (whole) {
        if (!a.tma_out) {
          for (int c0 = 0; c0 < t.ncols; c0 += 16) {
            uint32_t r[16];
            tmem_acc16<TN>(t.taddr, c0, r);
            epilogue_direct<TN>(a, t, row, c0, r);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(&acc_empty[acc]);
        } else if (a.swap) {
          for (int c0 = 0; c0 < t.ncols; c0 += 16) {
            uint32_t r[16];
            tmem_acc16<TN>(t.taddr, c0, r);
            if (c0 + 16 >= t.ncols) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) release_acc(&acc_empty[acc]);
            }
            emit_swap16<TN>(a, &map_out, t, quarter, lane, c0, r, st);
          }
        } else {
          const int step = wide ? 32 : 16;
          for (int c0 = 0; c0 < t.ncols; c0 += step) {
            uint32_t r0[16], r1[16];
            tmem_acc16<TN>(t.taddr, c0, r0);
            if (wide) tmem_acc16<TN>(t.taddr, c0 + 16, r1);
            if (c0 + step >= t.ncols) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) release_acc(&acc_empty[acc]);
            }
            emit_normal<TN>(a, &map_out, t, quarter, lane, c0, r0, r1, st);
          }
        }
      } else {
        // A piece of a split tile: add it into the tile's workspace slot in L2
        // (TMA reduce-add of int32 boxes {32 rows, 16 columns}).
        const int slot = split_slot(a, seg.tile);
        for (int c0 = 0; c0 < t.ncols; c0 += 16) {
          uint32_t r[16];
          tmem_acc16<TN>(t.taddr, c0, r);
          if (c0 + 16 >= t.ncols) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(&acc_empty[acc]);
          }
          uint8_t *buf = st.acquire(lane);
          uint32_t *b32 = reinterpret_cast<uint32_t *>(buf);
#pragma unroll
          for (int j = 0; j < 16; ++j) b32[j * 32 + lane] = r[j];
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&map_ws, buf, quarter * 32, slot * TN + c0);
            bulk_commit();
          }
        }
        if (lane == 0) {
          bulk_wait<0>();
          fence_proxy_async_global();
          __threadfence();
        }
        __syncwarp();
        named_bar_sync(1, kEpiWarps * 32);
        if (epi_tid == 0) {
          const int mine = seg.kb1 - seg.kb0;
          const int before = atomicAdd(a.counters + slot, mine);
          *last_flag = (before + mine == a.kblocks) ? 1 : 0;
        }
        named_bar_sync(1, kEpiWarps * 32);
        if (*last_flag) {
          // This piece completed the tile: read the sums, store, zero the slot.
          __threadfence();
          int *ws = a.ws + static_cast<size_t>(slot) * (kXRows * TN);
          const int step = (!a.swap && wide && a.tma_out) ? 32 : 16;
          for (int c0 = 0; c0 < t.ncols; c0 += step) {
            uint32_t r0[16], r1[16];
            // All loads first, then the zeroing stores: the accesses are ordered as
            // written, so interleaving them would serialise 16-32 L2 round trips.
#pragma unroll
            for (int j = 0; j < 16; ++j) r0[j] = static_cast<uint32_t>(ld_cg_s32(ws + (c0 + j) * kXRows + row));
            if (step == 32) {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                r1[j] = static_cast<uint32_t>(ld_cg_s32(ws + (c0 + 16 + j) * kXRows + row));
            }
#pragma unroll
            for (int j = 0; j < step; ++j) st_cg_s32(ws + (c0 + j) * kXRows + row, 0);
            if (!a.tma_out)
              epilogue_direct<TN>(a, t, row, c0, r0);
            else if (a.swap)
              emit_swap16<TN>(a, &map_out, t, quarter, lane, c0, r0, st);
            else
              emit_normal<TN>(a, &map_out, t, quarter, lane, c0, r0, r1, st);
          }
          if (epi_tid == 0) atomicExch(a.counters + slot, 0);
        }
      }
      if (++acc == L::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    st.drain(lane);
  }

  tc_fence_before();
  __syncthreads();
  // A pair's CTAs leave together: neither exits while the other may still signal its
  // barriers or the even CTA's MMAs may still read its shared memory.  The CTAs of a
  // split-K cluster likewise: none leaves while another may still push partial sums into
  // its shared memory (a receiver whose wait gave up included).
  if (kPair || a.cluster > 1) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem_base, L::kTmemCols);
    else
      tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map over an int8 [rows, K] matrix with row stride `ld` bytes, boxes of
// 128 bytes along K by `box_rows` rows, 128-byte swizzle, zero fill outside.
static int make_operand_map(CUtensorMap *map, const int8_t *ptr, int64_t rows, int64_t k,
                            int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(I8L_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(I8L_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d) for [%lld x %lld], ld %lld",
                     static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(k),
                     static_cast<long long>(ld));
  return I8L_OK;
}

// Tensor map over a row-major 2-D matrix of `rows` x `cols` elements (row stride
// `ld_bytes`), boxes of box_cols x box_rows.
static int make_map(CUtensorMap *map, CUtensorMapDataType type, const void *ptr, int64_t rows,
                    int64_t cols, int64_t ld_bytes, int box_cols, int box_rows,
                    CUtensorMapSwizzle swizzle, const char *what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(I8L_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, type, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(I8L_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d) for the %s map [%lld x %lld]",
                     static_cast<int>(r), what, static_cast<long long>(rows),
                     static_cast<long long>(cols));
  return I8L_OK;
}

static size_t smem_extra() { return 1024 + kStagingBytes + kScalBytes + 8 * 8 + 64; }

// Shared memory of one of two CTAs that share an SM (228 KB minus 1 KB reserved per CTA).
constexpr int kHalfSmem = 233472 / 2 - 1024;

// X and Y rows one CTA holds per stage (X: 128, or 64 for narrow tiles; Y: TN, or
// TN/2 for a CTA pair).
static int max_stages_for(int y_rows, int smem_optin, int x_rows = kXRows) {
  const int stage = x_rows * kBK + y_rows * kBK;
  const int avail = smem_optin - static_cast<int>(smem_extra()) - 16;
  return std::max(1, std::min(16, avail / (stage + 16)));
}

// Most bytes of partial sums one CTA of a split-K cluster of `c` receives: narrow tiles,
// the leader gets (c-1) slots of M token rows x TN int32; swap_ab tiles, every CTA gets
// the 16-column chunks it owns (one in c of TN/16, rank 0 the most) from each of the
// other (c-1), 128 rows x 16 int32 per chunk.
static long long cluster_recv_bytes(bool narrow, int M, int tn, int c) {
  if (narrow) return static_cast<long long>(c - 1) * M * tn * 4;
  return static_cast<long long>(c - 1) * ((tn / 16 + c - 1) / c) * 16 * kXRows * 4;
}

// Ring bytes a CTA of a split-K cluster of `c` swap_ab tiles needs in ring mode: its
// incoming slots ((c-1) senders x the chunks it owns) at the start and its outgoing
// chunks (those it does not own) at the end; the most over the ranks.
static long long cluster_ring_bytes(int tn, int c) {
  const int nch = tn / 16;
  long long worst = 0;
  for (int r = 0; r < c; ++r) {
    const int own = nch > r ? (nch - r + c - 1) / c : 0;
    worst = std::max(worst, static_cast<long long>((c - 1) * own + (nch - own)) * 16 * kXRows * 4);
  }
  return worst;
}

static bool valid_tok_tile(int t) { return t == 16 || t == 32 || t == 64 || t == 128 || t == 256; }

// Everything the launch needs, derived from the problem and the tile.
struct Plan {
  i8l_tile tile;
  int tn;  // Y tile rows (MMA N)
  int tiles_x, tiles_y, kblocks, total_tiles, dp_tiles, ctas;
  long long sk_iters;
  int slots;
  size_t ws_bytes;
  int cluster;  // CTAs per cluster splitting K of one tile (1 = none)
  int pair;     // CTA pairs (cta_group::2): tiles_x counts 256-row tiles
  int narrow;   // narrow decode tiles: <= 16 tokens x 256 weight rows, 64-row MMAs
};

// Cluster size (1..8, at most the k-blocks) whose grid of tiles x size CTAs, one per
// SM, keeps the most SMs streaming.  Ties go to the smaller cluster.
static int best_cluster(int tiles, int kblocks, int sms) {
  int best = 1;
  double best_util = 0.0;
  for (int cs = 1; cs <= 8 && cs <= kblocks; ++cs) {
    const long long ctas = static_cast<long long>(tiles) * cs;
    if (ctas > sms) break;
    const double util = static_cast<double>(ctas) / sms;
    if (util > best_util + 1e-9) {
      best_util = util;
      best = cs;
    }
  }
  return best;
}

static void default_tile(int M, int N, int K, i8l_tile *t) {
  (void)N;
  (void)K;
  *t = i8l_tile{};
  if (M <= 256) {
    t->swap_ab = 1;
    t->tok_tile = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
    t->w_tile = 128;
  } else {
    t->swap_ab = 0;
    t->tok_tile = 128;
    t->w_tile = 256;
  }
  t->group = 8;
}

static int make_plan(int M, int N, int K, const i8l_tile *user, Plan *p) {
  DeviceInfo di;
  int e = device_info(&di);
  if (e) return e;
  if (user && user->split == 5) {
    // CUDA-core tiles (gemv_sm100.cu): whole output columns per CTA, no workspace.
    GemvPlan gp;
    if ((e = gemv_plan(M, N, K, user, &gp))) return e;
    *p = Plan{};
    p->tile = *user;
    p->tile.stages = gp.stages;
    p->tile.ctas = gp.ctas;
    p->ctas = gp.ctas;
    return I8L_OK;
  }
  i8l_tile t;
  const bool auto_tile = user == nullptr || (user->tok_tile == 0 && user->w_tile == 0);
  if (auto_tile) {
    default_tile(M, N, K, &t);
    if (user) {
      if (user->stages) t.stages = user->stages;
      if (user->ctas) t.ctas = user->ctas;
      if (user->group) t.group = user->group;
      t.split = user->split;
      t.cluster = user->cluster;
      t.store = user->store;
      t.act = user->act;
    }
  } else {
    t = *user;
  }
  if (t.swap_ab) {
    if (!valid_tok_tile(t.tok_tile) || t.w_tile != 128)
      return set_error(I8L_ENOTSUP,
                       "swap_ab tile needs tok_tile in {16,32,64,128,256} and w_tile 128, got %dx%d",
                       t.tok_tile, t.w_tile);
    p->tn = t.tok_tile;
  } else {
    if (t.tok_tile != 128 || (t.w_tile != 128 && t.w_tile != 256))
      return set_error(I8L_ENOTSUP, "tile needs tok_tile 128 and w_tile in {128,256}, got %dx%d",
                       t.tok_tile, t.w_tile);
    p->tn = t.w_tile;
  }
  // Split mode 4: CTA pairs (cta_group::2) on 128-token x 256-weight tiles, each pair a
  // 256 x 256 tile; every CTA holds 128 token rows and 128 weight rows per stage.  The
  // library's choice for prefill tiles with long K (>= 32 k-blocks), where each SM's TMA
  // fill of 48 KB per k-block, not the tensor core, bounds the one-CTA tile.
  if (t.split == 0 && !t.swap_ab && p->tn == 256 && K >= 4096) t.split = 4;
  const bool pair = t.split == 4;
  if (pair && (t.swap_ab || p->tn != 256))
    return set_error(I8L_ENOTSUP, "CTA pairs (split 4) take tok_tile 128 x w_tile 256 tiles without swap_ab");
  p->pair = pair ? 1 : 0;
  // Narrow decode tiles: cluster split-K (split 3) on 128 x 256 tiles without swap_ab,
  // for batches of <= 16 tokens: 64-row token tiles, the weight on the MMA's N side.
  // Split 3 without swap_ab: narrow tiles for batches of <= 16 tokens, else 128-token
  // tiles with the weight on the MMA's N side and K split over a cluster.
  const bool narrow = t.split == 3 && !t.swap_ab && M <= 16;
  if (narrow && p->tn != 256)
    return set_error(I8L_ENOTSUP, "narrow tiles (split 3 without swap_ab, M <= 16) take w_tile 256");
  p->narrow = narrow ? 1 : 0;
  const int x_rows = narrow ? 64 : kXRows;
  const int max_st = max_stages_for(pair ? p->tn / 2 : p->tn, di.max_smem_optin, x_rows);
  if (t.stages <= 0) {
    t.stages = max_st;
    // Decode tiles: leave room for a second CTA per SM (the next kernel under PDL).
    if ((t.swap_ab && p->tn <= 64) || narrow)
      t.stages = std::max(2, std::min(max_st, max_stages_for(p->tn, kHalfSmem, x_rows)));
  }
  if (t.stages < 2 || t.stages > max_st)
    return set_error(I8L_ENOTSUP, "stages %d outside [2, %d] for this tile", t.stages, max_st);
  if (t.group <= 0) t.group = 1;
  const int rows_x = t.swap_ab ? N : M;
  const int rows_y = t.swap_ab ? M : N;
  p->tiles_x = narrow ? 1 : (rows_x + (pair ? 2 * kXRows : kXRows) - 1) / (pair ? 2 * kXRows : kXRows);
  p->tiles_y = (rows_y + p->tn - 1) / p->tn;
  p->kblocks = (K + kBK - 1) / kBK;
  p->total_tiles = p->tiles_x * p->tiles_y;
  const long long total_iters = static_cast<long long>(p->total_tiles) * p->kblocks;
  int ctas = t.ctas > 0 ? t.ctas : di.sms;
  int split = t.split;
  bool auto_cluster = t.cluster <= 0;  // cluster size left to the library (shrunk to fit below)
  p->cluster = 1;
  if (split == 0) {
    // Decode tiles with fewer tiles than SMs: split K inside thread-block clusters
    // when that keeps most SMs streaming; otherwise whole tiles.
    if (t.swap_ab && p->tn <= 64 && p->total_tiles < ctas) {
      // Cluster split-K when it fills clearly more SMs than whole tiles, else whole tiles.
      const int cs = best_cluster(p->total_tiles, p->kblocks, ctas);
      split = (cs > 1 && p->total_tiles * cs >= p->total_tiles + ctas / 4) ? 3 : 1;
    } else if (t.swap_ab && p->tn <= 64 && t.ctas <= 0 && p->total_tiles <= 2 * ctas) {
      // Decode tiles fit two per SM: one CTA per tile, all resident at once.
      split = 1;
      ctas = p->total_tiles;
    } else if (t.swap_ab && p->total_tiles < ctas && t.cluster <= 0) {
      // 128- and 256-token tiles on fewer tiles than SMs: cluster split-K while each CTA
      // keeps at least 8 k-blocks (measured on B200 at 128 tokens: down, 48 k-blocks,
      // cluster 4 12.2 against 19.2 µs whole; qkv, 16 k-blocks, cluster 2 within 6% of
      // whole tiles, cluster 4 50% slower).
      int cs = best_cluster(p->total_tiles, p->kblocks, ctas);
      while (cs > 1 && p->kblocks / cs < 8) --cs;
      split = cs > 1 ? 3 : 1;
      t.cluster = cs;
    } else {
      // Whole tiles.  Stream-K (split 2, on request) measured slower on every shape
      // tried on B200: 53.7 against 29.9 µs at 4096 x 4096 x 2048, 22.5 against 9.4 µs
      // at 128 x 4096 x 2048.
      split = 1;
    }
  }
  if (split == 3) {
    // Narrow tiles: the leader's operand ring receives (cluster-1) slots of M token rows
    // x TN int32.  Other tiles (swap_ab, or 128 tokens x TN weight rows): every CTA's ring
    // receives, from each of the other (cluster-1), the 16-column chunks it owns (one in
    // `cluster`, 128 rows x 16 int32).
    const long long ring = static_cast<long long>(t.stages) * (x_rows * kBK + p->tn * kBK);
    auto fits = [&](int c) {
      return (narrow ? cluster_recv_bytes(true, M, p->tn, c) : cluster_ring_bytes(p->tn, c)) <= ring;
    };
    int cs = t.cluster;
    if (cs <= 0) cs = best_cluster(p->total_tiles, p->kblocks, ctas);
    if (auto_cluster)
      while (cs > 1 && !fits(cs)) --cs;
    if (cs < 1 || cs > 8 || cs > p->kblocks || !fits(cs))
      return set_error(I8L_ENOTSUP,
                       "cluster size %d outside [1, min(8, k-blocks=%d)] or its partial sums "
                       "exceed the %lld-byte ring",
                       cs, p->kblocks, ring);
    if (cs == 1 && !narrow) split = 1;
    p->cluster = cs;
    ctas = p->total_tiles * cs;
    p->dp_tiles = p->total_tiles;
  }
  if (split == 1) {
    if (p->cluster == 1) ctas = std::min(ctas, p->total_tiles);
    p->dp_tiles = p->total_tiles;
  } else if (split == 2) {
    if (static_cast<long long>(ctas) > total_iters) ctas = static_cast<int>(total_iters);
    const int waves = p->total_tiles / ctas;
    if (p->total_tiles % ctas == 0)
      p->dp_tiles = p->total_tiles;
    else
      p->dp_tiles = waves >= 1 ? (waves - 1) * ctas : 0;
  } else if (split == 4) {
    // One pair (two CTAs, one cluster) per 256 x 256 tile, persistent over the tiles.
    const int pairs = std::max(1, std::min(p->total_tiles, (t.ctas > 0 ? t.ctas : di.sms) / 2));
    ctas = 2 * pairs;
    p->dp_tiles = p->total_tiles;
  } else if (split != 3) {
    return set_error(I8L_ENOTSUP,
                     "split mode %d unknown (0 auto, 1 whole, 2 stream-K, 3 cluster, 4 CTA pairs)", split);
  }
  t.split = split;
  t.cluster = p->cluster;
  t.ctas = ctas;
  p->ctas = ctas;
  // Direct activation loads: every token in one Y tile, one segment per CTA, and that
  // segment's k-blocks all in the ring at once.
  {
    const int seg_kb = p->cluster > 1 ? (p->kblocks + p->cluster - 1) / p->cluster : p->kblocks;
    const bool one_segment = p->cluster > 1 || (split == 1 && ctas >= p->total_tiles);
    const bool direct_ok = t.swap_ab && p->tiles_y == 1 && one_segment && seg_kb <= t.stages;
    if (t.act == 2 && !direct_ok)
      return set_error(I8L_ENOTSUP,
                       "direct activation loads need swap_ab, M <= tok_tile, one tile or cluster "
                       "segment per CTA and at most `stages` k-blocks per CTA");
    if (t.act < 0 || t.act > 2)
      return set_error(I8L_ENOTSUP, "act mode %d unknown (0 auto, 1 TMA, 2 direct loads)", t.act);
    t.act = (t.act == 2 || (t.act == 0 && direct_ok)) ? 2 : 1;
  }
  p->sk_iters = p->cluster > 1 ? 0 : static_cast<long long>(p->total_tiles - p->dp_tiles) * p->kblocks;
  p->slots = p->sk_iters > 0 ? std::max(1, ctas - 1) : 0;
  const size_t counters_bytes = ((static_cast<size_t>(p->slots) * 4 + 255) / 256) * 256;
  p->ws_bytes = p->slots ? counters_bytes + static_cast<size_t>(p->slots) * kXRows * p->tn * 4 : 0;
  p->tile = t;
  return I8L_OK;
}

template <int TN, int kVar = kVarOne>
static int launch_tn(const CUtensorMap &mx, const CUtensorMap &my, const CUtensorMap &mo,
                     const CUtensorMap &mw, const GemmArgs &a, int ctas, int stages,
                     cudaStream_t stream) {
  const size_t smem = SmemLayout<TN, kVar>::bytes(stages);
  // Largest dynamic shared memory already allowed, per device (the attribute is
  // set on the function as loaded in each device's context).
  static size_t configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64 || smem > configured[dev]) {
    e = cudaFuncSetAttribute(w8a8_gemm_sm100<TN, kVar>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemm smem)");
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  e = launch(w8a8_gemm_sm100<TN, kVar>, dim3(ctas), dim3(kThreads), smem, stream,
             kVar == kVarPair ? 2 : a.cluster, mx, my, mo,
             mw, a);
  if (e != cudaSuccess) return cuda_error(e, "gemm launch");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "gemm launch");
  return I8L_OK;
}

}  // namespace i8l

using namespace i8l;

extern "C" int i8l_default_tile(int32_t M, int32_t N, int32_t K, i8l_tile *tile_out) {
  if (!tile_out) return set_error(I8L_EINVAL, "tile_out is NULL");
  Plan p;
  int e = make_plan(M > 0 ? M : 1, N > 0 ? N : 1, K > 0 ? K : 16, nullptr, &p);
  if (e) return e;
  *tile_out = p.tile;
  return I8L_OK;
}

extern "C" size_t i8l_workspace_size(int32_t M, int32_t N, int32_t K, const i8l_tile *tile) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  Plan p;
  if (make_plan(M, N, K, tile, &p)) return 0;
  return p.ws_bytes;
}

namespace i8l {

// A bf16/fp16 activation quantised per token inside the GEMM (i8l_w8a8_mm_quant_act).
struct ActQuant {
  const void *x;
  int dtype;  // I8L_BF16 or I8L_F16
  int64_t ldx;  // elements
  int precise;
};

// The body of i8l_w8a8_mm and i8l_w8a8_mm_quant_act.  With aq, A is aq->x (read only
// by the kernel's direct activation loads; the tile must allow them).
static int gemm_run(const int8_t *A, int64_t lda, const int8_t *W, int64_t ldw, const float *sa,
                    int32_t sa_per_row, const float *sb, int32_t sb_per_col, const void *bias,
                    int32_t bias_dtype, void *out, int32_t out_dtype, int64_t ldc, int32_t M,
                    int32_t N, int32_t K, const i8l_tile *tile, void *workspace, size_t ws_bytes,
                    void *stream, const ActQuant *aq) {
  if (M < 0 || N < 0 || K < 0) return set_error(I8L_EINVAL, "negative size M=%d N=%d K=%d", M, N, K);
  if (out_dtype < I8L_BF16 || out_dtype > I8L_I32)
    return set_error(I8L_ENOTSUP, "output dtype code %d not supported", out_dtype);
  if (M == 0 || N == 0) return I8L_OK;
  if (K == 0) return set_error(I8L_ENOTSUP, "K=0 is not supported");
  if (!A || !W || !out) return set_error(I8L_EINVAL, "NULL operand pointer");
  if (K % 16) return set_error(I8L_ENOTSUP, "K=%d must be a multiple of 16", K);
  if (lda < K || ldw < K || ldc < N)
    return set_error(I8L_EINVAL, "leading dimensions lda=%lld ldw=%lld ldc=%lld too small",
                     static_cast<long long>(lda), static_cast<long long>(ldw),
                     static_cast<long long>(ldc));
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W)) % 16 || lda % 16 || ldw % 16)
    return set_error(I8L_ENOTSUP, "int8 operands and their row strides must be 16-byte aligned");
  const bool raw = out_dtype == I8L_I32;
  if (!raw) {
    if ((!sa && !aq) || !sb) return set_error(I8L_EINVAL, "NULL scale pointer");
    if (bias && (bias_dtype < I8L_BF16 || bias_dtype > I8L_F32))
      return set_error(I8L_ENOTSUP, "bias dtype code %d not supported", bias_dtype);
  }
  if (tile && tile->split == 5) {
    if (aq) {
      // CUDA-core tile: the kernel's prologue quantises the activation per token.
      const GemvPro pro{1, aq->x, aq->ldx, aq->dtype, nullptr, 0, nullptr, 0, nullptr, 0, 0.f,
                        aq->precise, 0};
      return gemv_run(nullptr, 0, W, ldw, nullptr, 0, sb, sb_per_col, bias, bias_dtype, out, out_dtype,
                      ldc, M, N, K, tile, stream, &pro);
    }
    return gemv_run(A, lda, W, ldw, sa, sa_per_row, sb, sb_per_col, bias, bias_dtype, out, out_dtype,
                    ldc, M, N, K, tile, stream);
  }
  Plan p;
  int e = make_plan(M, N, K, tile, &p);
  if (e) return e;
  if (aq && p.tile.act != 2)
    return set_error(I8L_ENOTSUP,
                     "fused activation quantisation needs direct activation loads: swap_ab, "
                     "M <= tok_tile, one tile or cluster segment per CTA and at most `stages` "
                     "k-blocks per CTA");
  if (p.ws_bytes > 0 && (workspace == nullptr || ws_bytes < p.ws_bytes))
    return set_error(I8L_EWORKSPACE, "workspace of %zu bytes needed, %zu given", p.ws_bytes,
                     workspace ? ws_bytes : static_cast<size_t>(0));
  if (workspace && reinterpret_cast<uintptr_t>(workspace) % 256)
    return set_error(I8L_EINVAL, "workspace must be 256-byte aligned");

  CUtensorMap mx, my;
  const bool swap = p.tile.swap_ab != 0;
  const int8_t *xp = swap ? W : A;
  const int8_t *yp = swap ? A : W;
  const int64_t xrows = swap ? N : M, yrows = swap ? M : N;
  const int64_t xld = swap ? ldw : lda, yld = swap ? lda : ldw;
  if ((e = make_operand_map(&mx, xp, xrows, K, xld, p.narrow ? 64 : kXRows))) return e;
  if ((e = make_operand_map(&my, yp, yrows, K, yld, p.pair ? p.tn / 2 : p.tn))) return e;

  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles_x = p.tiles_x;
  a.tiles_y = p.tiles_y;
  a.kblocks = p.kblocks;
  a.total_tiles = p.total_tiles;
  a.dp_tiles = p.dp_tiles;
  a.sk_iters = p.sk_iters;
  a.group = std::max(1, std::min(p.tile.group, p.tiles_x));
  a.stages = p.tile.stages;
  a.swap = swap ? 1 : 0;
  a.sa = sa;
  a.sb = sb;
  a.sa_per_row = sa_per_row ? 1 : 0;
  a.sb_per_col = sb_per_col ? 1 : 0;
  a.bias = raw ? nullptr : bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  a.ldc = ldc;
  const int esize = (out_dtype == I8L_BF16 || out_dtype == I8L_F16) ? 2 : 4;
  const bool aligned_out = reinterpret_cast<uintptr_t>(out) % 16 == 0 && (ldc * esize) % 16 == 0;
  a.vec_store = aligned_out ? 1 : 0;
  // Output path: TMA stores through shared memory, or plain stores (cheaper for the
  // few rows of a decode batch).  store: 0 auto, 1 TMA, 2 direct.
  // Narrow tiles always store directly (one warp writes the few token rows).
  // Cluster split-K on 128-token tiles stores directly (each CTA finishes 16-column chunks).
  const int store = (p.narrow || (p.cluster > 1 && !swap))
                        ? 2
                        : (tile && tile->store ? tile->store : ((swap && M <= 32) ? 2 : 1));
  CUtensorMap mo{}, mw{};
  if (aligned_out && store == 1) {
    static const CUtensorMapDataType kTypes[4] = {
        CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
        CU_TENSOR_MAP_DATA_TYPE_FLOAT32, CU_TENSOR_MAP_DATA_TYPE_INT32};
    // swap: boxes of 32 output columns x 16 tokens; else 64 bytes of columns x 32 rows.
    if (swap)
      e = make_map(&mo, kTypes[out_dtype], out, M, N, ldc * esize, 32, 16,
                   CU_TENSOR_MAP_SWIZZLE_NONE, "output");
    else
      e = make_map(&mo, kTypes[out_dtype], out, M, N, ldc * esize, 64 / esize, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B, "output");
    if (e) return e;
    a.tma_out = 1;
  }
  if (p.ws_bytes) {
    const size_t counters_bytes = ((static_cast<size_t>(p.slots) * 4 + 255) / 256) * 256;
    a.counters = static_cast<int *>(workspace);
    a.ws = reinterpret_cast<int *>(static_cast<uint8_t *>(workspace) + counters_bytes);
    // [slots * TN columns][128 rows] int32, reduced into in boxes of 32 rows x 16 columns.
    if ((e = make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, a.ws,
                      static_cast<int64_t>(p.slots) * p.tn, kXRows, kXRows * 4, 32, 16,
                      CU_TENSOR_MAP_SWIZZLE_NONE, "workspace")))
      return e;
  }
  a.status = status_ptr();
  a.cluster = p.cluster;
  a.act_direct = p.tile.act == 2 ? 1 : 0;
  a.pair = p.pair;
  a.act = A;
  a.lda = lda;
  if (aq) {
    a.act_quant = 1;
    a.act_src_dtype = aq->dtype;
    a.act_precise = aq->precise ? 1 : 0;
    a.act_src = aq->x;
    a.act_ld = aq->ldx;
  }
  // Early cluster mode needs every slot a CTA receives inside its staging area, which
  // plain stores leave unused.
  if (p.cluster > 1 && !a.tma_out)
    a.cluster_early = cluster_recv_bytes(p.narrow, M, p.tn, p.cluster) <= kStagingBytes ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (p.tn) {
    case 16:
      return launch_tn<16>(mx, my, mo, mw, a, p.ctas, a.stages, s);
    case 32:
      return launch_tn<32>(mx, my, mo, mw, a, p.ctas, a.stages, s);
    case 64:
      return launch_tn<64>(mx, my, mo, mw, a, p.ctas, a.stages, s);
    case 128:
      return launch_tn<128>(mx, my, mo, mw, a, p.ctas, a.stages, s);
    case 256:
      if (p.pair) return launch_tn<256, kVarPair>(mx, my, mo, mw, a, p.ctas, a.stages, s);
      if (p.narrow) return launch_tn<256, kVarNarrow>(mx, my, mo, mw, a, p.ctas, a.stages, s);
      return launch_tn<256>(mx, my, mo, mw, a, p.ctas, a.stages, s);
    default:
      return set_error(I8L_ENOTSUP, "no kernel for tile width %d", p.tn);
  }
}

}  // namespace i8l

extern "C" int i8l_w8a8_mm(const int8_t *A, int64_t lda, const int8_t *W, int64_t ldw,
                           const float *sa, int32_t sa_per_row, const float *sb,
                           int32_t sb_per_col, const void *bias, int32_t bias_dtype, void *out,
                           int32_t out_dtype, int64_t ldc, int32_t M, int32_t N, int32_t K,
                           const i8l_tile *tile, void *workspace, size_t ws_bytes, void *stream) {
  return gemm_run(A, lda, W, ldw, sa, sa_per_row, sb, sb_per_col, bias, bias_dtype, out, out_dtype,
                  ldc, M, N, K, tile, workspace, ws_bytes, stream, nullptr);
}

extern "C" int i8l_w8a8_mm_quant_act(const void *X, int32_t x_dtype, int64_t ldx, int32_t precise_div,
                                     const int8_t *W, int64_t ldw, const float *sb,
                                     int32_t sb_per_col, const void *bias, int32_t bias_dtype,
                                     void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N,
                                     int32_t K, const i8l_tile *tile, void *workspace,
                                     size_t ws_bytes, void *stream) {
  if (x_dtype != I8L_BF16 && x_dtype != I8L_F16)
    return set_error(I8L_ENOTSUP, "activation dtype code %d not supported (bf16 or fp16)", x_dtype);
  if (M > 0 && N > 0 && K > 0) {
    if (!X) return set_error(I8L_EINVAL, "NULL activation pointer");
    if (ldx < K) return set_error(I8L_EINVAL, "activation row stride %lld < K=%d", static_cast<long long>(ldx), K);
    if (reinterpret_cast<uintptr_t>(X) % 16 || (ldx * 2) % 16)
      return set_error(I8L_ENOTSUP, "the activation and its row stride must be 16-byte aligned");
  }
  const ActQuant aq{X, x_dtype, ldx, precise_div};
  // The int8 A pointer and stride stand in for X's bytes: only the direct loads read A,
  // and through aq.  (X's rows are 2*ldx bytes apart and hold at least K bytes.)
  return gemm_run(static_cast<const int8_t *>(X), ldx * 2, W, ldw, nullptr, 0, sb, sb_per_col, bias,
                  bias_dtype, out, out_dtype, ldc, M, N, K, tile, workspace, ws_bytes, stream, &aq);
}

// ------------------------------------------------------------------ no-allocation entry
//
// Some callers cannot allocate device memory at the point where they run a GEMM: a
// host that owns all device memory through its own fixed arena and forbids
// allocation inside its execute callback, code that must not hit cudaMalloc's
// implicit device synchronisation on a latency-critical path, or a foreign-language
// caller with no binding to an allocator.  For them, i8l_w8a8_mm_noalloc takes its
// split-K scratch from a fixed array compiled into this library.
//
// The array is a file-scope __device__ variable: every GPU that loads the library
// holds kNoAllocScratchBytes of it until the process exits.  Host code cannot use the
// array's name as a device address (on the host it is only a stand-in symbol), so the
// device address is looked up once per device with cudaGetSymbolAddress, with that
// device current, on the first call made on it.

namespace i8l {

constexpr size_t kNoAllocScratchBytes = I8L_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void *g_noalloc_addr[64];

// Device address of g_noalloc_scratch on the current device (resolved on first use).
static int noalloc_scratch(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(I8L_EINVAL, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return I8L_OK;
}

}  // namespace i8l

extern "C" int i8l_w8a8_mm_noalloc(const int8_t *A, int64_t lda, const int8_t *W, int64_t ldw,
                                   const float *sa, int32_t sa_per_row, const float *sb,
                                   int32_t sb_per_col, const void *bias, int32_t bias_dtype,
                                   void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N,
                                   int32_t K, const i8l_tile *tile, void *stream) {
  if (M < 0 || N < 0 || K < 0) return set_error(I8L_EINVAL, "negative size M=%d N=%d K=%d", M, N, K);
  // Scratch this problem needs under this tile (host arithmetic only).
  size_t need = 0;
  if (M > 0 && N > 0 && K > 0 && K % 16 == 0) {
    Plan p;
    if (make_plan(M, N, K, tile, &p) == I8L_OK) need = p.ws_bytes;
  }
  if (need > kNoAllocScratchBytes)
    return set_error(I8L_EWORKSPACE,
                     "i8l_w8a8_mm_noalloc: this problem needs %zu bytes of split-K scratch, more "
                     "than the library's fixed %zu; pass a tile with split=1 (no scratch) or call "
                     "i8l_w8a8_mm with a workspace",
                     need, kNoAllocScratchBytes);
  void *ws = nullptr;
  int e = noalloc_scratch(&ws);
  if (e) return e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The counters and partial-sum slots must start at zero.  Kernels leave them
  // zeroed, but a call that ended in an error may not have: clear them every call.
  if (need) {
    cudaError_t ce = cudaMemsetAsync(ws, 0, need, s);
    if (ce != cudaSuccess) return cuda_error(ce, "cudaMemsetAsync(no-alloc scratch)");
  }
  return i8l_w8a8_mm(A, lda, W, ldw, sa, sa_per_row, sb, sb_per_col, bias, bias_dtype, out,
                     out_dtype, ldc, M, N, K, tile, ws, kNoAllocScratchBytes, stream);
}
