/*
 * int8_linear_b200.h - C ABI of the B200 (sm_100a) W8A8 linear-layer library.
 *
 * Every entry point takes plain device pointers, element strides and sizes and a
 * CUDA stream handle (a cudaStream_t passed as void*; NULL is the legacy default
 * stream).  Nothing here allocates device memory: the caller owns every buffer,
 * including the split-K workspace.  Calls are asynchronous on the given stream and
 * never synchronise the host.
 *
 * Return codes: I8L_OK, or one of the I8L_E* codes; i8l_last_error() gives a
 * one-line message for the calling host thread.  I8L_ENOTSUP means "this kernel
 * does not take that shape/dtype/layout; the caller should fall back"; it maps to
 * int8_linear.NotSupported in the Python layer.  I8L_EINVAL maps to ValueError.
 *
 * The reference (AshrithaG/int8-linear) is a Python/Triton package with no native
 * ABI; each entry below replaces the Triton launch of one reference function, cited
 * by file:line inside that project.
 */
#ifndef INT8_LINEAR_B200_H
#define INT8_LINEAR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---------------------------------------------------------- */
#define I8L_OK 0
#define I8L_ENOTSUP 1   /* shape/dtype/layout the kernel declines (NotSupported)   */
#define I8L_EINVAL 2    /* inconsistent arguments (ValueError)                     */
#define I8L_ECUDA 3     /* a CUDA runtime/driver call failed (RuntimeError)        */
#define I8L_EWORKSPACE 4 /* workspace missing or smaller than i8l_workspace_size() */

/* ---- element type codes ---------------------------------------------------- */
#define I8L_BF16 0
#define I8L_F16 1
#define I8L_F32 2
#define I8L_I32 3 /* GEMM output only: the raw int32 product (reference raw=True) */

/* ---- GEMM tile selection ---------------------------------------------------- */
/*
 * One GEMM tile configuration.  A zero-initialised struct (or a NULL pointer)
 * asks the library for its own choice.
 *   swap_ab = 1: the weight rows fill the 128-row MMA M side and the tokens are the
 *                MMA N side, tok_tile in {16,32,64,128,256} (decode shapes);
 *   swap_ab = 0: tokens fill the 128-row MMA M side, w_tile in {128,256}.
 *   stages:      shared-memory ring depth (0 = the most that fits);
 *   ctas:        persistent CTAs (0 = one per SM);
 *   group:       tiles walked together along the 128-row side for L2 reuse (>=1);
 *   split:       how K is shared out (int32 partial sums are always reduced exactly):
 *                0 = the library's choice; 1 = whole tiles; 2 = stream-K over the SMs,
 *                partial sums reduced through the workspace; 3 = cluster split-K:
 *                the CTAs of a thread-block cluster split one tile's K and reduce over
 *                distributed shared memory, no workspace: swap_ab tiles of up to 256
 *                tokens and, without swap_ab above 16 tokens, 128-token tiles of w_tile
 *                weight rows, each CTA finishing one in `cluster` of the tile's 16-column
 *                chunks from the others' partial sums (plain stores for the latter);
 *                without swap_ab at most 16 tokens: narrow tiles, w_tile 256); 4 = CTA pairs
 *                (cta_group::2) on 128 x 256 tiles; 5 = CUDA-core tiles for batches of
 *                at most tok_tile in {1, 2, 4, 8, 16} tokens (w_tile 0, swap_ab 0): each CTA
 *                owns whole output columns (dp4a int8 dot products, no split-K, no
 *                workspace), its weight rows streamed into shared memory by 1-D bulk
 *                copies; `ctas` and `stages` apply;
 *   cluster:     CTAs per cluster for split = 3 (0 = the library's choice, <= 8);
 *   store:       output path: 0 = the library's choice, 1 = TMA stores through
 *                shared memory, 2 = plain stores;
 *   act:         activation path of swap_ab tiles: 0 = the library's choice, 1 = TMA
 *                loads, 2 = plain loads by the epilogue warps straight after the
 *                dependency wait (needs M <= tok_tile, one tile or cluster segment
 *                per CTA, and that segment's k-blocks all in the ring at once).
 */
typedef struct i8l_tile {
  int32_t swap_ab;
  int32_t tok_tile;
  int32_t w_tile;
  int32_t stages;
  int32_t ctas;
  int32_t group;
  int32_t split;
  int32_t cluster;
  int32_t store;
  int32_t act;
} i8l_tile;

/*
 * out[M,N] = (A[M,K] @ W[N,K]^T) * sa * sb + bias, int8 x int8 -> int32 on the
 * tcgen05 tensor cores, dequantised in fp32 in the epilogue and rounded once to the
 * output type.  With out_dtype == I8L_I32 the exact int32 product is stored and
 * sa/sb/bias are ignored.
 *
 *   A   int8, row m at A + m*lda  (K contiguous); lda*1 and A must be 16-byte aligned
 *   W   int8, row n at W + n*ldw  (K contiguous); this is the [K,N] view b_q with
 *       strides (1, ldw) that the reference takes; 16-byte alignment as for A
 *   sa  float32, M values (sa_per_row=1) or one value
 *   sb  float32, N values (sb_per_col=1) or one value
 *   bias NULL or N values of bias_dtype (I8L_BF16/I8L_F16/I8L_F32)
 *   out row m at out + m*ldc elements of out_dtype (I8L_BF16/F16/F32/I32)
 *   K must be a positive multiple of 16.
 *   workspace/ws_bytes: at least i8l_workspace_size(...) bytes, zero-filled by the
 *       caller ONCE when first allocated; every call leaves it zero-filled again.
 *       Calls that share a workspace must not overlap on the GPU.
 *
 * Replaces the reference's launcher w8a8_mm (int8_linear/kernel.py:202-257) and
 * its Triton kernel _w8a8_mm (int8_linear/kernel.py:63-124).
 */
int i8l_w8a8_mm(const int8_t *A, int64_t lda, const int8_t *W, int64_t ldw,
                const float *sa, int32_t sa_per_row, const float *sb,
                int32_t sb_per_col, const void *bias, int32_t bias_dtype,
                void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N,
                int32_t K, const i8l_tile *tile, void *workspace,
                size_t ws_bytes, void *stream);

/*
 * i8l_w8a8_mm with the activation's per-token quantisation fused into the GEMM:
 * X is the bf16 (x_dtype I8L_BF16) or fp16 (I8L_F16) activation [M,K], rows ldx
 * elements apart, 16-byte aligned.  The kernel quantises each token row as the plain
 * per-token quantiser does (scale = absmax/127, q = rint(x * 127/absmax) saturated to
 * [-128, 127], absmax over all K; precise_div = 1 for IEEE division, 0 for Triton's
 * full-range division) and multiplies; the result equals i8l_quant_rows followed by
 * i8l_w8a8_mm bit for bit, with one launch instead of two and no int8 copy of X in
 * HBM.  Other arguments as i8l_w8a8_mm (there is no sa).
 *
 * Tiles that take it: tensor-core tiles with direct activation loads (swap_ab,
 * M <= tok_tile, one tile or cluster segment per CTA, at most `stages` k-blocks per CTA;
 * tile->act 0 or 2), and CUDA-core tiles (split 5; the kernel quantises the batch in its
 * prologue, 16-byte aligned rows with strides a multiple of 8 elements); any other
 * returns I8L_ENOTSUP and the caller quantises separately.
 *
 * Replaces the reference's o_proj input path, vLLM's scaled_int8_quant followed by
 * w8a8_mm (bench/fuse_quant.py:234, int8_linear/vllm_fuse_patch.py:13-14, where the
 * reference notes that o_proj still quantises its own input).
 */
int i8l_w8a8_mm_quant_act(const void *X, int32_t x_dtype, int64_t ldx, int32_t precise_div,
                          const int8_t *W, int64_t ldw, const float *sb,
                          int32_t sb_per_col, const void *bias, int32_t bias_dtype,
                          void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N,
                          int32_t K, const i8l_tile *tile, void *workspace,
                          size_t ws_bytes, void *stream);

/*
 * add + RMSNorm + per-token quantisation of X followed by the GEMM with its result, in
 * one launch for decode batches of at most 8 tokens: the same bits as
 * i8l_add_rmsnorm_quant(x, residual, norm_weight) and then i8l_w8a8_mm(q, W, scale, sb),
 * without the int8 activation or its scales ever reaching HBM.  Every CTA of the
 * CUDA-core GEMM (split 5) normalises and quantises the whole batch itself, with the
 * standalone kernel's thread layout and reduction order, before its dot products; CTA 0
 * writes residual_out = x + residual (rounded to act_dtype), as the standalone kernel
 * does.  x, residual, residual_out: act_dtype (I8L_BF16/I8L_F16) rows of K values,
 * 16-byte aligned, row strides multiples of 8; residual and residual_out NULL together
 * for a plain RMSNorm.  Other arguments as i8l_w8a8_mm (there is no sa: the per-token
 * scales are the quantiser's).  tile: NULL or zeroed for the CUDA-core tile holding M,
 * else a split-5 tile; I8L_ENOTSUP for larger batches, other tiles, unaligned rows or a
 * K whose rows hold more than 8 vectors per thread at this batch (the caller then runs
 * the two steps).
 * Replaces the reference's decoder-layer pair add_rmsnorm_quant -> int8 linear
 * (int8_linear/vllm_fuse_patch.py:41-52, bench/fuse_quant.py:230-236).
 */
int i8l_rmsnorm_w8a8_mm(const void *x, int64_t ldx, const void *residual, int64_t ldr,
                        const void *norm_weight, int32_t act_dtype, int32_t w_dtype, float eps,
                        int32_t precise_div, void *residual_out, int64_t ldro, const int8_t *W,
                        int64_t ldw, const float *sb, int32_t sb_per_col, const void *bias,
                        int32_t bias_dtype, void *out, int32_t out_dtype, int64_t ldc, int32_t M,
                        int32_t N, int32_t K, const i8l_tile *tile, void *stream);

/*
 * SiLU-and-mul + per-token quantisation of gate_up = [gate | up] (rows of 2K values,
 * ld elements apart) followed by the GEMM with the [M, K] result, in one launch: the same
 * bits as i8l_silu_mul_quant and then i8l_w8a8_mm.  Same tile rules as
 * i8l_rmsnorm_w8a8_mm.  Replaces the reference's MLP pair silu_mul_quant -> down_proj
 * (int8_linear/vllm_fuse_patch.py:55-59, bench/fuse_quant.py:237-238).
 */
int i8l_silu_mul_w8a8_mm(const void *gate_up, int64_t ld, int32_t act_dtype, int32_t precise_div,
                         int32_t round_silu, const int8_t *W, int64_t ldw, const float *sb,
                         int32_t sb_per_col, const void *bias, int32_t bias_dtype, void *out,
                         int32_t out_dtype, int64_t ldc, int32_t M, int32_t N, int32_t K,
                         const i8l_tile *tile, void *stream);

/*
 * i8l_w8a8_mm for callers that cannot allocate device memory.  No counterpart in
 * the reference (its Triton kernel needed no scratch).
 *
 * Who needs it: a host that owns all device memory through a fixed arena and forbids
 * allocation inside its execute callback, a latency-critical path that must not run
 * into cudaMalloc's implicit device synchronisation, or a caller from another
 * language with no allocator binding.  The caller still passes the inputs and the
 * output; only the split-K scratch changes: it is a fixed array of
 * I8L_NOALLOC_SCRATCH_BYTES compiled into the library, which every GPU that loads the
 * library holds until the process exits.  This call allocates nothing.
 *
 * - A problem whose scratch (i8l_workspace_size for the same tile) exceeds
 *   I8L_NOALLOC_SCRATCH_BYTES is rejected with I8L_EWORKSPACE and a message naming
 *   both sizes; a tile with split = 1 needs no scratch.  With the default tiles,
 *   decode batches up to 64 tokens fit.
 * - The first call on a device looks up the array's device address
 *   (cudaGetSymbolAddress) with that device current; make that first call before
 *   any stream capture.
 * - Every call on a device shares the one array and clears the part it needs before
 *   its kernel runs, so calls whose GPU work overlaps (other streams, other host
 *   threads, graph branches) race: serialise them.
 */
#define I8L_NOALLOC_SCRATCH_BYTES (8u << 20)
int i8l_w8a8_mm_noalloc(const int8_t *A, int64_t lda, const int8_t *W, int64_t ldw,
                        const float *sa, int32_t sa_per_row, const float *sb,
                        int32_t sb_per_col, const void *bias, int32_t bias_dtype,
                        void *out, int32_t out_dtype, int64_t ldc, int32_t M, int32_t N,
                        int32_t K, const i8l_tile *tile, void *stream);

/*
 * Bytes of workspace i8l_w8a8_mm needs for this problem and tile (tile may be
 * NULL for the library's choice).  Host-only, no CUDA calls beyond a cached
 * device-property query.  Replaces nothing in the reference (Triton's kernel kept
 * no cross-CTA state); the workspace exists for the exact int32 split-K reduction.
 */
size_t i8l_workspace_size(int32_t M, int32_t N, int32_t K, const i8l_tile *tile);

/*
 * The tile the library picks when none is given (the untuned heuristic).
 * Replaces default_config (int8_linear/kernel.py:127-134).
 */
int i8l_default_tile(int32_t M, int32_t N, int32_t K, i8l_tile *tile_out);

/*
 * add + RMSNorm + per-token int8 quantisation, one token row per CTA:
 *   x' = x (+ residual) in fp32; rout = x' rounded to act_dtype (if residual);
 *   var = sum(x'^2)/K; xn = x' * rsqrt(var + eps);
 *   y = act(w_dtype(xn) * weight); scale = max|y|/127; q = rint(y*127/max|y|).
 * x, residual, rout: act_dtype (I8L_BF16 or I8L_F16), rows at ld* elements.
 * weight: K values of w_dtype (I8L_BF16/F16/F32).  residual/rout may be NULL
 * together.  q: int8 rows at ldq; scale: M float32.
 * Replaces add_rmsnorm_quant (int8_linear/fused_quant.py:95-110) and its kernel
 * _add_rmsnorm_quant_kernel (int8_linear/fused_quant.py:56-73) with the row
 * quantiser _quantize_row (int8_linear/fused_quant.py:41-53).
 */
int i8l_add_rmsnorm_quant(const void *x, int64_t ldx, const void *residual,
                          int64_t ldr, const void *weight, int32_t act_dtype,
                          int32_t w_dtype, int8_t *q, int64_t ldq, float *scale,
                          void *rout, int64_t ldro, int32_t M, int32_t K,
                          float eps, int32_t precise_div, void *stream);

/*
 * SiLU-and-mul + per-token int8 quantisation: gate = row[0:I], up = row[I:2I];
 *   a = g/(1+exp(-g)); a rounded to act_dtype if round_silu; y = act(a*u);
 *   then the row quantiser as above.
 * gate_up: act_dtype rows of 2I elements at ld; q: int8 rows at ldq; scale: M f32.
 * Replaces silu_mul_quant (int8_linear/fused_quant.py:113-124) and
 * _silu_mul_quant_kernel (int8_linear/fused_quant.py:76-88).
 */
int i8l_silu_mul_quant(const void *gate_up, int64_t ld, int32_t act_dtype,
                       int8_t *q, int64_t ldq, float *scale, int32_t M,
                       int32_t I, int32_t precise_div, int32_t round_silu,
                       void *stream);

/*
 * Plain dynamic per-token int8 quantisation of an act_dtype [M,K] matrix (rows at
 * ldx elements, so a column slice of a wider matrix needs no copy).  The same
 * row quantiser as above.  The reference reaches this step through vLLM's
 * scaled_int8_quant (called in bench/fuse_quant.py:234); its arithmetic is the
 * reference's torch `quant` (tests/test_fused_quant.py:26-31).
 */
int i8l_quant_rows(const void *x, int64_t ldx, int32_t act_dtype, int8_t *q,
                   int64_t ldq, float *scale, int32_t M, int32_t K,
                   int32_t precise_div, void *stream);

/*
 * The two quantisers above for a token row that is split across GPUs (the input of a
 * row-parallel linear under tensor parallelism).  With absmax_out (M floats) each
 * row's local max|y| is written and nothing is quantised; after the caller takes the
 * MAX over the GPUs, the call with absmax_in quantises with that shared absmax, so
 * each GPU's int8 values and scale are exactly those one GPU would compute for the
 * whole row.  Both pointers NULL: same as i8l_silu_mul_quant / i8l_quant_rows.  No
 * reference counterpart (the reference is single-GPU).
 */
int i8l_silu_mul_quant_ex(const void *gate_up, int64_t ld, int32_t act_dtype, int8_t *q,
                          int64_t ldq, float *scale, int32_t M, int32_t I,
                          int32_t precise_div, int32_t round_silu,
                          const float *absmax_in, float *absmax_out, void *stream);
int i8l_quant_rows_ex(const void *x, int64_t ldx, int32_t act_dtype, int8_t *q,
                      int64_t ldq, float *scale, int32_t M, int32_t K,
                      int32_t precise_div, const float *absmax_in, float *absmax_out,
                      void *stream);

/*
 * out[M,N] = cast(((float(acc) * sa) * sb) + bias) for an int32 product computed
 * elsewhere, e.g. the SUM over GPUs of a row-parallel layer's partial products: the
 * GEMM epilogue's arithmetic, so the result equals a one-GPU i8l_w8a8_mm bit for bit.
 * acc rows at lda, out rows at ldo (I8L_BF16/F16/F32).  Same role as the epilogue of
 * the reference kernel (int8_linear/kernel.py:105-120).
 */
int i8l_dequant_i32(const int32_t *acc, int64_t lda, const float *sa, int32_t sa_per_row,
                    const float *sb, int32_t sb_per_col, const void *bias,
                    int32_t bias_dtype, void *out, int32_t out_dtype, int64_t ldo,
                    int32_t M, int32_t N, void *stream);

/* One-line message for the last non-OK return on this host thread. */
const char *i8l_last_error(void);

/*
 * Device status word, written by kernels whose bounded waits gave up (a wait that
 * should take microseconds ran past its limit).  i8l_read_status() synchronises
 * the device and returns the word (0 = clean); i8l_clear_status() resets it.
 * No reference counterpart (Triton kernels have no in-kernel waits).
 */
int i8l_read_status(int32_t *status_out);
int i8l_clear_status(void);

/*
 * Programmatic dependent launch (process-wide, off by default).  When on, every kernel
 * of the library is launched so that it may start while the previous kernel in the
 * stream is still running: it sets up, and a GEMM loads the weight tiles of its first
 * pipeline stages, then waits for the previous kernel before reading activations or
 * scales or writing anything.  Only turn it on when weights (W, sb, bias, norm gamma)
 * are never written by the kernel launched just before (true for inference).
 * No reference counterpart (Triton launches are stream-ordered).
 */
int i8l_set_pdl(int32_t enable);
int32_t i8l_get_pdl(void);

/* Library version string and the compiled target, e.g. "0.1.0 sm_100a". */
const char *i8l_version(void);

/* ---- tensor parallelism over NVLink peer memory --------------------------------
 * A row-parallel W8A8 layer (o_proj, down) leaves every GPU an int32 partial product;
 * a row-split activation needs the global per-token absmax before it is quantised.
 * These entry points do the exchange themselves, GPU to GPU over NVLink, fused with
 * the computation that follows, in place of an NCCL collective plus a separate kernel.
 * Every GPU owns one exchange buffer (i8l_peer_alloc) and opens every peer's buffer
 * through its CUDA IPC handle (i8l_peer_open); the host exchanges the 64-byte handles
 * (e.g. torch.distributed.all_gather_object).  All GPUs must make the same calls in
 * the same order (SPMD); each call's waits for peers are bounded by timeout_ns, after
 * which the status word (i8l_read_status) holds bit 64 and the outputs are invalid.
 * No reference counterpart: the reference is single-GPU.
 */
#define I8L_MAX_RANKS 8
#define I8L_PEER_HANDLE_BYTES 64

typedef struct i8l_peer_comm {
  void *bases[I8L_MAX_RANKS]; /* every GPU's exchange buffer, this GPU's at [rank]  */
  uint32_t *epochs;           /* this GPU's call counters: max_rows zeroed uint32    */
  int32_t rank, world;        /* world <= I8L_MAX_RANKS                              */
  int64_t slot_bytes;         /* bytes per (parity, source) inbox slot, multiple of 16 */
  int32_t max_rows;           /* rows per call (and epoch counters)                  */
  uint64_t timeout_ns;        /* bound on each wait for a peer (0 = 2 s)             */
  /* Rows per call from which the row-parallel exchanges (i8l_tp_allreduce_*) run two-shot:
   * each GPU sums its 1/world of the columns from every GPU's partials (reduce-scatter)
   * and sends the sums to the others (all-gather), (world-1)/world x 16 bytes per column
   * sent instead of (world-1) x 8.  0 = the library's choice (16 rows with 4 or more
   * GPUs, else one-shot), < 0 = always one-shot.  Needs N % (4 x world) == 0. */
  int32_t two_shot_rows;
} i8l_peer_comm;

/* Bytes of one exchange buffer: 2 parities x world source slots (0 for a slot that is
 * no positive multiple of 16 or a world outside [1, I8L_MAX_RANKS]).  Data travels as
 * 8-byte words of {4-byte value, 4-byte call epoch}, so a row of N int32 takes 8*N
 * bytes of a slot and a row's absmax 16 bytes. */
size_t i8l_peer_buffer_bytes(int64_t slot_bytes, int32_t world);
/* cudaMalloc + zero an exchange buffer on the current device; writes its IPC handle
 * (I8L_PEER_HANDLE_BYTES) to handle_out. */
int i8l_peer_alloc(size_t bytes, void **ptr, void *handle_out);
/* Map a peer's exchange buffer from its IPC handle (peer access enabled lazily). */
int i8l_peer_open(const void *handle, void **ptr);
int i8l_peer_close(void *ptr);
int i8l_peer_free(void *ptr);

/* out[M,N] = cast(((float(sum over GPUs of partial) * sa) * sb) + bias): the one-GPU
 * GEMM epilogue applied to the exact int32 sum.  N and ldp multiples of 4, N <= 8192,
 * M*N*8 <= slot_bytes, M <= max_rows. */
int i8l_tp_allreduce_dequant(const i8l_peer_comm *comm, const int32_t *partial, int64_t ldp,
                             const float *sa, int32_t sa_per_row, const float *sb,
                             int32_t sb_per_col, const void *bias, int32_t bias_dtype, void *out,
                             int32_t out_dtype, int64_t ldo, int32_t M, int32_t N, void *stream);

/* The same sum and dequant to the activation dtype (h, written to h_out if not NULL),
 * then i8l_add_rmsnorm_quant(h, residual, weight) in the same pass: q, scale and
 * residual_out equal the separate calls bit for bit.  N % 8 == 0. */
int i8l_tp_allreduce_add_rmsnorm_quant(
    const i8l_peer_comm *comm, const int32_t *partial, int64_t ldp, const float *sa,
    int32_t sa_per_row, const float *sb, int32_t sb_per_col, const void *bias, int32_t bias_dtype,
    const void *residual, int64_t ldr, const void *weight, int32_t act_dtype, int32_t w_dtype,
    int8_t *q, int64_t ldq, float *scale, void *residual_out, int64_t ldro, void *h_out,
    int64_t ldh, int32_t M, int32_t N, float eps, int32_t precise_div, void *stream);

/* Per-token int8 of this GPU's column slice x[M, K] of rows split over the GPUs, with
 * the scale of the whole row (absmax = MAX over the GPUs): every GPU's q slice and the
 * (replicated) scale equal i8l_quant_rows on the whole row. */
int i8l_tp_quant_rows(const i8l_peer_comm *comm, const void *x, int64_t ldx, int32_t act_dtype,
                      int8_t *q, int64_t ldq, float *scale, int32_t M, int32_t K,
                      int32_t precise_div, void *stream);

/* The same for silu(gate)*up of this GPU's [gate_r | up_r] slice, [M, 2I] -> q [M, I]. */
int i8l_tp_silu_mul_quant(const i8l_peer_comm *comm, const void *gate_up, int64_t ld,
                          int32_t act_dtype, int8_t *q, int64_t ldq, float *scale, int32_t M,
                          int32_t I, int32_t precise_div, int32_t round_silu, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* INT8_LINEAR_B200_H */
