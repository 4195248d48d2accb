/*
 * lora_b200.h -- C ABI of the B200 (sm_100a) LoRA-linear kernels.
 *
 * Computes the LoRA linear  y = x.W^T + bias + sum_a s_a (x.A_a^T).B_a^T  and
 * its pieces, behind plain pointers and sizes so that any host language can
 * bind it (ctypes, cgo, JNI, N-API).  Storage layouts follow PyTorch / PEFT:
 *   W    = nn.Linear.weight   [N, K] row-major
 *   A    = lora_A.weight      [R, K] row-major
 *   B    = lora_B.weight      [N, R] row-major
 * Row strides ("ld*") are in elements; the innermost stride is always 1.
 *
 * Conventions shared by every entry point:
 *   - all tensor pointers are device pointers on the current CUDA device;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every launch
 *     goes on it and no entry point synchronises the host;
 *   - the return value is a lora_status; no exception crosses the ABI;
 *   - dtype is LORA_F16 or LORA_BF16 for activations and weights; some
 *     intermediate z buffers may be LORA_F32 where stated;
 *   - most kernels launch with programmatic dependent launch and may start
 *     while the kernel launched just before them on `stream` is still running.
 *     Until that kernel has completed they read only weights (w, a, b,
 *     lora_A / lora_B tables, offsets, ranks); activations, z, tile tables and
 *     every write come after.  So a kernel that WRITES a weight must not be the
 *     launch immediately before an entry point that reads it (any other launch,
 *     an event wait or a synchronisation in between is enough), or set the
 *     environment variable LORA_B200_PDL=0 (read once per process) for plain
 *     stream order throughout.
 *
 * Each declaration names the reference function (lishenghui/probe,
 * loraforge_kernels/, file:line) whose GPU work it replaces.
 */
#ifndef LORA_B200_H
#define LORA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LORA_API __attribute__((visibility("default")))
#else
#define LORA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum lora_status {
  LORA_OK = 0,
  LORA_ERR_SHAPE = 1,       /* inconsistent or unsupported sizes            */
  LORA_ERR_ALIGN = 2,       /* pointer / stride alignment not met           */
  LORA_ERR_DTYPE = 3,       /* unsupported dtype combination                */
  LORA_ERR_DEVICE = 4,      /* no usable sm_100 device                      */
  LORA_ERR_INDEX = 5,       /* adapter id / offset out of range             */
  LORA_ERR_CUDA = 6,        /* a CUDA runtime / driver call failed          */
  LORA_ERR_TIMEOUT = 7,     /* a bounded device wait ran out                */
  LORA_ERR_WORKSPACE = 8,   /* workspace missing or too small               */
  LORA_ERR_UNSUPPORTED = 9, /* valid request this build does not implement  */
  LORA_ERR_ARG = 10         /* NULL pointer or invalid argument             */
};

enum lora_dtype { LORA_F16 = 0, LORA_BF16 = 1, LORA_F32 = 2 };

/* Layout of a LoRA up-projection B as seen by the expand kernels. */
enum lora_b_layout {
  LORA_B_PEFT = 0,      /* B[n * ldb + j]  : lora_B.weight [N, R]            */
  LORA_B_RANK_MAJOR = 1 /* B[j * ldb + n]  : flat table [sum R, N]           */
};

/* ABI version of this library (bumped on any signature change). */
LORA_API int lora_b200_abi_version(void);

/* Human-readable name of a lora_status value. */
LORA_API const char* lora_b200_status_string(int status);

/* Reads and clears the device-side error word of `device` (a bounded wait
 * that ran out, or an adapter id out of range seen on the device).  Waits for
 * the device to finish its queued work.  *code = 0 when nothing was recorded.
 * No reference counterpart: the reference's Triton kernels have no device
 * error channel. */
LORA_API int lora_b200_device_error(int device, int* code);

/* ---------------------------------------------------------------------------
 * Dense fused LoRA GEMM on tcgen05 tensor cores (TMA -> smem -> TMEM).
 *
 *   out[M,N] = alpha * ( x[M,K] . w[N,K]^T  +  z[M,R] . bw[N,R]^T ) + bias[N]
 *
 * The second product is the LoRA expand folded in as an extra K-slice
 * ("K-concat"): z = s * x . A^T comes from lora_shrink, bw holds lora_B.weight
 * columns.  For accuracy the caller usually passes z as a hi/lo pair
 * [round(s.z) | s.z - round(s.z)] against bw = [B | B] (R = 2 * rank).
 * R = 0 (z, bw NULL) gives a plain linear.
 * lo_offset > 0 writes the result itself as a hi/lo pair: out[:, c] =
 * round(v) and out[:, c + lo_offset] = round(v - round(v)) (lo_offset >= N,
 * ldo >= N + lo_offset) -- the large-rank shrink producing such a z.
 * Requirements: 16-byte aligned pointers; ldx, ldw multiples of 8 and >= K;
 * K a multiple of 8; when R > 0, ldz, ldbw >= R and multiples of 8 (columns
 * beyond R are never read).  bias may be NULL.
 * Replaces: _fused_lora_gemm_kernel / fused_gemm (fused_linear.py:229-317),
 * _kconcat (fused_linear.py:676-677), the cuBLAS GEMM of _concat / _hybrid
 * (fused_linear.py:362-373) and cutlass_gemm (csrc/cutlass_gemm_gate.cu:91-106).
 * ------------------------------------------------------------------------- */
LORA_API int lora_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
              const void* bw, int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M,
              int64_t N, int64_t K, int64_t R, float alpha, int64_t lo_offset, int dtype, void* stream);
/* lora_gemm with a workspace for its split tail: when the tiles do not fill a
 * whole number of waves of resident CTA pairs, the tiles of the last, partial
 * wave are cut along K across the otherwise idle pairs; their fp32 partials
 * meet in the workspace and the last piece of each tile to finish sums them in
 * a fixed order (results do not depend on timing).  Workspace:
 * lora_gemm_workspace_size(M, N, K, R) bytes (0 = no split for this shape),
 * with a zeroed ticket region first, as lora_shrink's (its counters are
 * returned to zero by every call).  NULL or short workspace: no split.
 * Replaces the same reference functions as lora_gemm; the split is a B200
 * scheduling choice with no counterpart there. */
LORA_API size_t lora_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t R);
LORA_API int lora_gemm_ex(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                 const void* bw, int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M,
                 int64_t N, int64_t K, int64_t R, float alpha, int64_t lo_offset, int dtype,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Split-K rank shrink  z[M, z_width] = scale * x[M,K] . a[R,K]^T
 * Columns [R, z_width) of z are written with zeros.  z_dtype may be LORA_F32
 * or the input dtype.  z_split = 1 (input dtype only) also writes the
 * rounding residual: z[:, z_width + j] = round(v - round(v)), so [hi | lo]
 * carries ~16 mantissa bits into a K-concat expand (ldz >= 2 * z_width).
 * split_k slices of K run in separate CTAs; their fp32 partials are summed in
 * a fixed order by the last CTA to finish (no float atomics: the result is
 * deterministic).  split_k == 0 picks a value.
 * Workspace: lora_shrink_workspace_size() bytes.  It starts with a fixed
 * 256 KiB region of ticket counters that must be zero before the first use;
 * every call leaves them at zero again, so one workspace serves calls of any
 * shape (and CUDA-graph replays) without re-zeroing.  Calls that share one
 * workspace must not overlap on the GPU.
 * Replaces: _splitk_shrink_kernel + torch sum / splitk_lora_shrink
 * (splitk_lora.py:22-63,104-126), _splitk_shrink_partial / _splitk_shrink_atomic
 * (splitk_shrink.py:34-141), the x.A^T half of the fused_lora / tiled_lora /
 * classed_* / grouped_lora kernels (fused_lora.py:10-200) and build_ext's shrink
 * (fused_linear.py:662-673).
 * ------------------------------------------------------------------------- */
LORA_API size_t lora_shrink_workspace_size(int64_t M, int64_t R, int split_k);
LORA_API int lora_shrink_pick_split_k(int64_t M, int64_t K, int64_t R);
LORA_API int lora_shrink(const void* x, int64_t ldx, const void* a, int64_t lda, void* z, int64_t ldz,
                int z_dtype, int64_t z_width, int z_split, int64_t M, int64_t K, int64_t R,
                float scale, int dtype, int split_k, void* workspace, size_t workspace_bytes,
                void* stream);

/* The same split-K shrink for callers that cannot allocate device memory:
 * serving loops that cannot afford cudaMalloc's implicit device
 * synchronisation, or host frameworks that own all device memory and forbid
 * plugins from allocating.  It takes no
 * workspace: the ticket counters and partial sums live in an 8 MiB array of
 * device memory that the library holds on every GPU that loads it, until the
 * process exits.  The caller still passes x, a and z.  Limit: with split_k > 1
 * the partials need split_k * M * R * 4 bytes <= 8 MiB - 16 KiB
 * (lora_shrink_static_scratch_capacity()) and at most 4096 token tiles;
 * split_k == 0 picks the widest split that fits (down to 1, which needs no
 * scratch); an explicit split_k that does not fit returns LORA_ERR_WORKSPACE.
 * The first call on a device that splits K looks up the array's device
 * address (cudaGetSymbolAddress) and caches it.  A failed lookup returns
 * LORA_ERR_CUDA and is retried by the next call.  Device ordinals above 63 return LORA_ERR_DEVICE.
 * All calls share the one array: calls that overlap on the GPU (several
 * streams or threads) race and must be serialised on one stream.
 * No counterpart in the reference (its wrappers allocate per call). */
LORA_API size_t lora_shrink_static_scratch_capacity(void);
LORA_API int lora_shrink_static_scratch(const void* x, int64_t ldx, const void* a, int64_t lda,
                                        void* z, int64_t ldz, int z_dtype, int64_t z_width,
                                        int z_split, int64_t M, int64_t K, int64_t R, float scale,
                                        int dtype, int split_k, void* stream);

/* ---------------------------------------------------------------------------
 * Expand + add   out[M,N] = y[M,N] + scale * z[M,R] . B^T + bias[N]
 * y may be NULL (treated as zero) and may not alias out.  z is f32 or the
 * input dtype; an f32 z is carried into the tensor-core product as a
 * hi/lo pair of the input dtype (R <= 128), keeping ~16 mantissa bits.
 * b_layout selects LORA_B_PEFT ([N,R]) or LORA_B_RANK_MAJOR ([R,N]).
 * Replaces: _expand_add_kernel / expand_add (fused_linear.py:112-200),
 * _persistent_expand_add_kernel (splitk_lora.py:66-153) and the expand half of
 * the fused_lora / tiled_lora / classed_* / grouped_lora kernels
 * (fused_lora.py:10-200).
 * ------------------------------------------------------------------------- */
LORA_API int lora_expand_add(const void* y, int64_t ldy, const void* z, int64_t ldz, int z_dtype,
                    const void* b, int64_t ldb, int b_layout, const void* bias, void* out,
                    int64_t ldo, int64_t M, int64_t N, int64_t R, float scale, int dtype,
                    void* stream);

/* ---------------------------------------------------------------------------
 * Decode linear (small M): out[M,N] = x . w^T + scale * z . b^T + bias
 * Streams w once with split-K over CTAs; z ([M,R], input dtype or f32) comes
 * from lora_shrink and may be NULL when R == 0.  b is lora_B.weight [N,R].
 * scale * z is carried as a hi/lo pair of the input dtype.
 * M <= 256 when K, ldx and ldw are multiples of 8 and x, w are 16-byte
 * aligned (tcgen05 path: TMA-fed, K split over a thread-block cluster, no
 * workspace used); M <= 64 otherwise (register path, split-K through the
 * workspace).  Workspace: lora_decode_workspace_size() bytes, with the same
 * zeroed counter region as lora_shrink's.
 * Replaces: _decode_linear_kernel / build_decode_linear / decode_lora_linear
 * (decode_linear.py:13-100).
 * ------------------------------------------------------------------------- */
LORA_API size_t lora_decode_workspace_size(int64_t M, int64_t N, int split_k);
LORA_API int lora_decode_pick_split_k(int64_t M, int64_t N, int64_t K);
LORA_API int lora_decode_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z,
                       int64_t ldz, int z_dtype, const void* b, int64_t ldb, const void* bias,
                       void* out, int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t R,
                       float scale, int dtype, int split_k, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Small-M LoRA linear in one kernel: out[M,N] = x . w^T + scale * (x . a^T) . b^T + bias
 * a is lora_A.weight [R,K], b is lora_B.weight [N,R]; R == 0 (a, b NULL) gives
 * the base linear.  The shrink is computed inside the kernel that streams W
 * (z never written to memory).  M <= 256, R <= 128; K, ldx, ldw, lda
 * multiples of 8 and x, w, a 16-byte aligned, else LORA_ERR_UNSUPPORTED (use
 * lora_shrink + lora_decode_linear).
 * Up to 128 tokens (and ranks above 64) run the W-streaming skinny kernel,
 * where scale * z enters the expand as a hi/lo pair of the input dtype.  Above
 * 128 tokens with R <= 64 a split-K CTA-pair kernel runs instead (256-token
 * tiles, K split over a cluster, z kept in fp32); it exchanges partial tiles
 * through `workspace`, which must hold lora_linear_small_workspace_size(M, N, R)
 * bytes (16-byte aligned) and must not be used by a concurrent launch.  With a
 * smaller or NULL workspace the skinny kernel runs.
 * Replaces: decode_lora_linear (decode_linear.py:81-100) and the small-M
 * fused_lora_linear (fused_linear.py:527-551) -- shrink, expand and base in
 * one launch, where the reference re-derives x . A^T in every output tile.
 * ------------------------------------------------------------------------- */
LORA_API size_t lora_linear_small_workspace_size(int64_t M, int64_t N, int64_t R);
LORA_API int lora_linear_small(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* a, int64_t lda,
                               const void* b, int64_t ldb, const void* bias, void* out, int64_t ldo, int64_t M,
                               int64_t N, int64_t K, int64_t R, float scale, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Segmented multi-adapter LoRA (SGMV / BGMV).
 *
 * Adapter tables: a_flat rows (offsets[a] .. offsets[a]+ranks[a]) hold adapter
 * a's lora_A rows ([sum R, K] flat, or a padded [n, r_max, K] stack viewed as
 * [n*r_max, K] with offsets[a] = a*r_max).  B element (adapter a, rank j,
 * output n) is b[offsets[a]*N + j*b_sj + n*b_sn]: the flat rank-major table
 * [sum R, N] has (b_sj, b_sn) = (N, 1); a padded PEFT stack [n, N, r_max] has
 * (1, r_max).  offsets / ranks are int64 device arrays of n_adapters entries.
 *
 * lora_sgmv_schedule builds the tile list on the device: token blocks of 64
 * split wherever the adapter changes, from either per-token ids (ids[T]) or
 * segments (seg_start[S+1], seg_adapter[S]; pass ids = NULL).  The list lives
 * in `tiles`, an int32 buffer of lora_sgmv_tiles_size(T, S) bytes.  Ids out of
 * range become rank-0 tiles and set the device error word (LORA_ERR_INDEX).
 * Replaces the per-token / per-request adapter lookup of _ragged_shrink_kernel
 * (multilora.py:128-182), _bgmv_shrink_kernel (multilora.py:51-104),
 * _shrink / _expand of segmented_branch.py:12-60 and ragged_branch.py:6-40.
 * ------------------------------------------------------------------------- */
LORA_API size_t lora_sgmv_tiles_size(int64_t T, int64_t S);
LORA_API int lora_sgmv_schedule(const int64_t* ids, const int64_t* seg_start, const int64_t* seg_adapter,
                       int64_t T, int64_t S, int64_t n_adapters, int32_t* tiles,
                       size_t tiles_bytes, void* stream);

/* z[t, :] = scale * x[t] . A_{a(t)}^T for every token, zero beyond the
 * token's rank up to z_width.  Workspace: lora_sgmv_shrink_workspace_size()
 * bytes, with the same zeroed counter region as lora_shrink's.
 * rows (optional, int64 [T]): logical token t of the schedule reads x row
 * rows[t] and writes z row rows[t] (a gather / scatter by index, e.g. the
 * adapter-sorted order of lora_sgmv_sort or a rank bucket's positions);
 * NULL = identity. */
LORA_API size_t lora_sgmv_shrink_workspace_size(int64_t T, int64_t S, int64_t z_width, int split_k);
/* K split lora_sgmv_shrink uses when passed split_k <= 0 (size the workspace
 * with it).  No counterpart in the reference, whose segmented shrink does not
 * split K (segmented_branch.py:12-28). */
LORA_API int lora_sgmv_pick_split_k(int64_t T, int64_t K, int64_t r_max);
LORA_API int lora_sgmv_shrink(const void* x, int64_t ldx, const void* a_flat, int64_t lda,
                     const int64_t* offsets, const int64_t* ranks, int64_t n_adapters,
                     const int32_t* tiles, const int64_t* rows, void* z, int64_t ldz, int z_dtype, int64_t z_width,
                     int64_t T, int64_t S, int64_t K, int64_t r_max, float scale, int dtype,
                     int split_k, void* workspace, size_t workspace_bytes, void* stream);
/* lora_sgmv_shrink with the row count of a_flat ([a_rows, K]): knowing the
 * table's extent lets the tensor-core form (128-token blocks, adapter rows
 * gathered by TMA) bound its reads, so it is used when rows == NULL and the
 * rows are 16-byte aligned.  No counterpart in the reference (its shrink is
 * the Triton kernel of segmented_branch.py:12-28). */
LORA_API int lora_sgmv_shrink_ex(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                        const int64_t* offsets, const int64_t* ranks, int64_t n_adapters,
                        const int32_t* tiles, const int64_t* rows, void* z, int64_t ldz, int z_dtype,
                        int64_t z_width, int64_t T, int64_t S, int64_t K, int64_t r_max, float scale, int dtype,
                        int split_k, void* workspace, size_t workspace_bytes, void* stream);

/* out[t, :] = y[t, :] + scale * z[t, :r] . B_{a(t)}^T ; y may be NULL.
 * rows (optional): logical token t uses row rows[t] of y, z and out. */
LORA_API int lora_sgmv_expand(const void* y, int64_t ldy, const void* z, int64_t ldz, int z_dtype,
                     const void* b, int64_t b_sj, int64_t b_sn, const int64_t* offsets,
                     const int64_t* ranks, int64_t n_adapters, const int32_t* tiles,
                     const int64_t* rows, void* out,
                     int64_t ldo, int64_t T, int64_t S, int64_t N, int64_t r_max, float scale,
                     int dtype, void* stream);

/* The whole segmented branch in one call:
 *   out[t, :] = y[t, :] + (scale * x[t] . A_a^T) . B_a     a = adapter of t's tile
 * with a_flat [a_rows, K] (lda) and the rank-major b_flat [b_rows, N] (ldb,
 * each adapter's scale folded in, as the reference's tables), tiles from
 * lora_sgmv_schedule.  Three kernels on tensor cores: the shrink over (tile,
 * K slice) units writing fp32 partials, their sum in slice order into a
 * 16-bit hi/lo z, the expand over (tile, 256-column chunk) units with B and y
 * read by TMA.  y may be NULL (out = the LoRA term).  Workspace:
 * lora_sgmv_branch_workspace_size(T, S, K, r_max) bytes of scratch (no
 * zeroing needed; one buffer per stream).  Serves r_max <= 64, K and N
 * multiples of 64, leading dimensions multiples of 8, 16-byte aligned rows;
 * returns LORA_ERR_UNSUPPORTED otherwise (use lora_sgmv_shrink_ex +
 * lora_sgmv_expand).
 * Replaces the shrink / expand pair of ragged_branch.branch
 * (ragged_branch.py:6-40) and segmented_branch (segmented_branch.py:12-60). */
LORA_API size_t lora_sgmv_branch_workspace_size(int64_t T, int64_t S, int64_t K, int64_t r_max);
LORA_API int lora_sgmv_branch(const void* x, int64_t ldx, const void* y, int64_t ldy, const void* a_flat,
                     int64_t lda, int64_t a_rows, const void* b_flat, int64_t ldb, int64_t b_rows,
                     const int64_t* offsets, const int64_t* ranks, int64_t n_adapters, const int32_t* tiles,
                     void* out, int64_t ldo, int64_t T, int64_t S, int64_t K, int64_t N, int64_t r_max,
                     float scale, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Base linear and segmented branch in one GEMM:
 *   out[t, :] = x[t] . W^T + bias + (scale * x[t] . A_a^T) . B_a
 * W [N, K] (ldw), bias [N] or NULL, tables and tiles as lora_sgmv_branch.
 * The CTA-pair GEMM of lora_gemm takes, after each 256-token output tile's
 * base K blocks, one more k-block per adapter piece of the tile (the tokens
 * of one segment inside it): a block-diagonal slot of the tile's z (hi/lo
 * bf16 pair) against the adapter's B rows, read by TMA from b_flat.  The base
 * output is written once, with the adapters in it; no y is read or written.
 * Launches: the tile's pieces (one CTA), the unit shrink, the slot fill, the
 * GEMM.  Workspace: lora_sgmv_linear_workspace_size(T, S, K, r_max) bytes
 * (256-byte aligned, no zeroing; one buffer per stream); 0 when the batch's
 * worst case needs more than 512 MiB (per-token ids over ~8000 tokens): then
 * the call returns LORA_ERR_UNSUPPORTED.  S: the segment
 * count the tiles were scheduled from (0 for per-token ids).  Serves
 * r_max <= 64, K and N multiples of 64, leading dimensions multiples of 8,
 * 16-byte aligned rows; LORA_ERR_UNSUPPORTED otherwise (use lora_gemm +
 * lora_sgmv_branch).  No reference counterpart: it fuses the base
 * F.linear with ragged_branch.branch (ragged_branch.py:6-40) /
 * segmented_branch (segmented_branch.py:12-60), the fused base + multi-adapter
 * kernel the reference's serving notes ask for. */
LORA_API size_t lora_sgmv_linear_workspace_size(int64_t T, int64_t S, int64_t K, int64_t r_max);
LORA_API int lora_sgmv_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                     const void* a_flat, int64_t lda, int64_t a_rows, const void* b_flat, int64_t ldb,
                     int64_t b_rows, const int64_t* offsets, const int64_t* ranks, int64_t n_adapters,
                     const int32_t* tiles, void* out, int64_t ldo, int64_t T, int64_t S, int64_t K, int64_t N,
                     int64_t r_max, float scale, int dtype, void* workspace, size_t workspace_bytes,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LORA_B200_H */
