// Device-side tile schedule for the segmented multi-adapter kernels.
//
// A schedule is an int32 buffer built on the GPU by lora_sgmv_schedule:
//   [0]                              number of tiles (set by the schedule kernel)
//   [1]                              capacity (max_tiles, set by the host)
//   [2 .. 3 + max_tiles)             tile start token; entry [num_tiles] == T
//   [3 + max_tiles .. 3 + 2 max_tiles)  adapter id of each tile (-1 = skip / invalid)
//   [3 + 2 max_tiles .. + blocks + 1)   first tile of each 64-token block;
//                                       entry [blocks] == num_tiles
// Every tile covers <= 64 consecutive tokens that use the same adapter, and a
// tile starts at every multiple of 64, so the tiles of block b are exactly
// first[b] .. first[b+1].
#pragma once

#include <stdint.h>

namespace lora {

constexpr int kSgmvTileTokens = 64;

__host__ __device__ inline int64_t sgmv_max_tiles(int64_t T, int64_t S) {
  const int64_t blocks = (T + kSgmvTileTokens - 1) / kSgmvTileTokens;
  const int64_t boundaries = S > 0 ? S : T;
  return blocks + boundaries + 1;
}

__host__ __device__ inline int64_t sgmv_blocks(int64_t T) { return (T + kSgmvTileTokens - 1) / kSgmvTileTokens; }

__host__ __device__ inline int64_t sgmv_tiles_bytes(int64_t T, int64_t S) {
  const int64_t mt = sgmv_max_tiles(T, S);
  return (2 + (mt + 1) + mt + (sgmv_blocks(T) + 1)) * static_cast<int64_t>(sizeof(int32_t));
}

__device__ __forceinline__ int sgmv_num_tiles(const int32_t* tiles) { return tiles[0]; }
__device__ __forceinline__ int sgmv_tile_start(const int32_t* tiles, int i) { return tiles[2 + i]; }
__device__ __forceinline__ int sgmv_tile_adapter(const int32_t* tiles, int i) { return tiles[3 + tiles[1] + i]; }
__device__ __forceinline__ const int32_t* sgmv_block_first(const int32_t* tiles) { return tiles + 3 + 2 * tiles[1]; }

// Block-structured kernels of sgmv_block.cu (dense 64-token blocks, cp.async
// pipelines; the shrink's K splits are the CTAs of one thread-block cluster,
// reduced through distributed shared memory, so it needs no workspace).  They return LORA_ERR_UNSUPPORTED when a layout or alignment
// condition of their fast path does not hold; the caller then uses the
// per-tile kernels.
struct SgmvShrinkBlockArgs {
  const void* x;
  const void* a;
  void* z;
  const int64_t* offsets;
  const int64_t* ranks;
  const int32_t* tiles;
  const int64_t* rows;
  int* err;
  int64_t ldx, lda, ldz;
  int T, K, R, z_width, z_split, split_k, kslice;  // split_k CTAs of one cluster share a block
  float scale;
};
int launch_sgmv_shrink_block(const SgmvShrinkBlockArgs& p, int dtype, int z_dtype, int num_sms, void* stream);
int sgmv_shrink_block_split(int64_t T, int64_t K, int num_sms);
constexpr int kSgmvMaxClusterSplit = 8;  // portable cluster size

struct SgmvExpandBlockArgs {
  const void* y;
  const void* z;
  const void* b;
  void* out;
  const int64_t* offsets;
  const int64_t* ranks;
  const int32_t* tiles;
  const int64_t* rows;
  int* err;
  int64_t ldy, ldz, ldo, ldb;  // B element (adapter a, rank j, column n) at b[(offsets[a] + j) * ldb + n]
  int T, N, R;
  float scale;
};
int launch_sgmv_expand_block(const SgmvExpandBlockArgs& p, int dtype, int z_dtype, void* stream);

// Tensor-core segmented shrink (sgmv_tc.cu): 128-token blocks, every adapter of
// a block in one MMA chain, K slices reduced over a cluster.  Needs the row
// count of a_flat (bounds of its TMA reads), no row indirection, aligned rows.
int launch_sgmv_shrink_tc(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                          const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, void* z, int64_t ldz,
                          int z_dtype, int64_t z_width, int64_t T, int64_t K, int64_t r_max, float scale, int dtype,
                          int num_sms, int* err, void* stream);

// Unit-scheduled tensor-core segmented branch (sgmv_unit.cu): a shrink over
// (tile, K slice) units writing fp32 partials, a reduce kernel summing them in
// slice order, and an expand over (tile, 256-column chunk) units.  Needs the
// row counts of the tables (TMA bounds), no row indirection, aligned rows.
// The shrink's workspace: sgmv_unit_shrink_workspace() bytes of partials.
size_t sgmv_unit_shrink_workspace(int64_t T, int64_t K, int64_t r_max, int64_t max_tiles, int num_sms);
int launch_sgmv_shrink_unit(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                            const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t max_tiles,
                            void* z, int64_t ldz, int z_dtype, int64_t z_width, int64_t T, int64_t K, int64_t r_max,
                            float scale, int dtype, void* workspace, size_t workspace_bytes, int num_sms, int* err,
                            void* stream);
// The whole branch out = y + (x . A_a^T) . B_a in three launches (r_max <= 64,
// N and leading dimensions multiples of 8); LORA_ERR_UNSUPPORTED otherwise.
size_t sgmv_unit_branch_workspace(int64_t T, int64_t K, int64_t r_max, int64_t max_tiles, int num_sms);
int launch_sgmv_branch_unit(const void* x, int64_t ldx, const void* y, int64_t ldy, const void* a_flat, int64_t lda,
                            int64_t a_rows, const void* b_flat, int64_t ldb, int64_t b_rows, const int64_t* offsets,
                            const int64_t* ranks, const int32_t* tiles, int64_t max_tiles, void* out, int64_t ldo,
                            int64_t T, int64_t K, int64_t N, int64_t r_max, float scale, int dtype, void* workspace,
                            size_t workspace_bytes, int num_sms, int* err, void* stream);

// The shrink alone: fp32 partials [S][T][rpad16(r_max)] over S K slices
// (sgmv_unit_slices), zeros beyond each token's rank; for callers that reduce
// them themselves.
int sgmv_unit_slices(int64_t T, int64_t K, int num_sms);
int launch_sgmv_shrink_partials(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                                const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t max_tiles,
                                float* partial, int64_t T, int64_t K, int64_t r_max, int S, int dtype, int num_sms,
                                int* err, void* stream);

// Segmented LoRA linear in one CTA-pair GEMM (sgmv_linear.cu):
// out = x . W^T + bias + (branch), the adapters as a per-tile K tail.
// r_max <= 64, K and N multiples of 64, 16-byte aligned rows;
// LORA_ERR_UNSUPPORTED otherwise.  S = segment count the schedule was built
// from (0 for per-token ids): it bounds the schedule's tiles.
size_t sgmv_linear_workspace(int64_t T, int64_t S, int64_t K, int64_t r_max, int num_sms);
int launch_sgmv_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias, const void* a_flat,
                       int64_t lda, int64_t a_rows, const void* b_flat, int64_t ldb, int64_t b_rows,
                       const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t S, void* out,
                       int64_t ldo, int64_t T, int64_t K, int64_t N, int64_t r_max, float scale, int dtype,
                       void* workspace, size_t workspace_bytes, int num_sms, int* err, void* stream);

}  // namespace lora
