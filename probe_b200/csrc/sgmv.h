// Device-side tile schedule for the segmented multi-adapter kernels.
//
// A schedule is an int32 buffer built on the GPU by lora_sgmv_schedule:
//   [0]                       number of tiles (set by the schedule kernel)
//   [1]                       capacity (max_tiles, set by the host)
//   [2 .. 3 + max_tiles)      tile start token; entry [num_tiles] == T
//   [3 + max_tiles .. )       adapter id of each tile (-1 = skip / invalid)
// Every tile covers <= 64 consecutive tokens that use the same adapter.
#pragma once

#include <stdint.h>

namespace lora {

constexpr int kSgmvTileTokens = 64;

__host__ __device__ inline int64_t sgmv_max_tiles(int64_t T, int64_t S) {
  const int64_t blocks = (T + kSgmvTileTokens - 1) / kSgmvTileTokens;
  const int64_t boundaries = S > 0 ? S : T;
  return blocks + boundaries + 1;
}

__host__ __device__ inline int64_t sgmv_tiles_bytes(int64_t T, int64_t S) {
  const int64_t mt = sgmv_max_tiles(T, S);
  return (2 + (mt + 1) + mt) * static_cast<int64_t>(sizeof(int32_t));
}

__device__ __forceinline__ int sgmv_num_tiles(const int32_t* tiles) { return tiles[0]; }
__device__ __forceinline__ int sgmv_tile_start(const int32_t* tiles, int i) { return tiles[2 + i]; }
__device__ __forceinline__ int sgmv_tile_adapter(const int32_t* tiles, int i) { return tiles[3 + tiles[1] + i]; }

}  // namespace lora
