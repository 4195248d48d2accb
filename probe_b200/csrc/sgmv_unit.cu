// Segmented multi-adapter LoRA branch, unit-scheduled, on Blackwell tensor cores.
//
//   z[t, :r_a]  = scale * x[t] . A_a^T                       (shrink)
//   out[t, n]   = y[t, n] + sum_j z[t, j] * B[off_a + j, n]  (expand; scale of a folded into B)
//
// for every token t with adapter a = a(t), a(t) read from the device tile
// schedule (sgmv.h: tiles of <= 64 consecutive tokens sharing one adapter).
// Three kernels, chained with programmatic dependent launch:
//
// 1. Shrink.  Work units = (tile, K slice).  Every x row is read once per
//    call and every adapter row once per tile; persistent CTAs take the units
//    in a snake over a cost-sorted tile order (order_tiles), so they stay
//    balanced whatever the segment lengths and ranks.  Swap-AB MMA: the adapter rows are the M = 128
//    operand (only the first r16 rows are loaded; the other accumulator lanes
//    are never read), the tile's tokens the N = 16..64 operand, both K-major
//    tiles written by TMA with 128-byte swizzle; a double-buffered TMEM
//    accumulator lets one unit's MMAs overlap the previous unit's drain.  A
//    unit stores its fp32 partial [tokens x r_pad] (zeros beyond the rank, and
//    for tiles without an adapter) -- no cross-CTA protocol at all.
// 2. Reduce.  One thread per (token, 4 columns) sums the slices in slice
//    order (results do not depend on timing) and writes z: fp32 or 16-bit
//    [T, z_width], or, for the expand, the 16-bit pair
//    hi = round(s.z), lo = round(s.z - hi) as [T, 2 W] (W = 64).
// 3. Expand.  Work units = (tile, 256-column chunk); CTAs walk groups of two
//    consecutive units of a tile.  The producer loads a group's
//    [hi | lo] z rows once, into one of two z buffers, and for every unit the
//    adapter's B rows [r16 x 256] (rank-major table: an MN-major MMA operand)
//    and the tile's y rows, each in ONE TMA operation (3-D chunk boxes: on
//    B200 the operation count, not the bytes, limits a pipeline of small
//    boxes).  One thread issues M = 128 (the tile's tokens), N = 256 MMAs over
//    K = r16 (hi) + r16 (lo), then adds y with an identity MMA (K = the tile's
//    tokens, one nonzero product per output: exact), into a double-buffered
//    accumulator (2 x 256 TMEM columns).  Eight drain warps on the two lane
//    quadrants that hold the tokens convert and store out with 16-byte
//    stores, releasing the accumulator and the stage as soon as they have
//    read it.
//    Tiles of rank 0 or with an unknown adapter copy y to out.
//
// Roles per CTA: one TMA producer warp, one warp that owns TMEM and issues the
// MMAs, the rest epilogue.  Unit tables are looked up 32 units at a time by whole warps,
// off the issue path.  Every wait is bounded (an expired wait records an error
// and every role leaves its loop); no CTA waits for another.
// Reference semantics: ragged_branch.py:6-40 (per-token shrink / expand,
// rank-0 skip), segmented_branch.py:12-60, multilora.py:128-182, :295-347.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

namespace {

constexpr int kUnitBK = 64;  // K per stage (one 128-byte swizzle row)

bool encode_unit_map(CUtensorMap* map, const void* ptr, int dtype, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                     uint32_t box_outer) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kUnitBK), box_outer};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, dtype == LORA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D view of a row-major [rows, cols] matrix as {64-element chunk, row,
// chunk index}: one TMA box {64, box_rows, box_chunks} brings box_chunks
// consecutive 64-column chunks of box_rows rows in one operation, laid out in
// shared memory chunk-major ([chunk][row][64], 128-byte swizzled rows) -- the
// K-major (or MN-major) MMA operand layout.  TMA operations, not bytes, bound a
// small-box pipeline on B200, so this is how the unit kernels stream.
// cols must be a multiple of 64 (no chunk runs past a row).
bool encode_chunk_map(CUtensorMap* map, const void* ptr, int dtype, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                      uint32_t box_rows, uint32_t box_chunks) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr || cols % 64 != 0) return false;
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {ld_elems * 2, 128};
  cuuint32_t box[3] = {64, box_rows, box_chunks};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode(map, dtype == LORA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool unit_al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

cudaLaunchConfig_t pdl_config(int grid, int threads, size_t smem, void* stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cfg;
}

// ------------------------------------------------------------ unit lookups
// One unit's tile: token range, its adapter's first row and rank.
struct TileInfo {
  int ts, ntok, r;
  int64_t arow;
};

__device__ __forceinline__ TileInfo read_tile(const int32_t* tiles, const int64_t* offsets, const int64_t* ranks,
                                              int tile, int T, int R) {
  TileInfo ti{0, 0, 0, 0};
  ti.ts = sgmv_tile_start(tiles, tile);
  ti.ntok = min(sgmv_tile_start(tiles, tile + 1), T) - ti.ts;
  const int ad = sgmv_tile_adapter(tiles, tile);
  if (ad >= 0) {
    const int64_t rr = ranks[ad];
    ti.r = rr <= 0 ? 0 : static_cast<int>(rr < R ? rr : R);
    ti.arow = offsets[ad];
  }
  return ti;
}

// Unit order.  A unit's time is about its operand bytes, (r16 + n16) rows per
// K chunk or column chunk, and tiles range from 16 to 128 such rows: striding
// over the tiles in schedule order leaves the costliest CTA with ~1.4-1.7x the
// mean on C3.  So every CTA first computes the same order of the tile list --
// descending (r16 + n16), ties in schedule order: a stable counting sort by
// warp ballots, in shared memory -- and takes its units in a snake over the
// grid along that order (b, 2G-1-b, 2G+b, ...).  Which CTA runs a unit does not
// change any result.  Past kOrderMax tiles the tiles keep schedule order.
constexpr int kOrderMax = 1024;
constexpr int kOrderKeys = 12;  // buckets 0..10: (r16 + n16) / 16 = 12..2 (r <= 128, <= 64 tokens); 11: no work
constexpr int kOrderBytes = kOrderMax * 4 + kOrderMax + kOrderKeys * 33 * 4 + 16;  // order, keys, counters

__device__ int tile_bucket(const int32_t* tiles, const int64_t* ranks, int i, int T, int R) {
  const int ntok = min(sgmv_tile_start(tiles, i + 1), T) - sgmv_tile_start(tiles, i);
  const int ad = sgmv_tile_adapter(tiles, i);
  int r = 0;
  if (ad >= 0) {
    const int64_t rr = ranks[ad];
    r = rr <= 0 ? 0 : static_cast<int>(rr < R ? rr : R);
  }
  if (ntok <= 0 || r <= 0) return kOrderKeys - 1;
  const int b = 12 - ((r + 15) / 16 + (ntok + 15) / 16);
  return b < 0 ? 0 : (b > kOrderKeys - 2 ? kOrderKeys - 2 : b);
}

// All threads of the block call it; returns the order (shared memory) or
// nullptr past kOrderMax tiles.
__device__ const int* order_tiles(const int32_t* tiles, const int64_t* ranks, int T, int R, uint8_t* region) {
  const int n = sgmv_num_tiles(tiles);
  if (n > kOrderMax) return nullptr;
  int* order = reinterpret_cast<int*>(region);
  uint8_t* key = region + kOrderMax * 4;
  int* cursor = reinterpret_cast<int*>(region + kOrderMax * 5);  // [kOrderKeys], then [warp][kOrderKeys]
  int* wc = cursor + kOrderKeys;
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nwarps = nth >> 5;
  if (tid < kOrderKeys) cursor[tid] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += nth) {
    const int b = tile_bucket(tiles, ranks, i, T, R);
    key[i] = static_cast<uint8_t>(b);
    atomicAdd(&cursor[b], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int b = 0; b < kOrderKeys; ++b) {
      const int c = cursor[b];
      cursor[b] = acc;
      acc += c;
    }
  }
  __syncthreads();
  for (int base = 0; base < n; base += nth) {  // stable placement, one block-wide chunk at a time
    const int i = base + tid;
    const int b = i < n ? key[i] : -1;
    int below = 0;
    for (int k = 0; k < kOrderKeys; ++k) {
      const unsigned m = __ballot_sync(0xffffffffu, b == k);
      if (b == k) below = __popc(m & ((1u << lane) - 1u));
      if (lane == 0) wc[warp * kOrderKeys + k] = __popc(m);
    }
    __syncthreads();
    if (b >= 0) {
      int pos = cursor[b] + below;
      for (int w = 0; w < warp; ++w) pos += wc[w * kOrderKeys + b];
      order[pos] = i;
    }
    __syncthreads();
    if (tid < kOrderKeys) {
      int add = 0;
      for (int w = 0; w < nwarps; ++w) add += wc[w * kOrderKeys + tid];
      cursor[tid] += add;
    }
    __syncthreads();
  }
  return order;
}

// Walks this CTA's share of n units: unit k is the tile order[k / per_tile]
// (k / per_tile without an order), part k % per_tile.  With an order, CTA b
// takes positions b, 2G-1-b, 2G+b, ... (G CTAs); without, b, b + G, ...
// Warp-collective (lane l prefetches the tile of the (j + l)-th unit); every
// role walks the same sequence.
struct UnitWalk {
  int cta, ctas, n, per_tile, lane, j = 0;
  const int* order;
  TileInfo c;
  __device__ UnitWalk(int b, int g, int n_, int per, int l, const int* ord)
      : cta(b), ctas(g), n(n_), per_tile(per), lane(l), order(ord) {}
  __device__ int pos(int jj) const {
    return order != nullptr ? jj * ctas + ((jj & 1) ? ctas - 1 - cta : cta) : cta + jj * ctas;
  }
  template <typename Args>
  __device__ bool next(const Args& p, TileInfo& t, int& part) {
    const int u = pos(j);
    if (u >= n) return false;
    if ((j & 31) == 0) {
      const int uu = pos(j + lane);
      c = TileInfo{0, 0, 0, 0};
      if (uu < n) {
        const int tile = order != nullptr ? order[uu / per_tile] : uu / per_tile;
        c = read_tile(p.tiles, p.offsets, p.ranks, tile, p.T, p.R);
      }
    }
    const int src = j & 31;
    t.ts = __shfl_sync(0xffffffffu, c.ts, src);
    t.ntok = __shfl_sync(0xffffffffu, c.ntok, src);
    t.r = __shfl_sync(0xffffffffu, c.r, src);
    t.arow = __shfl_sync(0xffffffffu, c.arow, src);
    part = u - (u / per_tile) * per_tile;
    ++j;
    return true;
  }
};

// =================================================================== shrink
constexpr int kShThreads = 192;
constexpr int kShSlots = 12;   // stages in flight at most (barrier pairs)
constexpr int kShKC = 4;       // 64-wide K chunks per stage (one TMA operation per operand)
constexpr int kShRing = 200 * 1024;   // stage ring (bytes); stages take only what their tile needs
constexpr int kShSlack = 16 * 1024;   // the last chunk's M = 128 adapter view may reach past a stage

// A stage of unit (r16 adapter rows, n16 tokens) takes kShKC chunks of both:
// [kShKC][r16][128 B] then [kShKC][n16][128 B].  Stages are packed into the
// ring in issue order; one that would cross the ring's end starts at 0 and the
// skipped bytes count as its own.  Producer and MMA issuer walk the same
// units, so both compute the same offsets; only the producer waits for room.
struct ShRing {
  uint32_t head = 0;
  __device__ uint32_t place(uint32_t size, uint32_t& footprint) {
    const uint32_t off = head % kShRing;
    const uint32_t waste = off + size > kShRing ? kShRing - off : 0u;
    footprint = waste + size;
    head += footprint;
    return waste ? 0u : off;
  }
};
constexpr int kShAccCols = 64;  // one accumulator buffer: up to 64 tokens
constexpr uint32_t kShTmemCols = 2 * kShAccCols;

struct ShMaps {
  CUtensorMap a[8];  // a_flat chunk boxes: 16, 32, ..., 128 rows x kShKC chunks of 64 K
  CUtensorMap x[4];  // x chunk boxes: 16, 32, 48, 64 rows x kShKC chunks of 64 K
};

struct ShArgs {
  float* partial;  // [S][T][RP] fp32
  const int64_t* offsets;
  const int64_t* ranks;
  const int32_t* tiles;
  int* err;
  int T, K, R, RP;
  int num_kb, kb_per, S;   // kb_per: a multiple of kShKC
};

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kShThreads, 1) sgmv_shrink_unit_kernel(const __grid_constant__ ShMaps maps,
                                                                         const ShArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t bar_off = static_cast<uint32_t>(kShRing + kShSlack);
  if (static_cast<uint32_t>(smem - smem_raw) + bar_off + 512u + kOrderBytes > dynamic_smem_bytes()) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemLayout);
    return;
  }
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + bar_off);
  uint64_t* empty = full + kShSlots;
  uint64_t* acc_full = empty + kShSlots;  // [2]
  uint64_t* acc_empty = acc_full + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kShSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int h = 0; h < 8; ++h) tma_prefetch_desc(&maps.a[h]);
    for (int h = 0; h < 4; ++h) tma_prefetch_desc(&maps.x[h]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kShTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The schedule launched before this kernel writes the tile table: wait for
  // it before any global read.  The reduce launched next waits for this whole
  // grid before reading the partials, so it may start its set-up now.
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int n_units = sgmv_num_tiles(p.tiles) * p.S;
  const int* order = order_tiles(p.tiles, p.ranks, p.T, p.R, smem + bar_off + 512);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    UnitWalk walk(blockIdx.x, gridDim.x, n_units, p.S, lane, order);
    TileInfo u;
    int slice, issued = 0, released = 0;
    uint32_t freed = 0;
    uint32_t foot[kShSlots];
    ShRing ring;
    bool ok = true;
    while (ok && walk.next(p, u, slice)) {
      if (u.ntok <= 0 || u.r <= 0) continue;
      const int kb0 = slice * p.kb_per, kb1 = min(p.num_kb, kb0 + p.kb_per);
      const int r16 = (u.r + 15) & ~15, n16 = (u.ntok + 15) & ~15;
      const uint32_t size = static_cast<uint32_t>(kShKC * (r16 + n16) * 128);
      for (int kb = kb0; kb < kb1; kb += kShKC) {  // chunks past K arrive as zeros
        uint32_t footprint;
        const uint32_t start = ring.place(size, footprint);
        if (lane == 0) {
          // room for this stage: release the oldest stages (FIFO) until it fits
          while (ok && (issued - released == kShSlots || ring.head - freed > static_cast<uint32_t>(kShRing))) {
            const int rs = released % kShSlots;
            ok = mbar_wait_bounded(&empty[rs], static_cast<uint32_t>((released / kShSlots) & 1), abort_flag, p.err,
                                   kDevErrTimeoutEmpty);
            freed += foot[rs];
            ++released;
          }
          if (ok) {
            const int s = issued % kShSlots;
            foot[s] = footprint;
            uint8_t* st = smem + start;
            mbar_arrive_expect_tx(&full[s], size);
            tma_load_3d(&maps.a[(r16 >> 4) - 1], st, &full[s], 0, static_cast<int32_t>(u.arow), kb);
            tma_load_3d(&maps.x[(n16 >> 4) - 1], st + kShKC * r16 * 128, &full[s], 0, u.ts, kb);
          }
        }
        ++issued;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    UnitWalk walk(blockIdx.x, gridDim.x, n_units, p.S, lane, order);
    TileInfo u;
    int slice, cnt = 0, i = 0;
    ShRing ring;
    bool ok = true;
    const uint32_t idesc_base = umma_idesc_f16(128, 16, std::is_same<T, __nv_bfloat16>::value ? 1 : 0) &
                                ~(0x3Fu << 17);
    while (ok && walk.next(p, u, slice)) {
      if (u.ntok <= 0 || u.r <= 0) continue;
      const int kb0 = slice * p.kb_per, kb1 = min(p.num_kb, kb0 + p.kb_per);
      const int r16 = (u.r + 15) & ~15, n16 = (u.ntok + 15) & ~15;
      const uint32_t idesc = idesc_base | (static_cast<uint32_t>(n16 >> 3) << 17);
      const int buf = i & 1;
      const uint32_t aph = static_cast<uint32_t>((i >> 1) & 1);
      ++i;
      if (lane == 0) {
        ok = mbar_wait_bounded(&acc_empty[buf], aph ^ 1, abort_flag, p.err, kDevErrTimeoutAccEmpty);
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kShAccCols);
        const uint32_t size = static_cast<uint32_t>(kShKC * (r16 + n16) * 128);
        for (int kb = kb0; ok && kb < kb1; kb += kShKC) {
          uint32_t footprint;
          const uint32_t start = ring.place(size, footprint);
          const int st = cnt % kShSlots;
          const uint32_t phase = static_cast<uint32_t>((cnt / kShSlots) & 1);
          ++cnt;
          if (!mbar_wait_bounded(&full[st], phase, abort_flag, p.err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + start);
#pragma unroll
          for (int c = 0; c < kShKC; ++c) {
            // chunk c: adapter rows at c * r16 rows, tokens after all kShKC adapter chunks
            const uint64_t ad = umma_desc_sw128(sa + static_cast<uint32_t>(c * r16 * 128));
            const uint64_t xd = umma_desc_sw128(sa + static_cast<uint32_t>((kShKC * r16 + c * n16) * 128));
#pragma unroll
            for (int k = 0; k < kUnitBK / 16; ++k)
              tc_mma_f16(d, ad + static_cast<uint64_t>(2 * k), xd + static_cast<uint64_t>(2 * k), idesc,
                         (kb > kb0 || c > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[st]);
        }
        if (ok) tc_commit(&acc_full[buf]);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
  } else {
    // --------------------------------------------- epilogue (warps 2..5)
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31 = ranks
    const int j = quad * 32 + lane;
    const int et = threadIdx.x - 64;
    UnitWalk walk(blockIdx.x, gridDim.x, n_units, p.S, lane, order);
    TileInfo u;
    int slice, i = 0;
    bool ok = true;
    while (walk.next(p, u, slice)) {
      float* dst = p.partial + (static_cast<int64_t>(slice) * p.T + u.ts) * p.RP;
      if (u.ntok <= 0 || u.r <= 0) {
        // no products: this slice's partial rows are zero
        for (int idx = et; idx < u.ntok * (p.RP >> 2); idx += 128)
          reinterpret_cast<float4*>(dst)[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      const int buf = i & 1;
      const uint32_t aph = static_cast<uint32_t>((i >> 1) & 1);
      ++i;
      if (ok) ok = mbar_wait_bounded(&acc_full[buf], aph, abort_flag, p.err, kDevErrTimeoutAccFull);
      tc_fence_after();
      __syncwarp();
      if (ok && quad * 32 < p.RP) {
        for (int c0 = 0; c0 < u.ntok; c0 += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                 static_cast<uint32_t>(buf * kShAccCols + c0),
                             v);
          tmem_wait_ld();
          if (j < p.RP) {
            const int cn = min(32, u.ntok - c0);
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (e < cn) dst[static_cast<int64_t>(c0 + e) * p.RP + j] = j < u.r ? __uint_as_float(v[e]) : 0.f;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kShTmemCols);
  }
}

// =================================================================== reduce
namespace {
struct RedArgs {
  const float* partial;  // [S][T][RP]
  void* z;
  int64_t ldz;
  int T, RP, S, width;   // width: z columns (mode 0/1) or W (mode 2: [T, 2W])
  int mode;              // 0: fp32 z, 1: 16-bit z, 2: 16-bit [hi | lo]
  float scale;
};
}  // namespace

template <typename T>
__global__ void __launch_bounds__(256) sgmv_reduce_kernel(const RedArgs p) {
  pdl_wait();  // the partials come from the shrink launched just before
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int groups = (p.width + 3) >> 2;  // 4 columns per thread
  const int64_t total = static_cast<int64_t>(p.T) * groups;
  const int64_t slice = static_cast<int64_t>(p.T) * p.RP;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(idx / groups);
    const int c = static_cast<int>(idx - static_cast<int64_t>(t) * groups) * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (c < p.RP) {  // RP is a multiple of 4: the group is inside or outside the partial rows
      const float* src = p.partial + static_cast<int64_t>(t) * p.RP + c;
      for (int s = 0; s < p.S; ++s) {
        const float4 q = __ldcg(reinterpret_cast<const float4*>(src + s * slice));
        v[0] += q.x;
        v[1] += q.y;
        v[2] += q.z;
        v[3] += q.w;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] *= p.scale;
    }
    if (p.mode == 0) {
      float* z = static_cast<float*>(p.z) + static_cast<int64_t>(t) * p.ldz + c;
      for (int e = 0; e < 4 && c + e < p.width; ++e) z[e] = v[e];
    } else if (p.mode == 1) {
      T* z = static_cast<T*>(p.z) + static_cast<int64_t>(t) * p.ldz + c;
      for (int e = 0; e < 4 && c + e < p.width; ++e) z[e] = from_f32<T>(v[e]);
    } else {
      uint32_t hi[2], lo[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        hi[e] = pack2<T>(v[2 * e], v[2 * e + 1]);
        const float2 h = unpack2<T>(hi[e]);
        lo[e] = pack2<T>(v[2 * e] - h.x, v[2 * e + 1] - h.y);
      }
      T* z = static_cast<T*>(p.z) + static_cast<int64_t>(t) * p.ldz + c;
      *reinterpret_cast<uint2*>(z) = make_uint2(hi[0], hi[1]);
      *reinterpret_cast<uint2*>(z + p.width) = make_uint2(lo[0], lo[1]);
    }
  }
}

// =================================================================== expand
namespace {

// Warps: eight drain warps on TMEM lane quadrants 0 and 1 (the accumulator's
// 64 token rows), the TMA producer, the MMA issuer; warps 6, 7, 10 and 11
// have no role (a warp may only read the lane quadrant warp_id % 4).
constexpr int kExDrainWarps = 8;
constexpr int kExProducer = 2;
constexpr int kExIssuer = 3;
constexpr int kExThreads = 14 * 32;
constexpr int kExBN = 256;        // output columns per unit
constexpr int kExZW = 64;         // z_hl: [T, 2 * 64] (hi | lo), r_max <= 64
constexpr int kExSlots = 12;      // units in flight at most
constexpr int kExGroup = 2;       // column chunks of one tile walked together (one z load), default
// Shared memory: [identity 8 KB][z buffer 0][z buffer 1][stage ring][barriers].
// An M = 128 operand read from the identity or a z buffer spans 16 KB: its
// rows 64..127 are whatever follows (never drained), always inside the block.
constexpr int kExOffId = 0;                          // 64 x 64 identity, K-major, 128-byte swizzle
constexpr int kExZBytes = 2 * 64 * 128;              // one z buffer: 64 token rows of hi, then of lo
constexpr int kExOffZ = 64 * 128;
constexpr int kExOffRing = kExOffZ + 2 * kExZBytes;
constexpr int kExRing = 176 * 1024;
constexpr int kExOffBar = kExOffRing + kExRing;
constexpr int kExOffOrder = kExOffBar + 512;  // the tile order (order_tiles)
constexpr int kExSmem = kExOffOrder + kOrderBytes + 1024;
constexpr uint32_t kExTmemCols = 2 * kExBN;

__device__ __forceinline__ int ex_drain_index(int warp) {  // -1: not a drain warp
  return ((warp & 3) < 2 && warp < 14) ? (warp >> 2) * 2 + (warp & 1) : -1;
}

// A unit's stage: [B rows: 4 chunks x r16 x 128 B][y: 4 chunks x n16 x 128 B],
// packed into a ring in unit order (a stage that would cross the end starts
// at 0).  The producer places, the MMA issuer recomputes the same offsets; the
// drain frees a stage once the unit's MMAs (which read all of it) have
// completed.  z is not part of a stage: CTAs walk groups of kExGroup
// consecutive column chunks of a tile (in the cost order of order_tiles), and a
// group's z rows are loaded once into one of two z buffers.  Neighbouring CTAs
// take neighbouring groups, so the CTAs in flight cover whole rows of y and out.
struct ExRing {
  uint32_t head = 0;
  __device__ uint32_t place(uint32_t size, uint32_t& footprint) {
    const uint32_t off = head % kExRing;
    const uint32_t waste = off + size > kExRing ? kExRing - off : 0u;
    footprint = waste + size;
    head += footprint;
    return waste ? 0u : off;
  }
};

__device__ __forceinline__ uint32_t ex_stage_bytes(int r16, int n16) {
  return static_cast<uint32_t>((4 * r16 + 4 * n16) * 128);
}

struct ExMaps {
  CUtensorMap b[4];  // b_flat chunk boxes: 16/32/48/64 rows x 4 chunks of 64 columns
  CUtensorMap y[4];  // y chunk boxes: 16/32/48/64 rows x 4 chunks of 64 columns
  CUtensorMap z;     // z_hl [T, 128]: boxes of 64 columns x 64 rows
};

struct ExArgs {
  const void* y;  // only its address matters here (NULL: out = z.B)
  void* out;
  const int64_t* offsets;
  const int64_t* ranks;
  const int32_t* tiles;
  int* err;
  int64_t ldo, ldy;
  int T, N, R, n_chunks, group;
};

// Shared-memory descriptor of an MN-major operand written by TMA as 64-element
// (128-byte) wide chunks with 128-byte swizzle: K rows 128 B apart, 8-row
// groups 1024 B apart (SBO), 64-wide MN chunks `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

}  // namespace

// Per unit, with the tile's tokens as the M = 128 rows (rows 64..127 unused):
//   D[tok, col] = sum_j z_hi[tok, j] B[off + j, col] + sum_j z_lo[tok, j] B[off + j, col]
//               + sum_k I[tok, k] y[k, col]
// A = the z rows or a 64 x 64 identity (K-major), B = the adapter's B rows or
// the tile's y rows (MN-major, straight from the TMA chunk boxes), N = 256.
// The identity pass adds y exactly (one nonzero product per output), so the
// drain only converts and stores.
template <typename T>
__global__ void __launch_bounds__(kExThreads, 1) sgmv_expand_unit_kernel(const __grid_constant__ ExMaps maps,
                                                                         const ExArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if (static_cast<uint32_t>(smem - smem_raw) + static_cast<uint32_t>(kExOffOrder + kOrderBytes) > dynamic_smem_bytes()) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemLayout);
    return;
  }
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kExOffBar);  // B rows and y of a stage landed
  uint64_t* freed = full + kExSlots;                               // the unit's MMAs are done, stage reusable
  uint64_t* afull = freed + kExSlots;
  uint64_t* aempty = afull + 2;
  uint64_t* zfull = aempty + 2;
  uint64_t* zfree = zfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(zfree + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* ring_base = smem + kExOffRing;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dw = ex_drain_index(warp);
  const bool has_y = p.y != nullptr;
  if (threadIdx.x == 0) {
    for (int b = 0; b < kExSlots; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&freed[b], kExDrainWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], kExDrainWarps);
      mbar_init(&zfull[b], 1);
      mbar_init(&zfree[b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (dw >= 0) {
    // identity rows: row t holds 1 at K = t (16-byte granule t / 8, swizzled by t % 8)
    const uint32_t one_lo = pack2<T>(1.f, 0.f), one_hi = pack2<T>(0.f, 1.f);
    for (int g = dw * 32 + lane; g < 64 * 8; g += kExDrainWarps * 32) {
      const int t = g >> 3, logical = (g & 7) ^ (t & 7);
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      if (logical == (t >> 3)) w[(t & 7) >> 1] = (t & 1) ? one_hi : one_lo;
      *reinterpret_cast<uint4*>(smem + kExOffId + g * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    fence_proxy_async_smem();
  }
  if (warp == kExProducer && lane == 0) {
    tma_prefetch_desc(&maps.z);
    for (int h = 0; h < 4; ++h) {
      tma_prefetch_desc(&maps.b[h]);
      if (has_y) tma_prefetch_desc(&maps.y[h]);
    }
  }
  if (warp == kExIssuer) {
    tmem_alloc(tmem_slot, kExTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // z_hl comes from the reduce launched just before: wait before any global read.
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int gpt = (p.n_chunks + p.group - 1) / p.group;  // groups per tile
  const int n_groups = sgmv_num_tiles(p.tiles) * gpt;
  const int* order = order_tiles(p.tiles, p.ranks, p.T, p.R, smem + kExOffOrder);

  if (warp == kExProducer) {
    // ------------------------------------------------------------ producer
    UnitWalk walk(blockIdx.x, gridDim.x, n_groups, gpt, lane, order);
    TileInfo u;
    int grp, issued = 0, released = 0, runs = 0;
    uint32_t freed_bytes = 0;
    uint32_t foot[kExSlots];
    ExRing ring;
    bool ok = true;
    while (ok && walk.next(p, u, grp)) {
      if (u.ntok <= 0 || u.r <= 0) continue;
      const int r16 = (u.r + 15) & ~15, n16 = (u.ntok + 15) & ~15;
      if (lane == 0) {  // the tile's z rows, once per group (the buffer's group before last has finished its MMAs)
        const int zb = runs & 1;
        ok = mbar_wait_bounded(&zfree[zb], static_cast<uint32_t>(((runs >> 1) & 1) ^ 1), abort_flag, p.err,
                               kDevErrTimeoutEmpty);
        if (ok) {
          uint8_t* zs = smem + kExOffZ + zb * kExZBytes;
          mbar_arrive_expect_tx(&zfull[zb], kExZBytes);
          tma_load_2d(&maps.z, zs, &zfull[zb], 0, u.ts);                // hi
          tma_load_2d(&maps.z, zs + 64 * 128, &zfull[zb], kExZW, u.ts);  // lo
        }
      }
      ++runs;
      const int c_end = min(p.n_chunks, (grp + 1) * p.group);
      for (int chunk = grp * p.group; ok && chunk < c_end; ++chunk) {
        uint32_t footprint;
        const uint32_t start = ring.place(ex_stage_bytes(r16, n16), footprint);
        if (lane == 0) {
          while (ok && (issued - released == kExSlots || ring.head - freed_bytes > static_cast<uint32_t>(kExRing))) {
            const int rs = released % kExSlots;
            ok = mbar_wait_bounded(&freed[rs], static_cast<uint32_t>((released / kExSlots) & 1), abort_flag, p.err,
                                   kDevErrTimeoutEmpty);
            freed_bytes += foot[rs];
            ++released;
          }
          if (ok) {
            const int s = issued % kExSlots;
            const int c0 = chunk * (kExBN / 64);  // first 64-column chunk of the unit
            foot[s] = footprint;
            uint8_t* st = ring_base + start;
            mbar_arrive_expect_tx(&full[s], (4 * r16 + (has_y ? 4 * n16 : 0)) * 128);
            tma_load_3d(&maps.b[(r16 >> 4) - 1], st, &full[s], 0, static_cast<int32_t>(u.arow), c0);
            if (has_y) tma_load_3d(&maps.y[(n16 >> 4) - 1], st + 4 * r16 * 128, &full[s], 0, u.ts, c0);
          }
        }
        ++issued;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
  } else if (warp == kExIssuer) {
    // ---------------------------------------------------------- MMA issuer
    UnitWalk walk(blockIdx.x, gridDim.x, n_groups, gpt, lane, order);
    TileInfo u;
    int grp, i = 0, runs = 0;
    ExRing ring;
    bool ok = true;
    // M = 128 (tokens), N = 256 columns; A K-major, B MN-major (transpose-B bit 16)
    const uint32_t idesc = umma_idesc_f16(128, kExBN, std::is_same<T, __nv_bfloat16>::value ? 1 : 0) | (1u << 16);
    const uint32_t zbase = smem_u32(smem + kExOffZ), ring_u32 = smem_u32(ring_base);
    const uint64_t id_desc = umma_desc_sw128(smem_u32(smem + kExOffId));
    while (ok && walk.next(p, u, grp)) {
      if (u.ntok <= 0 || u.r <= 0) continue;
      const int r16 = (u.r + 15) & ~15, n16 = (u.ntok + 15) & ~15;
      const int zb = runs & 1;
      if (lane == 0) {
        if (runs > 0) tc_commit(&zfree[zb ^ 1]);  // every MMA of the previous group is issued
        ok = mbar_wait_bounded(&zfull[zb], static_cast<uint32_t>((runs >> 1) & 1), abort_flag, p.err,
                               kDevErrTimeoutFull);
      }
      ++runs;
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      const uint32_t zs = zbase + static_cast<uint32_t>(zb * kExZBytes);
      const int c_end = min(p.n_chunks, (grp + 1) * p.group);
      for (int chunk = grp * p.group; ok && chunk < c_end; ++chunk) {
        uint32_t footprint;
        const uint32_t start = ring.place(ex_stage_bytes(r16, n16), footprint);
        const int s = i % kExSlots, buf = i & 1;
        const uint32_t ph = static_cast<uint32_t>((i / kExSlots) & 1), aph = static_cast<uint32_t>((i >> 1) & 1);
        ++i;
        if (lane == 0) {
          ok = mbar_wait_bounded(&full[s], ph, abort_flag, p.err, kDevErrTimeoutFull) &&
               mbar_wait_bounded(&aempty[buf], aph ^ 1, abort_flag, p.err, kDevErrTimeoutAccEmpty);
          if (ok) {
            tc_fence_after();
            const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kExBN);
            const uint32_t bs = ring_u32 + start;
            for (int part = 0; part < 2; ++part) {  // z hi, then z lo
              const uint64_t zd = umma_desc_sw128(zs + static_cast<uint32_t>(part * 64 * 128));
              for (int ks = 0; ks < r16 / 16; ++ks)
                tc_mma_f16(d, zd + static_cast<uint64_t>(2 * ks),
                           umma_desc_sw128_mn(bs + static_cast<uint32_t>(ks * 2048), static_cast<uint32_t>(r16 * 128)),
                           idesc, (part > 0 || ks > 0) ? 1u : 0u);
            }
            if (has_y) {  // + y: identity x the tile's y rows (K = its tokens)
              const uint32_t ys = bs + static_cast<uint32_t>(4 * r16 * 128);
              for (int ks = 0; ks < n16 / 16; ++ks)
                tc_mma_f16(d, id_desc + static_cast<uint64_t>(2 * ks),
                           umma_desc_sw128_mn(ys + static_cast<uint32_t>(ks * 2048), static_cast<uint32_t>(n16 * 128)),
                           idesc, 1u);
            }
            tc_commit(&afull[buf]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
    }
  } else if (dw >= 0) {
    // ------------------------------------------------ drain (8 warps)
    const int quad = dw & 1;        // == warp % 4: TMEM lanes quad*32.. hold tokens quad*32..
    const int cb = (dw >> 1) * 64;  // this warp's 64-column block of the unit
    const int t = quad * 32 + lane;
    UnitWalk walk(blockIdx.x, gridDim.x, n_groups, gpt, lane, order);
    TileInfo u;
    int grp, i = 0;
    bool ok = true;
    while (walk.next(p, u, grp)) {
      const int c_end = min(p.n_chunks, (grp + 1) * p.group);
      if (u.ntok <= 0 || u.r <= 0) {
        // rank 0 / unknown adapter: out = y (zeros without y); warp dw copies tokens dw, dw + 8, ...
        for (int tt = dw; tt < u.ntok; tt += kExDrainWarps) {
          for (int col = grp * p.group * kExBN + lane * 2; col < c_end * kExBN && col < p.N; col += 64) {
            T* o = static_cast<T*>(p.out) + static_cast<int64_t>(u.ts + tt) * p.ldo + col;
            const T* yy = has_y ? static_cast<const T*>(p.y) + static_cast<int64_t>(u.ts + tt) * p.ldy + col : nullptr;
            *reinterpret_cast<uint32_t*>(o) = has_y ? *reinterpret_cast<const uint32_t*>(yy) : 0u;
          }
        }
        continue;
      }
      for (int chunk = grp * p.group; chunk < c_end; ++chunk) {
        const int n0 = chunk * kExBN;
        const int s = i % kExSlots, buf = i & 1;
        const uint32_t aph = static_cast<uint32_t>((i >> 1) & 1);
        ++i;
        if (ok) ok = mbar_wait_bounded(&afull[buf], aph, abort_flag, p.err, kDevErrTimeoutAccFull);
        tc_fence_after();
        __syncwarp();
        uint32_t v[64];
        if (ok) {
          const uint32_t ta =
              tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * kExBN + cb);
          tmem_ld_32x32b_x32(ta, v);
          tmem_ld_32x32b_x32(ta + 32, v + 32);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {  // accumulator read and the unit's MMAs done: both can be reused
          mbar_arrive(&aempty[buf]);
          mbar_arrive(&freed[s]);
        }
        if (ok && t < u.ntok && n0 + cb < p.N) {  // N is a multiple of 64
          T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(u.ts + t) * p.ldo + n0 + cb;
#pragma unroll
          for (int c = 0; c < 8; ++c) {  // 8 columns (16 bytes) per store
            uint32_t ow[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              ow[e] = pack2<T>(__uint_as_float(v[8 * c + 2 * e]), __uint_as_float(v[8 * c + 2 * e + 1]));
            *reinterpret_cast<uint4*>(orow + 8 * c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kExIssuer) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kExTmemCols);
  }
}

// ===================================================================== host
namespace {

// K slices of the shrink: about `per_sm` units per SM counting one tile per
// 64 tokens (the fewest any schedule of T tokens has), at least 4 k-blocks
// per slice, at most 16 slices.  It depends on T and K only, so per-token ids
// and segment tables describing the same batch sum their partials alike and
// give bit-identical results.
// One unit per SM: with the units in cost order (order_tiles), fewer and
// longer units keep more of a CTA's stages in flight and leave fewer partial
// slices to sum (C3: branch 64.9 against 67.6 us per call, fused linear
// 152-154 against 155 us, than four per SM).
constexpr int kUnitsPerSm = 1;

int unit_slices(int64_t T, int64_t K, int num_sms, int per_sm) {
  const int64_t kb = std::max<int64_t>((K + kUnitBK - 1) / kUnitBK, 1);
  const int64_t blocks = std::max<int64_t>((T + 63) / 64, 1);
  int64_t s = (per_sm * static_cast<int64_t>(num_sms) + blocks - 1) / blocks;
  s = std::max<int64_t>(1, std::min<int64_t>({s, 16, std::max<int64_t>(kb / 4, 1)}));
  const int64_t per = ((kb + s - 1) / s + kShKC - 1) / kShKC * kShKC;
  return static_cast<int>((kb + per - 1) / per);
}

inline int64_t rpad(int64_t r_max) { return (r_max + 15) / 16 * 16; }

int launch_shrink_units(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                        const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t max_tiles,
                        float* partial, int64_t T, int64_t K, int64_t r_max, int S, int dtype, int num_sms, int* err,
                        void* stream) {
  const int num_kb = static_cast<int>((K + kUnitBK - 1) / kUnitBK);
  const int kb_per = ((num_kb + S - 1) / S + kShKC - 1) / kShKC * kShKC;
  const size_t smem = static_cast<size_t>(kShRing + kShSlack) + 512 + kOrderBytes + 1024;
  ShMaps maps;
  for (int h = 0; h < 8; ++h)
    if (!encode_chunk_map(&maps.a[h], a_flat, dtype, static_cast<uint64_t>(a_rows), static_cast<uint64_t>(K),
                          static_cast<uint64_t>(lda), static_cast<uint32_t>(16 * (h + 1)), kShKC))
      return LORA_ERR_CUDA;
  for (int h = 0; h < 4; ++h)
    if (!encode_chunk_map(&maps.x[h], x, dtype, static_cast<uint64_t>(T), static_cast<uint64_t>(K),
                          static_cast<uint64_t>(ldx), static_cast<uint32_t>(16 * (h + 1)), kShKC))
      return LORA_ERR_CUDA;
  ShArgs a{};
  a.partial = partial;
  a.offsets = offsets;
  a.ranks = ranks;
  a.tiles = tiles;
  a.err = err;
  a.T = static_cast<int>(T);
  a.K = static_cast<int>(K);
  a.R = static_cast<int>(r_max);
  a.RP = static_cast<int>(rpad(r_max));
  a.num_kb = num_kb;
  a.kb_per = kb_per;
  a.S = S;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(max_tiles * S, num_sms)));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(grid, kShThreads, smem, stream, attr);
  if (dtype == LORA_BF16) {
    auto kernel = sgmv_shrink_unit_kernel<__nv_bfloat16>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return LORA_ERR_CUDA;
    return cudaLaunchKernelEx(&cfg, kernel, maps, a) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
  }
  auto kernel = sgmv_shrink_unit_kernel<__half>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return LORA_ERR_CUDA;
  return cudaLaunchKernelEx(&cfg, kernel, maps, a) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

int launch_reduce(const float* partial, int S, int64_t T, int64_t RP, void* z, int64_t ldz, int64_t width, int mode,
                  float scale, int dtype, int num_sms, void* stream) {
  RedArgs r{};
  r.partial = partial;
  r.z = z;
  r.ldz = ldz;
  r.T = static_cast<int>(T);
  r.RP = static_cast<int>(RP);
  r.S = S;
  r.width = static_cast<int>(width);
  r.mode = mode;
  r.scale = scale;
  const int64_t work = T * ((width + 3) / 4);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 8 * num_sms)));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(grid, 256, 0, stream, attr);
  if (dtype == LORA_BF16)
    return cudaLaunchKernelEx(&cfg, sgmv_reduce_kernel<__nv_bfloat16>, r) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
  return cudaLaunchKernelEx(&cfg, sgmv_reduce_kernel<__half>, r) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

// Column chunks per expand group: LORA_B200_EX_GROUP overrides the default
// (read once; tuning sweeps).
int expand_group(int64_t n_chunks) {
  static const int g = [] {
    const char* v = std::getenv("LORA_B200_EX_GROUP");
    const int parsed = v != nullptr ? std::atoi(v) : 0;
    return parsed > 0 ? parsed : kExGroup;
  }();
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(g, n_chunks)));
}

int launch_expand_units(const void* y, int64_t ldy, const void* z_hl, const void* b, int64_t b_rows, int64_t ldb,
                        const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t max_tiles,
                        void* out, int64_t ldo, int64_t T, int64_t N, int64_t r_max, int dtype, int num_sms, int* err,
                        void* stream) {
  const int64_t n_chunks = (N + kExBN - 1) / kExBN;
  ExMaps maps;
  for (int h = 0; h < 4; ++h) {
    if (!encode_chunk_map(&maps.b[h], b, dtype, static_cast<uint64_t>(b_rows), static_cast<uint64_t>(N),
                          static_cast<uint64_t>(ldb), static_cast<uint32_t>(16 * (h + 1)), kExBN / 64))
      return LORA_ERR_CUDA;
    if (y != nullptr) {
      if (!encode_chunk_map(&maps.y[h], y, dtype, static_cast<uint64_t>(T), static_cast<uint64_t>(N),
                            static_cast<uint64_t>(ldy), static_cast<uint32_t>(16 * (h + 1)), kExBN / 64))
        return LORA_ERR_CUDA;
    } else {
      maps.y[h] = maps.b[h];
    }
  }
  if (!encode_unit_map(&maps.z, z_hl, dtype, static_cast<uint64_t>(2 * kExZW), static_cast<uint64_t>(T),
                       static_cast<uint64_t>(2 * kExZW), 64))
    return LORA_ERR_CUDA;
  ExArgs a{};
  a.y = y;
  a.out = out;
  a.offsets = offsets;
  a.ranks = ranks;
  a.tiles = tiles;
  a.err = err;
  a.ldo = ldo;
  a.ldy = ldy;
  a.T = static_cast<int>(T);
  a.N = static_cast<int>(N);
  a.R = static_cast<int>(r_max);
  a.n_chunks = static_cast<int>(n_chunks);
  a.group = expand_group(n_chunks);
  const int64_t groups = max_tiles * ((n_chunks + a.group - 1) / a.group);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(groups, num_sms)));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(grid, kExThreads, kExSmem, stream, attr);
  if (dtype == LORA_BF16) {
    auto kernel = sgmv_expand_unit_kernel<__nv_bfloat16>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kExSmem) != cudaSuccess)
      return LORA_ERR_CUDA;
    return cudaLaunchKernelEx(&cfg, kernel, maps, a) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
  }
  auto kernel = sgmv_expand_unit_kernel<__half>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kExSmem) != cudaSuccess)
    return LORA_ERR_CUDA;
  return cudaLaunchKernelEx(&cfg, kernel, maps, a) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

bool shrink_units_ok(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows, int64_t T,
                     int64_t K, int64_t r_max, int64_t max_tiles) {
  if (r_max <= 0 || r_max > 128 || T <= 0 || K <= 0 || a_rows <= 0 || a_rows > INT32_MAX) return false;
  // whole 64-column chunks (the 3-D TMA view), 16-byte aligned rows
  if (K % 64 != 0 || ldx % 8 != 0 || lda % 8 != 0 || !unit_al16(x) || !unit_al16(a_flat)) return false;
  return T <= INT32_MAX / 2 && K <= INT32_MAX && max_tiles * 16 <= INT32_MAX;
}

// Bytes of the fp32 partials [S][T][rpad(r_max)], rounded up to 256.
size_t partial_bytes(int S, int64_t T, int64_t r_max) {
  return (static_cast<size_t>(S) * static_cast<size_t>(T) * static_cast<size_t>(rpad(r_max)) * sizeof(float) + 255) /
         256 * 256;
}

}  // namespace

size_t sgmv_unit_shrink_workspace(int64_t T, int64_t K, int64_t r_max, int64_t max_tiles, int num_sms) {
  return partial_bytes(unit_slices(T, K, num_sms, kUnitsPerSm), T, r_max);
}

int launch_sgmv_shrink_unit(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                            const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t max_tiles,
                            void* z, int64_t ldz, int z_dtype, int64_t z_width, int64_t T, int64_t K, int64_t r_max,
                            float scale, int dtype, void* workspace, size_t workspace_bytes, int num_sms, int* err,
                            void* stream) {
  if (!shrink_units_ok(x, ldx, a_flat, lda, a_rows, T, K, r_max, max_tiles)) return LORA_ERR_UNSUPPORTED;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  const int S = unit_slices(T, K, num_sms, kUnitsPerSm);
  if (workspace == nullptr || !unit_al16(workspace) ||
      workspace_bytes < sgmv_unit_shrink_workspace(T, K, r_max, max_tiles, num_sms))
    return LORA_ERR_UNSUPPORTED;
  float* partial = static_cast<float*>(workspace);
  int rc = launch_shrink_units(x, ldx, a_flat, lda, a_rows, offsets, ranks, tiles, max_tiles, partial, T, K, r_max, S,
                               dtype, num_sms, err, stream);
  if (rc != LORA_OK) return rc;
  return launch_reduce(partial, S, T, rpad(r_max), z, ldz, z_width, z_dtype == LORA_F32 ? 0 : 1, scale, dtype,
                       num_sms, stream);
}

size_t sgmv_unit_branch_workspace(int64_t T, int64_t K, int64_t r_max, int64_t max_tiles, int num_sms) {
  return partial_bytes(unit_slices(T, K, num_sms, kUnitsPerSm), T, r_max) +
         static_cast<size_t>(T) * 2 * kExZW * 2;
}

int launch_sgmv_branch_unit(const void* x, int64_t ldx, const void* y, int64_t ldy, const void* a_flat, int64_t lda,
                            int64_t a_rows, const void* b_flat, int64_t ldb, int64_t b_rows, const int64_t* offsets,
                            const int64_t* ranks, const int32_t* tiles, int64_t max_tiles, void* out, int64_t ldo,
                            int64_t T, int64_t K, int64_t N, int64_t r_max, float scale, int dtype, void* workspace,
                            size_t workspace_bytes, int num_sms, int* err, void* stream) {
  if (!shrink_units_ok(x, ldx, a_flat, lda, a_rows, T, K, r_max, max_tiles) || r_max > kExZW)
    return LORA_ERR_UNSUPPORTED;
  if (N <= 0 || N % 64 != 0 || ldb % 8 != 0 || ldo % 8 != 0 || b_rows <= 0 || b_rows > INT32_MAX ||
      !unit_al16(b_flat) || !unit_al16(out) || N > INT32_MAX / 2)
    return LORA_ERR_UNSUPPORTED;
  if (y != nullptr && (ldy % 8 != 0 || !unit_al16(y))) return LORA_ERR_UNSUPPORTED;
  if (max_tiles * ((N + kExBN - 1) / kExBN) > INT32_MAX) return LORA_ERR_UNSUPPORTED;
  if (workspace == nullptr || !unit_al16(workspace) ||
      workspace_bytes < sgmv_unit_branch_workspace(T, K, r_max, max_tiles, num_sms))
    return LORA_ERR_UNSUPPORTED;
  const int S = unit_slices(T, K, num_sms, kUnitsPerSm);
  float* partial = static_cast<float*>(workspace);
  void* z_hl = static_cast<char*>(workspace) + partial_bytes(S, T, r_max);
  int rc = launch_shrink_units(x, ldx, a_flat, lda, a_rows, offsets, ranks, tiles, max_tiles, partial, T, K, r_max, S,
                               dtype, num_sms, err, stream);
  if (rc != LORA_OK) return rc;
  rc = launch_reduce(partial, S, T, rpad(r_max), z_hl, 2 * kExZW, kExZW, 2, scale, dtype, num_sms, stream);
  if (rc != LORA_OK) return rc;
  return launch_expand_units(y, ldy, z_hl, b_flat, b_rows, ldb, offsets, ranks, tiles, max_tiles, out, ldo, T, N,
                             r_max, dtype, num_sms, err, stream);
}

int sgmv_unit_slices(int64_t T, int64_t K, int num_sms) { return unit_slices(T, K, num_sms, kUnitsPerSm); }

int launch_sgmv_shrink_partials(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                                const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t max_tiles,
                                float* partial, int64_t T, int64_t K, int64_t r_max, int S, int dtype, int num_sms,
                                int* err, void* stream) {
  if (!shrink_units_ok(x, ldx, a_flat, lda, a_rows, T, K, r_max, max_tiles)) return LORA_ERR_UNSUPPORTED;
  return launch_shrink_units(x, ldx, a_flat, lda, a_rows, offsets, ranks, tiles, max_tiles, partial, T, K, r_max, S,
                             dtype, num_sms, err, stream);
}

}  // namespace lora
