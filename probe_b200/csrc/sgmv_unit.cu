// Segmented multi-adapter shrink, unit-scheduled, on Blackwell tensor cores.
//
//   z[t, :r_a] = scale * x[t] . A_a^T   for every token t with adapter a(t)
//
// Work is cut into units = (tile of the device schedule, K slice): a tile is
// <= 64 consecutive tokens sharing one adapter, so a unit's operands are that
// tile's x rows and its adapter's rows over one K slice -- every x row is
// read once per call, every adapter row once per tile, and units are small
// (~100 KB) and alike, so persistent CTAs striding over them stay balanced
// whatever the segment lengths (no 128-token block with 400 adapter rows to
// wait for).
//
// MMA (swap-AB): the adapter rows are the M = 128 operand (only the first
// r16 rows are loaded; the other lanes of the accumulator are never read) and
// the tile's tokens the N = 16..64 operand, both K-major tiles written by TMA
// with 128-byte swizzle.  The accumulator (rank x tokens, fp32) is
// double-buffered in TMEM so the next unit's MMAs overlap this unit's drain.
//
// Split-K: each unit stores its fp32 partial in the workspace; the last unit
// of a tile to finish (atomic ticket in the workspace's counter region,
// returned to zero) sums the slices in slice order and writes z, so the
// result does not depend on timing.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner and MMA issuer,
// warps 2..5 epilogue.  Unit tables are looked up 32 units at a time by whole
// warps, off the issue path.  Every wait is bounded (an expired wait records
// an error and makes every role leave its loop); there are no inter-CTA waits.
// Reference semantics: ragged_branch.py:6-16 (per-token shrink, rank-0 skip),
// segmented_branch.py:12-28, multilora.py:128-182.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

namespace {

constexpr int kUnitThreads = 192;
constexpr int kUnitBK = 64;            // K per stage (one 128-byte swizzle row)
constexpr int kUnitMaxStages = 12;
constexpr int kUnitAccCols = 64;       // one accumulator buffer: up to 64 tokens
constexpr uint32_t kUnitTmemCols = 2 * kUnitAccCols;

struct UnitMaps {
  CUtensorMap a[8];  // a_flat boxes of 16, 32, ..., 128 rows x 64 K
  CUtensorMap x[4];  // x boxes of 16, 32, 48, 64 rows x 64 K
};

struct UnitArgs {
  void* z;
  float* partial;        // [S][T][R] fp32
  int* tickets;          // one per tile, zero on entry and on exit
  const int64_t* offsets;
  const int64_t* ranks;
  const int32_t* tiles;
  int* err;
  int64_t ldz;
  int T, K, R, z_width, z_f32;
  int num_kb, kb_per, S;
  int stages, stage_bytes, x_off;
  float scale;
};

// One unit's operands, as looked up from the schedule.
struct UnitInfo {
  int ts, ntok, r, kb0, kb1, tile, slice;
  int64_t arow;
  __device__ bool empty() const { return ntok <= 0 || r <= 0 || kb1 <= kb0; }
};

// Warp-collective: lane l looks up unit (first + l * stride); units past n get ntok = 0.
__device__ __forceinline__ void lookup_units(const UnitArgs& p, int first, int stride, int n, int lane, int& ts,
                                             int& ntok, int& r, int64_t& arow) {
  const int u = first + lane * stride;
  ts = 0;
  ntok = 0;
  r = 0;
  arow = 0;
  if (u < n) {
    const int tile = u / p.S;
    ts = sgmv_tile_start(p.tiles, tile);
    ntok = min(sgmv_tile_start(p.tiles, tile + 1), p.T) - ts;
    const int ad = sgmv_tile_adapter(p.tiles, tile);
    if (ad >= 0) {
      const int64_t rr = p.ranks[ad];
      r = rr <= 0 ? 0 : static_cast<int>(rr < p.R ? rr : p.R);
      arow = p.offsets[ad];
    }
  }
}

// Walks this CTA's units in order (every role the same sequence).  The warp
// calling it must be converged; `get` is collective.
struct UnitCursor {
  int first, stride, n, lane;
  int j = 0;                 // index in this CTA's sequence
  int c_ts, c_ntok, c_r;     // cached batch (per lane)
  int64_t c_arow;
  __device__ UnitCursor(int first_, int stride_, int n_, int lane_) : first(first_), stride(stride_), n(n_), lane(lane_) {}
  __device__ bool next(const UnitArgs& p, UnitInfo& info) {
    const int u = first + j * stride;
    if (u >= n) return false;
    if ((j & 31) == 0) lookup_units(p, u, stride, n, lane, c_ts, c_ntok, c_r, c_arow);
    const int src = j & 31;
    info.ts = __shfl_sync(0xffffffffu, c_ts, src);
    info.ntok = __shfl_sync(0xffffffffu, c_ntok, src);
    info.r = __shfl_sync(0xffffffffu, c_r, src);
    info.arow = __shfl_sync(0xffffffffu, c_arow, src);
    info.tile = u / p.S;
    info.slice = u - info.tile * p.S;
    info.kb0 = info.slice * p.kb_per;
    info.kb1 = min(p.num_kb, info.kb0 + p.kb_per);
    ++j;
    return true;
  }
};

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kUnitThreads, 1) sgmv_shrink_unit_kernel(const __grid_constant__ UnitMaps maps,
                                                                           const UnitArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t bar_off = static_cast<uint32_t>(p.stages * p.stage_bytes);
  if (static_cast<uint32_t>(smem - smem_raw) + bar_off + 512u > dynamic_smem_bytes() || p.stages > kUnitMaxStages) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemLayout);
    return;
  }
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + bar_off);
  uint64_t* empty = full + kUnitMaxStages;
  uint64_t* acc_full = empty + kUnitMaxStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kUnitMaxStages; ++s) {
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
    tmem_alloc(tmem_slot, kUnitTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The schedule kernel launched before this one writes the tile table: wait
  // for it before any global read.  The expand launched next waits for this
  // whole grid before reading z, so it may start its set-up now.
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int n_units = sgmv_num_tiles(p.tiles) * p.S;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    UnitCursor cur(blockIdx.x, gridDim.x, n_units, lane);
    UnitInfo u;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    while (ok && cur.next(p, u)) {
      if (u.empty()) continue;
      const int r16 = (u.r + 15) & ~15, n16 = (u.ntok + 15) & ~15;
      const uint32_t tx = static_cast<uint32_t>((r16 + n16) * kUnitBK * 2);
      for (int kb = u.kb0; kb < u.kb1; ++kb) {
        if (lane == 0) {
          ok = mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, kDevErrTimeoutEmpty);
          if (ok) {
            uint8_t* st = smem + stage * p.stage_bytes;
            mbar_arrive_expect_tx(&full[stage], tx);
            tma_load_2d(&maps.a[(r16 >> 4) - 1], st, &full[stage], kb * kUnitBK, static_cast<int32_t>(u.arow));
            tma_load_2d(&maps.x[(n16 >> 4) - 1], st + p.x_off, &full[stage], kb * kUnitBK, u.ts);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    UnitCursor cur(blockIdx.x, gridDim.x, n_units, lane);
    UnitInfo u;
    int stage = 0, buf = 0;
    uint32_t phase = 0, acc_phase[2] = {0u, 0u};
    bool ok = true;
    const uint32_t idesc_base = umma_idesc_f16(128, 16, std::is_same<T, __nv_bfloat16>::value ? 1 : 0) &
                                ~(0x3Fu << 17);
    while (ok && cur.next(p, u)) {
      if (u.empty()) continue;
      const int n16 = (u.ntok + 15) & ~15;
      const uint32_t idesc = idesc_base | (static_cast<uint32_t>(n16 >> 3) << 17);
      if (lane == 0) {
        ok = mbar_wait_bounded(&acc_empty[buf], acc_phase[buf] ^ 1, abort_flag, p.err, kDevErrTimeoutAccEmpty);
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kUnitAccCols);
        for (int kb = u.kb0; ok && kb < u.kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * p.stage_bytes);
          const uint64_t ad = umma_desc_sw128(sa);
          const uint64_t xd = umma_desc_sw128(sa + static_cast<uint32_t>(p.x_off));
#pragma unroll
          for (int k = 0; k < kUnitBK / 16; ++k)
            tc_mma_f16(d, ad + static_cast<uint64_t>(2 * k), xd + static_cast<uint64_t>(2 * k), idesc,
                       (kb > u.kb0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[stage]);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) tc_commit(&acc_full[buf]);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      acc_phase[buf] ^= 1;
      buf ^= 1;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31 = ranks
    const int et = threadIdx.x - 64;
    const int j = quad * 32 + lane;
    UnitCursor cur(blockIdx.x, gridDim.x, n_units, lane);
    UnitInfo u;
    int buf = 0;
    uint32_t acc_phase[2] = {0u, 0u};
    bool ok = true;
    auto store_z = [&](int t, int col, float v) {
      const int64_t off = static_cast<int64_t>(t) * p.ldz + col;
      if (p.z_f32)
        static_cast<float*>(p.z)[off] = v;
      else
        static_cast<T*>(p.z)[off] = from_f32<T>(v);
    };
    while (cur.next(p, u)) {
      if (u.empty()) {
        // no products: the first slice writes the tile's zero rows
        if (u.slice == 0 && u.ntok > 0)
          for (int idx = et; idx < u.ntok * p.z_width; idx += 128) store_z(u.ts + idx / p.z_width, idx % p.z_width, 0.f);
        continue;
      }
      if (ok) {
        ok = mbar_wait_bounded(&acc_full[buf], acc_phase[buf], abort_flag, p.err, kDevErrTimeoutAccFull);
        tc_fence_after();
      }
      __syncwarp();
      if (ok && quad * 32 < u.r) {
        float* dst = p.partial + (static_cast<int64_t>(u.slice) * p.T + u.ts) * p.R + j;
        for (int c0 = 0; c0 < u.ntok; c0 += 16) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                 static_cast<uint32_t>(buf * kUnitAccCols + c0),
                             v);
          tmem_wait_ld();
          if (j < u.r) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c0 + e < u.ntok) dst[static_cast<int64_t>(c0 + e) * p.R] = __uint_as_float(v[e]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      acc_phase[buf] ^= 1;
      buf ^= 1;
      if (!ok) continue;
      // split-K: the last slice of the tile to arrive sums the partials in order
      __threadfence();
      named_bar_sync(1, 128);
      if (et == 0) {
        const int old = atomicAdd(&p.tickets[u.tile], 1);
        const int last = old == p.S - 1;
        if (last) p.tickets[u.tile] = 0;  // every slice has arrived: return the ticket to zero
        *last_flag = last;
      }
      named_bar_sync(1, 128);
      if (*last_flag) {
        __threadfence();
        for (int idx = et; idx < u.ntok * p.z_width; idx += 128) {
          const int t = idx / p.z_width, col = idx - t * p.z_width;
          float v = 0.f;
          if (col < u.r) {
            const float* src = p.partial + (static_cast<int64_t>(u.ts) + t) * p.R + col;
            for (int s = 0; s < p.S; ++s) v += __ldcg(src + static_cast<int64_t>(s) * p.T * p.R);
            v *= p.scale;
          }
          store_z(u.ts + t, col, v);
        }
      }
      named_bar_sync(1, 128);  // last_flag is rewritten by the next unit
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kUnitTmemCols);
  }
}

namespace {

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

inline bool unit_al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

// Slices and workspace of the unit kernel: K cut into <= 16 slices of >= 512.
int sgmv_unit_split(int64_t K) {
  const int64_t kb = std::max<int64_t>((K + kUnitBK - 1) / kUnitBK, 1);
  int64_t s = std::min<int64_t>(16, std::max<int64_t>(1, (kb + 7) / 8));
  const int64_t per = (kb + s - 1) / s;
  return static_cast<int>((kb + per - 1) / per);
}

size_t sgmv_unit_workspace_bytes(int64_t T, int64_t r_max, int split) {
  return kCounterBytes + static_cast<size_t>(split) * static_cast<size_t>(T) * static_cast<size_t>(r_max) * 4;
}

int launch_sgmv_shrink_unit(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                            const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t max_tiles,
                            void* z, int64_t ldz, int z_dtype, int64_t z_width, int64_t T, int64_t K, int64_t r_max,
                            float scale, int dtype, int split, void* workspace, size_t workspace_bytes, int num_sms,
                            int* err, void* stream) {
  if (r_max <= 0 || r_max > 128 || T <= 0 || K <= 0 || a_rows <= 0 || a_rows > INT32_MAX) return LORA_ERR_UNSUPPORTED;
  if (K % 8 != 0 || ldx % 8 != 0 || lda % 8 != 0 || !unit_al16(x) || !unit_al16(a_flat)) return LORA_ERR_UNSUPPORTED;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (T > INT32_MAX / 2 || K > INT32_MAX || max_tiles > kMaxCounters) return LORA_ERR_UNSUPPORTED;
  const int num_kb = static_cast<int>((K + kUnitBK - 1) / kUnitBK);
  if (split <= 1) return LORA_ERR_UNSUPPORTED;  // the tickets live in a split-K workspace
  const int kb_per = (num_kb + split - 1) / split;
  split = (num_kb + kb_per - 1) / kb_per;
  if (max_tiles * split > INT32_MAX) return LORA_ERR_UNSUPPORTED;
  if (workspace == nullptr || workspace_bytes < sgmv_unit_workspace_bytes(T, r_max, split) || !unit_al16(workspace))
    return LORA_ERR_UNSUPPORTED;
  const int r16max = static_cast<int>((r_max + 15) / 16 * 16);
  // stage: adapter rows (the M = 128 view may run into the x rows after them,
  // whose lanes are never read) then 64 x rows; at least 16 KB so the view stays in the stage
  const int x_off = r16max * 128;
  const int stage_bytes = std::max(16384, ((x_off + 64 * 128) + 1023) & ~1023);
  const int smem_budget = 100 * 1024;  // two CTAs per SM
  int stages = std::min(kUnitMaxStages, (smem_budget - 1024 - 512) / stage_bytes);
  if (stages < 2) return LORA_ERR_UNSUPPORTED;
  const size_t smem = static_cast<size_t>(stages * stage_bytes) + 512 + 1024;

  UnitMaps maps;
  for (int h = 0; h < 8; ++h)
    if (!encode_unit_map(&maps.a[h], a_flat, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(a_rows),
                         static_cast<uint64_t>(lda), static_cast<uint32_t>(16 * (h + 1))))
      return LORA_ERR_CUDA;
  for (int h = 0; h < 4; ++h)
    if (!encode_unit_map(&maps.x[h], x, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(T),
                         static_cast<uint64_t>(ldx), static_cast<uint32_t>(16 * (h + 1))))
      return LORA_ERR_CUDA;
  UnitArgs a{};
  a.z = z;
  a.tickets = static_cast<int*>(workspace);
  a.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  a.offsets = offsets;
  a.ranks = ranks;
  a.tiles = tiles;
  a.err = err;
  a.ldz = ldz;
  a.T = static_cast<int>(T);
  a.K = static_cast<int>(K);
  a.R = static_cast<int>(r_max);
  a.z_width = static_cast<int>(z_width);
  a.z_f32 = z_dtype == LORA_F32 ? 1 : 0;
  a.num_kb = num_kb;
  a.kb_per = kb_per;
  a.S = split;
  a.stages = stages;
  a.stage_bytes = stage_bytes;
  a.x_off = x_off;
  a.scale = scale;

  const int64_t units = max_tiles * split;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(units, 2 * static_cast<int64_t>(num_sms))));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kUnitThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
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


// ===========================================================================
// Segmented multi-adapter expand, unit-scheduled, on Blackwell tensor cores.
//
//   out[t, n] = y[t, n] + scale * sum_j z[t, j] * B[offsets[a(t)] + j, n]
//
// Units = (tile, 256-column chunk of the output).  Per unit:
//   * the producer loads, by TMA, the adapter's B rows [r16 x 256] (the
//     rank-major flat table, columns contiguous: an MN-major MMA operand) and
//     the tile's y rows [n16 x 256], each as four 64-column boxes with
//     128-byte swizzle;
//   * two builder warps turn the tile's z (fp32 or 16-bit) into a bf16/f16
//     hi/lo pair hi = round(s.z), lo = round(s.z - hi) -- the K-major MMA
//     operand [tokens x (hi | lo)] -- written twice, to rows t and t + 64, so
//     the accumulator holds every token in two TMEM lane quadrants and all
//     four drain warps have work;
//   * one thread issues M = 128, N = 256 MMAs over K = r16 (hi) + r16 (lo)
//     into a double-buffered TMEM accumulator (2 x 256 columns);
//   * four drain warps add y (from shared memory) and store out with 16-byte
//     stores; lanes 0..63 take columns 0..127, lanes 64..127 columns 128..255.
// Units of rank 0 or with an unknown adapter copy y to out.  Every wait is
// bounded; there are no inter-CTA waits.
// Reference semantics: segmented_branch.py:31-47 (_expand), ragged_branch.py:18-27,
// multilora.py:295-347.
// ===========================================================================

namespace {

constexpr int kExThreads = 256;
constexpr int kExBN = 256;                 // output columns per unit
constexpr int kExBoxBytes = 64 * 128;      // one 64-column box of up to 64 rows
constexpr int kExStage = 4 * kExBoxBytes;  // four boxes: 256 columns
constexpr int kExZRegion = 128 * 128;      // 128 operand rows x 64 K (hi or lo)
constexpr int kExZOp = 2 * kExZRegion;     // hi | lo
constexpr int kExOffB = 0;
constexpr int kExOffY = 2 * kExStage;
constexpr int kExOffZ = 4 * kExStage;
constexpr int kExOffBar = kExOffZ + 2 * kExZOp;
constexpr int kExSmem = kExOffBar + 256 + 1024;
constexpr uint32_t kExTmemCols = 2 * kExBN;

struct ExpMaps {
  CUtensorMap b[4];  // b_flat [rows, N]: boxes of 64 columns x 16/32/48/64 rows
  CUtensorMap y[4];  // y [T, N]: boxes of 64 columns x 16/32/48/64 rows
};

struct ExpArgs {
  const void* z;
  const void* y;     // only its address matters here (NULL: out = z.B)
  void* out;
  const int64_t* offsets;
  const int64_t* ranks;
  const int32_t* tiles;
  int* err;
  int64_t ldz, ldo, ldy;
  int T, N, R, z_f32, n_chunks;
  float scale;
};

struct ExpUnit {
  int ts, ntok, r, n0;
  int64_t arow;
  __device__ bool empty() const { return ntok <= 0 || r <= 0; }
};

// Walks this CTA's (tile, chunk) units; tables looked up 32 units at a time by the whole warp.
struct ExpCursor {
  int first, stride, n, lane, j = 0;
  int c_ts, c_ntok, c_r;
  int64_t c_arow;
  __device__ ExpCursor(int f, int s, int n_, int l) : first(f), stride(s), n(n_), lane(l) {}
  __device__ bool next(const ExpArgs& p, ExpUnit& e) {
    const int u = first + j * stride;
    if (u >= n) return false;
    if ((j & 31) == 0) {
      const int uu = first + (j + lane) * stride;
      c_ts = c_ntok = c_r = 0;
      c_arow = 0;
      if (uu < n) {
        const int tile = uu / p.n_chunks;
        c_ts = sgmv_tile_start(p.tiles, tile);
        c_ntok = min(sgmv_tile_start(p.tiles, tile + 1), p.T) - c_ts;
        const int ad = sgmv_tile_adapter(p.tiles, tile);
        if (ad >= 0) {
          const int64_t rr = p.ranks[ad];
          c_r = rr <= 0 ? 0 : static_cast<int>(rr < p.R ? rr : p.R);
          c_arow = p.offsets[ad];
        }
      }
    }
    const int src = j & 31;
    e.ts = __shfl_sync(0xffffffffu, c_ts, src);
    e.ntok = __shfl_sync(0xffffffffu, c_ntok, src);
    e.r = __shfl_sync(0xffffffffu, c_r, src);
    e.arow = __shfl_sync(0xffffffffu, c_arow, src);
    e.n0 = (u % p.n_chunks) * kExBN;
    ++j;
    return true;
  }
};

// Shared-memory descriptor of an MN-major operand written by TMA as 64-element
// (128-byte) wide boxes with 128-byte swizzle: K rows 128 B apart, 8-row
// groups 1024 B apart (SBO), 64-wide MN groups `lbo` bytes apart (LBO).
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

template <typename T>
__global__ void __launch_bounds__(kExThreads, 1) sgmv_expand_unit_kernel(const __grid_constant__ ExpMaps maps,
                                                                         const ExpArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if (static_cast<uint32_t>(smem - smem_raw) + static_cast<uint32_t>(kExOffBar) + 256u > dynamic_smem_bytes()) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemLayout);
    return;
  }
  uint64_t* bfull = reinterpret_cast<uint64_t*>(smem + kExOffBar);
  uint64_t* bempty = bfull + 2;
  uint64_t* yfull = bempty + 2;
  uint64_t* yempty = yfull + 2;
  uint64_t* zfull = yempty + 2;
  uint64_t* zempty = zfull + 2;
  uint64_t* afull = zempty + 2;
  uint64_t* aempty = afull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool has_y = p.y != nullptr;
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bfull[b], 1);
      mbar_init(&bempty[b], 1);
      mbar_init(&yfull[b], 1);
      mbar_init(&yempty[b], 4);
      mbar_init(&zfull[b], 1);
      mbar_init(&zempty[b], 1);
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int h = 0; h < 4; ++h) {
      tma_prefetch_desc(&maps.b[h]);
      if (has_y) tma_prefetch_desc(&maps.y[h]);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kExTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // z comes from the shrink launched just before; the tile table from the
  // schedule before that: wait for both before any global read.
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int n_units = sgmv_num_tiles(p.tiles) * p.n_chunks;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    ExpCursor cur(blockIdx.x, gridDim.x, n_units, lane);
    ExpUnit u;
    int i = 0;
    bool ok = true;
    while (ok && cur.next(p, u)) {
      if (u.empty()) continue;
      const int r16 = (u.r + 15) & ~15, n16 = (u.ntok + 15) & ~15;
      const int s = i & 1;
      const uint32_t ph = static_cast<uint32_t>((i >> 1) & 1);
      if (lane == 0) {
        ok = mbar_wait_bounded(&bempty[s], ph ^ 1, abort_flag, p.err, kDevErrTimeoutEmpty);
        if (ok) {
          mbar_arrive_expect_tx(&bfull[s], static_cast<uint32_t>(4 * r16 * 128));
          for (int g = 0; g < 4; ++g)
            tma_load_2d(&maps.b[(r16 >> 4) - 1], smem + kExOffB + s * kExStage + g * kExBoxBytes, &bfull[s],
                        u.n0 + 64 * g, static_cast<int32_t>(u.arow));
        }
        if (ok && has_y) {
          ok = mbar_wait_bounded(&yempty[s], ph ^ 1, abort_flag, p.err, kDevErrTimeoutEmpty);
          if (ok) {
            mbar_arrive_expect_tx(&yfull[s], static_cast<uint32_t>(4 * n16 * 128));
            for (int g = 0; g < 4; ++g)
              tma_load_2d(&maps.y[(n16 >> 4) - 1], smem + kExOffY + s * kExStage + g * kExBoxBytes, &yfull[s],
                          u.n0 + 64 * g, u.ts);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++i;
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    ExpCursor cur(blockIdx.x, gridDim.x, n_units, lane);
    ExpUnit u;
    int i = 0;
    bool ok = true;
    // M = 128, N = 256, A (z) K-major, B (adapter rows) MN-major
    const uint32_t idesc = umma_idesc_f16(128, kExBN, std::is_same<T, __nv_bfloat16>::value ? 1 : 0) | (1u << 16);
    while (ok && cur.next(p, u)) {
      if (u.empty()) continue;
      const int r16 = (u.r + 15) & ~15;
      const int s = i & 1;
      const uint32_t ph = static_cast<uint32_t>((i >> 1) & 1);
      if (lane == 0) {
        ok = mbar_wait_bounded(&zfull[s], ph, abort_flag, p.err, kDevErrTimeoutFull) &&
             mbar_wait_bounded(&bfull[s], ph, abort_flag, p.err, kDevErrTimeoutFull) &&
             mbar_wait_bounded(&aempty[s], ph ^ 1, abort_flag, p.err, kDevErrTimeoutAccEmpty);
        if (ok) {
          tc_fence_after();
          const uint32_t d = tmem_base + static_cast<uint32_t>(s * kExBN);
          const uint32_t zs = smem_u32(smem + kExOffZ + s * kExZOp);
          const uint32_t bs = smem_u32(smem + kExOffB + s * kExStage);
          for (int h = 0; h < 2; ++h) {
            const uint64_t ad = umma_desc_sw128(zs + static_cast<uint32_t>(h * kExZRegion));
            for (int ks = 0; ks < r16 / 16; ++ks) {
              const uint64_t bd = umma_desc_sw128_mn(bs + static_cast<uint32_t>(ks * 2048), kExBoxBytes);
              tc_mma_f16(d, ad + static_cast<uint64_t>(2 * ks), bd, idesc, (h > 0 || ks > 0) ? 1u : 0u);
            }
          }
          tc_commit(&bempty[s]);
          tc_commit(&zempty[s]);
          tc_commit(&afull[s]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++i;
    }
  } else if (warp >= 6) {
    // ----------------------------------------------- z operand builders (64 threads)
    const int bt = threadIdx.x - 192;
    ExpCursor cur(blockIdx.x, gridDim.x, n_units, lane);
    ExpUnit u;
    int i = 0;
    bool ok = true;
    while (cur.next(p, u)) {
      if (u.empty()) continue;
      const int s = i & 1;
      const uint32_t ph = static_cast<uint32_t>((i >> 1) & 1);
      ++i;
      if (ok) ok = mbar_wait_bounded(&zempty[s], ph ^ 1, abort_flag, p.err, kDevErrTimeoutEmpty);
      if (!ok) continue;
      uint8_t* zop = smem + kExOffZ + s * kExZOp;
      const int r16 = (u.r + 15) & ~15;
      const int chunks = r16 >> 3;  // 8 ranks (16 bytes) per chunk
      for (int idx = bt; idx < 64 * chunks; idx += 64) {
        const int t = idx / chunks, c = idx - t * chunks;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
        if (t < u.ntok) {
          const int64_t base = static_cast<int64_t>(u.ts + t) * p.ldz + c * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (c * 8 + e < u.r)
              v[e] = p.z_f32 ? static_cast<const float*>(p.z)[base + e] : to_f32(static_cast<const T*>(p.z)[base + e]);
          }
        }
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = p.scale * v[2 * e], b = p.scale * v[2 * e + 1];
          hi[e] = pack2<T>(a, b);
          const float2 hv = unpack2<T>(hi[e]);
          lo[e] = pack2<T>(a - hv.x, b - hv.y);
        }
        const uint4 h4 = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        const uint4 l4 = make_uint4(lo[0], lo[1], lo[2], lo[3]);
#pragma unroll
        for (int dup = 0; dup < 2; ++dup) {
          const int row = t + 64 * dup;
          const int off = row * 128 + ((c ^ (row & 7)) << 4);
          *reinterpret_cast<uint4*>(zop + off) = h4;
          *reinterpret_cast<uint4*>(zop + kExZRegion + off) = l4;
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(2, 64);
      if (bt == 0) mbar_arrive(&zfull[s]);
    }
  } else {
    // --------------------------------------------------- drain (warps 2..5)
    const int quad = warp & 3;
    const int t = (quad * 32 + lane) & 63;  // lanes 64..127 repeat tokens 0..63
    const int half = quad >> 1;             // which 128 columns this warp stores
    ExpCursor cur(blockIdx.x, gridDim.x, n_units, lane);
    ExpUnit u;
    int i = 0;
    bool ok = true;
    while (cur.next(p, u)) {
      if (u.empty()) {
        // rank 0 / unknown adapter: out = y (zeros without y), this warp's token rows and columns
        for (int rr = 0; rr < 32; ++rr) {
          const int tt = (quad & 1) * 32 + rr;
          if (tt >= u.ntok) break;
          const int col = u.n0 + half * 128 + lane * 4;
          if (col >= p.N) continue;
          T* o = static_cast<T*>(p.out) + static_cast<int64_t>(u.ts + tt) * p.ldo + col;
          const T* yy = has_y ? static_cast<const T*>(p.y) + static_cast<int64_t>(u.ts + tt) * p.ldy + col : nullptr;
          if (col + 4 <= p.N) {
            uint2 v = has_y ? *reinterpret_cast<const uint2*>(yy) : make_uint2(0u, 0u);
            *reinterpret_cast<uint2*>(o) = v;
          } else {
            for (int e = 0; col + e < p.N; ++e) o[e] = has_y ? yy[e] : from_f32<T>(0.f);
          }
        }
        continue;
      }
      const int s = i & 1;
      const uint32_t ph = static_cast<uint32_t>((i >> 1) & 1);
      ++i;
      if (ok) ok = mbar_wait_bounded(&afull[s], ph, abort_flag, p.err, kDevErrTimeoutAccFull);
      if (ok && has_y) ok = mbar_wait_bounded(&yfull[s], ph, abort_flag, p.err, kDevErrTimeoutFull);
      tc_fence_after();
      __syncwarp();
      if (ok) {
        const uint8_t* ys = smem + kExOffY + s * kExStage;
        T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(u.ts + t) * p.ldo;
        const bool live = t < u.ntok;
#pragma unroll 1
        for (int cg = 0; cg < 8; ++cg) {
          const int col = half * 128 + cg * 16;  // within the unit's 256 columns
          uint32_t v[16];
          tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                 static_cast<uint32_t>(s * kExBN + col),
                             v);
          tmem_wait_ld();
          const int g = col >> 6, c0 = (col & 63) >> 3;
          uint4 yv[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
          if (has_y) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
              yv[h] = *reinterpret_cast<const uint4*>(ys + g * kExBoxBytes + t * 128 + (((c0 + h) ^ (t & 7)) << 4));
          }
          const int gcol = u.n0 + col;
          if (live && gcol < p.N) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t* yw = reinterpret_cast<const uint32_t*>(&yv[h]);
              uint32_t ow[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 yf = unpack2<T>(yw[e]);
                ow[e] = pack2<T>(yf.x + __uint_as_float(v[8 * h + 2 * e]), yf.y + __uint_as_float(v[8 * h + 2 * e + 1]));
              }
              if (gcol + 8 * h + 8 <= p.N) {
                *reinterpret_cast<uint4*>(orow + gcol + 8 * h) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
              } else {
                const T* ot = reinterpret_cast<const T*>(ow);
                for (int e = 0; gcol + 8 * h + e < p.N; ++e) orow[gcol + 8 * h + e] = ot[e];
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&aempty[s]);
        if (has_y) mbar_arrive(&yempty[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kExTmemCols);
  }
}

int launch_sgmv_expand_unit(const void* y, int64_t ldy, const void* z, int64_t ldz, int z_dtype, const void* b,
                            int64_t b_rows, int64_t ldb, const int64_t* offsets, const int64_t* ranks,
                            const int32_t* tiles, int64_t max_tiles, void* out, int64_t ldo, int64_t T, int64_t N,
                            int64_t r_max, float scale, int dtype, int num_sms, int* err, void* stream) {
  if (r_max <= 0 || r_max > 64 || T <= 0 || N <= 0 || b_rows <= 0 || b_rows > INT32_MAX) return LORA_ERR_UNSUPPORTED;
  if (N % 8 != 0 || ldb % 8 != 0 || ldo % 8 != 0 || !unit_al16(b) || !unit_al16(out)) return LORA_ERR_UNSUPPORTED;
  if (y != nullptr && (ldy % 8 != 0 || !unit_al16(y))) return LORA_ERR_UNSUPPORTED;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (T > INT32_MAX / 2 || N > INT32_MAX / 2) return LORA_ERR_UNSUPPORTED;
  const int64_t n_chunks = (N + kExBN - 1) / kExBN;
  if (max_tiles * n_chunks > INT32_MAX) return LORA_ERR_UNSUPPORTED;

  ExpMaps maps;
  for (int h = 0; h < 4; ++h) {
    if (!encode_unit_map(&maps.b[h], b, dtype, static_cast<uint64_t>(N), static_cast<uint64_t>(b_rows),
                         static_cast<uint64_t>(ldb), static_cast<uint32_t>(16 * (h + 1))))
      return LORA_ERR_CUDA;
    if (y != nullptr) {
      if (!encode_unit_map(&maps.y[h], y, dtype, static_cast<uint64_t>(N), static_cast<uint64_t>(T),
                           static_cast<uint64_t>(ldy), static_cast<uint32_t>(16 * (h + 1))))
        return LORA_ERR_CUDA;
    } else {
      maps.y[h] = maps.b[h];
    }
  }
  ExpArgs a{};
  a.z = z;
  a.y = y;
  a.out = out;
  a.offsets = offsets;
  a.ranks = ranks;
  a.tiles = tiles;
  a.err = err;
  a.ldz = ldz;
  a.ldo = ldo;
  a.ldy = ldy;
  a.T = static_cast<int>(T);
  a.N = static_cast<int>(N);
  a.R = static_cast<int>(r_max);
  a.z_f32 = z_dtype == LORA_F32 ? 1 : 0;
  a.n_chunks = static_cast<int>(n_chunks);
  a.scale = scale;

  const int64_t units = max_tiles * n_chunks;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(units, num_sms)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kExThreads);
  cfg.dynamicSmemBytes = kExSmem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
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

}  // namespace lora
