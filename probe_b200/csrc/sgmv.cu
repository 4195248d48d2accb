// Device-side tile scheduling for segmented multi-adapter LoRA.
//
// The serving batch arrives either as per-token adapter ids (ragged_branch,
// multilora BGMV) or as contiguous request segments (segmented_branch).  One
// 1024-thread CTA turns either form into a list of tiles of <= 64 consecutive
// tokens that share one adapter: a tile starts at every 64-token boundary and
// wherever the adapter changes.  The shrink / expand kernels then walk that
// list, so a segment's adapter rows are fetched once per 64 tokens instead of
// once per token, and no host synchronisation is needed (the tile count stays
// on the device).  Segments may have any length -- the Zipf-distributed
// request lengths of a real batch -- unlike the reference's segmented_branch,
// which requires equal-length requests (segmented_branch.py:50-53).
#include <algorithm>

#include "common.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

namespace {

// Segment tables up to this many entries are staged in shared memory, so the
// per-token lookups below cost no global round trips.
constexpr int kSchedSmemSegs = 4096;

// A segment boundary clamped to [-1, T+1]: comparisons against tokens in
// [0, T) are unchanged and the value fits an int.
__device__ __forceinline__ int clamp_start(int64_t v, int T) {
  return v < -1 ? -1 : (v > T + 1 ? T + 1 : static_cast<int>(v));
}

// Adapter of token t, or -1 (out of range / not covered by any segment).
struct AdapterLookup {
  const int64_t* ids;
  const int64_t* seg_start;
  const int64_t* seg_adapter;
  const int* s_start;    // shared-memory copy of seg_start (clamped to [-1, T+1]) or NULL
  const int* s_adapter;  // shared-memory copy of seg_adapter (-1 where out of range) or NULL
  int T, S, n_adapters;
  int* err;

  __device__ int start(int s) const {
    return s_start ? s_start[s] : clamp_start(seg_start[s], T);
  }

  __device__ int find_segment(int t) const {
    // largest s with seg_start[s] <= t, s in [0, S)
    int lo = 0, hi = S - 1, ans = -1;
    while (lo <= hi) {
      const int mid = (lo + hi) >> 1;
      if (start(mid) <= t) {
        ans = mid;
        lo = mid + 1;
      } else {
        hi = mid - 1;
      }
    }
    return ans;
  }

  __device__ int validate(int64_t a) const {
    if (a < 0 || a >= n_adapters) {
      record_error(err, kDevErrBadIndex);
      return -1;
    }
    return static_cast<int>(a);
  }

  // seg: running segment index for monotone walks (segment mode only)
  __device__ int operator()(int t, int& seg) const {
    if (ids != nullptr) return validate(ids[t]);
    while (seg + 1 < S && start(seg + 1) <= t) ++seg;
    if (seg < 0 || t < start(seg) || t >= start(seg + 1)) {
      record_error(err, kDevErrBadIndex);
      return -1;
    }
    return validate(s_adapter ? s_adapter[seg] : seg_adapter[seg]);
  }
};

// Exclusive prefix sum of `count` over the block, in thread order; `total`
// receives the sum.  Two block barriers; every thread of the block calls it.
__device__ int block_exclusive_scan(int count, int* warp_sum, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int incl = count;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? warp_sum[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += v;
    }
    warp_sum[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  total = warp_sum[nwarps - 1];
  return incl - count + (warp > 0 ? warp_sum[warp - 1] : 0);
}

// Segment i of a table that covers [0, T) in order: its tokens [a, b), its
// adapter (-1 if out of range) and whether a tile starts at a (a is a
// multiple of 64, or the token before it -- in the last non-empty segment
// before i -- has another adapter).  Tiles also start at every multiple of 64
// inside (a, b).
struct SegTiles {
  int a, b, ad;
  bool first;
  __device__ int count() const {
    return b > a ? (first ? 1 : 0) + (b - 1) / kSgmvTileTokens - a / kSgmvTileTokens : 0;
  }
};

__device__ SegTiles seg_tiles(int i, const int* s_start, const int* s_adapter) {
  SegTiles g{s_start[i], s_start[i + 1], s_adapter[i], false};
  if (g.b > g.a) {
    if (g.a % kSgmvTileTokens == 0) {
      g.first = true;
    } else {
      int j = i - 1;
      while (j >= 0 && s_start[j] == g.a) --j;  // skip empty segments
      g.first = j < 0 || s_adapter[j] != g.ad;
    }
  }
  return g;
}

// One tile entry: start token t, adapter ad, index idx (entries past
// max_tiles are counted but not stored).
__device__ __forceinline__ void put_tile(int32_t* tiles, int max_tiles, int idx, int t, int ad) {
  if (t % kSgmvTileTokens == 0) tiles[3 + 2 * max_tiles + t / kSgmvTileTokens] = min(idx, max_tiles);
  if (idx < max_tiles) {
    tiles[2 + idx] = t;
    tiles[3 + max_tiles + idx] = ad;
  }
}

}  // namespace

__global__ void __launch_bounds__(1024) sgmv_schedule_kernel(AdapterLookup look, int32_t* tiles, int max_tiles) {
  __shared__ int warp_sum[32];
  __shared__ int s_start[kSchedSmemSegs + 1];
  __shared__ int s_adapter[kSchedSmemSegs];
  const int tid = threadIdx.x, nth = blockDim.x;
  const int T = look.T;
  // Launched with programmatic serialization: the segment table (and the tile
  // buffer, which the kernel before may still read) wait for that kernel.  The
  // segmented shrink launched next may set up (barriers, TMEM) meanwhile; it
  // waits for this grid before reading the table.
  pdl_wait();
  if (tid == 0) pdl_launch_dependents();
  const bool staged = look.ids == nullptr && look.S <= kSchedSmemSegs;
  if (staged) {
    for (int i = tid; i <= look.S; i += nth) {
      s_start[i] = clamp_start(look.seg_start[i], T);
      if (i < look.S) {
        const int64_t a = look.seg_adapter[i];
        s_adapter[i] = (a < 0 || a >= look.n_adapters) ? -1 : static_cast<int>(a);
      }
    }
    look.s_start = s_start;
    look.s_adapter = s_adapter;
  }
  __syncthreads();
  // A staged table that covers [0, T) in order (the usual serving batch) is
  // tiled segment by segment: O(S) work instead of a walk over every token.
  bool by_segment = false;
  if (staged) {
    int ordered = 1;
    for (int i = tid; i < look.S; i += nth) ordered &= s_start[i] <= s_start[i + 1] ? 1 : 0;
    if (tid == 0) ordered &= (s_start[0] == 0 && s_start[look.S] == T) ? 1 : 0;
    by_segment = __syncthreads_and(ordered) != 0;
  }
  int total = 0;
  if (by_segment) {
    const int per = (look.S + nth - 1) / nth;  // contiguous segments per thread, in order
    const int s0 = min(look.S, tid * per), s1 = min(look.S, s0 + per);
    int count = 0;
    for (int i = s0; i < s1; ++i) {
      const SegTiles g = seg_tiles(i, s_start, s_adapter);
      if (g.b > g.a && g.ad < 0) record_error(look.err, kDevErrBadIndex);
      count += g.count();
    }
    int idx = block_exclusive_scan(count, warp_sum, total);
    for (int i = s0; i < s1; ++i) {
      const SegTiles g = seg_tiles(i, s_start, s_adapter);
      if (g.b <= g.a) continue;
      if (g.first) put_tile(tiles, max_tiles, idx++, g.a, g.ad);
      for (int m = (g.a / kSgmvTileTokens + 1) * kSgmvTileTokens; m < g.b; m += kSgmvTileTokens)
        put_tile(tiles, max_tiles, idx++, m, g.ad);
    }
  } else {
    // token by token: per-token ids, or a table with gaps, overlaps or more
    // than kSchedSmemSegs entries
    const int chunk = (T + nth - 1) / nth;
    const int c0 = min(T, tid * chunk), c1 = min(T, c0 + chunk);
    int seg = -1;
    if (look.ids == nullptr && c0 < c1) seg = look.find_segment(c0 > 0 ? c0 - 1 : 0);
    int prev = -2;
    if (c0 > 0 && c0 < c1) {
      int s2 = seg;
      prev = look(c0 - 1, s2);
      seg = s2;
    }
    int count = 0;
    {
      int s = seg, pv = prev;
      for (int t = c0; t < c1; ++t) {
        const int a = look(t, s);
        if ((t % kSgmvTileTokens) == 0 || a != pv) ++count;
        pv = a;
      }
    }
    int idx = block_exclusive_scan(count, warp_sum, total);
    int s = seg, pv = prev;
    for (int t = c0; t < c1; ++t) {
      const int a = look(t, s);
      if ((t % kSgmvTileTokens) == 0 || a != pv) put_tile(tiles, max_tiles, idx++, t, a);
      pv = a;
    }
  }
  if (tid == 0) {
    const int n = min(total, max_tiles);
    if (total > max_tiles) record_error(look.err, kDevErrBadIndex);
    tiles[0] = n;
    tiles[1] = max_tiles;
    tiles[2 + n] = T;
    tiles[3 + 2 * max_tiles + (T + kSgmvTileTokens - 1) / kSgmvTileTokens] = n;
  }
}

}  // namespace lora

using namespace lora;

extern "C" size_t lora_sgmv_tiles_size(int64_t T, int64_t S) {
  return static_cast<size_t>(sgmv_tiles_bytes(std::max<int64_t>(T, 0), std::max<int64_t>(S, 0)));
}

extern "C" int lora_sgmv_schedule(const int64_t* ids, const int64_t* seg_start, const int64_t* seg_adapter, int64_t T,
                                  int64_t S, int64_t n_adapters, int32_t* tiles, size_t tiles_bytes, void* stream) {
  if (tiles == nullptr) return LORA_ERR_ARG;
  if (T < 0 || S < 0 || n_adapters < 0 || T > INT32_MAX / 2) return LORA_ERR_SHAPE;
  if (ids == nullptr && (seg_start == nullptr || seg_adapter == nullptr || (S == 0 && T > 0))) return LORA_ERR_ARG;
  if (ids != nullptr) S = 0;
  if (tiles_bytes < lora_sgmv_tiles_size(T, S)) return LORA_ERR_WORKSPACE;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  AdapterLookup look{ids, seg_start, seg_adapter, nullptr, nullptr, static_cast<int>(T), static_cast<int>(S),
                     static_cast<int>(std::min<int64_t>(n_adapters, INT32_MAX)), device_info(dev).err_word};
  const int64_t mt = sgmv_max_tiles(T, S);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(1024);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, sgmv_schedule_kernel, look, tiles, static_cast<int>(mt)) == cudaSuccess
             ? LORA_OK
             : LORA_ERR_CUDA;
}
