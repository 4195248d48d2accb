// Rank shrink  z = scale * x . A^T  (the skinny, memory-bound half of LoRA).
//
// One kernel serves the single-adapter shrink (lora_shrink) and the
// segmented multi-adapter shrink (lora_sgmv_shrink):
//   - a work tile is <= 64 consecutive tokens that share one adapter;
//   - each warp multiplies 16 tokens against the adapter's R rows with
//     mma.sync m16n8k16 (fp32 accumulate).  Both operands are read with
//     16-byte loads, 32 contiguous bytes per thread: the K order inside a
//     64-wide step is permuted identically for x and A, which leaves the dot
//     product unchanged and keeps every access a full 32-byte sector;
//   - K is split over CTAs (blockIdx.y).  Each split writes fp32 partials to
//     the workspace; the last CTA to finish a tile (atomic ticket) sums them
//     in split order, so results are deterministic and no float atomics are
//     needed.  The ticket counters sit in a fixed region at the start of the
//     workspace and the last CTA of each tile returns its counter to zero;
//   - optionally z is written as a bf16/f16 hi/lo pair (hi = round(v),
//     lo = round(v - hi), lo at column + z_width): fed to a tensor-core
//     expand as two K-slices against a duplicated B, the pair carries ~16
//     mantissa bits, so the expand is as accurate as an fp32 one.
// With M <= 32 the four warps of a CTA also split their K slice and reduce
// through shared memory, so decode-sized shrinks still fill the machine.
//
// Reference semantics: splitk_lora.py:22-63,104-126 (fp32 partials + sum),
// splitk_shrink.py:34-141, multilora.py:128-182 (ragged table lookup),
// segmented_branch.py:12-28 and ragged_branch.py:6-16 (per-segment / per-token
// adapter, rank-0 skip).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

struct ShrinkArgs {
  const void* x;
  const void* a;
  void* z;
  float* partial;     // [split_k][M][pr] fp32, pr = partial row width
  int* counters;      // one per tile
  const int64_t* offsets;  // SGMV only
  const int64_t* ranks;    // SGMV only
  const int32_t* tiles;    // SGMV only: schedule (sgmv.h), NULL = plain shrink
  const int64_t* rows;     // SGMV only: logical token -> physical row (NULL = identity)
  int* err;
  int64_t ldx, lda, ldz;
  int M, K, R, z_width, pr;
  int n_adapters;
  int z_split;          // 1: also write lo = v - round(v) at column + z_width
  int split_k, kslice;  // kslice: multiple of 64
  int wt;               // token sub-tiles per CTA (1, 2, 4); 4 / wt warps split K
  int num_tiles_plain;
  float scale;
};

template <bool ALIGNED, typename T>
LORA_DEVINL uint4 load8(const T* row, int k, int k_end, bool valid) {
  if (!valid) return make_uint4(0, 0, 0, 0);
  if (ALIGNED) {
    if (k < k_end) return ldg_stream(row + k);
    return make_uint4(0, 0, 0, 0);
  }
  union {
    uint4 v;
    T e[8];
  } u;
#pragma unroll
  for (int i = 0; i < 8; ++i) u.e[i] = (k + i < k_end) ? row[k + i] : from_f32<T>(0.f);
  return u.v;
}

template <bool ALIGNED, typename T>
LORA_DEVINL uint4 load8_cached(const T* row, int k, int k_end, bool valid) {
  if (!valid) return make_uint4(0, 0, 0, 0);
  if (ALIGNED) {
    if (k < k_end) return __ldg(reinterpret_cast<const uint4*>(row + k));
    return make_uint4(0, 0, 0, 0);
  }
  return load8<false, T>(row, k, k_end, true);
}

// acc[nt][*] += x[row0 .. row0+16) . A[nt*8 .. nt*8+8)^T over the 64-wide K
// steps k_first, k_first + k_stride, ... < k_end.
LORA_DEVINL int64_t phys_row(const int64_t* rows, int64_t t) { return rows ? rows[t] : t; }

template <bool ALIGNED, typename T, int NT>
LORA_DEVINL void shrink_warp(const T* x, int64_t ldx, const int64_t* rows, int row0, int nrows, const T* a,
                             int64_t lda, int R, int k_first, int k_stride, int k_end, float (&acc)[NT][4]) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const bool v0 = g < nrows, v1 = g + 8 < nrows;
  const T* xr0 = x + phys_row(rows, row0 + (v0 ? g : 0)) * ldx;
  const T* xr1 = x + phys_row(rows, row0 + (v1 ? g + 8 : 0)) * ldx;
#pragma unroll 1
  for (int k = k_first; k < k_end; k += k_stride) {
    const int kc = k + 16 * q;
    const uint4 x00 = load8<ALIGNED>(xr0, kc, k_end, v0);
    const uint4 x01 = load8<ALIGNED>(xr0, kc + 8, k_end, v0);
    const uint4 x10 = load8<ALIGNED>(xr1, kc, k_end, v1);
    const uint4 x11 = load8<ALIGNED>(xr1, kc + 8, k_end, v1);
    const uint32_t wg[8] = {x00.x, x00.y, x00.z, x00.w, x01.x, x01.y, x01.z, x01.w};
    const uint32_t wh[8] = {x10.x, x10.y, x10.z, x10.w, x11.x, x11.y, x11.z, x11.w};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (nt * 8 >= R) break;
      const int n = nt * 8 + g;
      const bool vn = n < R;
      const T* ar = a + static_cast<int64_t>(vn ? n : 0) * lda;
      const uint4 a0 = load8_cached<ALIGNED>(ar, kc, k_end, vn);
      const uint4 a1 = load8_cached<ALIGNED>(ar, kc + 8, k_end, vn);
      const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t af[4] = {wg[2 * j], wh[2 * j], wg[2 * j + 1], wh[2 * j + 1]};
        const uint32_t bf[2] = {wa[2 * j], wa[2 * j + 1]};
        mma16816<T>(acc[nt], af, bf);
      }
    }
  }
}

// z_row[col] = v rounded to TZ; with split, z_row[col + width] = the residual.
template <typename TZ>
LORA_DEVINL void store_z(TZ* z_row, int col, int width, int split, float v) {
  const TZ hi = from_f32<TZ>(v);
  z_row[col] = hi;
  if (split) z_row[col + width] = from_f32<TZ>(v - to_f32(hi));
}

template <bool ALIGNED, typename T, typename TZ, int NT>
__global__ void __launch_bounds__(128) shrink_kernel(const ShrinkArgs p) {
  // A kernel launched after this one with programmatic serialization (the
  // decode GEMV) may start streaming W now; it reads z only after
  // griddepcontrol.wait, i.e. after this grid has completed.
  pdl_launch_dependents();
  __shared__ float red[4][16][NT * 8 + 1];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int wt = p.wt, wk = 4 / p.wt;
  const int t_sub = warp % wt, k_sub = warp / wt;
  const int tile_tokens = 16 * wt;
  const int ks = blockIdx.y;
  const int k_begin = ks * p.kslice;
  const int k_end = min(p.K, k_begin + p.kslice);
  const T* x = static_cast<const T*>(p.x);
  TZ* z = static_cast<TZ*>(p.z);

  const int num_tiles = p.tiles ? sgmv_num_tiles(p.tiles) : p.num_tiles_plain;
  for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
    // ---- resolve the tile: token range, adapter rows, rank
    int t0, t1, R;
    const T* a;
    if (p.tiles) {
      t0 = sgmv_tile_start(p.tiles, tile);
      t1 = sgmv_tile_start(p.tiles, tile + 1);
      const int ad = sgmv_tile_adapter(p.tiles, tile);
      if (ad >= 0) {
        R = static_cast<int>(p.ranks[ad] < p.R ? p.ranks[ad] : p.R);
        a = static_cast<const T*>(p.a) + p.offsets[ad] * p.lda;
      } else {
        R = 0;
        a = static_cast<const T*>(p.a);
      }
    } else {
      t0 = tile * tile_tokens;
      t1 = min(p.M, t0 + tile_tokens);
      R = p.R;
      a = static_cast<const T*>(p.a);
    }
    const int row0 = t0 + t_sub * 16;
    const int nrows = min(16, t1 - row0);

    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    if (nrows > 0 && R > 0)
      shrink_warp<ALIGNED, T, NT>(x, p.ldx, p.rows, row0, nrows, a, p.lda, R, k_begin + 64 * k_sub, 64 * wk, k_end,
                                  acc);

    // ---- reduce the K sub-slices of this CTA's warps through shared memory
    if (wk > 1) {
      if (k_sub > 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          red[warp][g][nt * 8 + 2 * q] = acc[nt][0];
          red[warp][g][nt * 8 + 2 * q + 1] = acc[nt][1];
          red[warp][g + 8][nt * 8 + 2 * q] = acc[nt][2];
          red[warp][g + 8][nt * 8 + 2 * q + 1] = acc[nt][3];
        }
      }
      __syncthreads();
      if (k_sub == 0) {
        for (int s = 1; s < wk; ++s) {
          const int w2 = t_sub + s * wt;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] += red[w2][g][nt * 8 + 2 * q];
            acc[nt][1] += red[w2][g][nt * 8 + 2 * q + 1];
            acc[nt][2] += red[w2][g + 8][nt * 8 + 2 * q];
            acc[nt][3] += red[w2][g + 8][nt * 8 + 2 * q + 1];
          }
        }
      }
    }

    // ---- write: final z (no split) or fp32 partials
    if (k_sub == 0 && nrows > 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = g + 8 * h;
          if (row >= nrows) continue;
          const int64_t t = row0 + row;
          const int64_t pt = phys_row(p.rows, t);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int col = nt * 8 + 2 * q + e;
            if (p.split_k == 1) {
              if (col < p.z_width)
                store_z<TZ>(z + pt * p.ldz, col, p.z_width, p.z_split, col < R ? p.scale * acc[nt][2 * h + e] : 0.f);
            } else if (col < p.pr) {
              p.partial[(static_cast<int64_t>(ks) * p.M + t) * p.pr + col] = acc[nt][2 * h + e];
            }
          }
        }
      }
      if (p.split_k == 1) {
        // zero-fill columns beyond the mma tiles up to z_width
        for (int row = 0; row < nrows; ++row)
          for (int col = NT * 8 + lane; col < p.z_width; col += 32)
            store_z<TZ>(z + phys_row(p.rows, row0 + row) * p.ldz, col, p.z_width, p.z_split, 0.f);
      }
    }

    if (p.split_k > 1) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.counters[tile], 1);
        s_last = (prev == p.split_k - 1);
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        const int ntok = t1 - t0;
        const int width = p.z_width;
        for (int idx = threadIdx.x; idx < ntok * width; idx += blockDim.x) {
          const int row = idx / width, col = idx - row * width;
          const int64_t t = t0 + row;
          float v = 0.f;
          if (col < R) {
            for (int s = 0; s < p.split_k; ++s) v += __ldcg(&p.partial[(static_cast<int64_t>(s) * p.M + t) * p.pr + col]);
            v *= p.scale;
          }
          store_z<TZ>(z + phys_row(p.rows, t) * p.ldz, col, width, p.z_split, v);
        }
        if (threadIdx.x == 0) p.counters[tile] = 0;
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------- host
namespace {

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int shrink_wt(int64_t M) { return M <= 16 ? 1 : (M <= 32 ? 2 : 4); }

template <bool AL, typename T, typename TZ>
int launch_shrink_nt(int nt, const ShrinkArgs& p, dim3 grid, cudaStream_t s) {
  switch (nt) {
    case 1: shrink_kernel<AL, T, TZ, 1><<<grid, 128, 0, s>>>(p); break;
    case 2: shrink_kernel<AL, T, TZ, 2><<<grid, 128, 0, s>>>(p); break;
    case 4: shrink_kernel<AL, T, TZ, 4><<<grid, 128, 0, s>>>(p); break;
    case 8: shrink_kernel<AL, T, TZ, 8><<<grid, 128, 0, s>>>(p); break;
    case 16: shrink_kernel<AL, T, TZ, 16><<<grid, 128, 0, s>>>(p); break;
    default: return LORA_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

template <typename T, typename TZ>
int launch_shrink_t(bool aligned, int nt, const ShrinkArgs& p, dim3 grid, cudaStream_t s) {
  return aligned ? launch_shrink_nt<true, T, TZ>(nt, p, grid, s) : launch_shrink_nt<false, T, TZ>(nt, p, grid, s);
}

inline int pick_nt(int64_t R) {
  if (R <= 8) return 1;
  if (R <= 16) return 2;
  if (R <= 32) return 4;
  if (R <= 64) return 8;
  return 16;
}

}  // namespace

int launch_shrink(const ShrinkArgs& p, int dtype, int z_dtype, bool aligned, dim3 grid, cudaStream_t s) {
  const int nt = pick_nt(p.R);
  if (dtype == LORA_BF16) {
    if (z_dtype == LORA_F32) return launch_shrink_t<__nv_bfloat16, float>(aligned, nt, p, grid, s);
    if (z_dtype == LORA_BF16) return launch_shrink_t<__nv_bfloat16, __nv_bfloat16>(aligned, nt, p, grid, s);
  } else if (dtype == LORA_F16) {
    if (z_dtype == LORA_F32) return launch_shrink_t<__half, float>(aligned, nt, p, grid, s);
    if (z_dtype == LORA_F16) return launch_shrink_t<__half, __half>(aligned, nt, p, grid, s);
  }
  return LORA_ERR_DTYPE;
}

// K slice per split: a multiple of 64.
int shrink_kslice(int64_t K, int split_k) {
  const int64_t steps = (K + 63) / 64;
  const int64_t per = (steps + split_k - 1) / split_k;
  return static_cast<int>(std::max<int64_t>(per, 1) * 64);
}

int shrink_pick_split_k_impl(int64_t tiles, int64_t K, int num_sms) {
  const int64_t steps = (K + 63) / 64;
  int64_t sk = (2 * static_cast<int64_t>(num_sms) + tiles - 1) / std::max<int64_t>(tiles, 1);
  sk = std::min<int64_t>(sk, std::max<int64_t>(steps / 4, 1));  // >= 256 of K per split
  sk = std::max<int64_t>(std::min<int64_t>(sk, 64), 1);
  // Fold the split so no slice is empty.
  const int kslice = shrink_kslice(K, static_cast<int>(sk));
  sk = (K + kslice - 1) / kslice;
  return static_cast<int>(std::max<int64_t>(sk, 1));
}

}  // namespace lora

using namespace lora;

namespace {
inline size_t round256(size_t v) { return (v + 255) / 256 * 256; }
}  // namespace

extern "C" size_t lora_shrink_workspace_size(int64_t M, int64_t R, int split_k) {
  if (M <= 0 || R <= 0 || split_k <= 1) return 256;
  const size_t partial = static_cast<size_t>(split_k) * M * R * sizeof(float);
  return kCounterBytes + round256(partial);
}

extern "C" int lora_shrink_pick_split_k(int64_t M, int64_t K, int64_t R) {
  (void)R;
  const int dev = current_device();
  const int sms = dev >= 0 ? device_info(dev).num_sms : 148;
  const int64_t tt = 16 * shrink_wt(M);
  return shrink_pick_split_k_impl((M + tt - 1) / tt, K, sms > 0 ? sms : 148);
}

extern "C" int lora_shrink(const void* x, int64_t ldx, const void* a, int64_t lda, void* z, int64_t ldz, int z_dtype,
                           int64_t z_width, int z_split, int64_t M, int64_t K, int64_t R, float scale, int dtype,
                           int split_k, void* workspace, size_t workspace_bytes, void* stream) {
  if (x == nullptr || a == nullptr || z == nullptr) return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (z_split != 0 && (z_split != 1 || z_dtype == LORA_F32)) return LORA_ERR_ARG;
  if (M < 0 || K < 0 || R < 0 || R > 128 || z_width < R) return LORA_ERR_SHAPE;
  if (M > INT32_MAX || K > INT32_MAX || ldz < z_width * (1 + z_split) || ldx < K || lda < K) return LORA_ERR_SHAPE;
  if (M == 0 || z_width == 0) return LORA_OK;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  const int wt = shrink_wt(M);
  const int64_t tiles = (M + 16 * wt - 1) / (16 * wt);
  if (R == 0 || K == 0) split_k = 1;
  if (split_k <= 0) split_k = shrink_pick_split_k_impl(tiles, K, info.num_sms);
  const int kslice = shrink_kslice(K, split_k);
  split_k = static_cast<int>(std::max<int64_t>((K + kslice - 1) / kslice, 1));

  ShrinkArgs p{};
  p.x = x;
  p.a = a;
  p.z = z;
  p.err = info.err_word;
  p.ldx = ldx;
  p.lda = lda;
  p.ldz = ldz;
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.R = static_cast<int>(R);
  p.z_width = static_cast<int>(z_width);
  p.z_split = z_split;
  p.pr = static_cast<int>(R);
  p.split_k = split_k;
  p.kslice = kslice;
  p.wt = wt;
  p.num_tiles_plain = static_cast<int>(tiles);
  p.scale = scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (split_k > 1) {
    const size_t need = lora_shrink_workspace_size(M, R, split_k);
    if (workspace == nullptr || workspace_bytes < need || !al16(workspace)) return LORA_ERR_WORKSPACE;
    if (tiles > kMaxCounters) return LORA_ERR_SHAPE;
    p.counters = static_cast<int*>(workspace);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  }
  const bool aligned = (K % 8 == 0) && (ldx % 8 == 0) && (lda % 8 == 0) && al16(x) && al16(a);
  const int64_t gx = std::min<int64_t>(tiles, std::max<int64_t>(1, (4 * static_cast<int64_t>(info.num_sms) + split_k - 1) / split_k));
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(split_k));
  return launch_shrink(p, dtype, z_dtype, aligned, grid, s);
}

extern "C" int lora_sgmv_pick_split_k(int64_t T, int64_t K, int64_t r_max) {
  if (T <= 0 || K <= 0 || r_max <= 0) return 1;
  const int dev = current_device();
  const int sms = dev >= 0 ? device_info(dev).num_sms : 148;
  return sgmv_shrink_block_split(T, K, sms > 0 ? sms : 148);
}

extern "C" size_t lora_sgmv_shrink_workspace_size(int64_t T, int64_t S, int64_t z_width, int split_k) {
  if (T <= 0 || z_width <= 0) return 256;
  // the unit-scheduled tensor-core shrink keeps its partials after the
  // counter region; its K split (<= 16, about one unit per SM over the tile
  // capacity) is bounded here without K, by four units per SM
  const int dev = current_device();
  const int sms = dev >= 0 ? device_info(dev).num_sms : 148;
  const int64_t blocks = std::max<int64_t>((T + 63) / 64, 1);
  const int64_t unit_split = std::min<int64_t>(16, (4 * static_cast<int64_t>(sms > 0 ? sms : 148) + blocks - 1) /
                                                       blocks);
  const size_t unit = kCounterBytes + round256(static_cast<size_t>(unit_split) * T * ((z_width + 15) / 16 * 16) * 4);
  if (split_k <= 1) return unit;
  const size_t partial = static_cast<size_t>(split_k) * T * z_width * sizeof(float);
  return std::max(unit, kCounterBytes + round256(partial));
}

namespace {
int sgmv_shrink_impl(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                     const int64_t* offsets, const int64_t* ranks, int64_t n_adapters, const int32_t* tiles,
                     const int64_t* rows, void* z, int64_t ldz, int z_dtype, int64_t z_width, int64_t T, int64_t S,
                     int64_t K, int64_t r_max, float scale, int dtype, int split_k, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (x == nullptr || a_flat == nullptr || offsets == nullptr || ranks == nullptr || tiles == nullptr || z == nullptr)
    return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (T < 0 || K < 0 || r_max < 0 || r_max > 128 || z_width < r_max || n_adapters < 0) return LORA_ERR_SHAPE;
  if (T > INT32_MAX / 2 || K > INT32_MAX || ldz < z_width || ldx < K || lda < K) return LORA_ERR_SHAPE;
  if (T == 0 || z_width == 0) return LORA_OK;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  if (r_max == 0 || K == 0) split_k = 1;
  if (split_k <= 0) split_k = sgmv_shrink_block_split(T, K, info.num_sms);
  const int kslice = shrink_kslice(K, split_k);
  split_k = static_cast<int>(std::max<int64_t>((K + kslice - 1) / kslice, 1));
  if (split_k > 1) {
    const size_t need = lora_sgmv_shrink_workspace_size(T, S, z_width, split_k);
    if (workspace == nullptr || workspace_bytes < need || !al16(workspace)) return LORA_ERR_WORKSPACE;
    if (sgmv_max_tiles(T, S) > kMaxCounters) return LORA_ERR_SHAPE;
  }

  // Tensor cores first: the unit-scheduled kernel (sgmv_unit.cu: (tile, K
  // slice) units over persistent CTAs, split-K through the workspace), else the
  // 128-token block kernel (sgmv_tc.cu, cluster split-K); both need the row
  // count of a_flat and no row indirection.  Then dense 64-token blocks on
  // mma.sync (sgmv_block.cu); the per-tile kernel below covers the layouts
  // none of them takes (unaligned rows, r_max > 128).
  if (rows == nullptr && a_rows > 0 && r_max > 0 && K > 0 && workspace != nullptr &&
      workspace_bytes > kCounterBytes) {
    const int rc = launch_sgmv_shrink_unit(x, ldx, a_flat, lda, a_rows, offsets, ranks, tiles, sgmv_max_tiles(T, S), z,
                                           ldz, z_dtype, z_width, T, K, r_max, scale, dtype,
                                           static_cast<char*>(workspace) + kCounterBytes,
                                           workspace_bytes - kCounterBytes, info.num_sms, info.err_word, stream);
    if (rc != LORA_ERR_UNSUPPORTED) return rc;
  }
  if (rows == nullptr && a_rows > 0 && r_max > 0 && K > 0) {
    const int rc = launch_sgmv_shrink_tc(x, ldx, a_flat, lda, a_rows, offsets, ranks, tiles, z, ldz, z_dtype, z_width,
                                         T, K, r_max, scale, dtype, info.num_sms, info.err_word, stream);
    if (rc != LORA_ERR_UNSUPPORTED) return rc;
  }
  if (r_max > 0 && K > 0) {
    SgmvShrinkBlockArgs bp{};
    bp.x = x;
    bp.a = a_flat;
    bp.z = z;
    bp.offsets = offsets;
    bp.ranks = ranks;
    bp.tiles = tiles;
    bp.rows = rows;
    bp.err = info.err_word;
    bp.ldx = ldx;
    bp.lda = lda;
    bp.ldz = ldz;
    bp.T = static_cast<int>(T);
    bp.K = static_cast<int>(K);
    bp.R = static_cast<int>(r_max);
    bp.z_width = static_cast<int>(z_width);
    bp.z_split = 0;
    // the block path splits K over the CTAs of a cluster (at most 8)
    bp.split_k = std::min(split_k, kSgmvMaxClusterSplit);
    bp.kslice = shrink_kslice(K, bp.split_k);
    bp.split_k = static_cast<int>(std::max<int64_t>((K + bp.kslice - 1) / bp.kslice, 1));
    bp.scale = scale;
    const int rc = launch_sgmv_shrink_block(bp, dtype, z_dtype, info.num_sms, stream);
    if (rc != LORA_ERR_UNSUPPORTED) return rc;
  }

  ShrinkArgs p{};
  p.x = x;
  p.a = a_flat;
  p.z = z;
  p.offsets = offsets;
  p.ranks = ranks;
  p.tiles = tiles;
  p.rows = rows;
  p.err = info.err_word;
  p.ldx = ldx;
  p.lda = lda;
  p.ldz = ldz;
  p.M = static_cast<int>(T);
  p.K = static_cast<int>(K);
  p.R = static_cast<int>(r_max);
  p.z_width = static_cast<int>(z_width);
  p.pr = static_cast<int>(z_width);
  p.n_adapters = static_cast<int>(std::min<int64_t>(n_adapters, INT32_MAX));
  p.split_k = split_k;
  p.kslice = kslice;
  p.wt = 4;
  p.scale = scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (split_k > 1) {
    p.counters = static_cast<int*>(workspace);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  }
  const bool aligned = (K % 8 == 0) && (ldx % 8 == 0) && (lda % 8 == 0) && al16(x) && al16(a_flat);
  const int64_t max_tiles = sgmv_max_tiles(T, S);
  const int64_t gx = std::min<int64_t>(
      max_tiles, std::max<int64_t>(1, (4 * static_cast<int64_t>(info.num_sms) + split_k - 1) / split_k));
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(split_k));
  return launch_shrink(p, dtype, z_dtype, aligned, grid, s);
}
}  // namespace

extern "C" int lora_sgmv_shrink(const void* x, int64_t ldx, const void* a_flat, int64_t lda, const int64_t* offsets,
                                const int64_t* ranks, int64_t n_adapters, const int32_t* tiles, const int64_t* rows,
                                void* z, int64_t ldz, int z_dtype, int64_t z_width, int64_t T, int64_t S, int64_t K,
                                int64_t r_max, float scale, int dtype, int split_k, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return sgmv_shrink_impl(x, ldx, a_flat, lda, 0, offsets, ranks, n_adapters, tiles, rows, z, ldz, z_dtype, z_width, T,
                          S, K, r_max, scale, dtype, split_k, workspace, workspace_bytes, stream);
}

extern "C" int lora_sgmv_shrink_ex(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                                   const int64_t* offsets, const int64_t* ranks, int64_t n_adapters,
                                   const int32_t* tiles, const int64_t* rows, void* z, int64_t ldz, int z_dtype,
                                   int64_t z_width, int64_t T, int64_t S, int64_t K, int64_t r_max, float scale,
                                   int dtype, int split_k, void* workspace, size_t workspace_bytes, void* stream) {
  if (a_rows < 0) return LORA_ERR_SHAPE;
  return sgmv_shrink_impl(x, ldx, a_flat, lda, a_rows, offsets, ranks, n_adapters, tiles, rows, z, ldz, z_dtype,
                          z_width, T, S, K, r_max, scale, dtype, split_k, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// Split-K shrink with library-held scratch.
//
// Some callers cannot call cudaMalloc: serving loops that cannot afford
// cudaMalloc's implicit device synchronisation, and host frameworks that own
// all device memory and forbid plugins from allocating.  lora_shrink_static_scratch takes no
// workspace: its ticket counters and fp32 partials live in the file-scope
// array below, which every GPU that loads this library holds until exit.
// Every call shares that array, so calls that overlap on the GPU (concurrent
// streams, several host threads) race; serialise them on one stream.
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;   // 8 MiB in total
constexpr size_t kStaticCounterBytes = size_t(16) << 10;  // 4096 ticket counters
constexpr size_t kStaticPartialBytes = kStaticScratchBytes - kStaticCounterBytes;

static __device__ __align__(256) unsigned char g_shrink_scratch[kStaticScratchBytes];

// Device address of g_shrink_scratch per device ordinal, looked up with that
// device current (in host code the array's name is only a stand-in).  Only a
// successful lookup is cached; a failed one is retried by the next call.
constexpr int kStaticMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_addr[kStaticMaxDevices];

int static_scratch(int dev, void** addr) {
  if (dev < 0 || dev >= kStaticMaxDevices) return LORA_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_shrink_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();  // leave no sticky status behind for the caller
      return LORA_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  return LORA_OK;
}

}  // namespace

extern "C" size_t lora_shrink_static_scratch_capacity(void) { return kStaticPartialBytes; }

extern "C" int lora_shrink_static_scratch(const void* x, int64_t ldx, const void* a, int64_t lda, void* z,
                                          int64_t ldz, int z_dtype, int64_t z_width, int z_split, int64_t M,
                                          int64_t K, int64_t R, float scale, int dtype, int split_k,
                                          void* stream) {
  if (x == nullptr || a == nullptr || z == nullptr) return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (z_split != 0 && (z_split != 1 || z_dtype == LORA_F32)) return LORA_ERR_ARG;
  if (M < 0 || K < 0 || R < 0 || R > 128 || z_width < R || split_k < 0) return LORA_ERR_SHAPE;
  if (M > INT32_MAX || K > INT32_MAX || ldz < z_width * (1 + z_split) || ldx < K || lda < K) return LORA_ERR_SHAPE;
  if (M == 0 || z_width == 0) return LORA_OK;
  // device_info() is not used here: it allocates the library's error word.
  const int dev = current_device();
  if (dev < 0) return LORA_ERR_DEVICE;
  int major = 0, minor = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return LORA_ERR_DEVICE;
  if (major != 10 || minor != 0) return LORA_ERR_DEVICE;

  const int wt = shrink_wt(M);
  const int64_t tiles = (M + 16 * wt - 1) / (16 * wt);
  const bool explicit_split = split_k > 0;
  if (R == 0 || K == 0) split_k = 1;
  if (split_k <= 0) split_k = shrink_pick_split_k_impl(tiles, K, sms > 0 ? sms : 148);
  auto fits = [&](int sk) {
    return sk == 1 || (static_cast<size_t>(sk) * M * R * sizeof(float) <= kStaticPartialBytes &&
                       tiles <= static_cast<int64_t>(kStaticCounterBytes / sizeof(int)));
  };
  if (!explicit_split)
    while (split_k > 1 && !fits(split_k)) --split_k;
  const int kslice = shrink_kslice(K, split_k);
  split_k = static_cast<int>(std::max<int64_t>((K + kslice - 1) / kslice, 1));
  if (!fits(split_k)) return LORA_ERR_WORKSPACE;  // would need more than the 8 MiB array holds

  ShrinkArgs p{};
  p.x = x;
  p.a = a;
  p.z = z;
  p.err = nullptr;
  p.ldx = ldx;
  p.lda = lda;
  p.ldz = ldz;
  p.M = static_cast<int>(M);
  p.K = static_cast<int>(K);
  p.R = static_cast<int>(R);
  p.z_width = static_cast<int>(z_width);
  p.z_split = z_split;
  p.pr = static_cast<int>(R);
  p.split_k = split_k;
  p.kslice = kslice;
  p.wt = wt;
  p.num_tiles_plain = static_cast<int>(tiles);
  p.scale = scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (split_k > 1) {
    void* scratch = nullptr;  // looked up only when the partials need it
    if (const int rc = static_scratch(dev, &scratch); rc != LORA_OK) return rc;
    p.counters = static_cast<int*>(scratch);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(scratch) + kStaticCounterBytes);
    // The tickets must start at zero; the array keeps whatever the last call left.
    if (cudaMemsetAsync(scratch, 0, static_cast<size_t>(tiles) * sizeof(int), s) != cudaSuccess)
      return LORA_ERR_CUDA;
  }
  const bool aligned = (K % 8 == 0) && (ldx % 8 == 0) && (lda % 8 == 0) && al16(x) && al16(a);
  const int64_t gx =
      std::min<int64_t>(tiles, std::max<int64_t>(1, (4 * static_cast<int64_t>(sms) + split_k - 1) / split_k));
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(split_k));
  return launch_shrink(p, dtype, z_dtype, aligned, grid, s);
}

extern "C" size_t lora_sgmv_branch_workspace_size(int64_t T, int64_t S, int64_t K, int64_t r_max) {
  if (T <= 0 || K <= 0 || r_max <= 0) return 256;
  const int dev = current_device();
  const int sms = dev >= 0 ? device_info(dev).num_sms : 148;
  return sgmv_unit_branch_workspace(T, K, r_max, sgmv_max_tiles(T, S), sms > 0 ? sms : 148);
}

extern "C" int lora_sgmv_branch(const void* x, int64_t ldx, const void* y, int64_t ldy, const void* a_flat,
                                int64_t lda, int64_t a_rows, const void* b_flat, int64_t ldb, int64_t b_rows,
                                const int64_t* offsets, const int64_t* ranks, int64_t n_adapters,
                                const int32_t* tiles, void* out, int64_t ldo, int64_t T, int64_t S, int64_t K,
                                int64_t N, int64_t r_max, float scale, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (x == nullptr || a_flat == nullptr || b_flat == nullptr || offsets == nullptr || ranks == nullptr ||
      tiles == nullptr || out == nullptr)
    return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (T < 0 || S < 0 || K < 0 || N < 0 || r_max < 0 || n_adapters < 0 || a_rows < 0 || b_rows < 0)
    return LORA_ERR_SHAPE;
  if (ldx < K || lda < K || ldb < N || ldo < N || (y != nullptr && ldy < N)) return LORA_ERR_SHAPE;
  if (y != nullptr && y == out) return LORA_ERR_ARG;
  if (T == 0 || N == 0) return LORA_OK;
  if (r_max == 0 || K == 0) return LORA_ERR_UNSUPPORTED;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  return launch_sgmv_branch_unit(x, ldx, y, ldy, a_flat, lda, a_rows, b_flat, ldb, b_rows, offsets, ranks, tiles,
                                 sgmv_max_tiles(T, S), out, ldo, T, K, N, r_max, scale, dtype, workspace,
                                 workspace_bytes, info.num_sms, info.err_word, stream);
}

extern "C" size_t lora_sgmv_linear_workspace_size(int64_t T, int64_t S, int64_t K, int64_t r_max) {
  if (T <= 0 || K <= 0 || r_max <= 0) return 256;
  const int dev = current_device();
  const int sms = dev >= 0 ? device_info(dev).num_sms : 148;
  return sgmv_linear_workspace(T, S, K, r_max, sms > 0 ? sms : 148);
}

extern "C" int lora_sgmv_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                                const void* a_flat, int64_t lda, int64_t a_rows, const void* b_flat, int64_t ldb,
                                int64_t b_rows, const int64_t* offsets, const int64_t* ranks, int64_t n_adapters,
                                const int32_t* tiles, void* out, int64_t ldo, int64_t T, int64_t S, int64_t K,
                                int64_t N, int64_t r_max, float scale, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (x == nullptr || w == nullptr || a_flat == nullptr || b_flat == nullptr || offsets == nullptr ||
      ranks == nullptr || tiles == nullptr || out == nullptr)
    return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (T < 0 || S < 0 || K < 0 || N < 0 || r_max < 0 || n_adapters < 0 || a_rows < 0 || b_rows < 0)
    return LORA_ERR_SHAPE;
  if (ldx < K || ldw < K || lda < K || ldb < N || ldo < N) return LORA_ERR_SHAPE;
  if (out == x || out == w) return LORA_ERR_ARG;
  if (T == 0 || N == 0) return LORA_OK;
  if (r_max == 0 || K == 0) return LORA_ERR_UNSUPPORTED;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  return launch_sgmv_linear(x, ldx, w, ldw, bias, a_flat, lda, a_rows, b_flat, ldb, b_rows, offsets, ranks, tiles, S,
                            out, ldo, T, K, N, r_max, scale, dtype, workspace, workspace_bytes, info.num_sms,
                            info.err_word, stream);
}
