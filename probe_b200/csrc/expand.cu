// Expand + add   out = y + scale * z . B^T (+ bias)   -- the output-sized,
// memory-bound half of LoRA.
//
// One kernel serves lora_expand_add (one adapter, every token) and
// lora_sgmv_expand (per-tile adapter from the device schedule).  A CTA owns a
// tile of <= 64 tokens x 128 output columns:
//   1. z[tile, :R] is staged in shared memory in the input dtype.  An fp32 z
//      (R <= 128) is staged as a hi/lo pair [round(z) | z - round(z)] and B
//      twice, so the 16-bit tensor-core product keeps ~16 mantissa bits of z
//      (the reference rounds z to the input dtype, tl.dot(z.to(b.dtype), b));
//   2. B[:R, n-chunk] is staged as [n][j] rows (from the PEFT [N,R] layout or
//      the rank-major flat table [sum R, N]) and re-staged only when the
//      adapter changes;
//   3. mma.sync m16n8k16 forms the 64x128 fp32 product;
//   4. the product goes through shared memory so that y is read and out is
//      written with coalesced 16-byte accesses.
// Reference semantics: _expand_add_kernel (fused_linear.py:112-200),
// _persistent_expand_add_kernel (splitk_lora.py:66-153), _bucket_expand_kernel
// (multilora.py:295-347), segmented_branch.py:31-47, ragged_branch.py:18-27.
#include <algorithm>

#include "common.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

constexpr int kExpTT = 64;   // tokens per tile
constexpr int kExpBN = 128;  // output columns per tile

struct ExpandArgs {
  const void* y;
  const void* z;
  const void* b;
  const void* bias;
  void* out;
  const int64_t* offsets;  // SGMV only
  const int64_t* ranks;    // SGMV only
  const int32_t* tiles;    // SGMV only (NULL = one adapter for all tokens)
  const int64_t* rows;     // SGMV only: logical token -> physical row (NULL = identity)
  int* err;
  int64_t ldy, ldz, ldo;
  int64_t b_sj, b_sn;      // B element (j, n) at b[base + j*b_sj + n*b_sn]
  int M, N, R, rp;         // rp = R rounded up to 16 (shared-memory width)
  int num_tiles_plain;
  float scale;
};

template <typename TZ>
__host__ __device__ inline bool expand_splits(int rp) {
  return sizeof(TZ) == 4 && rp <= 128;
}

template <typename T, typename TZ>
__global__ void __launch_bounds__(128) expand_kernel(const ExpandArgs p) {
  extern __shared__ uint8_t smem_raw[];
  const bool split = expand_splits<TZ>(p.rp);
  const int rs = (split ? 2 : 1) * p.rp + 8;  // padded row stride (elements) -> conflict-free fragments
  T* zs = reinterpret_cast<T*>(smem_raw);
  T* bs = zs + kExpTT * rs;
  float* cs = reinterpret_cast<float*>(bs + kExpBN * rs);
  constexpr int cstride = kExpBN + 8;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int n0 = blockIdx.y * kExpBN;
  const T* y = static_cast<const T*>(p.y);
  const TZ* z = static_cast<const TZ*>(p.z);
  const T* b = static_cast<const T*>(p.b);
  const T* bias = static_cast<const T*>(p.bias);
  T* out = static_cast<T*>(p.out);
  const bool vec = (p.ldo % 8 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                   (y == nullptr || ((p.ldy % 8 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0)));

  int staged_adapter = -2;
  const int num_tiles = p.tiles ? sgmv_num_tiles(p.tiles) : p.num_tiles_plain;
  for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
    int t0, t1, adapter, R;
    int64_t bbase = 0;
    if (p.tiles) {
      t0 = sgmv_tile_start(p.tiles, tile);
      t1 = sgmv_tile_start(p.tiles, tile + 1);
      adapter = sgmv_tile_adapter(p.tiles, tile);
      R = adapter >= 0 ? static_cast<int>(p.ranks[adapter] < p.R ? p.ranks[adapter] : p.R) : 0;
      if (adapter >= 0) bbase = p.offsets[adapter] * static_cast<int64_t>(p.N);
    } else {
      t0 = tile * kExpTT;
      t1 = min(p.M, t0 + kExpTT);
      adapter = 0;
      R = p.R;
    }
    const int ntok = t1 - t0;
    const int r16 = (R + 15) & ~15;

    if (R > 0) {
      // ---- stage B[:, n0:n0+128] as bs[n][j] (j < r16, zero beyond R / N)
      if (adapter != staged_adapter) {
        for (int idx = threadIdx.x; idx < kExpBN * r16; idx += blockDim.x) {
          int nn, j;
          if (p.b_sn == 1) {  // rank-major: consecutive threads walk n
            j = idx / kExpBN;
            nn = idx - j * kExpBN;
          } else {  // PEFT: consecutive threads walk j
            nn = idx / r16;
            j = idx - nn * r16;
          }
          const int n = n0 + nn;
          T v = from_f32<T>(0.f);
          if (j < R && n < p.N) v = b[bbase + static_cast<int64_t>(j) * p.b_sj + static_cast<int64_t>(n) * p.b_sn];
          bs[nn * rs + j] = v;
          if (split) bs[nn * rs + r16 + j] = v;
        }
        staged_adapter = adapter;
      }
      // ---- stage z[t0:t1, :R] as zs[t][j]
      for (int idx = threadIdx.x; idx < kExpTT * r16; idx += blockDim.x) {
        const int t = idx / r16, j = idx - t * r16;
        float v = 0.f;
        if (t < ntok && j < R) {
          const int64_t zr = p.rows ? p.rows[t0 + t] : static_cast<int64_t>(t0 + t);
          v = to_f32(z[zr * p.ldz + j]);
        }
        const T hi = from_f32<T>(v);
        zs[t * rs + j] = hi;
        if (split) zs[t * rs + r16 + j] = from_f32<T>(v - to_f32(hi));
      }
      __syncthreads();
      const int kk = split ? 2 * r16 : r16;

      // ---- 16 tokens x 128 columns per warp
      float acc[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      const T* za = zs + (warp * 16 + g) * rs + 2 * q;
      for (int k = 0; k < kk; k += 16) {
        uint32_t af[4];
        af[0] = *reinterpret_cast<const uint32_t*>(za + k);
        af[1] = *reinterpret_cast<const uint32_t*>(za + 8 * rs + k);
        af[2] = *reinterpret_cast<const uint32_t*>(za + k + 8);
        af[3] = *reinterpret_cast<const uint32_t*>(za + 8 * rs + k + 8);
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          const T* bb = bs + (nt * 8 + g) * rs + k + 2 * q;
          uint32_t bf[2];
          bf[0] = *reinterpret_cast<const uint32_t*>(bb);
          bf[1] = *reinterpret_cast<const uint32_t*>(bb + 8);
          mma16816<T>(acc[nt], af, bf);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        float* c0 = cs + (warp * 16 + g) * cstride + nt * 8 + 2 * q;
        *reinterpret_cast<float2*>(c0) = make_float2(acc[nt][0], acc[nt][1]);
        *reinterpret_cast<float2*>(c0 + 8 * cstride) = make_float2(acc[nt][2], acc[nt][3]);
      }
      __syncthreads();
    }

    // ---- epilogue: out = y + scale * acc + bias, 8 columns per thread
    for (int idx = threadIdx.x; idx < ntok * (kExpBN / 8); idx += blockDim.x) {
      const int t = idx / (kExpBN / 8);
      const int c8 = (idx - t * (kExpBN / 8)) * 8;
      const int n = n0 + c8;
      if (n >= p.N) continue;
      const int64_t row = p.rows ? p.rows[t0 + t] : static_cast<int64_t>(t0 + t);
      float v[8];
      if (R > 0) {
        const float4 a0 = *reinterpret_cast<const float4*>(cs + t * cstride + c8);
        const float4 a1 = *reinterpret_cast<const float4*>(cs + t * cstride + c8 + 4);
        v[0] = a0.x * p.scale; v[1] = a0.y * p.scale; v[2] = a0.z * p.scale; v[3] = a0.w * p.scale;
        v[4] = a1.x * p.scale; v[5] = a1.y * p.scale; v[6] = a1.z * p.scale; v[7] = a1.w * p.scale;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
      if (vec && n + 8 <= p.N) {
        if (y != nullptr) {
          const uint4 yv = *reinterpret_cast<const uint4*>(y + row * p.ldy + n);
          const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = unpack2<T>(yw[i]);
            v[2 * i] += f.x;
            v[2 * i + 1] += f.y;
          }
        }
        if (bias != nullptr) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] += to_f32(bias[n + i]);
        }
        uint4 o;
        o.x = pack2<T>(v[0], v[1]);
        o.y = pack2<T>(v[2], v[3]);
        o.z = pack2<T>(v[4], v[5]);
        o.w = pack2<T>(v[6], v[7]);
        *reinterpret_cast<uint4*>(out + row * p.ldo + n) = o;
      } else {
        for (int i = 0; i < 8 && n + i < p.N; ++i) {
          float w = v[i];
          if (y != nullptr) w += to_f32(y[row * p.ldy + n + i]);
          if (bias != nullptr) w += to_f32(bias[n + i]);
          out[row * p.ldo + n + i] = from_f32<T>(w);
        }
      }
    }
    __syncthreads();
  }
}

namespace {
inline size_t expand_smem(int rp, bool split) {
  return static_cast<size_t>(kExpTT + kExpBN) * ((split ? 2 : 1) * rp + 8) * 2 +
         static_cast<size_t>(kExpTT) * (kExpBN + 8) * 4;
}

template <typename T, typename TZ>
int launch_expand_t(const ExpandArgs& p, dim3 grid, cudaStream_t s) {
  const size_t smem = expand_smem(p.rp, expand_splits<TZ>(p.rp));
  auto kernel = expand_kernel<T, TZ>;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return LORA_ERR_CUDA;
  }
  kernel<<<grid, 128, smem, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}
}  // namespace

int launch_expand(const ExpandArgs& p, int dtype, int z_dtype, dim3 grid, cudaStream_t s) {
  if (dtype == LORA_BF16) {
    if (z_dtype == LORA_F32) return launch_expand_t<__nv_bfloat16, float>(p, grid, s);
    if (z_dtype == LORA_BF16) return launch_expand_t<__nv_bfloat16, __nv_bfloat16>(p, grid, s);
  } else if (dtype == LORA_F16) {
    if (z_dtype == LORA_F32) return launch_expand_t<__half, float>(p, grid, s);
    if (z_dtype == LORA_F16) return launch_expand_t<__half, __half>(p, grid, s);
  }
  return LORA_ERR_DTYPE;
}

int expand_grid_x(int64_t tiles, int64_t n_chunks, int num_sms) {
  const int64_t want = std::max<int64_t>(1, (8 * static_cast<int64_t>(num_sms) + n_chunks - 1) / n_chunks);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, want)));
}

}  // namespace lora

using namespace lora;

extern "C" int lora_expand_add(const void* y, int64_t ldy, const void* z, int64_t ldz, int z_dtype, const void* b,
                               int64_t ldb, int b_layout, const void* bias, void* out, int64_t ldo, int64_t M,
                               int64_t N, int64_t R, float scale, int dtype, void* stream) {
  if (out == nullptr) return LORA_ERR_ARG;
  if (R > 0 && (z == nullptr || b == nullptr)) return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (M < 0 || N < 0 || R < 0 || R > 256) return LORA_ERR_SHAPE;
  if (M > INT32_MAX || N > INT32_MAX || ldo < N || (y != nullptr && ldy < N) || (R > 0 && ldz < R)) return LORA_ERR_SHAPE;
  if (b_layout != LORA_B_PEFT && b_layout != LORA_B_RANK_MAJOR) return LORA_ERR_ARG;
  if (R > 0 && ((b_layout == LORA_B_PEFT && ldb < R) || (b_layout == LORA_B_RANK_MAJOR && ldb < N))) return LORA_ERR_SHAPE;
  if (y != nullptr && y == out) return LORA_ERR_ARG;
  if (M == 0 || N == 0) return LORA_OK;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  ExpandArgs p{};
  p.y = y;
  p.z = z;
  p.b = b;
  p.bias = bias;
  p.out = out;
  p.err = info.err_word;
  p.ldy = ldy;
  p.ldz = ldz;
  p.ldo = ldo;
  p.b_sj = b_layout == LORA_B_PEFT ? 1 : ldb;
  p.b_sn = b_layout == LORA_B_PEFT ? ldb : 1;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.R = static_cast<int>(R);
  p.rp = static_cast<int>((R + 15) / 16 * 16);
  const int64_t tiles = (M + kExpTT - 1) / kExpTT;
  p.num_tiles_plain = static_cast<int>(tiles);
  p.scale = scale;
  const int64_t nch = (N + kExpBN - 1) / kExpBN;
  if (nch > 65535) return LORA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(expand_grid_x(tiles, nch, info.num_sms)), static_cast<unsigned>(nch));
  return launch_expand(p, dtype, z_dtype, grid, static_cast<cudaStream_t>(stream));
}

extern "C" int lora_sgmv_expand(const void* y, int64_t ldy, const void* z, int64_t ldz, int z_dtype, const void* b,
                                int64_t b_sj, int64_t b_sn, const int64_t* offsets, const int64_t* ranks,
                                int64_t n_adapters, const int32_t* tiles, const int64_t* rows, void* out,
                                int64_t ldo, int64_t T,
                                int64_t S, int64_t N, int64_t r_max, float scale, int dtype, void* stream) {
  if (out == nullptr || tiles == nullptr || offsets == nullptr || ranks == nullptr) return LORA_ERR_ARG;
  if (r_max > 0 && (z == nullptr || b == nullptr)) return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (T < 0 || N < 0 || r_max < 0 || r_max > 256 || n_adapters < 0) return LORA_ERR_SHAPE;
  if (T > INT32_MAX / 2 || N > INT32_MAX || ldo < N || (y != nullptr && ldy < N) || (r_max > 0 && ldz < r_max))
    return LORA_ERR_SHAPE;
  if (b_sj <= 0 || b_sn <= 0) return LORA_ERR_ARG;
  if (y != nullptr && y == out) return LORA_ERR_ARG;
  if (T == 0 || N == 0) return LORA_OK;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  if (b_sn == 1 && r_max > 0) {
    // rank-major B: dense 64-token blocks (sgmv_block.cu)
    SgmvExpandBlockArgs bp{};
    bp.y = y;
    bp.z = z;
    bp.b = b;
    bp.out = out;
    bp.offsets = offsets;
    bp.ranks = ranks;
    bp.tiles = tiles;
    bp.rows = rows;
    bp.err = info.err_word;
    bp.ldy = ldy;
    bp.ldz = ldz;
    bp.ldo = ldo;
    bp.ldb = b_sj;
    bp.T = static_cast<int>(T);
    bp.N = static_cast<int>(N);
    bp.R = static_cast<int>(r_max);
    bp.scale = scale;
    const int rc = launch_sgmv_expand_block(bp, dtype, z_dtype, stream);
    if (rc != LORA_ERR_UNSUPPORTED) return rc;
  }
  ExpandArgs p{};
  p.y = y;
  p.z = z;
  p.b = b;
  p.out = out;
  p.offsets = offsets;
  p.ranks = ranks;
  p.tiles = tiles;
  p.rows = rows;
  p.err = info.err_word;
  p.ldy = ldy;
  p.ldz = ldz;
  p.ldo = ldo;
  p.b_sj = b_sj;
  p.b_sn = b_sn;
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(N);
  p.R = static_cast<int>(r_max);
  p.rp = static_cast<int>((r_max + 15) / 16 * 16);
  p.scale = scale;
  const int64_t nch = (N + kExpBN - 1) / kExpBN;
  if (nch > 65535) return LORA_ERR_SHAPE;
  const int64_t max_tiles = sgmv_max_tiles(T, S);
  dim3 grid(static_cast<unsigned>(expand_grid_x(max_tiles, nch, info.num_sms)), static_cast<unsigned>(nch));
  return launch_expand(p, dtype, z_dtype, grid, static_cast<cudaStream_t>(stream));
}
