// CTA-pair GEMM building blocks shared by gemm_tc.cu (dense fused LoRA GEMM)
// and sgmv_linear.cu (base GEMM with a per-tile segmented adapter tail).
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"
#include "runtime.h"

namespace lora {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
// CTA-pair GEMM: producer warp, MMA warp, then the epilogue warps (a multiple
// of 4: each TMEM lane quadrant drained by kPairEpiWarps / 4 warps splitting the
// columns).  Eight measured no faster than four on B200 (the epilogue is
// already hidden behind the next tile's mainloop), so four it is.
constexpr int kPairEpiWarps = 4;

struct GemmArgs {
  void* out;
  const void* bias;
  int* err;
  int64_t ldo;
  int64_t lo_offset;  // > 0: also write lo = v - round(v) at column + lo_offset
  int M, N, K, R;
  int num_kb_main, num_kb_tail, tail_last_k16;
  int num_m_tiles, num_n_tiles, num_tiles, group_m;
  int l2_hints;  // bit 0: W / B_dup evict_last; bit 1: x / z evict_first; bit 2: out evict_first
  float alpha;
  // Split tail (CTA-pair kernel): the first full_tiles tiles run whole; each
  // later tile is cut into `split` K ranges, one per pair, whose fp32 partials
  // meet in tail_ws and are summed by the last to finish (ticket per tile half).
  int full_tiles, split;
  float* tail_ws;
  int* tail_tickets;
};

// Work item `item` of the CTA-pair kernel: its tile and K-block range.
LORA_DEVINL void pair_item(int item, const GemmArgs& a, int num_kb, int& tile, int& kb0, int& kb1, int& unit) {
  if (item < a.full_tiles) {
    tile = item;
    kb0 = 0;
    kb1 = num_kb;
    unit = -1;
    return;
  }
  unit = item - a.full_tiles;
  tile = a.full_tiles + unit / a.split;
  const int slice = unit - (unit / a.split) * a.split;
  kb0 = (num_kb * slice) / a.split;
  kb1 = (num_kb * (slice + 1)) / a.split;
}

LORA_DEVINL void gemm_tile_coords(int tile, const GemmArgs& a, int& mt, int& nt) {
  const int group_size = a.group_m * a.num_n_tiles;
  const int group = tile / group_size;
  const int first_m = group * a.group_m;
  const int gm = min(a.num_m_tiles - first_m, a.group_m);
  const int in_group = tile - group * group_size;
  mt = first_m + in_group % gm;
  nt = in_group / gm;
}

template <int STAGES, int NW>
struct PairSmem {
  static constexpr int kABytes = 128 * kGemmBK * 2;
  static constexpr int kBBytes = NW * 128 * kGemmBK * 2;  // NW boxes of 128 W rows
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;
};

template <typename T>
LORA_DEVINL void epilogue_store16(const GemmArgs& args, T* out_row, const T* bias, int row, int col0, bool vec_ok,
                                  const uint32_t* r, uint64_t st_policy) {
  if (row >= args.M || col0 >= args.N) return;
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]) * args.alpha;
  if (bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (col0 + i < args.N) v[i] += to_f32(bias[col0 + i]);
  }
  if (args.lo_offset > 0 && vec_ok && (args.lo_offset % 8) == 0 && col0 + 16 <= args.N) {
    uint32_t hw[8], lw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const T h0 = from_f32<T>(v[2 * i]), h1 = from_f32<T>(v[2 * i + 1]);
      hw[i] = pack2<T>(to_f32(h0), to_f32(h1));
      lw[i] = pack2<T>(v[2 * i] - to_f32(h0), v[2 * i + 1] - to_f32(h1));
    }
    uint4* dh = reinterpret_cast<uint4*>(out_row + col0);
    uint4* dl = reinterpret_cast<uint4*>(out_row + col0 + args.lo_offset);
    dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
  } else if (args.lo_offset > 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (col0 + i < args.N) {
        const T hi = from_f32<T>(v[i]);
        out_row[col0 + i] = hi;
        out_row[col0 + i + args.lo_offset] = from_f32<T>(v[i] - to_f32(hi));
      }
    }
  } else if (vec_ok && col0 + 16 <= args.N) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = pack2<T>(v[2 * i], v[2 * i + 1]);
    uint4* dst = reinterpret_cast<uint4*>(out_row + col0);
    if (args.l2_hints & 4) {
      st_global_v4_hint(dst, make_uint4(w[0], w[1], w[2], w[3]), st_policy);
      st_global_v4_hint(dst + 1, make_uint4(w[4], w[5], w[6], w[7]), st_policy);
    } else {
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (col0 + i < args.N) out_row[col0 + i] = from_f32<T>(v[i]);
  }
}

// Tile width (1: 256 x 256, 2: 256 x 512) the CTA-pair GEMM picks for an
// M x N x K product without a split tail (gemm_tc.cu).
int gemm_pair_width(int64_t M, int64_t N, int64_t K, int num_sms);

// 2-D tiled TMA map (128-byte swizzle) over a row-major [outer, inner] matrix.
inline bool encode_tile_map(CUtensorMap* map, const void* ptr, int dtype, uint64_t inner, uint64_t outer,
                     uint64_t ld_elems, uint32_t box_inner, uint32_t box_outer) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, dtype == LORA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace lora
