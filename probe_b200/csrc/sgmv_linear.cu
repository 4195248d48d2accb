// Segmented multi-adapter LoRA linear in one tcgen05 GEMM.
//
//   out[t, n] = x[t] . W[n]^T + bias[n] + sum_j z[t, j] * B[off_a + j, n],
//   z[t, :r_a] = scale * x[t] . A_a^T,   a = a(t) from the device tile schedule
//
// The base GEMM and the adapter expand share one accumulator: every 256-token
// output tile of the CTA-pair GEMM runs its K/64 base k-blocks and then a
// "tail" of one stage per adapter piece of that tile -- a piece being a run of
// consecutive schedule tiles with one adapter, i.e. the tokens of one segment
// inside the 256-token tile.  A tail stage is a block-diagonal slice of the
// LoRA product: its A operand is a 256-row slot of z that holds the piece's
// tokens' z rows and zeros elsewhere, its B operand the adapter's rows of the
// rank-major B table, loaded by TMA straight from the table as an MN-major
// operand (no gathered copy).  So the branch costs no pass over y or out: the
// base output is written once with the adapters already in it.  This is the
// fused base + multi-adapter kernel the reference's serving path lacks (its
// ragged/segmented branch reads and rewrites the full base output,
// ragged_branch.py:6-40, segmented_branch.py:12-60).
//
// z travels as a bf16 hi/lo pair (hi = round(v), lo = round(v - hi)): a piece
// of rank <= 32 packs both into one 64-column slot (hi in columns 0..31, lo in
// 32..63; two MMA chains over the same B stage), a piece of rank 33..64 takes
// two slots.  Rank-0 pieces and tokens without a valid adapter add nothing.
//
// Launches (programmatic dependent launch between them):
//   1. pieces  (one CTA): per 256-token tile, its pieces -> slot table
//   2. shrink  (sgmv_unit.cu): fp32 partials of z over (tile, K slice) units
//   3. z fill: sums the partials in slice order into the hi/lo slots (zeros
//      outside each piece's rows)
//   4. the pair GEMM below.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "gemm_pair.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

namespace {

constexpr int kSlTile = 256;          // tokens per output tile (a CTA pair's M)
constexpr int kSlSlotCols = 64;       // z columns per slot (one 128-byte swizzle row)
constexpr int kSlStages = 6;
constexpr int kSlThreads = 1024;      // pieces kernel
constexpr int kSlMaxRank = 64;

// Slot record: {first token, end token, first B row, meta};
// meta = k16 steps (1..4) | part << 4, part 0 = hi|lo packed, 1 = hi, 2 = lo.
struct SlArgs {
  const int32_t* mt_first;  // [m_tiles + 1]: first slot of each 256-token tile
  const int4* slots;
};

// ------------------------------------------------------------------ pieces
// Walks the schedule tiles of output tile mt (those of its four 64-token
// blocks) and calls emit(t0, t1, b_row, k16, part) for every slot of its
// pieces, in token order.  Returns the number of slots.
template <typename Emit>
__device__ int tile_slots(const int32_t* tiles, const int64_t* offsets, const int64_t* ranks, int mt, int T, int R,
                          Emit&& emit) {
  const int32_t* first = sgmv_block_first(tiles);
  const int blocks = (T + kSgmvTileTokens - 1) / kSgmvTileTokens;
  const int b0 = mt * (kSlTile / kSgmvTileTokens);
  const int b1 = min(blocks, b0 + kSlTile / kSgmvTileTokens);
  const int i0 = first[b0], i1 = first[b1];
  int count = 0;
  int cur = -1, cur_r = 0, t0 = 0, t1 = 0;
  int64_t cur_row = 0;
  auto flush = [&]() {
    if (cur < 0 || cur_r <= 0) return;
    const int k16 = (cur_r + 15) >> 4;
    if (k16 <= 2) {
      emit(count, t0, t1, cur_row, k16, 0);
      ++count;
    } else {
      emit(count, t0, t1, cur_row, k16, 1);
      emit(count + 1, t0, t1, cur_row, k16, 2);
      count += 2;
    }
  };
  for (int i = i0; i < i1; ++i) {
    const int ad = sgmv_tile_adapter(tiles, i);
    const int ts = sgmv_tile_start(tiles, i);
    const int te = min(sgmv_tile_start(tiles, i + 1), T);
    if (ad == cur && ad >= 0 && ts == t1) {
      t1 = te;
      continue;
    }
    flush();
    cur = ad;
    t0 = ts;
    t1 = te;
    cur_r = 0;
    cur_row = 0;
    if (ad >= 0) {
      const int64_t rr = ranks[ad];
      cur_r = rr <= 0 ? 0 : static_cast<int>(rr < R ? rr : R);
      cur_row = offsets[ad];
    }
  }
  flush();
  return count;
}

__global__ void __launch_bounds__(kSlThreads) sgmv_linear_pieces_kernel(const int32_t* tiles, const int64_t* offsets,
                                                                        const int64_t* ranks, int T, int R,
                                                                        int m_tiles, int cap, int32_t* mt_first,
                                                                        int4* slots, int* err) {
  __shared__ int warp_sums[kSlThreads / 32];
  pdl_wait();  // the schedule launched before writes the tile table
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (m_tiles + kSlThreads - 1) / kSlThreads;  // contiguous tiles per thread
  const int mt0 = min(m_tiles, tid * per), mt1 = min(m_tiles, mt0 + per);
  auto none = [](int, int, int, int64_t, int, int) {};
  int mine = 0;
  for (int mt = mt0; mt < mt1; ++mt) mine += tile_slots(tiles, offsets, ranks, mt, T, R, none);
  // block-wide exclusive scan of the per-thread counts
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  int base = incl - mine + (warp > 0 ? warp_sums[warp - 1] : 0);
  const int total = warp_sums[kSlThreads / 32 - 1];
  if (total > cap) {  // cannot happen (a piece holds >= 1 schedule tile, <= 2 slots each); keep every write in bounds
    if (tid == 0) record_error(err, kDevErrBadIndex);
  }
  for (int mt = mt0; mt < mt1; ++mt) {
    mt_first[mt] = min(base, cap);
    const int b = base;
    const int n = tile_slots(tiles, offsets, ranks, mt, T, R,
                             [&](int k, int t0, int t1, int64_t row, int k16, int part) {
                               if (b + k < cap)
                                 slots[b + k] = make_int4(t0, t1, static_cast<int>(row), k16 | (part << 4));
                             });
    base += n;
  }
  if (tid == 0) mt_first[m_tiles] = min(total, cap);
}

// ------------------------------------------------------------------ z fill
// One thread per (slot, row, 8-column group): the slot's row holds token
// mt * 256 + row; inside the piece it gets the slice-ordered sum of the shrink
// partials (times scale) as hi or lo, elsewhere zeros.
struct FillArgs {
  const float* partial;  // [S][T][RP]
  const int32_t* mt_first;
  const int4* slots;
  void* z;  // [cap * 256][64]
  int T, RP, S, m_tiles, cap;
  float scale;
};

template <typename T>
__global__ void __launch_bounds__(256) sgmv_linear_zfill_kernel(const FillArgs p) {
  pdl_wait();  // partials from the shrink, slots from the pieces kernel before it
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int total = min(p.mt_first[p.m_tiles], p.cap);
  const int64_t work = static_cast<int64_t>(total) * kSlTile * 8;
  const int64_t slice = static_cast<int64_t>(p.T) * p.RP;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < work;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(idx / (kSlTile * 8));
    const int rem = static_cast<int>(idx - static_cast<int64_t>(e) * kSlTile * 8);
    const int row = rem >> 3, c = rem & 7;
    const int4 s = p.slots[e];
    const int part = (s.w >> 4) & 3;
    const int t = (s.x / kSlTile) * kSlTile + row;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    const int zg = part == 0 ? (c & 3) : c;  // z columns 8 zg .. 8 zg + 7
    const bool want_lo = part == 0 ? (c >= 4) : (part == 2);
    if (t >= s.x && t < s.y && t < p.T && zg * 8 < p.RP) {
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const float* src = p.partial + static_cast<int64_t>(t) * p.RP + zg * 8;
      for (int sl = 0; sl < p.S; ++sl) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(src + sl * slice));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(src + sl * slice + 4));
        v[0] += a.x;
        v[1] += a.y;
        v[2] += a.z;
        v[3] += a.w;
        v[4] += b.x;
        v[5] += b.y;
        v[6] += b.z;
        v[7] += b.w;
      }
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = v[2 * k] * p.scale, b = v[2 * k + 1] * p.scale;
        const uint32_t hi = pack2<T>(a, b);
        if (want_lo) {
          const float2 h = unpack2<T>(hi);
          w[k] = pack2<T>(a - h.x, b - h.y);
        } else {
          w[k] = hi;
        }
      }
      o = make_uint4(w[0], w[1], w[2], w[3]);
    }
    T* dst = static_cast<T*>(p.z) + (static_cast<int64_t>(e) * kSlTile + row) * kSlSlotCols + c * 8;
    *reinterpret_cast<uint4*>(dst) = o;
  }
}

// Shared-memory descriptor of an MN-major operand written by TMA as 64-element
// (128-byte) chunks with 128-byte swizzle: K rows 128 B apart, 8-row groups
// 1024 B apart (SBO), 64-wide MN chunks `lbo` bytes apart (LBO).
LORA_DEVINL uint64_t sl_desc_mn(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

struct SlMaps {
  CUtensorMap x, w, z;
  CUtensorMap b[4];  // B table chunk boxes: 16, 32, 48, 64 rows x 2 chunks of 64 columns
};

// Extra shared memory past the last stage: a tail stage's B operand takes at
// most half of a stage's B buffer, so even a reading of twice its extent
// stays inside the allocation.
constexpr int kSlGuardBytes = 16 * 1024;

}  // namespace

// The pair GEMM: 256 x 256 tiles (NW = 1 of gemm_tc2_kernel), base k-blocks
// then the tile's slots.  Roles and barriers as in gemm_tc2_kernel.
template <int STAGES, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    sgmv_linear_pair_kernel(const __grid_constant__ SlMaps maps, const GemmArgs args, const SlArgs sl) {
  using L = PairSmem<STAGES, 1>;
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kIdesc = umma_idesc_f16(256, 256, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
  constexpr uint32_t kIdescMN = kIdesc | (1u << 16);  // B (adapter rows) MN-major
  constexpr uint16_t kBoth = 0x3;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sm_a = smem;
  uint8_t* sm_b = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset + kSlGuardBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // 4 epilogue warps in each CTA of the pair
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.x);
    tma_prefetch_desc(&maps.w);
    tma_prefetch_desc(&maps.z);
    for (int h = 0; h < 4; ++h) tma_prefetch_desc(&maps.b[h]);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_items = args.num_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = pair; ok && item < num_items; item += npairs) {
        int mt, nt;
        gemm_tile_coords(item, args, mt, nt);
        const int e0 = sl.mt_first[mt], e1 = sl.mt_first[mt + 1];
        const int num_kb = args.num_kb_main + (e1 - e0);
        const int row_a = mt * 256 + static_cast<int>(rank) * 128;
        const int row_b = nt * 256 + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, args.err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          uint8_t* da = sm_a + stage * L::kABytes;
          uint8_t* db = sm_b + stage * L::kBBytes;
          if (kb < args.num_kb_main) {
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
            tma_load_2d_pair(&maps.x, da, bar, kb * kGemmBK, row_a);
            tma_load_2d_pair(&maps.w, db, bar, kb * kGemmBK, row_b);
          } else {
            const int e = e0 + kb - args.num_kb_main;
            const int4 s = sl.slots[e];
            const int k16 = s.w & 15;
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (L::kABytes + k16 * 16 * 128 * 2));
            tma_load_2d_pair(&maps.z, da, bar, 0, e * 256 + static_cast<int>(rank) * 128);
            tma_load_3d_pair(&maps.b[k16 - 1], db, bar, 0, s.z, row_b / 64);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (leader CTA only)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int item = pair; ok && item < num_items; item += npairs, ++local) {
        int mt, nt;
        gemm_tile_coords(item, args, mt, nt);
        const int e0 = sl.mt_first[mt], e1 = sl.mt_first[mt + 1];
        const int num_kb = args.num_kb_main + (e1 - e0);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1, abort_flag, args.err, kDevErrTimeoutAccEmpty))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 256);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sm_a + stage * L::kABytes));
          const uint32_t bs = smem_u32(sm_b + stage * L::kBBytes);
          if (kb < args.num_kb_main) {
            const uint64_t bdesc = umma_desc_sw128(bs);
            for (int k = 0; k < 4; ++k)
              tc_mma_f16_pair(d_tmem, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k),
                              kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
          } else {
            const int4 s = sl.slots[e0 + kb - args.num_kb_main];
            const int k16 = s.w & 15, part = (s.w >> 4) & 3;
            const uint32_t lbo = static_cast<uint32_t>(k16 * 16 * 128);  // chunk stride of the B box
            // hi columns at k-step 0.., lo (packed slot) at k-step 2..: same B rows
            for (int h = 0; h < (part == 0 ? 2 : 1); ++h)
              for (int ks = 0; ks < k16; ++ks)
                tc_mma_f16_pair(d_tmem, adesc + static_cast<uint64_t>(2 * (2 * h + ks)),
                                sl_desc_mn(bs + static_cast<uint32_t>(ks * 2048), lbo), kIdescMN, 1u);
          }
          tc_commit_pair(&empty[stage], kBoth);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) tc_commit_pair(&acc_full[acc], kBoth);
      }
    }
  } else {
    // ------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const T* bias = static_cast<const T*>(args.bias);
    const bool vec_ok = (args.ldo % 8) == 0 && (reinterpret_cast<uintptr_t>(args.out) % 16) == 0;
    const uint64_t st_policy = l2_policy_evict_first();
    int local = 0;
    for (int item = pair; item < num_items; item += npairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int mt, nt;
      gemm_tile_coords(item, args, mt, nt);
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, args.err, kDevErrTimeoutAccFull)) break;
      tc_fence_after();
      const int row = mt * 256 + static_cast<int>(rank) * 128 + quad * 32 + lane;
      T* out_row = static_cast<T*>(args.out) + static_cast<int64_t>(row) * args.ldo;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * 256);
#pragma unroll 1
      for (int c = 0; c < 256; c += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_row + c, r);
        tmem_wait_ld();
        epilogue_store16<T>(args, out_row, bias, row, nt * 256 + c, vec_ok, r, st_policy);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
    }
  }

  tc_fence_before();
  cluster_sync_all();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ===================================================================== host
namespace {

struct SlLayout {
  int64_t m_tiles, cap;  // output tiles, slot capacity
  size_t off_part, off_z, off_first, off_slots, bytes;
};

inline size_t round256(size_t v) { return (v + 255) / 256 * 256; }

SlLayout sl_layout(int64_t T, int64_t S, int64_t K, int64_t r_max, int num_sms) {
  SlLayout l{};
  l.m_tiles = (T + kSlTile - 1) / kSlTile;
  l.cap = 2 * sgmv_max_tiles(T, S);  // a piece holds >= 1 schedule tile and takes <= 2 slots
  l.off_part = 0;
  l.off_z = round256(sgmv_unit_shrink_workspace(T, K, r_max, sgmv_max_tiles(T, S), num_sms));
  l.off_first = l.off_z + round256(static_cast<size_t>(l.cap) * kSlTile * kSlSlotCols * 2);
  l.off_slots = l.off_first + round256(static_cast<size_t>(l.m_tiles + 1) * sizeof(int32_t));
  l.bytes = l.off_slots + round256(static_cast<size_t>(l.cap) * sizeof(int4));
  return l;
}

bool sl_chunk_map(CUtensorMap* map, const void* ptr, int dtype, uint64_t rows, uint64_t cols, uint64_t ld,
                  uint32_t box_rows) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr || cols % 64 != 0) return false;
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {ld * 2, 128};
  cuuint32_t box[3] = {64, box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode(map, dtype == LORA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool sl_al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T>
int launch_sl_pair(const SlMaps& maps, const GemmArgs& a, const SlArgs& sl, int pairs_cap, cudaStream_t stream) {
  using L = PairSmem<kSlStages, 1>;
  const size_t smem = L::kBytes + kSlGuardBytes;
  auto kernel = sgmv_linear_pair_kernel<kSlStages, T>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return LORA_ERR_CUDA;
  const int pairs = static_cast<int>(std::min<int64_t>(a.num_tiles, pairs_cap));
  kernel<<<2 * pairs, kGemmThreads, smem, stream>>>(maps, a, sl);
  return cudaGetLastError() == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

}  // namespace

size_t sgmv_linear_workspace(int64_t T, int64_t S, int64_t K, int64_t r_max, int num_sms) {
  return sl_layout(T, S, K, r_max, num_sms).bytes;
}

int launch_sgmv_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias, const void* a_flat,
                       int64_t lda, int64_t a_rows, const void* b_flat, int64_t ldb, int64_t b_rows,
                       const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, int64_t S, void* out,
                       int64_t ldo, int64_t T, int64_t K, int64_t N, int64_t r_max, float scale, int dtype,
                       void* workspace, size_t workspace_bytes, int num_sms, int* err, void* stream) {
  if (r_max <= 0 || r_max > kSlMaxRank || T <= 0 || K <= 0 || N <= 0) return LORA_ERR_UNSUPPORTED;
  if (K % 64 != 0 || N % 64 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0 || ldo % 8 != 0)
    return LORA_ERR_UNSUPPORTED;
  if (!sl_al16(x) || !sl_al16(w) || !sl_al16(a_flat) || !sl_al16(b_flat) || !sl_al16(out))
    return LORA_ERR_UNSUPPORTED;
  if (a_rows <= 0 || a_rows > INT32_MAX || b_rows <= 0 || b_rows > INT32_MAX || T > INT32_MAX / 2 ||
      N > INT32_MAX / 2 || K > INT32_MAX)
    return LORA_ERR_UNSUPPORTED;
  const SlLayout l = sl_layout(T, S, K, r_max, num_sms);
  if (l.cap * kSlTile > INT32_MAX || workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 ||
      workspace_bytes < l.bytes)
    return LORA_ERR_UNSUPPORTED;
  const int dev = current_device();
  if (dev < 0) return LORA_ERR_DEVICE;
  char* ws = static_cast<char*>(workspace);
  float* partial = reinterpret_cast<float*>(ws + l.off_part);
  void* zslots = ws + l.off_z;
  int32_t* mt_first = reinterpret_cast<int32_t*>(ws + l.off_first);
  int4* slots = reinterpret_cast<int4*>(ws + l.off_slots);
  const int64_t max_tiles = sgmv_max_tiles(T, S);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // 1. pieces -> slots
  {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kSlThreads);
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, sgmv_linear_pieces_kernel, tiles, offsets, ranks, static_cast<int>(T),
                           static_cast<int>(r_max), static_cast<int>(l.m_tiles), static_cast<int>(l.cap), mt_first,
                           slots, err) != cudaSuccess)
      return LORA_ERR_CUDA;
  }
  // 2. shrink partials
  const int n_slices = sgmv_unit_slices(T, K, num_sms);
  int rc = launch_sgmv_shrink_partials(x, ldx, a_flat, lda, a_rows, offsets, ranks, tiles, max_tiles, partial, T, K,
                                       r_max, n_slices, dtype, num_sms, err, stream);
  if (rc != LORA_OK) return rc;
  // 3. z slots
  {
    FillArgs f{};
    f.partial = partial;
    f.mt_first = mt_first;
    f.slots = slots;
    f.z = zslots;
    f.T = static_cast<int>(T);
    f.RP = static_cast<int>((r_max + 15) / 16 * 16);
    f.S = n_slices;
    f.m_tiles = static_cast<int>(l.m_tiles);
    f.cap = static_cast<int>(l.cap);
    f.scale = scale;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(static_cast<unsigned>(4 * num_sms));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    const cudaError_t e = dtype == LORA_BF16 ? cudaLaunchKernelEx(&cfg, sgmv_linear_zfill_kernel<__nv_bfloat16>, f)
                                             : cudaLaunchKernelEx(&cfg, sgmv_linear_zfill_kernel<__half>, f);
    if (e != cudaSuccess) return LORA_ERR_CUDA;
  }
  // 4. the pair GEMM
  SlMaps maps;
  if (!encode_tile_map(&maps.x, x, dtype, K, T, ldx, kGemmBK, 128)) return LORA_ERR_CUDA;
  if (!encode_tile_map(&maps.w, w, dtype, K, N, ldw, kGemmBK, 128)) return LORA_ERR_CUDA;
  if (!encode_tile_map(&maps.z, zslots, dtype, kSlSlotCols, static_cast<uint64_t>(l.cap) * kSlTile, kSlSlotCols,
                       kGemmBK, 128))
    return LORA_ERR_CUDA;
  for (int h = 0; h < 4; ++h)
    if (!sl_chunk_map(&maps.b[h], b_flat, dtype, static_cast<uint64_t>(b_rows), static_cast<uint64_t>(N),
                      static_cast<uint64_t>(ldb), static_cast<uint32_t>(16 * (h + 1))))
      return LORA_ERR_CUDA;
  GemmArgs a{};
  a.out = out;
  a.bias = bias;
  a.err = err;
  a.ldo = ldo;
  a.lo_offset = 0;
  a.M = static_cast<int>(T);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.R = 0;
  a.num_kb_main = static_cast<int>(K / kGemmBK);
  a.num_kb_tail = 0;
  a.tail_last_k16 = 4;
  a.num_m_tiles = static_cast<int>(l.m_tiles);
  a.num_n_tiles = static_cast<int>((N + 255) / 256);
  a.num_tiles = a.num_m_tiles * a.num_n_tiles;
  a.group_m = 8;
  a.l2_hints = 0;
  a.alpha = 1.0f;
  a.full_tiles = a.num_tiles;
  a.split = 1;
  a.tail_ws = nullptr;
  a.tail_tickets = nullptr;
  SlArgs sl{mt_first, slots};
  const int pairs_cap = std::max(1, num_sms / 2);
  return dtype == LORA_BF16 ? launch_sl_pair<__nv_bfloat16>(maps, a, sl, pairs_cap, s)
                            : launch_sl_pair<__half>(maps, a, sl, pairs_cap, s);
}

}  // namespace lora
