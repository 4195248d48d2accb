// Dense fused LoRA GEMM on Blackwell tensor cores.
//
//   out[M,N] = alpha * ( x[M,K] . W[N,K]^T + z[M,R] . Bw[N,R]^T ) + bias[N]
//
// The LoRA expand rides along as an extra K-slice: after the K/64 blocks of
// (x, W) the mainloop continues over ceil(R/64) blocks of (z, Bw) into the
// same TMEM accumulator, so the base output is written exactly once.  This is
// the B200 form of the reference's _kconcat ([x | s.z] @ [W | B]^T,
// fused_linear.py:622-677) without materialising the concatenated operands:
// two TMA descriptor pairs feed one accumulator.
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x64 x-tile + BNx64 W-tile per stage (128B swizzle)
//   warp 1      MMA issuer: tcgen05.mma M=128 N=BN K=16, fp32 accumulator in TMEM
//   warps 2..5  epilogue: tcgen05.ld -> alpha, bias, cast -> 32B stores
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap the
// mainloop of tile i+1.  Tiles are rasterised in GROUP_M bands so the W tiles
// of a band stay L2-resident (the reference's GROUP_M swizzle,
// fused_linear.py:245-254).  No TMA multicast.  Wide outputs use the
// CTA-pair form below (gemm_tc2_kernel); narrow ones (N < 256, e.g. a rank
// shrink) and small problems use this single-CTA kernel.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
// Shared with the segmented linear (sgmv_linear.cu): tile sizes, kernel
// arguments, work-item and tile coordinates, the pair stage layout, the
// epilogue store and the TMA map encoder.
#include "gemm_pair.cuh"
#include "runtime.h"

namespace lora {

template <int BN, int STAGES, typename T>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // barriers + alignment slack
};

template <int BN, int STAGES, typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_b,
                   const GemmArgs args) {
  using L = GemmSmem<BN, STAGES, T>;
  constexpr uint32_t kTmemCols = 2 * BN;  // 128, 256 or 512: a power of two >= 32
  constexpr uint32_t kIdesc = umma_idesc_f16(kGemmBM, BN, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sm_a = smem;
  uint8_t* sm_b = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    if (args.num_kb_tail > 0) {
      tma_prefetch_desc(&tm_z);
      tma_prefetch_desc(&tm_b);
    }
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = args.num_kb_main + args.num_kb_tail;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
        int mt, nt;
        gemm_tile_coords(tile, args, mt, nt);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, args.err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          if (kb < args.num_kb_main) {
            tma_load_2d(&tm_x, sm_a + stage * L::kABytes, &full[stage], kb * kGemmBK, mt * kGemmBM);
            tma_load_2d(&tm_w, sm_b + stage * L::kBBytes, &full[stage], kb * kGemmBK, nt * BN);
          } else {
            const int kt = kb - args.num_kb_main;
            tma_load_2d(&tm_z, sm_a + stage * L::kABytes, &full[stage], kt * kGemmBK, mt * kGemmBM);
            tma_load_2d(&tm_b, sm_b + stage * L::kBBytes, &full[stage], kt * kGemmBK, nt * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1, abort_flag, args.err,
                               kDevErrTimeoutAccEmpty)) {
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sm_a + stage * L::kABytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sm_b + stage * L::kBBytes));
          // The last tail block only holds ceil(R%64 / 16) non-zero K16 steps.
          const int nk = (kb == num_kb - 1 && args.num_kb_tail > 0) ? args.tail_last_k16 : 4;
          for (int k = 0; k < nk; ++k) {
            // +32 bytes per K16 step inside the 128B swizzle atom (>>4 => +2).
            tc_mma_f16(d_tmem, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k),
                       kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) tc_commit(&acc_full[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32) belong to this warp
    const T* bias = static_cast<const T*>(args.bias);
    const bool vec_ok = (args.ldo % 8) == 0 && (reinterpret_cast<uintptr_t>(args.out) % 16) == 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int mt, nt;
      gemm_tile_coords(tile, args, mt, nt);
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, args.err, kDevErrTimeoutAccFull)) break;
      tc_fence_after();
      const int row = mt * kGemmBM + quad * 32 + lane;
      T* out_row = static_cast<T*>(args.out) + static_cast<int64_t>(row) * args.ldo;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_row + c, r);
        tmem_wait_ld();
        const int col0 = nt * BN + c;
        if (row < args.M && col0 < args.N) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]) * args.alpha;
          if (bias != nullptr) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (col0 + i < args.N) v[i] += to_f32(bias[col0 + i]);
          }
          if (args.lo_offset > 0 && vec_ok && (args.lo_offset % 8) == 0 && col0 + 16 <= args.N) {
            // hi/lo pair: out[c] = round(v), out[c + lo_offset] = round(v - round(v))
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
            uint4 w0, w1;
            w0.x = pack2<T>(v[0], v[1]);
            w0.y = pack2<T>(v[2], v[3]);
            w0.z = pack2<T>(v[4], v[5]);
            w0.w = pack2<T>(v[6], v[7]);
            w1.x = pack2<T>(v[8], v[9]);
            w1.y = pack2<T>(v[10], v[11]);
            w1.z = pack2<T>(v[12], v[13]);
            w1.w = pack2<T>(v[14], v[15]);
            uint4* dst = reinterpret_cast<uint4*>(out_row + col0);
            dst[0] = w0;
            dst[1] = w1;
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (col0 + i < args.N) out_row[col0 + i] = from_f32<T>(v[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ----------------------------------------------------------- CTA-pair GEMM
//
// The same fused GEMM on 256x256 tiles shared by a cluster of two CTAs
// (tcgen05 cta_group::2).  Each CTA loads its own 128 rows of x (or z) and
// its own 128 rows of W (or B_dup) per 64-wide K block -- 32 KB per SM per
// block instead of 48 KB for a 128x256 single-CTA tile, with the same MMA work
// per SM -- and the leader's single thread issues M=256 N=256 K=16 MMAs that
// read both CTAs' shared memory and leave each CTA's 128 accumulator rows in
// its own TMEM.  Both CTAs' TMA loads complete on the leader's "full"
// barrier; the leader's commits arrive on the "empty" and "accumulator full"
// barriers of both CTAs; both CTAs' epilogues arrive on the leader's
// "accumulator empty" barrier.  No load uses cluster multicast.
// NW = 1: 256 x 256 tiles, two 256-column accumulators (the epilogue of one
// tile overlaps the mainloop of the next).  NW = 2: 256 x 512 tiles, two
// N = 256 MMAs per k-step sharing the x tile, so each SM takes in 48 KB per
// 64-deep k-block for twice the products of a 32 KB NW = 1 k-block (operand
// ingest per SM, not the tensor pipe, bounds the NW = 1 form on B200).  Both
// accumulator halves belong to the one tile; the epilogue frees them one at a
// time and the next tile's first MMAs into each half wait only for that half.
template <int STAGES, int NW, int EW, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(64 + 32 * EW, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_b,
                    const GemmArgs args) {
  using L = PairSmem<STAGES, NW>;
  constexpr uint32_t kTmemCols = 512;  // two 256-column fp32 accumulators
  constexpr int kTileN = 256 * NW;
  constexpr uint32_t kIdesc = umma_idesc_f16(256, 256, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
  constexpr uint16_t kBoth = 0x3;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sm_a = smem;
  uint8_t* sm_b = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

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
      mbar_init(&acc_empty[a], 2 * EW);  // every epilogue warp of both CTAs of the pair
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    if (args.num_kb_tail > 0) {
      tma_prefetch_desc(&tm_z);
      tma_prefetch_desc(&tm_b);
    }
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = args.num_kb_main + args.num_kb_tail;
  const int num_items = args.full_tiles + (args.num_tiles - args.full_tiles) * args.split;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_keep = l2_policy_evict_last();     // W, B_dup: reused by every M band
      const uint64_t pol_stream = l2_policy_evict_first();  // x, z
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = pair; ok && item < num_items; item += npairs) {
        int tile, kb0, kb1, unit;
        pair_item(item, args, num_kb, tile, kb0, kb1, unit);
        int mt, nt;
        gemm_tile_coords(tile, args, mt, nt);
        const int row_a = mt * 256 + static_cast<int>(rank) * 128;
        const int row_b = nt * kTileN + static_cast<int>(rank) * 128;  // + 256 for the second box
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, args.err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          const bool tail = kb >= args.num_kb_main;
          const CUtensorMap* ma = tail ? &tm_z : &tm_x;
          const CUtensorMap* mb = tail ? &tm_b : &tm_w;
          const int kc = (tail ? kb - args.num_kb_main : kb) * kGemmBK;
          if (args.l2_hints & 2)
            tma_load_2d_pair_hint(ma, sm_a + stage * L::kABytes, bar, kc, row_a, pol_stream);
          else
            tma_load_2d_pair(ma, sm_a + stage * L::kABytes, bar, kc, row_a);
#pragma unroll
          for (int h = 0; h < NW; ++h) {
            uint8_t* dst = sm_b + stage * L::kBBytes + h * (128 * kGemmBK * 2);
            if (args.l2_hints & 1)
              tma_load_2d_pair_hint(mb, dst, bar, kc, row_b + 256 * h, pol_keep);
            else
              tma_load_2d_pair(mb, dst, bar, kc, row_b + 256 * h);
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
        int tile, kb0, kb1, unit;
        pair_item(item, args, num_kb, tile, kb0, kb1, unit);
        // NW = 1: accumulator local & 1, its (local >> 1)-th use; NW = 2: both halves, every tile
        const int acc = NW == 1 ? (local & 1) : 0;
        const uint32_t acc_phase = NW == 1 ? ((local >> 1) & 1) : (local & 1);
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1, abort_flag, args.err, kDevErrTimeoutAccEmpty))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 256);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sm_a + stage * L::kABytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sm_b + stage * L::kBBytes));
          const int nk = (kb == num_kb - 1 && args.num_kb_tail > 0) ? args.tail_last_k16 : 4;
          for (int k = 0; k < nk; ++k)
            tc_mma_f16_pair(d_tmem, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k),
                            kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
          if constexpr (NW == 2) {
            if (kb == kb0) {  // the second half of the accumulator: free once the epilogue has drained it
              if (!mbar_wait_bounded(&acc_empty[1], acc_phase ^ 1, abort_flag, args.err, kDevErrTimeoutAccEmpty)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const uint64_t bdesc1 = umma_desc_sw128(smem_u32(sm_b + stage * L::kBBytes + 128 * kGemmBK * 2));
            for (int k = 0; k < nk; ++k)
              tc_mma_f16_pair(tmem_base + 256, adesc + static_cast<uint64_t>(2 * k),
                              bdesc1 + static_cast<uint64_t>(2 * k), kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
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
    // NW = 2: acc_full[0] per tile; the halves are released through
    // acc_empty[0] and acc_empty[1] as they are drained.  Warps 2 .. EW + 1:
    // lane quadrant warp % 4, columns [kCW * cpart, +kCW) of every 256-column half.
    constexpr int kCW = 256 / (EW / 4);
    const int quad = warp & 3;
    const int cpart = (warp - 2) >> 2;
    const T* bias = static_cast<const T*>(args.bias);
    const bool vec_ok = (args.ldo % 8) == 0 && (reinterpret_cast<uintptr_t>(args.out) % 16) == 0;
    const uint64_t st_policy = l2_policy_evict_first();
    int local = 0;
    for (int item = pair; item < num_items; item += npairs, ++local) {
      int tile, kb0, kb1, unit;
      pair_item(item, args, num_kb, tile, kb0, kb1, unit);
      const int acc = NW == 1 ? (local & 1) : 0;
      const uint32_t acc_phase = NW == 1 ? ((local >> 1) & 1) : (local & 1);
      int mt, nt;
      gemm_tile_coords(tile, args, mt, nt);
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, args.err, kDevErrTimeoutAccFull)) break;
      tc_fence_after();
      const int trow = static_cast<int>(rank) * 128 + quad * 32 + lane;  // row within the tile
      const int row = mt * 256 + trow;
      T* out_row = static_cast<T*>(args.out) + static_cast<int64_t>(row) * args.ldo;
      // split item: this CTA's 128 rows of the partial tile, fp32, kTileN wide
      float* part = unit < 0 ? nullptr
                             : args.tail_ws + (static_cast<int64_t>(unit) * 256 + trow) * kTileN;
#pragma unroll 1
      for (int h = 0; h < NW; ++h) {
        const int half = NW == 1 ? acc : h;  // TMEM accumulator drained in this round
        const uint32_t t_row =
            tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(half * 256);
#pragma unroll 1
        for (int c = kCW * cpart; c < kCW * cpart + kCW; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_row + c, r);
          tmem_wait_ld();
          if (part == nullptr) {
            epilogue_store16<T>(args, out_row, bias, row, nt * kTileN + h * 256 + c, vec_ok, r, st_policy);
          } else {
            float4* dst = reinterpret_cast<float4*>(part + h * 256 + c);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              dst[e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                   __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[half]), 0));
      }
      if (part != nullptr) {
        // The last of the tile's split items to store its partial (per CTA
        // half: ticket (tile, rank)) sums the partials in slice order.
        __threadfence();
        named_bar_sync(1, 32 * EW);
        if (threadIdx.x == 64) {
          int* ticket = args.tail_tickets + (tile - args.full_tiles) * 2 + static_cast<int>(rank);
          const int last = atomicAdd(ticket, 1) == args.split - 1;
          if (last) *ticket = 0;  // every slice has arrived: back to zero for the next call
          *last_flag = last;
        }
        named_bar_sync(1, 32 * EW);
        if (*last_flag) {
          __threadfence();
          const int first_unit = (tile - args.full_tiles) * args.split;
#pragma unroll 1
          for (int cc = 0; cc < NW * kCW; cc += 16) {
            const int c = (cc / kCW) * 256 + kCW * cpart + cc % kCW;  // this warp's columns of each half
            float v[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = 0.f;
            for (int sl = 0; sl < args.split; ++sl) {
              const float4* src = reinterpret_cast<const float4*>(
                  args.tail_ws + (static_cast<int64_t>(first_unit + sl) * 256 + trow) * kTileN + c);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float4 q = __ldcg(src + e);
                v[4 * e] += q.x;
                v[4 * e + 1] += q.y;
                v[4 * e + 2] += q.z;
                v[4 * e + 3] += q.w;
              }
            }
            uint32_t r[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(v[e]);
            epilogue_store16<T>(args, out_row, bias, row, nt * kTileN + c, vec_ok, r, st_policy);
          }
        }
        named_bar_sync(1, 32 * EW);  // last_flag is rewritten by the next split item
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its partner may still touch its shared memory
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------- host
namespace {


template <int BN, int STAGES, typename T>
int launch_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                const void* bw, int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M,
                int64_t N, int64_t K, int64_t R, float alpha, int64_t lo_offset, int dtype, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES, T>;
  const int dev = current_device();
  if (dev < 0) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);

  // The tail maps are exactly R wide: TMA fills the columns of the last
  // 64-wide box beyond R with zeros, so z and bw need no padding.
  CUtensorMap tm_x, tm_w, tm_z, tm_b;
  if (!encode_tile_map(&tm_x, x, dtype, K, M, ldx, kGemmBK, kGemmBM)) return LORA_ERR_CUDA;
  if (!encode_tile_map(&tm_w, w, dtype, K, N, ldw, kGemmBK, BN)) return LORA_ERR_CUDA;
  if (R > 0) {
    if (!encode_tile_map(&tm_z, z, dtype, R, M, ldz, kGemmBK, kGemmBM)) return LORA_ERR_CUDA;
    if (!encode_tile_map(&tm_b, bw, dtype, R, N, ldbw, kGemmBK, BN)) return LORA_ERR_CUDA;
  } else {
    tm_z = tm_x;
    tm_b = tm_w;
  }

  GemmArgs a;
  a.out = out;
  a.bias = bias;
  a.err = info.err_word;
  a.ldo = ldo;
  a.lo_offset = lo_offset;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.R = static_cast<int>(R);
  a.num_kb_main = static_cast<int>((K + kGemmBK - 1) / kGemmBK);
  a.num_kb_tail = static_cast<int>((R + kGemmBK - 1) / kGemmBK);
  const int tail_rem = static_cast<int>(R - static_cast<int64_t>(a.num_kb_tail - 1) * kGemmBK);
  a.tail_last_k16 = a.num_kb_tail > 0 ? (tail_rem + 15) / 16 : 4;
  a.num_m_tiles = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  a.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
  a.num_tiles = a.num_m_tiles * a.num_n_tiles;
  a.group_m = 8;
  a.l2_hints = 0;
  a.full_tiles = a.num_tiles;
  a.split = 1;
  a.tail_ws = nullptr;
  a.tail_tickets = nullptr;
  a.alpha = alpha;

  auto kernel = gemm_tc_kernel<BN, STAGES, T>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
  });
  if (attr_err[dev & 63] != cudaSuccess) return LORA_ERR_CUDA;
  const int grid = static_cast<int>(std::min<int64_t>(a.num_tiles, info.num_sms));
  kernel<<<grid, kGemmThreads, L::kBytes, stream>>>(tm_x, tm_w, tm_z, tm_b, a);
  return cudaGetLastError() == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

template <typename T>
int dispatch_gemm(int bn, const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                  const void* bw, int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                  int64_t K, int64_t R, float alpha, int64_t lo, int dtype, cudaStream_t stream) {
  switch (bn) {
    case 64:
      return launch_gemm<64, 8, T>(x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, R, alpha, lo, dtype,
                                   stream);
    case 128:
      return launch_gemm<128, 6, T>(x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, R, alpha, lo, dtype,
                                    stream);
    default:
      return launch_gemm<256, 4, T>(x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, R, alpha, lo, dtype,
                                    stream);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Tile width: narrow outputs (a rank-r shrink, N <= 128) get the narrowest
// tile that covers them; wide ones use 256 unless that leaves fewer than two
// waves of tiles on the machine.
namespace {

// Tuning knobs read from the environment (defaults are the tuned values).
int env_int(const char* name, int fallback) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == '\0') return fallback;
  const int parsed = std::atoi(v);
  return parsed > 0 || std::strcmp(v, "0") == 0 ? parsed : fallback;
}

// Split tail of the CTA-pair GEMM: with `pairs` resident pairs and `tiles`
// tiles, the last (tiles mod pairs) tiles are cut along K into `split` pieces
// (one per idle pair, each at least 4 k-blocks) when that leaves >= 2 pieces.
struct PairSplit {
  int full_tiles, split;
  size_t ws_bytes;  // workspace: ticket region + fp32 partials
};

// Splits pay only for long K: each piece's partial (256 x tile_n fp32) makes
// a round trip through L2 and the last piece to finish sums them, a cost that
// measured on B200 matched the time saved at K = 5120 and was clearly below it
// at K = 13824 (C5 shard shapes).
constexpr int kSplitMinKb = 128;

PairSplit pair_split_plan(int64_t tiles, int pairs, int num_kb, int tile_n) {
  PairSplit sp{static_cast<int>(tiles), 1, 0};
  if (pairs <= 0 || tiles <= 0 || num_kb < kSplitMinKb) return sp;
  const int64_t rem = tiles % pairs;
  if (rem == 0) return sp;
  int64_t s = pairs / rem;
  s = std::min<int64_t>(s, std::max(num_kb / 4, 1));
  s = std::min<int64_t>(s, 16);
  if (s < 2 || rem * 2 > kMaxCounters) return sp;
  sp.full_tiles = static_cast<int>(tiles - rem);
  sp.split = static_cast<int>(s);
  sp.ws_bytes = kCounterBytes + static_cast<size_t>(rem * s) * 256 * static_cast<size_t>(tile_n) * sizeof(float);
  return sp;
}

// Resident CTA pairs of gemm_tc2_kernel<STAGES, NW, EW> on this device (cached).
template <int STAGES, int NW, int EW, typename T>
int pair_capacity(int dev, const DeviceInfo& info, cudaError_t* attr_status) {
  using L = PairSmem<STAGES, NW>;
  auto kernel = gemm_tc2_kernel<STAGES, NW, EW, T>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  static int max_clusters[64];
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    int clusters = 0;
    if (attr_err[dev & 63] == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * info.num_sms);
      cfg.blockDim = dim3(64 + 32 * EW);
      cfg.dynamicSmemBytes = L::kBytes;
      if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        clusters = info.num_sms / 2;
      }
    }
    max_clusters[dev & 63] = clusters > 0 ? clusters : info.num_sms / 2;
  });
  *attr_status = attr_err[dev & 63];
  return max_clusters[dev & 63];
}

template <int STAGES, int NW, int EW, typename T>
int launch_gemm_pair(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                     const void* bw, int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                     int64_t K, int64_t R, float alpha, int64_t lo_offset, int dtype, void* ws, size_t ws_bytes,
                     cudaStream_t stream) {
  using L = PairSmem<STAGES, NW>;
  const int dev = current_device();
  if (dev < 0) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  CUtensorMap tm_x, tm_w, tm_z, tm_b;
  if (!encode_tile_map(&tm_x, x, dtype, K, M, ldx, kGemmBK, 128)) return LORA_ERR_CUDA;
  if (!encode_tile_map(&tm_w, w, dtype, K, N, ldw, kGemmBK, 128)) return LORA_ERR_CUDA;
  if (R > 0) {
    if (!encode_tile_map(&tm_z, z, dtype, R, M, ldz, kGemmBK, 128)) return LORA_ERR_CUDA;
    if (!encode_tile_map(&tm_b, bw, dtype, R, N, ldbw, kGemmBK, 128)) return LORA_ERR_CUDA;
  } else {
    tm_z = tm_x;
    tm_b = tm_w;
  }
  GemmArgs a;
  a.out = out;
  a.bias = bias;
  a.err = info.err_word;
  a.ldo = ldo;
  a.lo_offset = lo_offset;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.R = static_cast<int>(R);
  a.num_kb_main = static_cast<int>((K + kGemmBK - 1) / kGemmBK);
  a.num_kb_tail = static_cast<int>((R + kGemmBK - 1) / kGemmBK);
  const int tail_rem = static_cast<int>(R - static_cast<int64_t>(a.num_kb_tail - 1) * kGemmBK);
  a.tail_last_k16 = a.num_kb_tail > 0 ? (tail_rem + 15) / 16 : 4;
  a.num_m_tiles = static_cast<int>((M + 255) / 256);
  a.num_n_tiles = static_cast<int>((N + 256 * NW - 1) / (256 * NW));
  a.num_tiles = a.num_m_tiles * a.num_n_tiles;
  a.group_m = env_int("LORA_B200_GROUP_M", 8);
  // W (and B_dup) with L2 evict_last when W is large: it is re-read by every
  // band of M tiles while x streams through once (measured on B200 with the
  // replays of both settings interleaved: 32760 x 5120 -> 13824 4193 -> 3971 us,
  // 13824 -> 5120 3961 -> 3888, 5120 -> 5120 1530 -> 1505; 4096^3 unchanged,
  // 1536 x 1536 1.3 % slower).  LORA_B200_L2_HINTS overrides (1: W evict_last,
  // 2: x evict_first, 4: output stores evict_first).
  const int64_t w_bytes = (N * K + N * R) * 2;
  a.l2_hints = env_int("LORA_B200_L2_HINTS", w_bytes >= (int64_t{48} << 20) ? 1 : 0);
  a.alpha = alpha;

  auto kernel = gemm_tc2_kernel<STAGES, NW, EW, T>;
  cudaError_t attr_status = cudaSuccess;
  const int capacity = pair_capacity<STAGES, NW, EW, T>(dev, info, &attr_status);
  if (attr_status != cudaSuccess) return LORA_ERR_CUDA;
  a.full_tiles = a.num_tiles;
  a.split = 1;
  a.tail_ws = nullptr;
  a.tail_tickets = nullptr;
  if (ws != nullptr && env_int("LORA_B200_SPLIT_TAIL", 1) != 0) {
    const PairSplit sp = pair_split_plan(a.num_tiles, capacity, a.num_kb_main + a.num_kb_tail, 256 * NW);
    if (sp.split > 1 && ws_bytes >= sp.ws_bytes && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0) {
      a.full_tiles = sp.full_tiles;
      a.split = sp.split;
      a.tail_tickets = static_cast<int*>(ws);
      a.tail_ws = reinterpret_cast<float*>(static_cast<char*>(ws) + kCounterBytes);
    }
  }
  const int64_t items = a.full_tiles + static_cast<int64_t>(a.num_tiles - a.full_tiles) * a.split;
  const int pairs = static_cast<int>(std::min<int64_t>(items, capacity));
  kernel<<<2 * pairs, 64 + 32 * EW, L::kBytes, stream>>>(tm_x, tm_w, tm_z, tm_b, a);
  return cudaGetLastError() == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

// 256 x 512 pair tiles (NW = 2): a third less operand ingest per product
// than 256 x 256, at the price of an epilogue that only half overlaps the next
// tile.  Chosen when their waves of pairs, weighted by the tile's doubled work
// and the ~10% faster products, cost less than the 256 x 256 waves (4096^3:
// 2 waves of wide tiles against 4 of narrow ones, 20 % faster; 4095 x 5120^2:
// 3 against 5, narrow 45 % faster).
// LORA_B200_GEMM_WIDE=0 / 1 forces the choice (tuning sweeps).
// Waves of pair tiles, counting a split tail as the fraction of a wave each
// of its pieces takes (plus a little for the partials' round trip).
double pair_waves(int64_t tiles, int pairs, int num_kb, bool can_split) {
  const int64_t full = tiles / pairs, rem = tiles % pairs;
  if (rem == 0) return static_cast<double>(full);
  if (can_split) {
    const PairSplit sp = pair_split_plan(tiles, pairs, num_kb, 256);
    if (sp.split > 1) return static_cast<double>(full) + 1.0 / sp.split + 0.05;
  }
  return static_cast<double>(full + 1);
}

int pair_tile_width(int64_t M, int64_t N, int64_t K, int64_t R, int pairs, bool can_split) {
  static const int force = [] {  // -1: choose, 0 / 1: forced (read once)
    const char* v = std::getenv("LORA_B200_GEMM_WIDE");
    return (v != nullptr && (v[0] == '0' || v[0] == '1')) ? v[0] - '0' : -1;
  }();
  if (force == 0 || N <= 256) return 1;
  if (force == 1) return 2;
  const int64_t mt = (M + 255) / 256;
  const int num_kb = static_cast<int>((K + kGemmBK - 1) / kGemmBK + (R + kGemmBK - 1) / kGemmBK);
  // 256 < N <= 512 (the hi/lo output of a rank-224 shrink): one wide tile
  // covers every column, so x is read once instead of once per 256 columns
  // -- the whole cost of such a narrow, memory-bound product.
  if (N <= 512) return num_kb >= 48 ? 2 : 1;
  const int64_t tiles2 = mt * ((N + 511) / 512);
  // Short K: a 256 x 512 tile's epilogue is no longer hidden behind the next
  // tile's mainloop (measured at K = 1536: 256 x 256 tiles 25 % faster).
  if (num_kb < 48) return 1;
  const double w1 = pair_waves(mt * ((N + 255) / 256), pairs, num_kb, can_split);
  const double w2 = pair_waves(tiles2, pairs, num_kb, can_split);
  return 1.8 * w2 < w1 ? 2 : 1;
}

// Pair tiles when the output is wide and there are enough 256x256 tiles to
// keep every SM pair busy -- or, with a workspace for the split tail, when
// cutting the few tiles there are along K puts at least half the pairs to
// work (a rank-224 shrink of a few thousand tokens: 16 tiles become 64
// pieces instead of 64 single-CTA tiles on 64 SMs).  LORA_B200_GEMM=1sm /
// 2sm forces one or the other.
bool use_pair_tiles(int64_t M, int64_t N, int64_t K, int64_t R, int num_sms, bool can_split) {
  const char* force = std::getenv("LORA_B200_GEMM");
  if (force != nullptr && std::strcmp(force, "1sm") == 0) return false;
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  if (force != nullptr && std::strcmp(force, "2sm") == 0) return N > 128;
  if (N <= 128) return false;
  // Outputs wider than 128 columns (the rank-224 shrink included: one 256-wide
  // pair tile reads x once instead of twice) once the grid fills a wave of pairs.
  const int pairs = num_sms / 2;
  if (tiles >= pairs) return true;
  if (!can_split || env_int("LORA_B200_SPLIT_TAIL", 1) == 0) return false;
  const int num_kb = static_cast<int>((K + kGemmBK - 1) / kGemmBK + (R + kGemmBK - 1) / kGemmBK);
  const PairSplit sp = pair_split_plan(tiles, pairs, num_kb, 256);
  return sp.split > 1 && tiles * sp.split * 2 >= pairs;
}

}  // namespace

int gemm_pair_width(int64_t M, int64_t N, int64_t K, int num_sms) {
  return pair_tile_width(M, N, K, 0, num_sms / 2, false);
}

int gemm_pick_bn(int64_t M, int64_t N, int num_sms) {
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  const int64_t mt = (M + kGemmBM - 1) / kGemmBM;
  const int64_t tiles256 = mt * ((N + 255) / 256);
  if (tiles256 >= 2 * num_sms || N % 256 == 0) return 256;
  return 128;
}

}  // namespace lora

namespace lora {
namespace {

int gemm_impl(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz, const void* bw,
              int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t R,
              float alpha, int64_t lo_offset, int dtype, void* ws, size_t ws_bytes, void* stream) {
  if (x == nullptr || w == nullptr || out == nullptr) return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (M < 0 || N < 0 || K < 0 || R < 0) return LORA_ERR_SHAPE;
  if (M == 0 || N == 0) return LORA_OK;
  if (K == 0 && R == 0) return LORA_ERR_UNSUPPORTED;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || R > INT32_MAX) return LORA_ERR_SHAPE;
  if (ldx < K || ldw < K || ldo < N || lo_offset < 0 || (lo_offset > 0 && (lo_offset < N || ldo < N + lo_offset)))
    return LORA_ERR_SHAPE;
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0) return LORA_ERR_ALIGN;
  if (!aligned16(x) || !aligned16(w)) return LORA_ERR_ALIGN;
  if (K == 0) return LORA_ERR_UNSUPPORTED;
  if (R > 0) {
    if (z == nullptr || bw == nullptr) return LORA_ERR_ARG;
    if (ldz < R || ldbw < R) return LORA_ERR_SHAPE;
    if (ldz % 8 != 0 || ldbw % 8 != 0 || !aligned16(z) || !aligned16(bw)) return LORA_ERR_ALIGN;
  }
  const int dev = current_device();
  if (dev < 0) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  if (!info.is_sm100) return LORA_ERR_DEVICE;
  const int bn = gemm_pick_bn(M, N, info.num_sms);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (use_pair_tiles(M, N, K, R, info.num_sms, ws != nullptr)) {
    const int nw = pair_tile_width(M, N, K, R, info.num_sms / 2, ws != nullptr);
#define LORA_PAIR(ST, NWV)                                                                                        \
  (dtype == LORA_BF16                                                                                              \
       ? launch_gemm_pair<ST, NWV, kPairEpiWarps, __nv_bfloat16>(x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, \
                                                                 N, K, R, alpha, lo_offset, dtype, ws, ws_bytes, s)   \
       : launch_gemm_pair<ST, NWV, kPairEpiWarps, __half>(x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, \
                                                          R, alpha, lo_offset, dtype, ws, ws_bytes, s))
    return nw == 2 ? LORA_PAIR(4, 2) : LORA_PAIR(6, 1);
#undef LORA_PAIR
  }
  if (dtype == LORA_BF16)
    return dispatch_gemm<__nv_bfloat16>(bn, x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, R, alpha,
                                        lo_offset, dtype, s);
  return dispatch_gemm<__half>(bn, x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, R, alpha, lo_offset,
                               dtype, s);
}

}  // namespace
}  // namespace lora

extern "C" int lora_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                         const void* bw, int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M,
                         int64_t N, int64_t K, int64_t R, float alpha, int64_t lo_offset, int dtype, void* stream) {
  return lora::gemm_impl(x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, R, alpha, lo_offset, dtype,
                         nullptr, 0, stream);
}

extern "C" size_t lora_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t R) {
  using namespace lora;
  if (M <= 0 || N <= 0 || K <= 0 || R < 0 || M > INT32_MAX || N > INT32_MAX) return 0;
  const int dev = current_device();
  if (dev < 0) return 0;
  const DeviceInfo& info = device_info(dev);
  if (!info.is_sm100 || !use_pair_tiles(M, N, K, R, info.num_sms, true)) return 0;
  const int nw = pair_tile_width(M, N, K, R, info.num_sms / 2, true);
  cudaError_t st = cudaSuccess;
  const int capacity = nw == 2 ? pair_capacity<4, 2, kPairEpiWarps, __nv_bfloat16>(dev, info, &st)
                               : pair_capacity<6, 1, kPairEpiWarps, __nv_bfloat16>(dev, info, &st);
  if (st != cudaSuccess) return 0;
  const int64_t tiles = ((M + 255) / 256) * ((N + 256 * nw - 1) / (256 * nw));
  const int num_kb = static_cast<int>((K + kGemmBK - 1) / kGemmBK + (R + kGemmBK - 1) / kGemmBK);
  return pair_split_plan(tiles, capacity, num_kb, 256 * nw).ws_bytes;
}

extern "C" int lora_gemm_ex(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                            const void* bw, int64_t ldbw, const void* bias, void* out, int64_t ldo, int64_t M,
                            int64_t N, int64_t K, int64_t R, float alpha, int64_t lo_offset, int dtype,
                            void* workspace, size_t workspace_bytes, void* stream) {
  return lora::gemm_impl(x, ldx, w, ldw, z, ldz, bw, ldbw, bias, out, ldo, M, N, K, R, alpha, lo_offset, dtype,
                         workspace, workspace_bytes, stream);
}
