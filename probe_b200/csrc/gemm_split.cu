// Split-K CTA-pair LoRA linear for outputs with few 256x256 tiles (128 < M <= 256).
//
//   out[M,N] = x[M,K] . W[N,K]^T + bias[N] + scale * (x . A[R,K]^T) . B[N,R]^T   (R <= 64)
//
// A 256x4096 output (the reference's single fused linear at 256 tokens,
// fused_linear.py:296-317 / :652-677 for a 256-row batch) has only 16 tiles of
// 256x256: a persistent kernel would run 32 of the 148 SMs.  Here each tile is
// a cluster of 2 x S CTAs: a CTA pair (tcgen05 cta_group::2, M = 256 tokens,
// N = 256 output columns) for each of S contiguous K slices.
//
//   warp 0      TMA producer: per k-block this CTA's 128 x-rows, its 128 W-rows
//               and (R > 0) its 16 (32 for R > 32) lora_A rows, 128-byte swizzle
//   warp 1      MMA issuer in the even CTA of each pair: D (256x256, TMEM
//               columns 0..255) and the shrink D2 = x . A^T (256x32 or
//               256x64, columns from 256) from the same x tile; then the
//               expand of this K slice, D += [hi | lo](scale * D2) . [B | B]^T,
//               as two, four or eight more MMAs (the expand is linear, so each slice adds its own
//               part and no shrink partial ever leaves its CTA)
//   warps 2..5  epilogue, one thread per accumulator row; they stage [B | B]
//               in the swizzled operand layout while the mainloop runs
//
// Reduction over the S slices: the output columns of a tile are divided into
// S slices (16-column groups, as evenly as S allows), slice j owned by the
// CTAs of K split j.  Each epilogue thread copies its row of the columns it
// does not own from TMEM into an L2-resident workspace (16-byte stores,
// consecutive rows in consecutive lanes); one cluster barrier (release /
// acquire) orders those writes before each owner bulk-copies its slices back
// into its idle stage buffers (one cp.async.bulk per slice), adds them in
// split order to its own columns, adds the bias and writes bf16/f16 rows.
// The exchange goes through L2 rather than distributed shared memory: the
// SM-to-SM network moved these ~90 KB per CTA several times slower on B200.
// No TMA multicast and no atomics: results are deterministic.
//
// Launched with programmatic stream serialization: every CTA signals its
// dependents at once, and the producer loads the weight tiles (W, lora_A) of
// the first stages before griddepcontrol.wait, so in a chain of linears the
// next launch's prologue and weight prefetch overlap this one's tail.  x and
// every global write (workspace, out) come after the wait: only the weights,
// which no kernel of this library writes, are read early.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "gemm_split.h"
#include "runtime.h"

namespace lora {

namespace {

constexpr int kSpThreads = 192;
constexpr int kSpBK = 64;
// Pipeline depth and shrink width by the fused rank RZ: N of the shrink MMA
// is 32 (16 lora_A rows per CTA of the pair), 64 for ranks above 32, where the
// wider stages and two-atom expand operands leave room for 5 stages.
template <int RZ>
struct SplitCfg {
  static constexpr int kStages = RZ > 32 ? 5 : 6;
  static constexpr int kZN = RZ > 32 ? 64 : 32;
  static constexpr int kAtoms = RZ > 32 ? 2 : 1;  // 64-wide K atoms of [hi | lo] and [B | B]
};

struct SplitArgs {
  void* out;
  const void* bias;
  const void* b;  // lora_B [N, R] (fused form)
  float* ws;      // partial exchange (SplitWs layout)
  int* err;
  int64_t ldo, ldb;
  int M, N, R;
  int num_kb, kb_per;
  int num_n_tiles, num_tiles;
  float scale;
};

template <int S, int RZ>
struct SplitSmem {
  static constexpr int kX = 128 * kSpBK * 2;
  static constexpr int kW = 128 * kSpBK * 2;
  static constexpr int kStages = SplitCfg<RZ>::kStages;
  static constexpr int kA = RZ > 0 ? (SplitCfg<RZ>::kZN / 2) * kSpBK * 2 : 0;
  static constexpr int kStage = kX + kW + kA;  // multiple of 1024 (swizzle atoms stay aligned)
  // K split j owns output columns [col_lo(j), col_lo(j + 1)): the 16 groups of
  // 16 columns divided as evenly as S allows (S = 3: 80, 80, 96 columns).
  static constexpr LORA_DEVINL int col_lo(int j) { return (16 * j / S) * 16; }
  static constexpr int kCols = ((16 + S - 1) / S) * 16;  // widest owned slice
  static constexpr int kMain = kStages * kStage;
  // Expand operands (R > 0), 128 rows x 128 bytes each in the 128-byte swizzle
  // layout: [B | B | 0] for this CTA's 128 output columns after the stage
  // buffers, [hi | lo | 0](scale * z) for its 128 rows in the last 16 KB of the
  // stage buffers (free once the mainloop's MMAs are complete).
  static constexpr int kTile = 128 * 128 * SplitCfg<RZ>::kAtoms;  // atoms 16 KB apart
  static constexpr int kBt = kMain;
  static constexpr int kZt = kMain - kTile;
  static constexpr int kBarOffset = kMain + (RZ > 0 ? kTile : 0);
  static constexpr int kBytes = kBarOffset + 256 + 1024;
  static_assert(kStage % 1024 == 0, "stage buffers must keep 1024-byte alignment");
  static_assert(kBytes <= 227 * 1024, "shared memory budget");
};

// Workspace of one launch, in floats: per tile, pair half and owner split,
// S - 1 partial slices [owned columns / 4][128 rows][4], each slot sized for
// the widest slice.
template <int S>
struct SplitWs {
  static constexpr int64_t kSlice = 128 * SplitSmem<S, 0>::kCols;
  static constexpr int64_t kPerTile = 2LL * S * (S - 1) * kSlice;
  static LORA_DEVINL int64_t slice(int tile, int half, int owner, int slot) {
    return static_cast<int64_t>(tile) * kPerTile + ((static_cast<int64_t>(half) * S + owner) * (S - 1) + slot) * kSlice;
  }
};

template <typename T>
LORA_DEVINL void store_row16(T* out_row, int col0, int N, bool vec_ok, const float* v) {
  if (vec_ok && col0 + 16 <= N) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = pack2<T>(v[2 * i], v[2 * i + 1]);
    uint4* dst = reinterpret_cast<uint4*>(out_row + col0);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (col0 + i < N) out_row[col0 + i] = from_f32<T>(v[i]);
  }
}

// RZ = 0: plain linear; RZ = 16 / 32 / 64: fused shrink of rank <= RZ.
template <int S, int RZ, typename T>
__global__ void __launch_bounds__(kSpThreads, 1)
    gemm_split_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_a, const SplitArgs args) {
  using L = SplitSmem<S, RZ>;
  using W = SplitWs<S>;
  static_assert((S - 1) * W::kSlice * 4 <= L::kZt, "received partials stay clear of the z operand");
  constexpr uint32_t kTmemCols = 512;
  constexpr int kBf = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t kIdesc = umma_idesc_f16(256, 256, kBf);
  constexpr int kSpStages = L::kStages;
  constexpr int kSpZN = SplitCfg<RZ>::kZN;
  constexpr uint32_t kIdescZ = umma_idesc_f16(256, kSpZN, kBf);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + kSpStages;
  uint64_t* acc_full = empty + kSpStages;
  uint64_t* z_ready = acc_full + 1;   // leader: both CTAs' z operands written (4 warps each)
  uint64_t* exp_full = z_ready + 1;   // the expand MMAs are complete
  uint64_t* ws_full = exp_full + 1;   // the other splits' partials, bulk-loaded into the stage buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ws_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t half = rank & 1u;  // 0: the pair's MMA issuer
  const int split = static_cast<int>(rank >> 1);
  const uint32_t leader_rank = rank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(0x3u << (2 * split));
  const int tile = blockIdx.z;
  const int mt = tile / args.num_n_tiles;
  const int nt = tile - mt * args.num_n_tiles;
  const int kb0 = split * args.kb_per;
  const int kb1 = min(args.num_kb, kb0 + args.kb_per);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(z_ready, 8);
    mbar_init(exp_full, 1);
    mbar_init(ws_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    if (RZ > 0) tma_prefetch_desc(&tm_a);
  }
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of every CTA initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  bool have = false;  // epilogue threads: the accumulator (with this slice's expand) is complete
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const int row_a = mt * 256 + static_cast<int>(half) * 128;
      const int row_b = nt * 256 + static_cast<int>(half) * 128;
      // weights of the first stages before the grid dependency resolves, x after it
      const int npre = min(kSpStages, kb1 - kb0);
      for (int i = 0; i < npre; ++i) {
        if (half == 0) mbar_arrive_expect_tx(&full[i], 2 * L::kStage);
        const uint32_t bar = mapa_shared(smem_u32(&full[i]), leader_rank);
        uint8_t* st = smem + i * L::kStage;
        const int kc = (kb0 + i) * kSpBK;
        tma_load_2d_pair(&tm_w, st + L::kX, bar, kc, row_b);
        if (RZ > 0) tma_load_2d_pair(&tm_a, st + L::kX + L::kW, bar, kc, static_cast<int>(half) * (kSpZN / 2));
      }
      pdl_wait();
      for (int i = 0; i < npre; ++i)
        tma_load_2d_pair(&tm_x, smem + i * L::kStage, mapa_shared(smem_u32(&full[i]), leader_rank),
                         (kb0 + i) * kSpBK, row_a);
      stage = npre % kSpStages;
      phase = npre == kSpStages ? 1u : 0u;
      for (int kb = kb0 + npre; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, args.err, kDevErrTimeoutEmpty)) break;
        if (half == 0) mbar_arrive_expect_tx(&full[stage], 2 * L::kStage);
        const uint32_t bar = mapa_shared(smem_u32(&full[stage]), leader_rank);
        uint8_t* st = smem + stage * L::kStage;
        const int kc = kb * kSpBK;
        tma_load_2d_pair(&tm_x, st, bar, kc, row_a);
        tma_load_2d_pair(&tm_w, st + L::kX, bar, kc, row_b);
        if (RZ > 0) tma_load_2d_pair(&tm_a, st + L::kX + L::kW, bar, kc, static_cast<int>(half) * (kSpZN / 2));
        if (++stage == kSpStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (even CTA only)
    if (half == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.err, kDevErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sbase = smem_u32(smem + stage * L::kStage);
        const uint64_t adesc = umma_desc_sw128(sbase);
        const uint64_t bdesc = umma_desc_sw128(sbase + L::kX);
        for (int k = 0; k < 4; ++k)
          tc_mma_f16_pair(tmem_base, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k),
                          kIdesc, (kb > kb0 || k > 0) ? 1u : 0u);
        if (RZ > 0) {
          const uint64_t zdesc = umma_desc_sw128(sbase + L::kX + L::kW);
          for (int k = 0; k < 4; ++k)
            tc_mma_f16_pair(tmem_base + 256, adesc + static_cast<uint64_t>(2 * k),
                            zdesc + static_cast<uint64_t>(2 * k), kIdescZ, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        tc_commit_pair(&empty[stage], pair_mask);
        if (++stage == kSpStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) tc_commit_pair(acc_full, pair_mask);
      if (RZ > 0 && ok && mbar_wait_bounded(z_ready, 0, abort_flag, args.err, kDevErrTimeoutFull)) {
        // this slice's expand: D += [hi | lo](scale * z_s) . [B | B]^T, K = 2 * RZ
        fence_acq_rel_cluster();  // both CTAs' operand writes (released by their arrivals) are visible
        tc_fence_after();
        for (int k = 0; k < 2 * RZ / 16; ++k) {
          const int atom = k >> 2, kk = k & 3;
          const uint64_t adesc = umma_desc_sw128(smem_u32(smem + L::kZt + atom * 16384));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(smem + L::kBt + atom * 16384));
          tc_mma_f16_pair(tmem_base, adesc + static_cast<uint64_t>(2 * kk), bdesc + static_cast<uint64_t>(2 * kk),
                          kIdesc, 1u);
        }
        tc_commit_pair(exp_full, pair_mask);
      }
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int row_local = quad * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    if constexpr (RZ > 0) {
      // [B | B | 0] for this CTA's 128 output columns (one row per thread), in
      // the 128-byte swizzle layout the MMA reads (16-byte chunk c of row r at
      // chunk c ^ (r % 8)), written while the mainloop runs.
      const int r = threadIdx.x - 64;
      const int n = nt * 256 + static_cast<int>(half) * 128 + r;
      const T* brow = static_cast<const T*>(args.b) + static_cast<int64_t>(n < args.N ? n : 0) * args.ldb;
      T vals[RZ];
#pragma unroll
      for (int j = 0; j < RZ; ++j) vals[j] = (n < args.N && j < args.R) ? brow[j] : from_f32<T>(0.f);
#pragma unroll
      for (int c = 0; c < 8 * SplitCfg<RZ>::kAtoms; ++c) {  // 16-byte chunk c: K = 8c .. 8c + 7
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k0 = c * 8 + 2 * e;
          const float lo = k0 < 2 * RZ ? to_f32(vals[k0 % RZ]) : 0.f;
          const float hi = k0 + 1 < 2 * RZ ? to_f32(vals[(k0 + 1) % RZ]) : 0.f;
          w[e] = pack2<T>(lo, hi);
        }
        uint8_t* bt = smem + L::kBt + (c >> 3) * 16384 + r * 128;
        *reinterpret_cast<uint4*>(bt + (((c & 7) ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
    }
    have = mbar_wait_bounded(acc_full, 0, abort_flag, args.err, kDevErrTimeoutAccFull);
    have = __all_sync(0xffffffffu, have);  // tcgen05.ld below is warp-collective
    tc_fence_after();
    if constexpr (RZ > 0) {
      if (have) {
        // [hi | lo | 0](scale * z_s) for this row: the slice's shrink partial,
        // split into two 16-bit parts (about 16 significant bits together).
        float z[RZ];
#pragma unroll
        for (int c = 0; c < RZ; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_lane + static_cast<uint32_t>(256 + c), r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) z[c + i] = __uint_as_float(r[i]) * args.scale;
        }
        float part[2 * RZ];
#pragma unroll
        for (int j = 0; j < RZ; ++j) {
          const float h = to_f32(from_f32<T>(z[j]));
          part[j] = h;
          part[RZ + j] = z[j] - h;
        }
#pragma unroll
        for (int c = 0; c < 8 * SplitCfg<RZ>::kAtoms; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k0 = c * 8 + 2 * e;
            w[e] = pack2<T>(k0 < 2 * RZ ? part[k0] : 0.f, k0 + 1 < 2 * RZ ? part[k0 + 1] : 0.f);
          }
          uint8_t* zt = smem + L::kZt + (c >> 3) * 16384 + row_local * 128;
          *reinterpret_cast<uint4*>(zt + (((c & 7) ^ (row_local & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_release(mapa_shared(smem_u32(z_ready), leader_rank));
        have = mbar_wait_bounded(exp_full, 0, abort_flag, args.err, kDevErrTimeoutAccFull);
        have = __all_sync(0xffffffffu, have);
        tc_fence_after();
      }
    }
    if (have) {
      // Partials of the columns the other splits own, into the workspace.
#pragma unroll 1
      for (int jj = 1; jj < S; ++jj) {
        const int j = (split + jj) % S;
        const int slot = split < j ? split : split - 1;
        float4* dst = reinterpret_cast<float4*>(args.ws + W::slice(tile, half, j, slot)) + row_local;
        const int lo = L::col_lo(j), width = L::col_lo(j + 1) - lo;
#pragma unroll 1
        for (int c = 0; c < width; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_lane + static_cast<uint32_t>(lo + c), r);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 4; ++q)
            __stcg(dst + (c / 4 + q) * 128, make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                        __uint_as_float(r[4 * q + 2]),
                                                        __uint_as_float(r[4 * q + 3])));
        }
      }
      fence_proxy_async_global();  // the owners read these with bulk copies
    }
  }
  // Release / acquire over the cluster: every split's partials are in the
  // workspace before any owner reads them.
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();
  tc_fence_after();

  if (warp >= 2 && have) {
    const int quad = warp & 3;
    const int row_local = quad * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const int own_c0 = L::col_lo(split);
    const int own_w = L::col_lo(split + 1) - own_c0;
    // The other splits' partials of the owned columns, one bulk copy each,
    // into the idle stage buffers.
    float* rd = reinterpret_cast<float*>(smem);
    if (threadIdx.x == 64) {
      fence_proxy_async_global();
      mbar_arrive_expect_tx(ws_full, static_cast<uint32_t>((S - 1) * 128 * own_w * 4));
      for (int slot = 0; slot < S - 1; ++slot)
        bulk_load_g2s(rd + slot * W::kSlice, args.ws + W::slice(tile, half, split, slot),
                      static_cast<uint32_t>(128 * own_w * 4), ws_full);
    }
    const bool got = mbar_wait_bounded(ws_full, 0, abort_flag, args.err, kDevErrTimeoutSplitK);
    // TMEM loads are warp-collective: every lane runs the loop, rows >= M only skip their stores.
    const int row = mt * 256 + static_cast<int>(half) * 128 + row_local;
    T* out_row = static_cast<T*>(args.out) + static_cast<int64_t>(row < args.M ? row : 0) * args.ldo;
    const T* bias = static_cast<const T*>(args.bias);
    const bool vec_ok = (args.ldo % 8) == 0 && (reinterpret_cast<uintptr_t>(args.out) % 16) == 0;
#pragma unroll 1
    for (int c = 0; c < own_w; c += 16) {
      const int col0 = nt * 256 + own_c0 + c;
      if (col0 >= args.N) break;
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_lane + static_cast<uint32_t>(own_c0 + c), r);
      tmem_wait_ld();
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
#pragma unroll 1
      for (int slot = 0; slot < S - 1; ++slot) {
        const float4* src = reinterpret_cast<const float4*>(rd + slot * W::kSlice) + (c / 4) * 128 + row_local;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 p = src[q * 128];
          v[4 * q] += p.x;
          v[4 * q + 1] += p.y;
          v[4 * q + 2] += p.z;
          v[4 * q + 3] += p.w;
        }
      }
      if (bias != nullptr) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (col0 + i < args.N) v[i] += to_f32(bias[col0 + i]);
      }
      if (row < args.M && got) store_row16<T>(out_row, col0, args.N, vec_ok, v);
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // the pair's TMEM is released by both CTAs together
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

bool encode_map(CUtensorMap* map, const void* ptr, int dtype, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                uint32_t box_inner, uint32_t box_outer) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, dtype == LORA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int env_slices() {
  const char* v = std::getenv("LORA_B200_SPLIT_PAIR");
  if (v == nullptr || *v == '\0') return -1;
  return std::atoi(v);
}

template <int S, int RZ, typename T>
cudaLaunchConfig_t make_config(int tiles, cudaStream_t stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, S, static_cast<unsigned>(tiles));
  cfg.blockDim = dim3(kSpThreads);
  cfg.dynamicSmemBytes = SplitSmem<S, RZ>::kBytes;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = S;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Clusters of this instance that can be resident at once (0 if it cannot
// launch), queried once per device.
template <int S, int RZ, typename T>
int resident_clusters(int dev) {
  static std::once_flag once[64];
  static int value[64];
  std::call_once(once[dev & 63], [&] {
    auto kernel = gemm_split_pair_kernel<S, RZ, T>;
    int clusters = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SplitSmem<S, RZ>::kBytes) ==
        cudaSuccess) {
      cudaLaunchAttribute attr[1];
      cudaLaunchConfig_t cfg = make_config<S, RZ, T>(64, nullptr, attr);
      if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) clusters = 0;
    }
    cudaGetLastError();
    value[dev & 63] = clusters;
  });
  return value[dev & 63];
}

template <int RZ>
int resident_for(int S, int dtype, int dev) {
  if (dtype == LORA_BF16) {
    if (S == 4) return resident_clusters<4, RZ, __nv_bfloat16>(dev);
    if (S == 3) return resident_clusters<3, RZ, __nv_bfloat16>(dev);
    if (S == 2) return resident_clusters<2, RZ, __nv_bfloat16>(dev);
    return resident_clusters<1, RZ, __nv_bfloat16>(dev);
  }
  if (S == 4) return resident_clusters<4, RZ, __half>(dev);
  if (S == 3) return resident_clusters<3, RZ, __half>(dev);
  if (S == 2) return resident_clusters<2, RZ, __half>(dev);
  return resident_clusters<1, RZ, __half>(dev);
}

int resident(int S, int rz, int dtype, int dev) {
  if (rz == 0) return resident_for<0>(S, dtype, dev);
  if (rz == 16) return resident_for<16>(S, dtype, dev);
  if (rz == 32) return resident_for<32>(S, dtype, dev);
  return resident_for<64>(S, dtype, dev);
}

// K slices for a launch, or 0 (use another kernel): the most slices (4, 3, 2)
// whose 2 x S CTAs per tile fit the machine with every cluster resident in one
// wave (a second wave costs a whole extra mainloop), each slice keeping at
// least 8 k-blocks.  Wider outputs take one slice (no exchange), in as many
// waves of resident pairs as their tiles need: each wave costs about one
// 256 x 256 tile's mainloop, still well under the W-streaming kernel's time
// at these token counts.  LORA_B200_SPLIT_PAIR=0/1/2/3/4 forces the choice
// (for tuning sweeps).
int plan_slices(int64_t M, int64_t N, int64_t num_kb, int rz, int dtype, int dev, int num_sms) {
  if (M <= 0 || N <= 128 || num_kb <= 0) return 0;
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  if (tiles > 65535) return 0;
  const int forced = env_slices();
  if (forced == 0) return 0;
  if (forced >= 1 && forced <= 4)  // at least S k-blocks per slice, so that no slice is empty
    return (num_kb >= forced * forced && resident(forced, rz, dtype, dev) > 0) ? forced : 0;
  for (int S : {4, 3, 2}) {
    if (tiles * 2 * S > num_sms || num_kb < 8 * S) continue;
    if (tiles > resident(S, rz, dtype, dev)) continue;
    return S;
  }
  return (num_kb >= 8 && resident(1, rz, dtype, dev) > 0) ? 1 : 0;
}

template <int S, int RZ, typename T>
int launch_t(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& ta, const SplitArgs& a, int tiles,
             cudaStream_t stream) {
  auto kernel = gemm_split_pair_kernel<S, RZ, T>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SplitSmem<S, RZ>::kBytes) !=
      cudaSuccess)
    return LORA_ERR_CUDA;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = make_config<S, RZ, T>(tiles, stream, attr);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, tx, tw, ta, a) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

template <int RZ, typename T>
int launch_s(int S, const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& ta, const SplitArgs& a,
             int tiles, cudaStream_t stream) {
  if (S == 4) return launch_t<4, RZ, T>(tx, tw, ta, a, tiles, stream);
  if (S == 3) return launch_t<3, RZ, T>(tx, tw, ta, a, tiles, stream);
  if (S == 2) return launch_t<2, RZ, T>(tx, tw, ta, a, tiles, stream);
  return launch_t<1, RZ, T>(tx, tw, ta, a, tiles, stream);
}

template <int RZ>
int launch_rz(int dtype, int S, const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& ta,
              const SplitArgs& a, int tiles, cudaStream_t stream) {
  if (dtype == LORA_BF16) return launch_s<RZ, __nv_bfloat16>(S, tx, tw, ta, a, tiles, stream);
  return launch_s<RZ, __half>(S, tx, tw, ta, a, tiles, stream);
}

template <int S>
size_t ws_bytes_s(int64_t tiles) {
  return static_cast<size_t>(tiles * SplitWs<S>::kPerTile) * sizeof(float);
}

size_t ws_bytes(int S, int64_t tiles) {
  return S == 4 ? ws_bytes_s<4>(tiles) : (S == 3 ? ws_bytes_s<3>(tiles) : (S == 2 ? ws_bytes_s<2>(tiles) : 0));
}

int rz_for(int64_t R) { return R <= 0 ? 0 : (R <= 16 ? 16 : (R <= 32 ? 32 : 64)); }

}  // namespace

size_t split_pair_workspace_bytes(int64_t M, int64_t N, int64_t R) {
  if (M <= 0 || N <= 0 || R < 0 || R > kSplitMaxRank) return 0;
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  return std::max({ws_bytes(4, tiles), ws_bytes(3, tiles), ws_bytes(2, tiles)});
}

int launch_linear_split(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* a, int64_t lda,
                        const void* b, int64_t ldb, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                        int64_t K, int64_t R, float scale, int dtype, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream) {
  if (R < 0 || R > kSplitMaxRank || workspace == nullptr) return LORA_ERR_UNSUPPORTED;
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || !al16(x) || !al16(w) || !al16(workspace))
    return LORA_ERR_UNSUPPORTED;
  if (R > 0 && (a == nullptr || b == nullptr || lda % 8 != 0 || !al16(a))) return LORA_ERR_UNSUPPORTED;
  const int dev = current_device();
  if (dev < 0) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  const int rz = rz_for(R);
  const int64_t num_kb = (K + kSpBK - 1) / kSpBK;
  const int S = plan_slices(M, N, num_kb, rz, dtype, dev, info.num_sms);
  if (S == 0) return LORA_ERR_UNSUPPORTED;
  const int tiles = static_cast<int>(((M + 255) / 256) * ((N + 255) / 256));
  if (workspace_bytes < ws_bytes(S, tiles)) return LORA_ERR_UNSUPPORTED;
  CUtensorMap tx, tw, ta;
  if (!encode_map(&tx, x, dtype, K, M, ldx, kSpBK, 128)) return LORA_ERR_CUDA;
  if (!encode_map(&tw, w, dtype, K, N, ldw, kSpBK, 128)) return LORA_ERR_CUDA;
  // lora_A [R, K]: RZ / 2 rows per CTA of the pair, rows >= R zero-filled
  if (R > 0) {
    if (!encode_map(&ta, a, dtype, K, R, lda, kSpBK, rz > 32 ? 32 : 16)) return LORA_ERR_CUDA;
  } else {
    ta = tx;
  }
  SplitArgs args{};
  args.out = out;
  args.bias = bias;
  args.b = b;
  args.ws = static_cast<float*>(workspace);
  args.err = info.err_word;
  args.ldo = ldo;
  args.ldb = ldb;
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.R = static_cast<int>(R);
  args.num_kb = static_cast<int>(num_kb);
  args.kb_per = static_cast<int>((num_kb + S - 1) / S);
  args.num_n_tiles = static_cast<int>((N + 255) / 256);
  args.num_tiles = tiles;
  args.scale = scale;
  if (rz == 0) return launch_rz<0>(dtype, S, tx, tw, ta, args, tiles, stream);
  if (rz == 16) return launch_rz<16>(dtype, S, tx, tw, ta, args, tiles, stream);
  if (rz == 32) return launch_rz<32>(dtype, S, tx, tw, ta, args, tiles, stream);
  return launch_rz<64>(dtype, S, tx, tw, ta, args, tiles, stream);
}

}  // namespace lora
