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
// two slots.  (Rounding z to bf16 alone, as the reference's ragged expand does
// with z.to(b.dtype), ragged_branch.py:24-25, measured up to 0.13 max-abs
// error at rank 64 -- beyond the 2e-2 bar.)  Rank-0 pieces and tokens without
// a valid adapter add nothing.
//
// Launches (programmatic dependent launch between them):
//   1. pieces  (one CTA): per 256-token tile, its pieces -> slot table
//   2. shrink  (sgmv_unit.cu): fp32 partials of z over (tile, K slice) units
//   3. z fill: sums the partials in slice order into the hi/lo slots (zeros
//      outside each piece's rows and beyond its rank)
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
constexpr int kSlStages = 6;       // 256 x 256 tiles (256 x 512: 4 stages)
constexpr int kSlMaxRank = 64;

// Slot record: {first token, end token, first B row, meta};
// meta = k16 steps (1..4) | part << 4, part 0 = hi|lo packed, 1 = hi, 2 = lo.
struct SlArgs {
  const int32_t* mt_first;  // [m_tiles + 1]: first slot of each 256-token tile
  const int4* slots;
};

// ------------------------------------------------------------------ pieces
// One warp per 256-token output tile (warps stride over the tiles).  Lanes
// read 32 schedule tiles at a time in parallel; a piece starts at every
// schedule tile whose adapter differs from the one before it inside the output
// tile, and ends where the next piece starts (pieces cover the output tile,
// those without an adapter or of rank 0 included; those emit no slot).  A
// piece of rank <= 32 takes one slot, a larger one two.  Pass 1 counts each
// output tile's slots into mt_first, a block-wide scan turns the counts into
// first-slot offsets, pass 2 writes the slot records.  Every load of a pass is
// independent of the others, so a pass costs a few memory latencies.
constexpr int kSlPieceThreads = 1024;  // a warp per output tile up to 32 of them (8192 tokens): one walk each
constexpr int kSlPieceWarps = kSlPieceThreads / 32;

struct PieceWalk {
  const int32_t* tiles;
  const int64_t* offsets;
  const int64_t* ranks;
  int T, R;

  // Calls emit(k, t0, t1, b_row, k16, part) for the slots of output tile mt
  // (k = slot index within the tile, in token order) from every lane that owns
  // a slot; returns the tile's slot count (warp-uniform).
  template <typename Emit>
  __device__ int run(int mt, int lane, Emit&& emit) const {
    const int32_t* first = sgmv_block_first(tiles);
    const int blocks = (T + kSgmvTileTokens - 1) / kSgmvTileTokens;
    const int b0 = mt * (kSlTile / kSgmvTileTokens);
    const int b1 = min(blocks, b0 + kSlTile / kSgmvTileTokens);
    const int i0 = first[b0], i1 = first[b1];
    const int tile_end = min(T, (mt + 1) * kSlTile);
    int carry_ad = -2;  // adapter of the last schedule tile of the previous chunk
    int done = 0;       // slots emitted so far
    // a piece that starts in this chunk may end in a later one: its start is
    // kept until the next start (or the tile's end) is seen
    int open_t0 = -1, open_ad = -1;
    for (int c0 = i0; c0 < i1; c0 += 32) {
      const int i = c0 + lane;
      const bool valid = i < i1;
      const int ad = valid ? sgmv_tile_adapter(tiles, i) : -3;
      const int ts = valid ? sgmv_tile_start(tiles, i) : tile_end;
      int prev = __shfl_up_sync(0xffffffffu, ad, 1);
      if (lane == 0) prev = carry_ad;
      const bool starts = valid && (i == i0 || ad != prev);
      const uint32_t mask = __ballot_sync(0xffffffffu, starts);
      // the open piece (from an earlier chunk) ends at this chunk's first start
      if (open_t0 >= 0 && mask != 0u) {
        const int t1 = __shfl_sync(0xffffffffu, ts, __ffs(mask) - 1);
        done += emit_piece(done, open_t0, t1, open_ad, lane, emit);
        open_t0 = -1;
      }
      // pieces starting in this chunk: each ends at the next start in the chunk,
      // the last one stays open
      const uint32_t later = starts ? (mask & ~((2u << lane) - 1u)) : 0u;  // starts after this lane
      const int nxt = later ? __ffs(later) - 1 : -1;
      const int t1_local = __shfl_sync(0xffffffffu, ts, nxt >= 0 ? nxt : 0);
      // closed pieces of this chunk, in lane order
      const bool closes = starts && nxt >= 0;
      const int rr = (closes && ad >= 0) ? piece_rank(ad) : 0;
      const int nslot = rr <= 0 ? 0 : (rr <= 32 ? 1 : 2);
      int excl = nslot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, excl, o);
        if (lane >= o) excl += v;
      }
      const int total_c = __shfl_sync(0xffffffffu, excl, 31);
      excl -= nslot;
      if (nslot > 0) emit_slots(done + excl, ts, t1_local, static_cast<int>(offsets[ad]), rr, emit);
      done += total_c;
      if (mask != 0u) {
        const int last = 31 - __clz(mask);
        open_t0 = __shfl_sync(0xffffffffu, ts, last);
        open_ad = __shfl_sync(0xffffffffu, ad, last);
      }
      carry_ad = __shfl_sync(0xffffffffu, ad, min(31, i1 - 1 - c0));
    }
    if (open_t0 >= 0) done += emit_piece(done, open_t0, tile_end, open_ad, lane, emit);
    return done;
  }

  __device__ int piece_rank(int ad) const {
    const int64_t rr = ranks[ad];
    return rr <= 0 ? 0 : static_cast<int>(rr < R ? rr : R);
  }

  // The slots of one piece of rank rr > 0, from slot index k on.
  template <typename Emit>
  __device__ static void emit_slots(int k, int t0, int t1, int brow, int rr, Emit&& emit) {
    const int k16 = (rr + 15) >> 4;
    if (k16 <= 2) {
      emit(k, t0, t1, brow, k16, 0);
    } else {
      emit(k, t0, t1, brow, k16, 1);
      emit(k + 1, t0, t1, brow, k16, 2);
    }
  }

  // One piece known to the whole warp: lane 0 emits its slots; returns their count.
  template <typename Emit>
  __device__ int emit_piece(int k, int t0, int t1, int ad, int lane, Emit&& emit) const {
    const int rr = ad >= 0 ? piece_rank(ad) : 0;
    if (rr <= 0) return 0;
    if (lane == 0) emit_slots(k, t0, t1, static_cast<int>(offsets[ad]), rr, emit);
    return rr <= 32 ? 1 : 2;
  }
};

__global__ void __launch_bounds__(kSlPieceThreads) sgmv_linear_pieces_kernel(const int32_t* tiles,
                                                                             const int64_t* offsets,
                                                                             const int64_t* ranks, int T, int R,
                                                                             int m_tiles, int cap, int32_t* mt_first,
                                                                             int4* slots, int* err) {
  __shared__ int warp_sums[kSlPieceWarps];
  __shared__ int carry;
  pdl_wait();  // the schedule launched before writes the tile table
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const PieceWalk walk{tiles, offsets, ranks, T, R};
  // pass 1: slots per output tile
  for (int mt = warp; mt < m_tiles; mt += kSlPieceWarps) {
    const int n = walk.run(mt, lane, [](int, int, int, int, int, int) {});
    if (lane == 0) mt_first[mt] = n;
  }
  __syncthreads();
  // exclusive scan of mt_first[0 .. m_tiles) in chunks of the block
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int c0 = 0; c0 < m_tiles; c0 += kSlPieceThreads) {
    const int mt = c0 + tid;
    const int v = mt < m_tiles ? mt_first[mt] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    int before = carry;
    for (int w2 = 0; w2 < warp; ++w2) before += warp_sums[w2];
    if (mt < m_tiles) mt_first[mt] = min(before + incl - v, cap);
    __syncthreads();
    if (tid == kSlPieceThreads - 1) carry = before + incl;
    __syncthreads();
  }
  const int total = carry;
  if (total > cap && tid == 0) record_error(err, kDevErrBadIndex);  // cannot happen; keeps writes in bounds
  if (tid == 0) mt_first[m_tiles] = min(total, cap);
  __syncthreads();
  // pass 2: slot records
  for (int mt = warp; mt < m_tiles; mt += kSlPieceWarps) {
    const int base = mt_first[mt];
    walk.run(mt, lane, [&](int k, int t0, int t1, int row, int k16, int part) {
      if (base + k < cap) slots[base + k] = make_int4(t0, t1, row, k16 | (part << 4));
    });
  }
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

// Output tiles are taken heaviest row band first (most slots), and the pairs
// take them in a snake order (forward in even rounds, backward in odd ones),
// so a pair that drew a heavy band in one round draws a light one in the next.
// Bands beyond this many keep the plain raster.
constexpr int kSlSortMax = 256;

// Order of an item's k-blocks: its n slot stages spread evenly among the kbm
// base blocks (slot j after pos(j) base blocks).  A slot stage carries a few
// MMAs against a full stage's loads, so a run of them would leave the tensor
// pipe waiting on TMA latency; spread out, each hides behind the base blocks
// around it.  Producer and MMA issuer walk the same order.
struct KOrder {
  int kbm, n, j = 0, b = 0, next;
  __device__ KOrder(int kbm_, int n_) : kbm(kbm_), n(n_) { next = n > 0 ? pos(0) : kbm + 1; }
  __device__ int pos(int jj) const {
    return static_cast<int>((static_cast<int64_t>(jj + 1) * kbm) / (n + 1));
  }
  // true: slot stage j (in idx); false: base block (in idx)
  __device__ bool step(int& idx) {
    if (j < n && b >= next) {
      idx = j++;
      next = j < n ? pos(j) : kbm + 1;
      return true;
    }
    idx = b++;
    return false;
  }
};

}  // namespace

// The pair GEMM: 256 x 256 (NW = 1) or 256 x 512 (NW = 2) tiles as in
// gemm_tc2_kernel, base k-blocks then the tile's slots.  Roles and barriers as
// in gemm_tc2_kernel; NW = 2 keeps both TMEM halves for one tile and loads the
// slot's B rows as one box per 256-column half.
template <int STAGES, int NW, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    sgmv_linear_pair_kernel(const __grid_constant__ SlMaps maps, const GemmArgs args, const SlArgs sl) {
  using L = PairSmem<STAGES, NW>;
  constexpr int kTileN = 256 * NW;
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
  __shared__ int s_cost[kSlSortMax];
  __shared__ int s_order[kSlSortMax];
  const int m_tiles = args.num_m_tiles;
  const bool by_cost = m_tiles <= kSlSortMax;
  if (by_cost) {
    for (int m = threadIdx.x; m < m_tiles; m += blockDim.x) s_cost[m] = sl.mt_first[m + 1] - sl.mt_first[m];
    __syncthreads();
    for (int m = threadIdx.x; m < m_tiles; m += blockDim.x) {
      const int c = s_cost[m];
      int rank = 0;
      for (int j = 0; j < m_tiles; ++j) rank += (s_cost[j] > c) || (s_cost[j] == c && j < m);
      s_order[rank] = m;
    }
  }
  __syncthreads();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_items = args.num_tiles;
  // This pair's j-th output tile (false: none left); every role walks the same sequence.
  auto pair_tile = [&](int j, int& mt, int& nt) {
    const int item = j * npairs + ((j & 1) ? (npairs - 1 - pair) : pair);
    if (item >= num_items) return false;
    if (by_cost) {
      mt = s_order[item / args.num_n_tiles];
      nt = item - (item / args.num_n_tiles) * args.num_n_tiles;
    } else {
      gemm_tile_coords(item, args, mt, nt);
    }
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int mt, nt;
      for (int j = 0; ok && pair_tile(j, mt, nt); ++j) {
        const int e0 = sl.mt_first[mt], e1 = sl.mt_first[mt + 1];
        const int num_kb = args.num_kb_main + (e1 - e0);
        const int row_a = mt * 256 + static_cast<int>(rank) * 128;
        const int row_b = nt * kTileN + static_cast<int>(rank) * 128;  // + 256 for the second half
        KOrder order(args.num_kb_main, e1 - e0);
        for (int q = 0; q < num_kb; ++q) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, args.err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          uint8_t* da = sm_a + stage * L::kABytes;
          uint8_t* db = sm_b + stage * L::kBBytes;
          int kb;
          if (!order.step(kb)) {
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::kStageBytes);
            tma_load_2d_pair(&maps.x, da, bar, kb * kGemmBK, row_a);
#pragma unroll
            for (int h = 0; h < NW; ++h)
              tma_load_2d_pair(&maps.w, db + h * (128 * kGemmBK * 2), bar, kb * kGemmBK, row_b + 256 * h);
          } else {
            const int e = e0 + kb;
            const int4 s = sl.slots[e];
            const int k16 = s.w & 15;
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (L::kABytes + NW * k16 * 16 * 128 * 2));
            tma_load_2d_pair(&maps.z, da, bar, 0, e * 256 + static_cast<int>(rank) * 128);
#pragma unroll
            for (int h = 0; h < NW; ++h)
              tma_load_3d_pair(&maps.b[k16 - 1], db + h * (128 * kGemmBK * 2), bar, 0, s.z, (row_b + 256 * h) / 64);
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
      int mt, nt;
      for (int j = 0; ok && pair_tile(j, mt, nt); ++j, ++local) {
        const int e0 = sl.mt_first[mt], e1 = sl.mt_first[mt + 1];
        const int num_kb = args.num_kb_main + (e1 - e0);
        // NW = 1: accumulator local & 1, its (local >> 1)-th use; NW = 2: both halves, every tile
        const int acc = NW == 1 ? (local & 1) : 0;
        const uint32_t acc_phase = NW == 1 ? ((local >> 1) & 1) : (local & 1);
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1, abort_flag, args.err, kDevErrTimeoutAccEmpty))
          break;
        tc_fence_after();
        KOrder order(args.num_kb_main, e1 - e0);
        uint32_t accum = 0u;  // the item's first MMA into each half starts the sum
        for (int q = 0; q < num_kb; ++q) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (NW == 2 && q == 0) {  // the second half: free once the epilogue has drained it
            if (!mbar_wait_bounded(&acc_empty[1], acc_phase ^ 1, abort_flag, args.err, kDevErrTimeoutAccEmpty)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const uint64_t adesc = umma_desc_sw128(smem_u32(sm_a + stage * L::kABytes));
          int kb;
          const bool slot = order.step(kb);
#pragma unroll
          for (int hn = 0; hn < NW; ++hn) {
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>((NW == 1 ? acc : hn) * 256);
            const uint32_t bs = smem_u32(sm_b + stage * L::kBBytes + hn * (128 * kGemmBK * 2));
            if (!slot) {
              const uint64_t bdesc = umma_desc_sw128(bs);
              for (int k = 0; k < 4; ++k)
                tc_mma_f16_pair(d_tmem, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k),
                                kIdesc, (accum || k > 0) ? 1u : 0u);
            } else {
              const int4 s = sl.slots[e0 + kb];
              const int k16 = s.w & 15, part = (s.w >> 4) & 3;
              const uint32_t lbo = static_cast<uint32_t>(k16 * 16 * 128);  // chunk stride of the B box
              // hi columns at k-step 0.., lo (packed slot) at k-step 2..: same B rows
              for (int h = 0; h < (part == 0 ? 2 : 1); ++h)
                for (int ks = 0; ks < k16; ++ks)
                  tc_mma_f16_pair(d_tmem, adesc + static_cast<uint64_t>(2 * (2 * h + ks)),
                                  sl_desc_mn(bs + static_cast<uint32_t>(ks * 2048), lbo), kIdescMN,
                                  (accum || h > 0 || ks > 0) ? 1u : 0u);
            }
          }
          accum = 1u;
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
    int mt, nt;
    for (int j = 0; pair_tile(j, mt, nt); ++j, ++local) {
      const int acc = NW == 1 ? (local & 1) : 0;
      const uint32_t acc_phase = NW == 1 ? ((local >> 1) & 1) : (local & 1);
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, args.err, kDevErrTimeoutAccFull)) break;
      tc_fence_after();
      const int row = mt * 256 + static_cast<int>(rank) * 128 + quad * 32 + lane;
      T* out_row = static_cast<T*>(args.out) + static_cast<int64_t>(row) * args.ldo;
#pragma unroll 1
      for (int h = 0; h < NW; ++h) {
        const int half = NW == 1 ? acc : h;  // TMEM accumulator drained in this round
        const uint32_t t_row =
            tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(half * 256);
#pragma unroll 1
        for (int c = 0; c < 256; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_row + c, r);
          tmem_wait_ld();
          epilogue_store16<T>(args, out_row, bias, row, nt * kTileN + h * 256 + c, vec_ok, r, st_policy);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[half]), 0));
      }
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

template <int STAGES, int NW, typename T>
int launch_sl_pair(const SlMaps& maps, const GemmArgs& a, const SlArgs& sl, int pairs_cap, cudaStream_t stream) {
  using L = PairSmem<STAGES, NW>;
  const size_t smem = L::kBytes + kSlGuardBytes;
  auto kernel = sgmv_linear_pair_kernel<STAGES, NW, T>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return LORA_ERR_CUDA;
  const int pairs = static_cast<int>(std::min<int64_t>(a.num_tiles, pairs_cap));
  kernel<<<2 * pairs, kGemmThreads, smem, stream>>>(maps, a, sl);
  return cudaGetLastError() == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

}  // namespace

// The slot region is sized for the worst case the schedule allows (every
// schedule tile its own piece of two slots), 32 KB a slot.  Batches whose
// worst case exceeds this (per-token ids over more than ~8000 tokens) are
// declined: the base GEMM + branch path serves them.
constexpr size_t kSlMaxWorkspace = size_t{512} << 20;

size_t sgmv_linear_workspace(int64_t T, int64_t S, int64_t K, int64_t r_max, int num_sms) {
  const size_t bytes = sl_layout(T, S, K, r_max, num_sms).bytes;
  return bytes <= kSlMaxWorkspace ? bytes : 0;
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
  if (l.cap * kSlTile > INT32_MAX || l.bytes > kSlMaxWorkspace || workspace == nullptr ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 || workspace_bytes < l.bytes)
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
    cfg.blockDim = dim3(kSlPieceThreads);
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
  // tile width as the plain GEMM picks it for this shape (the tail adds a
  // few k-blocks per tile, not enough to change the choice)
  const int nw = gemm_pair_width(T, N, K, num_sms);
  a.num_n_tiles = static_cast<int>((N + 256 * nw - 1) / (256 * nw));
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
  if (nw == 2)
    return dtype == LORA_BF16 ? launch_sl_pair<4, 2, __nv_bfloat16>(maps, a, sl, pairs_cap, s)
                              : launch_sl_pair<4, 2, __half>(maps, a, sl, pairs_cap, s);
  return dtype == LORA_BF16 ? launch_sl_pair<kSlStages, 1, __nv_bfloat16>(maps, a, sl, pairs_cap, s)
                            : launch_sl_pair<kSlStages, 1, __half>(maps, a, sl, pairs_cap, s);
}

}  // namespace lora
