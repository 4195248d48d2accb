// Block-structured segmented multi-adapter LoRA kernels.
//
// The device schedule (sgmv.h) starts a tile at every multiple of 64 tokens,
// so each 64-token block of the batch holds a short list of tiles -- runs of
// tokens that share one adapter.  These kernels give one CTA a whole block:
// the token rows they stream (x for the shrink, y / out for the expand) are
// read and written densely, 64 rows at a time, whatever the segment lengths,
// and each tile of the block only selects which adapter rows multiply which
// token rows.  Zipf-distributed request lengths (most segments far shorter
// than 64 tokens) therefore cost no padding traffic.
//
// Both kernels keep their loads in flight with cp.async (16-byte, L1-bypassing)
// and feed mma.sync m16n8k16 through ldmatrix from padded or XOR-swizzled
// shared memory:
//   shrink  z[t, :r_a] = scale * x[t] . A_a^T
//     CTA = (block, K split); a 4-stage pipeline streams the block's x
//     [64 x 64] slice and the adapter rows of its tiles ([<=128 x 64]); rows of
//     a tile are masked into the product of that tile's adapter only.  Splits
//     write fp32 partials; the last CTA of a block (atomic ticket) sums them in
//     split order -- deterministic, no float atomics.
//   expand  out[t, :] = y[t, :] + scale * z[t, :r_a] . B_a
//     CTA = (block, 128 output columns); y and z of the block are fetched
//     once, each tile's B rows are staged in turn and accumulated into one
//     fp32 tile, and out is written with 16-byte stores.  An fp32 z is split
//     into a bf16/f16 hi/lo pair in registers, so the product keeps ~16
//     mantissa bits of z.
// Reference semantics: segmented_branch.py:12-60 (_shrink / _expand per
// request segment), ragged_branch.py:6-40 (per-token adapter, rank-0 skip),
// multilora.py:128-182 and :295-347 (ragged / bucketed shrink and expand).
#include <algorithm>

#include "common.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

namespace {

constexpr int kBT = kSgmvTileTokens;  // tokens per block (64)
constexpr int kShrStages = 4;
constexpr int kShrARows = 128;  // adapter rows staged per pass
constexpr int kExpBN = 128;     // output columns per expand CTA
constexpr int kExpStride = kExpBN + 8;  // padded row (elements): conflict-free fragments and ldmatrix

// The tiles of one 64-token block, in shared memory.
struct BlockTiles {
  int n;
  int lo[kBT], hi[kBT];  // token rows [lo, hi) relative to the block start
  int r[kBT];            // rank used (0 = nothing to add)
  int64_t arow[kBT];     // first adapter row in the flat tables
  // shrink only: passes over the adapter rows, each <= kShrARows rows
  int srow[kBT];         // first staged row of the tile within its pass
  int pass[kBT];
  int npass;
  int row_r[kBT];        // rank of the tile that owns each row
};

// Warp 0 reads the block's tiles; thread 0 then groups them into passes.
LORA_DEVINL void load_block_tiles(BlockTiles& bt, const int32_t* tiles, const int64_t* offsets,
                                  const int64_t* ranks, int R, int block, int tbase, int ntok) {
  const int tid = threadIdx.x;
  if (tid < 32) {
    const int nt_all = sgmv_num_tiles(tiles);
    const int32_t* first = sgmv_block_first(tiles);
    const int f0 = min(first[block], nt_all);
    const int f1 = max(f0, min(first[block + 1], nt_all));
    const int n = min(f1 - f0, kBT);
    for (int i = tid; i < n; i += 32) {
      const int ts = sgmv_tile_start(tiles, f0 + i), te = sgmv_tile_start(tiles, f0 + i + 1);
      const int ad = sgmv_tile_adapter(tiles, f0 + i);
      int r = 0;
      int64_t arow = 0;
      if (ad >= 0) {
        const int64_t rr = ranks[ad];
        r = rr <= 0 ? 0 : static_cast<int>(rr < R ? rr : R);
        arow = offsets[ad];
      }
      int lo = ts - tbase, hi = te - tbase;
      lo = lo < 0 ? 0 : (lo > ntok ? ntok : lo);
      hi = hi < lo ? lo : (hi > ntok ? ntok : hi);
      bt.lo[i] = lo;
      bt.hi[i] = hi;
      bt.r[i] = (hi > lo) ? r : 0;
      bt.arow[i] = arow;
    }
    if (tid == 0) bt.n = n;
  }
  __syncthreads();
  if (tid == 0) {
    int pass = 0, used = 0;
    for (int i = 0; i < bt.n; ++i) {
      const int r16 = (bt.r[i] + 15) & ~15;
      if (r16 == 0) {
        bt.pass[i] = -1;
        continue;
      }
      if (used + r16 > kShrARows) {
        ++pass;
        used = 0;
      }
      bt.pass[i] = pass;
      bt.srow[i] = used;
      used += r16;
    }
    bt.npass = used > 0 || pass > 0 ? pass + 1 : 0;
  }
  for (int row = tid; row < kBT; row += blockDim.x) {
    int rr = 0;
    for (int i = 0; i < bt.n; ++i)
      if (row >= bt.lo[i] && row < bt.hi[i]) rr = bt.r[i];
    bt.row_r[row] = rr;
  }
  __syncthreads();
}

// byte offset of 16-byte chunk c (0..7) of row r in a [rows][64] 16-bit tile, 128B-XOR swizzled
LORA_DEVINL uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }

LORA_DEVINL int64_t phys_row(const int64_t* rows, int64_t t) { return rows ? rows[t] : t; }

template <typename TZ>
LORA_DEVINL void store_z(TZ* z_row, int col, int width, int split, float v) {
  const TZ hi = from_f32<TZ>(v);
  z_row[col] = hi;
  if (split) z_row[col + width] = from_f32<TZ>(v - to_f32(hi));
}

// --------------------------------------------------------------------- shrink
// Launched as clusters of split_k CTAs along grid y: the CTAs of a cluster
// take the K slices of one block and sum their fp32 partial tiles through
// distributed shared memory in rank order (deterministic, no workspace).
template <typename T, typename TZ, int NT>
__global__ void __launch_bounds__(128) sgmv_shrink_block_kernel(const SgmvShrinkBlockArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr int kXBytes = kBT * 128;
  constexpr int kABytes = kShrARows * 128;
  constexpr int kStageBytes = kXBytes + kABytes;
  constexpr int kRS = NT * 8 + 8;  // partial-tile row stride (floats): conflict-free float2 stores
  static_assert(kBT * kRS * 4 <= kShrStages * kStageBytes, "partial tile must fit the stage buffers");
  BlockTiles& bt = *reinterpret_cast<BlockTiles*>(smem_raw + kShrStages * kStageBytes);
  __shared__ const T* s_arow[kShrARows];  // source row of each staged adapter row (NULL = zero)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int block = blockIdx.x, ks = blockIdx.y;
  const int cs = p.split_k;  // cluster size == number of K slices
  const int tbase = block * kBT;
  const int ntok = min(kBT, p.T - tbase);
  const int k0 = ks * p.kslice;
  const int k1 = min(p.K, k0 + p.kslice);
  const int nsteps = k1 > k0 ? (k1 - k0 + 63) / 64 : 0;
  const T* x = static_cast<const T*>(p.x);
  const T* a = static_cast<const T*>(p.a);
  TZ* z = static_cast<TZ*>(p.z);

  load_block_tiles(bt, p.tiles, p.offsets, p.ranks, p.R, block, tbase, ntok);

  // x rows this thread copies: rows (tid >> 3) + 16 i, chunk tid & 7
  const int xc = tid & 7;
  const T* xrow[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = (tid >> 3) + 16 * i;
    xrow[i] = row < ntok ? x + phys_row(p.rows, tbase + row) * p.ldx : nullptr;
  }
  // output rows this CTA of the cluster writes
  const int rank_in_cluster = static_cast<int>(cluster_ctarank());
  const int rpr = (ntok + cs - 1) / cs;
  const int out_r0 = min(ntok, rank_in_cluster * rpr), out_r1 = min(ntok, out_r0 + rpr);

  float acc[NT][4];
  const int row_a = 16 * warp + g, row_b = row_a + 8;
  float* red = reinterpret_cast<float*>(smem_raw);

  for (int pass = 0; pass < bt.npass; ++pass) {
    // ---- staged adapter rows of this pass
    int prow = 0;
    for (int i = 0; i < bt.n; ++i)
      if (bt.pass[i] == pass) prow = bt.srow[i] + ((bt.r[i] + 15) & ~15);
    for (int row = tid; row < kShrARows; row += blockDim.x) {
      const T* src = nullptr;
      for (int i = 0; i < bt.n; ++i) {
        if (bt.pass[i] != pass) continue;
        const int j = row - bt.srow[i];
        if (j >= 0 && j < bt.r[i]) src = a + (bt.arow[i] + j) * p.lda;
      }
      s_arow[row] = src;
    }
    __syncthreads();

    auto load_stage = [&](int step, int slot) {
      uint8_t* st = smem_raw + slot * kStageBytes;
      const int kc = k0 + step * 64 + xc * 8;
      const bool kin = kc < k1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = (tid >> 3) + 16 * i;
        const bool v = kin && xrow[i] != nullptr;
        cp_async16(st + swz(row, xc), v ? xrow[i] + kc : x, v ? 16 : 0);
      }
#pragma unroll
      for (int i = 0; i < kShrARows / 16; ++i) {
        const int row = (tid >> 3) + 16 * i;
        if (row >= prow) break;
        const T* src = s_arow[row];
        const bool v = kin && src != nullptr;
        cp_async16(st + kXBytes + swz(row, xc), v ? src + kc : a, v ? 16 : 0);
      }
    };

#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

#pragma unroll
    for (int s = 0; s < kShrStages - 1; ++s) {
      if (s < nsteps) load_stage(s, s);
      cp_async_commit();
    }
    for (int step = 0; step < nsteps; ++step) {
      cp_async_wait<kShrStages - 2>();
      __syncthreads();
      const int nxt = step + kShrStages - 1;
      if (nxt < nsteps) load_stage(nxt, nxt % kShrStages);
      cp_async_commit();

      const uint8_t* st = smem_raw + (step % kShrStages) * kStageBytes;
      const uint32_t xs = smem_u32(st), as = smem_u32(st + kXBytes);
      if (16 * warp < ntok) {
        uint32_t af[4][4];
#pragma unroll
        for (int k16 = 0; k16 < 4; ++k16)
          ldmatrix_x4(af[k16], xs + swz(16 * warp + (lane & 15), 2 * k16 + (lane >> 4)));
        for (int i = 0; i < bt.n; ++i) {
          if (bt.pass[i] != pass) continue;
          const int lo = bt.lo[i], hi = bt.hi[i];
          if (hi <= 16 * warp || lo >= 16 * warp + 16) continue;
          const bool ma = row_a >= lo && row_a < hi, mb = row_b >= lo && row_b < hi;
          const int npair = (bt.r[i] + 15) >> 4;
          const int sr = bt.srow[i];
#pragma unroll
          for (int k16 = 0; k16 < 4; ++k16) {
            const uint32_t am[4] = {ma ? af[k16][0] : 0u, mb ? af[k16][1] : 0u, ma ? af[k16][2] : 0u,
                                    mb ? af[k16][3] : 0u};
#pragma unroll
            for (int pp = 0; pp < NT / 2; ++pp) {
              if (pp >= npair) break;
              uint32_t bf[4];
              const int mi = lane >> 3;
              ldmatrix_x4(bf, as + swz(sr + pp * 16 + (mi >> 1) * 8 + (lane & 7), 2 * k16 + (mi & 1)));
              const uint32_t b0[2] = {bf[0], bf[1]}, b1[2] = {bf[2], bf[3]};
              mma16816<T>(acc[2 * pp], am, b0);
              mma16816<T>(acc[2 * pp + 1], am, b1);
            }
          }
        }
      }
    }
    cp_async_wait<0>();
    __syncthreads();  // every warp is done with the stage buffers: they now hold the partial tile

    if (16 * warp < ntok) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        *reinterpret_cast<float2*>(red + row_a * kRS + nt * 8 + 2 * q) = make_float2(acc[nt][0], acc[nt][1]);
        *reinterpret_cast<float2*>(red + row_b * kRS + nt * 8 + 2 * q) = make_float2(acc[nt][2], acc[nt][3]);
      }
    }
    cluster_sync_all();  // all partial tiles of the cluster are written

    // ---- this CTA's rows: sum the cluster's partials in rank order
    const uint32_t red_addr = smem_u32(red);
    for (int idx = tid; idx < (out_r1 - out_r0) * (NT * 2); idx += blockDim.x) {
      const int row = out_r0 + idx / (NT * 2);
      const int c4 = (idx % (NT * 2)) * 4;
      int ti = -1;
      for (int i = 0; i < bt.n; ++i)
        if (row >= bt.lo[i] && row < bt.hi[i]) ti = i;
      if (ti < 0 || bt.pass[ti] != pass) continue;
      const int r = bt.r[ti];
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      const uint32_t off = red_addr + static_cast<uint32_t>((row * kRS + c4) * 4);
      for (int s = 0; s < cs; ++s) {
        const float4 v = ld_dsmem_f4(mapa_shared(off, static_cast<uint32_t>(s)));
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
      TZ* zr = z + phys_row(p.rows, tbase + row) * p.ldz;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = c4 + e;
        if (col < p.z_width) store_z<TZ>(zr, col, p.z_width, p.z_split, col < r ? p.scale * vals[e] : 0.f);
      }
    }
    cluster_sync_all();  // peers have read this CTA's partial tile; the buffers may be reused
  }

  // ---- rows without a rank, and columns beyond the mma tiles, are zero
  for (int idx = tid; idx < (out_r1 - out_r0) * p.z_width; idx += blockDim.x) {
    const int row = out_r0 + idx / p.z_width, col = idx % p.z_width;
    if (bt.row_r[row] > 0 && col < NT * 8) continue;
    store_z<TZ>(z + phys_row(p.rows, tbase + row) * p.ldz, col, p.z_width, p.z_split, 0.f);
  }
}

// --------------------------------------------------------------------- expand
// out = y + scale * z . B over one 64-token block and 128 output columns.
// Each thread keeps the z values of its two fragment rows in registers (fp32),
// the B rows of all the block's tiles are staged at once (passes of <= 128
// rows), and every tile adds its adapter's product to the rows it owns.
template <typename T, typename TZ, int RZ>
__global__ void __launch_bounds__(128) sgmv_expand_block_kernel(const SgmvExpandBlockArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr bool kSplit = sizeof(TZ) == 4;
  constexpr int kRows = RZ > kShrARows ? RZ : kShrARows;  // staged B rows per pass
  T* ys = reinterpret_cast<T*>(smem_raw);
  T* bs = ys + kBT * kExpStride;
  BlockTiles& bt = *reinterpret_cast<BlockTiles*>(reinterpret_cast<uint8_t*>(bs + kRows * kExpStride));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int block = blockIdx.y;
  const int n0 = blockIdx.x * kExpBN;
  const int tbase = block * kBT;
  const int ntok = min(kBT, p.T - tbase);
  const T* y = static_cast<const T*>(p.y);
  const TZ* z = static_cast<const TZ*>(p.z);
  const T* b = static_cast<const T*>(p.b);
  const int row_a = 16 * warp + g, row_b = row_a + 8;

  // Launched with programmatic serialization behind the shrink that writes z:
  // the kernel waits for it before its first global read (the tile table may
  // come from a schedule launched just before, z from the shrink), so only its
  // set-up overlaps the kernel before it.
  pdl_wait();
  load_block_tiles(bt, p.tiles, p.offsets, p.ranks, p.R, block, tbase, ntok);

  // ---- y of the block (rows (tid >> 4) + 8 i, chunk tid & 15)
  const int ch = tid & 15;
  const bool col_in = n0 + ch * 8 < p.N;
  int64_t prow[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = (tid >> 4) + 8 * i;
    prow[i] = row < ntok ? phys_row(p.rows, tbase + row) : -1;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = (tid >> 4) + 8 * i;
    if (y != nullptr && prow[i] >= 0 && col_in)
      cp_async16(ys + row * kExpStride + ch * 8, y + prow[i] * p.ldy + n0 + ch * 8, 16);
  }
  cp_async_commit();

  // ---- z of this thread's fragment rows: zf[h][k16][kk][e] = z[row_h, 16 k16 + 8 kk + 2 q + e]
  float zf[2][RZ / 16][2][2];
  {
    const int64_t pa = row_a < ntok ? phys_row(p.rows, tbase + row_a) : -1;
    const int64_t pb = row_b < ntok ? phys_row(p.rows, tbase + row_b) : -1;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t pr = h ? pb : pa;
#pragma unroll
      for (int k16 = 0; k16 < RZ / 16; ++k16) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int c = 16 * k16 + 8 * kk + 2 * q;
          float2 v = make_float2(0.f, 0.f);
          if (pr >= 0 && c < p.R) {
            const TZ* zp = z + pr * p.ldz + c;
            v.x = to_f32(zp[0]);
            if (c + 1 < p.R) v.y = to_f32(zp[1]);
          }
          zf[h][k16][kk][0] = v.x;
          zf[h][k16][kk][1] = v.y;
        }
      }
    }
  }

  float acc[kExpBN / 8][4];
#pragma unroll
  for (int nt = 0; nt < kExpBN / 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  const uint32_t bsa = smem_u32(bs);

  for (int pass = 0; pass < bt.npass; ++pass) {
    if (pass > 0) __syncthreads();  // the previous pass's reads of bs are done
    for (int i = 0; i < bt.n; ++i) {
      if (bt.pass[i] != pass) continue;
      const int r = bt.r[i], r16 = (r + 15) & ~15, sr = bt.srow[i];
      for (int idx = tid; idx < r16 * 16; idx += blockDim.x) {
        const int j = idx >> 4, c = idx & 15;
        const bool v = j < r && n0 + c * 8 < p.N;
        cp_async16(bs + (sr + j) * kExpStride + c * 8, v ? b + (bt.arow[i] + j) * p.ldb + n0 + c * 8 : b,
                   v ? 16 : 0);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    for (int i = 0; i < bt.n; ++i) {
      if (bt.pass[i] != pass) continue;
      const int lo = bt.lo[i], hi = bt.hi[i];
      if (hi <= 16 * warp || lo >= 16 * warp + 16) continue;
      const bool ma = row_a >= lo && row_a < hi, mb = row_b >= lo && row_b < hi;
      const int r = bt.r[i], sr = bt.srow[i];
#pragma unroll
      for (int k16 = 0; k16 < RZ / 16; ++k16) {
        if (16 * k16 >= r) break;
        uint32_t ah[4], al[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const bool m = h ? mb : ma;
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const int c = 16 * k16 + 8 * kk + 2 * q;
            const float v0 = (m && c < r) ? zf[h][k16][kk][0] : 0.f;
            const float v1 = (m && c + 1 < r) ? zf[h][k16][kk][1] : 0.f;
            const T h0 = from_f32<T>(v0), h1 = from_f32<T>(v1);
            ah[h + 2 * kk] = pack2<T>(to_f32(h0), to_f32(h1));
            al[h + 2 * kk] = pack2<T>(v0 - to_f32(h0), v1 - to_f32(h1));
          }
        }
#pragma unroll
        for (int pp = 0; pp < kExpBN / 16; ++pp) {
          uint32_t bf[4];
          const int mi = lane >> 3;
          const int krow = sr + 16 * k16 + (mi & 1) * 8 + (lane & 7);
          const int ncol = pp * 16 + (mi >> 1) * 8;
          ldmatrix_x4_trans(bf, bsa + static_cast<uint32_t>((krow * kExpStride + ncol) * sizeof(T)));
          const uint32_t b0[2] = {bf[0], bf[1]}, b1[2] = {bf[2], bf[3]};
          mma16816<T>(acc[2 * pp], ah, b0);
          mma16816<T>(acc[2 * pp + 1], ah, b1);
          if (kSplit) {
            mma16816<T>(acc[2 * pp], al, b0);
            mma16816<T>(acc[2 * pp + 1], al, b1);
          }
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- out = y + scale * acc, assembled in ys, then 16-byte stores
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = h ? row_b : row_a;
    if (row >= ntok) continue;
#pragma unroll
    for (int nt = 0; nt < kExpBN / 8; ++nt) {
      const int col = nt * 8 + 2 * q;
      uint32_t* cell = reinterpret_cast<uint32_t*>(ys + row * kExpStride + col);
      const float2 yv = y != nullptr ? unpack2<T>(*cell) : make_float2(0.f, 0.f);
      *cell = pack2<T>(yv.x + p.scale * acc[nt][2 * h], yv.y + p.scale * acc[nt][2 * h + 1]);
    }
  }
  __syncthreads();
  T* out = static_cast<T*>(p.out);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = (tid >> 4) + 8 * i;
    if (prow[i] >= 0 && col_in)
      *reinterpret_cast<uint4*>(out + prow[i] * p.ldo + n0 + ch * 8) =
          *reinterpret_cast<const uint4*>(ys + row * kExpStride + ch * 8);
  }
}

template <typename T, typename TZ, int NT>
int launch_shrink_nt(const SgmvShrinkBlockArgs& p, dim3 grid, cudaStream_t s) {
  const size_t smem = kShrStages * (kBT * 128 + kShrARows * 128) + sizeof(BlockTiles);
  auto kernel = sgmv_shrink_block_kernel<T, TZ, NT>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return LORA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = grid.y;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

template <typename T, typename TZ>
int launch_shrink_t(const SgmvShrinkBlockArgs& p, dim3 grid, cudaStream_t s) {
  if (p.R <= 16) return launch_shrink_nt<T, TZ, 2>(p, grid, s);
  if (p.R <= 32) return launch_shrink_nt<T, TZ, 4>(p, grid, s);
  if (p.R <= 64) return launch_shrink_nt<T, TZ, 8>(p, grid, s);
  return launch_shrink_nt<T, TZ, 16>(p, grid, s);
}

template <typename T, typename TZ, int RZ>
int launch_expand_rz(const SgmvExpandBlockArgs& p, dim3 grid, cudaStream_t s) {
  constexpr int kRows = RZ > kShrARows ? RZ : kShrARows;
  const size_t smem = (kBT + kRows) * kExpStride * sizeof(T) + sizeof(BlockTiles);
  auto kernel = sgmv_expand_block_kernel<T, TZ, RZ>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return LORA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, p) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

template <typename T, typename TZ>
int launch_expand_t(const SgmvExpandBlockArgs& p, dim3 grid, cudaStream_t s) {
  if (p.R <= 64) return launch_expand_rz<T, TZ, 64>(p, grid, s);
  return launch_expand_rz<T, TZ, 128>(p, grid, s);
}

inline bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

int sgmv_shrink_block_split(int64_t T, int64_t K, int num_sms) {
  // Two CTAs fit an SM; pick the split that minimises waves x K-steps per CTA,
  // keeping >= 4 K-steps (256 of K) per split so the pipeline fills.
  const int64_t nb = std::max<int64_t>(sgmv_blocks(T), 1);
  const int64_t steps = std::max<int64_t>((K + 63) / 64, 1);
  const int64_t slots = 2 * static_cast<int64_t>(std::max(num_sms, 1));
  int best = 1;
  double best_cost = 1e300;
  for (int sk = 1; sk <= std::min<int64_t>(kSgmvMaxClusterSplit, std::max<int64_t>(steps / 4, 1)); ++sk) {
    const int64_t per = (steps + sk - 1) / sk;
    const int64_t used = (steps + per - 1) / per;  // splits that are not empty
    if (used != sk) continue;
    const int64_t waves = (nb * sk + slots - 1) / slots;
    const double cost = static_cast<double>(waves * per) + 0.05 * sk;
    if (cost < best_cost) {
      best_cost = cost;
      best = sk;
    }
  }
  return best;
}

int launch_sgmv_shrink_block(const SgmvShrinkBlockArgs& p, int dtype, int z_dtype, int num_sms, void* stream) {
  (void)num_sms;
  if (p.R > 128 || p.R <= 0) return LORA_ERR_UNSUPPORTED;
  if (p.K % 8 != 0 || p.ldx % 8 != 0 || p.lda % 8 != 0 || !al16(p.x) || !al16(p.a)) return LORA_ERR_UNSUPPORTED;
  const int64_t nb = sgmv_blocks(p.T);
  if (nb > INT32_MAX || p.split_k < 1 || p.split_k > kSgmvMaxClusterSplit) return LORA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(nb), static_cast<unsigned>(p.split_k));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LORA_BF16) {
    if (z_dtype == LORA_F32) return launch_shrink_t<__nv_bfloat16, float>(p, grid, s);
    if (z_dtype == LORA_BF16) return launch_shrink_t<__nv_bfloat16, __nv_bfloat16>(p, grid, s);
  } else if (dtype == LORA_F16) {
    if (z_dtype == LORA_F32) return launch_shrink_t<__half, float>(p, grid, s);
    if (z_dtype == LORA_F16) return launch_shrink_t<__half, __half>(p, grid, s);
  }
  return LORA_ERR_DTYPE;
}

int launch_sgmv_expand_block(const SgmvExpandBlockArgs& p, int dtype, int z_dtype, void* stream) {
  if (p.R > 128 || p.R <= 0) return LORA_ERR_UNSUPPORTED;
  if (p.N % 8 != 0 || p.ldb % 8 != 0 || p.ldo % 8 != 0 || !al16(p.b) || !al16(p.out)) return LORA_ERR_UNSUPPORTED;
  if (p.y != nullptr && (p.ldy % 8 != 0 || !al16(p.y))) return LORA_ERR_UNSUPPORTED;
  const int64_t nb = sgmv_blocks(p.T);
  const int64_t nch = (p.N + kExpBN - 1) / kExpBN;
  if (nb > 65535 || nch > INT32_MAX) return LORA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(nch), static_cast<unsigned>(nb));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LORA_BF16) {
    if (z_dtype == LORA_F32) return launch_expand_t<__nv_bfloat16, float>(p, grid, s);
    if (z_dtype == LORA_BF16) return launch_expand_t<__nv_bfloat16, __nv_bfloat16>(p, grid, s);
  } else if (dtype == LORA_F16) {
    if (z_dtype == LORA_F32) return launch_expand_t<__half, float>(p, grid, s);
    if (z_dtype == LORA_F16) return launch_expand_t<__half, __half>(p, grid, s);
  }
  return LORA_ERR_DTYPE;
}

}  // namespace lora
