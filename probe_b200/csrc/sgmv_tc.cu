// Segmented multi-adapter shrink on Blackwell tensor cores.
//
//   z[t, :r_a] = scale * x[t] . A_a^T   for every token t with adapter a(t)
//
// One CTA owns a 128-token block of the batch (the M = 128 operand of
// tcgen05.mma, fed by TMA) and one K slice.  The adapter rows of every tile in
// the block (a tile = a run of tokens with one adapter, from the device
// schedule) are gathered by TMA, one box per tile, into one N <= 256 operand,
// so a single MMA chain multiplies every token by every adapter present in
// its block; each token then takes its own adapter's columns from TMEM.  The
// wasted products are free -- the kernel streams x once and the tensor pipe
// is otherwise idle.  A pass holds up to 512 adapter rows (two MMAs of N <= 256
// into the two halves of TMEM); the stage stride is sized at run time to the
// block's widest pass, so narrow blocks keep more stages in flight.  Blocks
// whose adapters need more rows than one pass holds run in passes.  The K slices of a block are the CTAs of a cluster: each writes its
// per-token results to shared memory, pushes row slices to their owners with
// bulk shared::cluster copies, and each owner sums its rows in rank order
// (deterministic, no workspace) and writes z.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner and MMA issuer,
// warps 2..5 table setup and epilogue.  Every wait is bounded; every CTA
// reaches every cluster barrier.
// Reference semantics: segmented_branch.py:12-28 and ragged_branch.py:6-16
// (_shrink per request / token, rank-0 skip), multilora.py:128-182.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "runtime.h"
#include "sgmv.h"

namespace lora {

namespace {

constexpr int kTcBM = 128;         // tokens per CTA
constexpr int kTcBK = 64;          // K per stage
constexpr int kTcMmaN = 256;       // adapter rows per MMA (N)
constexpr int kTcPassMax = 512;    // adapter rows per pass (two MMAs, 512 TMEM columns)
constexpr int kTcMaxStages = 8;
constexpr int kTcThreads = 192;
constexpr int kTcMaxTiles = 128;   // a 128-token block holds at most 128 tiles
constexpr int kTcXBytes = kTcBM * kTcBK * 2;    // 16 KB

struct TcTiles {
  int n, npass;
  int stride, stages;                     // stage ring geometry for this block
  int lo[kTcMaxTiles], hi[kTcMaxTiles];  // rows [lo, hi) of the block
  int r[kTcMaxTiles];                     // rank used (0 = nothing)
  int srow[kTcMaxTiles];                  // first operand row within its pass
  int pass[kTcMaxTiles];
  int64_t arow[kTcMaxTiles];              // first row in a_flat
  int pass_rows[kTcMaxTiles];             // operand rows of each pass (multiple of 16)
  int row_tile[kTcBM];                    // tile of each row, -1 = none
};

// Shared memory: [stage ring][red][tile table][barriers].  Each stage is the
// x tile (16 KB) followed by the pass's adapter rows (128 B each), its stride
// rounded to 1 KB (swizzle atoms stay aligned).
struct TcLayout {
  int ring, rs, cs;
  int red_off, tab_off, bar_off, bytes;
  int rpr, slice_bytes;
  __host__ __device__ TcLayout(int ring_, int rmax16, int cs_) : ring(ring_), cs(cs_) {
    rs = rmax16 + 4;  // per-token result row (floats)
    red_off = ring;   // [128][rs] fp32, written pass by pass during the mainloop
    // slices pushed by the other CTAs land at offset 0 (stage buffers, idle by then)
    rpr = ((kTcBM + cs - 1) / cs + 7) & ~7;
    slice_bytes = rpr * rs * 4;
    tab_off = (red_off + kTcBM * rs * 4 + 1023) & ~1023;
    bar_off = (tab_off + static_cast<int>(sizeof(TcTiles)) + 15) & ~15;
    bytes = bar_off + 256 + 1024;
  }
};

__host__ __device__ inline int tc_stage_stride(int rows) { return (kTcXBytes + rows * 128 + 1023) & ~1023; }

}  // namespace

// lora_A gather maps, one per box height 16, 32, ..., 128 rows, so every tile's
// k-block comes in one TMA box of exactly its (16-rounded) rank: small boxes
// measured far slower per byte than tall ones on B200.
struct TcAMaps {
  CUtensorMap m[8];
};

struct SgmvTcArgs {
  void* z;
  const int64_t* offsets;
  const int64_t* ranks;
  const int32_t* tiles;
  int* err;
  int64_t ldz;
  int T, K, R, z_width, z_f32;
  int num_kb, kb_per, split, ring, rmax16, pass_cap;
  float scale;
};

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1) sgmv_shrink_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                                       const __grid_constant__ TcAMaps tm_a,
                                                                       const SgmvTcArgs p) {
  constexpr uint32_t kTmemCols = kTcPassMax;
  const TcLayout L(p.ring, p.rmax16, p.split);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  if (static_cast<uint32_t>(smem - smem_raw) + static_cast<uint32_t>(L.bar_off) + 160u > dynamic_smem_bytes()) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemLayout);
    return;
  }
  TcTiles& tb = *reinterpret_cast<TcTiles*>(smem + L.tab_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + kTcMaxStages;
  uint64_t* acc_full = empty + kTcMaxStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* rpull = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rpull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x, ks = blockIdx.y, cs = p.split;
  const int t0 = blk * kTcBM;
  const int ntok = min(kTcBM, p.T - t0);
  const int kb0 = ks * p.kb_per;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per);
  const int n_main = max(kb1 - kb0, 0);
  const int rs = L.rs;

  // Launched with programmatic serialization behind the schedule: barriers and
  // TMEM are set up while it finishes; every global read of the table, x and
  // a_flat comes after griddepcontrol.wait (the producer's loads follow the
  // table through the block barrier).  Dependents are signalled only after
  // that wait: the expand launched next reads the tile table before its own
  // wait, so the schedule that wrote it must be complete by then.

  // ---- tile table of the block (warps 2..5), barriers (thread 0), TMEM (warp 1)
  if (warp >= 2) {
    pdl_wait();
    if (threadIdx.x == 64) pdl_launch_dependents();
    const int et = threadIdx.x - 64;
    const int nt_all = sgmv_num_tiles(p.tiles);
    const int32_t* first = sgmv_block_first(p.tiles);
    const int nb64 = (p.T + kSgmvTileTokens - 1) / kSgmvTileTokens;
    const int f0 = min(first[min(2 * blk, nb64)], nt_all);
    const int f1 = max(f0, min(first[min(2 * blk + 2, nb64)], nt_all));
    const int n = min(f1 - f0, kTcMaxTiles);
    for (int i = et; i < n; i += 128) {
      const int ts = sgmv_tile_start(p.tiles, f0 + i), te = sgmv_tile_start(p.tiles, f0 + i + 1);
      const int ad = sgmv_tile_adapter(p.tiles, f0 + i);
      int r = 0;
      int64_t arow = 0;
      if (ad >= 0) {
        const int64_t rr = p.ranks[ad];
        r = rr <= 0 ? 0 : static_cast<int>(rr < p.R ? rr : p.R);
        arow = p.offsets[ad];
      }
      int lo = ts - t0, hi = te - t0;
      lo = lo < 0 ? 0 : (lo > ntok ? ntok : lo);
      hi = hi < lo ? lo : (hi > ntok ? ntok : hi);
      tb.lo[i] = lo;
      tb.hi[i] = hi;
      tb.r[i] = hi > lo ? r : 0;
      tb.arow[i] = arow;
    }
    for (int row = et; row < kTcBM; row += 128) tb.row_tile[row] = -1;
    named_bar_sync(1, 128);
    if (et == 0) {
      tb.n = n;
      int pass = 0, used = 0, widest = 16;
      for (int i = 0; i < n; ++i) {
        const int r16 = (tb.r[i] + 15) & ~15;
        if (r16 == 0) {
          tb.pass[i] = -1;
          continue;
        }
        if (used + r16 > p.pass_cap) {
          tb.pass_rows[pass] = used;
          widest = max(widest, used);
          ++pass;
          used = 0;
        }
        tb.pass[i] = pass;
        tb.srow[i] = used;
        used += r16;
      }
      if (used > 0) tb.pass_rows[pass] = used;
      widest = max(widest, used);
      tb.npass = used > 0 ? pass + 1 : 0;
      tb.stride = tc_stage_stride(widest);
      // at least 2: the host caps a pass at the rows two stages of the ring hold
      tb.stages = min(kTcMaxStages, L.ring / tb.stride);
    }
    named_bar_sync(1, 128);
    for (int i = et; i < n; i += 128)
      if (tb.pass[i] >= 0)
        for (int row = tb.lo[i]; row < tb.hi[i]; ++row) tb.row_tile[row] = i;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcMaxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(rpull, 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (cs > 1) {
      const int my_rows = min(kTcBM, (ks + 1) * L.rpr) - min(kTcBM, ks * L.rpr);
      mbar_arrive_expect_tx(rpull, static_cast<uint32_t>((cs - 1) * my_rows * rs * 4));
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    for (int h = 0; h < 8; ++h) tma_prefetch_desc(&tm_a.m[h]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (cs > 1) cluster_sync_all();  // every CTA's receive barrier exists before any push
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t idesc_base = umma_idesc_f16(kTcBM, 16, std::is_same<T, __nv_bfloat16>::value ? 1 : 0) &
                              ~(0x3Fu << 17);  // N field filled per pass
  float* red = reinterpret_cast<float*>(smem + L.red_off);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int pass = 0; ok && pass < tb.npass; ++pass) {
        const uint32_t tx = static_cast<uint32_t>(kTcXBytes + tb.pass_rows[pass] * kTcBK * 2);
        for (int i = 0; i < n_main; ++i) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int kc = (kb0 + i) * kTcBK;
          mbar_arrive_expect_tx(&full[stage], tx);
          uint8_t* xs = smem + stage * tb.stride;
          tma_load_2d(&tm_x, xs, &full[stage], kc, t0);
          uint8_t* as = xs + kTcXBytes;
          for (int ti = 0; ti < tb.n; ++ti) {
            if (tb.pass[ti] != pass) continue;
            const int r16 = (tb.r[ti] + 15) & ~15;
            tma_load_2d(&tm_a.m[(r16 >> 4) - 1], as + tb.srow[ti] * 128, &full[stage], kc,
                        static_cast<int32_t>(tb.arow[ti]));
          }
          if (++stage == tb.stages) {
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
      bool ok = true;
      for (int pass = 0; ok && pass < tb.npass; ++pass) {
        if (pass > 0) {
          if (!mbar_wait_bounded(acc_empty, (pass - 1) & 1, abort_flag, p.err, kDevErrTimeoutAccEmpty)) break;
          tc_fence_after();
        }
        // rows [0, 256) into TMEM columns [0, 256), the rest into [256, 512)
        const int rows = tb.pass_rows[pass];
        const int n0 = min(rows, kTcMmaN), n1 = rows - n0;
        const uint32_t idesc0 = idesc_base | (static_cast<uint32_t>(n0 >> 3) << 17);
        const uint32_t idesc1 = idesc_base | (static_cast<uint32_t>((n1 > 0 ? n1 : 16) >> 3) << 17);
        for (int i = 0; i < n_main; ++i) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xs = smem_u32(smem + stage * tb.stride);
          const uint64_t xd = umma_desc_sw128(xs);
          const uint64_t ad0 = umma_desc_sw128(xs + kTcXBytes);
          const uint64_t ad1 = umma_desc_sw128(xs + kTcXBytes + kTcMmaN * 128);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            tc_mma_f16(tmem_base, xd + static_cast<uint64_t>(2 * k), ad0 + static_cast<uint64_t>(2 * k), idesc0,
                       (i > 0 || k > 0) ? 1u : 0u);
            if (n1 > 0)
              tc_mma_f16(tmem_base + kTcMmaN, xd + static_cast<uint64_t>(2 * k), ad1 + static_cast<uint64_t>(2 * k),
                         idesc1, (i > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == tb.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) tc_commit(acc_full);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int my_tile = tb.row_tile[row];
    for (int pass = 0; pass < tb.npass; ++pass) {
      const bool ok = mbar_wait_bounded(acc_full, pass & 1, abort_flag, p.err, kDevErrTimeoutAccFull);
      tc_fence_after();
      __syncwarp();
      // every tile of this pass present in the warp's 32 rows: read its columns
      for (int ti = 0; ti < tb.n; ++ti) {
        if (tb.pass[ti] != pass || tb.hi[ti] <= quad * 32 || tb.lo[ti] >= quad * 32 + 32) continue;
        const int r16 = (tb.r[ti] + 15) & ~15;
        for (int c = 0; c < r16; c += 16) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                 static_cast<uint32_t>(tb.srow[ti] + c),
                             v);
          tmem_wait_ld();
          if (ok && my_tile == ti) {
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(red + row * rs + c + e) =
                  make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]), __uint_as_float(v[e + 2]),
                              __uint_as_float(v[e + 3]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
    if (cs > 1) fence_proxy_async_smem();  // red is read by bulk copies below
  }

  // ---------------------------------------------------------------- output
  const int my_r0 = min(kTcBM, ks * L.rpr), my_r1 = min(kTcBM, my_r0 + L.rpr);
  auto write_row_range = [&](int r0, int r1, auto&& value) {
    const int w = p.z_width;
    if (p.z_f32 && (w & 3) == 0 && (p.ldz & 3) == 0 && (reinterpret_cast<uintptr_t>(p.z) & 15) == 0) {
      // four columns per thread, 16-byte stores
      const int w4 = w >> 2;
      for (int idx = threadIdx.x; idx < (r1 - r0) * w4; idx += kTcThreads) {
        const int lr = idx / w4, j = (idx - lr * w4) * 4;
        const int row = r0 + lr;
        if (row >= ntok) continue;
        const int ti = tb.row_tile[row];
        const int r = ti >= 0 ? tb.r[ti] : 0;
        float4 v;
        v.x = j < r ? p.scale * value(lr, j) : 0.f;
        v.y = j + 1 < r ? p.scale * value(lr, j + 1) : 0.f;
        v.z = j + 2 < r ? p.scale * value(lr, j + 2) : 0.f;
        v.w = j + 3 < r ? p.scale * value(lr, j + 3) : 0.f;
        *reinterpret_cast<float4*>(static_cast<float*>(p.z) + static_cast<int64_t>(t0 + row) * p.ldz + j) = v;
      }
      return;
    }
    for (int idx = threadIdx.x; idx < (r1 - r0) * w; idx += kTcThreads) {
      const int lr = idx / w, j = idx - lr * w;
      const int row = r0 + lr;
      if (row >= ntok) continue;
      const int ti = tb.row_tile[row];
      const int r = ti >= 0 ? tb.r[ti] : 0;
      const float v = j < r ? p.scale * value(lr, j) : 0.f;
      const int64_t off = static_cast<int64_t>(t0 + row) * p.ldz + j;
      if (p.z_f32)
        static_cast<float*>(p.z)[off] = v;
      else
        static_cast<T*>(p.z)[off] = from_f32<T>(v);
    }
  };
  if (cs == 1) {
    __syncthreads();
    write_row_range(0, kTcBM, [&](int lr, int j) { return red[lr * rs + j]; });
  } else {
    __syncwarp();
    cluster_sync_all();  // every CTA's results are in red and every mainloop is over
    if (threadIdx.x < cs && threadIdx.x != ks) {
      const int o = threadIdx.x;
      const int q0 = min(kTcBM, o * L.rpr), q1 = min(kTcBM, q0 + L.rpr);
      if (q1 > q0) {
        const int slot = ks < o ? ks : ks - 1;
        bulk_push_to_peer(mapa_shared(smem_u32(smem) + static_cast<uint32_t>(slot * L.slice_bytes), static_cast<uint32_t>(o)),
                          red + q0 * rs, static_cast<uint32_t>((q1 - q0) * rs * 4),
                          mapa_shared(smem_u32(rpull), static_cast<uint32_t>(o)));
      }
    }
    const bool got = mbar_wait_bounded(rpull, 0, abort_flag, p.err, kDevErrTimeoutFull);
    const float* rst = reinterpret_cast<const float*>(smem);
    if (got)
      write_row_range(my_r0, my_r1, [&](int lr, int j) {
        float sum = 0.f;
        for (int s = 0; s < cs; ++s)
          sum += (s == ks) ? red[(my_r0 + lr) * rs + j] : rst[(s < ks ? s : s - 1) * (L.slice_bytes / 4) + lr * rs + j];
        return sum;
      });
    __syncwarp();
    cluster_sync_all();  // every push has landed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

namespace {

bool encode_map_tc(CUtensorMap* map, const void* ptr, int dtype, uint64_t inner, uint64_t outer, uint64_t ld_elems,
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

inline bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

template <typename T>
int launch_tc_t(const CUtensorMap& tx, const TcAMaps& ta, const SgmvTcArgs& p, dim3 grid, size_t smem,
                cudaStream_t s) {
  auto kernel = sgmv_shrink_tc_kernel<T>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return LORA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = grid.y;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, tx, ta, p) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

}  // namespace

int launch_sgmv_shrink_tc(const void* x, int64_t ldx, const void* a_flat, int64_t lda, int64_t a_rows,
                          const int64_t* offsets, const int64_t* ranks, const int32_t* tiles, void* z, int64_t ldz,
                          int z_dtype, int64_t z_width, int64_t T, int64_t K, int64_t r_max, float scale, int dtype,
                          int num_sms, int* err, void* stream) {
  if (r_max <= 0 || r_max > 128 || T <= 0 || K <= 0 || a_rows <= 0 || a_rows > INT32_MAX) return LORA_ERR_UNSUPPORTED;
  if (K % 8 != 0 || ldx % 8 != 0 || lda % 8 != 0 || !al16(x) || !al16(a_flat)) return LORA_ERR_UNSUPPORTED;
  if (z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  const int rmax16 = static_cast<int>((r_max + 15) / 16 * 16);
  const int num_kb = static_cast<int>((K + kTcBK - 1) / kTcBK);
  const int64_t nblk = (T + kTcBM - 1) / kTcBM;
  // K split: one wave of one CTA per SM, at least 4 k-blocks per slice, <= 8 (cluster size)
  int split = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_sms / std::max<int64_t>(nblk, 1), 8)));
  split = std::max(1, std::min(split, std::max(1, num_kb / 4)));
  const int kb_per = (num_kb + split - 1) / split;
  split = (num_kb + kb_per - 1) / kb_per;
  // the stage ring takes what the result rows, the table and the barriers leave
  const int ring = (227 * 1024 - (TcLayout(0, rmax16, split).bytes)) & ~2047;
  const TcLayout L(ring, rmax16, split);
  // a pass holds as many adapter rows as two stages of the ring can carry
  const int pass_cap = std::min(kTcPassMax, ((ring / 2 - kTcXBytes) / 128) & ~15);
  if (L.bytes > 227 * 1024 || L.slice_bytes * (split - 1) > L.ring || pass_cap < 128) return LORA_ERR_UNSUPPORTED;
  if (nblk > INT32_MAX) return LORA_ERR_SHAPE;

  CUtensorMap tx;
  TcAMaps ta;
  if (!encode_map_tc(&tx, x, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(T), static_cast<uint64_t>(ldx),
                     kTcBK, kTcBM))
    return LORA_ERR_CUDA;
  // a_flat [a_rows, K]: one box of r16 rows at each tile's first row; rows past
  // the table read as zeros, rows of the next adapter only reach discarded columns
  for (int h = 0; h < 8; ++h)
    if (!encode_map_tc(&ta.m[h], a_flat, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(a_rows),
                       static_cast<uint64_t>(lda), kTcBK, static_cast<uint32_t>(16 * (h + 1))))
      return LORA_ERR_CUDA;
  SgmvTcArgs p{};
  p.z = z;
  p.offsets = offsets;
  p.ranks = ranks;
  p.tiles = tiles;
  p.err = err;
  p.ldz = ldz;
  p.T = static_cast<int>(T);
  p.K = static_cast<int>(K);
  p.R = static_cast<int>(r_max);
  p.z_width = static_cast<int>(z_width);
  p.z_f32 = z_dtype == LORA_F32 ? 1 : 0;
  p.num_kb = num_kb;
  p.kb_per = kb_per;
  p.split = split;
  p.ring = ring;
  p.pass_cap = pass_cap;
  p.rmax16 = rmax16;
  p.scale = scale;
  dim3 grid(static_cast<unsigned>(nblk), static_cast<unsigned>(split), 1);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LORA_BF16) return launch_tc_t<__nv_bfloat16>(tx, ta, p, grid, L.bytes, s);
  return launch_tc_t<__half>(tx, ta, p, grid, L.bytes, s);
}

}  // namespace lora
