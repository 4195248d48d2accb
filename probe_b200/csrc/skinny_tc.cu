// Skinny fused LoRA linear on Blackwell tensor cores (small token counts).
//
//   out[M,N] = x[M,K] . W[N,K]^T + scale * z[M,R] . B[N,R]^T + bias[N],  M <= 256
//   with z = x . A^T given (lora_decode_linear) or computed in the same kernel
//   (lora_linear_small: the fused shrink below)
//
// With few tokens the cost is streaming W once, so the roles of the GEMM are
// swapped: 128 rows of W are the M=128 operand of tcgen05.mma and the tokens
// (padded to NB = 16 .. 128) are its N operand.  Each CTA owns one 128-row
// band of W and one K slice; the K slices of a band are the CTAs of one
// thread-block cluster, which add their fp32 partial tiles through
// distributed shared memory in rank order -- no workspace, no atomics,
// deterministic.  With a z input the LoRA expand is the cluster's last K
// slice: the band's B rows (128 rows x 64 ranks, zero beyond R) multiplied by
// [hi | lo] of scale * z, a bf16/f16 pair the epilogue warps write into shared
// memory once z is ready (griddepcontrol.wait: z may come from the shrink
// launched just before this kernel), so W streaming overlaps the shrink.
//
// Fused shrink: every stage also brings the k-block of lora_A (r16 rows), and
// a second set of MMAs (A rows as the 128-row operand, the same x tile as the
// N operand) accumulates z^T over the CTA's K slice in a second TMEM region.
// The expand is linear in z, so every CTA of the cluster turns its own partial
// z (its K slice's share) into the [hi | lo] operand of its own tail, and the
// partial tiles the cluster adds already carry the whole expand: no z partial
// crosses the cluster and no CTA waits for another's shrink -- one kernel for
// base GEMV, shrink and expand; z never leaves the chip.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner and MMA issuer,
// warps 2..5 z staging and epilogue (tcgen05.ld of their 32 TMEM lanes).
// Every wait is bounded; a CTA whose wait runs out still reaches both cluster
// barriers so its peers never hang.
// Reference: _decode_linear_kernel / decode_lora_linear (decode_linear.py:13-100),
// fused_lora_linear for small M (fused_linear.py:527-551).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "runtime.h"
#include "gemm_split.h"
#include "skinny.h"

namespace lora {

namespace {

constexpr int kSkBM = 128;  // W rows per CTA
constexpr int kSkBK = 64;   // K per stage
constexpr int kSkThreads = 192;
constexpr int kSkABytes = kSkBM * kSkBK * 2;  // 16 KB

struct SkinnyLayout {
  int nb, stages, rch, r16, fz, cs;
  int b_bytes, at_bytes;                            // x tile, A tile (fused shrink) per stage
  int rpr, slice_bytes, zpush_bytes;                // rows per owner, partial slice pushed to an owner, z partial size
  int at_off, a_off, b_off, bl_off, z_off, rst_off, zr_off, bar_off, bytes;
  __host__ __device__ SkinnyLayout(int nb_, int stages_, int rch_, int r16_ = 0, int fz_ = 0, int cs_ = 1)
      : nb(nb_), stages(stages_), rch(rch_), r16(r16_), fz(fz_), cs(cs_) {
    b_bytes = nb * kSkBK * 2;
    at_bytes = fz ? r16 * kSkBK * 2 : 0;
    at_off = 0;                                     // [stages][r16 x 64]: lora_A rows (fused shrink)
    a_off = at_off + stages * at_bytes;             // [stages][128 x 64]: W rows of the band
    b_off = a_off + stages * kSkABytes;             // [stages][nb x 64]: x tokens
    bl_off = b_off + stages * b_bytes;              // [rch][128 x 64]: lora_B rows of the band
    // [rch][hi, lo][nb x 64]: z as the tail's operand.  Staged from global z
    // during the mainloop, it needs its own space; built from the fused shrink
    // after the mainloop, it reuses the (then idle) stage buffers at offset 0.
    const int z_bytes = rch * 2 * b_bytes;
    const bool z_alias = fz && z_bytes <= bl_off;
    z_off = z_alias ? 0 : bl_off + rch * kSkABytes;
    const int end_a = z_alias ? bl_off + rch * kSkABytes : z_off + z_bytes;  // in use during the mainloop
    // After the mainloop and the tail, every CTA writes its fp32 partial tile
    // [128][nb + 4] at offset 0 and pushes row slices to their owners, which
    // receive them in rst: (cs - 1) slices of rpr rows, above the tile.
    const int red_bytes = kSkBM * (nb + 4) * 4;
    rpr = ((kSkBM + cs - 1) / cs + 7) & ~7;  // multiple of 8: 16-byte output stores
    slice_bytes = rpr * (nb + 4) * 4;
    rst_off = (red_bytes + 1023) & ~1023;
    const int rst_end = rst_off + (cs - 1) * slice_bytes;
    // Fused shrink: this CTA's z partial (zr), written after its own mainloop
    // but while other CTAs' mainloops (and their pushes into rst) may still
    // run, so above everything the mainloop and rst use.  [r16][nb + 4]
    // (lora_A rows as the MMA's M), or [128][r16 + 4] with 128-token tiles.
    const int zr_floats = nb == 128 ? kSkBM * (r16 + 4) : r16 * (nb + 4);
    zpush_bytes = fz ? zr_floats * 4 : 0;
    const int zr_bytes = fz ? ((zpush_bytes + 1023) & ~1023) : 0;
    int top = end_a > rst_end ? end_a : rst_end;
    zr_off = (top + 1023) & ~1023;
    bar_off = zr_off + zr_bytes;
    bytes = bar_off + 256 + 1024;                   // barriers, tmem slot, flags + alignment slack
  }
};

}  // namespace

template <int NB, typename T>
__global__ void __launch_bounds__(kSkThreads, 1) skinny_linear_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                   const __grid_constant__ CUtensorMap tm_x,
                                                                   const __grid_constant__ CUtensorMap tm_a,
                                                                   const SkinnyArgs p) {
  constexpr int kNbc = NB < 16 ? 16 : NB;
  constexpr uint32_t kIdesc = umma_idesc_f16(kSkBM, NB, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
  constexpr int kRS = NB + 4;  // partial-tile row stride (floats)
  // Fused shrink with 128-token tiles: tokens are the MMA's 128 rows and the
  // r16 lora_A rows its N (8x less tensor work than padding A to 128 rows).
  constexpr bool kZSwap = (NB == 128);
  const SkinnyLayout L(NB, p.stages, p.rch, p.r16, p.fuse, p.split);
  const uint32_t kIdescZ = umma_idesc_f16(kSkBM, p.r16 > 0 ? p.r16 : 16, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
  const int zrs = kZSwap ? p.r16 + 4 : NB + 4;  // z-partial row stride (floats)
  const uint32_t tmem_cols = p.fuse ? (2 * kNbc <= 32 ? 32u : static_cast<uint32_t>(2 * kNbc))
                                    : (kNbc <= 32 ? 32u : static_cast<uint32_t>(kNbc));

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  // Layout check (uniform over the grid, so a failing launch returns from every
  // CTA before any cluster barrier): the aligned layout must fit the allocation.
  if (static_cast<uint32_t>(smem - smem_raw) + static_cast<uint32_t>(L.bar_off) + 160u > dynamic_smem_bytes()) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemLayout);
    return;
  }
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + 8;
  uint64_t* acc_full = empty + 8;
  uint64_t* z_ready = acc_full + 1;
  uint64_t* tail_full = z_ready + 1;
  uint64_t* rpull = tail_full + 1;  // every CTA: the other CTAs' slices of its rows have arrived
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rpull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kSkBM;      // first W row (output feature)
  const int ks = blockIdx.y;              // K slice == rank in the cluster
  const int tok0 = blockIdx.z * NB;       // first token
  const int cs = p.split;
  const int kb0 = ks * p.kb_per;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per);
  // CTAs with a LoRA tail: every K slice with the fused shrink (each expands
  // its own partial z), only the last one with a z input (the full z, once).
  const bool tail = (p.fuse || ks == cs - 1) && p.R > 0;
  const int n_main = max(kb1 - kb0, 0);
  // Bands start their K slice at different k-blocks, so the W requests in flight
  // across the grid spread over many column offsets.
  const int rot = (n_main > 0 && p.rotate) ? static_cast<int>((blockIdx.x * 5u + blockIdx.z * 3u) % n_main) : 0;
  const int stage_tx = kSkABytes + L.b_bytes + L.at_bytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(z_ready, 128);
    mbar_init(tail_full, 1);
    mbar_init(rpull, 1);
    *abort_flag = 0;
    fence_mbar_init();
    // Arm the receive barriers now: peers' bulk pushes may complete their bytes
    // before this CTA reaches its wait.
    if (cs > 1) {
      const int my_rows = min(kSkBM, (ks + 1) * L.rpr) - min(kSkBM, ks * L.rpr);
      mbar_arrive_expect_tx(rpull, static_cast<uint32_t>((cs - 1) * my_rows * kRS * 4));
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
    if (p.fuse) tma_prefetch_desc(&tm_a);
  }
  if (threadIdx.x == 0 && p.early) pdl_launch_dependents();
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (cs > 1) cluster_sync_all();  // every CTA's receive barriers exist before any push
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_z = tmem_base + static_cast<uint32_t>(kNbc);  // fused shrink accumulator
  bool acc_ok = false;  // epilogue: the accumulator is complete

  // ================================================================ phase A
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // Stages are filled kgroup at a time and W is fetched as br-row boxes
      // interleaved across the group's k-blocks (defaults: one stage, one
      // 128-row box; the interleaved forms are tuning knobs that measured
      // slower on B200).
      const int kg = p.kgroup, br = p.box_rows;
      bool ok = true;
      int i0 = 0;
      if (kg == 1) {
        // Launched behind another kernel: the weights (W, lora_A) of the first
        // stages load before the grid dependency resolves, x after it.
        const int npre = min(L.stages, n_main);
        for (int j = 0; j < npre; ++j) {
          mbar_arrive_expect_tx(&full[j], stage_tx);
          const int kb = kb0 + (j + rot < n_main ? j + rot : j + rot - n_main);
          for (int r0 = 0; r0 < kSkBM; r0 += br)
            tma_load_2d(&tm_w, smem + L.a_off + j * kSkABytes + r0 * 128, &full[j], kb * kSkBK, n0 + r0);
          if (p.fuse) tma_load_2d(&tm_a, smem + L.at_off + j * L.at_bytes, &full[j], kb * kSkBK, 0);
        }
        pdl_wait();
        for (int j = 0; j < npre; ++j) {
          const int kb = kb0 + (j + rot < n_main ? j + rot : j + rot - n_main);
          tma_load_2d(&tm_x, smem + L.b_off + j * L.b_bytes, &full[j], kb * kSkBK, tok0);
        }
        stage = npre % L.stages;
        phase = npre == L.stages ? 1u : 0u;
        i0 = npre;
      } else {
        pdl_wait();
      }
      for (int i = i0; ok && i < n_main; i += kg) {
        const int cnt = min(kg, n_main - i);
        const int st0 = stage;  // the group fills stages st0, st0+1, ... (mod stages)
        for (int j = 0; j < cnt; ++j) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], stage_tx);
          if (++stage == L.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        for (int r0 = 0; r0 < kSkBM; r0 += br)
          for (int j = 0; j < cnt; ++j) {
            const int sj = (st0 + j) % L.stages;
            const int ii = i + j;
            const int kb = kb0 + (ii + rot < n_main ? ii + rot : ii + rot - n_main);
            tma_load_2d(&tm_w, smem + L.a_off + sj * kSkABytes + r0 * 128, &full[sj], kb * kSkBK, n0 + r0);
          }
        for (int j = 0; j < cnt; ++j) {
          const int sj = (st0 + j) % L.stages;
          const int ii = i + j;
          const int kb = kb0 + (ii + rot < n_main ? ii + rot : ii + rot - n_main);
          tma_load_2d(&tm_x, smem + L.b_off + sj * L.b_bytes, &full[sj], kb * kSkBK, tok0);
          if (p.fuse) tma_load_2d(&tm_a, smem + L.at_off + sj * L.at_bytes, &full[sj], kb * kSkBK, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t accumulate = 0;
      for (int i = 0; ok && i < n_main; ++i) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, kDevErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t adesc = umma_desc_sw128(smem_u32(smem + L.a_off + stage * kSkABytes));
        const uint64_t bdesc = umma_desc_sw128(smem_u32(smem + L.b_off + stage * L.b_bytes));
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(tmem_base, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k), kIdesc,
                     (accumulate | static_cast<uint32_t>(k)) ? 1u : 0u);
        if (p.fuse) {
          const uint64_t zdesc = umma_desc_sw128(smem_u32(smem + L.at_off + stage * L.at_bytes));
          if (kZSwap) {
            // z[tokens, r16] += x[128 x 64] . A[r16 x 64]^T
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_f16(tmem_z, bdesc + static_cast<uint64_t>(2 * k), zdesc + static_cast<uint64_t>(2 * k), kIdescZ,
                         (accumulate | static_cast<uint32_t>(k)) ? 1u : 0u);
          } else {
            // z^T[A rows, tokens] += A[r16 (of 128) x 64] . x[NB x 64]^T; rows >= r16 are never read back
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_f16(tmem_z, zdesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k), kIdesc,
                         (accumulate | static_cast<uint32_t>(k)) ? 1u : 0u);
          }
        }
        accumulate = 1;
        tc_commit(&empty[stage]);
        if (++stage == L.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) tc_commit(acc_full);
    }
  } else {
    // ------------------------------------------------ epilogue warps, phase A
    const int et = threadIdx.x - 64;  // 0..127
    if (tail) {
      // lora_B rows n0 .. n0+128, ranks c*64 .. c*64+64 (zero beyond N and R), SW128 K-major.
      // 16-byte rows: every chunk is one cp.async (zero-filled past R), all in
      // flight together; other row pitches take element loads.
      const T* bsrc = static_cast<const T*>(p.b);
      if (p.b_vec) {
        for (int idx = et; idx < p.rch * kSkBM * 8; idx += 128) {
          const int c = idx / (kSkBM * 8);
          const int rem = idx - c * kSkBM * 8;
          const int row = rem >> 3, ch = rem & 7;
          const int n = n0 + row;
          const int j0 = c * kSkBK + ch * 8;
          const int nbytes = (n < p.N && j0 < p.R) ? 2 * min(8, p.R - j0) : 0;
          cp_async16(smem + L.bl_off + c * kSkABytes + row * 128 + ((ch ^ (row & 7)) << 4),
                     nbytes ? bsrc + static_cast<int64_t>(n) * p.ldb + j0 : bsrc, static_cast<uint32_t>(nbytes));
        }
        cp_async_commit();
        cp_async_wait<0>();
      } else {
        for (int idx = et; idx < p.rch * kSkBM * 8; idx += 128) {
          const int c = idx / (kSkBM * 8);
          const int rem = idx - c * kSkBM * 8;
          const int row = rem >> 3, ch = rem & 7;
          const int n = n0 + row;
          const int j0 = c * kSkBK + ch * 8;
          union {
            uint4 u;
            T e[8];
          } v;
          v.u = make_uint4(0u, 0u, 0u, 0u);
          if (n < p.N && j0 < p.R) {
            const T* src = bsrc + static_cast<int64_t>(n) * p.ldb + j0;
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (j0 + e < p.R) v.e[e] = src[e];
          }
          *reinterpret_cast<uint4*>(smem + L.bl_off + c * kSkABytes + row * 128 + ((ch ^ (row & 7)) << 4)) = v.u;
        }
      }
      if (p.fuse) fence_proxy_async_smem();  // the z path below fences once for both
      if (!p.fuse) {
        pdl_wait();  // z may be written by the kernel launched just before this one
        // [hi | lo] of scale * z for tokens tok0 .. tok0+NB, ranks c*64 .. c*64+64, SW128 K-major
        for (int idx = et; idx < p.rch * NB * 8; idx += 128) {
          const int c = idx / (NB * 8);
          const int rem = idx - c * NB * 8;
          const int row = rem >> 3, ch = rem & 7;
          const int t = tok0 + row;
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = c * kSkBK + ch * 8 + e;
            float zv = 0.f;
            if (t < p.M && j < p.R)
              zv = p.z_f32 ? static_cast<const float*>(p.z)[static_cast<int64_t>(t) * p.ldz + j]
                           : to_f32(static_cast<const T*>(p.z)[static_cast<int64_t>(t) * p.ldz + j]);
            v[e] = p.scale * zv;
          }
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const T h0 = from_f32<T>(v[2 * e]), h1 = from_f32<T>(v[2 * e + 1]);
            hw[e] = pack2<T>(to_f32(h0), to_f32(h1));
            lw[e] = pack2<T>(v[2 * e] - to_f32(h0), v[2 * e + 1] - to_f32(h1));
          }
          const uint32_t off = static_cast<uint32_t>(row * 128 + ((ch ^ (row & 7)) << 4));
          *reinterpret_cast<uint4*>(smem + L.z_off + (2 * c) * L.b_bytes + off) =
              make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(smem + L.z_off + (2 * c + 1) * L.b_bytes + off) =
              make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        mbar_arrive(z_ready);
      }
    }
    acc_ok = mbar_wait_bounded(acc_full, 0, abort_flag, p.err, kDevErrTimeoutAccFull);
    tc_fence_after();
    if (p.fuse) {
      const int quad = warp & 3;
      float* zred = reinterpret_cast<float*>(smem + L.zr_off);
      if (kZSwap) {
        // this CTA's partial z (TMEM lanes = tokens) -> zred[token][rank]
        __syncwarp();
        const int row = quad * 32 + lane;
        for (int c = 0; c < p.r16; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tmem_z + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(c), r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(zred + row * zrs + c + i) =
                make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2]),
                            __uint_as_float(r[i + 3]));
        }
      } else if (quad * 32 < p.r16) {
        // this CTA's partial z^T (TMEM lanes = lora_A rows) -> zred[rank][token]
        __syncwarp();
        const int row = quad * 32 + lane;
#pragma unroll
        for (int c = 0; c < NB; c += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tmem_z + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(c), r);
          tmem_wait_ld();
          if (row < p.r16) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
              *reinterpret_cast<float4*>(zred + row * zrs + c + i) =
                  make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2]),
                              __uint_as_float(r[i + 3]));
          }
        }
      }
      // Every epilogue warp's rows of zred are written before any thread
      // reads them in phase B.
      named_bar_sync(1, 128);
    }
  }

  // ================================================================ phase B
  if (tail) {
    if (p.fuse && warp >= 2) {
      // scale * (this K slice's partial z) -> [hi | lo] operand tiles
      const int et = threadIdx.x - 64;
      const float* zown = reinterpret_cast<const float*>(smem + L.zr_off);
      auto zsum4 = [&](int off) { return *reinterpret_cast<const float4*>(zown + off); };
      if (kZSwap) {
        // one item = token t, 8 ranks (one 16-byte chunk of the hi and of the lo tile)
        const int items = NB * p.rch * 8;
        for (int idx = et; idx < items; idx += 128) {
          const int t = idx / (p.rch * 8);
          const int j8 = (idx % (p.rch * 8)) * 8;  // first of 8 ranks
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = 0.f;
          if (j8 < p.R && tok0 + t < p.M) {
            const float4 a0 = zsum4(t * zrs + j8), a1 = zsum4(t * zrs + j8 + 4);
            v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
            v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
          }
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = (j8 + e < p.R) ? p.scale * v[e] : 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const T h0 = from_f32<T>(v[2 * e]), h1 = from_f32<T>(v[2 * e + 1]);
            hw[e] = pack2<T>(to_f32(h0), to_f32(h1));
            lw[e] = pack2<T>(v[2 * e] - to_f32(h0), v[2 * e + 1] - to_f32(h1));
          }
          const int c = j8 / kSkBK, ch = (j8 % kSkBK) >> 3;
          const uint32_t off = static_cast<uint32_t>(t * 128 + ((ch ^ (t & 7)) << 4));
          *reinterpret_cast<uint4*>(smem + L.z_off + (2 * c) * L.b_bytes + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(smem + L.z_off + (2 * c + 1) * L.b_bytes + off) =
              make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      } else {
        const int items = p.rch * kSkBK * (NB / 4);
        for (int idx = et; idx < items; idx += 128) {
          const int j = idx / (NB / 4);          // rank (0 .. rch*64)
          const int t4 = (idx % (NB / 4)) * 4;   // first of 4 tokens
          float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
          if (j < p.R) sum = zsum4(j * zrs + t4);
          const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
          const int c = j / kSkBK, jj = j % kSkBK, ch = jj >> 3, e = jj & 7;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int row = t4 + q;  // token row of the operand tile
            const float v = (tok0 + row < p.M) ? p.scale * vals[q] : 0.f;
            const T hi = from_f32<T>(v);
            const T lo = from_f32<T>(v - to_f32(hi));
            const uint32_t off = static_cast<uint32_t>(row * 128 + ((ch ^ (row & 7)) << 4) + e * 2);
            *reinterpret_cast<T*>(smem + L.z_off + (2 * c) * L.b_bytes + off) = hi;
            *reinterpret_cast<T*>(smem + L.z_off + (2 * c + 1) * L.b_bytes + off) = lo;
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(z_ready);
    }
    if (warp == 1 && lane == 0) {
      // LoRA tail: lora_B rows of the band against [hi | lo] of scale * z
      bool ok = mbar_wait_bounded(z_ready, 0, abort_flag, p.err, kDevErrTimeoutFull);
      tc_fence_after();
      for (int c = 0; ok && c < p.rch; ++c) {
        const int nk = min(4, (p.R - c * kSkBK + 15) / 16);
        const uint64_t adesc = umma_desc_sw128(smem_u32(smem + L.bl_off + c * kSkABytes));
        const uint64_t hdesc = umma_desc_sw128(smem_u32(smem + L.z_off + (2 * c) * L.b_bytes));
        const uint64_t ldesc = umma_desc_sw128(smem_u32(smem + L.z_off + (2 * c + 1) * L.b_bytes));
        for (int k = 0; k < nk; ++k) {
          tc_mma_f16(tmem_base, adesc + static_cast<uint64_t>(2 * k), hdesc + static_cast<uint64_t>(2 * k), kIdesc,
                     1u);
          tc_mma_f16(tmem_base, adesc + static_cast<uint64_t>(2 * k), ldesc + static_cast<uint64_t>(2 * k), kIdesc,
                     1u);
        }
      }
      if (ok) tc_commit(tail_full);
    }
    if (warp >= 2) {
      acc_ok = acc_ok && mbar_wait_bounded(tail_full, 0, abort_flag, p.err, kDevErrTimeoutAccFull);
      tc_fence_after();
    }
  }

  // ================================================================ phase C
  // partial tile: TMEM -> registers -> shared memory at offset 0, below zr_off
  // (the operand buffers there are free: every TMA load was consumed by an MMA
  // before acc_full fired, and the tail's operands before tail_full)
  float* red = reinterpret_cast<float*>(smem);
  const T* bias = static_cast<const T*>(p.bias);
  T* out = static_cast<T*>(p.out);
  if (warp >= 2) {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // W row within the band
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    __syncwarp();
#pragma unroll
    for (int c = 0; c < NB; c += 16) {
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(c), r);
      tmem_wait_ld();
      if (cs == 1) {
        const int n = n0 + row;
        if (acc_ok && n < p.N) {
          const float bv = bias != nullptr ? to_f32(bias[n]) : 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = tok0 + c + i;
            if (t < p.M) out[static_cast<int64_t>(t) * p.ldo + n] = from_f32<T>(__uint_as_float(r[i]) + bv);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(red + row * kRS + c + i) =
              make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2]),
                          __uint_as_float(r[i + 3]));
      }
    }
    if (cs > 1) fence_proxy_async_smem();  // the partial tile is read by bulk copies below
  }
  if (cs > 1) {
    __syncwarp();
    cluster_sync_all();  // every CTA's partial tile is written and every mainloop is over
    // Push rows [o*rpr, (o+1)*rpr) of this CTA's partial tile to owner o (slot = this rank,
    // skipping o's own), one bulk copy per owner.
    if (threadIdx.x < cs && threadIdx.x != ks) {
      const int o = threadIdx.x;
      const int q0 = min(kSkBM, o * L.rpr), q1 = min(kSkBM, q0 + L.rpr);
      if (q1 > q0) {
        const int slot = ks < o ? ks : ks - 1;
        bulk_push_to_peer(
            mapa_shared(smem_u32(smem + L.rst_off) + static_cast<uint32_t>(slot * L.slice_bytes), static_cast<uint32_t>(o)),
            red + q0 * kRS, static_cast<uint32_t>((q1 - q0) * kRS * 4), mapa_shared(smem_u32(rpull), static_cast<uint32_t>(o)));
      }
    }
    // this CTA's rows: its own partial plus the pushed slices, summed in rank order
    const int r0 = min(kSkBM, ks * L.rpr), r1 = min(kSkBM, r0 + L.rpr);
    const bool got = mbar_wait_bounded(rpull, 0, abort_flag, p.err, kDevErrTimeoutFull);
    const float* rst = reinterpret_cast<const float*>(smem + L.rst_off);
    // one item = token t, 8 consecutive features (one 16-byte store of out)
    const bool vec_out = (p.ldo % 8 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15u) == 0);
    const int groups = (r1 - r0) / 8;
    const int items = NB * groups;
    for (int idx = threadIdx.x; got && idx < items; idx += kSkThreads) {
      const int t = idx % NB;            // consecutive threads: consecutive tokens (conflict-free columns)
      const int lr = (idx / NB) * 8;     // first of 8 rows within the slice
      const int n = n0 + r0 + lr;
      if (n >= p.N || tok0 + t >= p.M) continue;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
      for (int s = 0; s < cs; ++s) {
        const float* src = (s == ks ? red + (r0 + lr) * kRS : rst + (s < ks ? s : s - 1) * (L.slice_bytes / 4) + lr * kRS) + t;
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] += src[e * kRS];
      }
      T* dst = out + static_cast<int64_t>(tok0 + t) * p.ldo + n;
      if (vec_out && n + 8 <= p.N) {
        float bv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) bv[e] = bias != nullptr ? to_f32(bias[n + e]) : 0.f;
        *reinterpret_cast<uint4*>(dst) = make_uint4(pack2<T>(v[0] + bv[0], v[1] + bv[1]), pack2<T>(v[2] + bv[2], v[3] + bv[3]),
                                                    pack2<T>(v[4] + bv[4], v[5] + bv[5]), pack2<T>(v[6] + bv[6], v[7] + bv[7]));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (n + e < p.N) dst[e] = from_f32<T>(v[e] + (bias != nullptr ? to_f32(bias[n + e]) : 0.f));
      }
    }
    __syncwarp();
    cluster_sync_all();  // every push has landed: no CTA's partial tile is read any more
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

namespace {

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

inline bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int pick_nb(int64_t M) { return M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128)); }

// CTAs of this kernel that fit one SM (shared memory bound; TMEM and threads allow more).
int ctas_per_sm(const SkinnyLayout& L, int smem_per_sm) { return std::max(1, smem_per_sm / (L.bytes + 1024)); }

struct SkinnyPlan {
  int stages, split;
};

// Pipeline depth and K split chosen together.  Measured on B200 (M = 1..256,
// W 11008 x 4096): a grid that needs a second wave costs a whole extra pass,
// two-stage pipelines stream ~20% slower than deeper ones, and beyond three
// stages depth no longer matters.  A plan's cost is therefore
//   waves x ((CTAs per SM in a wave) x (K blocks per CTA + fill) / efficiency + F)
// with F ~ 16 K-block times of prologue, reduction and epilogue per wave.

// LORA_B200_SKINNY="stages,split" pins the plan (read once; for tuning sweeps).
SkinnyPlan forced_plan() {
  static const SkinnyPlan forced = [] {
    SkinnyPlan f{0, 0};
    const char* v = std::getenv("LORA_B200_SKINNY");
    if (v != nullptr && std::sscanf(v, "%d,%d", &f.stages, &f.split) != 2) f = SkinnyPlan{0, 0};
    return f;
  }();
  return forced;
}

int tune_env(const char* name, int fallback) {
  const char* v = std::getenv(name);
  return (v != nullptr && v[0] >= '0' && v[0] <= '9') ? std::atoi(v) : fallback;
}

// Token counts above this go to the split-K CTA-pair kernel (gemm_split.cu):
// 256-token tiles read x once per 256 W rows instead of once per 128.
// LORA_B200_SPLIT_MIN_M overrides the threshold (tuning sweeps).
int split_min_rows() {
  static const int m = tune_env("LORA_B200_SPLIT_MIN_M", 128);
  return m;
}

int rotate_env() {
  static const int r = [] {
    const char* v = std::getenv("LORA_B200_SKINNY_ROTATE");
    return (v != nullptr && v[0] == '0') ? 0 : 1;
  }();
  return r;
}

SkinnyPlan plan_skinny(int nb, int rch, int r16, int fz, int64_t tiles, int64_t steps, int num_sms, int smem_per_sm,
                       int split_req) {
  const SkinnyPlan f = forced_plan();
  if (f.stages >= 2 && f.split >= 1 && SkinnyLayout(nb, f.stages, rch, r16, fz, f.split).bytes <= 227 * 1024) {
    const int s = static_cast<int>(std::min<int64_t>(std::min(f.split, kSkinnyMaxSplit), steps));
    return SkinnyPlan{std::min(f.stages, 8), s};
  }
  SkinnyPlan best{2, 1};
  double best_cost = 1e300;
  for (int st = 2; st <= 6; ++st) {
    if (SkinnyLayout(nb, st, rch, r16, fz, 1).bytes > 227 * 1024) break;
    for (int s = 1; s <= kSkinnyMaxSplit && s <= steps; ++s) {
      const SkinnyLayout L(nb, st, rch, r16, fz, s);
      if (L.bytes > 227 * 1024) continue;
      const int c = ctas_per_sm(L, smem_per_sm);
      const int64_t slots = static_cast<int64_t>(num_sms) * c;
      if (split_req > 0 && s != std::min<int64_t>(split_req, std::min<int64_t>(kSkinnyMaxSplit, steps))) continue;
      const int64_t per = (steps + s - 1) / s;
      if ((steps + per - 1) / per != s) continue;  // no empty slice
      const int64_t ctas = tiles * s;
      const int64_t waves = (ctas + slots - 1) / slots;
      const int64_t per_sm = (std::min(ctas, slots) + num_sms - 1) / num_sms;
      const double eff = st >= 3 ? 1.0 : 0.8;
      const double cost = static_cast<double>(waves) * (static_cast<double>(per_sm * (per + 2)) / eff + 16.0) +
                          0.01 * s - 0.001 * st;
      if (cost < best_cost) {
        best_cost = cost;
        best = SkinnyPlan{st, s};
      }
    }
  }
  return best;
}

template <int NB, typename T>
int launch_nb(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ta, const SkinnyArgs& p, dim3 grid,
              size_t smem, bool pdl, cudaStream_t s) {
  auto kernel = skinny_linear_kernel<NB, T>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return LORA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kSkThreads);
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
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, tw, tx, ta, p) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

template <typename T>
int launch_t(int nb, const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ta, const SkinnyArgs& p,
             dim3 grid, size_t smem, bool pdl, cudaStream_t s) {
  switch (nb) {
    case 16: return launch_nb<16, T>(tw, tx, ta, p, grid, smem, pdl, s);
    case 32: return launch_nb<32, T>(tw, tx, ta, p, grid, smem, pdl, s);
    case 64: return launch_nb<64, T>(tw, tx, ta, p, grid, smem, pdl, s);
    case 128: return launch_nb<128, T>(tw, tx, ta, p, grid, smem, pdl, s);
    default: return LORA_ERR_UNSUPPORTED;
  }
}

}  // namespace

int skinny_pick_split(int64_t M, int64_t N, int64_t K, int64_t R, int num_sms, int smem_per_sm) {
  const int nb = pick_nb(M);
  const int rch = R > 0 ? static_cast<int>((R + 63) / 64) : 0;
  const int64_t tiles = ((N + kSkBM - 1) / kSkBM) * ((M + nb - 1) / nb);
  const int64_t steps = std::max<int64_t>((K + kSkBK - 1) / kSkBK, 1);
  return plan_skinny(nb, rch, 0, 0, tiles, steps, num_sms, smem_per_sm, 0).split;
}

int launch_skinny_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                         int z_f32, const void* a, int64_t lda, const void* b, int64_t ldb, const void* bias,
                         void* out, int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t R, float scale, int dtype,
                         int split, int num_sms, int smem_per_sm, int* err, void* stream) {
  const int fuse = (R > 0 && a != nullptr) ? 1 : 0;
  if (M <= 0 || M > kSkinnyMaxM || R > 128 || K <= 0) return LORA_ERR_UNSUPPORTED;
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || !al16(x) || !al16(w)) return LORA_ERR_UNSUPPORTED;
  if (fuse && (lda % 8 != 0 || !al16(a))) return LORA_ERR_UNSUPPORTED;
  const int nb = pick_nb(M);
  const int rch = R > 0 ? static_cast<int>((R + 63) / 64) : 0;
  const int r16 = fuse ? static_cast<int>((R + 15) / 16 * 16) : 0;
  const int num_kb = static_cast<int>((K + kSkBK - 1) / kSkBK);
  const int64_t tiles = ((N + kSkBM - 1) / kSkBM) * ((M + nb - 1) / nb);
  const SkinnyPlan plan = plan_skinny(nb, rch, r16, fuse, tiles, num_kb, num_sms, smem_per_sm, split);
  const int stages = plan.stages;
  split = plan.split;
  const int kb_per = (num_kb + split - 1) / split;
  split = (num_kb + kb_per - 1) / kb_per;
  const SkinnyLayout L(nb, stages, rch, r16, fuse, split);
  if (L.bytes > 227 * 1024) return LORA_ERR_UNSUPPORTED;

  // W box rows (128: one box per k-block; smaller boxes measured slower on B200)
  const int box_rows_pre = tune_env("LORA_B200_SKINNY_BR", 128);
  const uint32_t wbox = (box_rows_pre == 8 || box_rows_pre == 16 || box_rows_pre == 32 || box_rows_pre == 64 ||
                         box_rows_pre == 128) ? static_cast<uint32_t>(box_rows_pre) : 128u;
  CUtensorMap tw, tx, ta;
  if (!encode_map(&tw, w, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ldw),
                  kSkBK, wbox))
    return LORA_ERR_CUDA;
  if (!encode_map(&tx, x, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(ldx),
                  kSkBK, static_cast<uint32_t>(nb)))
    return LORA_ERR_CUDA;
  if (fuse) {
    // lora_A [R, K]: boxes of r16 rows, rows R .. r16 filled with zeros
    if (!encode_map(&ta, a, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(R), static_cast<uint64_t>(lda),
                    kSkBK, static_cast<uint32_t>(r16)))
      return LORA_ERR_CUDA;
  } else {
    ta = tw;
  }
  SkinnyArgs p{};
  p.out = out;
  p.bias = bias;
  p.z = z;
  p.b = b;
  p.ldb = ldb;
  p.b_vec = (ldb % 8 == 0 && al16(b)) ? 1 : 0;
  p.err = err;
  p.ldo = ldo;
  p.ldz = ldz;
  p.z_f32 = z_f32;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.R = static_cast<int>(R);
  p.num_kb = num_kb;
  p.kb_per = kb_per;
  p.split = split;
  p.stages = stages;
  p.rch = rch;
  p.r16 = r16;
  p.fuse = fuse;
  p.scale = scale;
  p.rotate = rotate_env();
  p.kgroup = std::max(1, std::min(tune_env("LORA_B200_SKINNY_KG", 1), std::min(stages, 8)));
  p.box_rows = static_cast<int>(wbox);
  const int64_t bands = (N + kSkBM - 1) / kSkBM;
  const int64_t ttiles = (M + nb - 1) / nb;
  if (bands > INT32_MAX || ttiles > 65535) return LORA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(bands), static_cast<unsigned>(split), static_cast<unsigned>(ttiles));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Every form runs with programmatic serialization: the weights of the first
  // stages load before griddepcontrol.wait, x after it, and the z-consuming
  // form's epilogue waits again before reading z (the shrink launched just
  // before it).  The forms without a z input signal their own dependents at once.
  p.early = (fuse || R == 0) ? 1 : 0;
  const bool pdl = pdl_enabled();
  if (dtype == LORA_BF16) return launch_t<__nv_bfloat16>(nb, tw, tx, ta, p, grid, L.bytes, pdl, s);
  return launch_t<__half>(nb, tw, tx, ta, p, grid, L.bytes, pdl, s);
}

}  // namespace lora

using namespace lora;

extern "C" size_t lora_linear_small_workspace_size(int64_t M, int64_t N, int64_t R) {
  return M > split_min_rows() ? split_pair_workspace_bytes(M, N, R) : 0;
}

extern "C" int lora_linear_small(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* a, int64_t lda,
                                 const void* b, int64_t ldb, const void* bias, void* out, int64_t ldo, int64_t M,
                                 int64_t N, int64_t K, int64_t R, float scale, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (x == nullptr || w == nullptr || out == nullptr) return LORA_ERR_ARG;
  if (R > 0 && (a == nullptr || b == nullptr)) return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (M < 0 || N < 0 || K < 0 || R < 0 || M > kSkinnyMaxM || R > 128) return LORA_ERR_SHAPE;
  if (N > INT32_MAX || K > INT32_MAX || ldx < K || ldw < K || ldo < N) return LORA_ERR_SHAPE;
  if (R > 0 && (lda < K || ldb < R)) return LORA_ERR_SHAPE;
  if (M == 0 || N == 0) return LORA_OK;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  if (M > split_min_rows()) {  // 256-token CTA-pair tiles, K split over a cluster
    const int rc = launch_linear_split(x, ldx, w, ldw, a, lda, b, ldb, bias, out, ldo, M, N, K, scale != 0.f ? R : 0,
                                       scale, dtype, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
    if (rc != LORA_ERR_UNSUPPORTED) return rc;
  }
  return launch_skinny_linear(x, ldx, w, ldw, nullptr, 0, 0, R > 0 ? a : nullptr, lda, b, ldb, bias, out, ldo, M, N,
                              K, R, scale, dtype, 0, info.num_sms, info.smem_per_sm, info.err_word, stream);
}
