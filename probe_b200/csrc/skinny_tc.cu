// Skinny fused LoRA linear on Blackwell tensor cores (small token counts).
//
//   out[M,N] = x[M,K] . W[N,K]^T + scale * z[M,R] . B[N,R]^T + bias[N],  M <= 256
//
// With few tokens the cost is streaming W once, so the roles of the GEMM are
// swapped: 128 rows of W are the M=128 operand of tcgen05.mma and the tokens
// (padded to NB = 16 .. 128) are its N operand.  Each CTA owns one 128-row
// band of W and one K slice; the K slices of a band are the CTAs of one
// thread-block cluster, which add their fp32 partial tiles through
// distributed shared memory in rank order -- no workspace, no atomics,
// deterministic.  The LoRA expand is the cluster's last K slice: one TMA tile
// of B (128 rows x 64 ranks, zero beyond R) multiplied by [hi | lo] of
// scale * z, a bf16/f16 pair the epilogue warps write into shared memory once
// z is ready (griddepcontrol.wait: z may come from the shrink launched just
// before this kernel), so W streaming overlaps the shrink.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner and MMA issuer,
// warps 2..5 z staging and epilogue (tcgen05.ld of their 32 TMEM lanes).
// Every wait is bounded; a CTA whose wait runs out still reaches both cluster
// barriers so its peers never hang.
// Reference: _decode_linear_kernel / decode_lora_linear (decode_linear.py:13-100),
// fused_lora_linear for small M (fused_linear.py:527-551).
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "runtime.h"
#include "skinny.h"

namespace lora {

namespace {

constexpr int kSkBM = 128;  // W rows per CTA
constexpr int kSkBK = 64;   // K per stage
constexpr int kSkThreads = 192;
constexpr int kSkABytes = kSkBM * kSkBK * 2;  // 16 KB

struct SkinnyLayout {
  int nb, stages, rch;
  int b_bytes, a_off, b_off, bl_off, z_off, bar_off, bytes;
  __host__ __device__ SkinnyLayout(int nb_, int stages_, int rch_) : nb(nb_), stages(stages_), rch(rch_) {
    b_bytes = nb * kSkBK * 2;
    a_off = 0;
    b_off = stages * kSkABytes;
    bl_off = b_off + stages * b_bytes;             // [rch][128 x 64]: lora_B rows of the band
    z_off = bl_off + rch * kSkABytes;              // [rch][hi, lo][nb x 64]
    // After the mainloop the fp32 partial tile [128][nb + 4] reuses the space
    // from offset 0; the barriers sit above whichever region is larger.
    const int red_bytes = kSkBM * (nb + 4) * 4;
    const int end = z_off + rch * 2 * b_bytes;
    bar_off = ((end > red_bytes ? end : red_bytes) + 1023) & ~1023;
    bytes = bar_off + 256 + 1024;                   // barriers, tmem slot, flags + alignment slack
  }
};

}  // namespace

template <int NB, typename T>
__global__ void __launch_bounds__(kSkThreads) skinny_linear_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                   const __grid_constant__ CUtensorMap tm_x,
                                                                   const SkinnyArgs p) {
  constexpr uint32_t kTmemCols = NB < 32 ? 32 : NB;
  constexpr uint32_t kIdesc = umma_idesc_f16(kSkBM, NB, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
  constexpr int kRS = NB + 4;  // partial-tile row stride (floats)
  const SkinnyLayout L(NB, p.stages, p.rch);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + 8;
  uint64_t* acc_full = empty + 8;
  uint64_t* z_ready = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(z_ready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // Layout check (uniform over the grid, so a failing launch returns from every
  // CTA before any cluster barrier): the aligned layout must fit the allocation.
  if (static_cast<uint32_t>(smem - smem_raw) + static_cast<uint32_t>(L.bar_off) + 160u > dynamic_smem_bytes()) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrSmemLayout);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kSkBM;      // first W row (output feature)
  const int ks = blockIdx.y;              // K slice == rank in the cluster
  const int tok0 = blockIdx.z * NB;       // first token
  const int cs = p.split;
  const int kb0 = ks * p.kb_per;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per);
  const bool tail = (ks == cs - 1) && p.R > 0;
  const int n_main = max(kb1 - kb0, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < L.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(z_ready, 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool acc_ok = false;  // epilogue: the accumulator is complete

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < n_main; ++i) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, kDevErrTimeoutEmpty)) break;
        const int kb = kb0 + i;
        mbar_arrive_expect_tx(&full[stage], kSkABytes + L.b_bytes);
        tma_load_2d(&tm_w, smem + L.a_off + stage * kSkABytes, &full[stage], kb * kSkBK, n0);
        tma_load_2d(&tm_x, smem + L.b_off + stage * L.b_bytes, &full[stage], kb * kSkBK, tok0);
        if (++stage == L.stages) {
          stage = 0;
          phase ^= 1;
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
        for (int k = 0; k < 4; ++k) {
          tc_mma_f16(tmem_base, adesc + static_cast<uint64_t>(2 * k), bdesc + static_cast<uint64_t>(2 * k), kIdesc,
                     accumulate);
          accumulate = 1;
        }
        tc_commit(&empty[stage]);
        if (++stage == L.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      // LoRA tail: lora_B rows of the band against [hi | lo] of scale * z
      if (ok && tail) {
        if (!mbar_wait_bounded(z_ready, 0, abort_flag, p.err, kDevErrTimeoutFull)) ok = false;
        tc_fence_after();
        for (int c = 0; ok && c < p.rch; ++c) {
          const int nk = min(4, (p.R - c * kSkBK + 15) / 16);
          const uint64_t adesc = umma_desc_sw128(smem_u32(smem + L.bl_off + c * kSkABytes));
          const uint64_t hdesc = umma_desc_sw128(smem_u32(smem + L.z_off + (2 * c) * L.b_bytes));
          const uint64_t ldesc = umma_desc_sw128(smem_u32(smem + L.z_off + (2 * c + 1) * L.b_bytes));
          for (int k = 0; k < nk; ++k) {
            tc_mma_f16(tmem_base, adesc + static_cast<uint64_t>(2 * k), hdesc + static_cast<uint64_t>(2 * k), kIdesc,
                       accumulate);
            accumulate = 1;
            tc_mma_f16(tmem_base, adesc + static_cast<uint64_t>(2 * k), ldesc + static_cast<uint64_t>(2 * k), kIdesc,
                       1u);
          }
        }
      }
      if (ok) tc_commit(acc_full);
    }
  } else {
    // ------------------------------------------ z staging, then the epilogue
    const int et = threadIdx.x - 64;  // 0..127
    if (tail) {
      // lora_B rows n0 .. n0+128, ranks c*64 .. c*64+64 (zero beyond N and R), SW128 K-major
      const T* bsrc = static_cast<const T*>(p.b);
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
          if (p.b_vec && j0 + 8 <= p.R) {
            v.u = *reinterpret_cast<const uint4*>(src);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (j0 + e < p.R) v.e[e] = src[e];
          }
        }
        *reinterpret_cast<uint4*>(smem + L.bl_off + c * kSkABytes + row * 128 + ((ch ^ (row & 7)) << 4)) = v.u;
      }
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
        *reinterpret_cast<uint4*>(smem + L.z_off + (2 * c) * L.b_bytes + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(smem + L.z_off + (2 * c + 1) * L.b_bytes + off) =
            make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive(z_ready);
    }
    acc_ok = mbar_wait_bounded(acc_full, 0, abort_flag, p.err, kDevErrTimeoutAccFull);
    tc_fence_after();
  }

  // ---- partial tile: TMEM -> registers -> shared memory at offset 0, below bar_off
  //      (the operand buffers there are free: every TMA load was consumed by an
  //      MMA before acc_full fired)
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
  }
  if (cs > 1) {
    __syncwarp();
    cluster_sync_all();  // every partial tile of the cluster is in shared memory
    // rows [ks*rpr, ...) of the band: sum the cluster's partials in rank order
    const int rpr = (kSkBM + cs - 1) / cs;
    const int r0 = ks * rpr, r1 = min(kSkBM, r0 + rpr);
    const uint32_t red_addr = smem_u32(red);
    for (int idx = threadIdx.x; idx < (r1 - r0) * (NB / 4); idx += kSkThreads) {
      const int c4 = (idx / (r1 - r0)) * 4;
      const int row = r0 + idx % (r1 - r0);
      const int n = n0 + row;
      if (n >= p.N || tok0 + c4 >= p.M) continue;
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      const uint32_t off = red_addr + static_cast<uint32_t>((row * kRS + c4) * 4);
      for (int s = 0; s < cs; ++s) {
        const float4 v = ld_dsmem_f4(mapa_shared(off, static_cast<uint32_t>(s)));
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      const float bv = bias != nullptr ? to_f32(bias[n]) : 0.f;
      const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = tok0 + c4 + e;
        if (t < p.M) out[static_cast<int64_t>(t) * p.ldo + n] = from_f32<T>(vals[e] + bv);
      }
    }
    __syncwarp();
    cluster_sync_all();  // peers are done reading this CTA's partial tile
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
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
int ctas_per_sm(int nb, int stages, int rch, int smem_per_sm) {
  const SkinnyLayout L(nb, stages, rch);
  return std::max(1, smem_per_sm / (L.bytes + 1024));
}

// Deepest pipeline (2..4 stages) that still lets the most CTAs share an SM.
int pick_stages(int nb, int rch, int smem_per_sm) {
  int best = 2, best_ctas = ctas_per_sm(nb, 2, rch, smem_per_sm);
  for (int st = 3; st <= 4; ++st) {
    const int c = ctas_per_sm(nb, st, rch, smem_per_sm);
    if (c >= std::min(best_ctas, 3)) {
      best = st;
      best_ctas = c;
    }
  }
  return best;
}

template <int NB, typename T>
int launch_nb(const CUtensorMap& tw, const CUtensorMap& tx, const SkinnyArgs& p, dim3 grid, size_t smem,
              cudaStream_t s) {
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
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, tw, tx, p) == cudaSuccess ? LORA_OK : LORA_ERR_CUDA;
}

template <typename T>
int launch_t(int nb, const CUtensorMap& tw, const CUtensorMap& tx, const SkinnyArgs& p, dim3 grid, size_t smem,
             cudaStream_t s) {
  switch (nb) {
    case 16: return launch_nb<16, T>(tw, tx, p, grid, smem, s);
    case 32: return launch_nb<32, T>(tw, tx, p, grid, smem, s);
    case 64: return launch_nb<64, T>(tw, tx, p, grid, smem, s);
    case 128: return launch_nb<128, T>(tw, tx, p, grid, smem, s);
    default: return LORA_ERR_UNSUPPORTED;
  }
}

}  // namespace

int skinny_pick_split(int64_t M, int64_t N, int64_t K, int64_t R, int num_sms, int smem_per_sm) {
  const int nb = pick_nb(M);
  const int rch = R > 0 ? static_cast<int>((R + 63) / 64) : 0;
  const int64_t tiles = ((N + kSkBM - 1) / kSkBM) * ((M + nb - 1) / nb);
  const int64_t steps = std::max<int64_t>((K + kSkBK - 1) / kSkBK, 1);
  const int64_t slots = static_cast<int64_t>(num_sms) * ctas_per_sm(nb, pick_stages(nb, rch, smem_per_sm), rch, smem_per_sm);
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= kSkinnyMaxSplit && s <= steps; ++s) {
    const int64_t per = (steps + s - 1) / s;
    if ((steps + per - 1) / per != s) continue;  // no empty slice
    const int64_t waves = (tiles * s + slots - 1) / slots;
    const double cost = static_cast<double>(waves * (per + 3)) + 0.1 * s;  // +3: pipeline fill and reduction
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

int launch_skinny_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                         int z_f32, const void* b, int64_t ldb, const void* bias, void* out, int64_t ldo, int64_t M,
                         int64_t N, int64_t K, int64_t R, float scale, int dtype, int split, int num_sms,
                         int smem_per_sm, int* err, void* stream) {
  if (M <= 0 || M > kSkinnyMaxM || R > 128 || K <= 0) return LORA_ERR_UNSUPPORTED;
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || !al16(x) || !al16(w)) return LORA_ERR_UNSUPPORTED;
  const int nb = pick_nb(M);
  const int rch = R > 0 ? static_cast<int>((R + 63) / 64) : 0;
  const int stages = pick_stages(nb, rch, smem_per_sm);
  const SkinnyLayout L(nb, stages, rch);
  if (L.bytes > 227 * 1024) return LORA_ERR_UNSUPPORTED;
  const int num_kb = static_cast<int>((K + kSkBK - 1) / kSkBK);
  if (split <= 0) split = skinny_pick_split(M, N, K, R, num_sms, smem_per_sm);
  split = std::max(1, std::min(split, std::min(kSkinnyMaxSplit, num_kb)));
  const int kb_per = (num_kb + split - 1) / split;
  split = (num_kb + kb_per - 1) / kb_per;

  CUtensorMap tw, tx;
  if (!encode_map(&tw, w, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ldw),
                  kSkBK, kSkBM))
    return LORA_ERR_CUDA;
  if (!encode_map(&tx, x, dtype, static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(ldx),
                  kSkBK, static_cast<uint32_t>(nb)))
    return LORA_ERR_CUDA;
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
  p.scale = scale;
  const int64_t bands = (N + kSkBM - 1) / kSkBM;
  const int64_t ttiles = (M + nb - 1) / nb;
  if (bands > INT32_MAX || ttiles > 65535) return LORA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(bands), static_cast<unsigned>(split), static_cast<unsigned>(ttiles));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LORA_BF16) return launch_t<__nv_bfloat16>(nb, tw, tx, p, grid, L.bytes, s);
  return launch_t<__half>(nb, tw, tx, p, grid, L.bytes, s);
}

}  // namespace lora
