// Decode-shaped full LoRA linear (M <= 64 tokens):
//
//   out[M,N] = x . W^T + scale * z . B^T + bias
//
// The cost is streaming W ([N,K], e.g. 90 MB for Llama-7B up_proj) once, so
// the kernel is organised around HBM bandwidth:
//   - CTA = 4 warps = 64 rows of W, K split over blockIdx.y so that
//     (N/64) x split_k CTAs cover every SM several times;
//   - each warp streams its 16 W rows with 16-byte no-L1-allocate loads, 4
//     K-steps of 64 in flight, and multiplies them against the token slice
//     staged in shared memory with mma.sync m16n8k16 in swap-AB form (W rows
//     are the 16-row operand, tokens the 8-column operand);
//   - the LoRA expand is one more K-slice on the last split: [x | s.z] against
//     [W | B], so the output is written once (the decode analogue of the
//     reference's K-concat, fused_linear.py:622-677).  s.z is staged as a
//     bf16/f16 hi/lo pair against B twice, so the expand keeps ~16 mantissa
//     bits of z (the reference rounds z to the input dtype first,
//     decode_linear.py:42-44; pass z already rounded to reproduce that);
//   - splits write fp32 partials; the last CTA of a row block (atomic
//     ticket) sums them in split order and adds the bias, then returns the
//     ticket to zero (fixed counter region at the start of the workspace).
// When z is produced by the kernel right before this one, programmatic
// dependent launch lets W streaming start before z is ready: z is only read
// after griddepcontrol.wait.
// Reference: _decode_linear_kernel / decode_lora_linear (decode_linear.py:13-100).
#include <algorithm>

#include "common.cuh"
#include "runtime.h"
#include "skinny.h"

namespace lora {

struct DecodeArgs {
  const void* x;
  const void* w;
  const void* z;
  const void* b;
  const void* bias;
  void* out;
  float* partial;  // [split_k][M][N]
  int* counters;   // one per 64-row block
  int* err;
  int64_t ldx, ldw, ldz, ldb, ldo;
  int M, N, K, R, r16;
  int split_k, kslice;  // kslice multiple of 64
  float scale;
};

template <bool ALIGNED, typename T, int TG>
__global__ void __launch_bounds__(128) decode_kernel(const DecodeArgs p) {
  extern __shared__ uint8_t smem_raw[];
  T* xs = reinterpret_cast<T*>(smem_raw);
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int ks = blockIdx.y;
  const int k0 = ks * p.kslice;
  const int k1 = min(p.K, k0 + p.kslice);
  const bool last_split = (ks == p.split_k - 1);
  const bool has_tail = last_split && p.R > 0;
  const int kmain = ((k1 - k0) + 63) & ~63;               // main columns in xs (64-padded)
  const int kcols = kmain + (has_tail ? ((2 * p.r16 + 63) & ~63) : 0);
  const int xstride = kcols + 8;
  const int n_row0 = blockIdx.x * 64 + warp * 16;
  const T* x = static_cast<const T*>(p.x);
  const T* w = static_cast<const T*>(p.w);

  // Launched with programmatic serialization: x (and z for the tail) may be
  // written by the kernel launched just before this one, so the kernel waits
  // for it before its first global access.
  pdl_wait();

  // ---- stage x[:, k0:k1) (zero padded to TG*8 tokens and 64 columns)
  for (int idx = threadIdx.x; idx < TG * 8 * (kmain / 8); idx += blockDim.x) {
    const int m = idx / (kmain / 8);
    const int c = (idx - m * (kmain / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (m < p.M) {
      const T* row = x + static_cast<int64_t>(m) * p.ldx;
      if (ALIGNED) {
        if (k0 + c < k1) v = *reinterpret_cast<const uint4*>(row + k0 + c);
      } else {
        union { uint4 u; T e[8]; } t;
#pragma unroll
        for (int i = 0; i < 8; ++i) t.e[i] = (k0 + c + i < k1) ? row[k0 + c + i] : from_f32<T>(0.f);
        v = t.u;
      }
    }
    *reinterpret_cast<uint4*>(xs + m * xstride + c) = v;
  }
  __syncthreads();

  float acc[TG][4];
#pragma unroll
  for (int i = 0; i < TG; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  const int ra = n_row0 + g, rb = n_row0 + g + 8;
  const bool va = ra < p.N, vb = rb < p.N;
  const T* wa = w + static_cast<int64_t>(va ? ra : 0) * p.ldw;
  const T* wb = w + static_cast<int64_t>(vb ? rb : 0) * p.ldw;

  auto mma_step = [&](const uint32_t* wg, const uint32_t* wh, int kl) {
#pragma unroll
    for (int tg = 0; tg < TG; ++tg) {
      const T* xr = xs + (tg * 8 + g) * xstride + kl + 16 * q;
      const uint4 xa = *reinterpret_cast<const uint4*>(xr);
      const uint4 xb = *reinterpret_cast<const uint4*>(xr + 8);
      const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t af[4] = {wg[2 * j], wh[2 * j], wg[2 * j + 1], wh[2 * j + 1]};
        const uint32_t bf[2] = {xw[2 * j], xw[2 * j + 1]};
        mma16816<T>(acc[tg], af, bf);
      }
    }
  };

  // ---- main K slice: 4 steps of 64 in flight
  constexpr int U = 4;
  int kl = 0;
  for (; kl + U * 64 <= kmain; kl += U * 64) {
    uint4 la[U][2], lb[U][2];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int kc = k0 + kl + u * 64 + 16 * q;
      if (ALIGNED) {
        la[u][0] = (va && kc < k1) ? ldg_stream(wa + kc) : make_uint4(0, 0, 0, 0);
        la[u][1] = (va && kc + 8 < k1) ? ldg_stream(wa + kc + 8) : make_uint4(0, 0, 0, 0);
        lb[u][0] = (vb && kc < k1) ? ldg_stream(wb + kc) : make_uint4(0, 0, 0, 0);
        lb[u][1] = (vb && kc + 8 < k1) ? ldg_stream(wb + kc + 8) : make_uint4(0, 0, 0, 0);
      } else {
        union { uint4 u4; T e[8]; } t0, t1, t2, t3;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          t0.e[i] = (va && kc + i < k1) ? wa[kc + i] : from_f32<T>(0.f);
          t1.e[i] = (va && kc + 8 + i < k1) ? wa[kc + 8 + i] : from_f32<T>(0.f);
          t2.e[i] = (vb && kc + i < k1) ? wb[kc + i] : from_f32<T>(0.f);
          t3.e[i] = (vb && kc + 8 + i < k1) ? wb[kc + 8 + i] : from_f32<T>(0.f);
        }
        la[u][0] = t0.u4; la[u][1] = t1.u4; lb[u][0] = t2.u4; lb[u][1] = t3.u4;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t wg[8] = {la[u][0].x, la[u][0].y, la[u][0].z, la[u][0].w,
                              la[u][1].x, la[u][1].y, la[u][1].z, la[u][1].w};
      const uint32_t wh[8] = {lb[u][0].x, lb[u][0].y, lb[u][0].z, lb[u][0].w,
                              lb[u][1].x, lb[u][1].y, lb[u][1].z, lb[u][1].w};
      mma_step(wg, wh, kl + u * 64);
    }
  }
  for (; kl < kmain; kl += 64) {
    const int kc = k0 + kl + 16 * q;
    uint4 a0, a1, b0, b1;
    if (ALIGNED) {
      a0 = (va && kc < k1) ? ldg_stream(wa + kc) : make_uint4(0, 0, 0, 0);
      a1 = (va && kc + 8 < k1) ? ldg_stream(wa + kc + 8) : make_uint4(0, 0, 0, 0);
      b0 = (vb && kc < k1) ? ldg_stream(wb + kc) : make_uint4(0, 0, 0, 0);
      b1 = (vb && kc + 8 < k1) ? ldg_stream(wb + kc + 8) : make_uint4(0, 0, 0, 0);
    } else {
      union { uint4 u4; T e[8]; } t0, t1, t2, t3;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        t0.e[i] = (va && kc + i < k1) ? wa[kc + i] : from_f32<T>(0.f);
        t1.e[i] = (va && kc + 8 + i < k1) ? wa[kc + 8 + i] : from_f32<T>(0.f);
        t2.e[i] = (vb && kc + i < k1) ? wb[kc + i] : from_f32<T>(0.f);
        t3.e[i] = (vb && kc + 8 + i < k1) ? wb[kc + 8 + i] : from_f32<T>(0.f);
      }
      a0 = t0.u4; a1 = t1.u4; b0 = t2.u4; b1 = t3.u4;
    }
    const uint32_t wg[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t wh[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    mma_step(wg, wh, kl);
  }

  // ---- LoRA tail on the last split: [hi(s.z) | lo(s.z)] against [B | B]
  if (has_tail) {
    const int r16 = p.r16;
    const int tcols = (2 * r16 + 63) & ~63;
    __syncthreads();
    for (int idx = threadIdx.x; idx < TG * 8 * r16; idx += blockDim.x) {
      const int m = idx / r16, j = idx - m * r16;
      float v = 0.f;
      if (m < p.M && j < p.R) {
        if (p.ldz < 0) v = static_cast<const float*>(p.z)[static_cast<int64_t>(m) * (-p.ldz) + j];
        else v = to_f32(static_cast<const T*>(p.z)[static_cast<int64_t>(m) * p.ldz + j]);
      }
      v *= p.scale;
      const T hi = from_f32<T>(v);
      xs[m * xstride + kmain + j] = hi;
      xs[m * xstride + kmain + r16 + j] = from_f32<T>(v - to_f32(hi));
    }
    for (int idx = threadIdx.x; idx < TG * 8 * (tcols - 2 * r16); idx += blockDim.x) {
      const int m = idx / (tcols - 2 * r16), j = idx - m * (tcols - 2 * r16);
      xs[m * xstride + kmain + 2 * r16 + j] = from_f32<T>(0.f);
    }
    __syncthreads();
    const T* bsrc = static_cast<const T*>(p.b);
    for (int kt = 0; kt < tcols; kt += 64) {
      uint32_t wg[8], wh[8];
      const int kc = kt + 16 * q;
      union { uint4 u4[2]; T e[16]; } ua, ub;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int c = kc + i;
        const int j = c < r16 ? c : c - r16;  // both halves multiply the same B columns
        const bool vj = c < 2 * r16 && j < p.R;
        ua.e[i] = (va && vj) ? bsrc[static_cast<int64_t>(ra) * p.ldb + j] : from_f32<T>(0.f);
        ub.e[i] = (vb && vj) ? bsrc[static_cast<int64_t>(rb) * p.ldb + j] : from_f32<T>(0.f);
      }
      wg[0] = ua.u4[0].x; wg[1] = ua.u4[0].y; wg[2] = ua.u4[0].z; wg[3] = ua.u4[0].w;
      wg[4] = ua.u4[1].x; wg[5] = ua.u4[1].y; wg[6] = ua.u4[1].z; wg[7] = ua.u4[1].w;
      wh[0] = ub.u4[0].x; wh[1] = ub.u4[0].y; wh[2] = ub.u4[0].z; wh[3] = ub.u4[0].w;
      wh[4] = ub.u4[1].x; wh[5] = ub.u4[1].y; wh[6] = ub.u4[1].z; wh[7] = ub.u4[1].w;
      mma_step(wg, wh, kmain + kt);
    }
  }

  // ---- outputs: acc[tg][0..1] = (row g, tokens tg*8+2q, +1), acc[tg][2..3] = row g+8
  T* out = static_cast<T*>(p.out);
  const T* bias = static_cast<const T*>(p.bias);
  if (p.split_k == 1) {
#pragma unroll
    for (int tg = 0; tg < TG; ++tg) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int n = (e < 2) ? ra : rb;
        const int m = tg * 8 + 2 * q + (e & 1);
        if (n < p.N && m < p.M) {
          float v = acc[tg][e];
          if (bias != nullptr) v += to_f32(bias[n]);
          out[static_cast<int64_t>(m) * p.ldo + n] = from_f32<T>(v);
        }
      }
    }
    return;
  }
#pragma unroll
  for (int tg = 0; tg < TG; ++tg) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int n = (e < 2) ? ra : rb;
      const int m = tg * 8 + 2 * q + (e & 1);
      if (n < p.N && m < p.M) p.partial[(static_cast<int64_t>(ks) * p.M + m) * p.N + n] = acc[tg][e];
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&p.counters[blockIdx.x], 1) == p.split_k - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int nb = blockIdx.x * 64;
  for (int idx = threadIdx.x; idx < p.M * 64; idx += blockDim.x) {
    const int m = idx / 64, n = nb + (idx & 63);
    if (n >= p.N) continue;
    float v = 0.f;
    for (int s = 0; s < p.split_k; ++s) v += __ldcg(&p.partial[(static_cast<int64_t>(s) * p.M + m) * p.N + n]);
    if (bias != nullptr) v += to_f32(bias[n]);
    out[static_cast<int64_t>(m) * p.ldo + n] = from_f32<T>(v);
  }
  if (threadIdx.x == 0) p.counters[blockIdx.x] = 0;
}

namespace {
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int decode_kslice_cap(int64_t M) {
  // keep the staged token slice <= 64 KB: (8*TG tokens) x kslice x 2 bytes
  const int64_t tok = ((M + 7) / 8) * 8;
  int64_t cap = (64 * 1024) / (tok * 2);
  cap = (cap / 64) * 64;
  return static_cast<int>(std::max<int64_t>(cap, 64));
}

template <bool AL, typename T, int TG>
int launch_decode_tg(const DecodeArgs& p, dim3 grid, size_t smem, cudaStream_t s) {
  auto kernel = decode_kernel<AL, T, TG>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
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

template <bool AL, typename T>
int launch_decode_al(int tg, const DecodeArgs& p, dim3 grid, size_t smem, cudaStream_t s) {
  switch (tg) {
    case 1: return launch_decode_tg<AL, T, 1>(p, grid, smem, s);
    case 2: return launch_decode_tg<AL, T, 2>(p, grid, smem, s);
    case 4: return launch_decode_tg<AL, T, 4>(p, grid, smem, s);
    case 8: return launch_decode_tg<AL, T, 8>(p, grid, smem, s);
    default: return LORA_ERR_UNSUPPORTED;
  }
}

int decode_pick_split_k_impl(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int64_t blocks = (N + 63) / 64;
  const int64_t steps = (K + 63) / 64;
  const int cap = decode_kslice_cap(M);
  int64_t sk_min = (K + cap - 1) / cap;
  int64_t sk = (3 * static_cast<int64_t>(num_sms) + blocks - 1) / blocks;
  sk = std::max(sk, sk_min);
  sk = std::min<int64_t>(sk, std::max<int64_t>(steps, 1));
  return static_cast<int>(std::max<int64_t>(sk, 1));
}
}  // namespace

}  // namespace lora

using namespace lora;

namespace {
inline size_t round256(size_t v) { return (v + 255) / 256 * 256; }
}  // namespace

extern "C" size_t lora_decode_workspace_size(int64_t M, int64_t N, int split_k) {
  if (M <= 0 || N <= 0 || split_k <= 1) return 256;
  const size_t partial = static_cast<size_t>(split_k) * M * N * sizeof(float);
  return kCounterBytes + round256(partial);
}

extern "C" int lora_decode_pick_split_k(int64_t M, int64_t N, int64_t K) {
  const int dev = current_device();
  const int sms = dev >= 0 ? device_info(dev).num_sms : 148;
  if (M > 64) return 1;  // only the tensor-core path, which needs no workspace, takes M > 64
  return decode_pick_split_k_impl(M, N, K, sms > 0 ? sms : 148);
}

extern "C" int lora_decode_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                                  int z_dtype, const void* b, int64_t ldb, const void* bias, void* out, int64_t ldo,
                                  int64_t M, int64_t N, int64_t K, int64_t R, float scale, int dtype, int split_k,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (x == nullptr || w == nullptr || out == nullptr) return LORA_ERR_ARG;
  if (R > 0 && (z == nullptr || b == nullptr)) return LORA_ERR_ARG;
  if (dtype != LORA_BF16 && dtype != LORA_F16) return LORA_ERR_DTYPE;
  if (R > 0 && z_dtype != LORA_F32 && z_dtype != dtype) return LORA_ERR_DTYPE;
  if (M < 0 || N < 0 || K < 0 || R < 0 || M > kSkinnyMaxM || R > 128) return LORA_ERR_SHAPE;
  if (N > INT32_MAX || K > INT32_MAX || ldx < K || ldw < K || ldo < N) return LORA_ERR_SHAPE;
  if (R > 0 && (ldz < R || ldb < R)) return LORA_ERR_SHAPE;
  if (M == 0 || N == 0) return LORA_OK;
  const int dev = current_device();
  if (dev < 0 || !device_info(dev).is_sm100) return LORA_ERR_DEVICE;
  const DeviceInfo& info = device_info(dev);
  {
    // Tensor-core path: TMA-fed tcgen05 with the K split over a cluster (skinny_tc.cu).
    const int rc = launch_skinny_linear(x, ldx, w, ldw, z, ldz, z_dtype == LORA_F32 ? 1 : 0, nullptr, 0, b, ldb, bias,
                                        out, ldo, M, N, K, R, scale, dtype, split_k, info.num_sms, info.smem_per_sm,
                                        info.err_word, stream);
    if (rc != LORA_ERR_UNSUPPORTED) return rc;
  }
  if (M > 64) return LORA_ERR_SHAPE;  // the register-path kernel below covers M <= 64
  if (split_k <= 0) split_k = decode_pick_split_k_impl(M, N, K, info.num_sms);
  const int cap = decode_kslice_cap(M);
  const int64_t steps = std::max<int64_t>((K + 63) / 64, 1);
  int64_t per = (steps + split_k - 1) / split_k;
  int kslice = static_cast<int>(std::min<int64_t>(per * 64, cap));
  if (kslice <= 0) kslice = 64;
  split_k = static_cast<int>(std::max<int64_t>((K + kslice - 1) / kslice, 1));
  const int tg_need = static_cast<int>((M + 7) / 8);
  const int tg = tg_need <= 1 ? 1 : (tg_need <= 2 ? 2 : (tg_need <= 4 ? 4 : 8));
  DecodeArgs p{};
  p.x = x;
  p.w = w;
  p.z = z;
  p.b = b;
  p.bias = bias;
  p.out = out;
  p.err = info.err_word;
  p.ldx = ldx;
  p.ldw = ldw;
  p.ldz = (z_dtype == LORA_F32) ? -ldz : ldz;  // sign carries the z dtype
  p.ldb = ldb;
  p.ldo = ldo;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.R = static_cast<int>(R);
  p.r16 = static_cast<int>((R + 15) / 16 * 16);
  p.split_k = split_k;
  p.kslice = kslice;
  p.scale = scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (split_k > 1) {
    const size_t need = lora_decode_workspace_size(M, N, split_k);
    if (workspace == nullptr || workspace_bytes < need || !al16(workspace)) return LORA_ERR_WORKSPACE;
    if ((N + 63) / 64 > kMaxCounters) return LORA_ERR_SHAPE;
    p.counters = static_cast<int*>(workspace);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
  }
  const int64_t tail_cols = R > 0 ? (2 * p.r16 + 63) / 64 * 64 : 0;
  const size_t smem = static_cast<size_t>(tg * 8) * (kslice + tail_cols + 8) * 2;
  const bool aligned = (K % 8 == 0) && (ldx % 8 == 0) && (ldw % 8 == 0) && al16(x) && al16(w);
  const int64_t blocks = (N + 63) / 64;
  if (split_k > 65535) return LORA_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(split_k));
  if (dtype == LORA_BF16)
    return aligned ? launch_decode_al<true, __nv_bfloat16>(tg, p, grid, smem, s)
                   : launch_decode_al<false, __nv_bfloat16>(tg, p, grid, smem, s);
  return aligned ? launch_decode_al<true, __half>(tg, p, grid, smem, s)
                 : launch_decode_al<false, __half>(tg, p, grid, smem, s);
}
