// Skinny tensor-core LoRA linear (skinny_tc.cu): small token counts, W
// streamed once through TMA, K split over the CTAs of a cluster.
#pragma once

#include <stdint.h>

namespace lora {

constexpr int kSkinnyMaxM = 256;   // tokens
constexpr int kSkinnyMaxSplit = 8; // portable cluster size

struct SkinnyArgs {
  void* out;
  const void* bias;
  const void* z;
  const void* b;
  int* err;
  int64_t ldo, ldz, ldb;
  int z_f32, b_vec;
  int M, N, R;
  int num_kb, kb_per, split, stages, rch;
  float scale;
};

// Returns LORA_ERR_UNSUPPORTED when the shape or alignment is outside this
// kernel's domain (the caller then uses the register-path decode kernel).
int launch_skinny_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                         int z_f32, const void* b, int64_t ldb, const void* bias, void* out, int64_t ldo, int64_t M,
                         int64_t N, int64_t K, int64_t R, float scale, int dtype, int split, int num_sms,
                         int smem_per_sm, int* err, void* stream);
int skinny_pick_split(int64_t M, int64_t N, int64_t K, int64_t R, int num_sms, int smem_per_sm);

}  // namespace lora
