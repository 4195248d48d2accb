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
  int r16, fuse;  // fused shrink: lora_A rows per stage (R rounded to 16), on/off
  int rotate;    // start each band's K slice at a different k-block
  int kgroup;    // stages filled together (W boxes interleaved across their k-blocks)
  int box_rows;  // rows per W box
  int early;     // signal dependents at the start (forms without a z input); every form loads the
                 // weights of its first stages before griddepcontrol.wait, x and every global write after it
  float scale;
};

// Returns LORA_ERR_UNSUPPORTED when the shape or alignment is outside this
// kernel's domain (the caller then uses the register-path decode kernel).
// z given (a == NULL), or the shrink fused into the kernel (a = lora_A [R, K], z unused).
int launch_skinny_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* z, int64_t ldz,
                         int z_f32, const void* a, int64_t lda, const void* b, int64_t ldb, const void* bias,
                         void* out, int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t R, float scale, int dtype,
                         int split, int num_sms, int smem_per_sm, int* err, void* stream);
int skinny_pick_split(int64_t M, int64_t N, int64_t K, int64_t R, int num_sms, int smem_per_sm);

}  // namespace lora
