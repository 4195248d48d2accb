// Split-K CTA-pair LoRA linear (gemm_split.cu): outputs with too few 256x256
// tiles to fill the machine, K split over the CTA pairs of a cluster and the
// partial tiles exchanged through an L2-resident workspace.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

namespace lora {

constexpr int kSplitMaxRank = 64;  // fused shrink: lora_A rows held in the second accumulator

// Workspace the split kernel may need for this shape (0 if it never runs it).
size_t split_pair_workspace_bytes(int64_t M, int64_t N, int64_t R);

// out = x . W^T + bias + scale * (x . A^T) . B^T with the shrink accumulated
// beside the base tile and the expand applied to each owned column slice in
// fp32 (A = lora_A [R, K], B = lora_B [N, R] with row pitch ldb, R <= 64;
// R == 0: the plain linear).  Returns LORA_ERR_UNSUPPORTED when the shape,
// alignment or workspace is outside this kernel, or another kernel fits it
// better.
int launch_linear_split(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* a, int64_t lda,
                        const void* b, int64_t ldb, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                        int64_t K, int64_t R, float scale, int dtype, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream);

}  // namespace lora
