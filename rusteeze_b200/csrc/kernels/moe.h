// Host-visible declarations of the MoE routing / permutation / combine kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {

struct MoeRouteParams {
  const __nv_bfloat16* h;   // [M, ldh] hidden states
  int ldh;
  const __nv_bfloat16* wr;  // [E, H] router weight
  int M, H, E, topk;
  int e_lo, ne;             // local experts [e_lo, e_lo + ne)
  int renormalize;          // weights renormalised over the selected k
  float* topk_w;            // [M, topk]
  int* topk_id;             // [M, topk]
  int* counts;              // [ne], zeroed by the caller
};

struct MoePermuteParams {
  const __nv_bfloat16* h;
  int ldh;
  const int* topk_id;       // [M, topk]
  const int* counts;        // [ne]
  int M, H, topk, e_lo, ne;
  int* fill;                // [ne], zeroed by the caller
  int* grp_off;             // [ne + 1] 128-aligned segment starts (written)
  int* grp_end;             // [ne] valid-row ends (written)
  int* pos_of;              // [M * topk] row of each pair in x_perm, -1 if not local
  __nv_bfloat16* x_perm;    // [M * topk + 128 * ne, H]
};

struct MoeCombineParams {
  const __nv_bfloat16* y;   // expert outputs, row pos_of[t, k]
  int ldy;
  const int* pos_of;
  const float* topk_w;
  const __nv_bfloat16* residual;  // optional [M, H]
  __nv_bfloat16* out;       // [M, H]
  int M, H, topk;
};

int moe_route_launch(const MoeRouteParams& p, cudaStream_t st);
int moe_permute_launch(const MoePermuteParams& p, cudaStream_t st);
int moe_combine_launch(const MoeCombineParams& p, cudaStream_t st);

}  // namespace rz
