// Host-visible declarations of the fused tensor-parallel layer-boundary kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_bf16.h"

namespace rz {

struct RsNormAgParams {
  const __nv_bfloat16* slots;          // local slot buffer [world][rs_rows][H]
  const uint32_t* rs_flag;             // local reduce-scatter flags [m tiles][n_tiles][4][world]
  int n_tiles;                         // n tiles of the producing GEMM
  int reduce;                          // 0: no reduce-scatter input, x = resid_in rows
  const __nv_bfloat16* resid_in;       // [M, H] replicated input when reduce == 0
  __nv_bfloat16* residual;             // [rs_rows, H] this rank's residual shard (in/out)
  const __nv_bfloat16* w;              // RMSNorm weight [H]
  float eps, offset;
  __nv_bfloat16* gather[kMaxTpRanks];  // every rank's gather buffer [rows, H]
  uint32_t* ag_flag[kMaxTpRanks];      // every rank's all-gather flags [rows / kAgRowBlock]
  int rank, world, M, rs_rows, H;
  const uint32_t* epoch_ptr;
  uint32_t call_idx;
  int* status;
};

int rs_norm_ag_launch(const RsNormAgParams& p, cudaStream_t st);
int tp_epoch_bump_launch(uint32_t* ep, cudaStream_t st);

}  // namespace rz
