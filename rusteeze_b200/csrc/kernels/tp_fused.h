// Host-visible declarations of the fused tensor-parallel layer-boundary kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_bf16.h"

namespace rz {

constexpr int kRsNormAgMaxH = 8192;   // hidden sizes the add+RMSNorm+all-gather kernel holds in registers

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
  // MoE combine mode (moe_topk > 0): slots hold [topk][rs_rows][H] expert outputs (already
  // weighted by the gates), each row k-slot released by its own flag moe_flag[k * rs_rows + row]
  int moe_topk;
  const uint32_t* moe_flag;
  // MXFP8 output (mx != 0): the normalised rows go out as e4m3 with power-of-two 1x128
  // scales, in the block-scaled GEMM's scale-chunk layout, to every rank's gather_q
  // [rows, H] and gather_sf [row tiles][H / 128][512] instead of the bf16 gather buffer
  int mx;
  uint8_t* gather_q[kMaxTpRanks];
  uint8_t* gather_sf[kMaxTpRanks];
  uint32_t jitter_ns;                  // race testing: random pauses before stores and flags (0: off)
};

// Expert-parallel combine: every local (token, slot) pair's weighted expert output row goes
// to the token's owner, slot k, over NVLink; one release flag per written row.
struct MoeCombinePeerParams {
  const __nv_bfloat16* y;           // expert outputs (rows of the expert-sorted buffer)
  const int* pos_of;                // [M * topk] row of each pair in y, -1 if the expert is not local
  const float* topk_w;              // [M * topk]
  __nv_bfloat16* slot[kMaxTpRanks]; // every rank's slot buffer [topk][rs_rows][H]
  uint32_t* flag[kMaxTpRanks];      // every rank's moe flags [topk][rs_rows]
  int M, H, topk, rs_rows;
  const uint32_t* epoch_ptr;
  uint32_t call_idx;
  uint32_t jitter_ns;               // race testing: random pause before each flag (0: off)
};

int rs_norm_ag_launch(const RsNormAgParams& p, cudaStream_t st);
int moe_combine_peer_launch(const MoeCombinePeerParams& p, cudaStream_t st);
// waits (bounded) until the all-gather flags of rows [0, M) carry this call's epoch
int ag_wait_launch(const uint32_t* ag_flag, int M, const uint32_t* epoch_ptr, uint32_t call_idx, int* status,
                   cudaStream_t st);
int tp_epoch_bump_launch(uint32_t* ep, cudaStream_t st);

}  // namespace rz
