// Host-visible declarations of the tcgen05 GEMM launcher.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {

// kEpiSiluMulMx: SiLU(gate)*up written as e4m3 (q_out, row stride ldd) plus UE8M0 1x128
// scales (sf_out, [ceil(M/128)][N/256] chunks); BN = 256 only.
enum GemmEpilogue : int { kEpiNone = 0, kEpiSiluMul = 1, kEpiPeerRS = 2, kEpiSiluMulMx = 3 };
// The bindings take the epilogue with the gate activation in bit 8 of the same argument:
// epi | kGateGelu makes the gated epilogues compute GELU(tanh)(gate) * up instead of SiLU.
constexpr int kGateGelu = 1 << 8;

constexpr int kMaxTpRanks = 8;
constexpr int kAgRowBlock = 8;    // rows per all-gather flag

struct GemmParams {
  int M, N, K;
  int k_splits;        // >= 1
  int k_blocks;        // filled by the launcher
  int kb_per_split;    // filled by the launcher
  int m_tiles, n_tiles;
  __nv_bfloat16* D;    // output, leading dimension ldd
  int ldd;
  float* partial;      // [k_splits][M][N] fp32 workspace when k_splits > 1
  const __nv_bfloat16* bias;      // [N] or nullptr
  const __nv_bfloat16* residual;  // [M][ldr] or nullptr (kEpiNone only)
  int ldr;
  int epi;
  int gate_act;        // gated epilogues (kEpiSiluMul / kEpiSiluMulMx): 0 SiLU, 1 GELU (tanh)
  int* status;
  const uint8_t* sfa;  // MXFP8 only: A scales, [ceil(M/128)][K/128] chunks of 512 bytes
  const uint8_t* sfb;  // MXFP8 only: B scales, [N/128][K/128] chunks of 512 bytes
  // grouped (MoE) mode: device arrays, 128-aligned segment starts [num_groups + 1]
  // and valid-row ends [num_groups]; B is num_groups matrices of N rows
  const int* grp_off;
  const int* grp_end;
  int num_groups;
  // tensor-parallel fusion (sequence-sharded rows: rank o owns rows [o*rs_rows, (o+1)*rs_rows))
  //   kEpiPeerRS: every finished tile row is stored into its owner's slot buffer
  //     rs_slot[o] + ((tp_rank * rs_rows + local row) * N) over NVLink, then each epilogue
  //     warp releases rs_flag[o][((m_tile * n_tiles + n_tile) * 8 + quarter * 2 + column half)
  //     * tp_world + tp_rank] for its 32 rows x half the tile's columns;
  //   ag_flag != null: before loading an A tile, the producer waits for the
  //     all-gather flags of its rows (one per kAgRowBlock rows, rows < ag_rows).
  __nv_bfloat16* rs_slot[kMaxTpRanks];
  uint32_t* rs_flag[kMaxTpRanks];
  int rs_rows;
  int tp_rank, tp_world;
  const uint32_t* ag_flag;
  int ag_rows;
  const uint32_t* epoch_ptr;   // device step counter; flags carry (*epoch_ptr) * 256 + call_idx + 1
  uint32_t call_idx;
  uint8_t* q_out;              // kEpiSiluMulMx outputs
  uint8_t* sf_out;
  uint32_t jitter_ns;          // kEpiPeerRS race testing: random pauses before stores and flags (0: off)
};

constexpr int kMaxGemmGroups = 64;

struct GemmPlan {
  int bn;
  int k_splits;
  double cost;
};

GemmPlan plan_gemm(int M, int N, int K, int epi, int max_splits = 16);
__global__ void gemm_splitk_reduce(GemmParams p);
int gemm_bf16_launch(const GemmParams& p, const void* A, int lda, const void* B, int ldb, int bn,
                     cudaStream_t stream);
// Grouped GEMM over expert-sorted rows (see GemmParams::grp_off); k_splits must be 1.
int gemm_grouped_launch(const GemmParams& p, const void* A, int lda, int64_t a_rows, const void* B, int ldb,
                        int bn, bool mx, cudaStream_t stream);
// MXFP8 (e4m3 operands, UE8M0 scales per 32 K-elements): K % 128 == 0, N % 128 == 0, bn in {128, 256}.
GemmPlan plan_gemm_mxf8(int M, int N, int K, int epi, int max_splits = 16);
int gemm_mxf8_launch(const GemmParams& p, const void* A, int lda, const void* B, int ldb, int bn,
                     cudaStream_t stream);
// bf16 [M, K] (row stride ldx) -> e4m3 [M, K] + scale chunks for ceil(M/128) row blocks.
int quant_mxf8_act_launch(void* xq, uint8_t* sfa, const __nv_bfloat16* x, int M, int K, int ldx,
                          cudaStream_t stream);
int make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int elem_bytes, int64_t rows,
                 int64_t cols, int64_t ld, int box_rows, int box_cols);
int num_sms();

}  // namespace rz
