// Peer-memory communication kernels (NVLink P2P / NVSwitch) for tensor and expert parallelism.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {
constexpr int kMaxRanks = 8;
constexpr int kMaxArBlocks = 128;
}  // namespace rz
