// Launch parameters shared by the grouped Wgrad kernel and its host launcher.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace wgrad {

constexpr int kMaxDevices = 64;  // device ordinals with per-device launch state

#ifndef WGRAD_PROFILE
#define WGRAD_PROFILE 0
#endif

// Slots of the per-role cycle counters (WGRAD_PROFILE builds), summed over CTAs.
enum ProfSlot : int {
  kProfProducerWaitStage = 0,   // producer: waits for a free operand stage
  kProfProducerWaitScales = 1,  // producer: waits for a free scale stage
  kProfMmaWait = 2,             // MMA warp: waits for a free TMEM buffer + a full stage
  kProfMmaIssue = 3,            // MMA warp: issuing the K block's UMMAs and commits
  kProfEpiWait = 4,             // promotion warp: waits for the partial + scales
  kProfEpiPromote = 5,          // promotion warp: TMEM loads + fp32 promotion of a K block
  kProfEpiStore = 6,            // promotion warp: BF16/fp32 staging + TMA store issue of a tile
  kProfEpiStoreWait = 7,        // promotion warp: wait for the previous tile's store to read smem
  kProfKBlocks = 8,             // count: K blocks promoted (first promotion warp)
  kProfTiles = 9,               // count: output tiles stored
  kProfCtas = 10,               // count: CTAs
  kProfSfConvert = 11,          // UE8M0 scale-factor writer: scale loads, E8M0 conversion, shared stores
  kProfSfPublish = 12,          // UE8M0 scale-factor writer: proxy fence and barrier arrivals
  kProfLoadLatency = 13,        // operand stage: producer issue -> MMA warp sees it full
  kProfSfSync = 14,             // UE8M0 scale-factor writer: warp vote after its barrier wait
  kProfSfLoad = 15,             // UE8M0 scale-factor writer: scale loads and E8M0 conversion
  kProfMmaTileWait = 16,        // UE8M0 MMA warp: wait for a free accumulator at a tile's start
  kProfCtaCycles = 17,          // whole CTA: cycles from the end of set-up to the final barrier
  kProfSlots = 24,
};

#ifndef WGRAD_DEBUG_MODES
#define WGRAD_DEBUG_MODES 0
#endif

// Known-answer kernel modes (instrumented builds only, -DWGRAD_DEBUG_MODES=1),
// selected like the reference's KERNEL_LAB_WGRAD_KERNEL_MODE (gemm_sm90.py:139-175):
//   coord_m / coord_n  out[e, m, n] = m / n            (pins the tile -> output mapping)
//   scale_only         out = 2^20 * sum_b sa[b,m] sb[b,n]  (pins scale indexing, :5271-5292)
//   unscaled           out = sum_k A[m,k] B[n,k]       (the FP8 product alone, :2820-2868)
enum KernelMode : int { kModeNormal = 0, kModeCoordM = 1, kModeCoordN = 2, kModeScaleOnly = 3, kModeUnscaled = 4 };

// Test-only failure injection (SM100_WGRAD_DEBUG_INJECT=withhold_first_load):
// the producer announces its first stage's bytes without issuing the copy.
constexpr int kInjectWithholdFirstLoad = 1;

struct GemmParams {
  const float* sa;              // lhs scales [total_blocks][m]
  const float* sb;              // rhs scales [total_blocks][n]
  void* out;                    // [E][m][n]
  const int32_t* block_offsets; // [E+1]
  const int32_t* k_row_offsets; // [E+1]
  const int32_t* expert_order;  // [E] or nullptr
  int num_experts;
  int m, n;
  int bn;                       // tile N (128, 192 or 256)
  int bm;                       // tile M: 128, or 256 for a CTA pair (cta_group::2)
  int tiles_n;
  int tiles_per_expert;
  int num_tiles;
  int out_f32;
  int accumulate;
  int has_operands;             // 0 when the operand K extent is empty
  int epi_warps;                // promotion warps: 8, or 16 (bn 256 only)
  int inject;                   // test-only failure injection (kInject*), 0 in normal use
  int mode;                     // KernelMode; only instrumented builds honour a non-zero mode
  int ue8m0;                    // 1: scales are powers of two, applied by block-scaled UMMAs (bn 192)
};

cudaError_t launch_grouped_wgrad(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                                 const GemmParams& p, int grid, cudaStream_t stream);


}  // namespace wgrad
