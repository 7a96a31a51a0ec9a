// Scale-block metadata and tile-schedule builder (device side).
//
// Restates build_wgrad_scale_block_meta (src/sm90_fp8_wgrad/block_meta.py:252-349)
// and its packed-layout helper _build_wgmma_layout_cpu (block_meta.py:181-212)
// as one single-CTA CUDA kernel, so building metadata needs no host loop:
//   counts[e]            = cu[e+1] - cu[e]                      (:274)
//   blocks_per_expert[e] = ceil(counts[e] / 128)                (:278)
//   block_offsets        = exclusive prefix sum of blocks        (:279-282)
//   padded_cu_seqlens_k  = 128 * block_offsets                   (:284)
//   block_row_start[b]   = cu[e] + 128 * j   (j-th block of e)   (:288-294)
//   block_row_count[b]   = min(128, cu[e] + counts[e] - row0)
//   wgmma_cu_seqlens_k   = prefix sum of ceil32(counts)          (:191-197)
//   wgmma_block_row_start[b] = wgmma_cu[e] + 128 * j             (:199-210)
//   tail_valid_rows = counts % 128, tail_wgmma_atoms = ceil(tail / 32),
//   has_tail = tail != 0, tail_copy_k = 128 if has_tail else 0 (masked128
//   policy, block_meta.py:97-99, 131-141)
// It also writes the tile-schedule order used by the grouped GEMM: experts
// sorted by descending block count (longest-processing-time first), ties kept
// in expert order. For more than LPT_MAX_EXPERTS experts the order is identity.
#include <cuda_runtime.h>
#include <cub/block/block_scan.cuh>

#include <cstdint>

#include "../../include/sm100_fp8_wgrad.h"

namespace wgrad {

namespace {

constexpr int META_THREADS = 1024;
constexpr int64_t LPT_MAX_EXPERTS = 16384;

__global__ void __launch_bounds__(META_THREADS, 1)
    build_meta_kernel(const int32_t* __restrict__ cu, int64_t num_experts, Sm100WgradMetaOut out) {
  using Scan = cub::BlockScan<long long, META_THREADS>;
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ long long carry_blocks, carry_wgmma;
  __shared__ int bad;

  const int tid = threadIdx.x;
  if (tid == 0) {
    carry_blocks = 0;
    carry_wgmma = 0;
    bad = 0;
  }
  __syncthreads();

  // Pass 1: per-expert fields and the two prefix sums.
  for (int64_t base = 0; base < num_experts; base += META_THREADS) {
    const int64_t e = base + tid;
    long long cnt = 0;
    if (e < num_experts) {
      cnt = static_cast<long long>(cu[e + 1]) - static_cast<long long>(cu[e]);
      if (cnt < 0) {
        atomicExch(&bad, 1);
        cnt = 0;
      }
    }
    const long long blocks = (cnt + 127) / 128;
    const long long wg = ((cnt + 31) / 32) * 32;
    long long blocks_excl, wg_excl;
    Scan(scan_tmp).ExclusiveSum(blocks, blocks_excl);
    __syncthreads();
    Scan(scan_tmp).ExclusiveSum(wg, wg_excl);
    __syncthreads();
    const long long bo = carry_blocks + blocks_excl;
    const long long wo = carry_wgmma + wg_excl;
    if (e < num_experts) {
      const int tail = static_cast<int>(cnt % 128);
      out.blocks_per_expert[e] = static_cast<int32_t>(blocks);
      out.block_offsets[e] = static_cast<int32_t>(bo);
      out.padded_cu_seqlens_k[e] = static_cast<int32_t>(bo * 128);
      out.wgmma_cu_seqlens_k[e] = static_cast<int32_t>(wo);
      out.tail_valid_rows[e] = tail;
      out.tail_wgmma_atoms[e] = (tail + 31) / 32;
      out.tail_copy_k[e] = tail != 0 ? 128 : 0;
      out.has_tail[e] = tail != 0 ? 1 : 0;
    }
    __syncthreads();
    if (e == num_experts - 1 || (tid == META_THREADS - 1 && e < num_experts)) {
      carry_blocks = bo + blocks;
      carry_wgmma = wo + wg;
    }
    __syncthreads();
  }
  const long long total_blocks = carry_blocks;
  if (tid == 0) {
    out.block_offsets[num_experts] = static_cast<int32_t>(total_blocks);
    out.padded_cu_seqlens_k[num_experts] = static_cast<int32_t>(total_blocks * 128);
    out.wgmma_cu_seqlens_k[num_experts] = static_cast<int32_t>(carry_wgmma);
  }
  const bool fits = total_blocks <= out.block_capacity;
  __syncthreads();

  // Pass 2: per-block arrays (one thread per expert, looping over its blocks).
  if (fits && !bad) {
    for (int64_t e = tid; e < num_experts; e += META_THREADS) {
      const int64_t b0 = out.block_offsets[e];
      const int64_t nb = out.blocks_per_expert[e];
      const int64_t row_start = cu[e];
      const int64_t row_end = cu[e + 1];
      const int64_t wg_start = out.wgmma_cu_seqlens_k[e];
      for (int64_t j = 0; j < nb; ++j) {
        const int64_t r0 = row_start + 128 * j;
        out.block_row_start[b0 + j] = static_cast<int32_t>(r0);
        out.block_row_count[b0 + j] = static_cast<int32_t>(min(static_cast<int64_t>(128), row_end - r0));
        out.wgmma_block_row_start[b0 + j] = static_cast<int32_t>(wg_start + 128 * j);
      }
    }
  }

  // Pass 3: LPT schedule order (stable, descending block count).
  if (num_experts <= LPT_MAX_EXPERTS) {
    for (int64_t e = tid; e < num_experts; e += META_THREADS) {
      const int32_t mine = out.blocks_per_expert[e];
      int64_t rank = 0;
      for (int64_t j = 0; j < num_experts; ++j) {
        const int32_t other = out.blocks_per_expert[j];
        rank += (other > mine) || (other == mine && j < e);
      }
      out.expert_order[rank] = static_cast<int32_t>(e);
    }
  } else {
    for (int64_t e = tid; e < num_experts; e += META_THREADS) out.expert_order[e] = static_cast<int32_t>(e);
  }

  if (tid == 0) {
    out.totals[0] = static_cast<int64_t>(cu[num_experts]);
    out.totals[1] = total_blocks * 128;
    out.totals[2] = carry_wgmma;
    out.totals[3] = total_blocks;
    out.totals[4] = bad ? 1 : (fits ? 0 : 2);
  }
}

}  // namespace

cudaError_t launch_build_meta(const int32_t* cu, int64_t num_experts, const Sm100WgradMetaOut& out,
                              cudaStream_t stream) {
  build_meta_kernel<<<1, META_THREADS, 0, stream>>>(cu, num_experts, out);
  return cudaGetLastError();
}

}  // namespace wgrad
