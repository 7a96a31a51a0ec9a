// sm100_fp8_grouped_wgrad_noalloc: the scale-product GEMM (the one kernel of
// this library that needs device scratch: the hi/lo split scales it feeds to
// its TF32 UMMA) with that scratch taken from a fixed array compiled into the
// library instead of a caller-provided workspace.
//
// For callers that cannot allocate device memory: a host binding over this
// C ABI that owns only the input and output buffers it was handed (a Go, Java
// or Rust wrapper with no CUDA allocator of its own), or a serving process that
// reserves its whole device-memory budget at start-up and forbids allocations
// afterwards. Neither can hand sm100_fp8_grouped_wgrad a workspace.
//
// The array below is a module-scope __device__ variable: every GPU that loads
// the library holds kNoAllocScratchBytes of it until the process exits. In host
// code its name is only a host-side stand-in, never a device address; the
// device address is looked up once per device with cudaGetSymbolAddress while
// that device is current, on the first call of the entry point on it (so that
// first call should come before any stream capture).
//
// Every call shares the one array, and it keeps the last call's contents.
// Calls that overlap on the GPU (different streams, or different host threads
// on the same device) race on it: serialise them. Nothing in it has to start
// at zero: each call's scale-operand kernel writes every entry the GEMM then
// reads (the split scales of the launched experts' blocks), and the GEMM's TMA
// boxes read nothing else (rows past M or N are zero-filled by the TMA unit).
//
// This entry point calls no cudaMalloc, cudaFree or other allocating routine
// (it also skips the pinned host error mirror that the other entry points set
// up: poll errors of its launches with sm100_wgrad_device_error).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/sm100_fp8_wgrad.h"
#include "wgrad_gemm.cuh"

namespace {

constexpr int64_t kNoAllocScratchBytes = 64ll << 20;  // 64 MiB per device

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device (looked up once per
// device, with that device current), or nullptr if the lookup failed.
void* noalloc_scratch_ptr() {
  static std::once_flag flags[wgrad::kMaxDevices];
  static void* ptrs[wgrad::kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= wgrad::kMaxDevices) return nullptr;
  std::call_once(flags[dev], [dev] {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) == cudaSuccess) ptrs[dev] = ptr;
    else (void)cudaGetLastError();
  });
  return ptrs[dev];
}

}  // namespace

extern "C" {

int sm100_fp8_grouped_wgrad_noalloc(const Sm100WgradArgs* a, void* stream) {
  if (a == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->out == nullptr || a->block_offsets == nullptr || a->k_row_offsets == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->num_experts < 0 || a->m <= 0 || a->n <= 0 || a->k_rows < 0 || a->total_blocks < 0)
    return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->out_dtype != SM100_WGRAD_OUT_BF16 && a->out_dtype != SM100_WGRAD_OUT_F32) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->tile_config != SM100_WGRAD_TILE_AUTO && a->tile_config != SM100_WGRAD_TILE_256x256_SP &&
      a->tile_config != SM100_WGRAD_TILE_256x256_SP_W16)
    return SM100_WGRAD_ERR_UNSUPPORTED;
  if (a->m % 16 != 0 || a->n % 16 != 0) return SM100_WGRAD_ERR_UNSUPPORTED;
  if (a->m > (1 << 30) || a->n > (1 << 30) || a->num_experts > (1 << 30)) return SM100_WGRAD_ERR_UNSUPPORTED;
  if (!aligned16(a->out)) return SM100_WGRAD_ERR_INVALID_ARG;
  const bool has_operands = a->k_rows > 0 && a->total_blocks > 0;
  if (has_operands) {
    if (a->lhs_data == nullptr || a->rhs_data == nullptr || a->lhs_scales == nullptr || a->rhs_scales == nullptr)
      return SM100_WGRAD_ERR_INVALID_ARG;
    if (a->lhs_pitch % 16 != 0 || a->rhs_pitch % 16 != 0 || a->lhs_pitch < a->k_rows || a->rhs_pitch < a->k_rows)
      return SM100_WGRAD_ERR_INVALID_ARG;
    if (!aligned16(a->lhs_data) || !aligned16(a->rhs_data) || !aligned16(a->lhs_scales) ||
        !aligned16(a->rhs_scales))
      return SM100_WGRAD_ERR_INVALID_ARG;
    // Larger problems need the caller-provided workspace of sm100_fp8_grouped_wgrad.
    if (sp_workspace_bytes(a->total_blocks, a->m, a->n) > kNoAllocScratchBytes) return SM100_WGRAD_ERR_UNSUPPORTED;
  }
  if (a->num_experts == 0) return SM100_WGRAD_OK;

  DeviceInfo info;
  int st = device_info(&info);
  if (st != SM100_WGRAD_OK) return st;
  if (info.major != 10 || info.minor != 0) return SM100_WGRAD_ERR_UNSUPPORTED_ARCH;

  const int32_t tile = a->tile_config == SM100_WGRAD_TILE_256x256_SP_W16 ? SM100_WGRAD_TILE_256x256_SP_W16
                                                                          : SM100_WGRAD_TILE_256x256_SP;
  void* opa = nullptr;
  void* opb = nullptr;
  CUtensorMap ta{}, tb{}, to{}, tsa{}, tsb{};
  if (has_operands) {
    uint8_t* scratch = static_cast<uint8_t*>(noalloc_scratch_ptr());
    if (scratch == nullptr) return SM100_WGRAD_ERR_LAUNCH;
    opa = scratch;
    opb = scratch + sp_workspace_lhs_bytes(a->total_blocks, a->m);
    st = encode_operand_map(&ta, a->lhs_data, a->k_rows, a->m, a->lhs_pitch, 128);
    if (st != SM100_WGRAD_OK) return st;
    st = encode_operand_map(&tb, a->rhs_data, a->k_rows, a->n, a->rhs_pitch, 64);
    if (st != SM100_WGRAD_OK) return st;
    st = encode_scale_operand_map(&tsa, opa, a->m, a->total_blocks, 128);
    if (st != SM100_WGRAD_OK) return st;
    st = encode_scale_operand_map(&tsb, opb, a->n, a->total_blocks, 64);
    if (st != SM100_WGRAD_OK) return st;
  }
  st = encode_out_map(&to, a->out, a->out_dtype == SM100_WGRAD_OUT_F32, a->num_experts, a->m, a->n,
                      tile == SM100_WGRAD_TILE_256x256_SP_W16);
  if (st != SM100_WGRAD_OK) return st;

  wgrad::GemmParams p{};
  p.sa = a->lhs_scales;
  p.sb = a->rhs_scales;
  p.out = a->out;
  p.block_offsets = a->block_offsets;
  p.k_row_offsets = a->k_row_offsets;
  p.expert_order = a->expert_order;
  p.num_experts = static_cast<int>(a->num_experts);
  p.m = static_cast<int>(a->m);
  p.n = static_cast<int>(a->n);
  p.bn = 256;
  p.bm = 256;
  p.tiles_n = static_cast<int>((a->n + 255) / 256);
  const int64_t tpe = ((a->m + 255) / 256) * p.tiles_n;
  const int64_t num_tiles = tpe * a->num_experts;
  if (num_tiles > INT32_MAX) return SM100_WGRAD_ERR_UNSUPPORTED;
  p.tiles_per_expert = static_cast<int>(tpe);
  p.num_tiles = static_cast<int>(num_tiles);
  p.out_f32 = a->out_dtype == SM100_WGRAD_OUT_F32;
  p.accumulate = a->accumulate != 0;
  p.has_operands = has_operands ? 1 : 0;
  p.epi_warps = tile == SM100_WGRAD_TILE_256x256_SP_W16 ? 16 : 8;
  p.mode = wgrad::kModeNormal;
  p.inject = 0;
  p.ue8m0 = 0;

  int grid = info.sm_count;
  if (a->max_ctas > 0 && a->max_ctas < grid) grid = a->max_ctas;
  if (2 * num_tiles < grid) grid = static_cast<int>(2 * num_tiles);
  grid &= ~1;
  if (grid < 2) grid = 2;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (has_operands) {
    const cudaError_t e = wgrad::launch_scale_operands(a->lhs_scales, a->rhs_scales, opa, opb, a->m, a->n,
                                                       a->block_offsets, p.num_experts, a->total_blocks,
                                                       info.sm_count, s);
    if (e != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  }
  const cudaError_t e = wgrad::launch_grouped_wgrad_sp(ta, tb, tsa, tsb, to, p, grid, s);
  return e == cudaSuccess ? SM100_WGRAD_OK : SM100_WGRAD_ERR_LAUNCH;
}

}  // extern "C"
