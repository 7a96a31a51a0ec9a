// C-ABI entry points of the grouped FP8 Wgrad engine (declared in
// include/sm100_fp8_wgrad.h). Host-side argument validation, TMA descriptor
// encoding and kernel launch; no entry point synchronises the stream.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/sm100_fp8_wgrad.h"
#include "ptx.cuh"
#include "wgrad_gemm.cuh"

namespace wgrad {
cudaError_t launch_quantize_1x128(const void* x, int x_dtype, int64_t cols, const int32_t* gather_idx,
                                  const int32_t* block_row_start, const int32_t* block_row_count,
                                  int64_t total_blocks, void* q, int64_t q_pitch, const int32_t* q_row_start,
                                  bool q_zero_fill, void* kq, int64_t kq_pitch, const int32_t* kq_row_start,
                                  float* scales, int block_rows, int64_t x_rows, bool ue8m0, cudaStream_t stream);
cudaError_t launch_build_meta(const int32_t* cu, int64_t num_experts, const Sm100WgradMetaOut& out,
                              cudaStream_t stream);
cudaError_t launch_scale_operands(const float* sa, const float* sb, void* opa, void* opb, int64_t m, int64_t n,
                                  const int32_t* block_offsets, int num_experts, int64_t total_blocks, int sm_count,
                                  cudaStream_t stream);
cudaError_t launch_grouped_wgrad_sp(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa,
                                    const CUtensorMap& tsb, const CUtensorMap& to, const GemmParams& p, int grid,
                                    cudaStream_t stream);
}  // namespace wgrad

#ifndef WGRAD_OPERAND_L2_PROMOTION
#define WGRAD_OPERAND_L2_PROMOTION CU_TENSOR_MAP_L2_PROMOTION_L2_256B
#endif

namespace {

using wgrad::GemmParams;

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  });
  return fn;
}

// Tensor maps encoded for earlier launches, keyed by every argument of the
// encoding (device, element type, rank, base address, extents, strides, box,
// swizzle, L2 promotion). A map depends only on those values, never on the
// memory's contents, so a hit is exact. A launch needs three to five maps;
// the cache saves their encoding on repeated launches over the same buffers
// (the reference caches its compiled launch per shape, gemm_sm90.py:5388-5409).
struct MapKey {
  int dev, dtype, rank, swizzle, promo;
  const void* ptr;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  bool operator==(const MapKey& o) const {
    return dev == o.dev && dtype == o.dtype && rank == o.rank && swizzle == o.swizzle && promo == o.promo &&
           ptr == o.ptr && std::memcmp(dims, o.dims, sizeof(dims)) == 0 &&
           std::memcmp(strides, o.strides, sizeof(strides)) == 0 && std::memcmp(box, o.box, sizeof(box)) == 0;
  }
};

int cached_encode(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* ptr, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swizzle,
                  CUtensorMapL2promotion promo) {
  constexpr int kSlots = 64;
  static std::mutex mu;
  static MapKey keys[kSlots];
  static CUtensorMap maps[kSlots];
  static int used = 0, next = 0;
  MapKey k{};
  if (cudaGetDevice(&k.dev) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  k.dtype = static_cast<int>(dtype);
  k.rank = rank;
  k.swizzle = static_cast<int>(swizzle);
  k.promo = static_cast<int>(promo);
  k.ptr = ptr;
  for (int i = 0; i < rank; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
    if (i + 1 < rank) k.strides[i] = strides[i];
  }
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i) {
      if (keys[i] == k) {
        *map = maps[i];
        return SM100_WGRAD_OK;
      }
    }
  }
  auto encode = get_encode_fn();
  if (encode == nullptr) return SM100_WGRAD_ERR_LAUNCH;
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = encode(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(ptr), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return SM100_WGRAD_ERR_TENSOR_MAP;
  std::lock_guard<std::mutex> lock(mu);
  keys[next] = k;
  maps[next] = *map;
  next = (next + 1) % kSlots;
  if (used < kSlots) ++used;
  return SM100_WGRAD_OK;
}

// Per-device capability check and SM count, cached.
struct DeviceInfo {
  int sm_count = 0;
  int major = 0;
  int minor = 0;
};

int device_info(DeviceInfo* info) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool have[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return SM100_WGRAD_ERR_LAUNCH;
  if (!have[dev]) {
    DeviceInfo d;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return SM100_WGRAD_ERR_LAUNCH;
    cache[dev] = d;
    have[dev] = true;
  }
  *info = cache[dev];
  return SM100_WGRAD_OK;
}

// Per-device host-mapped mirror of the device error word: one pinned word,
// mapped into the device's address space and published to the kernels'
// g_device_error_host once (a synchronous symbol copy on the first call of
// any entry point on that device, which must therefore not be inside a CUDA
// stream capture). Null when pinned mapped memory is unavailable.
volatile unsigned int* error_mirror(int dev) {
  static std::once_flag flags[wgrad::kMaxDevices];
  static volatile unsigned int* words[wgrad::kMaxDevices] = {};
  if (dev < 0 || dev >= wgrad::kMaxDevices) return nullptr;
  std::call_once(flags[dev], [dev] {
    void* h = nullptr;
    if (cudaHostAlloc(&h, sizeof(unsigned int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
      (void)cudaGetLastError();
      return;
    }
    *static_cast<volatile unsigned int*>(h) = 0u;
    void* d = nullptr;
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess ||
        cudaMemcpyToSymbol(wgrad::g_device_error_host, &d, sizeof(d)) != cudaSuccess) {
      (void)cudaGetLastError();
      cudaFreeHost(h);
      return;
    }
    words[dev] = static_cast<volatile unsigned int*>(h);
  });
  return words[dev];
}

int check_arch(DeviceInfo* info) {
  const int st = device_info(info);
  if (st != SM100_WGRAD_OK) return st;
  // sm_100a code runs on compute capability 10.0 only.
  if (info->major != 10 || info->minor != 0) return SM100_WGRAD_ERR_UNSUPPORTED_ARCH;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  (void)error_mirror(dev);
  return SM100_WGRAD_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// FP8 operand [cols][pitch] bytes, box = 128 K-bytes x box_rows columns, 128B swizzle.
int encode_operand_map(CUtensorMap* map, const void* data, int64_t k_rows, int64_t cols, int64_t pitch,
                       int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k_rows), static_cast<cuuint64_t>(cols)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
  const cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(box_rows)};
  return cached_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, data, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                       WGRAD_OPERAND_L2_PROMOTION);
}

// Output [E][M][N]; box = (64 bf16 | 32 fp32) columns x 32 rows x 1 expert,
// 128B swizzle; narrow_bf16: 32-column bf16 boxes (64-byte rows, 64B swizzle).
int encode_out_map(CUtensorMap* map, void* out, int out_f32, int64_t e, int64_t m, int64_t n,
                   bool narrow_bf16 = false) {
  const int64_t esz = out_f32 ? 4 : 2;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m), static_cast<cuuint64_t>(e)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(n * esz), static_cast<cuuint64_t>(m * n * esz)};
  const bool narrow = narrow_bf16 && !out_f32;
  const cuuint32_t box[3] = {out_f32 || narrow ? 32u : 64u, 32u, 1u};
  return cached_encode(map, out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, dims,
                       strides, box, narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

// Split-scale operand of the scale-product kernel: [blocks][cols][4] fp32
// (16 B per scale), read as boxes of 8 x box_rows x 1 with 32-byte swizzling;
// the box's four K elements past the 16-byte row lie outside the tensor and
// are zero-filled by the TMA unit.
int encode_scale_operand_map(CUtensorMap* map, void* data, int64_t cols, int64_t blocks, int box_rows) {
  const cuuint64_t dims[3] = {4u, static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(blocks)};
  const cuuint64_t strides[2] = {16u, static_cast<cuuint64_t>(cols * 16)};
  const cuuint32_t box[3] = {8u, static_cast<cuuint32_t>(box_rows), 1u};
  return cached_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, data, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_32B,
                       CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

// Workspace of the scale-product kernel: the split lhs scales [blocks][m][4]
// fp32, then (256-byte aligned) the split rhs scales [blocks][n][4].
int64_t sp_workspace_lhs_bytes(int64_t blocks, int64_t m) { return (blocks * m * 16 + 255) / 256 * 256; }
int64_t sp_workspace_bytes(int64_t blocks, int64_t m, int64_t n) {
  return sp_workspace_lhs_bytes(blocks, m) + blocks * n * 16;
}

int pick_bn(int32_t tile_config, int64_t n) {
  if (tile_config == SM100_WGRAD_TILE_256x256_SP || tile_config == SM100_WGRAD_TILE_256x256_SP_W16) return 256;
  if (tile_config == SM100_WGRAD_TILE_128x128 || tile_config == SM100_WGRAD_TILE_128x128_2CTA) return 128;
  if (tile_config == SM100_WGRAD_TILE_128x192_W12 || tile_config == SM100_WGRAD_TILE_128x192_UE8M0) return 192;
  if (tile_config == SM100_WGRAD_TILE_128x256 || tile_config == SM100_WGRAD_TILE_128x256_W8 ||
      tile_config == SM100_WGRAD_TILE_128x256_W16 || tile_config == SM100_WGRAD_TILE_256x256_PAIR ||
      tile_config == SM100_WGRAD_TILE_256x256_PAIR_W16)
    return 256;
  // auto: the wide tile halves operand re-reads per output byte; a narrow N
  // would only fill it with zero columns.
  return n <= 128 ? 128 : 256;
}

// Average 128-row K blocks per expert at or below which the 256-wide tile runs
// 16 promotion warps: such launches are bound by output stores and per-block
// latency, which more warps overlap; deeper K favours 8 warps.
constexpr int64_t kShortKBlocksPerExpert = 2;

int pick_epi_warps(int32_t tile_config, int bn, int64_t total_blocks, int64_t num_experts) {
  if (tile_config == SM100_WGRAD_TILE_128x128_2CTA) return 4;
  if (tile_config == SM100_WGRAD_TILE_128x192_W12 || tile_config == SM100_WGRAD_TILE_128x192_UE8M0) return 12;
  if (bn != 256 || tile_config == SM100_WGRAD_TILE_128x256_W8 || tile_config == SM100_WGRAD_TILE_256x256_PAIR) return 8;
  if (tile_config == SM100_WGRAD_TILE_128x256_W16 || tile_config == SM100_WGRAD_TILE_256x256_PAIR_W16 ||
      tile_config == SM100_WGRAD_TILE_256x256_SP_W16)
    return 16;
  if (tile_config == SM100_WGRAD_TILE_256x256_SP) return 8;
  return total_blocks <= kShortKBlocksPerExpert * num_experts ? 16 : 8;
}

// Automatic choice between the 128 x 256 single-CTA tile and the 256 x 256
// CTA pair: the pair moves a third less operand data per SM per K block but
// pays more per tile (two CTAs meet at every partial and at the tile's end),
// so it is chosen for long contractions over experts with many output tiles.
// Measured interleaved on B200: the pair is 2-3 % faster on DeepSeek-V3 32k
// (8.5 K blocks and 224-448 pair tiles per expert) and its skewed routing,
// the single-CTA tile 3-7 % faster on DeepSeek-V3 4k-16k and Qwen3 32k.
constexpr int64_t kPairMinBlocksPerExpert = 8;
constexpr int64_t kPairMinTilesPerExpert = 64;

int32_t resolve_tile(const Sm100WgradArgs* a) {
  if (a->tile_config != SM100_WGRAD_TILE_AUTO) return a->tile_config;
#if WGRAD_DEBUG_MODES
  // the known-answer modes run on the single-CTA kernels only
  if (const char* km = std::getenv("KERNEL_LAB_WGRAD_KERNEL_MODE"); km != nullptr && km[0] != '\0' &&
      std::strcmp(km, "normal") != 0)
    return SM100_WGRAD_TILE_AUTO;
#endif
  const int64_t pair_tiles = ((a->m + 255) / 256) * ((a->n + 255) / 256);
  if (a->n > 128 && pair_tiles >= kPairMinTilesPerExpert &&
      a->total_blocks >= kPairMinBlocksPerExpert * a->num_experts)
    return SM100_WGRAD_TILE_256x256_PAIR;
  return SM100_WGRAD_TILE_AUTO;
}

}  // namespace

extern "C" {

const char* sm100_wgrad_version(void) { return "0.1.0"; }

const char* sm100_wgrad_status_string(int status) {
  switch (status) {
    case SM100_WGRAD_OK: return "ok";
    case SM100_WGRAD_ERR_INVALID_ARG: return "invalid argument";
    case SM100_WGRAD_ERR_UNSUPPORTED_ARCH: return "unsupported GPU architecture (requires sm_100a / B200)";
    case SM100_WGRAD_ERR_LAUNCH: return "CUDA launch or driver call failed";
    case SM100_WGRAD_ERR_TENSOR_MAP: return "TMA descriptor encoding failed";
    case SM100_WGRAD_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case SM100_WGRAD_ERR_UNSUPPORTED: return "unsupported shape or option";
    default: return "unknown status";
  }
}

int sm100_fp8_grouped_wgrad(const Sm100WgradArgs* a, void* stream) {
  if (a == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->out == nullptr || a->block_offsets == nullptr || a->k_row_offsets == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->num_experts < 0 || a->m <= 0 || a->n <= 0 || a->k_rows < 0 || a->total_blocks < 0)
    return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->out_dtype != SM100_WGRAD_OUT_BF16 && a->out_dtype != SM100_WGRAD_OUT_F32) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->tile_config < SM100_WGRAD_TILE_AUTO || a->tile_config > SM100_WGRAD_TILE_256x256_SP_W16)
    return SM100_WGRAD_ERR_INVALID_ARG;
  // TMA: output row pitch and scale-vector chunks must be 16-byte multiples.
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
  }
  if (a->num_experts == 0) return SM100_WGRAD_OK;

  DeviceInfo info;
  int st = check_arch(&info);
  if (st != SM100_WGRAD_OK) return st;

  const int32_t tile = resolve_tile(a);
  const int bn = pick_bn(tile, a->n);
  const bool sp = tile == SM100_WGRAD_TILE_256x256_SP || tile == SM100_WGRAD_TILE_256x256_SP_W16;
  const bool pair = sp || tile == SM100_WGRAD_TILE_256x256_PAIR || tile == SM100_WGRAD_TILE_256x256_PAIR_W16;
  const int bm = pair ? 256 : 128;
  CUtensorMap ta{}, tb{}, to{}, tsa{}, tsb{};
  void* opa = nullptr;
  void* opb = nullptr;
  if (sp && has_operands) {
    const int64_t need = sp_workspace_bytes(a->total_blocks, a->m, a->n);
    if (a->workspace == nullptr || a->workspace_bytes < need || (reinterpret_cast<uintptr_t>(a->workspace) & 255u))
      return SM100_WGRAD_ERR_INVALID_ARG;
    opa = a->workspace;
    opb = static_cast<uint8_t*>(a->workspace) + sp_workspace_lhs_bytes(a->total_blocks, a->m);
  }
  if (has_operands) {
    st = encode_operand_map(&ta, a->lhs_data, a->k_rows, a->m, a->lhs_pitch, 128);
    if (st != SM100_WGRAD_OK) return st;
    // a pair CTA loads half of the rhs tile's rows (the scale-product kernel:
    // half of each 128-column half)
    st = encode_operand_map(&tb, a->rhs_data, a->k_rows, a->n, a->rhs_pitch, sp ? 64 : (pair ? bn / 2 : bn));
    if (st != SM100_WGRAD_OK) return st;
    if (sp) {
      st = encode_scale_operand_map(&tsa, opa, a->m, a->total_blocks, 128);
      if (st != SM100_WGRAD_OK) return st;
      st = encode_scale_operand_map(&tsb, opb, a->n, a->total_blocks, 64);
      if (st != SM100_WGRAD_OK) return st;
    }
  }
  st = encode_out_map(&to, a->out, a->out_dtype == SM100_WGRAD_OUT_F32, a->num_experts, a->m, a->n,
                      tile == SM100_WGRAD_TILE_256x256_SP_W16);
  if (st != SM100_WGRAD_OK) return st;

  GemmParams p{};
  p.sa = a->lhs_scales;
  p.sb = a->rhs_scales;
  p.out = a->out;
  p.block_offsets = a->block_offsets;
  p.k_row_offsets = a->k_row_offsets;
  p.expert_order = a->expert_order;
  p.num_experts = static_cast<int>(a->num_experts);
  p.m = static_cast<int>(a->m);
  p.n = static_cast<int>(a->n);
  p.bn = bn;
  p.bm = bm;
  p.tiles_n = static_cast<int>((a->n + bn - 1) / bn);
  const int64_t tiles_m = (a->m + bm - 1) / bm;
  const int64_t tpe = tiles_m * p.tiles_n;
  const int64_t num_tiles = tpe * a->num_experts;
  if (num_tiles > INT32_MAX) return SM100_WGRAD_ERR_UNSUPPORTED;
  p.tiles_per_expert = static_cast<int>(tpe);
  p.num_tiles = static_cast<int>(num_tiles);
  p.out_f32 = a->out_dtype == SM100_WGRAD_OUT_F32;
  p.accumulate = a->accumulate != 0;
  p.has_operands = has_operands ? 1 : 0;
  p.epi_warps = pick_epi_warps(tile, bn, a->total_blocks, a->num_experts);
  // Known-answer kernel modes (KERNEL_LAB_WGRAD_KERNEL_MODE, as the reference)
  // and the test-only failure injection exist in the debug-modes library only;
  // the product library reads no environment variable.
  p.mode = wgrad::kModeNormal;
  p.inject = 0;
#if WGRAD_DEBUG_MODES
  if (const char* km = std::getenv("KERNEL_LAB_WGRAD_KERNEL_MODE"); km != nullptr && km[0] != '\0' &&
      std::strcmp(km, "normal") != 0) {
    if (std::strcmp(km, "coord_m") == 0) p.mode = wgrad::kModeCoordM;
    else if (std::strcmp(km, "coord_n") == 0) p.mode = wgrad::kModeCoordN;
    else if (std::strcmp(km, "scale_only") == 0) p.mode = wgrad::kModeScaleOnly;
    else if (std::strcmp(km, "unscaled") == 0) p.mode = wgrad::kModeUnscaled;
    else return SM100_WGRAD_ERR_INVALID_ARG;
  }
  // Test-only failure injection of the bounded-wait path.
  if (const char* inject = std::getenv("SM100_WGRAD_DEBUG_INJECT");
      inject != nullptr && std::strcmp(inject, "withhold_first_load") == 0)
    p.inject = wgrad::kInjectWithholdFirstLoad;
#endif
  p.ue8m0 = tile == SM100_WGRAD_TILE_128x192_UE8M0 ? 1 : 0;
  // The known-answer modes instrument the promotion loop, which the UE8M0 kernel does not have.
  if (p.ue8m0 && p.mode != wgrad::kModeNormal) return SM100_WGRAD_ERR_UNSUPPORTED;
  if (pair && !sp && p.mode != wgrad::kModeNormal) return SM100_WGRAD_ERR_UNSUPPORTED;

  int grid = info.sm_count * (p.epi_warps == 4 ? 2 : 1);  // the 4-warp tile runs two CTAs per SM
  if (a->max_ctas > 0 && a->max_ctas < grid) grid = a->max_ctas;
  if (pair) {
    // one cluster of two CTAs per tile at most; whole clusters only
    if (2 * num_tiles < grid) grid = static_cast<int>(2 * num_tiles);
    grid &= ~1;
    if (grid < 2) grid = 2;
  } else if (num_tiles < grid) {
    grid = static_cast<int>(num_tiles);
  }
  if (sp) {
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (has_operands) {
      cudaError_t e = wgrad::launch_scale_operands(a->lhs_scales, a->rhs_scales, opa, opb, a->m, a->n,
                                                   a->block_offsets, p.num_experts, a->total_blocks, info.sm_count, s);
      if (e != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
    }
    const cudaError_t e = wgrad::launch_grouped_wgrad_sp(ta, tb, tsa, tsb, to, p, grid, s);
    return e == cudaSuccess ? SM100_WGRAD_OK : SM100_WGRAD_ERR_LAUNCH;
  }
  const cudaError_t err = wgrad::launch_grouped_wgrad(ta, tb, to, p, grid, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SM100_WGRAD_OK : SM100_WGRAD_ERR_LAUNCH;
}

int sm100_wgrad_workspace_bytes(const Sm100WgradArgs* a, int64_t* bytes) {
  if (a == nullptr || bytes == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->m <= 0 || a->n <= 0 || a->total_blocks < 0) return SM100_WGRAD_ERR_INVALID_ARG;
  const bool sp = a->tile_config == SM100_WGRAD_TILE_256x256_SP || a->tile_config == SM100_WGRAD_TILE_256x256_SP_W16;
  *bytes = sp ? sp_workspace_bytes(a->total_blocks, a->m, a->n) : 0;
  return SM100_WGRAD_OK;
}

int sm100_wgrad_quantize_1x128(const void* x, int32_t x_dtype, int64_t valid_rows, int64_t cols,
                               const int32_t* block_row_start, const int32_t* block_row_count,
                               int64_t total_blocks, void* q_data, int64_t q_pitch, float* scales, void* stream) {
  if (x_dtype != 0 && x_dtype != 1) return SM100_WGRAD_ERR_INVALID_ARG;
  if (valid_rows < 0 || cols < 0 || total_blocks < 0) return SM100_WGRAD_ERR_INVALID_ARG;
  if (total_blocks == 0 || cols == 0) return SM100_WGRAD_OK;
  if (x == nullptr && valid_rows > 0) return SM100_WGRAD_ERR_INVALID_ARG;
  if (block_row_start == nullptr || block_row_count == nullptr || q_data == nullptr || scales == nullptr)
    return SM100_WGRAD_ERR_INVALID_ARG;
  if (q_pitch % 16 != 0 || q_pitch < total_blocks * 128 || !aligned16(q_data)) return SM100_WGRAD_ERR_INVALID_ARG;
  if (total_blocks > INT32_MAX) return SM100_WGRAD_ERR_UNSUPPORTED;
  DeviceInfo info;
  const int st = check_arch(&info);
  if (st != SM100_WGRAD_OK) return st;
  const cudaError_t err = wgrad::launch_quantize_1x128(x, x_dtype, cols, nullptr, block_row_start, block_row_count,
                                                       total_blocks, q_data, q_pitch, nullptr, true, nullptr, 0,
                                                       nullptr, scales, 128, valid_rows, false,
                                                       static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SM100_WGRAD_OK : SM100_WGRAD_ERR_LAUNCH;
}

int sm100_wgrad_quantize_1x128_ex(const Sm100WgradQuantArgs* a, void* stream) {
  if (a == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->x_dtype != 0 && a->x_dtype != 1) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->cols < 0 || a->total_blocks < 0 || a->q_pitch < 0 || a->kq_pitch < 0) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->total_blocks == 0 || a->cols == 0) return SM100_WGRAD_OK;
  if (a->x == nullptr || a->block_row_start == nullptr || a->block_row_count == nullptr || a->q_data == nullptr ||
      a->scales == nullptr)
    return SM100_WGRAD_ERR_INVALID_ARG;
  const int block_rows = a->block_rows == 0 ? 128 : a->block_rows;
  if (block_rows != 32 && block_rows != 64 && block_rows != 128) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->gather_idx != nullptr && a->x_rows <= 0) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->q_row_start == nullptr && (a->q_pitch < a->total_blocks * block_rows || a->q_pitch % 16 != 0))
    return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->kq_data != nullptr && a->kq_row_start == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->scale_format != 0 && a->scale_format != 1) return SM100_WGRAD_ERR_INVALID_ARG;
  if (a->total_blocks > INT32_MAX) return SM100_WGRAD_ERR_UNSUPPORTED;
  DeviceInfo info;
  const int st = check_arch(&info);
  if (st != SM100_WGRAD_OK) return st;
  const cudaError_t err = wgrad::launch_quantize_1x128(
      a->x, a->x_dtype, a->cols, a->gather_idx, a->block_row_start, a->block_row_count, a->total_blocks, a->q_data,
      a->q_pitch, a->q_row_start, a->q_zero_fill != 0, a->kq_data, a->kq_pitch, a->kq_row_start, a->scales,
      block_rows, a->x_rows, a->scale_format == 1, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SM100_WGRAD_OK : SM100_WGRAD_ERR_LAUNCH;
}

int sm100_wgrad_build_meta(const int32_t* cu_seqlens_k, int64_t num_experts, const Sm100WgradMetaOut* out,
                           void* stream) {
  if (cu_seqlens_k == nullptr || out == nullptr || num_experts < 0) return SM100_WGRAD_ERR_INVALID_ARG;
  if (out->totals == nullptr || out->block_offsets == nullptr || out->padded_cu_seqlens_k == nullptr ||
      out->wgmma_cu_seqlens_k == nullptr || out->expert_order == nullptr ||
      (num_experts > 0 && (out->blocks_per_expert == nullptr || out->tail_valid_rows == nullptr ||
                           out->tail_wgmma_atoms == nullptr || out->tail_copy_k == nullptr ||
                           out->has_tail == nullptr)) ||
      out->block_capacity < 0)
    return SM100_WGRAD_ERR_INVALID_ARG;
  if (out->block_capacity > 0 &&
      (out->block_row_start == nullptr || out->block_row_count == nullptr || out->wgmma_block_row_start == nullptr))
    return SM100_WGRAD_ERR_INVALID_ARG;
  DeviceInfo info;
  const int st = check_arch(&info);
  if (st != SM100_WGRAD_OK) return st;
  const cudaError_t err = wgrad::launch_build_meta(cu_seqlens_k, num_experts, *out, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? SM100_WGRAD_OK : SM100_WGRAD_ERR_LAUNCH;
}

int sm100_wgrad_profile_counters(uint64_t* counters, int32_t n) {
  if (counters == nullptr || n < 0) return SM100_WGRAD_ERR_INVALID_ARG;
#if WGRAD_PROFILE
  unsigned long long v[wgrad::kProfSlots] = {0};
  if (cudaMemcpyFromSymbol(v, wgrad::g_wgrad_prof, sizeof(v)) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  const unsigned long long z[wgrad::kProfSlots] = {0};
  if (cudaMemcpyToSymbol(wgrad::g_wgrad_prof, z, sizeof(z)) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  for (int i = 0; i < n && i < wgrad::kProfSlots; ++i) counters[i] = v[i];
  return SM100_WGRAD_OK;
#else
  return SM100_WGRAD_ERR_UNSUPPORTED;  // library built without WGRAD_PROFILE
#endif
}

int sm100_wgrad_device_error(int32_t* code) {
  if (code == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, wgrad::g_device_error, sizeof(v)) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  if (v != 0 && cudaMemcpyToSymbol(wgrad::g_device_error, &zero, sizeof(zero)) != cudaSuccess)
    return SM100_WGRAD_ERR_LAUNCH;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    if (volatile unsigned int* w = error_mirror(dev)) *w = 0u;  // reported here: nothing left pending
  }
  *code = static_cast<int32_t>(v);
  return SM100_WGRAD_OK;
}

int sm100_wgrad_poll_device_error(int32_t* code) {
  if (code == nullptr) return SM100_WGRAD_ERR_INVALID_ARG;
  *code = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  volatile unsigned int* w = error_mirror(dev);
  if (w == nullptr) return SM100_WGRAD_ERR_UNSUPPORTED;
  const unsigned int v = *w;
  if (v != 0u) *w = 0u;
  *code = static_cast<int32_t>(v);
  return SM100_WGRAD_OK;
}

#if WGRAD_TRACE
// Event trace of CTAs 0 and 1 (trace builds only; not part of the product ABI).
SM100_WGRAD_API int sm100_wgrad_trace_read(uint64_t* out, int32_t n) {
  if (out == nullptr || n < 0) return SM100_WGRAD_ERR_INVALID_ARG;
  static unsigned long long buf[2 * wgrad::kTraceBlocks * wgrad::kTraceEvents];
  if (cudaMemcpyFromSymbol(buf, wgrad::g_wgrad_trace, sizeof(buf)) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  for (int i = 0; i < n && i < static_cast<int>(sizeof(buf) / 8); ++i) out[i] = buf[i];
  static const unsigned long long zero[2 * wgrad::kTraceBlocks * wgrad::kTraceEvents] = {};
  if (cudaMemcpyToSymbol(wgrad::g_wgrad_trace, zero, sizeof(zero)) != cudaSuccess) return SM100_WGRAD_ERR_LAUNCH;
  return SM100_WGRAD_OK;
}
#endif

int sm100_wgrad_build_flags(void) {
  return (WGRAD_DEBUG_MODES ? SM100_WGRAD_BUILD_DEBUG_MODES : 0) | (WGRAD_PROFILE ? SM100_WGRAD_BUILD_PROFILE : 0);
}

}  // extern "C"
