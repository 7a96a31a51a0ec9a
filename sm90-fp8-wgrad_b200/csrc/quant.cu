// 1x128 FP8 e4m3 quantiser for grouped Wgrad operands (padded layout).
//
// Restates the Triton kernel _quantize_grouped_wgrad_128x1_kernel
// (src/sm90_fp8_wgrad/quant.py:105-167) as a plain CUDA kernel:
//   for each 128-row scale block b and column c
//     amax        = max_{k < row_count[b]} |x[row_start[b] + k, c]|      (:141-145)
//     scale[b, c] = max(amax / 448, 1e-12)                               (:145-146)
//     q[c][128 b + k] = e4m3(x / scale)  for k < row_count[b]            (:139, :149-154)
//     q[c][128 b + k] = 0                for row_count[b] <= k < 128    (zero fill, :236-237)
// The division is IEEE fp32 (x / scale, not x * (1 / scale)) and the e4m3
// conversion is round-to-nearest-even with saturation to the finite range, so
// the bytes are reproducible on the CPU.
//
// Layouts: the padded operand (row b*128 + k, rows past the block's count
// written as zeros), or the packed storage of the reference's packed layout
// mode (quant.py:196-266: valid rows at block_row_start[b] + k in `data`, and a
// second copy at wgmma_block_row_start[b] + k in the zero-initialised
// `kernel_data`). An optional gather index reads the rows straight from a
// token-major activation (row r of the grouped operand = x row gather_idx[r]),
// which fuses the expert-major gather of the MoE backward into the quantiser.
//
// Scale blocks are 128 rows (the GEMM's contract) or, for the reference's
// compact tail operands (quant.py:273-307), 32 or 64 rows: block b then
// occupies padded rows [block_rows * b, block_rows * (b + 1)).
//
// HBM-bound transpose: a CTA reads a 128-row x 64-column BF16 tile with
// 16-byte coalesced loads, reduces column amax through shared memory and
// writes each column's 128 FP8 bytes as one contiguous 128-byte segment
// (the operand is K-contiguous per column).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace wgrad {

namespace {

constexpr int QBLOCK_ROWS = 128;
constexpr int QBLOCK_COLS = 64;
constexpr int QTHREADS = 256;

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* src, float (&v)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* src, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(src));
  const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename T>
__device__ __forceinline__ float load1(const T* src);
template <>
__device__ __forceinline__ float load1<__nv_bfloat16>(const __nv_bfloat16* src) {
  return __bfloat162float(src[0]);
}
template <>
__device__ __forceinline__ float load1<float>(const float* src) {
  return src[0];
}

// grid: (total_blocks, ceil(cols / 64)); block: 256 threads.
// Destination of the quantised bytes: column c's byte k of block b goes to
// q[c * pitch + row_start[b] + k] (row_start == nullptr: 128 b, the padded
// layout). zero_fill also writes the zero rows k >= row_count of the block.
struct QuantDst {
  uint8_t* q;
  int64_t pitch;
  const int32_t* row_start;
  bool zero_fill;
};

template <typename T>
__global__ void __launch_bounds__(QTHREADS) quantize_1x128_kernel(const T* __restrict__ x, int64_t cols,
                                                                  const int32_t* __restrict__ gather_idx,
                                                                  const int32_t* __restrict__ block_row_start,
                                                                  const int32_t* __restrict__ block_row_count,
                                                                  QuantDst d0, QuantDst d1,
                                                                  float* __restrict__ scales, bool vec_ok,
                                                                  int block_rows, int64_t x_rows) {
  __shared__ float tile[QBLOCK_ROWS][QBLOCK_COLS + 1];
  __shared__ float s_amax[4][QBLOCK_COLS];
  __shared__ float s_scale[QBLOCK_COLS];

  const int b = blockIdx.x;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * QBLOCK_COLS;
  const int64_t row0 = __ldg(block_row_start + b);
  const int rows = __ldg(block_row_count + b);
  const int ncols = static_cast<int>(min(static_cast<int64_t>(QBLOCK_COLS), cols - c0));
  const int tid = threadIdx.x;

  // Load: 8 threads per row (8 columns each), 32 rows per pass.
  {
    const int sub = tid & 7;
    const int r_in = tid >> 3;
    const int cc = sub * 8;
#pragma unroll
    for (int pass = 0; pass < QBLOCK_ROWS / 32; ++pass) {
      const int r = pass * 32 + r_in;
      float v[8];
      if (r < rows && cc < ncols) {
        int64_t xrow = gather_idx != nullptr ? static_cast<int64_t>(__ldg(gather_idx + row0 + r)) : row0 + r;
        if (gather_idx != nullptr && (xrow < 0 || xrow >= x_rows)) {
          // Out-of-range gather index: read nothing, flag the device error word.
          record_device_error(kDevBadGatherIndex);
          xrow = -1;
        }
        const T* src = x + (xrow < 0 ? 0 : xrow) * cols + c0 + cc;
        if (xrow < 0) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = 0.f;
        } else if (vec_ok && cc + 8 <= ncols) {
          load8<T>(src, v);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = (cc + i < ncols) ? load1<T>(src + i) : 0.f;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) tile[r][cc + i] = v[i];
    }
  }
  __syncthreads();

  // Column amax: 4 threads per column, 32 rows each.
  {
    const int col = tid & 63;
    const int part = tid >> 6;
    float m = 0.f;
#pragma unroll 8
    for (int r = part * 32; r < part * 32 + 32; ++r) m = fmaxf(m, fabsf(tile[r][col]));
    s_amax[part][col] = m;
  }
  __syncthreads();
  if (tid < QBLOCK_COLS) {
    const float amax = fmaxf(fmaxf(s_amax[0][tid], s_amax[1][tid]), fmaxf(s_amax[2][tid], s_amax[3][tid]));
    const float scale = fmaxf(__fdiv_rn(amax, 448.0f), 1.0e-12f);
    s_scale[tid] = scale;
    if (tid < ncols) scales[static_cast<int64_t>(b) * cols + c0 + tid] = scale;
  }
  __syncthreads();

  // Store: each 16-row chunk of column c's bytes as one 16-byte vector when the
  // destination is aligned and the chunk is entirely written, else bytewise.
  for (int idx = tid; idx < QBLOCK_COLS * 8; idx += QTHREADS) {
    const int col = idx >> 3;
    const int chunk = idx & 7;
    if (col >= ncols) continue;
    const float s = s_scale[col];
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = chunk * 16 + i * 4;
      const float f0 = __fdiv_rn(tile[k + 0][col], s);
      const float f1 = __fdiv_rn(tile[k + 1][col], s);
      const float f2 = __fdiv_rn(tile[k + 2][col], s);
      const float f3 = __fdiv_rn(tile[k + 3][col], s);
      const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f0, f1), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(f2, f3), __NV_SATFINITE, __NV_E4M3);
      w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      const QuantDst& d = o == 0 ? d0 : d1;
      if (d.q == nullptr) continue;
      const int64_t start = d.row_start != nullptr ? static_cast<int64_t>(__ldg(d.row_start + b))
                                                   : static_cast<int64_t>(b) * block_rows;
      const int limit = d.zero_fill ? block_rows : rows;  // rows k < limit are written
      if (chunk * 16 >= limit) continue;
      uint8_t* dst = d.q + (c0 + col) * d.pitch + start + chunk * 16;
      if (chunk * 16 + 16 <= limit && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      } else {
        for (int i = 0; i < 16 && chunk * 16 + i < limit; ++i) dst[i] = static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3)));
      }
    }
  }
}

}  // namespace

cudaError_t launch_quantize_1x128(const void* x, int x_dtype, int64_t cols, const int32_t* gather_idx,
                                  const int32_t* block_row_start, const int32_t* block_row_count,
                                  int64_t total_blocks, void* q, int64_t q_pitch, const int32_t* q_row_start,
                                  bool q_zero_fill, void* kq, int64_t kq_pitch, const int32_t* kq_row_start,
                                  float* scales, int block_rows, int64_t x_rows, cudaStream_t stream) {
  if (total_blocks == 0 || cols == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(total_blocks), static_cast<unsigned>((cols + QBLOCK_COLS - 1) / QBLOCK_COLS));
  const QuantDst d0{static_cast<uint8_t*>(q), q_pitch, q_row_start, q_zero_fill};
  const QuantDst d1{static_cast<uint8_t*>(kq), kq_pitch, kq_row_start, false};
  if (x_dtype == 0) {
    const bool vec_ok = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    quantize_1x128_kernel<__nv_bfloat16><<<grid, QTHREADS, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), cols, gather_idx, block_row_start, block_row_count, d0, d1, scales,
        vec_ok, block_rows, x_rows);
  } else {
    const bool vec_ok = (cols % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    quantize_1x128_kernel<float><<<grid, QTHREADS, 0, stream>>>(static_cast<const float*>(x), cols, gather_idx,
                                                               block_row_start, block_row_count, d0, d1, scales,
                                                               vec_ok, block_rows, x_rows);
  }
  return cudaGetLastError();
}

}  // namespace wgrad
