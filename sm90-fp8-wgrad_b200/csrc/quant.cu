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
// HBM-bound transpose: a CTA owns one scale block x a strip of 64 columns.
// Every thread issues its 16-byte row loads before writing them to shared
// memory (16 KB BF16 tiles, so eight CTAs share an SM); then each thread walks
// one column slice (amax, then x / scale), and the FP8 bytes leave through a
// column-major staging area as full 128-byte lines of the K-contiguous operand.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ptx.cuh"

namespace wgrad {

namespace {

constexpr int QBLOCK_ROWS = 128;
constexpr int QTHREADS = 256;

// Column strip of one CTA: 64 columns (a 16 KB BF16 or 32 KB fp32 tile);
// TPR threads per tile row, one 16-byte vector each, ROW_PASSES passes.
template <typename T>
struct QTile {
  static constexpr int VEC = 16 / static_cast<int>(sizeof(T));
  static constexpr int COLS = 64;
  static constexpr int TPR = COLS / VEC;                      // threads per tile row
  static constexpr int ROWS_PER_PASS = QTHREADS / TPR;
  static constexpr int ROW_PASSES = QBLOCK_ROWS / ROWS_PER_PASS;
  static constexpr int PARTS = QTHREADS / COLS;               // row parts per column
  static constexpr int ROWS_PER_PART = QBLOCK_ROWS / PARTS;   // 64 (bf16) or 32 (fp32)
};

__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(float v) { return v; }
template <typename T>
__device__ __forceinline__ T zero_of();
template <>
__device__ __forceinline__ __nv_bfloat16 zero_of<__nv_bfloat16>() { return __float2bfloat16(0.f); }
template <>
__device__ __forceinline__ float zero_of<float>() { return 0.f; }

constexpr int QSTAGE_PITCH = 144;  // bytes per staged FP8 column (128 + 16 pad)

// x / s rounded to nearest even, for the quantiser's positive scale s, from the
// correctly rounded reciprocal rs = RN(1/s) and one FMA correction step
// (Markstein's theorem, IBM J. Res. Dev. 34(1), 1990; also Muller et al.,
// Handbook of Floating-Point Arithmetic, sec. 4.7): q0 = RN(x rs) is faithful,
// the remainder x - s q0 is exact in one FMA, and RN(q0 + rem rs) is the
// correctly rounded quotient when nothing overflows or underflows. Quotients
// small enough for the remainder to underflow are far below the smallest e4m3
// subnormal (they encode as zero either way). The sign of a zero quotient is
// taken from x, as IEEE division gives it; an infinite scale uses the
// division directly.
__device__ __forceinline__ float div_rn_by_scale(float x, float s, float rs, bool finite_scale) {
  if (!finite_scale) return __fdiv_rn(x, s);
  const float q0 = x * rs;
  const float rem = fmaf(-q0, s, x);
  const float q1 = fmaf(rem, rs, q0);
  return __int_as_float(__float_as_int(q1) | (__float_as_int(x) & static_cast<int>(0x80000000u)));
}

// Smallest power of two >= s, for a positive normal s (the clamped scale is at
// least 1e-12): a set mantissa bit moves the value up to the next exponent.
// Infinity and NaN stay as they are.
__device__ __forceinline__ float round_up_pow2(float s) {
  const uint32_t bits = __float_as_uint(s);
  if ((bits & 0x7F800000u) == 0x7F800000u || (bits & 0x7FFFFFu) == 0u) return s;
  return __uint_as_float((bits & 0xFF800000u) + 0x800000u);
}

// grid: (total_blocks, ceil(cols / QTile<T>::COLS)); block: 256 threads.
// Destination of the quantised bytes: column c's byte k of block b goes to
// q[c * pitch + row_start[b] + k] (row_start == nullptr: block_rows * b, the
// padded layout). zero_fill also writes the zero rows k >= row_count.
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
                                                                  int block_rows, int64_t x_rows, bool ue8m0) {
  using Q = QTile<T>;
  // The tile keeps the input type (16 KB BF16, 32 KB fp32): row-major 16-byte writes, and the
  // column walks below read 32 consecutive columns per warp, so neither side
  // has shared-memory bank conflicts.
  __shared__ __align__(16) T tile[QBLOCK_ROWS][Q::COLS];
  __shared__ float s_amax[Q::PARTS][Q::COLS];
  __shared__ float s_scale[Q::COLS];

  const int b = blockIdx.x;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * Q::COLS;
  const int64_t row0 = __ldg(block_row_start + b);
  const int rows = __ldg(block_row_count + b);
  const int ncols = static_cast<int>(min(static_cast<int64_t>(Q::COLS), cols - c0));
  const int tid = threadIdx.x;

  // Load: all eight 16-byte loads of a thread are issued before any is
  // written to shared memory, so 32 KB per CTA are in flight at once.
  {
    const int cc = (tid % Q::TPR) * Q::VEC;
    const int r_in = tid / Q::TPR;
    uint4 buf[Q::ROW_PASSES];
#pragma unroll
    for (int pass = 0; pass < Q::ROW_PASSES; ++pass) {
      const int r = pass * Q::ROWS_PER_PASS + r_in;
      buf[pass] = make_uint4(0u, 0u, 0u, 0u);
      if (r < rows && cc < ncols) {
        int64_t xrow = gather_idx != nullptr ? static_cast<int64_t>(__ldg(gather_idx + row0 + r)) : row0 + r;
        if (gather_idx != nullptr && (xrow < 0 || xrow >= x_rows)) {
          // Out-of-range gather index: read nothing, flag the device error word.
          record_device_error(kDevBadGatherIndex);
          continue;  // zeros
        }
        const T* src = x + xrow * cols + c0 + cc;
        if (vec_ok && cc + Q::VEC <= ncols) {
          buf[pass] = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
          T v[Q::VEC];
#pragma unroll
          for (int i = 0; i < Q::VEC; ++i) v[i] = (cc + i < ncols) ? src[i] : zero_of<T>();
          buf[pass] = *reinterpret_cast<const uint4*>(v);
        }
      }
    }
#pragma unroll
    for (int pass = 0; pass < Q::ROW_PASSES; ++pass) {
      *reinterpret_cast<uint4*>(&tile[pass * Q::ROWS_PER_PASS + r_in][cc]) = buf[pass];
    }
  }
  __syncthreads();

  // Column amax: thread (col, part) walks ROWS_PER_PART rows of one column.
  const int col = tid % Q::COLS;
  const int part = tid / Q::COLS;
  const int k_begin = part * Q::ROWS_PER_PART;
  {
    float m = 0.f;
#pragma unroll 16
    for (int k = k_begin; k < k_begin + Q::ROWS_PER_PART; ++k) m = fmaxf(m, fabsf(to_f(tile[k][col])));
    s_amax[part][col] = m;
  }
  __syncthreads();
  if (tid < Q::COLS) {
    float amax = s_amax[0][tid];
#pragma unroll
    for (int pp = 1; pp < Q::PARTS; ++pp) amax = fmaxf(amax, s_amax[pp][tid]);
    float scale = fmaxf(__fdiv_rn(amax, 448.0f), 1.0e-12f);
    if (ue8m0) scale = round_up_pow2(scale);
    s_scale[tid] = scale;
    if (tid < ncols) scales[static_cast<int64_t>(b) * cols + c0 + tid] = scale;
  }
  __syncthreads();
  // Quantise the column slice into registers: 16 rows -> one 16-byte word.
  constexpr int CH = Q::ROWS_PER_PART / 16;
  uint4 qv[CH];
  if (col < ncols) {
    const float s = s_scale[col];
    const float rs = __frcp_rn(s);
    const bool finite_scale = isfinite(s);
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = k_begin + ch * 16 + i * 4;
        float f[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) f[j] = div_rn_by_scale(to_f(tile[k + j][col]), s, rs, finite_scale);
        const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[0], f[1]), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(f[2], f[3]), __NV_SATFINITE, __NV_E4M3);
        w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
      }
      qv[ch] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  __syncthreads();  // the input tile is no longer read: reuse it as FP8 staging

  // Stage column-major (column c's 128 bytes at c * QSTAGE_PITCH; the 16-byte
  // pad spreads the 16-byte stores of consecutive columns over all banks),
  // then write each column's bytes as full 128-byte lines, 8 threads a line.
  uint8_t* stage = reinterpret_cast<uint8_t*>(&tile[0][0]);
  if (col < ncols) {
#pragma unroll
    for (int ch = 0; ch < CH; ++ch)
      *reinterpret_cast<uint4*>(stage + col * QSTAGE_PITCH + k_begin + ch * 16) = qv[ch];
  }
  __syncthreads();
  for (int idx = tid; idx < ncols * 8; idx += QTHREADS) {
    const int c = idx >> 3;
    const int k0 = (idx & 7) * 16;
    if (k0 >= block_rows) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + c * QSTAGE_PITCH + k0);
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      const QuantDst& d = o == 0 ? d0 : d1;
      if (d.q == nullptr) continue;
      const int limit = d.zero_fill ? block_rows : rows;  // rows k < limit are written
      if (k0 >= limit) continue;
      const int64_t start = d.row_start != nullptr ? static_cast<int64_t>(__ldg(d.row_start + b))
                                                   : static_cast<int64_t>(b) * block_rows;
      uint8_t* dst = d.q + (c0 + c) * d.pitch + start + k0;
      if (k0 + 16 <= limit && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        for (int i = 0; i < 16 && k0 + i < limit; ++i) dst[i] = static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3)));
      }
    }
  }
}

}  // namespace

cudaError_t launch_quantize_1x128(const void* x, int x_dtype, int64_t cols, const int32_t* gather_idx,
                                  const int32_t* block_row_start, const int32_t* block_row_count,
                                  int64_t total_blocks, void* q, int64_t q_pitch, const int32_t* q_row_start,
                                  bool q_zero_fill, void* kq, int64_t kq_pitch, const int32_t* kq_row_start,
                                  float* scales, int block_rows, int64_t x_rows, bool ue8m0, cudaStream_t stream) {
  if (total_blocks == 0 || cols == 0) return cudaSuccess;
  const int strip = x_dtype == 0 ? QTile<__nv_bfloat16>::COLS : QTile<float>::COLS;
  const dim3 grid(static_cast<unsigned>(total_blocks), static_cast<unsigned>((cols + strip - 1) / strip));
  const QuantDst d0{static_cast<uint8_t*>(q), q_pitch, q_row_start, q_zero_fill};
  const QuantDst d1{static_cast<uint8_t*>(kq), kq_pitch, kq_row_start, false};
  if (x_dtype == 0) {
    const bool vec_ok = (cols % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    quantize_1x128_kernel<__nv_bfloat16><<<grid, QTHREADS, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), cols, gather_idx, block_row_start, block_row_count, d0, d1, scales,
        vec_ok, block_rows, x_rows, ue8m0);
  } else {
    const bool vec_ok = (cols % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    quantize_1x128_kernel<float><<<grid, QTHREADS, 0, stream>>>(static_cast<const float*>(x), cols, gather_idx,
                                                               block_row_start, block_row_count, d0, d1, scales,
                                                               vec_ok, block_rows, x_rows, ue8m0);
  }
  return cudaGetLastError();
}

}  // namespace wgrad
