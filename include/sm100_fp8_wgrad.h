/*
 * sm100_fp8_wgrad.h -- C ABI of the B200 (sm_100a) grouped FP8 Wgrad engine.
 *
 * The engine computes, for every expert e of a sparse MoE layer,
 *
 *   out[e, m, n] = sum_{b in blocks(e)} sum_{k in b}
 *                    lhs_q[k, m] * lhs_s[b, m] * rhs_q[k, n] * rhs_s[b, n]
 *
 * where the contraction index k runs over the expert's token rows, grouped in
 * 128-row scale blocks b, lhs_q / rhs_q are FP8 e4m3 and lhs_s / rhs_s are fp32.
 * The two MoE weight gradients are two calls:
 *   dW_down[e]    = grad_y_e^T       @ hidden_e   (lhs = grad_y,       rhs = hidden)
 *   dW_gate_up[e] = grad_gate_up_e^T @ x_e        (lhs = grad_gate_up, rhs = x)
 *
 * Everything here is plain C: device pointers, sizes and a CUDA stream passed
 * as void*. Every entry point returns an int status (SM100_WGRAD_OK == 0) and
 * never synchronises the stream. The caller owns and allocates all buffers.
 *
 * Memory layouts (identical to the reference operator contract):
 *   FP8 operand data  : [cols][pitch] bytes, K (token rows) contiguous; the
 *                       reference exposes it as a logical [K_rows, cols] view
 *                       with stride (1, pitch). pitch % 16 == 0.
 *   scales            : [total_blocks][cols] fp32, row-major.
 *   out               : [E][M][N] bf16 or fp32, row-major (contiguous).
 *   block_offsets     : [E+1] int32, prefix sum of ceil(rows_e / 128).
 *   k_row_offsets     : [E+1] int32, first operand K row of each expert
 *                       (padded layout: 128 * block_offsets).
 */
#ifndef SM100_FP8_WGRAD_H_
#define SM100_FP8_WGRAD_H_

#include <stdint.h>

#if defined(__GNUC__)
#define SM100_WGRAD_API __attribute__((visibility("default")))
#else
#define SM100_WGRAD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define SM100_WGRAD_OK 0
#define SM100_WGRAD_ERR_INVALID_ARG 1      /* null pointer, bad size, bad stride or alignment */
#define SM100_WGRAD_ERR_UNSUPPORTED_ARCH 2 /* device is not compute capability 10.0 (B200)    */
#define SM100_WGRAD_ERR_LAUNCH 3           /* CUDA launch / attribute / driver call failed   */
#define SM100_WGRAD_ERR_TENSOR_MAP 4       /* cuTensorMapEncodeTiled rejected a descriptor   */
#define SM100_WGRAD_ERR_DEVICE_TIMEOUT 5   /* a device-side bounded wait expired             */
#define SM100_WGRAD_ERR_UNSUPPORTED 6      /* shape or option outside the supported envelope */

#define SM100_WGRAD_OUT_BF16 0
#define SM100_WGRAD_OUT_F32 1

/* Tile configurations selectable through Sm100WgradArgs.tile_config.
 * AUTO picks the 256x256 CTA pair (below) when the experts average at least
 * 8 128-row blocks and each expert has at least 64 256x256 output tiles, and
 * a single-CTA tile otherwise, its N width by shape; AUTO and 128x256 pick the
 * number of promotion warps of the 256-wide single-CTA tile by K depth (16
 * when the experts average few 128-row blocks, 8 otherwise); the _W8 / _W16
 * forms force it. */
#define SM100_WGRAD_TILE_AUTO 0
#define SM100_WGRAD_TILE_128x256 1
#define SM100_WGRAD_TILE_128x128 2
#define SM100_WGRAD_TILE_128x256_W8 3
#define SM100_WGRAD_TILE_128x256_W16 4
#define SM100_WGRAD_TILE_128x128_2CTA 5   /* 128x128 tile, two CTAs (pipelines) per SM */
#define SM100_WGRAD_TILE_128x192_W12 6    /* 128x192 tile, 12 promotion warps          */
/* 128x192 tile for UE8M0 scales: every scale must be a positive power of two
 * (the quantiser's scale_format 1); the tensor core applies them as E8M0 block
 * scales (tcgen05.mma kind::mxf8f6f4.block_scale) and no fp32 promotion runs.
 * A scale with mantissa bits set is taken as 1.0 and sets device error 6
 * (reported by sm100_wgrad_poll_device_error / sm100_wgrad_device_error).
 * Never chosen by the C ABI's AUTO; the Python operator selects it for AUTO
 * when both operands carry scale_format == "ue8m0". */
#define SM100_WGRAD_TILE_128x192_UE8M0 7
/* 256x256 tile over a pair of CTAs (a cluster of two on neighbouring SMs):
 * tcgen05.mma cta_group::2 with each CTA loading its 128 rows of lhs and half
 * of the rhs tile, 8 promotion warps per CTA. */
#define SM100_WGRAD_TILE_256x256_PAIR 8
#define SM100_WGRAD_TILE_256x256_PAIR_W16 9   /* the same with 16 promotion warps per CTA */
/* 256x256 tile over a CTA pair whose per-block scale product lhs_s (x) rhs_s
 * is computed by a TF32 UMMA on hi/lo splits of the scales, so the fp32
 * promotion is one fused multiply-add per element. Needs a device workspace
 * of sm100_wgrad_workspace_bytes() bytes (256-byte aligned) for the split
 * scales, written by the call itself. */
#define SM100_WGRAD_TILE_256x256_SP 10
#define SM100_WGRAD_TILE_256x256_SP_W16 11   /* the same with 16 promotion warps per CTA */

typedef struct Sm100WgradArgs {
  const void* lhs_data;      /* FP8 e4m3 [M][lhs_pitch]                              */
  int64_t lhs_pitch;         /* bytes between consecutive columns (m) of lhs        */
  const float* lhs_scales;   /* [total_blocks][M]                                    */
  const void* rhs_data;      /* FP8 e4m3 [N][rhs_pitch]                              */
  int64_t rhs_pitch;         /* bytes between consecutive columns (n) of rhs        */
  const float* rhs_scales;   /* [total_blocks][N]                                    */
  void* out;                 /* [E][M][N]                                            */
  int32_t out_dtype;         /* SM100_WGRAD_OUT_BF16 or SM100_WGRAD_OUT_F32          */
  int32_t accumulate;        /* 0: out = result, 1: out += result                    */
  int64_t num_experts;       /* E                                                    */
  int64_t m;                 /* M (lhs columns)                                      */
  int64_t n;                 /* N (rhs columns)                                      */
  int64_t k_rows;            /* operand K extent (rows stored per column)            */
  int64_t total_blocks;      /* number of 128-row scale blocks                       */
  const int32_t* block_offsets;  /* device [E+1]                                     */
  const int32_t* k_row_offsets;  /* device [E+1]                                     */
  const int32_t* expert_order;   /* device [E] schedule order (LPT), or NULL = 0..E-1 */
  int32_t tile_config;       /* SM100_WGRAD_TILE_*                                   */
  int32_t max_ctas;          /* persistent grid cap, 0 = one CTA per SM              */
  void* workspace;           /* device scratch, 256-byte aligned (see
                                sm100_wgrad_workspace_bytes); NULL when it needs 0   */
  int64_t workspace_bytes;   /* size of workspace                                    */
} Sm100WgradArgs;

/*
 * Grouped FP8 Wgrad GEMM (one launch of the persistent tcgen05 kernel).
 * Replaces fp8_grouped_wgrad_sm90_impl, src/sm90_fp8_wgrad/gemm_sm90.py:5526-5899
 * (the TVM-FFI launch of the CuTe-DSL kernel at gemm_sm90.py:5886), called from
 * fp8_grouped_wgrad_sm90, src/sm90_fp8_wgrad/interface.py:243-255.
 * Unlike the reference (gemm_sm90.py:5676) it performs no device->host read.
 * Layouts: padded (k_row_offsets = 128 * block_offsets) or the reference's
 * packed mode (k_row_offsets = wgmma_cu_seqlens_k, 32-row aligned expert
 * starts, operands = kernel_data with >= 127 zero guard rows); an expert's last
 * scale block multiplies only its ceil(rows / 32) valid 32-row K slices.
 * A launch over an expert sub-range [e0, e1) passes num_experts = e1 - e0 and
 * block_offsets / k_row_offsets / out offset by e0 (their values stay absolute).
 * The product library reads no environment variable. A library built with
 * -DWGRAD_DEBUG_MODES=1 (sm100_wgrad_build_flags) reads, per launch,
 * KERNEL_LAB_WGRAD_KERNEL_MODE (the reference's known-answer modes coord_m /
 * coord_n / scale_only / unscaled) and SM100_WGRAD_DEBUG_INJECT (test-only).
 */
SM100_WGRAD_API int sm100_fp8_grouped_wgrad(const Sm100WgradArgs* args, void* stream);

/*
 * Device workspace (bytes) that sm100_fp8_grouped_wgrad needs for these
 * arguments: total_blocks * (m + n) * 16 (+ alignment) for
 * SM100_WGRAD_TILE_256x256_SP(_W16), 0 for every other tile configuration. The
 * reference allocates its scratch inside the launcher (gemm_sm90.py:5526-5899,
 * through the framework's allocator); here the caller owns it.
 */
SM100_WGRAD_API int sm100_wgrad_workspace_bytes(const Sm100WgradArgs* args, int64_t* bytes);

/*
 * The scale-product GEMM (SM100_WGRAD_TILE_256x256_SP, or _SP_W16; AUTO means
 * _SP) for callers that cannot allocate device memory, such as a host binding
 * that owns only the buffers it was given, or a process that reserves all of
 * its device memory up front. It needs no workspace: the split scales live in
 * a 64 MiB array compiled into the library (every GPU that loads the library
 * holds it until exit), so args->workspace is ignored and a problem whose
 * sm100_wgrad_workspace_bytes exceeds 64 MiB is refused with
 * SM100_WGRAD_ERR_UNSUPPORTED. All calls share that array: calls that overlap
 * on the GPU (other streams, other threads on the same device) race, so
 * serialise them. The first call on a device looks up the array's device
 * address (make it before any stream capture). It allocates nothing, and
 * device errors of its launches are read with sm100_wgrad_device_error.
 * No counterpart in the reference: its launcher always allocates through the
 * framework.
 */
SM100_WGRAD_API int sm100_fp8_grouped_wgrad_noalloc(const Sm100WgradArgs* args, void* stream);

/*
 * 1x128 FP8 quantiser: per (128-row block b, column c)
 *   amax = max_{k < row_count[b]} |x[row_start[b] + k, c]|
 *   scale[b, c] = max(amax / 448, 1e-12)
 *   q[c][128 b + k] = e4m3_rne_satfinite(x / scale)  (0 for k >= row_count[b])
 * x is BF16 (x_dtype 0) or fp32 (x_dtype 1) row-major [valid_rows][cols].
 * Replaces the Triton kernel _quantize_grouped_wgrad_128x1_kernel,
 * src/sm90_fp8_wgrad/quant.py:105-167, launched from
 * quantize_grouped_wgrad_operand_128x1, quant.py:175-270 (padded layout).
 */
SM100_WGRAD_API int sm100_wgrad_quantize_1x128(const void* x, int32_t x_dtype, int64_t valid_rows, int64_t cols,
                               const int32_t* block_row_start, const int32_t* block_row_count,
                               int64_t total_blocks, void* q_data, int64_t q_pitch, float* scales,
                               void* stream);

/*
 * 1x128 FP8 quantiser, general form: the same math as sm100_wgrad_quantize_1x128
 * with the destinations of the reference's two layout modes and an optional
 * row gather.
 *   x row of grouped row r : gather_idx ? gather_idx[r] : r     (token-major
 *                            activation read through the MoE routing gather,
 *                            fusing the gather of synthetic.py:132-150 into
 *                            the quantiser; NULL = x is already grouped)
 *   q_data                 : byte k of block b, column c at
 *                            q[c * q_pitch + q_row_start[b] + k]
 *                            (q_row_start NULL = 128 b: the padded layout);
 *                            q_zero_fill != 0 also writes rows k >= count as 0
 *   kq_data (optional)     : second copy at kq[c * kq_pitch + kq_row_start[b] + k],
 *                            valid rows only (the caller zero-fills the buffer)
 * Padded layout: quant.py:222-247; packed layout (data at block_row_start,
 * kernel_data at wgmma_block_row_start): quant.py:196-266 and the Triton
 * kernel's PACKED_LAYOUT / STORE_KERNEL_DATA branches, quant.py:129-167.
 */
typedef struct Sm100WgradQuantArgs {
  const void* x;                  /* BF16 (x_dtype 0) or fp32 (1), row-major [x_rows][cols] */
  int32_t x_dtype;
  int64_t cols;
  const int32_t* gather_idx;      /* [valid_rows] or NULL                                 */
  const int32_t* block_row_start; /* [total_blocks] first grouped row of each block       */
  const int32_t* block_row_count; /* [total_blocks] valid rows of each block              */
  int64_t total_blocks;
  void* q_data;
  int64_t q_pitch;
  const int32_t* q_row_start;     /* [total_blocks] or NULL                               */
  int32_t q_zero_fill;
  void* kq_data;                  /* or NULL                                              */
  int64_t kq_pitch;
  const int32_t* kq_row_start;    /* [total_blocks], required with kq_data                */
  float* scales;                  /* [total_blocks][cols]                                 */
  int32_t block_rows;             /* rows per scale block: 128 (0 means 128), or 32 / 64 for
                                     the compact tail operands of quant.py:273-307        */
  int64_t x_rows;                 /* rows of x; required with gather_idx (an index outside
                                     [0, x_rows) reads zeros and sets device error 5)      */
  int32_t scale_format;           /* 0: fp32 scale max(amax / 448, 1e-12) as the reference;
                                     1: that scale rounded up to a power of two (UE8M0, for
                                     SM100_WGRAD_TILE_128x192_UE8M0)                       */
} Sm100WgradQuantArgs;

SM100_WGRAD_API int sm100_wgrad_quantize_1x128_ex(const Sm100WgradQuantArgs* args, void* stream);

/*
 * Scale-block metadata builder (device side, no host sync).
 * From cu_seqlens_k [E+1] it writes the per-expert arrays
 *   blocks_per_expert[E], block_offsets[E+1], padded_cu_seqlens_k[E+1],
 *   wgmma_cu_seqlens_k[E+1] (32-row aligned), tail_valid_rows[E],
 *   tail_wgmma_atoms[E], tail_copy_k[E], has_tail[E] (uint8), expert_order[E]
 * and the per-block arrays (capacity block_capacity entries)
 *   block_row_start, block_row_count, wgmma_block_row_start
 * plus totals[5] = {valid_rows, padded_rows, wgmma_rows, total_blocks, status}
 * (status != 0 means cu_seqlens_k was not monotonic or block_capacity was too
 * small). Replaces build_wgrad_scale_block_meta,
 * src/sm90_fp8_wgrad/block_meta.py:252-349 (CPU loops at :288-294).
 */
typedef struct Sm100WgradMetaOut {
  int32_t* blocks_per_expert;
  int32_t* block_offsets;
  int32_t* padded_cu_seqlens_k;
  int32_t* wgmma_cu_seqlens_k;
  int32_t* tail_valid_rows;
  int32_t* tail_wgmma_atoms;
  int32_t* tail_copy_k;
  uint8_t* has_tail;
  int32_t* expert_order;
  int32_t* block_row_start;
  int32_t* block_row_count;
  int32_t* wgmma_block_row_start;
  int64_t block_capacity;
  int64_t* totals;
} Sm100WgradMetaOut;

SM100_WGRAD_API int sm100_wgrad_build_meta(const int32_t* cu_seqlens_k, int64_t num_experts, const Sm100WgradMetaOut* out,
                           void* stream);

/* Reads and clears the device error word of the current device (synchronous;
 * diagnostics only, never call it inside a timed region). Writes one of the
 * device error codes to *code: 0 none; 1, 2, 3 a bounded wait of the GEMM's
 * producer, MMA or epilogue role expired; 4 bad tile; 5 a quantiser gather
 * index outside [0, x_rows); 6 a scale given to the UE8M0 kernel that is not a
 * positive power of two. The first error since the last read is kept. */
SM100_WGRAD_API int sm100_wgrad_device_error(int32_t* code);

/* Non-blocking form of sm100_wgrad_device_error: reads (and clears) a pinned,
 * host-mapped copy of the device error word that every failing kernel writes
 * with a system-scope fence, so a caller learns of a device-side failure of an
 * earlier launch (a bounded wait that gave up, a bad gather index, a non-UE8M0
 * scale) without synchronising the stream: *code is 0 when no launch that has
 * finished so far recorded an error since the last poll or read. The reference
 * has no device error channel (its failures surface as exceptions of the
 * framework). The mirror is set up by the first call of any entry point on a
 * device (a synchronous symbol copy: make that first call outside any CUDA
 * stream capture); returns SM100_WGRAD_ERR_UNSUPPORTED if pinned mapped memory
 * was unavailable. */
SM100_WGRAD_API int sm100_wgrad_poll_device_error(int32_t* code);

/* Compile-time features of the loaded library (bit mask). */
#define SM100_WGRAD_BUILD_DEBUG_MODES 1 /* known-answer modes + test-only failure injection */
#define SM100_WGRAD_BUILD_PROFILE 2     /* per-role cycle counters                          */
SM100_WGRAD_API int sm100_wgrad_build_flags(void);

/* Per-role cycle counters of the grouped GEMM, summed over CTAs since the last
 * read (synchronous; reads and clears). Only a library built with
 * -DWGRAD_PROFILE=1 (build_ext.py --profile) records them; the product build
 * returns SM100_WGRAD_ERR_UNSUPPORTED. 24 slots. 0-10: producer wait for a
 * stage, producer wait for a scale stage, MMA wait, MMA issue, promotion wait,
 * promotion, tile store, wait for the previous store, K blocks, tiles, CTAs;
 * 11-12: UE8M0 scale-factor writer conversion and publication; 13: operand
 * stage latency (TMA issue to the MMA warp seeing the stage full); 14-15: UE8M0
 * writer vote and scale loads; 16: UE8M0 MMA wait for a free accumulator. The
 * UE8M0 kernel records its scale-factor writer in slots 4-5 and its epilogue's
 * accumulator wait in slot 7. 17: cycles from a CTA's start to its exit. */
SM100_WGRAD_API int sm100_wgrad_profile_counters(uint64_t* counters, int32_t n);

/* Human-readable text of a status code (static storage). */
SM100_WGRAD_API const char* sm100_wgrad_status_string(int status);

/* Library version, e.g. "0.1.0". */
SM100_WGRAD_API const char* sm100_wgrad_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SM100_FP8_WGRAD_H_ */
