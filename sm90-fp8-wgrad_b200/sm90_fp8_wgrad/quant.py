"""FP8 grouped Wgrad operands and the 1x128 quantiser.

``Fp8GroupedWgradOperand`` keeps the reference's data contract
(src/sm90_fp8_wgrad/quant.py:33-44): ``data`` is a logical [K_rows, cols]
float8_e4m3fn view with stride (1, pitch) -- physically [cols][pitch] bytes,
K contiguous, which is exactly the K-major operand layout tcgen05 reads --
and ``scales`` is fp32 [total_blocks, cols].

``quantize_grouped_wgrad_operand_128x1`` runs the CUDA quantiser
(``sm100_wgrad_quantize_1x128_ex``), replacing the reference's Triton kernel
(quant.py:105-167), for the padded and the packed layout;
``quantize_grouped_wgrad_operand_128x1_gather`` fuses the expert-major row
gather into it. Both are input preparation, outside the timed region.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .block_meta import WgradScaleBlockMeta
from .layout_mode import (
    LAYOUT_MODE_PACKED,
    LAYOUT_MODE_PADDED,
    PACKED_TAIL_TMA_ADAPTIVE32_64_128,
    PACKED_TAIL_TMA_ADAPTIVE32_64_TWOPHASE,
    PACKED_TAIL_TMA_ADAPTIVE64,
    PACKED_TAIL_TMA_MASKED128,
    resolve_packed_tail_tma_mode,
    resolve_wgrad_layout_mode,
)

FP8_MAX_E4M3 = 448.0
FP8_SCALE_EPS = 1.0e-12


@dataclass(frozen=True)
class Fp8GroupedWgradOperand:
    """FP8 operand: ``data`` logical [K_rows, cols] (stride (1, pitch)),
    ``scales`` [total_blocks, cols] fp32; ``kernel_data`` is the packed-layout
    launch copy [cols, K] (unused by the padded layout). ``scale_format``
    "ue8m0" marks scales that the quantiser rounded up to powers of two; the
    GEMM then applies them as tensor-core block scales (still stored as fp32).
    """

    data: torch.Tensor
    scales: torch.Tensor
    kernel_data: torch.Tensor | None = None
    scale_format: str = "fp32"


SCALE_FORMATS = ("fp32", "ue8m0")


def _check_scale_format(scale_format: str) -> int:
    if scale_format not in SCALE_FORMATS:
        raise RuntimeError(f"scale_format must be one of {SCALE_FORMATS}, got {scale_format!r}")
    return _lib.SCALE_UE8M0 if scale_format == "ue8m0" else _lib.SCALE_FP32


# ------------------------------------------------------- packed-layout helpers
# Same selection rules as the reference (quant.py:47-95): which K offsets,
# block starts and guard rows the packed launch copy uses.
def packed_kernel_data_uses_tma_slots(meta: WgradScaleBlockMeta) -> bool:
    return resolve_packed_tail_tma_mode(meta.packed_tail_tma_mode) != PACKED_TAIL_TMA_MASKED128


def packed_kernel_data_block_row_start(meta: WgradScaleBlockMeta) -> torch.Tensor:
    return meta.tma_block_row_start if packed_kernel_data_uses_tma_slots(meta) else meta.wgmma_block_row_start


def packed_kernel_data_cu_seqlens_k(meta: WgradScaleBlockMeta) -> torch.Tensor:
    return meta.tma_cu_seqlens_k if packed_kernel_data_uses_tma_slots(meta) else meta.wgmma_cu_seqlens_k


def packed_kernel_data_base_rows(meta: WgradScaleBlockMeta) -> int:
    return int(meta.tma_rows) if packed_kernel_data_uses_tma_slots(meta) else int(meta.wgmma_rows)


_GUARD_ROWS = {
    PACKED_TAIL_TMA_MASKED128: 127,
    PACKED_TAIL_TMA_ADAPTIVE64: 63,
    PACKED_TAIL_TMA_ADAPTIVE32_64_128: 127,
    PACKED_TAIL_TMA_ADAPTIVE32_64_TWOPHASE: 31,
}


def packed_kernel_data_guard_rows(meta: WgradScaleBlockMeta) -> int:
    if packed_kernel_data_base_rows(meta) <= 0:
        return 0
    return _GUARD_ROWS[resolve_packed_tail_tma_mode(meta.packed_tail_tma_mode)]


def packed_kernel_data_storage_rows(meta: WgradScaleBlockMeta) -> int:
    return packed_kernel_data_base_rows(meta) + packed_kernel_data_guard_rows(meta)


def operand_pitch(k_rows: int) -> int:
    """K pitch of an operand: a multiple of 128 bytes, at least 128
    (reference quant.py:222-230)."""
    return max(128, (int(k_rows) + 127) // 128 * 128)


def _quantize(x: torch.Tensor, gather_idx: torch.Tensor | None, meta: WgradScaleBlockMeta,
              layout_mode: str | None, scale_format: str = "fp32") -> Fp8GroupedWgradOperand:
    """Shared body of the two quantiser entry points (one CUDA launch)."""
    fmt = _check_scale_format(scale_format)
    if x.ndim != 2:
        raise RuntimeError(f"expected x_grouped [valid_TK,N], got {tuple(x.shape)}")
    if not x.is_cuda:
        raise RuntimeError("x_grouped must be CUDA")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError(f"x_grouped must be bf16 or fp32, got {x.dtype}")
    if not x.is_contiguous():
        x = x.contiguous()
    n = int(x.shape[1])
    if gather_idx is None and int(meta.valid_rows) != int(x.shape[0]):
        raise RuntimeError("meta.cu_seqlens_k[-1] must match x_grouped rows")
    if int(meta.padded_rows) != int(meta.total_blocks) * int(meta.block_k):
        raise RuntimeError("metadata padded_rows must equal total_blocks * block_k")
    mode = resolve_wgrad_layout_mode(layout_mode)
    block_rows = int(meta.block_k)
    if block_rows not in (32, 64, 128):
        raise RuntimeError(f"meta.block_k must be 32, 64 or 128, got {block_rows}")
    if block_rows != 128 and mode != LAYOUT_MODE_PADDED:
        raise RuntimeError("32/64-row scale blocks use the padded layout")
    dev = x.device
    scales = torch.empty((int(meta.total_blocks), n), device=dev, dtype=torch.float32)
    args = _lib.Sm100WgradQuantArgs()
    args.x = x.data_ptr()
    args.x_dtype = 0 if x.dtype == torch.bfloat16 else 1
    args.cols = n
    args.gather_idx = gather_idx.data_ptr() if gather_idx is not None else None
    args.block_row_start = meta.block_row_start.data_ptr()
    args.block_row_count = meta.block_row_count.data_ptr()
    args.total_blocks = int(meta.total_blocks)
    args.scales = scales.data_ptr()
    args.block_rows = block_rows
    args.x_rows = int(x.shape[0])
    args.scale_format = fmt
    kernel_q = None
    if mode == LAYOUT_MODE_PADDED:
        q_rows = int(meta.padded_rows)
        pitch = operand_pitch(q_rows)
        storage = torch.empty((n, pitch), device=dev, dtype=torch.float8_e4m3fn)
        if pitch > q_rows:
            storage[:, q_rows:].view(torch.uint8).zero_()
        args.q_row_start = None           # row 128 b + k
        args.q_zero_fill = 1              # rows past each block's count are zero
    else:
        assert mode == LAYOUT_MODE_PACKED
        # reference quant.py:211-247: compact logical data on valid rows (128-byte
        # K pitch) plus the zero-initialised launch copy with its TMA guard rows.
        q_rows = int(meta.valid_rows)
        pitch = operand_pitch(q_rows)
        storage = torch.empty((n, pitch), device=dev, dtype=torch.float8_e4m3fn)
        kernel_rows = packed_kernel_data_storage_rows(meta)
        aligned_k = max(16, (kernel_rows + 15) // 16 * 16)
        kernel_q = torch.zeros((n, aligned_k), device=dev, dtype=torch.float8_e4m3fn)
        args.q_row_start = meta.block_row_start.data_ptr()
        args.q_zero_fill = 0
        args.kq_data = kernel_q.data_ptr()
        args.kq_pitch = aligned_k
        args.kq_row_start = packed_kernel_data_block_row_start(meta).data_ptr()
    args.q_data = storage.data_ptr()
    args.q_pitch = pitch
    q = storage.as_strided((q_rows, n), (1, pitch))
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream().cuda_stream
        _lib.raise_pending_device_error()
        _lib.check(lib.sm100_wgrad_quantize_1x128_ex(ctypes.byref(args), stream), "sm100_wgrad_quantize_1x128_ex")
    return Fp8GroupedWgradOperand(q, scales, kernel_data=kernel_q, scale_format=scale_format)


def quantize_grouped_wgrad_operand_128x1(
    x_grouped: torch.Tensor,
    meta: WgradScaleBlockMeta,
    *,
    block_n: int = 32,
    layout_mode: str | None = None,
    scale_format: str = "fp32",
) -> Fp8GroupedWgradOperand:
    """Quantise expert-major grouped rows [valid_rows, cols] (BF16 or fp32)
    into an FP8 operand with 1x128 fp32 scales (reference quant.py:175-270).

    ``scale_format`` "fp32" (default) is the reference's scale
    max(amax / 448, 1e-12); "ue8m0" rounds that scale up to the next power of
    two (an extension: the reference has no such mode), so that
    ``fp8_grouped_wgrad_sm90`` can apply it as a tensor-core block scale.

    ``layout_mode`` "padded" stores each expert in whole 128-row slots
    (zero-filled tails); "packed" stores ``data`` on the valid rows only and a
    launch copy ``kernel_data`` [cols, K] at the packed tail policy's block
    starts (``wgmma_block_row_start`` for masked128) with its guard rows, as
    the reference does. ``block_n`` is accepted for signature compatibility
    (the CUDA kernel tiles 64 columns per CTA).
    """
    del block_n
    return _quantize(x_grouped, None, meta, layout_mode, scale_format)


def quantize_grouped_wgrad_operand_128x1_gather(
    x: torch.Tensor,
    gather_idx: torch.Tensor,
    meta: WgradScaleBlockMeta,
    *,
    layout_mode: str | None = None,
    scale_format: str = "fp32",
) -> Fp8GroupedWgradOperand:
    """Gather + quantise in one pass: row r of the expert-major operand is row
    ``gather_idx[r]`` of the token-major activation ``x`` [tokens, cols].

    Equal, byte for byte, to ``quantize_grouped_wgrad_operand_128x1(x[gather_idx], meta)``
    without materialising the grouped BF16 copy (the reference harness builds
    it with a separate gather, synthetic.py:132-150 and :243-244).
    """
    if gather_idx.ndim != 1 or not gather_idx.is_cuda:
        raise RuntimeError("gather_idx must be a 1-D CUDA tensor")
    if int(gather_idx.numel()) != int(meta.valid_rows):
        raise RuntimeError(f"gather_idx has {int(gather_idx.numel())} rows, metadata {int(meta.valid_rows)}")
    if gather_idx.device != x.device:
        raise RuntimeError("gather_idx and x must be on the same device")
    idx = gather_idx if gather_idx.dtype == torch.int32 else gather_idx.to(torch.int32)
    return _quantize(x, idx.contiguous(), meta, layout_mode, scale_format)


def quantize_grouped_wgrad_operand_tail_k(
    x_grouped: torch.Tensor,
    tail_indices: torch.Tensor,
    tail_meta: WgradScaleBlockMeta,
    *,
    block_n: int = 32,
) -> Fp8GroupedWgradOperand:
    """Quantise compact per-expert tail rows (reference quant.py:273-307).

    Row r of the compact tail operand is row ``tail_indices[r]`` of the
    expert-major ``x_grouped``; it is quantised with ``tail_meta.block_k``-row
    (32 or 64) scale blocks into the padded layout, block b at rows
    [block_k * b, block_k * (b + 1)). The reference gathers with
    ``index_select`` and then quantises; here the gather is fused into the
    quantiser's loads. An index outside ``x_grouped`` reads zeros and sets
    device error 5 (``sm100_wgrad_device_error``) instead of faulting.
    """
    del block_n
    if tail_indices.ndim != 1:
        raise RuntimeError(f"expected tail_indices [tail_rows], got {tuple(tail_indices.shape)}")
    if not tail_indices.is_cuda:
        raise RuntimeError("tail_indices must be CUDA")
    if int(tail_meta.block_k) not in (32, 64):
        raise RuntimeError(f"tail_meta.block_k must be 32 or 64, got {tail_meta.block_k}")
    if x_grouped.ndim != 2:
        raise RuntimeError(f"expected x_grouped [valid_TK,N], got {tuple(x_grouped.shape)}")
    if not x_grouped.is_cuda:
        raise RuntimeError("x_grouped must be CUDA")
    if int(tail_meta.valid_rows) != int(tail_indices.numel()):
        raise RuntimeError("tail_meta.valid_rows must match compact tail source rows")
    if tail_indices.device != x_grouped.device:
        raise RuntimeError("tail_indices and x_grouped must be on the same device")
    idx = tail_indices if tail_indices.dtype == torch.int32 else tail_indices.to(torch.int32)
    return _quantize(x_grouped, idx.contiguous(), tail_meta, LAYOUT_MODE_PADDED)
