"""FP8 grouped Wgrad operands and the 1x128 quantiser.

``Fp8GroupedWgradOperand`` keeps the reference's data contract
(src/sm90_fp8_wgrad/quant.py:33-44): ``data`` is a logical [K_rows, cols]
float8_e4m3fn view with stride (1, pitch) -- physically [cols][pitch] bytes,
K contiguous, which is exactly the K-major operand layout tcgen05 reads --
and ``scales`` is fp32 [total_blocks, cols].

``quantize_grouped_wgrad_operand_128x1`` runs the CUDA quantiser
(``sm100_wgrad_quantize_1x128``), replacing the reference's Triton kernel
(quant.py:105-167). It is input preparation, outside the timed region.
"""
from __future__ import annotations

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
    launch copy [cols, K] (unused by the padded layout)."""

    data: torch.Tensor
    scales: torch.Tensor
    kernel_data: torch.Tensor | None = None


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


def quantize_grouped_wgrad_operand_128x1(
    x_grouped: torch.Tensor,
    meta: WgradScaleBlockMeta,
    *,
    block_n: int = 32,
    layout_mode: str | None = None,
) -> Fp8GroupedWgradOperand:
    """Quantise expert-major grouped rows [valid_rows, cols] (BF16 or fp32)
    into the padded FP8 operand layout with 1x128 fp32 scales.

    ``block_n`` is accepted for signature compatibility (the CUDA kernel tiles
    64 columns per CTA).
    """
    del block_n
    if x_grouped.ndim != 2:
        raise RuntimeError(f"expected x_grouped [valid_TK,N], got {tuple(x_grouped.shape)}")
    if not x_grouped.is_cuda:
        raise RuntimeError("x_grouped must be CUDA")
    if x_grouped.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError(f"x_grouped must be bf16 or fp32, got {x_grouped.dtype}")
    if not x_grouped.is_contiguous():
        x_grouped = x_grouped.contiguous()
    valid_tk, n = map(int, x_grouped.shape)
    if int(meta.valid_rows) != valid_tk:
        raise RuntimeError("meta.cu_seqlens_k[-1] must match x_grouped rows")
    if int(meta.padded_rows) != int(meta.total_blocks) * int(meta.block_k):
        raise RuntimeError("metadata padded_rows must equal total_blocks * block_k")
    mode = resolve_wgrad_layout_mode(layout_mode)
    if mode == LAYOUT_MODE_PACKED:
        raise RuntimeError("packed layout is not implemented by the B200 engine yet; use layout_mode='padded'")
    assert mode == LAYOUT_MODE_PADDED

    q_rows = int(meta.padded_rows)
    pitch = operand_pitch(q_rows)
    storage = torch.empty((n, pitch), device=x_grouped.device, dtype=torch.float8_e4m3fn)
    if pitch > q_rows:
        storage[:, q_rows:].view(torch.uint8).zero_()
    q = storage.as_strided((q_rows, n), (1, pitch))
    scales = torch.empty((int(meta.total_blocks), n), device=x_grouped.device, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(x_grouped.device):
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(
            lib.sm100_wgrad_quantize_1x128(
                x_grouped.data_ptr(), 0 if x_grouped.dtype == torch.bfloat16 else 1, valid_tk, n,
                meta.block_row_start.data_ptr(), meta.block_row_count.data_ptr(), int(meta.total_blocks),
                storage.data_ptr(), pitch, scales.data_ptr(), stream,
            ),
            "sm100_wgrad_quantize_1x128",
        )
    return Fp8GroupedWgradOperand(q, scales, kernel_data=None)


def quantize_grouped_wgrad_operand_tail_k(
    x_grouped: torch.Tensor,
    tail_indices: torch.Tensor,
    tail_meta: WgradScaleBlockMeta,
    *,
    block_n: int = 32,
) -> Fp8GroupedWgradOperand:
    """Quantise compact per-expert tail rows (reference quant.py:273-307)."""
    if tail_indices.ndim != 1:
        raise RuntimeError(f"expected tail_indices [tail_rows], got {tuple(tail_indices.shape)}")
    if not tail_indices.is_cuda:
        raise RuntimeError("tail_indices must be CUDA")
    if int(tail_meta.block_k) not in (32, 64):
        raise RuntimeError(f"tail_meta.block_k must be 32 or 64, got {tail_meta.block_k}")
    raise RuntimeError("tail_k operands use 32/64-row scale blocks, which the B200 engine does not run")
