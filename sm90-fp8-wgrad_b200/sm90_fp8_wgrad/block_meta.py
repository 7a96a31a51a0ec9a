"""Scale-block metadata for grouped FP8 Wgrad.

The dataclasses keep the reference's field names and meaning
(src/sm90_fp8_wgrad/block_meta.py:16-90) so harness code that reads them works
unchanged. ``build_wgrad_scale_block_meta`` runs on the GPU: one launch of the
CUDA metadata kernel (``sm100_wgrad_build_meta``) replaces the reference's
Python loops (block_meta.py:288-294), followed by one small device->host read
of the totals (the reference also syncs here, block_meta.py:273; metadata is
built outside the timed Wgrad region).

Added field: ``expert_order`` -- the tile-schedule order the GEMM walks
(experts by descending 128-row block count, longest first).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .layout_mode import (
    PACKED_TAIL_TMA_ADAPTIVE32_64_128,
    PACKED_TAIL_TMA_ADAPTIVE32_64_TWOPHASE,
    PACKED_TAIL_TMA_ADAPTIVE64,
    PACKED_TAIL_TMA_MASKED128,
    resolve_packed_tail_tma_mode,
)

BLOCK_K = 128
WGMMA_K_ALIGNMENT = 32


@dataclass(frozen=True)
class WgradScaleBlockMeta:
    """Per-expert 128-row scale-block layout of the grouped Wgrad operands.

    ``cu_seqlens_k``        valid expert-major row offsets [E+1]
    ``padded_cu_seqlens_k`` 128 * block_offsets: K offsets of the padded layout
    ``wgmma_cu_seqlens_k``  packed offsets with each expert rounded up to 32 rows
    ``tma_cu_seqlens_k``    packed offsets of the tail-copy policy
    ``block_offsets``       prefix sum of ceil(rows / 128) [E+1]
    ``block_row_start/count`` first valid row and valid row count of each block
    """

    cu_seqlens_k: torch.Tensor
    padded_cu_seqlens_k: torch.Tensor
    wgmma_cu_seqlens_k: torch.Tensor
    tma_cu_seqlens_k: torch.Tensor
    blocks_per_expert: torch.Tensor
    block_offsets: torch.Tensor
    block_row_start: torch.Tensor
    wgmma_block_row_start: torch.Tensor
    tma_block_row_start: torch.Tensor
    block_row_count: torch.Tensor
    tail_valid_rows: torch.Tensor
    tail_wgmma_atoms: torch.Tensor
    tail_copy_k: torch.Tensor
    has_tail: torch.Tensor
    block_k: int
    valid_rows: int
    padded_rows: int
    wgmma_rows: int
    tma_rows: int
    wgmma_k_alignment: int
    total_blocks: int
    packed_tail_tma_mode: str
    expert_order: torch.Tensor | None = None

    @property
    def num_experts(self) -> int:
        return int(self.cu_seqlens_k.numel()) - 1


@dataclass(frozen=True)
class WgradFullBlockSplit:
    """Full 128-row blocks only, plus compact indices of each expert's ragged tail."""

    full_meta: WgradScaleBlockMeta
    tail_indices: torch.Tensor
    tail_cu_seqlens_k: torch.Tensor
    full_rows: int
    tail_rows: int


@dataclass(frozen=True)
class WgradTailBlockMeta:
    """Compact metadata of each expert's final partial block (tail rows only)."""

    meta: WgradScaleBlockMeta
    tail_indices: torch.Tensor
    tail_rows: int
    tail_block_k: int


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.int32).contiguous()


def _tail_copy_k(tail_rows: torch.Tensor, mode: str) -> torch.Tensor:
    """Rows a tail TMA copy moves under each packed-tail policy
    (reference block_meta.py:92-121)."""
    mode = resolve_packed_tail_tma_mode(mode)
    zero = torch.zeros_like(tail_rows)
    has = tail_rows != 0
    if mode == PACKED_TAIL_TMA_MASKED128:
        k = torch.full_like(tail_rows, 128)
    elif mode == PACKED_TAIL_TMA_ADAPTIVE64:
        k = torch.where(tail_rows <= 64, 64, 128).to(tail_rows.dtype)
    elif mode == PACKED_TAIL_TMA_ADAPTIVE32_64_128:
        k = torch.where(tail_rows <= 32, 32, torch.where(tail_rows <= 64, 64, 128)).to(tail_rows.dtype)
    elif mode == PACKED_TAIL_TMA_ADAPTIVE32_64_TWOPHASE:
        k = (tail_rows + 31) // 32 * 32
    else:  # pragma: no cover - resolve_packed_tail_tma_mode rejects it
        raise RuntimeError(f"unsupported packed tail TMA mode: {mode!r}")
    return torch.where(has, k, zero)


def _exclusive_cumsum(x: torch.Tensor) -> torch.Tensor:
    out = torch.zeros(x.numel() + 1, dtype=torch.int64, device=x.device)
    if x.numel():
        out[1:] = torch.cumsum(x.to(torch.int64), 0)
    return out


def _block_starts(per_expert_start: torch.Tensor, blocks: torch.Tensor, total_blocks: int, step: int) -> torch.Tensor:
    """start[b] = per_expert_start[e(b)] + step * (b - block_offsets[e(b)])."""
    e_of_block = torch.repeat_interleave(
        torch.arange(blocks.numel(), device=blocks.device), blocks.to(torch.int64), output_size=total_blocks
    )
    offsets = _exclusive_cumsum(blocks)
    j = torch.arange(total_blocks, device=blocks.device, dtype=torch.int64) - offsets[e_of_block]
    return per_expert_start[e_of_block].to(torch.int64) + step * j


def build_wgrad_scale_block_meta(
    cu_seqlens_k: torch.Tensor,
    *,
    block_k: int = 128,
    packed_tail_tma_mode: str | None = None,
) -> WgradScaleBlockMeta:
    """Build 128-row scale metadata for grouped valid-row Wgrad operands.

    Same contract as the reference (block_meta.py:252-349): ``cu_seqlens_k`` is
    a CUDA int tensor [E+1] of expert-major valid-row offsets.
    """
    if cu_seqlens_k.ndim != 1:
        raise RuntimeError(f"expected cu_seqlens_k [E+1], got {tuple(cu_seqlens_k.shape)}")
    if not cu_seqlens_k.is_cuda:
        raise RuntimeError("cu_seqlens_k must be a CUDA tensor")
    if int(block_k) != BLOCK_K:
        raise RuntimeError("FP8 Wgrad scale block must be 128 for this project")
    if int(cu_seqlens_k.numel()) < 1:
        raise RuntimeError("cu_seqlens_k must have at least one entry")
    mode = resolve_packed_tail_tma_mode(packed_tail_tma_mode)
    cu = _i32(cu_seqlens_k)
    dev = cu.device
    e_count = int(cu.numel()) - 1
    lib = _lib.load()

    # Upper bound on blocks: every valid row in its own expert tail + one per expert.
    valid_upper = int(cu[-1].item()) if e_count >= 0 else 0
    capacity = valid_upper // BLOCK_K + e_count + 1
    i32 = dict(dtype=torch.int32, device=dev)
    blocks = torch.empty(e_count, **i32)
    block_offsets = torch.empty(e_count + 1, **i32)
    padded_cu = torch.empty(e_count + 1, **i32)
    wgmma_cu = torch.empty(e_count + 1, **i32)
    tail_valid = torch.empty(e_count, **i32)
    tail_atoms = torch.empty(e_count, **i32)
    tail_copy_masked = torch.empty(e_count, **i32)
    has_tail_u8 = torch.empty(e_count, dtype=torch.uint8, device=dev)
    order = torch.empty(max(e_count, 1), **i32)
    row_start = torch.empty(capacity, **i32)
    row_count = torch.empty(capacity, **i32)
    wgmma_start = torch.empty(capacity, **i32)
    totals = torch.zeros(5, dtype=torch.int64, device=dev)

    out = _lib.Sm100WgradMetaOut(
        blocks.data_ptr(), block_offsets.data_ptr(), padded_cu.data_ptr(), wgmma_cu.data_ptr(),
        tail_valid.data_ptr(), tail_atoms.data_ptr(), tail_copy_masked.data_ptr(), has_tail_u8.data_ptr(),
        order.data_ptr(), row_start.data_ptr(), row_count.data_ptr(), wgmma_start.data_ptr(),
        capacity, totals.data_ptr(),
    )
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        _lib.check(lib.sm100_wgrad_build_meta(cu.data_ptr(), e_count, ctypes.byref(out), stream),
                   "sm100_wgrad_build_meta")
    valid_rows, padded_rows, wgmma_rows, total_blocks, status = (int(v) for v in totals.cpu().tolist())
    if status == 1:
        raise RuntimeError("cu_seqlens_k must be monotonic")
    if status != 0:
        raise RuntimeError(f"metadata builder failed (status {status})")

    counts = (cu[1:] - cu[:-1]).to(torch.int64)
    tail_copy = _tail_copy_k(tail_valid, mode)
    tma_counts = counts // BLOCK_K * BLOCK_K + tail_copy.to(torch.int64)
    tma_cu = _exclusive_cumsum(tma_counts)
    tma_rows = int(tma_cu[-1].item())
    tma_start = _block_starts(tma_cu[:-1], blocks, total_blocks, BLOCK_K)
    if tma_rows > padded_rows:
        raise RuntimeError("adaptive TMA rows must not exceed padded128 rows")

    return WgradScaleBlockMeta(
        cu_seqlens_k=cu,
        padded_cu_seqlens_k=padded_cu,
        wgmma_cu_seqlens_k=wgmma_cu,
        tma_cu_seqlens_k=_i32(tma_cu),
        blocks_per_expert=blocks,
        block_offsets=block_offsets,
        block_row_start=row_start[:total_blocks],
        wgmma_block_row_start=wgmma_start[:total_blocks],
        tma_block_row_start=_i32(tma_start),
        block_row_count=row_count[:total_blocks],
        tail_valid_rows=tail_valid,
        tail_wgmma_atoms=tail_atoms,
        tail_copy_k=_i32(tail_copy),
        has_tail=has_tail_u8.to(torch.bool),
        block_k=BLOCK_K,
        valid_rows=valid_rows,
        padded_rows=padded_rows,
        wgmma_rows=wgmma_rows,
        tma_rows=tma_rows,
        wgmma_k_alignment=WGMMA_K_ALIGNMENT,
        total_blocks=total_blocks,
        packed_tail_tma_mode=mode,
        expert_order=order[:e_count],
    )


def _meta_from_counts(
    counts: torch.Tensor,
    row_start_per_expert: torch.Tensor,
    *,
    block_k: int,
    valid_rows: int,
    cu_valid: torch.Tensor,
) -> WgradScaleBlockMeta:
    """Metadata whose every field is the padded/identity layout of ``counts``
    with blocks of ``block_k`` rows (diagnostic tail/full-split variants,
    reference block_meta.py:144-178)."""
    dev = counts.device
    blocks = (counts + block_k - 1) // block_k
    bo = _exclusive_cumsum(blocks)
    total_blocks = int(bo[-1].item())
    padded_cu = bo * block_k
    starts = _block_starts(row_start_per_expert, blocks, total_blocks, block_k)
    e_of_block = torch.repeat_interleave(torch.arange(counts.numel(), device=dev), blocks, output_size=total_blocks)
    ends = (row_start_per_expert + counts)[e_of_block]
    lens = torch.clamp(ends - starts, max=block_k)
    tail = counts % block_k
    has_tail = tail != 0
    tail_copy = torch.where(has_tail, (tail + block_k - 1) // block_k * block_k, torch.zeros_like(tail))
    return WgradScaleBlockMeta(
        cu_seqlens_k=_i32(cu_valid),
        padded_cu_seqlens_k=_i32(padded_cu),
        wgmma_cu_seqlens_k=_i32(padded_cu),
        tma_cu_seqlens_k=_i32(padded_cu),
        blocks_per_expert=_i32(blocks),
        block_offsets=_i32(bo),
        block_row_start=_i32(starts),
        wgmma_block_row_start=_i32(torch.arange(total_blocks, device=dev) * block_k),
        tma_block_row_start=_i32(starts),
        block_row_count=_i32(lens),
        tail_valid_rows=_i32(tail),
        tail_wgmma_atoms=_i32((tail + 31) // 32),
        tail_copy_k=_i32(tail_copy),
        has_tail=has_tail,
        block_k=int(block_k),
        valid_rows=int(valid_rows),
        padded_rows=int(padded_cu[-1].item()),
        wgmma_rows=int(padded_cu[-1].item()),
        tma_rows=int(padded_cu[-1].item()),
        wgmma_k_alignment=WGMMA_K_ALIGNMENT,
        total_blocks=total_blocks,
        packed_tail_tma_mode=PACKED_TAIL_TMA_MASKED128,
        expert_order=None,
    )


def _check_cu(cu_seqlens_k: torch.Tensor, require_cuda: bool = True) -> torch.Tensor:
    if cu_seqlens_k.ndim != 1:
        raise RuntimeError(f"expected cu_seqlens_k [E+1], got {tuple(cu_seqlens_k.shape)}")
    if require_cuda and not cu_seqlens_k.is_cuda:
        raise RuntimeError("cu_seqlens_k must be a CUDA tensor")
    cu = cu_seqlens_k.to(torch.int64)
    if bool((cu[1:] < cu[:-1]).any().item()):
        raise RuntimeError("cu_seqlens_k must be monotonic")
    return cu


def _ragged_ranges(starts: torch.Tensor, lens: torch.Tensor) -> torch.Tensor:
    total = int(lens.sum().item())
    owner = torch.repeat_interleave(torch.arange(lens.numel(), device=lens.device), lens, output_size=total)
    base = _exclusive_cumsum(lens)
    return starts[owner] + torch.arange(total, device=lens.device) - base[owner]


def build_wgrad_tail_block_meta(
    cu_seqlens_k: torch.Tensor,
    *,
    tail_block_k: int = 64,
    full_block_k: int = 128,
    _require_cuda: bool = True,
) -> WgradTailBlockMeta:
    """Compact metadata for each expert's final partial 128-row block
    (reference block_meta.py:352-465). Host-side tensor logic; the reference
    also requires a CUDA ``cu_seqlens_k``."""
    cu = _check_cu(cu_seqlens_k, _require_cuda)
    if int(tail_block_k) not in (32, 64):
        raise RuntimeError("tail_block_k must be 32 or 64")
    if int(full_block_k) != BLOCK_K:
        raise RuntimeError("full_block_k must stay 128 for the current Wgrad contract")
    counts = cu[1:] - cu[:-1]
    tail = counts % BLOCK_K
    tail_src_start = cu[:-1] + counts - tail
    tail_indices = _ragged_ranges(tail_src_start, tail)
    tail_cu = _exclusive_cumsum(tail)
    meta = _meta_from_counts(tail, tail_cu[:-1], block_k=int(tail_block_k), valid_rows=int(tail_indices.numel()),
                             cu_valid=tail_cu)
    return WgradTailBlockMeta(meta=meta, tail_indices=tail_indices.to(torch.long).contiguous(),
                              tail_rows=int(tail_indices.numel()), tail_block_k=int(tail_block_k))


def build_wgrad_full_block_split(
    cu_seqlens_k: torch.Tensor, *, block_k: int = 128, _require_cuda: bool = True
) -> WgradFullBlockSplit:
    """Full-block-only metadata plus compact tail-row indices
    (reference block_meta.py:468-575)."""
    cu = _check_cu(cu_seqlens_k, _require_cuda)
    if int(block_k) != BLOCK_K:
        raise RuntimeError("FP8 Wgrad scale block must be 128 for this project")
    counts = cu[1:] - cu[:-1]
    full = counts // BLOCK_K * BLOCK_K
    tail = counts - full
    meta = _meta_from_counts(full, cu[:-1], block_k=BLOCK_K, valid_rows=int(cu[-1].item()), cu_valid=cu)
    tail_indices = _ragged_ranges(cu[:-1] + full, tail)
    return WgradFullBlockSplit(
        full_meta=meta,
        tail_indices=tail_indices.to(torch.long).contiguous(),
        tail_cu_seqlens_k=_i32(_exclusive_cumsum(tail)),
        full_rows=int(full.sum().item()),
        tail_rows=int(tail.sum().item()),
    )
