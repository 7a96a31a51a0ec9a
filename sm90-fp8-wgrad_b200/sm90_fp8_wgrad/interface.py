"""Public grouped FP8 Wgrad operator (the drop-in boundary).

``fp8_grouped_wgrad_sm90`` keeps the reference signature, validation messages
and error type (src/sm90_fp8_wgrad/interface.py:28-69, 128-256); its body is a
single call of the C-ABI entry point ``sm100_fp8_grouped_wgrad`` on the
current CUDA stream. Unlike the reference implementation
(gemm_sm90.py:5676) the call performs no device->host synchronisation, so
back-to-back calls queue on the stream without host round trips.
"""
from __future__ import annotations

import ctypes
import os
from typing import Literal

import torch

from . import _lib
from .block_meta import WgradScaleBlockMeta
from .layout_mode import LAYOUT_MODE_PACKED, resolve_wgrad_layout_mode
from .quant import (
    Fp8GroupedWgradOperand,
    packed_kernel_data_base_rows,
    packed_kernel_data_cu_seqlens_k,
    packed_kernel_data_guard_rows,
)

# tuned_config names accepted by the reference (gemm_sm90.py:265-509), mapped
# onto the B200 tile shapes. The SM90 cluster/pingpong variants have no
# separate meaning on tcgen05: every name resolves to the persistent kernel
# with a 128-row tile and the N width listed here (0 = choose by shape).
# Tile configs whose kernel needs a workspace (sm100_wgrad_workspace_bytes > 0).
_SP_TILES = frozenset((_lib.TILE_256x256_SP, _lib.TILE_256x256_SP_W16))

TUNED_CONFIGS: dict[str, int] = {
    "default": _lib.TILE_AUTO,
    "optB_coop128_default": _lib.TILE_AUTO,
    "down_128x192": _lib.TILE_128x256,
    "down_128x128_pingpong": _lib.TILE_128x128,
    "down_128x256": _lib.TILE_128x256,
    "down_64x256": _lib.TILE_128x256,
    "down_128x192_coop": _lib.TILE_128x256,
    "down_128x256_coop": _lib.TILE_128x256,
    "down_64x192": _lib.TILE_128x256,
    "down_64x192_coop": _lib.TILE_128x256,
    "gate_64x256": _lib.TILE_128x256,
    "gate_64x192": _lib.TILE_128x256,
    "gate_128x192": _lib.TILE_128x256,
    "gate_128x256": _lib.TILE_128x256,
    "gate_128x256_coop": _lib.TILE_128x256,
    "gate_256x256_coop": _lib.TILE_128x256,
    "gate_64x256_coop": _lib.TILE_128x256,
    "gate_128x128": _lib.TILE_128x128,
    "gate_256x128": _lib.TILE_128x128,
    "optA_down_64x128_dbacc": _lib.TILE_128x128,
    "optA_gate_64x128_dbacc": _lib.TILE_128x128,
    "optB_down_64x128_wg_pingpong": _lib.TILE_128x128,
    "optB_gate_64x128_wg_pingpong": _lib.TILE_128x128,
    "tail64_64x128": _lib.TILE_128x128,
    "tail64_64x256": _lib.TILE_128x256,
    "tail32_64x128": _lib.TILE_128x128,
    # B200-native names
    "sm100_128x256": _lib.TILE_128x256,
    "sm100_128x128": _lib.TILE_128x128,
    "sm100_128x256_w8": _lib.TILE_128x256_W8,     # 8 promotion warps
    "sm100_128x256_w16": _lib.TILE_128x256_W16,   # 16 promotion warps
    "sm100_128x128_2cta": _lib.TILE_128x128_2CTA,  # two 128x128 pipelines (CTAs) per SM
    "sm100_128x192_w12": _lib.TILE_128x192_W12,    # 192-column tile, 12 promotion warps
    "sm100_128x192_ue8m0": _lib.TILE_128x192_UE8M0,  # power-of-two scales as tensor-core block scales
    "sm100_256x256_pair": _lib.TILE_256x256_PAIR,    # CTA pair (cta_group::2), half of B per SM
    "sm100_256x256_pair_w16": _lib.TILE_256x256_PAIR_W16,  # the same, 16 promotion warps per CTA
    "sm100_256x256_sp": _lib.TILE_256x256_SP,  # CTA pair, scale product on the tensor core, one FMA per element
    "sm100_256x256_sp_w16": _lib.TILE_256x256_SP_W16,  # the same, 16 promotion warps per CTA
}


# KERNEL_LAB_WGRAD_KERNEL_MODE values (reference gemm_sm90.py:139-175) with a B200
# counterpart: the known-answer modes, honoured by the debug-modes library
# (build_ext.py --debug-modes). The reference's other values select variants of
# the SM90 kernel's structure and have no meaning here.
B200_KERNEL_MODES = ("normal", "coord_m", "coord_n", "scale_only", "unscaled")


def _kernel_mode() -> str:
    mode = os.environ.get("KERNEL_LAB_WGRAD_KERNEL_MODE", "").strip()
    if mode and mode not in B200_KERNEL_MODES:
        raise RuntimeError(
            f"KERNEL_LAB_WGRAD_KERNEL_MODE={mode!r} selects an SM90 kernel variant with no B200 counterpart; "
            f"B200 modes: {', '.join(B200_KERNEL_MODES)}"
        )
    return mode or "normal"


def _check_fp8_operand(name: str, operand: Fp8GroupedWgradOperand) -> None:
    """Operand checks of the reference (interface.py:28-69)."""
    if operand.data.dtype != torch.float8_e4m3fn:
        raise RuntimeError(f"{name}.data must be torch.float8_e4m3fn, got {operand.data.dtype}")
    if operand.scales.dtype != torch.float32:
        raise RuntimeError(f"{name}.scales must be torch.float32, got {operand.scales.dtype}")
    if operand.data.ndim != 2 or operand.scales.ndim != 2:
        raise RuntimeError(f"{name} must have data [K,N] and scales [B,N]")
    if int(operand.data.shape[1]) != int(operand.scales.shape[1]):
        raise RuntimeError(f"{name} data/scales column mismatch")
    if int(operand.data.stride(0)) != 1:
        raise RuntimeError(
            f"{name}.data must be FP8 K-major logical [K,N] with stride(0) == 1, "
            f"got stride={tuple(operand.data.stride())}"
        )
    if int(operand.data.stride(1)) % 16 != 0:
        raise RuntimeError(
            f"{name}.data leading dimension must be divisible by 16 for FP8 TMA, "
            f"got stride={tuple(operand.data.stride())}"
        )
    if not operand.scales.is_contiguous():
        raise RuntimeError(f"{name}.scales must be contiguous")


def _auto_tuned_config(m: int, n: int) -> str:
    """Shape-keyed config selection with the reference's env overrides
    (interface.py:72-84)."""
    fallback = os.environ.get("KERNEL_LAB_WGRAD_AUTO_FALLBACK", "default").strip() or "default"
    if int(m) == 2048 and int(n) == 768:
        return os.environ.get("KERNEL_LAB_WGRAD_AUTO_DOWN", fallback).strip() or fallback
    if int(m) == 1536 and int(n) == 2048:
        return os.environ.get("KERNEL_LAB_WGRAD_AUTO_GATE_UP", fallback).strip() or fallback
    return fallback


def _check_int_vector(name: str, t: torch.Tensor, length: int, device: torch.device) -> None:
    if t.dtype != torch.int32:
        raise RuntimeError(f"{name} must be int32")
    if t.ndim != 1 or int(t.shape[0]) != length:
        raise RuntimeError(f"{name} shape must be [{length}], got {tuple(t.shape)}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if t.device != device:
        raise RuntimeError(f"{name} must be on {device}, got {t.device}")


def fp8_grouped_wgrad_sm90(
    lhs: Fp8GroupedWgradOperand,
    rhs: Fp8GroupedWgradOperand,
    out: torch.Tensor,
    meta: WgradScaleBlockMeta,
    *,
    output_layout: Literal["emn"] = "emn",
    tuned_config: str = "default",
    accumulate: bool = False,
    expert_range: tuple[int, int] | None = None,
) -> torch.Tensor:
    """Grouped scaled FP8 Wgrad (runs the sm_100a engine; name kept for drop-in).

    Contract (reference interface.py:138-155):
      lhs.data   logical [K_rows, M], stride(0) == 1, stride(1) % 16 == 0
      rhs.data   logical [K_rows, N], same layout
      lhs.scales [total_blocks, M], rhs.scales [total_blocks, N]   fp32
      out        [E, M, N] bf16 or fp32, contiguous

      out[e, m, n] (+)= sum_b sum_{k in b} lhs_q[k,m] lhs_s[b,m] rhs_q[k,n] rhs_s[b,n]

    with b over expert e's 128-row scale blocks; experts without rows give 0.
    Runs on the current CUDA stream of ``out``'s device; returns ``out``.

    ``expert_range=(e0, e1)`` (B200 addition, keyword only) computes only
    out[e0:e1] and leaves the other experts untouched: one launch over that
    expert range of the same operands and metadata, bit-identical to the
    corresponding slice of a full launch. It lets a caller overlap the
    device-to-host copy of finished experts with the rest of the GEMM.

    When both operands carry ``scale_format == "ue8m0"`` (power-of-two
    scales from ``quantize_grouped_wgrad_operand_128x1(..., scale_format="ue8m0")``),
    the default config runs the block-scaled kernel: the same sum, with the
    scales applied inside the tensor core instead of a per-block fp32 promotion.
    """
    kernel_mode = _kernel_mode()
    if kernel_mode != "normal" and not _lib.build_flags() & _lib.BUILD_DEBUG_MODES:
        raise RuntimeError(
            f"kernel mode {kernel_mode!r} needs the debug-modes library: build it with "
            "`python sm90-fp8-wgrad_b200/build_ext.py --debug-modes` and load it with SM100_WGRAD_LIB=<path>"
        )
    layout_mode = resolve_wgrad_layout_mode()
    _check_fp8_operand("lhs", lhs)
    _check_fp8_operand("rhs", rhs)
    packed = layout_mode == LAYOUT_MODE_PACKED
    expected_k_rows = int(meta.valid_rows) if packed else int(meta.padded_rows)
    if lhs.data.shape[0] != rhs.data.shape[0]:
        raise RuntimeError(
            "lhs/rhs K_rows mismatch: "
            f"lhs={tuple(lhs.data.shape)} stride={tuple(lhs.data.stride())} "
            f"rhs={tuple(rhs.data.shape)} stride={tuple(rhs.data.stride())} "
            f"layout_mode={layout_mode!r}"
        )
    if int(lhs.data.shape[0]) != expected_k_rows:
        raise RuntimeError(
            f"operand K_rows does not match metadata for layout_mode={layout_mode!r}: "
            f"got {int(lhs.data.shape[0])}, expected {expected_k_rows}"
        )
    if packed:
        # reference interface.py:191-209: the launch copy must cover the packed
        # K offsets plus the tail policy's TMA guard rows.
        base_rows = packed_kernel_data_base_rows(meta)
        for name, operand in (("lhs", lhs), ("rhs", rhs)):
            kd = operand.kernel_data
            if kd is None:
                raise RuntimeError(f"packed {name}.kernel_data is required")
            if int(kd.shape[1]) < base_rows:
                raise RuntimeError(
                    f"packed {name}.kernel_data K rows must cover meta.wgmma_rows: "
                    f"got {tuple(kd.shape)}, expected at least K={base_rows}"
                )
            guard = packed_kernel_data_guard_rows(meta)
            if base_rows > 0 and int(kd.shape[1]) < base_rows + guard:
                raise RuntimeError(
                    f"packed {name}.kernel_data must include a {guard}-row TMA guard: "
                    f"got K={int(kd.shape[1])}, expected at least {base_rows + guard}"
                )
            if kd.dtype != torch.float8_e4m3fn or kd.ndim != 2 or int(kd.stride(1)) != 1 or int(kd.stride(0)) % 16:
                raise RuntimeError(f"packed {name}.kernel_data must be float8_e4m3fn [cols, K] with K contiguous")
    if int(getattr(meta, "block_k", 128)) != 128:
        raise RuntimeError(
            f"metadata block_k must be 128 (the kernel's K block and scale block), got {int(meta.block_k)}; "
            "tail metadata with 32/64-row blocks feeds quantize_grouped_wgrad_operand_tail_k, not this operator"
        )
    if lhs.scales.shape[0] != rhs.scales.shape[0]:
        raise RuntimeError("lhs/rhs scale block count mismatch")
    if int(lhs.scales.shape[0]) != int(meta.total_blocks):
        raise RuntimeError("scale block count does not match metadata")
    if out.ndim != 3:
        raise RuntimeError(f"expected out [E,M,N], got {tuple(out.shape)}")
    if out.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError(f"out dtype must be bf16 or fp32, got {out.dtype}")
    if output_layout != "emn":
        raise RuntimeError("only contiguous [E,M,N] output is implemented for the benchmark")
    if not out.is_contiguous():
        raise RuntimeError("custom FP8 Wgrad output must be contiguous [E,M,N]")
    if not out.is_cuda:
        raise RuntimeError("out must be a CUDA tensor")
    experts, m, n = map(int, out.shape)
    if int(lhs.data.shape[1]) != m or int(rhs.data.shape[1]) != n:
        raise RuntimeError(
            f"out [E,M,N]={tuple(out.shape)} does not match lhs cols {int(lhs.data.shape[1])} "
            f"and rhs cols {int(rhs.data.shape[1])}"
        )
    dev = out.device
    for name, t in (("lhs.data", lhs.data), ("rhs.data", rhs.data), ("lhs.scales", lhs.scales),
                    ("rhs.scales", rhs.scales)):
        if t.device != dev:
            raise RuntimeError(f"{name} must be on {dev}, got {t.device}")
    _check_int_vector("cu_seqlens_k", packed_kernel_data_cu_seqlens_k(meta) if packed else meta.padded_cu_seqlens_k,
                      experts + 1, dev)
    _check_int_vector("block_offsets", meta.block_offsets, experts + 1, dev)
    order = meta.expert_order
    if order is not None:
        _check_int_vector("expert_order", order, experts, dev)
    resolved = _auto_tuned_config(m, n) if tuned_config == "auto" else str(tuned_config)
    if resolved not in TUNED_CONFIGS:
        raise RuntimeError(f"unknown Wgrad config {resolved!r}; choices={sorted(TUNED_CONFIGS)}")

    args = _lib.Sm100WgradArgs()
    if packed:
        lk, rk = lhs.kernel_data, rhs.kernel_data
        args.lhs_data, args.lhs_pitch = lk.data_ptr(), int(lk.stride(0))
        args.rhs_data, args.rhs_pitch = rk.data_ptr(), int(rk.stride(0))
        kernel_k_rows = min(int(lk.shape[1]), int(rk.shape[1]))
        k_row_offsets = packed_kernel_data_cu_seqlens_k(meta)
    else:
        args.lhs_data, args.lhs_pitch = lhs.data.data_ptr(), int(lhs.data.stride(1))
        args.rhs_data, args.rhs_pitch = rhs.data.data_ptr(), int(rhs.data.stride(1))
        kernel_k_rows = expected_k_rows
        k_row_offsets = meta.padded_cu_seqlens_k
    args.lhs_scales = lhs.scales.data_ptr()
    args.rhs_scales = rhs.scales.data_ptr()
    args.out = out.data_ptr()
    args.out_dtype = _lib.OUT_BF16 if out.dtype == torch.bfloat16 else _lib.OUT_F32
    args.accumulate = 1 if accumulate else 0
    args.num_experts = experts
    args.m = m
    args.n = n
    args.k_rows = kernel_k_rows
    args.total_blocks = int(meta.total_blocks)
    args.block_offsets = meta.block_offsets.data_ptr()
    args.k_row_offsets = k_row_offsets.data_ptr()
    args.expert_order = order.data_ptr() if order is not None and experts > 0 else None
    if expert_range is not None:
        e0, e1 = (int(v) for v in expert_range)
        if not 0 <= e0 <= e1 <= experts:
            raise RuntimeError(f"expert_range {expert_range!r} outside [0, {experts}]")
        # The kernel reads block_offsets[e] / k_row_offsets[e] (absolute block
        # and row indices), so a sub-range is a pointer offset of those arrays
        # and of out; the expert order falls back to natural order.
        args.num_experts = e1 - e0
        args.out = out.data_ptr() + e0 * m * n * out.element_size()
        args.block_offsets = meta.block_offsets.data_ptr() + 4 * e0
        args.k_row_offsets = k_row_offsets.data_ptr() + 4 * e0
        args.expert_order = None
    ue8m0_operands = all(getattr(op, "scale_format", "fp32") == "ue8m0" for op in (lhs, rhs))
    if resolved == "sm100_128x192_ue8m0" and not ue8m0_operands:
        raise RuntimeError("tuned_config 'sm100_128x192_ue8m0' needs both operands quantised with scale_format='ue8m0'")
    if TUNED_CONFIGS[resolved] == _lib.TILE_AUTO and ue8m0_operands and kernel_mode == "normal":
        # Power-of-two scales on both sides: the tensor core applies them, no fp32 promotion.
        resolved = "sm100_128x192_ue8m0"
    args.tile_config = TUNED_CONFIGS[resolved]
    args.max_ctas = int(os.environ.get("SM100_WGRAD_MAX_CTAS", "0") or 0)
    lib = _lib.load()
    if torch.cuda.current_device() == dev.index:
        status = _launch(lib, args, dev)
    else:
        with torch.cuda.device(dev):
            status = _launch(lib, args, dev)
    _lib.check(status, "sm100_fp8_grouped_wgrad")
    return out


def _current_stream_handle(index: int) -> int:
    """Raw cudaStream_t of the device's current stream (the cheap accessor
    where this torch has it)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return raw(index) if raw is not None else torch.cuda.current_stream(index).cuda_stream


def _launch(lib, args, dev: torch.device) -> int:
    """The C-ABI call, with ``dev`` current: first surface a device-side failure
    of an earlier launch (bounded wait that gave up, mislabelled UE8M0 scales,
    bad gather index) without a sync, then size the workspace (only the
    scale-product configs have one), then launch on the current stream."""
    _lib.raise_pending_device_error()
    workspace = None
    if args.tile_config in _SP_TILES:
        need = ctypes.c_int64(0)
        _lib.check(lib.sm100_wgrad_workspace_bytes(ctypes.byref(args), ctypes.byref(need)),
                   "sm100_wgrad_workspace_bytes")
        if need.value > 0:
            # Scratch for the split scales, from the caching allocator on the
            # launch stream; it is released when the launch has consumed it.
            workspace = torch.empty(int(need.value), dtype=torch.uint8, device=dev)
            args.workspace, args.workspace_bytes = workspace.data_ptr(), int(need.value)
    return lib.sm100_fp8_grouped_wgrad(ctypes.byref(args), _current_stream_handle(dev.index))


# B200-native alias of the same operator.
fp8_grouped_wgrad_sm100 = fp8_grouped_wgrad_sm90


def check_device_errors(device: torch.device | int | None = None) -> None:
    """Synchronise ``device`` and raise RuntimeError if any launch of this
    library on it recorded a device-side error (a bounded wait that gave up,
    a UE8M0-labelled operand whose scales are not powers of two, a quantiser
    gather index out of range). Clears the error."""
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        torch.cuda.synchronize()
        _lib.raise_device_error(_lib.device_error(), "recorded on this device")
