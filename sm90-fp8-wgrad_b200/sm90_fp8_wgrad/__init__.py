"""B200 (sm_100a) grouped FP8 Wgrad engine behind the sm90_fp8_wgrad operator API.

Public names match the reference package (src/sm90_fp8_wgrad/__init__.py:21-37)
so harness code importing ``sm90_fp8_wgrad`` runs unchanged against this
engine. All GPU work goes through the C-ABI library ``libsm100_fp8_wgrad.so``.
"""
from __future__ import annotations

from .block_meta import (
    WgradFullBlockSplit,
    WgradScaleBlockMeta,
    WgradTailBlockMeta,
    build_wgrad_full_block_split,
    build_wgrad_scale_block_meta,
    build_wgrad_tail_block_meta,
)
from .checks import (
    assert_scaled_wgrad_close,
    deepseek_calc_diff,
    ref_scaled_wgrad,
    scaled_wgrad_error,
    scaled_wgrad_stats,
)
from .interface import check_device_errors, fp8_grouped_wgrad_sm90, fp8_grouped_wgrad_sm100
from .quant import (
    Fp8GroupedWgradOperand,
    quantize_grouped_wgrad_operand_128x1,
    quantize_grouped_wgrad_operand_128x1_gather,
    quantize_grouped_wgrad_operand_tail_k,
)

__all__ = [
    "Fp8GroupedWgradOperand",
    "WgradFullBlockSplit",
    "WgradScaleBlockMeta",
    "WgradTailBlockMeta",
    "assert_scaled_wgrad_close",
    "build_wgrad_full_block_split",
    "build_wgrad_scale_block_meta",
    "build_wgrad_tail_block_meta",
    "check_device_errors",
    "deepseek_calc_diff",
    "fp8_grouped_wgrad_sm90",
    "fp8_grouped_wgrad_sm100",
    "quantize_grouped_wgrad_operand_128x1",
    "quantize_grouped_wgrad_operand_128x1_gather",
    "quantize_grouped_wgrad_operand_tail_k",
    "ref_scaled_wgrad",
    "scaled_wgrad_error",
    "scaled_wgrad_stats",
]
