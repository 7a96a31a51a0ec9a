"""Operand layout modes and their environment switches.

Same names, values and environment variables as the reference
(src/sm90_fp8_wgrad/layout_mode.py:6-82), because harness code selects the
layout through ``KERNEL_LAB_WGRAD_LAYOUT_MODE`` (synthetic.py:218 of the
reference) and packed-tail policies through ``KERNEL_LAB_WGRAD_PACKED_TAIL_TMA``.

* ``padded``  -- every expert's K rows are materialised in whole 128-row
  blocks (zero filled past the valid rows). This is the layout the B200 kernel
  runs.
* ``packed``  -- FP8 rows stay compact on valid K rows; scales keep 128-row
  blocks. Metadata for it is built; the GEMM does not run it yet and raises.
"""
from __future__ import annotations

import os

LAYOUT_MODE_PADDED = "padded"
LAYOUT_MODE_PACKED = "packed"
WGRAD_LAYOUT_MODES = (LAYOUT_MODE_PADDED, LAYOUT_MODE_PACKED)

PACKED_TAIL_TMA_MASKED128 = "masked128"
PACKED_TAIL_TMA_ADAPTIVE64 = "adaptive64"
PACKED_TAIL_TMA_ADAPTIVE32_64_128 = "adaptive32_64_128"
PACKED_TAIL_TMA_ADAPTIVE32_64_TWOPHASE = "adaptive32_64_twophase"
PACKED_TAIL_TMA_MODES = (
    PACKED_TAIL_TMA_MASKED128,
    PACKED_TAIL_TMA_ADAPTIVE64,
    PACKED_TAIL_TMA_ADAPTIVE32_64_128,
    PACKED_TAIL_TMA_ADAPTIVE32_64_TWOPHASE,
)

LAYOUT_ENV = "KERNEL_LAB_WGRAD_LAYOUT_MODE"
PACKED_TAIL_ENV = "KERNEL_LAB_WGRAD_PACKED_TAIL_TMA"


def _resolve(value: str | None, env: str, default: str, allowed: tuple[str, ...]) -> str:
    raw = os.environ.get(env, default) if value is None else value
    mode = str(raw).strip().lower()
    if mode not in allowed:
        raise RuntimeError(f"{env} must be one of {allowed}; got {raw!r}")
    return mode


def resolve_wgrad_layout_mode(value: str | None = None, *, default: str = LAYOUT_MODE_PADDED) -> str:
    """Explicit value, else the environment variable, else ``default``."""
    return _resolve(value, LAYOUT_ENV, default, WGRAD_LAYOUT_MODES)


def resolve_packed_tail_tma_mode(value: str | None = None, *, default: str = PACKED_TAIL_TMA_MASKED128) -> str:
    return _resolve(value, PACKED_TAIL_ENV, default, PACKED_TAIL_TMA_MODES)
