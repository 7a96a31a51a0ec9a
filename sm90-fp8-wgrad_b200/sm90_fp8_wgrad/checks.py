"""Numerical checks of the grouped Wgrad contract (harness API).

Same functions and semantics as the reference's checks module
(src/sm90_fp8_wgrad/checks.py): the dequantised-FP8 fp32 reference product and
DeepSeek's ``calc_diff`` metric ``1 - 2 sum(x y) / sum(x^2 + y^2)`` evaluated
in chunks. These are verification utilities that run with PyTorch on whatever
device the tensors live on; they are never called by the operator itself.
"""
from __future__ import annotations

import os
from typing import Iterable, Iterator

import torch

from .block_meta import WgradScaleBlockMeta
from .quant import Fp8GroupedWgradOperand


def _block_rows(operand: Fp8GroupedWgradOperand, meta: WgradScaleBlockMeta, b: int) -> torch.Tensor:
    """Valid rows of scale block ``b`` of a padded operand as fp32 [rows, cols]
    (reference checks.py:17-39, padded branch: data rows 128 b ...)."""
    rows = int(meta.block_row_count[b].item())
    row0 = b * int(meta.block_k)
    return operand.data[row0 : row0 + rows].float()


def _expert_product(lhs, rhs, meta, e: int, m: int, n: int, device) -> torch.Tensor:
    acc = torch.zeros((m, n), device=device, dtype=torch.float32)
    b0 = int(meta.block_offsets[e].item())
    b1 = int(meta.block_offsets[e + 1].item())
    for b in range(b0, b1):
        lq = _block_rows(lhs, meta, b) * lhs.scales[b].view(1, m)
        rq = _block_rows(rhs, meta, b) * rhs.scales[b].view(1, n)
        acc += lq.T @ rq
    return acc


def ref_scaled_wgrad(
    lhs: Fp8GroupedWgradOperand,
    rhs: Fp8GroupedWgradOperand,
    meta: WgradScaleBlockMeta,
    *,
    out_dtype: torch.dtype,
) -> torch.Tensor:
    """Dequantised FP8 reference [E, M, N] (reference checks.py:42-61)."""
    e_count = int(meta.cu_seqlens_k.numel()) - 1
    m = int(lhs.data.shape[1])
    n = int(rhs.data.shape[1])
    out = torch.zeros((e_count, m, n), device=lhs.data.device, dtype=torch.float32)
    for e in range(e_count):
        out[e] = _expert_product(lhs, rhs, meta, e, m, n, lhs.data.device)
    return out.to(out_dtype)


def iter_ref_scaled_wgrad_by_expert(
    lhs: Fp8GroupedWgradOperand,
    rhs: Fp8GroupedWgradOperand,
    meta: WgradScaleBlockMeta,
    *,
    out_dtype: torch.dtype,
) -> Iterator[tuple[int, torch.Tensor]]:
    """Per-expert references without materialising [E, M, N] (checks.py:64-86)."""
    e_count = int(meta.cu_seqlens_k.numel()) - 1
    m = int(lhs.data.shape[1])
    n = int(rhs.data.shape[1])
    for e in range(e_count):
        yield e, _expert_product(lhs, rhs, meta, e, m, n, lhs.data.device).to(out_dtype)


def scaled_wgrad_error(actual: torch.Tensor, expected: torch.Tensor) -> tuple[float, float, float]:
    """(max |a-e|, max |a-e| / max(|e|, 1e-6), max |e|); inf when non-finite
    (checks.py:89-101)."""
    a = actual.float()
    x = expected.float()
    diff = (a - x).abs()
    max_abs_ref = float(torch.nan_to_num(x.abs(), nan=float("inf")).max().item()) if x.numel() else 0.0
    if not bool(torch.isfinite(a).all()) or not bool(torch.isfinite(x).all()) or not bool(torch.isfinite(diff).all()):
        return float("inf"), float("inf"), max_abs_ref
    if diff.numel() == 0:
        return 0.0, 0.0, max_abs_ref
    return float(diff.max().item()), float((diff / x.abs().clamp_min(1.0e-6)).max().item()), max_abs_ref


def _chunks(actual: torch.Tensor, expected: torch.Tensor, max_elements: int):
    if tuple(actual.shape) != tuple(expected.shape):
        raise RuntimeError(f"calc_diff shape mismatch: actual={tuple(actual.shape)} expected={tuple(expected.shape)}")
    if actual.numel() <= max_elements or actual.ndim == 0:
        yield actual, expected
        return
    if actual.ndim == 1:
        step = max(1, max_elements)
    else:
        step = max(1, max_elements // max(1, int(actual[0].numel())))
    for i in range(0, int(actual.shape[0]), step):
        a, x = actual[i : i + step], expected[i : i + step]
        if a.numel() > max_elements and a.ndim > 1 and int(a.shape[0]) == 1:
            yield from _chunks(a[0], x[0], max_elements)
        else:
            yield a, x


def _calc_diff_sums(pairs: Iterable[tuple[torch.Tensor, torch.Tensor]]) -> float:
    max_chunk = int(os.environ.get("SM90_WGRAD_CALC_DIFF_CHUNK_ELEMENTS", "8388608"))
    num = 0.0
    den = 0.0
    with torch.no_grad():
        for actual, expected in pairs:
            for a, x in _chunks(actual, expected, max_chunk):
                a = a.detach().to(torch.float32)
                x = x.detach().to(torch.float32)
                num += float((a * x).sum().item())
                den += float((a * a + x * x).sum().item())
    if den == 0.0:
        return 0.0
    return float(1.0 - 2.0 * num / den)


def _deepgemm_importable() -> bool:
    try:
        import deep_gemm.testing  # noqa: F401
    except Exception:
        return False
    return True


def deepseek_calc_diff(actual: torch.Tensor, expected: torch.Tensor, *, require_deepgemm: bool = True) -> float:
    """DeepSeek/DeepGEMM ``calc_diff`` (checks.py:104-144), chunked formula.
    With ``require_deepgemm`` the DeepGEMM package must be importable, as in
    the reference, so a server run cannot silently switch metrics."""
    if require_deepgemm and not _deepgemm_importable():
        raise RuntimeError("DeepGEMM calc_diff is required but not importable")
    return _calc_diff_sums([(actual, expected)])


def deepseek_calc_diff_stream(pairs, *, require_deepgemm: bool = True) -> float:
    """calc_diff accumulated over streamed (actual, expected) pairs (checks.py:190-223)."""
    if require_deepgemm and not _deepgemm_importable():
        raise RuntimeError("DeepGEMM calc_diff is required but not importable")
    return _calc_diff_sums(pairs)


def scaled_wgrad_stats(actual: torch.Tensor, expected: torch.Tensor, *,
                       require_deepgemm_calc_diff: bool = True) -> dict[str, float]:
    return {"deepseek_calc_diff": deepseek_calc_diff(actual, expected, require_deepgemm=require_deepgemm_calc_diff)}


def assert_scaled_wgrad_close(
    actual: torch.Tensor,
    expected: torch.Tensor,
    *,
    out_dtype: torch.dtype,
    deepseek_diff_limit: float = 1.0e-3,
    require_deepgemm_calc_diff: bool = True,
) -> dict[str, float]:
    """Raise RuntimeError when calc_diff exceeds the gate (checks.py:241-258)."""
    del out_dtype
    stats = scaled_wgrad_stats(actual, expected, require_deepgemm_calc_diff=require_deepgemm_calc_diff)
    stats["deepseek_diff_limit"] = float(deepseek_diff_limit)
    if stats["deepseek_calc_diff"] > float(deepseek_diff_limit):
        raise RuntimeError(f"custom scaled FP8 Wgrad DeepSeek calc_diff check failed: {stats}")
    return stats
