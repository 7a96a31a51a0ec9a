"""CPU oracle for the grouped FP8 Wgrad path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this module, and only as the checker or the timed CPU
baseline. The product path (the sm90_fp8_wgrad package and its C-ABI library)
never imports or calls it.

It restates, in numpy, the reference's algorithm for every step of the path:

* scale-block metadata      -- build_wgrad_scale_block_meta,
                               src/sm90_fp8_wgrad/block_meta.py:252-349
                               (+ _build_wgmma_layout_cpu :181-212,
                               _build_tma_layout_cpu :124-178,
                               _select_tail_copy_k :92-121)
* 1x128 FP8 quantiser       -- _quantize_grouped_wgrad_128x1_kernel,
                               src/sm90_fp8_wgrad/quant.py:129-167 and the
                               padded operand layout of quant.py:222-247
* packed operand layout     -- quant.py:196-266 (data / kernel_data rows)
* fp32 -> e4m3 conversion   -- round to nearest even, saturating to +-448
                               (written from the e4m3fn format definition:
                               1 sign, 4 exponent bits with bias 7, 3 mantissa
                               bits, no infinities, max finite 448)
* dequantised reference     -- ref_scaled_wgrad, src/sm90_fp8_wgrad/checks.py:42-61
* DeepSeek calc_diff        -- _deepseek_calc_diff_chunked, checks.py:175-187
* error summary             -- scaled_wgrad_error, checks.py:89-101

Parity pin: tests/golden/make_golden.py imports the reference package from
its source tree (metadata builder, ref_scaled_wgrad, calc_diff) and commits
its outputs under tests/golden/; tests/test_oracle_golden.py checks this
module against them. The reference's Triton quantiser needs a GPU and cannot
run in the fixture container; its golden bytes come from a PyTorch
transliteration of quant.py:129-167 (PyTorch's own e4m3 cast), an
implementation independent of the bit construction here.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

BLOCK_K = 128
FP8_MAX = np.float32(448.0)
SCALE_EPS = np.float32(1.0e-12)


# ------------------------------------------------------------------ metadata
@dataclass
class OracleMeta:
    cu_seqlens_k: np.ndarray          # int64 [E+1]
    blocks_per_expert: np.ndarray     # int64 [E]
    block_offsets: np.ndarray         # int64 [E+1]
    padded_cu_seqlens_k: np.ndarray   # int64 [E+1]
    wgmma_cu_seqlens_k: np.ndarray    # int64 [E+1]
    tma_cu_seqlens_k: np.ndarray      # int64 [E+1]
    block_row_start: np.ndarray       # int64 [B]
    block_row_count: np.ndarray       # int64 [B]
    wgmma_block_row_start: np.ndarray # int64 [B]
    tma_block_row_start: np.ndarray   # int64 [B]
    tail_valid_rows: np.ndarray
    tail_wgmma_atoms: np.ndarray
    tail_copy_k: np.ndarray
    has_tail: np.ndarray
    valid_rows: int
    padded_rows: int
    wgmma_rows: int
    tma_rows: int
    total_blocks: int


def _tail_copy_k(tail: np.ndarray, mode: str) -> np.ndarray:
    """block_meta.py:92-121."""
    has = tail != 0
    if mode == "masked128":
        k = np.full_like(tail, 128)
    elif mode == "adaptive64":
        k = np.where(tail <= 64, 64, 128)
    elif mode == "adaptive32_64_128":
        k = np.where(tail <= 32, 32, np.where(tail <= 64, 64, 128))
    elif mode == "adaptive32_64_twophase":
        k = (tail + 31) // 32 * 32
    else:
        raise ValueError(mode)
    return np.where(has, k, 0).astype(np.int64)


def build_meta(cu_seqlens_k, packed_tail_tma_mode: str = "masked128") -> OracleMeta:
    """Loop-for-loop restatement of block_meta.py:271-349."""
    cu = np.asarray(cu_seqlens_k, dtype=np.int64)
    counts = cu[1:] - cu[:-1]
    if (counts < 0).any():
        raise RuntimeError("cu_seqlens_k must be monotonic")
    blocks = (counts + BLOCK_K - 1) // BLOCK_K
    bo = np.zeros(len(counts) + 1, dtype=np.int64)
    bo[1:] = np.cumsum(blocks)
    total = int(bo[-1])
    padded_cu = bo * BLOCK_K
    starts = np.zeros(total, dtype=np.int64)
    lens = np.zeros(total, dtype=np.int64)
    cur = 0
    for e, k_e in enumerate(counts.tolist()):                       # :288-294
        for b in range(int(blocks[e])):
            row0 = int(cu[e]) + b * BLOCK_K
            starts[cur] = row0
            lens[cur] = min(BLOCK_K, int(cu[e]) + int(k_e) - row0)
            cur += 1
    wg_counts = (counts + 31) // 32 * 32                             # :188-191
    wg_cu = np.zeros(len(counts) + 1, dtype=np.int64)
    wg_cu[1:] = np.cumsum(wg_counts)
    tail = counts % BLOCK_K
    tail_copy = _tail_copy_k(tail, packed_tail_tma_mode)
    tma_counts = counts // BLOCK_K * BLOCK_K + tail_copy
    tma_cu = np.zeros(len(counts) + 1, dtype=np.int64)
    tma_cu[1:] = np.cumsum(tma_counts)
    wg_starts = np.zeros(total, dtype=np.int64)
    tma_starts = np.zeros(total, dtype=np.int64)
    cur = 0
    for e in range(len(counts)):                                     # :199-210, :159-166
        for j in range(int(blocks[e])):
            wg_starts[cur] = wg_cu[e] + j * BLOCK_K
            tma_starts[cur] = tma_cu[e] + j * BLOCK_K
            cur += 1
    return OracleMeta(
        cu_seqlens_k=cu, blocks_per_expert=blocks, block_offsets=bo, padded_cu_seqlens_k=padded_cu,
        wgmma_cu_seqlens_k=wg_cu, tma_cu_seqlens_k=tma_cu, block_row_start=starts, block_row_count=lens,
        wgmma_block_row_start=wg_starts, tma_block_row_start=tma_starts, tail_valid_rows=tail,
        tail_wgmma_atoms=(tail + 31) // 32, tail_copy_k=tail_copy, has_tail=tail != 0,
        valid_rows=int(cu[-1]), padded_rows=int(padded_cu[-1]), wgmma_rows=int(wg_cu[-1]),
        tma_rows=int(tma_cu[-1]), total_blocks=total,
    )


def lpt_expert_order(blocks_per_expert: np.ndarray) -> np.ndarray:
    """Experts by descending block count, ties in expert order (stable)."""
    return np.argsort(-np.asarray(blocks_per_expert, dtype=np.int64), kind="stable").astype(np.int64)


# ------------------------------------------------------------ e4m3 encoding
def e4m3_encode(v) -> np.ndarray:
    """fp32 -> e4m3fn bytes, round to nearest even, saturating finite.

    Normal numbers 2^-6 <= |v| <= 448 have 3 mantissa bits, so the spacing of
    representable values at exponent floor(log2|v|) = p is 2^(p-3);
    subnormals have fixed spacing 2^-9. Rounding |v| to a multiple of that
    spacing with np.rint (ties to even) in float64 is exact.
    """
    v = np.asarray(v, dtype=np.float32).astype(np.float64)
    sign = np.signbit(v)
    a = np.abs(v)
    nan = np.isnan(a)
    a = np.where(nan, 0.0, a)
    _, ex = np.frexp(a)                          # a = f * 2^ex, f in [0.5, 1)
    p = ex - 1                                   # floor(log2 a) for a > 0
    spacing = np.where(a >= 2.0 ** -6, np.ldexp(1.0, p - 3), 2.0 ** -9)
    q = np.rint(a / spacing) * spacing
    q = np.minimum(q, 448.0)                     # satfinite
    normal = q >= 2.0 ** -6
    _, qex = np.frexp(np.where(normal, q, 1.0))
    qp = qex - 1
    exp_field = np.where(normal, qp + 7, 0)
    man_field = np.where(normal, np.rint((q / np.ldexp(1.0, qp) - 1.0) * 8.0), np.rint(q / 2.0 ** -9))
    code = (exp_field.astype(np.int64) << 3) | man_field.astype(np.int64)
    code = np.where(nan, 0x7F, code)
    return (code | (sign.astype(np.int64) << 7)).astype(np.uint8)


def e4m3_decode(b) -> np.ndarray:
    """e4m3fn bytes -> fp32 (0x7F / 0xFF decode to NaN)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


# ----------------------------------------------------------------- quantiser
@dataclass
class OracleOperand:
    data: np.ndarray    # uint8 [cols][pitch] (K contiguous), the padded layout
    scales: np.ndarray  # float32 [total_blocks][cols]
    k_rows: int

    def block_values(self, b: int, rows: int) -> np.ndarray:
        """Dequantisation input: FP8 values of block b's valid rows as fp32 [rows, cols]."""
        return e4m3_decode(self.data[:, b * BLOCK_K : b * BLOCK_K + rows]).T


def round_up_pow2(scale: np.ndarray) -> np.ndarray:
    """UE8M0 scale (an extension with no counterpart in the reference): the
    smallest power of two >= the positive fp32 scale, by its bit pattern -- a
    set mantissa bit moves the value to the next exponent; inf / NaN stay."""
    bits = np.asarray(scale, dtype=np.float32).view(np.uint32)
    special = (bits & np.uint32(0x7F800000)) == np.uint32(0x7F800000)
    exact = (bits & np.uint32(0x7FFFFF)) == 0
    up = (bits & np.uint32(0xFF800000)) + np.uint32(0x800000)
    return np.where(special | exact, bits, up).astype(np.uint32).view(np.float32)


def quantize_blocks(x: np.ndarray, block_row_start, block_row_count, block_k: int, padded_rows: int,
                    scale_format: str = "fp32") -> OracleOperand:
    """quant.py:129-167 for any scale-block height (the kernel's BLOCK_K is
    meta.block_k, quant.py:258): block b's valid rows are quantised with
    per-column amax/448 scales into padded rows block_k * b + k (quant.py:139),
    pitch = max(128, ceil(K/128)*128) and padded rows zero (quant.py:222-247).
    ``scale_format="ue8m0"`` rounds each scale up to a power of two first."""
    x = np.asarray(x, dtype=np.float32)
    cols = x.shape[1]
    nblocks = len(block_row_start)
    pitch = max(BLOCK_K, (padded_rows + BLOCK_K - 1) // BLOCK_K * BLOCK_K)
    data = np.zeros((cols, pitch), dtype=np.uint8)
    scales = np.empty((nblocks, cols), dtype=np.float32)
    for b in range(nblocks):
        r0, n = int(block_row_start[b]), int(block_row_count[b])
        blk = x[r0 : r0 + n]                                         # valid rows only (mask k < row_count)
        amax = np.abs(blk).max(axis=0) if n else np.zeros(cols, np.float32)
        scale = np.maximum((amax / FP8_MAX).astype(np.float32), SCALE_EPS)  # fp32 division, eps floor
        if scale_format == "ue8m0":
            scale = round_up_pow2(scale)
        scales[b] = scale
        q = (blk / scale[None, :]).astype(np.float32)                # x / scale, fp32
        data[:, b * block_k : b * block_k + n] = e4m3_encode(q).T
    return OracleOperand(data=data, scales=scales, k_rows=padded_rows)


def quantize_1x128(x: np.ndarray, meta: OracleMeta, scale_format: str = "fp32") -> OracleOperand:
    """The padded 128-row operand (quant.py:129-167, :222-247)."""
    x = np.asarray(x, dtype=np.float32)
    if x.ndim != 2 or x.shape[0] != meta.valid_rows:
        raise RuntimeError("x must be [valid_rows, cols]")
    return quantize_blocks(x, meta.block_row_start, meta.block_row_count, BLOCK_K, meta.padded_rows, scale_format)


_PACKED_GUARD_ROWS = {"masked128": 127, "adaptive64": 63, "adaptive32_64_128": 127, "adaptive32_64_twophase": 31}


def packed_layout(op: OracleOperand, meta: OracleMeta, mode: str = "masked128") -> tuple[np.ndarray, np.ndarray]:
    """Packed-layout storage of a quantised operand (same FP8 bytes, other rows).

    quant.py:196-266 with the Triton kernel's PACKED_LAYOUT and STORE_KERNEL_DATA
    branches (quant.py:133-167): ``data`` [cols, valid_rows] holds block b's valid
    rows at block_row_start[b] + k; ``kernel_data`` [cols, base + guard] (zeros
    elsewhere) holds them at the policy's block starts -- wgmma_block_row_start
    for masked128, tma_block_row_start for the adaptive policies
    (quant.py:47-95) -- with the guard rows of quant.py:66-83.
    """
    cols = op.data.shape[0]
    data = np.zeros((cols, meta.valid_rows), dtype=np.uint8)
    tma = mode != "masked128"
    base = meta.tma_rows if tma else meta.wgmma_rows
    starts = meta.tma_block_row_start if tma else meta.wgmma_block_row_start
    guard = _PACKED_GUARD_ROWS[mode] if base > 0 else 0
    kernel = np.zeros((cols, base + guard), dtype=np.uint8)
    for b in range(meta.total_blocks):
        n = int(meta.block_row_count[b])
        src = op.data[:, b * BLOCK_K : b * BLOCK_K + n]
        r0 = int(meta.block_row_start[b])
        data[:, r0 : r0 + n] = src
        k0 = int(starts[b])
        kernel[:, k0 : k0 + n] = src
    return data, kernel


# ------------------------------------------------------- dequantised product
def ref_scaled_wgrad(lhs: OracleOperand, rhs: OracleOperand, meta: OracleMeta) -> np.ndarray:
    """checks.py:42-61: out[e] = sum_b (lhs_q sa)^T (rhs_q sb) in fp32 [E, M, N]."""
    e_count = len(meta.cu_seqlens_k) - 1
    m, n = lhs.data.shape[0], rhs.data.shape[0]
    out = np.zeros((e_count, m, n), dtype=np.float32)
    for e in range(e_count):
        for b in range(int(meta.block_offsets[e]), int(meta.block_offsets[e + 1])):
            rows = int(meta.block_row_count[b])
            lq = lhs.block_values(b, rows) * lhs.scales[b][None, :]
            rq = rhs.block_values(b, rows) * rhs.scales[b][None, :]
            out[e] += lq.T @ rq
    return out


def ref_scaled_wgrad_experts(lhs: OracleOperand, rhs: OracleOperand, meta: OracleMeta, experts) -> np.ndarray:
    """ref_scaled_wgrad restricted to the listed experts, [len(experts), M, N]."""
    m, n = lhs.data.shape[0], rhs.data.shape[0]
    out = np.zeros((len(experts), m, n), dtype=np.float32)
    for i, e in enumerate(experts):
        for b in range(int(meta.block_offsets[e]), int(meta.block_offsets[e + 1])):
            rows = int(meta.block_row_count[b])
            out[i] += (lhs.block_values(b, rows) * lhs.scales[b][None, :]).T @ (
                rhs.block_values(b, rows) * rhs.scales[b][None, :])
    return out


def calc_diff(actual, expected) -> float:
    """checks.py:175-187: 1 - 2 sum(x y) / sum(x^2 + y^2), float64 sums."""
    a = np.asarray(actual, dtype=np.float64).ravel()
    x = np.asarray(expected, dtype=np.float64).ravel()
    den = float((a * a + x * x).sum())
    if den == 0.0:
        return 0.0
    return float(1.0 - 2.0 * float((a * x).sum()) / den)


def scaled_wgrad_error(actual, expected) -> tuple[float, float, float]:
    """checks.py:89-101: (max abs, max rel with |ref| floored at 1e-6, max |ref|)."""
    a = np.asarray(actual, dtype=np.float32)
    x = np.asarray(expected, dtype=np.float32)
    d = np.abs(a - x)
    max_ref = float(np.nan_to_num(np.abs(x), nan=np.inf).max()) if x.size else 0.0
    if not (np.isfinite(a).all() and np.isfinite(x).all() and np.isfinite(d).all()):
        return float("inf"), float("inf"), max_ref
    if d.size == 0:
        return 0.0, 0.0, max_ref
    return float(d.max()), float((d / np.maximum(np.abs(x), 1e-6)).max()), max_ref


def bf16_round(x) -> np.ndarray:
    """fp32 -> nearest-even bf16, returned as fp32 (for comparing BF16 outputs)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------ PyTorch CPU restatements
# The reference's CPU-capable path is PyTorch itself (ref_scaled_wgrad runs on
# CPU tensors, checks.py:42-61). These restatements time that algorithm on the
# host cores for the benchmark's CPU baseline and reference arm.
def quantize_1x128_torch(x, counts):
    """Padded 1x128 quantisation of grouped rows x [R, cols] (torch, CPU) with
    per-expert row counts; returns (data uint8 [cols][pitch], scales [B, cols],
    block_offsets list, block_row_count list). Same math as quantize_1x128."""
    import torch

    x = x.float()
    cols = x.shape[1]
    bo = [0]
    rc = []
    starts = []
    r = 0
    for c in counts:
        nb = (int(c) + BLOCK_K - 1) // BLOCK_K
        for j in range(nb):
            starts.append(r + j * BLOCK_K)
            rc.append(min(BLOCK_K, int(c) - j * BLOCK_K))
        bo.append(bo[-1] + nb)
        r += int(c)
    total = bo[-1]
    pitch = max(BLOCK_K, total * BLOCK_K)
    data = torch.zeros((cols, pitch), dtype=torch.uint8)
    scales = torch.empty((total, cols), dtype=torch.float32)
    for b in range(total):
        blk = x[starts[b] : starts[b] + rc[b]]
        s = torch.clamp_min(blk.abs().amax(dim=0) / 448.0, 1.0e-12)
        scales[b] = s
        q = (blk / s[None, :]).to(torch.float8_e4m3fn).view(torch.uint8)
        data[:, b * BLOCK_K : b * BLOCK_K + rc[b]] = q.T
    return data, scales, bo, rc


def ref_scaled_wgrad_torch(lhs_data, lhs_scales, rhs_data, rhs_scales, block_offsets, block_row_count, experts):
    """checks.py:42-61 on CPU tensors: per expert, per 128-row block,
    out[e] += (lhs_q * sa)^T @ (rhs_q * sb) in fp32."""
    import torch

    m, n = lhs_data.shape[0], rhs_data.shape[0]
    out = torch.zeros((len(experts), m, n), dtype=torch.float32)
    for i, e in enumerate(experts):
        for b in range(int(block_offsets[e]), int(block_offsets[e + 1])):
            rows = int(block_row_count[b])
            lq = lhs_data[:, b * BLOCK_K : b * BLOCK_K + rows].view(torch.float8_e4m3fn).float().T
            rq = rhs_data[:, b * BLOCK_K : b * BLOCK_K + rows].view(torch.float8_e4m3fn).float().T
            out[i] += (lq * lhs_scales[b].view(1, m)).T @ (rq * rhs_scales[b].view(1, n))
    return out
