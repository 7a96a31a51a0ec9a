"""Generate the golden fixtures in tests/golden/ from the reference implementation.

Run in a container where the reference source tree is available:

    python tests/golden/make_golden.py --reference-src <path to reference>/src

It imports the reference package ``sm90_fp8_wgrad`` (pure Python) and records:

* meta_cases.npz     -- build_wgrad_scale_block_meta (block_meta.py:252-349) for
                        edge-case routings under every packed-tail policy, plus
                        build_wgrad_tail_block_meta (:352-465) and
                        build_wgrad_full_block_split (:468-575).
                        The reference requires a CUDA ``cu_seqlens_k``; a
                        Tensor subclass reporting ``is_cuda`` lets it run on CPU.
* quant_small.npz    -- 1x128 quantiser bytes and scales. The reference's Triton
                        kernel (quant.py:105-167) needs a GPU, so its math is
                        transliterated here in PyTorch (masked amax, fp32
                        ``amax / 448`` floored at 1e-12, ``x / scale``,
                        ``tensor.to(torch.float8_e4m3fn)``).
* quant_triton.npz   -- the reference's own quantiser, end to end: its launcher
                        quantize_grouped_wgrad_operand_128x1 (quant.py:175-270)
                        and Triton kernel (quant.py:105-167), run on CPU under
                        the Triton interpreter (TRITON_INTERPRET=1, set before
                        triton is imported), padded and packed layouts. The
                        interpreter converts fp32 to e4m3 in software and
                        differs from the GPU's round-to-nearest-even satfinite
                        conversion in two ways: a quotient exactly halfway
                        between two e4m3 values goes to the larger magnitude,
                        and a round-up that should carry into the next binade
                        does not. The fixture stores the interpreter's bytes;
                        the test explains every byte that differs from the
                        oracle by one of those two rules.
* wgrad_small.npz    -- ref_scaled_wgrad (checks.py:42-61) fp32 outputs and the
                        reference calc_diff (checks.py:175-187) of known pairs.
* c1_tiny.npz        -- the tiny benchmark configuration (E=8, top-2, H=256,
                        I=128, T=1024, seed 0): counts, SHA-256 of every FP8
                        operand and scale buffer, and per-expert sums plus a
                        strided sample of the reference outputs.

Inputs are drawn with numpy's PCG64 generator (``case_inputs``) so the tests
regenerate them without the reference.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

# The reference's Triton quantiser runs on CPU through the Triton interpreter;
# the switch must be set before anything imports triton.
os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from golden_inputs import C1, META_CASES, SMALL_CASES, bf16_from_f32, case_inputs  # noqa: E402


class _CudaLike(torch.Tensor):
    """Makes the reference's ``is_cuda`` guard accept a CPU tensor."""

    @property
    def is_cuda(self):  # type: ignore[override]
        return True


def _plain(t: torch.Tensor) -> np.ndarray:
    return t.as_subclass(torch.Tensor).detach().cpu().numpy()


def _meta_arrays(meta, prefix: str) -> dict:
    out = {}
    for f in ("cu_seqlens_k", "padded_cu_seqlens_k", "wgmma_cu_seqlens_k", "tma_cu_seqlens_k",
              "blocks_per_expert", "block_offsets", "block_row_start", "wgmma_block_row_start",
              "tma_block_row_start", "block_row_count", "tail_valid_rows", "tail_wgmma_atoms",
              "tail_copy_k", "has_tail"):
        out[f"{prefix}.{f}"] = _plain(getattr(meta, f)).astype(np.int64)
    for f in ("block_k", "valid_rows", "padded_rows", "wgmma_rows", "tma_rows", "total_blocks"):
        out[f"{prefix}.{f}"] = np.int64(getattr(meta, f))
    return out


def torch_quantize_like_triton(x_bf16: torch.Tensor, meta) -> tuple[np.ndarray, np.ndarray]:
    """PyTorch transliteration of quant.py:129-167 for the padded layout."""
    x = x_bf16.float()
    n = x.shape[1]
    total = int(meta.total_blocks)
    pitch = max(128, (int(meta.padded_rows) + 127) // 128 * 128)
    data = np.zeros((n, pitch), dtype=np.uint8)
    scales = np.zeros((total, n), dtype=np.float32)
    starts = _plain(meta.block_row_start)
    counts = _plain(meta.block_row_count)
    for b in range(total):
        r0, rows = int(starts[b]), int(counts[b])
        vals = torch.zeros((128, n), dtype=torch.float32)
        vals[:rows] = x[r0 : r0 + rows]
        amax = vals.abs().amax(dim=0)
        scale = torch.clamp_min(amax / 448.0, 1.0e-12)
        scales[b] = scale.numpy()
        q = (vals / scale[None, :]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        data[:, b * 128 : b * 128 + rows] = q[:rows].T
    return data, scales


def reference_triton_quantize(x_bf16: torch.Tensor, meta, ref_quant, layout: str) -> dict:
    """The reference launcher + Triton kernel under the interpreter, on CPU.
    Returns the operand storage bytes ([cols][pitch]), the packed launch copy
    ([cols][K], packed layout only) and the scales."""
    op = ref_quant.quantize_grouped_wgrad_operand_128x1(x_bf16.as_subclass(_CudaLike), meta, layout_mode=layout)
    data = op.data.as_subclass(torch.Tensor)             # logical [K, cols], K contiguous
    out = {"storage": data.t().contiguous().view(torch.uint8).numpy().copy(),   # [cols][K]
           "scales": op.scales.as_subclass(torch.Tensor).numpy().copy()}
    if op.kernel_data is not None:
        out["kernel_data"] = op.kernel_data.as_subclass(torch.Tensor).view(torch.uint8).numpy().copy()
    return out


def _operand(data: np.ndarray, scales: np.ndarray, k_rows: int, ref_quant):
    storage = torch.from_numpy(data.copy()).view(torch.float8_e4m3fn)
    view = storage.as_strided((k_rows, data.shape[0]), (1, data.shape[1]))
    return ref_quant.Fp8GroupedWgradOperand(view, torch.from_numpy(scales.copy()))


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    import sm90_fp8_wgrad.block_meta as ref_meta
    import sm90_fp8_wgrad.checks as ref_checks
    import sm90_fp8_wgrad.quant as ref_quant

    def cu_of(counts):
        cu = torch.zeros(len(counts) + 1, dtype=torch.int32)
        if counts:
            cu[1:] = torch.cumsum(torch.tensor(counts, dtype=torch.int32), 0)
        return cu.as_subclass(_CudaLike)

    # ---------------------------------------------------------- metadata cases
    meta_out = {}
    for name, counts in META_CASES.items():
        meta_out[f"{name}.counts"] = np.asarray(counts, dtype=np.int64)
        for mode in ("masked128", "adaptive64", "adaptive32_64_128", "adaptive32_64_twophase"):
            m = ref_meta.build_wgrad_scale_block_meta(cu_of(counts), packed_tail_tma_mode=mode)
            meta_out.update(_meta_arrays(m, f"{name}.{mode}"))
        for tbk in (32, 64):
            t = ref_meta.build_wgrad_tail_block_meta(cu_of(counts), tail_block_k=tbk)
            meta_out.update(_meta_arrays(t.meta, f"{name}.tail{tbk}"))
            meta_out[f"{name}.tail{tbk}.tail_indices"] = _plain(t.tail_indices).astype(np.int64)
        s = ref_meta.build_wgrad_full_block_split(cu_of(counts))
        meta_out.update(_meta_arrays(s.full_meta, f"{name}.full"))
        meta_out[f"{name}.full.tail_indices"] = _plain(s.tail_indices).astype(np.int64)
        meta_out[f"{name}.full.tail_cu_seqlens_k"] = _plain(s.tail_cu_seqlens_k).astype(np.int64)
        meta_out[f"{name}.full.full_rows"] = np.int64(s.full_rows)
        meta_out[f"{name}.full.tail_rows"] = np.int64(s.tail_rows)
    np.savez_compressed(HERE / "meta_cases.npz", **meta_out)

    # --------------------------------------------- small quantiser + wgrad cases
    q_out, w_out = {}, {}
    for name, spec in SMALL_CASES.items():
        inp = case_inputs(spec)
        meta = ref_meta.build_wgrad_scale_block_meta(cu_of(spec["counts"]))
        ops = {}
        for key in ("lhs_down", "rhs_down", "lhs_gate", "rhs_gate"):
            x = torch.from_numpy(bf16_from_f32(inp[key])).view(torch.bfloat16)
            data, scales = torch_quantize_like_triton(x, meta)
            q_out[f"{name}.{key}.data"] = data
            q_out[f"{name}.{key}.scales"] = scales
            ops[key] = _operand(data, scales, int(meta.padded_rows), ref_quant)
        for stage, (lk, rk) in {"down": ("lhs_down", "rhs_down"), "gate": ("lhs_gate", "rhs_gate")}.items():
            ref = ref_checks.ref_scaled_wgrad(ops[lk], ops[rk], meta, out_dtype=torch.float32)
            w_out[f"{name}.{stage}.ref_f32"] = ref.numpy()
            w_out[f"{name}.{stage}.ref_bf16"] = ref.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
            # calc_diff of the bf16-rounded reference against the fp32 one
            w_out[f"{name}.{stage}.calc_diff_bf16_vs_f32"] = np.float64(
                ref_checks._deepseek_calc_diff_chunked(ref.to(torch.bfloat16).float(), ref))
            max_abs, max_rel, max_ref = ref_checks.scaled_wgrad_error(ref.to(torch.bfloat16), ref)
            w_out[f"{name}.{stage}.error_bf16_vs_f32"] = np.asarray([max_abs, max_rel, max_ref], np.float64)
    np.savez_compressed(HERE / "quant_small.npz", **q_out)

    # ------------------- the reference's Triton quantiser itself (interpreter)
    t_out = {"generator": np.asarray("reference quantize_grouped_wgrad_operand_128x1 + Triton kernel, "
                                     "TRITON_INTERPRET=1 on CPU")}
    for name, spec in SMALL_CASES.items():
        inp = case_inputs(spec)
        meta = ref_meta.build_wgrad_scale_block_meta(cu_of(spec["counts"]))
        for key in ("lhs_down", "rhs_down", "lhs_gate", "rhs_gate"):
            x = torch.from_numpy(bf16_from_f32(inp[key])).view(torch.bfloat16)
            for layout in ("padded", "packed"):
                r = reference_triton_quantize(x, meta, ref_quant, layout)
                for k, v in r.items():
                    t_out[f"{name}.{key}.{layout}.{k}"] = v
    np.savez_compressed(HERE / "quant_triton.npz", **t_out)
    np.savez_compressed(HERE / "wgrad_small.npz", **w_out)

    # ---------------------------------------------------------- tiny C1 config
    inp = case_inputs(C1)
    meta = ref_meta.build_wgrad_scale_block_meta(cu_of(C1["counts"]))
    c1 = {"counts": np.asarray(C1["counts"], np.int64)}
    ops = {}
    for key in ("lhs_down", "rhs_down", "lhs_gate", "rhs_gate"):
        x = torch.from_numpy(bf16_from_f32(inp[key])).view(torch.bfloat16)
        data, scales = torch_quantize_like_triton(x, meta)
        c1[f"{key}.data_sha256"] = np.asarray(_sha(data))
        c1[f"{key}.scales_sha256"] = np.asarray(_sha(scales))
        ops[key] = _operand(data, scales, int(meta.padded_rows), ref_quant)
    for stage, (lk, rk) in {"down": ("lhs_down", "rhs_down"), "gate": ("lhs_gate", "rhs_gate")}.items():
        ref = ref_checks.ref_scaled_wgrad(ops[lk], ops[rk], meta, out_dtype=torch.float32).numpy()
        c1[f"{stage}.expert_sum"] = ref.reshape(ref.shape[0], -1).sum(axis=1, dtype=np.float64)
        c1[f"{stage}.expert_sumsq"] = (ref.astype(np.float64) ** 2).reshape(ref.shape[0], -1).sum(axis=1)
        flat = ref.reshape(-1)
        idx = np.arange(0, flat.size, 97, dtype=np.int64)
        c1[f"{stage}.sample_idx"] = idx
        c1[f"{stage}.sample"] = flat[idx]
    np.savez_compressed(HERE / "c1_tiny.npz", **c1)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
