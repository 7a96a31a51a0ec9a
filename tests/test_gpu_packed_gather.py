"""GPU parity of the packed layout mode and the fused gather + quantiser.

Packed layout (reference quant.py:196-266, interface.py:173-241): operand bytes
in ``data`` and ``kernel_data`` bit-exact against the oracle's packed layout of
the same quantised operand, for every packed tail policy; the grouped GEMM
over the packed operands equal, bit for bit, to the padded-layout result (the
skipped tail K slices only ever multiplied zeros). Fused gather: quantising
token-major rows through a gather index is byte-identical to gathering first.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import wgrad_oracle as O
from golden_inputs import C1, SMALL_CASES, case_inputs

pytestmark = pytest.mark.gpu

POLICIES = ("masked128", "adaptive64", "adaptive32_64_128", "adaptive32_64_twophase")
EDGE_COUNTS = [1, 31, 32, 33, 63, 64, 65, 127, 128, 129, 0, 255, 256, 257]


def _cu(counts):
    return np.concatenate([[0], np.cumsum(np.asarray(counts, np.int64))]).astype(np.int64)


def _bytes(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).cpu().numpy()


@pytest.mark.parametrize("policy", POLICIES)
@pytest.mark.parametrize("case", ["edge", "c1"])
def test_packed_operand_bytes_match_oracle(cuda_device, case, policy):
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta, quantize_grouped_wgrad_operand_128x1

    counts = EDGE_COUNTS if case == "edge" else C1["counts"]
    rng = np.random.Generator(np.random.PCG64(11))
    x = rng.standard_normal((sum(counts), 96), dtype=np.float32)
    om = O.build_meta(_cu(counts), packed_tail_tma_mode=policy)
    data_ref, kernel_ref = O.packed_layout(O.quantize_1x128(x, om), om, policy)
    meta = build_wgrad_scale_block_meta(torch.from_numpy(_cu(counts)).to(cuda_device, torch.int32),
                                        packed_tail_tma_mode=policy)
    op = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(x).to(cuda_device), meta, layout_mode="packed")
    got = _bytes(op.data.t())                       # [cols, valid_rows]
    np.testing.assert_array_equal(got, data_ref)
    kd = _bytes(op.kernel_data)
    assert kd.shape[1] >= kernel_ref.shape[1]
    np.testing.assert_array_equal(kd[:, : kernel_ref.shape[1]], kernel_ref)
    assert not kd[:, kernel_ref.shape[1]:].any()
    np.testing.assert_array_equal(op.scales.cpu().numpy().view(np.uint32),
                                  O.quantize_1x128(x, om).scales.view(np.uint32))


@pytest.mark.parametrize("policy", POLICIES)
@pytest.mark.parametrize("case", sorted(SMALL_CASES) + ["c1", "edge"])
def test_packed_gemm_equals_padded(cuda_device, case, policy, monkeypatch):
    from sm90_fp8_wgrad import (build_wgrad_scale_block_meta, fp8_grouped_wgrad_sm90,
                                quantize_grouped_wgrad_operand_128x1)

    if case == "edge":
        spec = {"counts": EDGE_COUNTS, "tokens": 600, "hidden": 144, "intermediate": 80, "seed": 5}
    else:
        spec = C1 if case == "c1" else SMALL_CASES[case]
    inp = case_inputs(spec)
    meta = build_wgrad_scale_block_meta(torch.from_numpy(_cu(spec["counts"])).to(cuda_device, torch.int32),
                                        packed_tail_tma_mode=policy)
    e = len(spec["counts"])
    for lk, rk in (("lhs_down", "rhs_down"), ("lhs_gate", "rhs_gate")):
        outs = {}
        for mode in ("padded", "packed"):
            monkeypatch.setenv("KERNEL_LAB_WGRAD_LAYOUT_MODE", mode)
            lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp[lk]).to(cuda_device).to(torch.bfloat16),
                                                       meta, layout_mode=mode)
            rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp[rk]).to(cuda_device).to(torch.bfloat16),
                                                       meta, layout_mode=mode)
            out = torch.full((e, lhs.data.shape[1], rhs.data.shape[1]), float("nan"), device=cuda_device,
                             dtype=torch.bfloat16)
            fp8_grouped_wgrad_sm90(lhs, rhs, out, meta)
            outs[mode] = out
        torch.cuda.synchronize()
        assert torch.isfinite(outs["padded"].float()).all()
        assert torch.equal(outs["padded"].view(torch.int16), outs["packed"].view(torch.int16)), (case, policy, lk)


def test_packed_operator_rejects_missing_guard(cuda_device, monkeypatch):
    from sm90_fp8_wgrad import (Fp8GroupedWgradOperand, build_wgrad_scale_block_meta, fp8_grouped_wgrad_sm90,
                                quantize_grouped_wgrad_operand_128x1)

    counts = [40, 0, 130]
    meta = build_wgrad_scale_block_meta(torch.from_numpy(_cu(counts)).to(cuda_device, torch.int32))
    x = torch.randn(sum(counts), 32, device=cuda_device)
    op = quantize_grouped_wgrad_operand_128x1(x, meta, layout_mode="packed")
    short = Fp8GroupedWgradOperand(op.data, op.scales, kernel_data=op.kernel_data[:, : meta.wgmma_rows])
    out = torch.empty((3, 32, 32), device=cuda_device, dtype=torch.bfloat16)
    monkeypatch.setenv("KERNEL_LAB_WGRAD_LAYOUT_MODE", "packed")
    with pytest.raises(RuntimeError, match="guard"):
        fp8_grouped_wgrad_sm90(short, op, out, meta)
    with pytest.raises(RuntimeError, match="kernel_data is required"):
        fp8_grouped_wgrad_sm90(Fp8GroupedWgradOperand(op.data, op.scales), op, out, meta)


@pytest.mark.parametrize("mode", ["padded", "packed"])
def test_fused_gather_quantiser_equals_gather_then_quantise(cuda_device, mode):
    from sm90_fp8_wgrad import (build_wgrad_scale_block_meta, quantize_grouped_wgrad_operand_128x1,
                                quantize_grouped_wgrad_operand_128x1_gather)
    from sm90_fp8_wgrad.routing import make_routing

    routing = make_routing(tokens=1024, experts=8, top_k=2, route="zipf", seed=3)
    x = torch.randn(1024, 264, device=cuda_device).to(torch.bfloat16)
    idx = routing.gather_idx.to(cuda_device)
    cu = torch.from_numpy(_cu(routing.counts)).to(cuda_device, torch.int32)
    meta = build_wgrad_scale_block_meta(cu)
    fused = quantize_grouped_wgrad_operand_128x1_gather(x, idx, meta, layout_mode=mode)
    ref = quantize_grouped_wgrad_operand_128x1(x.index_select(0, idx.long()).contiguous(), meta, layout_mode=mode)
    assert torch.equal(_t(fused.data), _t(ref.data))
    assert torch.equal(fused.scales.view(torch.int32), ref.scales.view(torch.int32))
    if mode == "packed":
        assert torch.equal(fused.kernel_data.view(torch.uint8), ref.kernel_data.view(torch.uint8))


def _t(d: torch.Tensor) -> torch.Tensor:
    pitch = d.stride(1)
    return d.as_strided((d.shape[1], pitch), (pitch, 1)).view(torch.uint8)[:, : d.shape[0]]
