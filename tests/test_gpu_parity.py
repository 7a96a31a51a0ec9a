"""GPU parity: the CUDA metadata builder, quantiser and grouped Wgrad GEMM
(all through the C-ABI library) against the CPU oracle.

Tolerances (FP8 operands are identical bytes on both sides, so only the
accumulation order and the final rounding differ):
  * metadata, FP8 bytes and scales: bit-exact;
  * BF16 output vs the oracle's fp32 result: DeepSeek calc_diff <= 1e-5 (the
    contract gate), calc_diff vs the BF16-rounded oracle <= 1e-6, and
    elementwise |gpu - ref| <= 2^-7 |ref| + 1e-5 max|ref| (one BF16 ulp plus
    fp32 accumulation-order noise);
  * fp32 output: calc_diff <= 1e-9, |gpu - ref| <= 1e-4 |ref| + 1e-6 max|ref|.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import wgrad_oracle as O
from golden_inputs import C1, SMALL_CASES, case_inputs

pytestmark = pytest.mark.gpu

STAGES = {"down": ("lhs_down", "rhs_down"), "gate": ("lhs_gate", "rhs_gate")}


def _cu(counts):
    return np.concatenate([[0], np.cumsum(np.asarray(counts, np.int64))]).astype(np.int64)


def _gpu_case(spec, dev, x_dtype=torch.bfloat16):
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta, quantize_grouped_wgrad_operand_128x1

    cu = torch.from_numpy(_cu(spec["counts"])).to(device=dev, dtype=torch.int32)
    meta = build_wgrad_scale_block_meta(cu)
    inp = case_inputs(spec)
    ops = {k: quantize_grouped_wgrad_operand_128x1(torch.from_numpy(v).to(dev).to(x_dtype), meta)
           for k, v in inp.items()}
    return meta, inp, ops


def _oracle_case(spec):
    meta = O.build_meta(_cu(spec["counts"]))
    inp = case_inputs(spec)
    return meta, {k: O.quantize_1x128(v, meta) for k, v in inp.items()}


def _check_bf16(out_gpu: torch.Tensor, ref: np.ndarray):
    got = out_gpu.float().cpu().numpy()
    assert np.isfinite(got).all()
    if ref.size == 0 or not np.abs(ref).max() > 0:
        np.testing.assert_array_equal(got, 0.0)
        return {"calc_diff": 0.0}
    cd = O.calc_diff(got, ref)
    cd_b = O.calc_diff(got, O.bf16_round(ref))
    assert cd <= 1e-5, cd
    assert cd_b <= 1e-6, cd_b
    scale = float(np.abs(ref).max())
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-5 * scale)
    return {"calc_diff": cd, "calc_diff_bf16": cd_b, "max_rel": O.scaled_wgrad_error(got, ref)[1]}


def _check_f32(out_gpu: torch.Tensor, ref: np.ndarray):
    got = out_gpu.cpu().numpy()
    assert np.isfinite(got).all()
    if not np.abs(ref).max() > 0:
        np.testing.assert_array_equal(got, 0.0)
        return
    assert O.calc_diff(got, ref) <= 1e-9
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-6 * float(np.abs(ref).max()))


@pytest.mark.parametrize("case", sorted(SMALL_CASES) + ["c1"])
def test_meta_builder_matches_oracle(cuda_device, case):
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta

    spec = C1 if case == "c1" else SMALL_CASES[case]
    om = O.build_meta(_cu(spec["counts"]))
    gm = build_wgrad_scale_block_meta(torch.from_numpy(_cu(spec["counts"])).to(cuda_device, torch.int32))
    for f in ("padded_cu_seqlens_k", "wgmma_cu_seqlens_k", "tma_cu_seqlens_k", "blocks_per_expert",
              "block_offsets", "block_row_start", "wgmma_block_row_start", "tma_block_row_start",
              "block_row_count", "tail_valid_rows", "tail_wgmma_atoms", "tail_copy_k", "has_tail"):
        np.testing.assert_array_equal(getattr(gm, f).cpu().numpy().astype(np.int64),
                                      np.asarray(getattr(om, f)).astype(np.int64), err_msg=f)
    for f in ("valid_rows", "padded_rows", "wgmma_rows", "tma_rows", "total_blocks"):
        assert getattr(gm, f) == getattr(om, f), f
    np.testing.assert_array_equal(gm.expert_order.cpu().numpy(), O.lpt_expert_order(om.blocks_per_expert))


@pytest.mark.parametrize("counts", [[0, 0, 0, 0], [1, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256, 257],
                                    [70000, 0, 17, 4096], list(range(0, 3000, 7))])
def test_meta_builder_edge_routings(cuda_device, counts):
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta

    om = O.build_meta(_cu(counts))
    gm = build_wgrad_scale_block_meta(torch.from_numpy(_cu(counts)).to(cuda_device, torch.int32))
    for f in ("block_offsets", "block_row_start", "block_row_count", "wgmma_cu_seqlens_k", "wgmma_block_row_start"):
        np.testing.assert_array_equal(getattr(gm, f).cpu().numpy().astype(np.int64), getattr(om, f), err_msg=f)
    assert gm.total_blocks == om.total_blocks


def test_meta_builder_rejects_non_monotonic(cuda_device):
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta

    with pytest.raises(RuntimeError, match="monotonic"):
        build_wgrad_scale_block_meta(torch.tensor([0, 10, 5], dtype=torch.int32, device=cuda_device))


@pytest.mark.parametrize("case", sorted(SMALL_CASES) + ["c1"])
def test_quantiser_bit_exact(cuda_device, case):
    spec = C1 if case == "c1" else SMALL_CASES[case]
    meta, inp, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    for k, op in ops.items():
        pitch = op.data.stride(1)
        storage = op.data.as_strided((op.data.shape[1], pitch), (pitch, 1)).view(torch.uint8).cpu().numpy()
        np.testing.assert_array_equal(storage[:, : om.padded_rows], oops[k].data[:, : om.padded_rows], err_msg=k)
        np.testing.assert_array_equal(op.scales.cpu().numpy().view(np.uint32), oops[k].scales.view(np.uint32),
                                      err_msg=k)


def test_quantiser_fp32_input_and_odd_columns(cuda_device):
    """fp32 source, a column count that is not a multiple of the 64-column tile."""
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta, quantize_grouped_wgrad_operand_128x1

    counts = [5, 200, 0, 129]
    rng = np.random.Generator(np.random.PCG64(3))
    x = (rng.standard_normal((sum(counts), 72), dtype=np.float32) * np.float32(3.0))
    x[7, 3] = 0.0
    x[:, 5] = 0.0                                  # all-zero column -> scale floor 1e-12
    om = O.build_meta(_cu(counts))
    ref = O.quantize_1x128(x, om)
    meta = build_wgrad_scale_block_meta(torch.from_numpy(_cu(counts)).to(cuda_device, torch.int32))
    op = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(x).to(cuda_device), meta)
    pitch = op.data.stride(1)
    storage = op.data.as_strided((72, pitch), (pitch, 1)).view(torch.uint8).cpu().numpy()
    np.testing.assert_array_equal(storage[:, : om.padded_rows], ref.data[:, : om.padded_rows])
    np.testing.assert_array_equal(op.scales.cpu().numpy().view(np.uint32), ref.scales.view(np.uint32))


@pytest.mark.parametrize("tuned_config", ["default", "sm100_128x128", "sm100_128x256_w8", "sm100_128x256_w16",
                                          "sm100_128x128_2cta", "sm100_128x192_w12", "sm100_256x256_pair",
                                          "sm100_256x256_pair_w16", "sm100_256x256_sp", "sm100_256x256_sp_w16"])
@pytest.mark.parametrize("case", sorted(SMALL_CASES) + ["c1"])
def test_grouped_wgrad_matches_oracle(cuda_device, case, tuned_config):
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = C1 if case == "c1" else SMALL_CASES[case]
    meta, _, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    e = len(spec["counts"])
    for stage, (lk, rk) in STAGES.items():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        out = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)  # poison
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=tuned_config)
        torch.cuda.synchronize()
        ref = O.ref_scaled_wgrad(oops[lk], oops[rk], om)
        _check_bf16(out, ref)
    from sm90_fp8_wgrad import _lib

    assert _lib.device_error() == 0


@pytest.mark.parametrize("tuned_config", ["default", "sm100_128x256_w8", "sm100_128x256_w16", "sm100_128x128_2cta",
                                          "sm100_128x192_w12", "sm100_256x256_pair", "sm100_256x256_sp", "sm100_256x256_sp_w16"])
def test_grouped_wgrad_fp32_out_and_accumulate(cuda_device, tuned_config):
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = SMALL_CASES["mixed"]
    meta, _, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    e = len(spec["counts"])
    lk, rk = STAGES["gate"]
    m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
    ref = O.ref_scaled_wgrad(oops[lk], oops[rk], om)
    out = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.float32)
    fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=tuned_config)
    _check_f32(out, ref)
    base = torch.randn((e, m, n), device=cuda_device, dtype=torch.float32) * float(np.abs(ref).max())
    acc = base.clone()
    fp8_grouped_wgrad_sm90(ops[lk], ops[rk], acc, meta, accumulate=True, tuned_config=tuned_config)
    _check_f32(acc - base, ref)
    base16 = base.to(torch.bfloat16)
    acc16 = base16.clone()
    fp8_grouped_wgrad_sm90(ops[lk], ops[rk], acc16, meta, accumulate=True, tuned_config=tuned_config)
    expect = O.bf16_round(base16.float().cpu().numpy() + ref)
    got = acc16.float().cpu().numpy()
    np.testing.assert_allclose(got, expect, rtol=2 ** -7, atol=1e-5 * float(np.abs(expect).max()))


@pytest.mark.parametrize("tuned_config", ["default", "sm100_128x256_w8", "sm100_128x256_w16", "sm100_128x128_2cta",
                                          "sm100_128x192_w12", "sm100_256x256_pair", "sm100_256x256_pair_w16",
                                          "sm100_256x256_sp", "sm100_256x256_sp_w16"])
@pytest.mark.parametrize("hidden,inter", [(144, 80), (272, 48), (512, 128)])
def test_grouped_wgrad_ragged_tiles(cuda_device, hidden, inter, tuned_config):
    """M, N not multiples of the 128 x 256 tile; empty experts; long K."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = {"counts": [0, 640, 3, 129, 0, 1100], "tokens": 700, "hidden": hidden, "intermediate": inter, "seed": 5}
    meta, _, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    for stage, (lk, rk) in STAGES.items():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        out = torch.full((6, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=tuned_config)
        _check_bf16(out, O.ref_scaled_wgrad(oops[lk], oops[rk], om))


def test_interface_validation_errors(cuda_device):
    from sm90_fp8_wgrad import Fp8GroupedWgradOperand, fp8_grouped_wgrad_sm90

    spec = SMALL_CASES["single"]
    meta, _, ops = _gpu_case(spec, cuda_device)
    lhs, rhs = ops["lhs_down"], ops["rhs_down"]
    out = torch.empty((1, lhs.data.shape[1], rhs.data.shape[1]), device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        fp8_grouped_wgrad_sm90(Fp8GroupedWgradOperand(lhs.data.view(torch.uint8), lhs.scales), rhs, out, meta)
    with pytest.raises(RuntimeError, match="out dtype"):
        fp8_grouped_wgrad_sm90(lhs, rhs, out.half(), meta)
    with pytest.raises(RuntimeError, match="unknown Wgrad config"):
        fp8_grouped_wgrad_sm90(lhs, rhs, out, meta, tuned_config="nope")
    with pytest.raises(RuntimeError, match="contiguous"):
        fp8_grouped_wgrad_sm90(lhs, rhs, out.transpose(1, 2), meta)


@pytest.mark.parametrize("tuned_config", ["default", "sm100_256x256_sp", "sm100_256x256_sp_w16"])
@pytest.mark.parametrize("splits", [[0, 2, 5, 8], [0, 0, 3, 3, 8], [0, 8]])
def test_expert_range_launches_equal_full_launch(cuda_device, splits, tuned_config):
    """out[e0:e1] from expert-range launches equals the full launch bit for bit
    (experts are independent); the experts outside a range stay untouched."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = C1
    meta, _, ops = _gpu_case(spec, cuda_device)
    e = len(spec["counts"])
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        full = torch.empty((e, m, n), device=cuda_device, dtype=torch.bfloat16)
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], full, meta, tuned_config=tuned_config)
        part = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        for a, b in zip(splits[:-1], splits[1:]):
            fp8_grouped_wgrad_sm90(ops[lk], ops[rk], part, meta, expert_range=(a, b), tuned_config=tuned_config)
            assert torch.isnan(part[b:].float()).all() or b == e
        assert torch.equal(part.view(torch.int16), full.view(torch.int16))
    with pytest.raises(RuntimeError, match="expert_range"):
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], full, meta, expert_range=(3, 2))


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("tuned_config", ["default", "sm100_128x256_w8", "sm100_128x256_w16", "sm100_128x128_2cta",
                                          "sm100_128x192_w12", "sm100_256x256_pair", "sm100_256x256_pair_w16",
                                          "sm100_256x256_sp", "sm100_256x256_sp_w16"])
def test_accumulate_on_ragged_tiles(cuda_device, tuned_config, out_dtype):
    """out += result where M, N are not multiples of the tile (the previous output
    comes in through TMA boxes that reach past M and N) and experts are empty."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = {"counts": [0, 640, 3, 129, 0, 1100], "tokens": 700, "hidden": 272, "intermediate": 48, "seed": 9}
    meta, _, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        ref = O.ref_scaled_wgrad(oops[lk], oops[rk], om)
        gen = torch.Generator(device=cuda_device).manual_seed(3)
        base = (torch.randn((6, m, n), device=cuda_device, generator=gen) * float(np.abs(ref).max())).to(out_dtype)
        acc = base.clone()
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], acc, meta, accumulate=True, tuned_config=tuned_config)
        expect = base.float().cpu().numpy() + ref
        if out_dtype == torch.bfloat16:
            expect = O.bf16_round(expect)
            np.testing.assert_allclose(acc.float().cpu().numpy(), expect, rtol=2 ** -7,
                                       atol=1e-5 * float(np.abs(expect).max()))
        else:
            _check_f32(acc - base, ref)


def test_legacy_quantiser_entry_point(cuda_device):
    """sm100_wgrad_quantize_1x128 (the plain C entry, padded layout) called through
    ctypes the way a C-ABI user would: bytes and scales bit-exact to the oracle."""
    import ctypes

    from sm90_fp8_wgrad import _lib, build_wgrad_scale_block_meta

    spec = SMALL_CASES["mixed"]
    meta = build_wgrad_scale_block_meta(torch.from_numpy(_cu(spec["counts"])).to(cuda_device, torch.int32))
    om, oops = _oracle_case(spec)
    inp = case_inputs(spec)
    lib = _lib.load()
    for k, v in inp.items():
        x = torch.from_numpy(v).to(cuda_device).to(torch.bfloat16).contiguous()
        rows, cols = x.shape
        pitch = max(128, (int(meta.padded_rows) + 127) // 128 * 128)
        q = torch.zeros((cols, pitch), device=cuda_device, dtype=torch.uint8)
        scales = torch.empty((int(meta.total_blocks), cols), device=cuda_device, dtype=torch.float32)
        st = lib.sm100_wgrad_quantize_1x128(
            ctypes.c_void_p(x.data_ptr()), 0, rows, cols, ctypes.c_void_p(meta.block_row_start.data_ptr()),
            ctypes.c_void_p(meta.block_row_count.data_ptr()), int(meta.total_blocks), ctypes.c_void_p(q.data_ptr()),
            pitch, ctypes.c_void_p(scales.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == _lib.OK, st
        torch.cuda.synchronize()
        np.testing.assert_array_equal(q[:, : om.padded_rows].cpu().numpy(), oops[k].data[:, : om.padded_rows], err_msg=k)
        np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), oops[k].scales.view(np.uint32), err_msg=k)


@pytest.mark.parametrize("counts", [[0, 0, 0, 0], [300], [(e * 7) % 4 for e in range(1024)]],
                         ids=["all_empty", "one_expert", "1024_tiny_experts"])
@pytest.mark.parametrize("tuned_config", ["default", "sm100_128x256_w16", "sm100_128x128_2cta", "sm100_256x256_pair",
                                          "sm100_256x256_sp", "sm100_256x256_sp_w16"])
def test_grouped_wgrad_edge_expert_sets(cuda_device, counts, tuned_config):
    """Every expert empty (no K rows at all: the launch has no operands and writes
    zeros), a single expert, and 1,024 experts of 0-3 rows each."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = {"counts": counts, "tokens": max(8, sum(counts)), "hidden": 144, "intermediate": 80, "seed": 13}
    meta, _, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    e = len(counts)
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        out = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=tuned_config)
        _check_bf16(out, O.ref_scaled_wgrad(oops[lk], oops[rk], om))
