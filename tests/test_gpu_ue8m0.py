"""GPU parity of the UE8M0 path: the quantiser with power-of-two scales
(scale_format="ue8m0") and the block-scaled grouped Wgrad kernel
(tcgen05.mma kind::mxf8f6f4.block_scale, tuned_config "sm100_128x192_ue8m0"),
both through the C-ABI library, against the CPU oracle.

The reference has no UE8M0 mode; its contract formula still defines the result:
out[e,m,n] = sum_b sum_k qa[k,m] sa[b,m] qb[k,n] sb[b,n] (interface.py:149-155),
which the oracle evaluates in fp32 on the same FP8 bytes and scales. Tolerances
are those of the promotion kernels' parity tests (test_gpu_parity.py): BF16 out
calc_diff <= 1e-5 (contract gate) and <= 1e-6 against the BF16-rounded oracle;
fp32 out calc_diff <= 1e-9 and |gpu - ref| <= 1e-4 |ref| + 1e-6 max|ref|.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

import wgrad_oracle as O
from golden_inputs import C1, SMALL_CASES, case_inputs
from test_gpu_parity import STAGES, _check_bf16, _check_f32, _cu

pytestmark = pytest.mark.gpu

UE8M0 = "sm100_128x192_ue8m0"


def _gpu_case(spec, dev, scale_format="ue8m0"):
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta, quantize_grouped_wgrad_operand_128x1

    meta = build_wgrad_scale_block_meta(torch.from_numpy(_cu(spec["counts"])).to(device=dev, dtype=torch.int32))
    inp = case_inputs(spec)
    ops = {k: quantize_grouped_wgrad_operand_128x1(torch.from_numpy(v).to(dev).to(torch.bfloat16), meta,
                                                   scale_format=scale_format)
           for k, v in inp.items()}
    return meta, ops


def _oracle_case(spec):
    meta = O.build_meta(_cu(spec["counts"]))
    return meta, {k: O.quantize_1x128(v, meta, "ue8m0") for k, v in case_inputs(spec).items()}


def _device_error():
    from sm90_fp8_wgrad import _lib

    return _lib.device_error()


@pytest.mark.parametrize("case", sorted(SMALL_CASES) + ["c1"])
def test_ue8m0_quantiser_bit_exact(cuda_device, case):
    spec = C1 if case == "c1" else SMALL_CASES[case]
    _, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    for k, op in ops.items():
        assert op.scale_format == "ue8m0"
        pitch = op.data.stride(1)
        storage = op.data.as_strided((op.data.shape[1], pitch), (pitch, 1)).view(torch.uint8).cpu().numpy()
        np.testing.assert_array_equal(storage[:, : om.padded_rows], oops[k].data[:, : om.padded_rows], err_msg=k)
        bits = op.scales.cpu().numpy().view(np.uint32)
        np.testing.assert_array_equal(bits, oops[k].scales.view(np.uint32), err_msg=k)
        assert not (bits & 0x7FFFFF).any(), "every scale is a power of two"


@pytest.mark.parametrize("tuned_config", ["default", UE8M0])
@pytest.mark.parametrize("case", sorted(SMALL_CASES) + ["c1"])
def test_ue8m0_gemm_matches_oracle(cuda_device, case, tuned_config):
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = C1 if case == "c1" else SMALL_CASES[case]
    meta, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    e = len(spec["counts"])
    _device_error()
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        out = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=tuned_config)
        torch.cuda.synchronize()
        _check_bf16(out, O.ref_scaled_wgrad(oops[lk], oops[rk], om))
    assert _device_error() == 0


def test_ue8m0_default_dispatch_and_promotion_kernel_agree(cuda_device):
    """Default config on UE8M0 operands runs the block-scaled kernel (bit-equal
    to the explicit config); the promotion kernel on the same operands gives
    the same sum to fp32 rounding."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = {"counts": [0, 640, 3, 129, 0, 1100, 77], "tokens": 800, "hidden": 272, "intermediate": 208, "seed": 9}
    meta, ops = _gpu_case(spec, cuda_device)
    e = len(spec["counts"])
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        outs = {}
        for cfg in ("default", UE8M0, "sm100_128x256"):
            outs[cfg] = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.float32)
            fp8_grouped_wgrad_sm90(ops[lk], ops[rk], outs[cfg], meta, tuned_config=cfg)
        torch.cuda.synchronize()
        assert torch.equal(outs["default"], outs[UE8M0])
        a, b = outs[UE8M0].cpu().numpy(), outs["sm100_128x256"].cpu().numpy()
        assert O.calc_diff(a, b) <= 1e-10
        np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-6 * float(np.abs(b).max()))


def test_ue8m0_fp32_out_and_accumulate(cuda_device):
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = SMALL_CASES["mixed"]
    meta, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    e = len(spec["counts"])
    lk, rk = STAGES["gate"]
    m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
    ref = O.ref_scaled_wgrad(oops[lk], oops[rk], om)
    out = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.float32)
    fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=UE8M0)
    _check_f32(out, ref)
    base = torch.randn((e, m, n), device=cuda_device, dtype=torch.float32) * float(np.abs(ref).max())
    acc = base.clone()
    fp8_grouped_wgrad_sm90(ops[lk], ops[rk], acc, meta, accumulate=True, tuned_config=UE8M0)
    _check_f32(acc - base, ref)
    base16 = base.to(torch.bfloat16)
    acc16 = base16.clone()
    fp8_grouped_wgrad_sm90(ops[lk], ops[rk], acc16, meta, accumulate=True, tuned_config=UE8M0)
    expect = O.bf16_round(base16.float().cpu().numpy() + ref)
    np.testing.assert_allclose(acc16.float().cpu().numpy(), expect, rtol=2 ** -7,
                               atol=1e-5 * float(np.abs(expect).max()))


@pytest.mark.parametrize("hidden,inter", [(144, 80), (272, 48), (512, 208)])
def test_ue8m0_ragged_tiles(cuda_device, hidden, inter):
    """M, N not multiples of the 128 x 192 tile; empty experts; long K."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = {"counts": [0, 640, 3, 129, 0, 1100], "tokens": 700, "hidden": hidden, "intermediate": inter, "seed": 5}
    meta, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        out = torch.full((6, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=UE8M0)
        _check_bf16(out, O.ref_scaled_wgrad(oops[lk], oops[rk], om))


@pytest.mark.parametrize("counts", [[0, 0, 0, 0], [300], [(e * 7) % 4 for e in range(1024)]],
                         ids=["all_empty", "one_expert", "1024_tiny_experts"])
def test_ue8m0_edge_expert_sets(cuda_device, counts):
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = {"counts": counts, "tokens": max(8, sum(counts)), "hidden": 144, "intermediate": 80, "seed": 13}
    meta, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    e = len(counts)
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        out = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=UE8M0)
        _check_bf16(out, O.ref_scaled_wgrad(oops[lk], oops[rk], om))


def test_ue8m0_packed_layout_and_expert_range(cuda_device, monkeypatch):
    """Packed layout (masked tail UMMAs) and an expert sub-range launch."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    monkeypatch.setenv("KERNEL_LAB_WGRAD_LAYOUT_MODE", "packed")
    spec = {"counts": [5, 200, 0, 129, 31, 64], "tokens": 300, "hidden": 144, "intermediate": 80, "seed": 21}
    meta, ops = _gpu_case(spec, cuda_device)
    om, oops = _oracle_case(spec)
    e = len(spec["counts"])
    for lk, rk in STAGES.values():
        m, n = ops[lk].data.shape[1], ops[rk].data.shape[1]
        ref = O.ref_scaled_wgrad(oops[lk], oops[rk], om)
        out = torch.full((e, m, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=UE8M0)
        _check_bf16(out, ref)
        part = torch.full_like(out, float("nan"))
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], part, meta, tuned_config=UE8M0, expert_range=(1, 4))
        torch.cuda.synchronize()
        assert torch.equal(part[1:4], out[1:4])
        assert torch.isnan(part[0]).all() and torch.isnan(part[4:]).all()


def test_ue8m0_config_needs_ue8m0_operands(cuda_device):
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = SMALL_CASES["single"]
    meta, ops = _gpu_case(spec, cuda_device, scale_format="fp32")
    lk, rk = STAGES["down"]
    out = torch.empty((1, ops[lk].data.shape[1], ops[rk].data.shape[1]), device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="ue8m0"):
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta, tuned_config=UE8M0)


def test_ue8m0_kernel_flags_scales_that_are_not_powers_of_two(cuda_device):
    """fp32 scales labelled UE8M0: the kernel reads them as 1.0 and sets device
    error 6 (no fault, the context stays usable)."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    spec = SMALL_CASES["single"]
    meta, ops = _gpu_case(spec, cuda_device, scale_format="fp32")
    lk, rk = STAGES["down"]
    lhs = dataclasses.replace(ops[lk], scale_format="ue8m0")
    rhs = dataclasses.replace(ops[rk], scale_format="ue8m0")
    out = torch.empty((1, lhs.data.shape[1], rhs.data.shape[1]), device=cuda_device, dtype=torch.bfloat16)
    _device_error()
    fp8_grouped_wgrad_sm90(lhs, rhs, out, meta, tuned_config=UE8M0)
    torch.cuda.synchronize()
    assert _device_error() == 6
    assert _device_error() == 0  # read-and-clear


def test_mislabelled_ue8m0_scales_raise(cuda_device):
    """The error reaches the caller without a synchronisation: the next call of
    the operator raises, and so does the explicit check."""
    from sm90_fp8_wgrad import check_device_errors, fp8_grouped_wgrad_sm90

    spec = SMALL_CASES["single"]
    meta, ops = _gpu_case(spec, cuda_device, scale_format="fp32")
    lk, rk = STAGES["down"]
    lhs = dataclasses.replace(ops[lk], scale_format="ue8m0")
    rhs = dataclasses.replace(ops[rk], scale_format="ue8m0")
    out = torch.empty((1, lhs.data.shape[1], rhs.data.shape[1]), device=cuda_device, dtype=torch.bfloat16)
    _device_error()
    fp8_grouped_wgrad_sm90(lhs, rhs, out, meta)          # auto selects the UE8M0 kernel from the label
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device error 6"):
        fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta)
    with pytest.raises(RuntimeError, match="device error 6"):
        check_device_errors(cuda_device)
    fp8_grouped_wgrad_sm90(ops[lk], ops[rk], out, meta)  # reported once: the context is usable
    check_device_errors(cuda_device)
