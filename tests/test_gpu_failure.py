"""Failure detection on the GPU without a fault (bounded waits).

Every mbarrier wait of the GEMM gives up after a bounded time, records the
role that gave up in the device error word and lets the CTA exit cleanly.
A test-only injection (``SM100_WGRAD_DEBUG_INJECT=withhold_first_load``) makes
the producer announce its first stage's bytes without issuing the copy, so the
consumers' waits run out. The launch must finish in seconds, the error word
must name a timed-out role (1 producer, 2 MMA, 3 epilogue), and the CUDA
context must stay usable: the next normal launch is exact.
"""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import wgrad_oracle as O
from golden_inputs import C1, case_inputs

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_context_survives(cuda_device, monkeypatch):
    from sm90_fp8_wgrad import (_lib, build_wgrad_scale_block_meta, fp8_grouped_wgrad_sm90,
                                quantize_grouped_wgrad_operand_128x1)

    counts = C1["counts"]
    cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    meta = build_wgrad_scale_block_meta(torch.from_numpy(cu).to(cuda_device, torch.int32))
    inp = case_inputs(C1)
    lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["lhs_gate"]).to(cuda_device).to(torch.bfloat16), meta)
    rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["rhs_gate"]).to(cuda_device).to(torch.bfloat16), meta)
    out = torch.full((len(counts), lhs.data.shape[1], rhs.data.shape[1]), float("nan"), device=cuda_device,
                     dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert _lib.device_error() in (0, 1, 2, 3, 4, 5)   # clear anything left by earlier tests

    monkeypatch.setenv("SM100_WGRAD_DEBUG_INJECT", "withhold_first_load")
    t0 = time.time()
    fp8_grouped_wgrad_sm90(lhs, rhs, out, meta)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    code = _lib.device_error()
    assert code in (1, 2, 3), code
    assert elapsed < 60.0

    monkeypatch.delenv("SM100_WGRAD_DEBUG_INJECT")
    fp8_grouped_wgrad_sm90(lhs, rhs, out, meta)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    om = O.build_meta(cu)
    ref = O.ref_scaled_wgrad(O.quantize_1x128(inp["lhs_gate"], om), O.quantize_1x128(inp["rhs_gate"], om), om)
    assert O.calc_diff(out.float().cpu().numpy(), ref) <= 1e-5
