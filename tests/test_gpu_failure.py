"""Failure detection on the GPU without a fault (bounded waits).

Every mbarrier wait of the GEMM gives up after a bounded time, records the
role that gave up in the device error word (and its host-mapped mirror) and
lets the CTA exit cleanly. A test-only injection that exists only in the
debug-modes library (``SM100_WGRAD_DEBUG_INJECT=withhold_first_load``) makes
the producer announce its first stage's bytes without issuing the copy, so the
consumers' waits run out. The launch must finish in seconds; without any
synchronisation by the caller the NEXT call of the operator must raise
``RuntimeError`` naming a timed-out role (1 producer, 2 MMA, 3 epilogue); and
the CUDA context must stay usable: the following normal launch is exact.
Runs in a child process because the library is chosen per process
(SM100_WGRAD_LIB), for the promotion kernel and the scale-product pair kernel.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
DEBUG_LIB = ROOT / "sm90-fp8-wgrad_b200" / "sm90_fp8_wgrad" / "_lib" / "libsm100_fp8_wgrad_debug.so"

CHILD = r"""
import json, os, sys, time, torch
import numpy as np
import wgrad_oracle as O
from golden_inputs import C1, case_inputs
from sm90_fp8_wgrad import (_lib, build_wgrad_scale_block_meta, check_device_errors, fp8_grouped_wgrad_sm90,
                            quantize_grouped_wgrad_operand_128x1)
cfg = sys.argv[1]
dev = torch.device("cuda:0")
assert _lib.build_flags() & _lib.BUILD_DEBUG_MODES
counts = C1["counts"]
cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
meta = build_wgrad_scale_block_meta(torch.from_numpy(cu).to(dev, torch.int32))
inp = case_inputs(C1)
lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["lhs_gate"]).to(dev).to(torch.bfloat16), meta)
rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["rhs_gate"]).to(dev).to(torch.bfloat16), meta)
out = torch.full((len(counts), lhs.data.shape[1], rhs.data.shape[1]), float("nan"), device=dev, dtype=torch.bfloat16)
torch.cuda.synchronize()
res = {}
os.environ["SM100_WGRAD_DEBUG_INJECT"] = "withhold_first_load"
t0 = time.time()
fp8_grouped_wgrad_sm90(lhs, rhs, out, meta, tuned_config=cfg)
torch.cuda.synchronize()
res["elapsed_s"] = time.time() - t0
del os.environ["SM100_WGRAD_DEBUG_INJECT"]
try:
    fp8_grouped_wgrad_sm90(lhs, rhs, out, meta, tuned_config=cfg)
    res["next_call"] = "returned"
except RuntimeError as exc:
    res["next_call"] = str(exc)
res["code"] = _lib.device_error()
fp8_grouped_wgrad_sm90(lhs, rhs, out, meta, tuned_config=cfg)
check_device_errors(dev)
om = O.build_meta(cu)
ref = O.ref_scaled_wgrad(O.quantize_1x128(inp["lhs_gate"], om), O.quantize_1x128(inp["rhs_gate"], om), om)
res["calc_diff_after"] = float(O.calc_diff(out.float().cpu().numpy(), ref))
print(json.dumps(res))
"""


@pytest.mark.parametrize("tuned_config", ["default", "sm100_256x256_sp"])
def test_bounded_wait_expires_next_call_raises_context_survives(cuda_device, tuned_config):
    if not DEBUG_LIB.is_file():
        pytest.fail(f"{DEBUG_LIB} missing: build it with build_ext.py --debug-modes")
    env = dict(os.environ, SM100_WGRAD_LIB=str(DEBUG_LIB))
    env.pop("SM100_WGRAD_DEBUG_INJECT", None)
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT / "sm90-fp8-wgrad_b200"), str(ROOT / "tests" / "golden"),
                                         str(ROOT / "oracle"), env.get("PYTHONPATH", "")])
    res = subprocess.run([sys.executable, "-c", CHILD, tuned_config], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-3000:]
    got = json.loads(res.stdout.strip().splitlines()[-1])
    assert got["elapsed_s"] < 60.0, got
    assert "device error" in got["next_call"] and "timeout" in got["next_call"], got
    assert got["code"] in (1, 2, 3), got
    assert got["calc_diff_after"] <= 1e-5, got


def test_product_library_ignores_the_injection_switch(cuda_device, monkeypatch):
    """The product library reads no environment variable: the test-only switch
    changes nothing there."""
    import numpy as np
    import torch

    import wgrad_oracle as O
    from golden_inputs import C1, case_inputs
    from sm90_fp8_wgrad import (_lib, build_wgrad_scale_block_meta, check_device_errors, fp8_grouped_wgrad_sm90,
                                quantize_grouped_wgrad_operand_128x1)

    assert not _lib.build_flags() & _lib.BUILD_DEBUG_MODES
    counts = C1["counts"]
    cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    meta = build_wgrad_scale_block_meta(torch.from_numpy(cu).to(cuda_device, torch.int32))
    inp = case_inputs(C1)
    lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["lhs_gate"]).to(cuda_device).to(torch.bfloat16), meta)
    rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["rhs_gate"]).to(cuda_device).to(torch.bfloat16), meta)
    out = torch.full((len(counts), lhs.data.shape[1], rhs.data.shape[1]), float("nan"), device=cuda_device,
                     dtype=torch.bfloat16)
    check_device_errors(cuda_device)
    monkeypatch.setenv("SM100_WGRAD_DEBUG_INJECT", "withhold_first_load")
    fp8_grouped_wgrad_sm90(lhs, rhs, out, meta)
    check_device_errors(cuda_device)
    om = O.build_meta(cu)
    ref = O.ref_scaled_wgrad(O.quantize_1x128(inp["lhs_gate"], om), O.quantize_1x128(inp["rhs_gate"], om), om)
    assert O.calc_diff(out.float().cpu().numpy(), ref) <= 1e-5
