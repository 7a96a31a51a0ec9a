"""Known-answer kernel modes (debug-modes library, -DWGRAD_DEBUG_MODES=1).

The reference's KERNEL_LAB_WGRAD_KERNEL_MODE debug modes (gemm_sm90.py:139-175)
pin pieces of the GEMM separately; here each is asserted, for every tile
configuration, on the C1 shape with fp32 output:
  coord_m / coord_n  every output element holds its m / n coordinate (tile -> output mapping)
  scale_only         out[e] = 2^20 * sum over e's blocks of sa[b, m] sb[b, n] (scale indexing)
  unscaled           out[e] = sum over e's K rows of A[k, m] B[k, n] (the FP8 product alone;
                     the tensor core accumulates FP8 products within a K block with less
                     than fp32 precision -- the reason the reference promotes every
                     128-row block -- so its normwise bound is 1e-3)
Runs in a child process because the library is chosen per process (SM100_WGRAD_LIB).
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
import json, os, sys, torch
import numpy as np
from golden_inputs import C1, case_inputs
from sm90_fp8_wgrad import build_wgrad_scale_block_meta, fp8_grouped_wgrad_sm90, quantize_grouped_wgrad_operand_128x1
dev = torch.device("cuda:0")
counts = C1["counts"]
cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
meta = build_wgrad_scale_block_meta(torch.from_numpy(cu).to(dev, torch.int32))
inp = case_inputs(C1)
bo = meta.block_offsets.cpu().tolist()
pcu = meta.padded_cu_seqlens_k.cpu().tolist()
res = {}
for lk, rk in (("lhs_down", "rhs_down"), ("lhs_gate", "rhs_gate")):
    lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp[lk]).to(dev).to(torch.bfloat16), meta)
    rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp[rk]).to(dev).to(torch.bfloat16), meta)
    e, m, n = len(counts), lhs.data.shape[1], rhs.data.shape[1]
    a = lhs.data.float().double().cpu()          # [K_p, M]
    b = rhs.data.float().double().cpu()          # [K_p, N]
    sa = lhs.scales.double().cpu()
    sb = rhs.scales.double().cpu()
    expect = {
        "coord_m": torch.arange(m, dtype=torch.float64)[None, :, None].expand(e, m, n),
        "coord_n": torch.arange(n, dtype=torch.float64)[None, None, :].expand(e, m, n),
        "scale_only": torch.stack([2.0 ** 20 * sum((sa[blk][:, None] * sb[blk][None, :] for blk in range(bo[x], bo[x + 1])),
                                                  torch.zeros(m, n, dtype=torch.float64)) for x in range(e)]),
        "unscaled": torch.stack([a[pcu[x]:pcu[x + 1]].T @ b[pcu[x]:pcu[x + 1]] for x in range(e)]),
    }
    for mode, ref in expect.items():
        os.environ["KERNEL_LAB_WGRAD_KERNEL_MODE"] = mode
        out = torch.full((e, m, n), float("nan"), device=dev, dtype=torch.float32)
        fp8_grouped_wgrad_sm90(lhs, rhs, out, meta, tuned_config=sys.argv[1])
        torch.cuda.synchronize()
        got = out.double().cpu()
        # normwise: the largest error over the largest reference value (sums of
        # FP8 products cancel, so elementwise relative errors are meaningless)
        err = float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
        res[f"{lk}:{mode}"] = {"max_rel_err": err, "finite": bool(torch.isfinite(got).all())}
    os.environ["KERNEL_LAB_WGRAD_KERNEL_MODE"] = "normal"
print(json.dumps(res))
"""


@pytest.mark.parametrize("tuned_config", ["default", "sm100_128x256_w8", "sm100_128x256_w16", "sm100_128x128",
                                          "sm100_128x128_2cta"])
def test_known_answer_modes(cuda_device, tuned_config):
    if not DEBUG_LIB.is_file():   # instrumented build (build() makes it; nvcc is on the GPU box too)
        sys.path.insert(0, str(ROOT / "sm90-fp8-wgrad_b200"))
        import build_ext

        build_ext.build(debug_modes=True)
    env = dict(os.environ, SM100_WGRAD_LIB=str(DEBUG_LIB))
    env.pop("KERNEL_LAB_WGRAD_KERNEL_MODE", None)
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT / "sm90-fp8-wgrad_b200"), str(ROOT / "tests" / "golden"),
                                         env.get("PYTHONPATH", "")])
    res = subprocess.run([sys.executable, "-c", CHILD, tuned_config], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    got = json.loads(res.stdout.strip().splitlines()[-1])
    for key, r in got.items():
        assert r["finite"], key
        tol = {"coord_m": 0.0, "coord_n": 0.0, "scale_only": 1e-5, "unscaled": 1e-3}[key.split(":")[1]]
        assert r["max_rel_err"] <= tol, (key, r)


def test_product_library_refuses_known_answer_modes(cuda_device, monkeypatch):
    """The product build has no debug branches: a known-answer mode is refused."""
    import torch

    from golden_inputs import C1, case_inputs
    from sm90_fp8_wgrad import build_wgrad_scale_block_meta, fp8_grouped_wgrad_sm90, quantize_grouped_wgrad_operand_128x1
    import numpy as np

    counts = C1["counts"]
    cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    meta = build_wgrad_scale_block_meta(torch.from_numpy(cu).to(cuda_device, torch.int32))
    inp = case_inputs(C1)
    lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["lhs_gate"]).to(cuda_device).to(torch.bfloat16), meta)
    rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["rhs_gate"]).to(cuda_device).to(torch.bfloat16), meta)
    out = torch.empty((len(counts), lhs.data.shape[1], rhs.data.shape[1]), device=cuda_device, dtype=torch.float32)
    monkeypatch.setenv("KERNEL_LAB_WGRAD_KERNEL_MODE", "coord_m")
    with pytest.raises(RuntimeError, match="debug-modes library"):
        fp8_grouped_wgrad_sm90(lhs, rhs, out, meta)
