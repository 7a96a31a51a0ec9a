"""Per-role cycle counters of the GEMM (library built with -DWGRAD_PROFILE=1).

Runs one launch through the profile library in a child process (the library
is chosen per process by SM100_WGRAD_LIB) and checks the counts exactly: the
first promotion warp of each CTA counts the K blocks of every tile it
promotes (sum = tiles per expert x total K blocks), the tiles stored and the
CTAs; the cycle counters are positive.
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
PROFILE_LIB = ROOT / "sm90-fp8-wgrad_b200" / "sm90_fp8_wgrad" / "_lib" / "libsm100_fp8_wgrad_profile.so"

CHILD = r"""
import json, sys, torch
import numpy as np
from golden_inputs import C1, case_inputs
from sm90_fp8_wgrad import (_lib, build_wgrad_scale_block_meta, fp8_grouped_wgrad_sm90,
                            quantize_grouped_wgrad_operand_128x1)
dev = torch.device("cuda:0")
counts = C1["counts"]
cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
meta = build_wgrad_scale_block_meta(torch.from_numpy(cu).to(dev, torch.int32))
inp = case_inputs(C1)
lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["lhs_gate"]).to(dev).to(torch.bfloat16), meta)
rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp["rhs_gate"]).to(dev).to(torch.bfloat16), meta)
out = torch.empty((len(counts), lhs.data.shape[1], rhs.data.shape[1]), device=dev, dtype=torch.bfloat16)
_lib.profile_counters()
fp8_grouped_wgrad_sm90(lhs, rhs, out, meta, tuned_config=sys.argv[1])
torch.cuda.synchronize()
print(json.dumps({"counters": _lib.profile_counters(), "m": int(lhs.data.shape[1]), "n": int(rhs.data.shape[1]),
                  "experts": len(counts), "total_blocks": int(meta.total_blocks)}))
"""


@pytest.mark.parametrize("tuned_config,bn", [("sm100_128x256_w8", 256), ("sm100_128x256_w16", 256),
                                             ("sm100_128x128", 128)])
def test_profile_counters_count_every_block(cuda_device, tuned_config, bn):
    if not PROFILE_LIB.is_file():   # instrumented build (build() makes it; nvcc is on the GPU box too)
        sys.path.insert(0, str(ROOT / "sm90-fp8-wgrad_b200"))
        import build_ext

        build_ext.build(profile=True)
    env = dict(os.environ, SM100_WGRAD_LIB=str(PROFILE_LIB))
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT / "sm90-fp8-wgrad_b200"), str(ROOT / "tests" / "golden"),
                                         env.get("PYTHONPATH", "")])
    res = subprocess.run([sys.executable, "-c", CHILD, tuned_config], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    d = json.loads(res.stdout.strip().splitlines()[-1])
    c = d["counters"]
    assert c is not None
    tiles_per_expert = -(-d["m"] // 128) * -(-d["n"] // bn)
    assert c["tiles"] == tiles_per_expert * d["experts"]
    assert c["k_blocks"] == tiles_per_expert * d["total_blocks"]
    assert c["ctas"] >= 1
    for k in ("mma_issue", "epi_promote", "epi_store", "epi_wait", "mma_wait"):
        assert c[k] > 0, (k, c)
