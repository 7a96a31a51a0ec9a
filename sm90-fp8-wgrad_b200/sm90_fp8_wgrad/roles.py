"""Per-role cycle counters of the grouped GEMM on a synthetic workload.

Needs the profile library (``python sm90-fp8-wgrad_b200/build_ext.py --profile``),
selected with ``SM100_WGRAD_LIB``::

    SM100_WGRAD_LIB=sm90-fp8-wgrad_b200/sm90_fp8_wgrad/_lib/libsm100_fp8_wgrad_profile.so \\
        python -m sm90_fp8_wgrad.roles --workload dsv3_32k

For each GEMM (down, gate_up) one warm launch, then one counted launch: the
counters of every CTA (producer, MMA warp, first promotion warp) summed and
divided by the K blocks promoted, in SM cycles per K block.
"""
from __future__ import annotations

import argparse
import json

# (experts, top_k, hidden, intermediate, tokens, route) of the benchmark workloads
WORKLOADS = {
    "dsv3_32k": (256, 8, 7168, 2048, 32768, "uniform"),
    "dsv3_4k": (256, 8, 7168, 2048, 4096, "uniform"),
    "qwen3_32k": (128, 8, 2048, 768, 32768, "uniform"),
}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sm90_fp8_wgrad.roles", description=__doc__.split("\n\n")[0])
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="dsv3_32k")
    ap.add_argument("--tuned-config", default="default")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--scale-format", choices=("fp32", "ue8m0"), default="fp32")
    a = ap.parse_args(argv)

    import torch

    from . import _lib
    from .routing import make_routing
    from .synthetic import make_synthetic_wgrad_inputs, run_custom_down, run_custom_gate_up

    if _lib.profile_counters() is None:
        raise RuntimeError("the loaded library has no counters: build it with build_ext.py --profile and "
                           "point SM100_WGRAD_LIB at libsm100_fp8_wgrad_profile.so")
    e, k, h, i, t, route = WORKLOADS[a.workload]
    routing = make_routing(tokens=t, experts=e, top_k=k, route=route, seed=a.seed)
    inp = make_synthetic_wgrad_inputs(tokens=t, experts=e, top_k=k, hidden=h, intermediate=i, route=route,
                                      seed=a.seed, device=torch.device("cuda", torch.cuda.current_device()),
                                      routing=routing, scale_format=a.scale_format)
    inp.drop_sources()
    for name, fn in (("down", run_custom_down), ("gate_up", run_custom_gate_up)):
        fn(inp, tuned_config=a.tuned_config)
        torch.cuda.synchronize()
        _lib.profile_counters()                     # clear
        fn(inp, tuned_config=a.tuned_config)
        torch.cuda.synchronize()
        c = _lib.profile_counters()
        blocks = max(c["k_blocks"], 1)
        per_block = {key: round(v / blocks) for key, v in c.items()
                     if key not in ("k_blocks", "tiles", "ctas") and (v or not key.startswith(("sf_", "mma_tile")))}
        # load_latency is summed by the MMA warp over every K block it waited for
        per_block["load_latency"] = round(c.get("load_latency", 0) / max(c["k_blocks"], 1))
        # the CTA's whole run (set-up excluded) per K block: the period every role shares
        per_block["period"] = round(c.get("cta_cycles", 0) / blocks)
        print(json.dumps({"workload": a.workload, "gemm": name, "ctas": c["ctas"],
                          "k_blocks_per_cta": round(c["k_blocks"] / max(c["ctas"], 1)),
                          "tiles_per_cta": round(c["tiles"] / max(c["ctas"], 1)),
                          "cycles_per_k_block": per_block}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
