"""Per-K-block event timeline of the grouped GEMM (trace builds only).

Build the trace library and load it with ``SM100_WGRAD_LIB``::

    python sm90-fp8-wgrad_b200/build_ext.py --trace 1      # or --trace 2
    cd sm90-fp8-wgrad_b200
    SM100_WGRAD_LIB=sm90_fp8_wgrad/_lib/libsm100_fp8_wgrad_trace1.so \\
        python -m sm90_fp8_wgrad.timeline --workload dsv3_32k --tuned-config sm100_256x256_pair

One warm gate_up launch, then one traced launch; prints, for CTA 0 (and its
pair peer, CTA 1), the SM clock64 stamps of the first 40 K blocks relative to
the earliest stamp. Trace 1: MMA issuer ready / issued, promotion warp wait
start / partial ready / buffer released / block done (scale-product kernel:
ready/issued of its second half in the last two columns; promotion kernels:
tile start and tile decoded, on the first block of each tile). Trace 2: promotion
warp ready, chunks 0-3 in registers, released, done, next wait start.
"""
from __future__ import annotations

import argparse
import ctypes

from .roles import WORKLOADS

NAMES = {1: ["mma_ready", "mma_issued", "epi_wait_start", "epi_ready", "epi_released", "epi_done",
             "mma_h1_ready", "mma_h1_issued"],
         2: ["epi_ready", "c0", "c1", "c2", "c3", "released", "done", "wait_start"]}


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sm90_fp8_wgrad.timeline", description=__doc__.split("\n\n")[0])
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="dsv3_32k")
    ap.add_argument("--tuned-config", default="default")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--blocks", type=int, default=40)
    a = ap.parse_args(argv)

    import torch

    from . import _lib
    from .routing import make_routing
    from .synthetic import make_synthetic_wgrad_inputs, run_custom_gate_up

    lib = _lib.load()
    if not hasattr(lib, "sm100_wgrad_trace_read"):
        raise RuntimeError("the loaded library is not a trace build: build_ext.py --trace 1 and SM100_WGRAD_LIB")
    kind = 2 if str(_lib.library_path()).endswith("trace2.so") else 1
    lib.sm100_wgrad_trace_read.argtypes = [ctypes.POINTER(ctypes.c_uint64), ctypes.c_int32]
    e, k, h, i, t, route = WORKLOADS[a.workload]
    inp = make_synthetic_wgrad_inputs(tokens=t, experts=e, top_k=k, hidden=h, intermediate=i, route=route,
                                      seed=a.seed, device=torch.device("cuda", torch.cuda.current_device()),
                                      routing=make_routing(tokens=t, experts=e, top_k=k, route=route, seed=a.seed))
    inp.drop_sources()
    buf = (ctypes.c_uint64 * (2 * 64 * 8))()
    for _ in range(2):                       # warm launch, then the traced one (each read clears)
        run_custom_gate_up(inp, tuned_config=a.tuned_config)
        torch.cuda.synchronize()
        _lib.check(lib.sm100_wgrad_trace_read(buf, 2 * 64 * 8), "sm100_wgrad_trace_read")
    for cta in (0, 1):
        rows = [[int(buf[(cta * 64 + b) * 8 + ev]) for ev in range(8)] for b in range(64)]
        stamps = [v for r in rows for v in r if v]
        if not stamps:
            continue
        base = min(stamps)
        print(f"CTA {cta} ({a.workload}, {a.tuned_config}): SM cycles from the first stamp")
        print("blk " + " ".join(f"{n:>14s}" for n in NAMES[kind]))
        for b in range(min(a.blocks, 64)):
            print(f"{b:3d} " + " ".join(f"{(v - base) if v else -1:14d}" for v in rows[b]))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
