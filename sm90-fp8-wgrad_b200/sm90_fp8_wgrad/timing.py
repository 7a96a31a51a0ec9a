"""CUDA-event timing and FLOP accounting (harness API).

Same semantics as the reference (src/sm90_fp8_wgrad/timing.py): per repeat,
``warmup_iters`` untimed calls, then ``active_iters`` calls bracketed by two
CUDA events on the current stream; the per-call time is the elapsed time over
``active_iters``. FLOPs count valid rows only: down 2 R H I, gate/up 2 R (2I) H.
"""
from __future__ import annotations

import statistics
from dataclasses import asdict, dataclass
from typing import Callable

import torch


@dataclass(frozen=True)
class TimingStats:
    mean_ms: float
    median_ms: float
    min_ms: float
    p90_ms: float
    p95_ms: float
    std_ms: float
    repeats: list[float]

    def to_dict(self) -> dict:
        return asdict(self)


def summarize_ms(values: list[float]) -> TimingStats:
    if not values:
        raise RuntimeError("cannot summarize an empty timing list")
    v = sorted(float(x) for x in values)

    def pct(p: float) -> float:
        return v[min(len(v) - 1, max(0, int(round((len(v) - 1) * p))))]

    return TimingStats(
        mean_ms=float(statistics.mean(v)),
        median_ms=float(statistics.median(v)),
        min_ms=v[0],
        p90_ms=pct(0.90),
        p95_ms=pct(0.95),
        std_ms=float(statistics.pstdev(v)) if len(v) > 1 else 0.0,
        repeats=v,
    )


def time_cuda(fn: Callable[[], None], *, warmup_iters: int, active_iters: int, repeat: int) -> TimingStats:
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for timing")
    if int(active_iters) <= 0:
        raise RuntimeError("active_iters must be positive")
    if int(repeat) <= 0:
        raise RuntimeError("repeat must be positive")
    per_call: list[float] = []
    for _ in range(int(repeat)):
        for _ in range(int(warmup_iters)):
            fn()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(int(active_iters)):
            fn()
        t1.record()
        t1.synchronize()
        per_call.append(float(t0.elapsed_time(t1)) / float(active_iters))
    return summarize_ms(per_call)


def valid_wgrad_flops(valid_rows: int, hidden: int, intermediate: int) -> tuple[float, float, float]:
    """(down, gate_up, total) FLOPs over valid rows."""
    down = 2.0 * valid_rows * hidden * intermediate
    gate_up = 2.0 * valid_rows * (2 * intermediate) * hidden
    return down, gate_up, down + gate_up


def tflops(flops: float, ms: float) -> float:
    return 0.0 if float(ms) <= 0.0 else float(flops) / (float(ms) * 1.0e-3) / 1.0e12
