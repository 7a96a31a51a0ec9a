#!/usr/bin/env python3
"""Grouped FP8 Wgrad benchmark (one JSON line on rank 0).

A step is the hot path over one batch: the two grouped Wgrad GEMMs of an MoE
MLP backward (dW_down and dW_gate_up) through the public operator
``fp8_grouped_wgrad_sm90``. Default workload: DeepSeek-V3 shape (E=256, top-8,
H=7168, I=2048), T=32768 tokens, uniform top-8 routing, experts sharded
contiguously over the ranks (expert parallelism, no collective in the timed
region). Inputs (5.4 GB of FP8 operands, 22.5 GB of BF16 outputs at 1 GPU) are
larger than the 126 MB L2, so no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...

``--impl reference`` times the reference's CPU path (the dequantise-then-matmul
algorithm of checks.py:42-61, restated in oracle/) on the host cores, on a
bounded sample of the same workload; only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "sm90-fp8-wgrad_b200"))

import torch  # noqa: E402

WORKLOADS = {
    # name: (experts, top_k, hidden, intermediate, tokens, route)
    "dsv3_32k": (256, 8, 7168, 2048, 32768, "uniform"),
    "dsv3_16k": (256, 8, 7168, 2048, 16384, "uniform"),
    "dsv3_8k": (256, 8, 7168, 2048, 8192, "uniform"),
    "dsv3_4k": (256, 8, 7168, 2048, 4096, "uniform"),
    "dsv3_skewed_32k": (256, 8, 7168, 2048, 32768, "zipf"),
    "qwen3_32k": (128, 8, 2048, 768, 32768, "uniform"),
    "large_expert_16k": (32, 2, 6144, 9216, 16384, "zipf"),
    "many_small_32k": (512, 10, 4096, 1024, 32768, "zipf"),
    "tiny": (8, 2, 256, 128, 1024, "uniform"),
}
# H100 numbers of the reference kernel for the same per-GPU problem
# (README.md:141, :189 of the reference; TFLOP/s).
H100_REFERENCE_TFLOPS = {"dsv3_32k": 446.1, "qwen3_32k": 455.1, "dsv3_16k": 395.0, "dsv3_8k": 314.0,
                         "dsv3_4k": 223.0}
NOMINAL_FP8_TFLOPS = 4500.0


def log(msg: str) -> None:
    print(f"[bench] {msg}", file=sys.stderr, flush=True)


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "_fallback": True}


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region.

    In-process NVML (read-only queries) every ~10 ms from a background thread,
    started right before the first timed launch and stopped after the final
    synchronize, so every sample lies inside the timed region; the device is
    matched to the CUDA device by PCI bus id. Falls back to ``nvidia-smi -lms
    100`` when NVML is unavailable."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: torch.device, gpu_index: int):
        self.dev = dev
        self.gpu_index = gpu_index
        self.proc = None
        self.thread = None
        self.lines: list[str] = []
        self.rows: list[tuple[float, float, list[str]]] = []
        self.stop_flag = threading.Event()
        self.nvml = None
        self.handle = None

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.dev)
        bus = getattr(props, "pci_bus_id", None)
        if bus is not None:
            bus_id = f"{getattr(props, 'pci_domain_id', 0):08X}:{bus:02X}:{getattr(props, 'pci_device_id', 0):02X}.0"
            try:
                return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus_id)
            except pynvml.NVMLError:
                pass
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu_index)

    def _nvml_loop(self) -> None:
        nv, h = self.nvml, self.handle
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self.stop_flag.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.rows.append((mhz, max_mhz, ["active" if reasons & b else "not active" for b in bits]))
            except Exception:
                break
            time.sleep(0.01)

    def start(self) -> None:
        try:
            self.nvml, self.handle = self._nvml_handle()
            self.thread = threading.Thread(target=self._nvml_loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read_smi, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read_smi(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        source = "nvml"
        if self.nvml is not None:
            self.stop_flag.set()
            if self.thread is not None:
                self.thread.join(timeout=2)
        elif self.proc is not None:
            source = "nvidia-smi"
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            for ln in self.lines:
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    self.rows.append((float(parts[1]), float(parts[2]), [p.lower() for p in parts[5:9]]))
                except ValueError:
                    continue
        else:
            return None
        rows = self.rows
        if not rows:
            return None
        mhz = sorted(r[0] for r in rows)
        reasons = sorted({self.NAMES[i] for r in rows for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": mhz[len(mhz) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows), "sm_mhz_min": mhz[0], "source": source}


def _all_finite(t: torch.Tensor, experts_per_chunk: int = 16) -> bool:
    """isfinite over [E, M, N] in expert chunks (bounded temporary memory)."""
    return all(bool(torch.isfinite(t[e:e + experts_per_chunk]).all()) for e in range(0, t.shape[0], experts_per_chunk))


def validate_outputs(inp, layout: str, world: int, dev) -> dict:
    """After the timed region, as the reference's benchmark does
    (benchmark_wgrad.py:209-214, :360-414): every expert of both GEMMs checked,
    streamed by expert, against an fp32 dequantise-then-matmul of the same FP8
    operands; DeepSeek calc_diff accumulated over the whole output of each GEMM
    (against the reference rounded to BF16, the reference's metric, and against
    the fp32 reference) within the 1e-5 gate; every output finite and every
    empty expert exactly zero. Max over ranks; experts checked summed."""
    from sm90_fp8_wgrad.matrix import check_all_experts

    r = check_all_experts(inp, layout)
    ok_local = r["finite"] and r["empty_experts_zero"]

    def mx(v: float) -> float:
        return _max_over_ranks(v if math.isfinite(v) else 1e30, world, dev)

    out = {"calc_diff_max": mx(r["calc_diff_max"]), "calc_diff_vs_fp32_max": mx(r["calc_diff_vs_fp32_max"]),
           "worst_expert_calc_diff": mx(r["worst_expert_calc_diff"]), "calc_diff_gate": 1e-5,
           "max_rel_err_normwise": mx(r["max_rel_err_normwise"]),
           "experts_checked": int(_sum_over_ranks(float(r["experts_checked"]), world, dev)),
           "experts_total": int(_sum_over_ranks(float(sum(1 for c in inp.counts if c > 0)), world, dev)),
           "scope": "every expert, streamed (reference benchmark_wgrad.py:360-414)"}
    bad = _max_over_ranks(0.0 if ok_local else 1.0, world, dev)
    out["finite_and_empty_zero"] = bad == 0.0
    out["passed"] = bool(bad == 0.0 and out["calc_diff_max"] <= 1e-5 and out["calc_diff_vs_fp32_max"] <= 1e-5)
    return out


def flops_of(inp) -> tuple[float, float]:
    r = inp.valid_rows
    down = 2.0 * r * inp.hidden * inp.intermediate
    return down, 2.0 * down


def hbm_bytes_of(inp) -> float:
    """Algorithmic HBM bytes of one step: FP8 operands, fp32 scales, BF16 outputs."""
    h, i, e = inp.hidden, inp.intermediate, inp.experts
    # operand rows the GEMM streams: 128-row slots (padded) or 32-row-aligned segments (packed)
    pad = inp.meta.wgmma_rows if inp.grad_y_q.kernel_data is not None else inp.meta.padded_rows
    blocks = inp.meta.total_blocks
    return float(pad * (2 * h + 3 * i) + blocks * (2 * h + 3 * i) * 4 + e * 3 * h * i * 2)


# ---------------------------------------------------------------- CPU leg
def _host_threads() -> int:
    """Every host core this process may run on (affinity-aware)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_reference_sample(workload: str, seed: int, target_s: float, max_experts: int | None = None,
                         expert_range: tuple[int, int] | None = None) -> dict:
    """Time the reference's CPU algorithm (dequantise + fp32 matmul per 128-row
    block, checks.py:42-61; restated in oracle/) on a bounded sample of the
    workload: experts of ``expert_range`` (the whole problem by default; a
    rank's contiguous shard at N > 1), biggest first, down + gate_up, until
    ~target_s seconds of CPU work. Returns the rate over the sample and what
    the sample was (experts, FLOP, seconds)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import wgrad_oracle as O
    from sm90_fp8_wgrad.routing import make_routing

    e_all, top_k, h, i, t, route = WORKLOADS[workload]
    routing = make_routing(tokens=t, experts=e_all, top_k=top_k, route=route, seed=seed)
    e0, e1 = expert_range if expert_range is not None else (0, e_all)
    gen = torch.Generator().manual_seed(seed + 99)
    flops = 0.0
    elapsed = 0.0
    done = 0
    order = sorted(range(e0, e1), key=lambda e: -routing.counts[e])  # biggest first: fewer, longer samples
    for e in order:
        c = routing.counts[e]
        if c == 0:
            continue
        lhs_d = torch.randn((c, h), generator=gen).mul_(0.01).to(torch.bfloat16)
        rhs_d = torch.randn((c, i), generator=gen).to(torch.bfloat16)
        lhs_g = torch.randn((c, 2 * i), generator=gen).mul_(0.01).to(torch.bfloat16)
        rhs_g = torch.randn((c, h), generator=gen).to(torch.bfloat16)
        q = [O.quantize_1x128_torch(x, [c]) for x in (lhs_d, rhs_d, lhs_g, rhs_g)]
        bo, rc = q[0][2], q[0][3]
        t0 = time.perf_counter()
        O.ref_scaled_wgrad_torch(q[0][0], q[0][1], q[1][0], q[1][1], bo, rc, [0])
        O.ref_scaled_wgrad_torch(q[2][0], q[2][1], q[3][0], q[3][1], bo, rc, [0])
        elapsed += time.perf_counter() - t0
        flops += 6.0 * c * h * i
        done += 1
        if elapsed >= target_s or (max_experts is not None and done >= max_experts):
            break
    return {
        "value": flops / elapsed / 1e12 if elapsed > 0 else 0.0,
        "unit": "TFLOP/s",
        "cores": int(torch.get_num_threads()),
        "kind": "port",
        "sample": f"{done} of experts [{e0},{e1}) of {workload} (down+gate_up, {flops / 1e9:.0f} GFLOP, "
                  f"{elapsed:.1f} s, torch fp32 on CPU)",
        "seconds": elapsed,
        "flops": flops,
        "experts": done,
    }


def run_reference(args) -> None:
    """The reference's CPU path on the host cores (rank 0 only). A step is a
    bounded sample of the workload this GPU count gives one GPU (the whole
    problem at N=1, the first rank's contiguous expert shard at N>1): the
    biggest experts of that problem until ~cpu_seconds/steps of CPU work.
    ``steps`` and ``ms_per_step`` describe exactly the timed samples; the
    time the whole per-GPU problem would take at the measured rate is under
    ``extrapolated``, a separate key."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from sm90_fp8_wgrad.routing import make_routing, shard_experts

    torch.set_num_threads(_host_threads())
    e_all, top_k, h, i, t, route = WORKLOADS[args.workload]
    shard = shard_experts(e_all, world, 0)
    routing = make_routing(tokens=t, experts=e_all, top_k=top_k, route=route, seed=args.seed)
    shard_flops = 6.0 * h * i * sum(routing.counts[shard[0]:shard[1]])
    secs, flops, sample = [], [], None
    for s in range(args.warmup + args.steps):
        res = cpu_reference_sample(args.workload, args.seed, target_s=args.cpu_seconds / max(1, args.steps),
                                   expert_range=shard)
        if s >= args.warmup:
            secs.append(res["seconds"])
            flops.append(res["flops"])
            sample = res
    value = sum(flops) / sum(secs) / 1e12
    line = {
        "impl": "reference",
        "metric": "grouped Wgrad FP8 TFLOP/s (down + gate_up per step)",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": sum(secs) / len(secs) * 1e3,
        "step": f"a bounded sample of the per-GPU problem: {sample['experts']} experts of shard "
                f"[{shard[0]},{shard[1]}), {sample['flops'] / 1e9:.0f} GFLOP per step",
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8e4m3->f32",
        "data": "synthetic",
        "config": workload_config(args.workload, world),
        "cpu_baseline": {k: sample[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "extrapolated": {"full_per_gpu_step_ms": shard_flops / (value * 1e12) * 1e3 if value > 0 else None,
                         "full_per_gpu_step_gflop": shard_flops / 1e9,
                         "how": "whole per-GPU problem's FLOP at the measured sample rate (not measured)"},
        "gpu_launches": 0,
    }
    line["cpu_baseline"]["value"] = value
    print(json.dumps(line), flush=True)


def workload_config(workload: str, world: int, layout: str = "padded", scale_format: str = "fp32") -> dict:
    e_all, top_k, h, i, t, route = WORKLOADS[workload]
    return {"workload": workload, "experts": e_all, "top_k": top_k, "hidden": h, "intermediate": i,
            "tokens": t, "route": route, "parallelism": f"ep{world}", "layout": layout,
            "scale_format": scale_format,
            "l2": "inputs larger than L2 (no flush needed)" if workload not in ("tiny",) else "flush"}


# ---------------------------------------------------------------- GPU arm
def _max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _barrier(world: int, dev) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[dev.index])
    torch.cuda.synchronize(dev)


def _profile_traffic(workload: str):
    """DRAM bytes per launch of the grouped Wgrad kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "grouped_wgrad_traffic.json"
    if not p.is_file():
        return None
    try:
        return json.loads(p.read_text()).get(workload)
    except Exception:
        return None


def _tensor_rate_tflops(dev, sm_mhz: float) -> float:
    """Dense FP8 tensor rate of the whole GPU at an SM clock: 8,192 MACs per SM cycle."""
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    return sms * 8192 * 2 * sm_mhz * 1e6 / 1e12


def library_fp8_rate(dev, gpu_index: int, seconds: float = 3.0) -> dict:
    """cuBLAS FP8 GEMM on the same GPU, for context beside the grouped Wgrad rate.

    ``torch._scaled_mm`` on 8192^3 e4m3 operands with one scale per tensor (no
    per-block promotion; cuBLAS offers 1x128 block scaling only on sm_90):
    best of 10 launches (burst) and back-to-back launches for ``seconds``
    (sustained, under the board power limit), with the SM clock seen meanwhile.
    """
    n = 8192
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)
    flops = 2.0 * n ** 3

    def gemm():
        return torch._scaled_mm(a, b, one, one, out_dtype=torch.bfloat16)

    for _ in range(3):
        gemm()
    torch.cuda.synchronize(dev)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gemm()
        e1.record()
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1))
    clocks = ClockSampler(dev, gpu_index)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    t0 = time.perf_counter()
    e0.record()
    while time.perf_counter() - t0 < seconds:
        for _ in range(20):
            gemm()
        launches += 20
        torch.cuda.synchronize(dev)
    e1.record()
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    return {"what": "cuBLAS FP8 e4m3 GEMM 8192^3, per-tensor scales (torch._scaled_mm), bf16 out",
            "burst_tflops": flops / (best * 1e-3) / 1e12,
            "sustained_tflops": flops * launches / (e0.elapsed_time(e1) * 1e-3) / 1e12,
            "sustained_seconds": seconds, "sustained_clocks": clk}


def run_ours(args) -> None:
    rank, world, local_rank = dist_env()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
    from sm90_fp8_wgrad import _lib
    from sm90_fp8_wgrad.routing import make_routing, shard_experts
    from sm90_fp8_wgrad.synthetic import make_synthetic_wgrad_inputs, run_custom_down, run_custom_gate_up

    e_all, top_k, h, i, t, route = WORKLOADS[args.workload]
    routing = make_routing(tokens=t, experts=e_all, top_k=top_k, route=route, seed=args.seed)
    e0, e1 = shard_experts(e_all, world, rank)
    t_setup = time.perf_counter()
    inp = make_synthetic_wgrad_inputs(tokens=t, experts=e_all, top_k=top_k, hidden=h, intermediate=i, route=route,
                                      seed=args.seed, device=dev, expert_range=(e0, e1), routing=routing,
                                      layout_mode=args.layout, scale_format=args.scale_format)
    inp.drop_sources()
    torch.cuda.empty_cache()
    torch.cuda.synchronize(dev)
    log(f"rank {rank}: experts [{e0},{e1}) rows {inp.valid_rows} padded {inp.meta.padded_rows} "
        f"setup {time.perf_counter() - t_setup:.1f}s")

    def step():
        run_custom_down(inp, tuned_config=args.tuned_config)
        run_custom_gate_up(inp, tuned_config=args.tuned_config)

    for _ in range(args.warmup):
        step()
    _barrier(world, dev)
    if _lib.device_error() != 0:
        raise RuntimeError("device error word set after warm-up")

    stream = torch.cuda.current_stream(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(dev, dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else
                          int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    _barrier(world, dev)
    clocks.start()
    for s in range(args.steps):
        evs[s][0].record(stream)
        run_custom_down(inp, tuned_config=args.tuned_config)
        evs[s][1].record(stream)
        run_custom_gate_up(inp, tuned_config=args.tuned_config)
        evs[s][2].record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    _barrier(world, dev)
    total_ms = evs[0][0].elapsed_time(evs[-1][2])
    step_ms = sorted(e[0].elapsed_time(e[2]) for e in evs)   # per-step spread (timing.py: mean/min/p90)
    down_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    gate_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    local_ms = total_ms / args.steps
    ms = _max_over_ranks(local_ms, world, dev)
    f_down, f_gate = flops_of(inp)
    total_flops = _sum_over_ranks(f_down + f_gate, world, dev)
    value = total_flops / (ms * 1e-3) / 1e12
    err = _lib.device_error()
    if err != 0:
        raise RuntimeError(f"device error word {err} after the timed region")
    check = validate_outputs(inp, args.layout, world, dev)

    peaks = measured_peaks()
    fp8_peak = 2.0 * float(peaks["bf16_tflops"])
    step_bytes = hbm_bytes_of(inp)
    t_tc = (f_down + f_gate) / (fp8_peak * 1e12)
    t_hbm = step_bytes / (float(peaks["hbm_gbs"]) * 1e9)
    bound = "tensor" if t_tc >= t_hbm else "hbm"
    gate_flops_tf = f_gate / (gate_ms * 1e-3) / 1e12
    down_flops_tf = f_down / (down_ms * 1e-3) / 1e12
    kname = ("grouped_wgrad_ue8m0_kernel (gate_up launch)" if args.scale_format == "ue8m0"
             else "grouped_wgrad_kernel, AUTO tile (gate_up launch)")
    if bound == "tensor":
        roof = {"bound": "tensor", "kernel": kname,
                "achieved": gate_flops_tf, "peak": fp8_peak, "unit": "TFLOP/s", "frac": gate_flops_tf / fp8_peak,
                "peak_source": "2 x measured bf16 cuBLAS burst (MEASURED_PEAKS.json)"
                               + (" fallback" if peaks.get("_fallback") else ""),
                "pct_of_nominal_fp8_4500": gate_flops_tf / NOMINAL_FP8_TFLOPS}
    else:
        gate_bytes = step_bytes * 2.0 / 3.0
        gbs = gate_bytes / (gate_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": kname, "achieved": gbs,
                "peak": float(peaks["hbm_gbs"]), "unit": "GB/s", "frac": gbs / float(peaks["hbm_gbs"]),
                "peak_source": "measured copy bandwidth (MEASURED_PEAKS.json)"}
    # DRAM bytes per gate_up launch from a committed ncu capture of the same
    # workload (not a counter of this run); the capture is of the 1-GPU launch,
    # so at N > 1 it is scaled by this rank's share of experts.
    traffic = _profile_traffic(args.workload) if args.scale_format == "fp32" else None
    roof["traffic"] = None if traffic is None else float(traffic) * (e1 - e0) / e_all
    roof["traffic_unit"] = "DRAM bytes per gate_up launch"
    roof["traffic_source"] = ("committed ncu capture (dram__bytes_read.sum + dram__bytes_write.sum), not measured "
                              "in this run" + ("; scaled by this rank's share of experts" if world > 1 else ""))
    roof["step_roofline_ms"] = max(t_tc, t_hbm) * 1e3
    roof["step_roofline_frac"] = max(t_tc, t_hbm) * 1e3 / local_ms

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(inp, args, world, dev, f_down + f_gate)
    lib_rate = None
    if rank == 0 and world == 1 and not args.no_library_rate:
        lib_rate = library_fp8_rate(dev, clocks.gpu_index)
        lib_rate["pct_burst"] = value / lib_rate["burst_tflops"]
        lib_rate["pct_sustained"] = value / lib_rate["sustained_tflops"]
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(_host_threads())   # after the GPU timing: all host cores for the CPU leg
        cpu = cpu_reference_sample(args.workload, args.seed, target_s=args.cpu_seconds)
        for key in ("seconds", "flops", "experts"):
            cpu.pop(key, None)

    if rank == 0:
        line = {
            "metric": "grouped Wgrad FP8 TFLOP/s (down + gate_up per step)",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": (value / H100_REFERENCE_TFLOPS[args.workload]) if (
                world == 1 and args.workload in H100_REFERENCE_TFLOPS) else None,
            "vs_baseline_ref": "published reference sm90 kernel figure on H100, same per-GPU problem",
            "dtype": "fp8e4m3->f32acc->bf16",
            "data": "synthetic",
            "config": dict(workload_config(args.workload, world, args.layout, args.scale_format), tuned_config=args.tuned_config),
            "stages_ms": {"down": down_ms, "gate_up": gate_ms},
            "stages_tflops": {"down": down_flops_tf, "gate_up": gate_flops_tf},
            "pct_of_fp8_peak": value / world / fp8_peak,
            "pct_of_nominal_fp8": value / world / NOMINAL_FP8_TFLOPS,
            # The tensor pipe's own rate: 8,192 FP8 MACs per SM cycle (512 cycles per
            # 128 x 256 x 128 UMMA block, measured by a UMMA microbenchmark) on every
            # SM, at the boost clock and at the SM clock seen during the timed region.
            "pct_of_tensor_rate_boost": value / world / _tensor_rate_tflops(dev, float(peaks.get("sm_max_mhz", 1965))),
            "pct_of_tensor_rate_at_clock": (value / world / _tensor_rate_tflops(dev, clk["sm_mhz"])
                                            if clk and clk.get("sm_mhz") else None),
            "tflops_per_gpu_per_ghz": (value / world / (clk["sm_mhz"] / 1000.0) if clk and clk.get("sm_mhz") else None),
            "hbm_gbs_step": step_bytes / (local_ms * 1e-3) / 1e9,
            # This run's grouped Wgrad rate as a fraction of a plain cuBLAS FP8 GEMM's
            # (no promotion) on the same GPU, burst and sustained at the power limit.
            "library_fp8": lib_rate,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "ms_per_step_min": step_ms[0],
            "ms_per_step_p90": step_ms[min(len(step_ms) - 1, int(round(0.9 * (len(step_ms) - 1))))],
            "clocks": clk,
            "check": check,
            "gpu_launches": 2 * args.steps,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_e2e(inp, args, world, dev, step_flops) -> dict:
    """Same metric through the public API with host buffers: every step copies
    its inputs (FP8 operands, scales, metadata) from pinned host memory to the
    device, runs both GEMMs and copies both gradients back to pinned host memory.

    The step is pipelined over three streams, as a caller of the operator would
    run it: the inputs go host-to-device on one copy stream (the down GEMM's
    first, so it can start early); the GEMMs run on the compute stream in
    expert chunks (``expert_range`` launches, bit-identical to one launch); and
    each finished chunk of gradients goes device-to-host on a second copy stream
    while the next chunks compute. Consecutive steps only wait where they reuse
    a buffer (next inputs after this step's GEMMs, a chunk's output after its
    previous copy-out)."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90

    def storage_of(op):
        if op.kernel_data is not None:        # packed layout: the launch copy is what the GEMM reads
            return op.kernel_data
        pitch = op.data.stride(1)
        return op.data.as_strided((op.data.shape[1], pitch), (pitch, 1))

    m = inp.meta
    meta_in = [m.padded_cu_seqlens_k, m.wgmma_cu_seqlens_k, m.block_offsets, m.expert_order]
    down_in = [storage_of(inp.grad_y_q), inp.grad_y_q.scales, storage_of(inp.hidden_q), inp.hidden_q.scales]
    gate_in = [storage_of(inp.grad_gate_up_q), inp.grad_gate_up_q.scales, storage_of(inp.x_q), inp.x_q.scales]
    outs = [inp.down_out_bf16, inp.gate_up_out_bf16]

    def pinned_like(t):
        try:
            return torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        except RuntimeError:
            return torch.empty(t.shape, dtype=t.dtype)

    groups = [meta_in + down_in, gate_in]
    host_in = [[pinned_like(t) for t in g] for g in groups]
    for hg, dg in zip(host_in, groups):
        for h_t, d_t in zip(hg, dg):
            h_t.copy_(d_t)
    host_out = [pinned_like(t) for t in outs]
    h2d = sum(t.numel() * t.element_size() for g in host_in for t in g)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    steps = max(1, min(args.steps, args.e2e_steps))

    experts = inp.experts
    n_chunks = max(1, min(16, experts))
    bounds = [experts * c // n_chunks for c in range(n_chunks + 1)]
    chunks = [(a, b) for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
    s_h2d, s_cmp, s_d2h = (torch.cuda.Stream(dev) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in groups]
    ev_cmp = [[torch.cuda.Event() for _ in chunks] for _ in outs]
    ev_out = [[torch.cuda.Event() for _ in chunks] for _ in outs]
    ev_gemms_done = torch.cuda.Event()
    gemms = [(inp.grad_y_q, inp.hidden_q), (inp.grad_gate_up_q, inp.x_q)]

    def step():
        s_h2d.wait_event(ev_gemms_done)               # the previous step's GEMMs are done reading
        with torch.cuda.stream(s_h2d):
            for g, (hg, dg) in enumerate(zip(host_in, groups)):
                for h_t, d_t in zip(hg, dg):
                    d_t.copy_(h_t, non_blocking=True)
                ev_in[g].record(s_h2d)
        for g, ((lhs, rhs), out) in enumerate(zip(gemms, outs)):
            s_cmp.wait_event(ev_in[g])
            for c, (e0, e1) in enumerate(chunks):
                s_cmp.wait_event(ev_out[g][c])         # the previous copy-out of this chunk is done
                with torch.cuda.stream(s_cmp):
                    fp8_grouped_wgrad_sm90(lhs, rhs, out, m, expert_range=(e0, e1), tuned_config=args.tuned_config)
                ev_cmp[g][c].record(s_cmp)
                s_d2h.wait_event(ev_cmp[g][c])
                with torch.cuda.stream(s_d2h):
                    host_out[g][e0:e1].copy_(out[e0:e1], non_blocking=True)
                ev_out[g][c].record(s_d2h)
        ev_gemms_done.record(s_cmp)

    step()
    torch.cuda.synchronize(dev)
    _barrier(world, dev)
    stream = torch.cuda.current_stream(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for s_ in (s_h2d, s_cmp, s_d2h):
        s_.wait_event(t0)
    for _ in range(steps):
        step()
    for s_ in (s_h2d, s_cmp, s_d2h):
        e_ = torch.cuda.Event()
        e_.record(s_)
        stream.wait_event(e_)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = _max_over_ranks(t0.elapsed_time(t1) / steps, world, dev)
    flops = _sum_over_ranks(step_flops, world, dev)
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
            "pinned": bool(host_in[0][0].is_pinned()), "chunks": len(chunks), "streams": 3}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="dsv3_32k")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--layout", choices=("padded", "packed"), default="padded",
                    help="operand layout (KERNEL_LAB_WGRAD_LAYOUT_MODE of the reference)")
    ap.add_argument("--scale-format", choices=("fp32", "ue8m0"), default="fp32",
                    help="fp32: the reference's amax/448 scales (default, the headline); ue8m0: scales "
                         "rounded up to powers of two, applied by the block-scaled kernel")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tuned-config", default="default",
                    help="tuned_config passed to fp8_grouped_wgrad_sm90 (default: the library's automatic choice)")
    ap.add_argument("--no-library-rate", action="store_true",
                    help="skip the cuBLAS FP8 GEMM rate measured after the timed region (about 5 s)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        log("warm-up raised to 3 (timing rule)")
        args.warmup = 3
    rank, world, _ = dist_env()
    if world != args.gpus and "RANK" in os.environ:
        log(f"--gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
