"""Model-shape x sequence-length x expert-parallel benchmark matrix, and its
Markdown renderer.

Counterpart of the reference's sweep tooling: ``scripts/sweep_seq_lens.py``
(a token-count sweep of one shape), ``scripts/run_model_shape_matrix.sh`` (the
model shapes of ``MODEL_SPECS`` at :33-38, EP sizes, both routes) and
``scripts/render_matrix_results.py`` (results -> publishable Markdown).

Usage::

    python -m sm90_fp8_wgrad.matrix run --models all --ep 1,8 --route both \\
        --tokens-list 4k,8k,16k,32k --output-dir artifacts/matrix
    python -m sm90_fp8_wgrad.matrix render artifacts/matrix/results.jsonl

Expert parallelism (``--ep-mode``):

* ``shard`` (default) -- the global routing of ``tokens`` tokens over all
  experts is drawn once; rank r of EP owns experts [r E/EP, (r+1) E/EP) and
  exactly their rows, which is what one GPU of a real expert-parallel run
  computes. The ranks exchange nothing, so the EP step time is the maximum
  over ranks of the per-rank time. Ranks are timed one after another on the
  current GPU, or, under torchrun with WORLD_SIZE == EP, one per GPU at the
  same time (max over ranks by all-reduce).
* ``proxy-real`` / ``proxy-stress`` -- the reference's single-GPU EP proxy
  (run_model_shape_matrix.sh:74-77): local experts = E/EP routed over by
  ``tokens`` (real) or ``tokens * EP`` (stress) tokens.

Each case is timed with CUDA events (down, gate/up and the total step, the
reference's three timed callables, benchmark_wgrad.py) and checked: the
longest and the shortest non-empty expert of every rank are recomputed with
an fp32 dequantise-then-matmul of the same FP8 operands and compared with the
DeepSeek calc_diff gate (checks.py:175-187); empty experts must be zero.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time
from dataclasses import asdict, dataclass
from pathlib import Path

MODEL_SPECS: dict[str, tuple[str, int, int, int, int]] = {
    # key: (display name, experts, top_k, hidden, intermediate)
    "qwen3_30b": ("Qwen3-30B-A3B", 128, 8, 2048, 768),
    "deepseek_v3": ("DeepSeek-V3", 256, 8, 7168, 2048),
    "minimax_m3": ("MiniMax-M3", 128, 4, 6144, 3072),
    "qwen3_5_397b_a17b": ("Qwen3.5-397B-A17B", 512, 10, 4096, 1024),
}
ROUTE_CHOICES = ("balanced", "skewed", "uniform", "zipf")
EP_MODES = ("shard", "proxy-real", "proxy-stress")


@dataclass(frozen=True)
class Case:
    model: str
    tokens: int
    ep: int
    route: str


def parse_token_count(text: str) -> int:
    """'4096', '4k', '4ki', '32_768' -> tokens (k = 1024, as the reference)."""
    t = str(text).strip().lower().replace("_", "")
    if not t:
        raise RuntimeError("empty token count")
    scale = 1
    for suffix in ("kib", "ki", "k"):
        if t.endswith(suffix):
            scale, t = 1024, t[: -len(suffix)]
            break
    value = int(float(t) * scale)
    if value <= 0:
        raise RuntimeError(f"token count must be positive, got {text!r}")
    return value


def _csv(text: str) -> list[str]:
    return [p.strip() for p in str(text).split(",") if p.strip()]


def parse_models(text: str) -> list[str]:
    names = _csv(text)
    if names == ["all"]:
        return list(MODEL_SPECS)
    for n in names:
        if n not in MODEL_SPECS:
            raise RuntimeError(f"unknown model {n!r}; choices: all,{','.join(MODEL_SPECS)}")
    return names


def parse_model_spec(text: str) -> tuple[str, tuple[str, int, int, int, int]]:
    """'name:experts:top_k:hidden:intermediate' -> a custom MODEL_SPECS entry."""
    parts = str(text).split(":")
    if len(parts) != 5:
        raise RuntimeError("--model-spec wants name:experts:top_k:hidden:intermediate")
    name = parts[0]
    e, k, h, i = (int(p) for p in parts[1:])
    if min(e, k, h, i) <= 0 or k > e:
        raise RuntimeError(f"invalid model spec {text!r}")
    return name, (name, e, k, h, i)


def enumerate_cases(models: list[str], tokens: list[int], eps: list[int], routes: list[str]) -> list[Case]:
    cases = []
    for m in models:
        experts = MODEL_SPECS[m][1]
        for ep in eps:
            if ep <= 0 or experts % ep != 0:
                raise RuntimeError(f"EP={ep} does not divide the {experts} experts of {m}")
            for route in routes:
                for t in tokens:
                    cases.append(Case(m, int(t), int(ep), route))
    return cases


def _route_name(route: str) -> str:
    """The matrix's route names follow the reference (balanced / skewed); the
    BASELINE-style token-level routings (uniform / zipf) are accepted too."""
    if route not in ROUTE_CHOICES:
        raise RuntimeError(f"route must be one of {ROUTE_CHOICES}, got {route!r}")
    return route


def rank_problems(case: Case, ep_mode: str, seed: int):
    """[(routing, expert_range, local_tokens)] for every EP rank of the case."""
    from .routing import make_routing, shard_experts

    _, experts, top_k, _, _ = MODEL_SPECS[case.model]
    route = _route_name(case.route)
    if ep_mode == "shard":
        routing = make_routing(tokens=case.tokens, experts=experts, top_k=top_k, route=route, seed=seed)
        return [(routing, shard_experts(experts, case.ep, r), case.tokens) for r in range(case.ep)]
    if ep_mode not in EP_MODES:
        raise RuntimeError(f"ep-mode must be one of {EP_MODES}")
    local_e = experts // case.ep
    local_t = case.tokens * (case.ep if ep_mode == "proxy-stress" else 1)
    routing = make_routing(tokens=local_t, experts=local_e, top_k=min(top_k, local_e), route=route, seed=seed)
    return [(routing, (0, local_e), local_t)]


def _calc_diff(x, y) -> float:
    x = x.double()
    y = y.double()
    denom = float((x * x + y * y).sum())
    return 0.0 if denom == 0.0 else 1.0 - 2.0 * float((x * y).sum()) / denom


def check_sampled_experts(inp, layout: str, with_rel_err: bool = False):
    """Max calc_diff over the sampled experts (longest and shortest non-empty)
    against an fp32 dequantise-then-matmul of the same FP8 operands (the
    reference's ref_scaled_wgrad, checks.py:42-61); second value: every sampled
    output is finite and every empty expert is exactly zero. With
    ``with_rel_err`` a third value: the largest normwise relative error
    max|out - ref| / max|ref| over the sampled experts.
    An expert's operand rows start at padded_cu_seqlens_k[e] in the padded
    layout and at cu_seqlens_k[e] (valid rows only) in the packed layout."""
    import torch

    counts = inp.counts
    nonempty = [e for e, c in enumerate(counts) if c > 0]
    zeros_ok = all(not inp.down_out_bf16[e].any() and not inp.gate_up_out_bf16[e].any()
                   for e, c in enumerate(counts) if c == 0)
    if not nonempty:
        return (0.0, zeros_ok, 0.0) if with_rel_err else (0.0, zeros_ok)
    sample = sorted({max(nonempty, key=lambda e: counts[e]), min(nonempty, key=lambda e: counts[e])})
    cu = (inp.meta.padded_cu_seqlens_k if layout == "padded" else inp.meta.cu_seqlens_k).cpu().tolist()
    bo = inp.meta.block_offsets.cpu().tolist()

    def deq(op, k0, k1, b0):
        rows = k1 - k0
        nb = (rows + 127) // 128
        return op.data[k0:k1].float() * op.scales[b0:b0 + nb].repeat_interleave(128, dim=0)[:rows]

    worst, worst_rel = 0.0, 0.0
    for e in sample:
        k0, k1, b0 = cu[e], cu[e + 1], bo[e]
        for lhs, rhs, out in ((inp.grad_y_q, inp.hidden_q, inp.down_out_bf16),
                              (inp.grad_gate_up_q, inp.x_q, inp.gate_up_out_bf16)):
            ref = deq(lhs, k0, k1, b0).t() @ deq(rhs, k0, k1, b0)
            got = out[e].float()
            if not bool(torch.isfinite(got).all()):
                return (math.inf, False, math.inf) if with_rel_err else (math.inf, False)
            worst = max(worst, _calc_diff(got, ref))
            worst_rel = max(worst_rel, float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30)))
    return (worst, zeros_ok, worst_rel) if with_rel_err else (worst, zeros_ok)


def check_all_experts(inp, layout: str) -> dict:
    """Whole-output correctness, streamed by expert as the reference's benchmark
    does (scripts/benchmark_wgrad.py:360-414, checks.py:64-86 and :190-223):
    for every expert of both GEMMs, an fp32 dequantise-then-matmul of the same
    FP8 operands on the GPU (``float32_matmul_precision("highest")``, no TF32);
    DeepSeek calc_diff accumulated over all experts of a GEMM, against the
    reference rounded to the output dtype (the reference's metric) and against
    the fp32 reference itself; the worst single expert; the normwise max
    relative error max|out - ref| / max|ref|; every output finite and every
    empty expert exactly zero. Runs after the timed region."""
    import torch

    counts = inp.counts
    cu = (inp.meta.padded_cu_seqlens_k if layout == "padded" else inp.meta.cu_seqlens_k).cpu().tolist()
    bo = inp.meta.block_offsets.cpu().tolist()
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")

    def deq(op, k0, k1, b0):
        rows = k1 - k0
        nb = (rows + 127) // 128
        return op.data[k0:k1].float() * op.scales[b0:b0 + nb].repeat_interleave(128, dim=0)[:rows]

    res = {"experts_checked": 0, "finite": True, "empty_experts_zero": True, "worst_expert_calc_diff": 0.0,
           "max_rel_err_normwise": 0.0}
    try:
        for name, lhs, rhs, out in (("down", inp.grad_y_q, inp.hidden_q, inp.down_out_bf16),
                                    ("gate_up", inp.grad_gate_up_q, inp.x_q, inp.gate_up_out_bf16)):
            num = den = num32 = den32 = 0.0
            max_abs = max_ref = 0.0
            for e, c in enumerate(counts):
                got = out[e].float()
                if c == 0:
                    res["empty_experts_zero"] &= not bool(got.any())
                    continue
                k0, k1, b0 = cu[e], cu[e + 1], bo[e]
                ref = deq(lhs, k0, k1, b0).t() @ deq(rhs, k0, k1, b0)
                if not bool(torch.isfinite(got).all()):
                    res["finite"] = False
                ref_r = ref.to(out.dtype).float()
                xy, xx, yy = (float((got * ref_r).sum()), float((got * got).sum()), float((ref_r * ref_r).sum()))
                num, den = num + xy, den + xx + yy
                num32 += float((got.double() * ref.double()).sum())
                den32 += float((got.double() ** 2).sum() + (ref.double() ** 2).sum())
                if xx + yy > 0:
                    res["worst_expert_calc_diff"] = max(res["worst_expert_calc_diff"], 1.0 - 2.0 * xy / (xx + yy))
                max_abs = max(max_abs, float((got - ref).abs().max()))
                max_ref = max(max_ref, float(ref.abs().max()))
                if name == "down":
                    res["experts_checked"] += 1  # each expert counted once (both of its GEMMs are checked)
                del got, ref, ref_r
            res[f"{name}_calc_diff"] = 0.0 if den == 0 else 1.0 - 2.0 * num / den
            res[f"{name}_calc_diff_vs_fp32"] = 0.0 if den32 == 0 else 1.0 - 2.0 * num32 / den32
            res["max_rel_err_normwise"] = max(res["max_rel_err_normwise"], max_abs / max(max_ref, 1e-30))
    finally:
        torch.set_float32_matmul_precision(prev)
    res["calc_diff_max"] = max(res.get("down_calc_diff", 0.0), res.get("gate_up_calc_diff", 0.0))
    res["calc_diff_vs_fp32_max"] = max(res.get("down_calc_diff_vs_fp32", 0.0), res.get("gate_up_calc_diff_vs_fp32", 0.0))
    return res


def run_rank(case: Case, routing, expert_range, local_tokens: int, *, seed: int, layout: str, tuned_config: str,
             warmup: int, active: int, repeat: int, device) -> dict:
    """Time and check one EP rank's problem on ``device``."""
    import torch

    from .synthetic import make_synthetic_wgrad_inputs, run_custom_down, run_custom_gate_up, run_custom_total
    from .timing import time_cuda, valid_wgrad_flops

    _, _, top_k, hidden, inter = MODEL_SPECS[case.model]
    inp = make_synthetic_wgrad_inputs(tokens=local_tokens, experts=routing.experts, top_k=routing.top_k,
                                      hidden=hidden, intermediate=inter, route=routing.route, seed=seed,
                                      device=device, layout_mode=layout, expert_range=expert_range,
                                      routing=routing)
    inp.drop_sources()
    timing = {}
    for name, fn in (("down", run_custom_down), ("gate_up", run_custom_gate_up), ("total", run_custom_total)):
        stats = time_cuda(lambda fn=fn: fn(inp, tuned_config=tuned_config), warmup_iters=warmup,
                          active_iters=active, repeat=repeat)
        timing[name] = stats.to_dict()
    run_custom_total(inp, tuned_config=tuned_config)
    torch.cuda.synchronize()
    diff, zeros_ok, rel = check_sampled_experts(inp, layout, with_rel_err=True)
    rows = inp.valid_rows
    padded = int(inp.meta.padded_rows)
    blocks = int(inp.meta.total_blocks)
    e_local = inp.experts
    _, _, flops = valid_wgrad_flops(rows, hidden, inter)
    hbm = (padded * (2 * hidden + 3 * inter) + blocks * (2 * hidden + 3 * inter) * 4
           + e_local * 3 * hidden * inter * 2)
    out = {"valid_rows": rows, "padded_rows": padded, "blocks": blocks, "local_experts": e_local,
           "local_tokens": local_tokens, "flops": flops, "hbm_bytes": hbm, "timing": timing,
           "calc_diff": diff, "max_rel_err": rel, "empty_experts_zero": zeros_ok}
    del inp
    torch.cuda.empty_cache()
    return out


def _dist_world() -> tuple[int, int]:
    try:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            return dist.get_rank(), dist.get_world_size()
    except ImportError:
        pass
    return 0, 1


def _reduce_over_ranks(value: float, op: str) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64,
                     device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def run_case(case: Case, *, ep_mode: str, seed: int, layout: str, tuned_config: str, warmup: int, active: int,
             repeat: int, diff_gate: float, fp8_peak_tflops: float | None, device) -> dict:
    problems = rank_problems(case, ep_mode, seed)
    rank, world = _dist_world()
    concurrent = world > 1 and ep_mode == "shard"
    if concurrent and world != case.ep:
        raise RuntimeError(f"under torchrun the EP size must equal WORLD_SIZE ({world}), got {case.ep}")
    mine = [rank] if concurrent else list(range(len(problems)))
    per_rank = []
    for r in mine:
        routing, erange, local_tokens = problems[r]
        res = run_rank(case, routing, erange, local_tokens, seed=seed, layout=layout, tuned_config=tuned_config,
                       warmup=warmup, active=active, repeat=repeat, device=device)
        res["rank"] = r
        per_rank.append(res)
    step = max(p["timing"]["total"]["mean_ms"] for p in per_rank)
    job_flops = sum(p["flops"] for p in per_rank)
    diff = max(p["calc_diff"] for p in per_rank)
    rel_err = max(p["max_rel_err"] for p in per_rank)
    zeros_ok = all(p["empty_experts_zero"] for p in per_rank)
    gpus = len(per_rank)
    if concurrent:
        step = _reduce_over_ranks(step, "max")
        job_flops = _reduce_over_ranks(job_flops, "sum")
        diff = _reduce_over_ranks(diff, "max")
        rel_err = _reduce_over_ranks(rel_err, "max")
        zeros_ok = _reduce_over_ranks(0.0 if zeros_ok else 1.0, "max") == 0.0
        gpus = world
    name, experts, top_k, hidden, inter = MODEL_SPECS[case.model]
    # The slowest rank sets the step, so the job's rate per GPU is
    # (all ranks' FLOPs / number of ranks) / step time.
    per_gpu_tflops = job_flops / gpus / (step * 1e-3) / 1e12 if step > 0 else 0.0
    slow = max(per_rank, key=lambda p: p["timing"]["total"]["mean_ms"])
    row = {
        "model": case.model, "model_name": name, "experts": experts, "top_k": top_k, "hidden": hidden,
        "intermediate": inter, "tokens": case.tokens, "ep": case.ep, "ep_mode": ep_mode, "route": case.route,
        "layout": layout, "tuned_config": tuned_config, "seed": seed,
        "step_ms": step, "per_gpu_tflops": per_gpu_tflops,
        "pct_fp8_peak": (100.0 * per_gpu_tflops / fp8_peak_tflops) if fp8_peak_tflops else None,
        "slowest_rank": slow["rank"], "slowest_rank_hbm_gbs": slow["hbm_bytes"] / (slow["timing"]["total"]["mean_ms"] * 1e-3) / 1e9,
        "imbalance": (step / (sum(p["timing"]["total"]["mean_ms"] for p in per_rank) / len(per_rank))
                      if not concurrent else None),
        "calc_diff": diff, "max_rel_err": rel_err, "diff_gate": diff_gate, "empty_experts_zero": zeros_ok,
        "passed": bool(diff <= diff_gate and zeros_ok), "ranks": per_rank if not concurrent else None,
    }
    return row


# ------------------------------------------------------------------ rendering
def _fmt(v, spec: str, missing: str = "-") -> str:
    if v is None or (isinstance(v, float) and not math.isfinite(v)):
        return missing
    return format(v, spec)


def token_label(tokens: int) -> str:
    return f"{tokens // 1024}k" if tokens % 1024 == 0 else str(tokens)


def render_markdown(rows: list[dict], *, title: str = "Grouped FP8 Wgrad on B200: model-shape matrix") -> str:
    """Markdown tables (one per model) of matrix rows, ordered by route, EP, tokens."""
    lines = [f"# {title}", ""]
    if not rows:
        return "\n".join(lines + ["(no results)", ""])
    meta = rows[0]
    lines.append(f"Layout `{meta.get('layout')}`, config `{meta.get('tuned_config')}`, "
                 f"EP mode `{meta.get('ep_mode')}`, seed {meta.get('seed')}. Step = down + gate/up "
                 "Wgrad; FLOPs count valid rows only (6 H I R); EP step time is the slowest rank; "
                 "max rel err = max|out - ref| / max|ref| over the checked experts.")
    lines.append("")
    by_model: dict[str, list[dict]] = {}
    for r in rows:
        by_model.setdefault(r["model"], []).append(r)
    for model, rs in by_model.items():
        r0 = rs[0]
        lines.append(f"## {r0['model_name']} (E={r0['experts']}, top-{r0['top_k']}, H={r0['hidden']}, "
                     f"I={r0['intermediate']})")
        lines.append("")
        lines.append("| route | EP | tokens | step ms | TFLOP/s per GPU | % FP8 peak | slowest-rank HBM GB/s "
                     "| imbalance | calc_diff | max rel err | ok |")
        lines.append("|---|---:|---:|---:|---:|---:|---:|---:|---:|---:|:-:|")
        for r in sorted(rs, key=lambda x: (x["route"], x["ep"], x["tokens"])):
            lines.append(
                f"| {r['route']} | {r['ep']} | {token_label(r['tokens'])} | {_fmt(r['step_ms'], '.3f')} "
                f"| {_fmt(r['per_gpu_tflops'], '.0f')} | {_fmt(r.get('pct_fp8_peak'), '.1f')} "
                f"| {_fmt(r.get('slowest_rank_hbm_gbs'), '.0f')} | {_fmt(r.get('imbalance'), '.2f')} "
                f"| {_fmt(r['calc_diff'], '.2e')} | {_fmt(r.get('max_rel_err'), '.1e')} "
                f"| {'yes' if r['passed'] else 'NO'} |")
        lines.append("")
    return "\n".join(lines)


def load_rows(path: str | os.PathLike) -> list[dict]:
    rows = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line:
                rows.append(json.loads(line))
    return rows


# ------------------------------------------------------------------ CLI
def _parse(argv: list[str] | None) -> argparse.Namespace:
    p = argparse.ArgumentParser(prog="python -m sm90_fp8_wgrad.matrix", description=__doc__.split("\n\n")[0])
    sub = p.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run", help="run the matrix and write results.jsonl + results.md")
    r.add_argument("--models", default="all")
    r.add_argument("--model-spec", action="append", default=[],
                   help="extra shape name:experts:top_k:hidden:intermediate (may repeat)")
    r.add_argument("--ep", default="1")
    r.add_argument("--ep-mode", choices=EP_MODES, default="shard")
    r.add_argument("--route", default="both", help="balanced, skewed, both, uniform or zipf (comma list)")
    r.add_argument("--tokens-list", default="4096,8192,16384,32768")
    r.add_argument("--warmup-iters", type=int, default=5)
    r.add_argument("--active-iters", type=int, default=20)
    r.add_argument("--repeat", type=int, default=1)
    r.add_argument("--seed", type=int, default=1234)
    r.add_argument("--layout", choices=("padded", "packed"), default="padded")
    r.add_argument("--tuned-config", default="default")
    r.add_argument("--diff-gate", type=float, default=1.0e-3)
    r.add_argument("--fp8-peak-tflops", type=float, default=None,
                   help="denominator of the '% FP8 peak' column (omitted when not given)")
    r.add_argument("--output-dir", default="artifacts/matrix")
    r.add_argument("--dry-run", action="store_true", help="list the cases and exit")
    d = sub.add_parser("render", help="render results.jsonl as Markdown")
    d.add_argument("results")
    d.add_argument("-o", "--output", default=None)
    return p.parse_args(argv)


def main(argv: list[str] | None = None) -> int:
    a = _parse(argv)
    if a.cmd == "render":
        md = render_markdown(load_rows(a.results))
        if a.output:
            Path(a.output).write_text(md)
        else:
            sys.stdout.write(md)
        return 0

    for spec in a.model_spec:
        name, entry = parse_model_spec(spec)
        MODEL_SPECS[name] = entry
    models = parse_models(a.models) if a.models else []
    models += [parse_model_spec(s)[0] for s in a.model_spec if parse_model_spec(s)[0] not in models]
    routes = ["balanced", "skewed"] if a.route == "both" else [_route_name(x) for x in _csv(a.route)]
    cases = enumerate_cases(models, [parse_token_count(t) for t in _csv(a.tokens_list)],
                            [int(x) for x in _csv(a.ep)], routes)
    if a.dry_run:
        for c in cases:
            print(json.dumps(asdict(c)))
        return 0

    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("the matrix run needs a CUDA device")
    own_group = False
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            own_group = True
    device = torch.device("cuda", torch.cuda.current_device())
    rank, _ = _dist_world()
    out_dir = Path(a.output_dir)
    if rank == 0:
        out_dir.mkdir(parents=True, exist_ok=True)
    results = out_dir / "results.jsonl"
    rows = []
    for c in cases:
        t0 = time.time()
        row = run_case(c, ep_mode=a.ep_mode, seed=a.seed, layout=a.layout, tuned_config=a.tuned_config,
                       warmup=a.warmup_iters, active=a.active_iters, repeat=a.repeat, diff_gate=a.diff_gate,
                       fp8_peak_tflops=a.fp8_peak_tflops, device=device)
        row["wall_s"] = time.time() - t0
        rows.append(row)
        if rank == 0:
            with open(results, "a") as f:
                f.write(json.dumps(row) + "\n")
            print(f"{c.model} ep{c.ep} {c.route} {token_label(c.tokens)}: {row['step_ms']:.3f} ms "
                  f"{row['per_gpu_tflops']:.0f} TF/GPU calc_diff {row['calc_diff']:.2e} "
                  f"{'ok' if row['passed'] else 'FAIL'}", flush=True)
    if rank == 0:
        (out_dir / "results.md").write_text(render_markdown(load_rows(results)))
    if own_group:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0 if all(r["passed"] for r in rows) else 1


if __name__ == "__main__":
    sys.exit(main())
