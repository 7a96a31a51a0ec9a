"""Synthetic grouped Wgrad inputs (harness API).

``make_synthetic_wgrad_inputs`` keeps the reference signature
(src/sm90_fp8_wgrad/synthetic.py:191-288) and result fields, with:

* the routes of ``routing.py`` (``uniform`` and ``zipf`` added to the
  reference's ``balanced`` / ``skewed``),
* value scales of the benchmark configurations: activations (x, hidden)
  ~ N(0, 1), gradients (dout, grad_gate_up) ~ N(0, grad_std) with
  grad_std = 0.01 by default (``grad_std=1.0`` reproduces the reference's
  all-N(0,1) draw),
* ``expert_range`` for expert-parallel shards: only the rows routed to experts
  [e0, e1) are materialised, and the outputs have e1 - e0 experts.

Sources are drawn on the device with a seeded ``torch.Generator`` (seed + 17,
as in the reference); quantisation and metadata run on the GPU.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from .block_meta import WgradScaleBlockMeta, build_wgrad_scale_block_meta
from .checks import scaled_wgrad_error
from .interface import fp8_grouped_wgrad_sm90
from .layout_mode import LAYOUT_MODE_PADDED
from .quant import Fp8GroupedWgradOperand, quantize_grouped_wgrad_operand_128x1
from .routing import Routing, make_routing, routing_from_counts, shard_routing


@dataclass
class SyntheticWgradInputs:
    tokens: int
    experts: int
    top_k: int
    hidden: int
    intermediate: int
    dtype: torch.dtype
    route: str
    counts: list[int]
    cu_seqlens_k: torch.Tensor
    x_gather_idx: torch.Tensor
    x_bf16: torch.Tensor | None
    dout_bf16: torch.Tensor | None
    hidden_grouped_bf16: torch.Tensor | None
    grad_gate_up_grouped_bf16: torch.Tensor | None
    grad_y_grouped_bf16: torch.Tensor | None
    x_grouped_bf16: torch.Tensor | None
    meta: WgradScaleBlockMeta
    grad_y_q: Fp8GroupedWgradOperand | None
    hidden_q: Fp8GroupedWgradOperand | None
    grad_gate_up_q: Fp8GroupedWgradOperand | None
    x_q: Fp8GroupedWgradOperand | None
    down_out_bf16: torch.Tensor | None
    gate_up_out_bf16: torch.Tensor | None

    @property
    def valid_rows(self) -> int:
        return int(sum(self.counts))

    def drop_sources(self) -> None:
        """Release the BF16 source tensors (keeps FP8 operands and outputs)."""
        self.x_bf16 = self.dout_bf16 = None
        self.hidden_grouped_bf16 = self.grad_gate_up_grouped_bf16 = None
        self.grad_y_grouped_bf16 = self.x_grouped_bf16 = None


def dtype_from_name(name: str) -> torch.dtype:
    key = str(name).strip().lower()
    if key in ("bf16", "bfloat16"):
        return torch.bfloat16
    if key in ("fp32", "float32"):
        return torch.float32
    raise RuntimeError(f"unsupported dtype {name!r}")


def load_counts_file(path) -> list[int]:
    """JSON list / {"counts": [...]} or CSV (last column) of per-expert counts
    (reference synthetic.py:62-84)."""
    import csv
    import json
    from pathlib import Path

    p = Path(path)
    if p.suffix.lower() == ".json":
        data = json.loads(p.read_text(encoding="utf-8"))
        if isinstance(data, dict):
            data = data.get("counts", data.get("expert_counts"))
        if not isinstance(data, list):
            raise RuntimeError("counts JSON must be a list or contain a 'counts' list")
        return [int(v) for v in data]
    counts = []
    with p.open("r", encoding="utf-8", newline="") as f:
        for row in csv.reader(f):
            if not row or row[0].strip().startswith("#"):
                continue
            counts.append(int(row[-1]))
    if not counts:
        raise RuntimeError(f"no counts found in {p}")
    return counts


def make_expert_counts(*, tokens: int, top_k: int, experts: int, route: str, seed: int,
                       counts_file: str | None = None) -> list[int]:
    if counts_file:
        counts = load_counts_file(counts_file)
        if len(counts) != int(experts):
            raise RuntimeError(f"counts file has {len(counts)} experts, expected {experts}")
        if sum(counts) != int(tokens) * int(top_k):
            raise RuntimeError(f"counts sum {sum(counts)} does not match tokens*top_k {int(tokens) * int(top_k)}")
        return counts
    return make_routing(tokens=tokens, experts=experts, top_k=top_k, route=route, seed=seed).counts


def counts_to_cu_seqlens(counts: list[int], *, device: torch.device) -> torch.Tensor:
    cu = torch.zeros(len(counts) + 1, dtype=torch.int64)
    if counts:
        cu[1:] = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0)
    return cu.to(device=device, dtype=torch.int32).contiguous()


def route_stats(counts: list[int], meta: WgradScaleBlockMeta) -> dict:
    s = sorted(int(v) for v in counts)
    return {
        "experts": len(counts),
        "valid_rows": int(sum(counts)),
        "padded_rows": int(meta.padded_rows),
        "wgmma_rows": int(meta.wgmma_rows),
        "tma_rows": int(meta.tma_rows),
        "total_blocks": int(meta.total_blocks),
        "min_rows_per_expert": s[0] if s else 0,
        "median_rows_per_expert": s[len(s) // 2] if s else 0,
        "max_rows_per_expert": s[-1] if s else 0,
        "padding_overhead_ratio": float(meta.padded_rows) / float(max(1, sum(counts))),
        "packed_tail_tma_mode": str(meta.packed_tail_tma_mode),
    }


def make_synthetic_wgrad_inputs(
    *,
    tokens: int,
    experts: int = 128,
    top_k: int = 8,
    hidden: int = 2048,
    intermediate: int = 768,
    route: str = "skewed",
    seed: int = 1234,
    counts_file: str | None = None,
    dtype: torch.dtype = torch.bfloat16,
    device: torch.device | None = None,
    layout_mode: str = LAYOUT_MODE_PADDED,
    build_fp8_operands: bool = True,
    allocate_custom_outputs: bool = True,
    grad_std: float = 0.01,
    expert_range: tuple[int, int] | None = None,
    routing: Routing | None = None,
    scale_format: str = "fp32",
) -> SyntheticWgradInputs:
    if device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA is required to build Wgrad benchmark inputs")
        device = torch.device("cuda")
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("CUDA device is required")
    # The launch path resolves the layout from this variable, as in the reference.
    os.environ["KERNEL_LAB_WGRAD_LAYOUT_MODE"] = str(layout_mode)

    if routing is None:
        if counts_file:
            routing = routing_from_counts(
                make_expert_counts(tokens=tokens, top_k=top_k, experts=experts, route=route, seed=seed,
                                   counts_file=counts_file), tokens, top_k, seed)
        else:
            routing = make_routing(tokens=tokens, experts=experts, top_k=top_k, route=route, seed=seed)
    e0, e1 = expert_range if expert_range is not None else (0, int(experts))
    local = shard_routing(routing, e0, e1)
    e_local = e1 - e0

    cu = counts_to_cu_seqlens(local.counts, device=device)
    gather = local.gather_idx.to(device)
    meta = build_wgrad_scale_block_meta(cu, block_k=128)

    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed) + 17)
    rows = local.valid_rows
    x = torch.randn((int(tokens), int(hidden)), device=device, dtype=dtype, generator=gen)
    dout = torch.randn((int(tokens), int(hidden)), device=device, dtype=dtype, generator=gen).mul_(grad_std)
    hidden_grouped = torch.randn((rows, int(intermediate)), device=device, dtype=dtype, generator=gen)
    grad_gate_up_grouped = torch.randn((rows, 2 * int(intermediate)), device=device, dtype=dtype,
                                       generator=gen).mul_(grad_std)
    grad_y_grouped = dout.index_select(0, gather).contiguous()
    x_grouped = x.index_select(0, gather).contiguous()

    if build_fp8_operands:
        grad_y_q = quantize_grouped_wgrad_operand_128x1(grad_y_grouped, meta, layout_mode=layout_mode,
                                                        scale_format=scale_format)
        hidden_q = quantize_grouped_wgrad_operand_128x1(hidden_grouped, meta, layout_mode=layout_mode,
                                                        scale_format=scale_format)
        grad_gate_up_q = quantize_grouped_wgrad_operand_128x1(grad_gate_up_grouped, meta, layout_mode=layout_mode,
                                                        scale_format=scale_format)
        x_q = quantize_grouped_wgrad_operand_128x1(x_grouped, meta, layout_mode=layout_mode,
                                                        scale_format=scale_format)
    else:
        grad_y_q = hidden_q = grad_gate_up_q = x_q = None

    if allocate_custom_outputs:
        down_out = torch.empty((e_local, int(hidden), int(intermediate)), device=device, dtype=torch.bfloat16)
        gate_up_out = torch.empty((e_local, 2 * int(intermediate), int(hidden)), device=device, dtype=torch.bfloat16)
    else:
        down_out = gate_up_out = None

    return SyntheticWgradInputs(
        tokens=int(tokens), experts=e_local, top_k=int(top_k), hidden=int(hidden),
        intermediate=int(intermediate), dtype=dtype, route=str(route), counts=list(local.counts),
        cu_seqlens_k=cu, x_gather_idx=gather.to(torch.int32), x_bf16=x, dout_bf16=dout,
        hidden_grouped_bf16=hidden_grouped, grad_gate_up_grouped_bf16=grad_gate_up_grouped,
        grad_y_grouped_bf16=grad_y_grouped, x_grouped_bf16=x_grouped, meta=meta,
        grad_y_q=grad_y_q, hidden_q=hidden_q, grad_gate_up_q=grad_gate_up_q, x_q=x_q,
        down_out_bf16=down_out, gate_up_out_bf16=gate_up_out,
    )


def run_custom_down(inp: SyntheticWgradInputs, *, tuned_config: str = "default") -> None:
    if inp.grad_y_q is None or inp.hidden_q is None or inp.down_out_bf16 is None:
        raise RuntimeError("custom down requires FP8 operands and a down output buffer")
    fp8_grouped_wgrad_sm90(inp.grad_y_q, inp.hidden_q, inp.down_out_bf16, inp.meta, tuned_config=tuned_config)


def run_custom_gate_up(inp: SyntheticWgradInputs, *, tuned_config: str = "default") -> None:
    if inp.grad_gate_up_q is None or inp.x_q is None or inp.gate_up_out_bf16 is None:
        raise RuntimeError("custom gate/up requires FP8 operands and a gate/up output buffer")
    fp8_grouped_wgrad_sm90(inp.grad_gate_up_q, inp.x_q, inp.gate_up_out_bf16, inp.meta, tuned_config=tuned_config)


def run_custom_total(inp: SyntheticWgradInputs, *, tuned_config: str = "default") -> None:
    run_custom_down(inp, tuned_config=tuned_config)
    run_custom_gate_up(inp, tuned_config=tuned_config)


def finite_status(tensors: dict[str, torch.Tensor]) -> dict[str, bool]:
    out = {}
    with torch.no_grad():
        for name, t in tensors.items():
            ok = True
            flat = t.detach().reshape(-1)
            step = int(os.environ.get("SM90_WGRAD_FINITE_CHECK_CHUNK_ELEMENTS", "8388608"))
            for i in range(0, flat.numel(), step):
                if not bool(torch.isfinite(flat[i : i + step]).all().item()):
                    ok = False
                    break
            out[name] = ok
    return out


def error_summary(actual: torch.Tensor, expected: torch.Tensor) -> dict[str, float]:
    max_abs, max_rel, max_abs_ref = scaled_wgrad_error(actual, expected)
    return {"max_abs": max_abs, "max_rel": max_rel, "max_abs_ref": max_abs_ref}
