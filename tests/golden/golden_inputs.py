"""Seeded inputs of the golden fixtures (shared by make_golden.py and the tests).

Values come from numpy's PCG64 generator and are rounded to BF16 (nearest
even), so fixtures can be regenerated bit for bit without the reference.
Activations (x, hidden) ~ N(0, 1); gradients (dout, grad_gate_up) ~ N(0, 0.01).
"""
from __future__ import annotations

import numpy as np


def bf16_from_f32(x: np.ndarray) -> np.ndarray:
    """fp32 -> BF16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def uniform_topk_counts(tokens: int, experts: int, top_k: int, seed: int) -> tuple[list[int], np.ndarray]:
    """Each token picks top_k distinct experts uniformly (PCG64 seed); returns
    per-expert counts and the expert-major token gather index."""
    rng = np.random.Generator(np.random.PCG64(seed))
    choice = np.argsort(rng.random((tokens, experts)), axis=1, kind="stable")[:, :top_k]
    flat_e = choice.reshape(-1)
    flat_t = np.repeat(np.arange(tokens), top_k)
    order = np.argsort(flat_e, kind="stable")
    counts = np.bincount(flat_e, minlength=experts)
    return [int(c) for c in counts], flat_t[order]


def _c1_spec() -> dict:
    counts, gather = uniform_topk_counts(1024, 8, 2, 0)
    return {"counts": counts, "gather": gather, "tokens": 1024, "hidden": 256, "intermediate": 128, "seed": 0}


C1 = _c1_spec()

SMALL_CASES = {
    "mixed": {"counts": [0, 1, 31, 32, 33, 127, 128, 129, 300], "tokens": 400, "hidden": 64,
              "intermediate": 32, "seed": 11},
    "single": {"counts": [257], "tokens": 300, "hidden": 32, "intermediate": 16, "seed": 12},
    "all_empty": {"counts": [0, 0, 0], "tokens": 8, "hidden": 32, "intermediate": 16, "seed": 13},
}

META_CASES = {
    "all_empty": [0, 0, 0, 0],
    "tails": [1, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256, 257],
    "single": [1000],
    "zeros_mixed": [0, 5, 0, 300, 0],
    "large": [4096, 0, 17, 70000, 129, 1],
    "one_empty": [0],
}


def case_inputs(spec: dict) -> dict:
    """Grouped fp32 sources of a case (BF16-representable values):
    lhs_down = grad_y [R, H], rhs_down = hidden [R, I],
    lhs_gate = grad_gate_up [R, 2I], rhs_gate = x_grouped [R, H]."""
    counts = spec["counts"]
    rows = int(sum(counts))
    t, h, i = int(spec["tokens"]), int(spec["hidden"]), int(spec["intermediate"])
    rng = np.random.Generator(np.random.PCG64(int(spec["seed"]) + 17))
    x = rng.standard_normal((t, h), dtype=np.float32)
    dout = rng.standard_normal((t, h), dtype=np.float32) * np.float32(0.01)
    hidden = rng.standard_normal((rows, i), dtype=np.float32)
    grad_gu = rng.standard_normal((rows, 2 * i), dtype=np.float32) * np.float32(0.01)
    gather = spec.get("gather")
    if gather is None:
        gather = np.concatenate([(np.arange(c) + 7919 * e) % max(1, t) for e, c in enumerate(counts)]
                                + [np.zeros(0, np.int64)]).astype(np.int64)
    r = lambda a: bf16_to_f32(bf16_from_f32(a))  # noqa: E731
    return {
        "lhs_down": r(dout[gather]),
        "rhs_down": r(hidden),
        "lhs_gate": r(grad_gu),
        "rhs_gate": r(x[gather]),
    }
