"""Seeded MoE routing generators and expert sharding.

Routes (all deterministic for a given seed, generated on the CPU):

* ``uniform``  -- each token picks ``top_k`` distinct experts uniformly at
  random (the "balanced" routing of the benchmark configurations).
* ``zipf``     -- expert probability p_e proportional to 1 / (rank + 1)^alpha
  over a seeded random permutation of the experts (alpha = 1.2 by default),
  ``top_k`` distinct experts per token drawn without replacement. Sampling
  without replacement proportional to p is done with the Gumbel-top-k
  construction (top-k of log p + Gumbel noise).
* ``balanced`` / ``skewed`` -- the reference's count generators
  (src/sm90_fp8_wgrad/synthetic.py:87-121): equal counts, or Zipf-1.15
  multinomial counts with replacement over rows. They produce counts only; the
  grouped rows then use the reference's deterministic gather index
  (synthetic.py:132-150).

Expert parallelism shards experts contiguously: rank r of g owns experts
[r E / g, (r + 1) E / g) and exactly the expert-major rows routed to them.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

ROUTES = ("uniform", "zipf", "balanced", "skewed")


@dataclass(frozen=True)
class Routing:
    """Expert-major routing of ``tokens`` tokens over ``experts`` experts.

    counts[e]    rows routed to expert e
    gather_idx   [sum(counts)] token id of every expert-major row
    """

    tokens: int
    experts: int
    top_k: int
    route: str
    seed: int
    counts: list[int]
    gather_idx: torch.Tensor  # int64, CPU

    @property
    def valid_rows(self) -> int:
        return int(sum(self.counts))

    def cu_seqlens(self) -> list[int]:
        cu = [0]
        for c in self.counts:
            cu.append(cu[-1] + int(c))
        return cu


def _token_choices_to_routing(choice: torch.Tensor, tokens: int, experts: int, top_k: int, route: str,
                              seed: int) -> Routing:
    flat_e = choice.reshape(-1)
    flat_t = torch.arange(tokens, dtype=torch.int64).repeat_interleave(top_k)
    order = torch.argsort(flat_e, stable=True)
    counts = torch.bincount(flat_e, minlength=experts)
    return Routing(tokens, experts, top_k, route, seed, [int(c) for c in counts.tolist()],
                   flat_t[order].contiguous())


def reference_gather_idx(counts: list[int], tokens: int) -> torch.Tensor:
    """Deterministic expert-major gather index of the reference harness
    (synthetic.py:132-150): row r of expert e reads token (r + 7919 e) mod T."""
    parts = [torch.remainder(torch.arange(int(c), dtype=torch.int64) + e * 7919, max(1, int(tokens)))
             for e, c in enumerate(counts) if int(c) > 0]
    return torch.cat(parts) if parts else torch.empty(0, dtype=torch.int64)


def make_routing(*, tokens: int, experts: int, top_k: int, route: str, seed: int,
                 zipf_alpha: float = 1.2) -> Routing:
    tokens, experts, top_k, seed = int(tokens), int(experts), int(top_k), int(seed)
    if route not in ROUTES:
        raise RuntimeError(f"route must be one of {ROUTES}, got {route!r}")
    if top_k > experts or top_k <= 0 or tokens < 0:
        raise RuntimeError(f"invalid routing shape tokens={tokens} experts={experts} top_k={top_k}")
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    if route == "uniform":
        keys = torch.rand((tokens, experts), generator=gen)
        choice = torch.topk(keys, top_k, dim=1).indices
        return _token_choices_to_routing(choice, tokens, experts, top_k, route, seed)
    if route == "zipf":
        ranks = torch.arange(1, experts + 1, dtype=torch.float64)
        p = 1.0 / torch.pow(ranks, float(zipf_alpha))
        p = p / p.sum()
        p = p[torch.randperm(experts, generator=gen)]
        u = torch.rand((tokens, experts), generator=gen, dtype=torch.float64).clamp_(1e-300, 1.0)
        keys = torch.log(p).unsqueeze(0) - torch.log(-torch.log(u))
        choice = torch.topk(keys, top_k, dim=1).indices
        return _token_choices_to_routing(choice, tokens, experts, top_k, route, seed)
    valid = tokens * top_k
    if route == "balanced":
        base, rem = divmod(valid, experts)
        counts = [base + (1 if e < rem else 0) for e in range(experts)]
    else:  # skewed: reference generator, Zipf 1.15 with replacement over rows
        ranks = torch.arange(1, experts + 1, dtype=torch.float64)
        p = 1.0 / torch.pow(ranks, 1.15)
        p = (p / p.sum())[torch.randperm(experts, generator=gen)]
        counts = torch.multinomial(p, valid, replacement=True, generator=gen).bincount(minlength=experts).tolist()
    return Routing(tokens, experts, top_k, route, seed, [int(c) for c in counts],
                   reference_gather_idx(counts, tokens))


def routing_from_counts(counts: list[int], tokens: int, top_k: int = 1, seed: int = 0) -> Routing:
    counts = [int(c) for c in counts]
    return Routing(int(tokens), len(counts), int(top_k), "counts", int(seed), counts,
                   reference_gather_idx(counts, tokens))


def shard_experts(experts: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous expert range [e0, e1) owned by ``rank``."""
    if experts % world_size != 0:
        raise RuntimeError(f"experts={experts} must divide evenly over world_size={world_size}")
    per = experts // world_size
    return rank * per, (rank + 1) * per


def shard_routing(routing: Routing, e0: int, e1: int) -> Routing:
    """The rows of experts [e0, e1) (a contiguous slice of the expert-major order)."""
    cu = routing.cu_seqlens()
    return Routing(routing.tokens, e1 - e0, routing.top_k, routing.route, routing.seed,
                   routing.counts[e0:e1], routing.gather_idx[cu[e0]:cu[e1]].clone())
