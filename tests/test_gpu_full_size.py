"""GPU parity at the benchmark's full sizes (BASELINE.json configs C2-C5).

The CPU oracle cannot finish a 23-TFLOP problem in seconds, so at these sizes
the check is per expert: after both grouped GEMMs of a full-size problem ran
through the public operator, a sample of experts (the longest, the shortest
non-empty, a random one, and every empty one) is recomputed with a plain
PyTorch fp32 dequantise-then-matmul of the same FP8 bytes and scales -- the
reference's own algorithm (src/sm90_fp8_wgrad/checks.py:42-61) -- and compared
with DeepSeek calc_diff <= 1e-5 (the contract gate, checks.py:175-187).
Empty experts must come out exactly zero. Multi-GPU configs are checked on
the 1/8 expert shard that one GPU of the 8-GPU run computes.
"""
from __future__ import annotations

import random

import pytest
import torch

pytestmark = pytest.mark.gpu

# name: (experts, top_k, hidden, intermediate, tokens, route, shards)
CONFIGS = {
    "dsv3_32k": (256, 8, 7168, 2048, 32768, "uniform", 1),
    "dsv3_4k": (256, 8, 7168, 2048, 4096, "uniform", 1),
    "qwen3_32k": (128, 8, 2048, 768, 32768, "uniform", 1),
    "dsv3_skewed_32k": (256, 8, 7168, 2048, 32768, "zipf", 1),
    "large_expert_16k_shard": (32, 2, 6144, 9216, 16384, "zipf", 8),
    "many_small_32k_shard": (512, 10, 4096, 1024, 32768, "zipf", 8),
}


def _dequant(op, k0: int, k1: int, b0: int) -> torch.Tensor:
    """fp32 [rows, cols] of operand rows k0..k1 (blocks from b0): whole 128-row
    blocks in the padded layout, valid rows only in the packed layout."""
    rows = op.data[k0:k1].float()
    nb = (k1 - k0 + 127) // 128
    scale = op.scales[b0:b0 + nb].repeat_interleave(128, dim=0)[: k1 - k0]
    return rows * scale


def _calc_diff(x: torch.Tensor, y: torch.Tensor) -> float:
    x = x.double()
    y = y.double()
    denom = (x * x + y * y).sum()
    if denom == 0:
        return 0.0
    return float(1.0 - 2.0 * (x * y).sum() / denom)


@pytest.mark.parametrize("name,layout", [(n, "padded") for n in sorted(CONFIGS)] +
                         [("dsv3_skewed_32k", "packed"), ("many_small_32k_shard", "packed")])
def test_full_size_sampled_experts(cuda_device, name, layout):
    from sm90_fp8_wgrad.routing import make_routing, shard_experts
    from sm90_fp8_wgrad.synthetic import make_synthetic_wgrad_inputs, run_custom_down, run_custom_gate_up

    experts, top_k, hidden, inter, tokens, route, shards = CONFIGS[name]
    routing = make_routing(tokens=tokens, experts=experts, top_k=top_k, route=route, seed=1234)
    e0, e1 = shard_experts(experts, shards, 0)
    inp = make_synthetic_wgrad_inputs(tokens=tokens, experts=experts, top_k=top_k, hidden=hidden,
                                      intermediate=inter, route=route, seed=1234, device=cuda_device,
                                      expert_range=(e0, e1), routing=routing, layout_mode=layout)
    inp.drop_sources()
    run_custom_down(inp)
    run_custom_gate_up(inp)
    torch.cuda.synchronize()

    counts = inp.counts
    cu = (inp.meta.padded_cu_seqlens_k if layout == "padded" else inp.meta.cu_seqlens_k).cpu().tolist()
    bo = inp.meta.block_offsets.cpu().tolist()
    nonempty = [e for e, c in enumerate(counts) if c > 0]
    sample = {max(nonempty, key=lambda e: counts[e]), min(nonempty, key=lambda e: counts[e]),
              random.Random(7).choice(nonempty)}
    empty = [e for e, c in enumerate(counts) if c == 0]

    for e in sorted(sample):
        k0, k1, b0 = cu[e], cu[e + 1], bo[e]
        for lhs, rhs, out in ((inp.grad_y_q, inp.hidden_q, inp.down_out_bf16),
                              (inp.grad_gate_up_q, inp.x_q, inp.gate_up_out_bf16)):
            ref = _dequant(lhs, k0, k1, b0).t() @ _dequant(rhs, k0, k1, b0)
            got = out[e].float()
            assert torch.isfinite(got).all()
            cd = _calc_diff(got, ref)
            assert cd <= 1e-5, (name, layout, e, counts[e], cd)
    for e in empty:
        assert not inp.down_out_bf16[e].any() and not inp.gate_up_out_bf16[e].any(), (name, e)


@pytest.mark.parametrize("policy", ["adaptive64", "adaptive32_64_twophase"])
def test_full_size_packed_tail_policies(cuda_device, monkeypatch, policy):
    """Packed layout with the adaptive tail-copy policies at full size (their
    kernel_data offsets and guard rows differ from masked128): every sampled
    expert of the skewed DeepSeek-V3 32k problem within the gate."""
    from sm90_fp8_wgrad.layout_mode import PACKED_TAIL_ENV
    from sm90_fp8_wgrad.matrix import check_sampled_experts
    from sm90_fp8_wgrad.routing import make_routing
    from sm90_fp8_wgrad.synthetic import make_synthetic_wgrad_inputs, run_custom_down, run_custom_gate_up

    monkeypatch.setenv(PACKED_TAIL_ENV, policy)
    experts, top_k, hidden, inter, tokens, route, _ = CONFIGS["dsv3_skewed_32k"]
    routing = make_routing(tokens=tokens, experts=experts, top_k=top_k, route=route, seed=1234)
    inp = make_synthetic_wgrad_inputs(tokens=tokens, experts=experts, top_k=top_k, hidden=hidden,
                                      intermediate=inter, route=route, seed=1234, device=cuda_device,
                                      routing=routing, layout_mode="packed")
    assert inp.meta.packed_tail_tma_mode == policy
    inp.drop_sources()
    run_custom_down(inp)
    run_custom_gate_up(inp)
    torch.cuda.synchronize()
    diff, zeros_ok, rel = check_sampled_experts(inp, "packed", with_rel_err=True)
    assert zeros_ok and diff <= 1e-5, (policy, diff, rel)


def test_full_size_accumulate_and_expert_ranges(cuda_device):
    """DeepSeek-V3 32k down GEMM: 16 expert-range launches equal one launch bit for
    bit, and accumulate=True into fp32 adds exactly the launch's result to the
    previous contents (sampled experts vs the fp32 reference)."""
    from sm90_fp8_wgrad import fp8_grouped_wgrad_sm90
    from sm90_fp8_wgrad.routing import make_routing
    from sm90_fp8_wgrad.synthetic import make_synthetic_wgrad_inputs

    experts, top_k, hidden, inter, tokens, route, _ = CONFIGS["dsv3_32k"]
    routing = make_routing(tokens=tokens, experts=experts, top_k=top_k, route=route, seed=1234)
    inp = make_synthetic_wgrad_inputs(tokens=tokens, experts=experts, top_k=top_k, hidden=hidden,
                                      intermediate=inter, route=route, seed=1234, device=cuda_device,
                                      routing=routing)
    inp.drop_sources()
    lhs, rhs, meta = inp.grad_y_q, inp.hidden_q, inp.meta
    full = torch.empty_like(inp.down_out_bf16)
    fp8_grouped_wgrad_sm90(lhs, rhs, full, meta)
    part = torch.empty_like(full)
    for c in range(16):
        fp8_grouped_wgrad_sm90(lhs, rhs, part, meta, expert_range=(c * experts // 16, (c + 1) * experts // 16))
    torch.cuda.synchronize()
    assert torch.equal(part.view(torch.int16), full.view(torch.int16))

    base = torch.full(full.shape, 0.25, device=cuda_device, dtype=torch.float32)
    fp8_grouped_wgrad_sm90(lhs, rhs, base, meta, accumulate=True)
    torch.cuda.synchronize()
    base -= 0.25                      # the accumulated result minus the initial value
    counts = inp.counts
    nonempty = [e for e, c in enumerate(counts) if c > 0]
    cu = meta.padded_cu_seqlens_k.cpu().tolist()
    bo = meta.block_offsets.cpu().tolist()
    for e in (max(nonempty, key=lambda x: counts[x]), min(nonempty, key=lambda x: counts[x])):
        k0, k1, b0 = cu[e], cu[e + 1], bo[e]
        ref = _dequant(lhs, k0, k1, b0).t() @ _dequant(rhs, k0, k1, b0)
        assert _calc_diff(base[e], ref) <= 1e-5


@pytest.mark.parametrize("name", ["dsv3_32k", "dsv3_skewed_32k"])
def test_full_size_every_expert(cuda_device, name):
    """Whole-output correctness at full size, as the reference's benchmark
    checks it (scripts/benchmark_wgrad.py:360-414): every expert of both GEMMs
    against an fp32 dequantise-then-matmul of the same FP8 operands, DeepSeek
    calc_diff accumulated over the whole output of each GEMM (vs the reference
    rounded to BF16, the reference's metric, and vs the fp32 reference) within
    1e-5; every output finite, every empty expert zero."""
    from sm90_fp8_wgrad.matrix import check_all_experts
    from sm90_fp8_wgrad.routing import make_routing
    from sm90_fp8_wgrad.synthetic import make_synthetic_wgrad_inputs, run_custom_down, run_custom_gate_up

    experts, top_k, hidden, inter, tokens, route, _ = CONFIGS[name]
    routing = make_routing(tokens=tokens, experts=experts, top_k=top_k, route=route, seed=1234)
    inp = make_synthetic_wgrad_inputs(tokens=tokens, experts=experts, top_k=top_k, hidden=hidden,
                                      intermediate=inter, route=route, seed=1234, device=cuda_device,
                                      routing=routing)
    inp.drop_sources()
    run_custom_down(inp)
    run_custom_gate_up(inp)
    torch.cuda.synchronize()
    r = check_all_experts(inp, "padded")
    assert r["experts_checked"] == sum(1 for c in inp.counts if c > 0), r
    assert r["finite"] and r["empty_experts_zero"], r
    assert r["calc_diff_max"] <= 1e-5 and r["calc_diff_vs_fp32_max"] <= 1e-5, r


def test_full_size_quantiser_sampled_blocks_bit_exact(cuda_device):
    """The CUDA quantiser's bytes and scales at DeepSeek-V3 32k size, on sampled
    (scale block, 64-column strip) pieces of all four operands, bit for bit
    against the oracle's restatement of the reference quantiser
    (quant.py:129-167) applied to the same BF16 rows."""
    import numpy as np

    import wgrad_oracle as O
    from sm90_fp8_wgrad.routing import make_routing
    from sm90_fp8_wgrad.synthetic import make_synthetic_wgrad_inputs

    experts, top_k, hidden, inter, tokens, route, _ = CONFIGS["dsv3_32k"]
    routing = make_routing(tokens=tokens, experts=experts, top_k=top_k, route=route, seed=1234)
    inp = make_synthetic_wgrad_inputs(tokens=tokens, experts=experts, top_k=top_k, hidden=hidden,
                                      intermediate=inter, route=route, seed=1234, device=cuda_device,
                                      routing=routing, allocate_custom_outputs=False)
    torch.cuda.synchronize()
    rs = inp.meta.block_row_start.cpu().numpy()
    rc = inp.meta.block_row_count.cpu().numpy()
    rng = random.Random(11)
    pairs = ((inp.grad_y_grouped_bf16, inp.grad_y_q), (inp.hidden_grouped_bf16, inp.hidden_q),
             (inp.grad_gate_up_grouped_bf16, inp.grad_gate_up_q), (inp.x_grouped_bf16, inp.x_q))
    checked = 0
    for src, op in pairs:
        cols = src.shape[1]
        pitch = op.data.stride(1)
        storage = op.data.as_strided((cols, pitch), (pitch, 1))
        for _ in range(12):
            b = rng.randrange(int(inp.meta.total_blocks))
            c0 = rng.randrange(cols // 64) * 64
            r0, n = int(rs[b]), int(rc[b])
            x = src[r0:r0 + n, c0:c0 + 64].float().cpu().numpy()
            ref = O.quantize_blocks(x, [0], [n], 128, 128)
            got = storage[c0:c0 + 64, b * 128:(b + 1) * 128].view(torch.uint8).cpu().numpy()
            np.testing.assert_array_equal(got, ref.data[:, :128], err_msg=f"block {b} cols {c0}")
            np.testing.assert_array_equal(op.scales[b, c0:c0 + 64].cpu().numpy().view(np.uint32),
                                          ref.scales[0].view(np.uint32), err_msg=f"scales block {b} cols {c0}")
            checked += 1
    assert checked == 48
