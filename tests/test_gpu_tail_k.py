"""GPU parity of the compact tail-K quantiser (reference quant.py:273-307).

``quantize_grouped_wgrad_operand_tail_k`` gathers each expert's final partial
128-row block (the rows ``build_wgrad_tail_block_meta`` lists in
``tail_indices``, reference block_meta.py:352-465) and quantises them with 32-
or 64-row scale blocks into the padded layout. Bytes and scales are compared
bit-exactly with the CPU oracle's quantiser run on the same gathered rows.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import wgrad_oracle as O

pytestmark = pytest.mark.gpu

CASES = {
    "edge": [1, 31, 32, 33, 63, 64, 65, 127, 128, 129, 0, 255, 256, 257, 200],
    "no_tail": [128, 256, 0, 384],
    "one_expert": [77],
}


def _cu(counts):
    return np.concatenate([[0], np.cumsum(np.asarray(counts, np.int64))]).astype(np.int64)


@pytest.mark.parametrize("tail_block_k", [32, 64])
@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_tail_k_operand_matches_oracle(cuda_device, case, tail_block_k, dtype):
    from sm90_fp8_wgrad import build_wgrad_tail_block_meta, quantize_grouped_wgrad_operand_tail_k

    counts = CASES[case]
    cols = 80
    rng = np.random.Generator(np.random.PCG64(29))
    x = torch.from_numpy(rng.standard_normal((sum(counts), cols), dtype=np.float32)).to(dtype)
    tm = build_wgrad_tail_block_meta(torch.from_numpy(_cu(counts)).to(cuda_device, torch.int32),
                                     tail_block_k=tail_block_k)
    meta = tm.meta
    op = quantize_grouped_wgrad_operand_tail_k(x.to(cuda_device), tm.tail_indices, meta)
    torch.cuda.synchronize()

    src = x.float().numpy()[tm.tail_indices.cpu().numpy()]
    ref = O.quantize_blocks(src, meta.block_row_start.cpu().numpy(), meta.block_row_count.cpu().numpy(),
                            tail_block_k, int(meta.padded_rows))
    assert tuple(op.data.shape) == (int(meta.padded_rows), cols)
    got = op.data.t().contiguous().view(torch.uint8).cpu().numpy()     # [cols, padded_rows]
    np.testing.assert_array_equal(got, ref.data[:, : int(meta.padded_rows)])
    np.testing.assert_array_equal(op.scales.cpu().numpy().view(np.uint32), ref.scales.view(np.uint32))
    pitch = op.data.stride(1)
    assert pitch == max(128, (int(meta.padded_rows) + 127) // 128 * 128)


def test_tail_k_bad_index_sets_device_error(cuda_device):
    """An out-of-range tail index reads zeros and sets device error 5; nothing
    outside the source tensor is read."""
    from sm90_fp8_wgrad import _lib, build_wgrad_tail_block_meta, quantize_grouped_wgrad_operand_tail_k

    lib = _lib.load()
    code = ctypes.c_int32(0)
    assert lib.sm100_wgrad_device_error(ctypes.byref(code)) == 0       # clear
    counts = [40, 10]
    tm = build_wgrad_tail_block_meta(torch.tensor(_cu(counts), dtype=torch.int32, device=cuda_device),
                                     tail_block_k=32)
    x = torch.ones((sum(counts), 32), device=cuda_device, dtype=torch.bfloat16)
    bad = tm.tail_indices.clone()
    bad[3] = 10_000
    op = quantize_grouped_wgrad_operand_tail_k(x, bad, tm.meta)
    torch.cuda.synchronize()
    assert lib.sm100_wgrad_device_error(ctypes.byref(code)) == 0
    assert code.value == 5
    assert not op.data.t()[:, 3].view(torch.uint8).any()                # the bad row quantised as zeros
    assert lib.sm100_wgrad_device_error(ctypes.byref(code)) == 0 and code.value == 0


def test_tail_k_bad_index_raises_at_next_call(cuda_device):
    """Without any synchronisation by the caller, the next quantiser call raises."""
    from sm90_fp8_wgrad import _lib, build_wgrad_tail_block_meta, quantize_grouped_wgrad_operand_tail_k

    _lib.device_error()
    counts = [40, 10]
    tm = build_wgrad_tail_block_meta(torch.tensor(_cu(counts), dtype=torch.int32, device=cuda_device),
                                     tail_block_k=32)
    x = torch.ones((sum(counts), 32), device=cuda_device, dtype=torch.bfloat16)
    bad = tm.tail_indices.clone()
    bad[3] = 10_000
    quantize_grouped_wgrad_operand_tail_k(x, bad, tm.meta)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device error 5"):
        quantize_grouped_wgrad_operand_tail_k(x, tm.tail_indices, tm.meta)
    assert _lib.device_error() == 5
    quantize_grouped_wgrad_operand_tail_k(x, tm.tail_indices, tm.meta)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def test_tail_k_rejects_bad_arguments(cuda_device):
    from sm90_fp8_wgrad import build_wgrad_tail_block_meta, quantize_grouped_wgrad_operand_tail_k

    tm = build_wgrad_tail_block_meta(torch.tensor([0, 40], dtype=torch.int32, device=cuda_device), tail_block_k=64)
    x = torch.zeros((40, 16), device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="valid_rows"):
        quantize_grouped_wgrad_operand_tail_k(x, tm.tail_indices[:-1], tm.meta)
    with pytest.raises(RuntimeError, match="x_grouped"):
        quantize_grouped_wgrad_operand_tail_k(x[0], tm.tail_indices, tm.meta)
    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_grouped_wgrad_operand_tail_k(x, tm.tail_indices.cpu(), tm.meta)
