"""The allocation-free entry point, sm100_fp8_grouped_wgrad_noalloc.

Some callers of this library cannot allocate device memory: a host binding
over the C ABI that owns only the input and output buffers it was handed, or a
serving process that reserves its whole device-memory budget at start-up.
Such a caller cannot pass the workspace that the scale-product GEMM
(SM100_WGRAD_TILE_256x256_SP) needs for its split scales, so the library also
exports a variant that takes that scratch from a fixed 64 MiB array compiled
into it. These tests call it through the C ABI (ctypes) and check that its
output equals the workspace entry point's output for the same kernel, bit for
bit and within the oracle's calc_diff gate, on two calls in a row (the array
keeps the previous call's contents), and that a problem needing more scratch
than the array holds is refused. The file sorts last so that a run stopping at
its first failure has run every other test before it; it also passes alone in
a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import wgrad_oracle as O
from golden_inputs import C1, case_inputs

pytestmark = pytest.mark.gpu


def _args(lib_mod, lhs, rhs, out, meta, tile, workspace=None):
    a = lib_mod.Sm100WgradArgs()
    a.lhs_data, a.lhs_pitch = lhs.data.data_ptr(), int(lhs.data.stride(1))
    a.rhs_data, a.rhs_pitch = rhs.data.data_ptr(), int(rhs.data.stride(1))
    a.lhs_scales, a.rhs_scales = lhs.scales.data_ptr(), rhs.scales.data_ptr()
    a.out = out.data_ptr()
    a.out_dtype = lib_mod.OUT_BF16 if out.dtype == torch.bfloat16 else lib_mod.OUT_F32
    a.accumulate = 0
    a.num_experts, a.m, a.n = (int(v) for v in out.shape)
    a.k_rows = int(meta.padded_rows)
    a.total_blocks = int(meta.total_blocks)
    a.block_offsets = meta.block_offsets.data_ptr()
    a.k_row_offsets = meta.padded_cu_seqlens_k.data_ptr()
    a.expert_order = meta.expert_order.data_ptr() if meta.expert_order is not None else None
    a.tile_config = tile
    a.max_ctas = 0
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), int(workspace.numel())
    return a


@pytest.mark.parametrize("tile_name", ["TILE_256x256_SP", "TILE_256x256_SP_W16"])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, tile_name, out_dtype):
    from sm90_fp8_wgrad import _lib, build_wgrad_scale_block_meta, quantize_grouped_wgrad_operand_128x1

    lib = _lib.load()
    tile = getattr(_lib, tile_name)
    counts = C1["counts"]
    cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    meta = build_wgrad_scale_block_meta(torch.from_numpy(cu).to(cuda_device, torch.int32))
    inp = case_inputs(C1)
    om = O.build_meta(cu)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    for lk, rk in (("lhs_down", "rhs_down"), ("lhs_gate", "rhs_gate")):
        lhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp[lk]).to(cuda_device).to(torch.bfloat16), meta)
        rhs = quantize_grouped_wgrad_operand_128x1(torch.from_numpy(inp[rk]).to(cuda_device).to(torch.bfloat16), meta)
        shape = (len(counts), lhs.data.shape[1], rhs.data.shape[1])
        want = torch.full(shape, float("nan"), device=cuda_device, dtype=out_dtype)
        probe = _args(_lib, lhs, rhs, want, meta, tile)
        need = ctypes.c_int64(0)
        assert lib.sm100_wgrad_workspace_bytes(ctypes.byref(probe), ctypes.byref(need)) == _lib.OK
        ws = torch.empty(int(need.value), device=cuda_device, dtype=torch.uint8)
        assert lib.sm100_fp8_grouped_wgrad(ctypes.byref(_args(_lib, lhs, rhs, want, meta, tile, ws)), stream) == _lib.OK
        ref = O.ref_scaled_wgrad(O.quantize_1x128(inp[lk], om), O.quantize_1x128(inp[rk], om), om)
        for call in range(2):   # the array keeps the first call's contents when the second one starts
            got = torch.full(shape, float("nan"), device=cuda_device, dtype=out_dtype)
            status = lib.sm100_fp8_grouped_wgrad_noalloc(ctypes.byref(_args(_lib, lhs, rhs, got, meta, tile)), stream)
            assert status == _lib.OK, (call, _lib.status_string(status))
            torch.cuda.synchronize(cuda_device)
            assert torch.equal(got.view(torch.int16 if out_dtype == torch.bfloat16 else torch.int32),
                               want.view(torch.int16 if out_dtype == torch.bfloat16 else torch.int32)), (lk, call)
            assert O.calc_diff(got.float().cpu().numpy(), ref) <= 1e-5, (lk, call)
    assert _lib.device_error() == 0


def test_noalloc_refuses_problems_beyond_its_array(cuda_device):
    """A problem whose split scales exceed the 64 MiB array is refused before
    any device work (the caller must use the workspace entry point)."""
    from sm90_fp8_wgrad import _lib

    lib = _lib.load()
    a = _lib.Sm100WgradArgs()
    a.lhs_data = a.rhs_data = a.lhs_scales = a.rhs_scales = a.out = 4096
    a.block_offsets = a.k_row_offsets = 4096
    a.lhs_pitch = a.rhs_pitch = 1 << 20
    a.num_experts, a.m, a.n = 256, 7168, 2048
    a.k_rows, a.total_blocks = 1 << 20, 2173          # DeepSeek-V3 32k: ~320 MB of split scales
    a.tile_config = _lib.TILE_256x256_SP
    assert lib.sm100_fp8_grouped_wgrad_noalloc(ctypes.byref(a), None) == _lib.ERR_UNSUPPORTED
    a.tile_config = _lib.TILE_128x256                  # another kernel: not this entry point's
    assert lib.sm100_fp8_grouped_wgrad_noalloc(ctypes.byref(a), None) == _lib.ERR_UNSUPPORTED
