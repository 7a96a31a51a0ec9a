"""CPU checks of the oracle's UE8M0 option (power-of-two scales), the checker
the GPU tests of the UE8M0 quantiser and kernel compare against. The reference
has no such mode; these pin the rounding rule itself."""
from __future__ import annotations

import numpy as np

import wgrad_oracle as O
from golden_inputs import SMALL_CASES, case_inputs


def test_round_up_pow2_is_the_smallest_power_of_two_not_below():
    rng = np.random.Generator(np.random.PCG64(7))
    s = (rng.random(10_000, dtype=np.float32) * np.float32(1e6) + np.float32(1e-12)).astype(np.float32)
    s[:4] = np.array([1.0, 0.5, 2.0 ** -40, 3.0], np.float32)
    r = O.round_up_pow2(s)
    bits = r.view(np.uint32)
    assert not (bits & 0x7FFFFF).any()                       # powers of two
    assert (r >= s).all() and (r < 2 * s).all()                # smallest one >= s
    np.testing.assert_array_equal(r[:4], np.array([1.0, 0.5, 2.0 ** -40, 4.0], np.float32))
    assert np.isinf(O.round_up_pow2(np.array([np.inf], np.float32))).all()


def test_ue8m0_quantisation_bounds_and_exact_scaling():
    spec = SMALL_CASES["mixed"]
    cu = np.concatenate([[0], np.cumsum(spec["counts"])]).astype(np.int64)
    meta = O.build_meta(cu)
    for name, x in case_inputs(spec).items():
        op32 = O.quantize_1x128(x, meta)
        op = O.quantize_1x128(x, meta, "ue8m0")
        np.testing.assert_array_equal(op.scales, O.round_up_pow2(op32.scales), err_msg=name)
        q = O.e4m3_decode(op.data)
        assert np.abs(q).max() <= 448.0
        # x / s with a power-of-two s is exact before the e4m3 rounding: the
        # dequantised value stays within half an e4m3 step of x
        for b in range(meta.total_blocks):
            n = int(meta.block_row_count[b])
            if n == 0:
                continue
            r0 = int(meta.block_row_start[b])
            deq = op.block_values(b, n) * op.scales[b][None, :]
            err = np.abs(deq - x[r0:r0 + n])
            assert (err <= np.abs(x[r0:r0 + n]) * 2.0 ** -4 + op.scales[b][None, :] * 2.0 ** -9).all(), name
