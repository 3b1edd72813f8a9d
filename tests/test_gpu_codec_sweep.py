"""Exhaustive GPU sweeps of the production codec paths against the reference.

The requantisers of the decode, prefill and codec kernels build every code
byte from two device functions: the block scale byte of a 16-element block
(block_scale_code: amax/6 through the reference's scale-encoder rules) and
the E2M1 encoder of y * inv (e2m1_encode8: hardware round-to-nearest-even
corrected to the reference's ties-to-the-smaller-magnitude rule).
gdn_b200_selftest_codec runs those same functions over consecutive fp32 bit
patterns, and these tests compare every finite input with:
  * the reference's own code from oracle/_ref (its encoder on amax/6, and its
    nvfp4_quantise_host for E2M1), in the reference's scale mode;
  * the oracle (itself pinned exhaustively to the reference by
    tests/test_oracle.py) for the E4M3FN-range mode and for |v| in (6, 8),
    where the reference quantiser cannot be driven at inverse scale 1.
Reference: src/kernel/gdn_state_update_ref.cu:93-141,
src/intrinsics/gdn_fp4_intrinsics.cuh:71-123.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FINITE_POS_END = 0x7F800000   # first non-finite bit pattern
SIX_BITS = 0x40C00000         # 6.0f
EIGHT_BITS = 0x41000000       # 8.0f
CHUNK = 1 << 27


def _gpu(which: int, lo: int, n: int, mode: int = 0) -> np.ndarray:
    from gdn_b200 import ops
    out = ops.codec_selftest(which, lo, n, mode)
    return out.cpu().numpy()


def _check(lo: int, got: np.ndarray, want: np.ndarray, what: str) -> None:
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (what, [(hex(lo + int(i)), int(got[i]), int(want[i])) for i in bad[:8]])


def test_block_scale_code_every_finite_amax_matches_reference(cuda, ref_lib):
    """All 2^31 - 2^23 finite block maxima >= 0 (0 included), reference scale mode."""
    for lo in range(0, FINITE_POS_END, CHUNK):
        n = min(CHUNK, FINITE_POS_END - lo)
        _check(lo, _gpu(0, lo, n, 0), ref_lib.ref_block_scale_sweep(lo, n), "scale ref240")


def test_block_scale_code_every_finite_amax_fn448(cuda, oracle_lib):
    """The same sweep in the E4M3FN-range mode, against the oracle."""
    for lo in range(0, FINITE_POS_END, CHUNK):
        n = min(CHUNK, FINITE_POS_END - lo)
        _check(lo, _gpu(0, lo, n, 1), oracle_lib.block_scale_sweep(lo, n, 1), "scale fn448")


@pytest.mark.parametrize("sign", [0, 0x80000000])
def test_e2m1_encoder_every_value_up_to_6_matches_reference(cuda, ref_lib, sign):
    """Every fp32 v with |v| <= 6 (either sign, -0 included) at inverse scale 1:
    the nibble equals the reference quantiser's."""
    for lo in range(0, SIX_BITS + 1, CHUNK):
        n = min(CHUNK, SIX_BITS + 1 - lo)
        _check(sign + lo, _gpu(1, sign + lo, n), ref_lib.ref_e2m1_sweep(sign + lo, n), "e2m1")


@pytest.mark.parametrize("sign", [0, 0x80000000])
def test_e2m1_encoder_6_to_8_saturates_like_reference(cuda, oracle_lib, sign):
    """6 < |v| < 8: the reference scan gives magnitude code 7 (|a - 6| < |a - 4|);
    checked against the oracle's restatement of that scan."""
    lo, n = sign + SIX_BITS + 1, EIGHT_BITS - SIX_BITS - 1
    got = _gpu(1, lo, n)
    _check(lo, got, oracle_lib.e2m1_sweep(lo, n), "e2m1 (6, 8)")
    assert (got & 7 == 7).all()
