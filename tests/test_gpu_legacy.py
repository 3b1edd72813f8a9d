"""GPU parity of the legacy op (launch_gdn_state_update, launch_gdn_ref and
torch.ops.gdn_sm120.state_update) with the reference's own op path, compiled
from its sources (oracle/_ref/libgdn_ref.so) and run on the same GPU, on the
reference's M3 gate inputs (tests/test_gdn_correctness.cu:199-218 of the
reference: srand(42); d = 512, 1024, 2048; (alpha, beta) = (.9, .1),
(.8, .2), (.95, .05))."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

M3_CASES = ((512, 0.9, 0.1), (1024, 0.8, 0.2), (2048, 0.95, 0.05))


def _m3_inputs(oracle_lib):
    out = []
    for (d, S, k, v), (d2, a, b) in zip(oracle_lib.m3_fixture(tuple(c[0] for c in M3_CASES)), M3_CASES):
        assert d == d2
        sd, ss = oracle_lib.quantise(S, 0)  # == the reference quantiser (tests/test_oracle.py)
        out.append((d, a, b, sd, ss, oracle_lib.bf16_bits(k), oracle_lib.bf16_bits(v)))
    return out


def _dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:  # bf16 bit patterns travel as int16
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


def _ref_op(ref_lib, sd, ss, kb, vb, a, b, d):
    """The reference's launch_gdn_state_update (GPU kernel + host quantiser)."""
    S_data, S_scales, k, v = _dev(sd), _dev(ss), _dev(kb), _dev(vb)
    od = torch.empty_like(S_data)
    os_ = torch.empty_like(S_scales)
    torch.cuda.synchronize()
    rc = ref_lib.ref().launch_gdn_state_update(S_data.data_ptr(), S_scales.data_ptr(), k.data_ptr(), v.data_ptr(),
                                               od.data_ptr(), os_.data_ptr(), a, b, d, None)
    torch.cuda.synchronize()
    assert rc == 0
    return od.cpu().numpy(), os_.cpu().numpy()


def _ref_f32(ref_lib, sd, ss, kb, vb, a, b, d):
    S_data, S_scales, k, v = _dev(sd), _dev(ss), _dev(kb), _dev(vb)
    out = torch.empty(d * d, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ref_lib.ref().launch_gdn_ref(S_data.data_ptr(), S_scales.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                 a, b, d, None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _ours(sd, ss, kb, vb, a, b, d, rounding=None):
    from gdn_b200 import ops
    od, os_ = ops.legacy_state_update(_dev(sd), _dev(ss), _dev(kb).view(torch.bfloat16),
                                      _dev(vb).view(torch.bfloat16), a, b, d, rounding=rounding)
    torch.cuda.synchronize()
    return od.cpu().numpy(), os_.cpu().numpy()


def test_default_rounding_matches_reference_binary_fp32(cuda, ref_lib, oracle_lib):
    """launch_gdn_ref: our fused kernel equals the reference's two kernels bit
    for bit.  The rounding the reference entry points use is the one its
    compiled line uses; the per-call variants show that the comparison can
    tell the three roundings apart."""
    from gdn_b200 import ops
    d, a, b, sd, ss, kb, vb = _m3_inputs(oracle_lib)[0]
    ref = _ref_f32(ref_lib, sd, ss, kb, vb, a, b, d)
    args = (_dev(sd), _dev(ss), _dev(kb).view(torch.bfloat16), _dev(vb).view(torch.bfloat16), a, b, d)
    mismatch = {}
    for var in range(3):
        out = ops.legacy_ref_update(*args, rounding=var).cpu().numpy()
        mismatch[var] = int((out.view(np.uint32) != ref.view(np.uint32)).sum())
    default = ops.legacy_ref_update(*args).cpu().numpy()
    assert np.array_equal(default.view(np.uint32), ref.view(np.uint32))
    assert mismatch[ops.LEGACY_REFERENCE_ROUNDING] == 0, mismatch
    assert sum(1 for m in mismatch.values() if m == 0) == 1, f"variants indistinguishable: {mismatch}"


def test_per_call_rounding_leaves_reference_entry_unchanged(cuda, oracle_lib):
    """A call with another rounding changes nothing for later default calls:
    there is no process-wide rounding state."""
    from gdn_b200 import ops
    d, a, b, sd, ss, kb, vb = _m3_inputs(oracle_lib)[0]
    before = _ours(sd, ss, kb, vb, a, b, d)
    for var in (0, 2):
        _ours(sd, ss, kb, vb, a, b, d, rounding=var)
    after = _ours(sd, ss, kb, vb, a, b, d)
    for x, y in zip(before, after):
        np.testing.assert_array_equal(x, y)
    ref = _ours(sd, ss, kb, vb, a, b, d, rounding=ops.LEGACY_REFERENCE_ROUNDING)
    for x, y in zip(before, ref):
        np.testing.assert_array_equal(x, y)
    with pytest.raises(Exception):
        _ours(sd, ss, kb, vb, a, b, d, rounding=3)


@pytest.mark.parametrize("case", range(3))
def test_state_update_bytes_equal_reference_op(cuda, ref_lib, oracle_lib, case):
    d, a, b, sd, ss, kb, vb = _m3_inputs(oracle_lib)[case]
    rd, rs = _ref_op(ref_lib, sd, ss, kb, vb, a, b, d)
    od, os_ = _ours(sd, ss, kb, vb, a, b, d)
    np.testing.assert_array_equal(os_, rs)
    np.testing.assert_array_equal(od, rd)
    # the reference's own gate metric (max relative error <= 5%) holds trivially
    ours = oracle_lib.dequantise(od, os_)
    refq = oracle_lib.dequantise(rd, rs)
    rel = np.abs(ours - refq) / np.maximum(np.abs(refq), 1e-6)
    assert rel.max() <= 0.05


@pytest.mark.parametrize("d", [4, 12, 16, 48])
def test_small_and_unaligned_d(cuda, ref_lib, oracle_lib, d):
    """d % 16 != 0 (blocks straddle rows) and tiny states, against the reference op."""
    rng = np.random.default_rng(d)
    S = rng.uniform(-4, 4, d * d).astype(np.float32)
    sd, ss = oracle_lib.quantise(S, 0)
    kb = oracle_lib.bf16_bits(rng.uniform(-1, 1, d).astype(np.float32))
    vb = oracle_lib.bf16_bits(rng.uniform(-1, 1, d).astype(np.float32))
    rd, rs = _ref_op(ref_lib, sd, ss, kb, vb, 0.9, 0.1, d)
    od, os_ = _ours(sd, ss, kb, vb, 0.9, 0.1, d)
    np.testing.assert_array_equal(os_, rs)
    np.testing.assert_array_equal(od, rd)


def test_in_place_update(cuda, oracle_lib):
    from gdn_b200 import ops
    d, a, b, sd, ss, kb, vb = _m3_inputs(oracle_lib)[0]
    expect_d, expect_s = _ours(sd, ss, kb, vb, a, b, d)
    S_data, S_scales = _dev(sd), _dev(ss)
    ops.legacy_state_update(S_data, S_scales, _dev(kb).view(torch.bfloat16), _dev(vb).view(torch.bfloat16), a, b, d,
                            out=(S_data, S_scales))
    np.testing.assert_array_equal(S_data.cpu().numpy(), expect_d)
    np.testing.assert_array_equal(S_scales.cpu().numpy(), expect_s)


def test_torch_op_matches_c_abi(cuda, oracle_lib):
    from gdn_b200 import gdn_op
    gdn_op.load_gdn_op()
    d, a, b, sd, ss, kb, vb = _m3_inputs(oracle_lib)[1]
    od, os_ = torch.ops.gdn_sm120.state_update(_dev(sd), _dev(ss), _dev(kb).view(torch.bfloat16),
                                               _dev(vb).view(torch.bfloat16), a, b, d)
    ed, es = _ours(sd, ss, kb, vb, a, b, d)
    np.testing.assert_array_equal(od.cpu().numpy(), ed)
    np.testing.assert_array_equal(os_.cpu().numpy(), es)
    # shapes and dtypes of the reference op (tests/test_vllm_integration.py:180-196)
    assert od.shape == (d * d // 2,) and os_.shape == (d * d // 16,)
    assert od.dtype == torch.uint8 and os_.dtype == torch.uint8


def test_torch_op_rejects_bad_inputs(cuda):
    from gdn_b200 import gdn_op
    gdn_op.load_gdn_op()
    d = 32
    S = torch.zeros(d * d // 2, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(d * d // 16, dtype=torch.uint8, device="cuda")
    k = torch.zeros(d, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        torch.ops.gdn_sm120.state_update(S, sc, k.float(), k, 0.9, 0.1, d)
    with pytest.raises(RuntimeError):
        torch.ops.gdn_sm120.state_update(S[:-1], sc, k, k, 0.9, 0.1, d)
    with pytest.raises(RuntimeError):
        torch.ops.gdn_sm120.state_update(S.cpu(), sc, k, k, 0.9, 0.1, d)
