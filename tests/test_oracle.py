"""CPU tests: pin the oracle to the reference before trusting it.

1. Decode tables against the reference's unit-test golden tables
   (tests/unit/m1_intrinsics.hpp:22-58).
2. Quantiser and scale encoder against vectors produced by the reference's own
   host code (tests/golden/ref_quantise_vectors.npz, see make_golden.py) and,
   where oracle/_ref is built, against that code directly.
3. Internal consistency of the new parts (global scale, recurrent vs chunked
   forms, the decode step against an f64 recurrence).
"""
from __future__ import annotations

import json
import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _bits(x: float) -> int:
    return int(np.float32(x).view(np.uint32))


def test_ue4m3_decode_matches_reference_unit_table(oracle_lib):
    tab = json.loads((GOLDEN / "reference_decode_tables.json").read_text())["kUE4M3ExpectedBits"]
    o = oracle_lib.oracle()
    got = [_bits(o.orc_scale_decode(b, 0)) for b in range(256)]
    assert got == tab


def test_e2m1_decode_matches_reference_unit_table_where_valid(oracle_lib):
    tab = json.loads((GOLDEN / "reference_decode_tables.json").read_text())["kE2M1ExpectedBits"]
    o = oracle_lib.oracle()
    for code in list(range(0, 6)) + list(range(8, 14)):
        assert _bits(o.orc_e2m1_decode(code)) == tab[code], code
    # codes 6/7/14/15: the product decoder's standard NVFP4 values
    assert [o.orc_e2m1_decode(c) for c in (6, 7, 14, 15)] == [4.0, 6.0, -4.0, -6.0]


def test_quantise_matches_reference_golden_vectors(oracle_lib):
    g = np.load(GOLDEN / "ref_quantise_vectors.npz")
    codes, scales = oracle_lib.quantise(g["x"], 0)
    np.testing.assert_array_equal(scales, g["scales"])
    np.testing.assert_array_equal(codes, g["codes"])


def test_scale_encode_matches_reference_golden_vectors(oracle_lib):
    g = np.load(GOLDEN / "ref_quantise_vectors.npz")
    o = oracle_lib.oracle()
    got = np.array([o.orc_scale_encode(float(v), 0) for v in g["enc_in"]], np.uint8)
    np.testing.assert_array_equal(got, g["enc_out"])


def test_scale_encode_sweep_matches_compiled_reference(ref_lib):
    # every 61st bit pattern over the whole 32-bit space (70 M inputs)
    count = (1 << 32) // 61
    a = ref_lib.scale_encode_sweep(0, 61, count, 0)
    b = ref_lib.ref_scale_encode_sweep(0, 61, count)
    np.testing.assert_array_equal(a, b)


# Bit patterns of the finite non-negative floats, and of |v| <= 6.
FINITE_POS_END = 0x7F800000          # first non-finite pattern
SIX_BITS = 0x40C00000                # 6.0f
EIGHT_BITS = 0x41000000              # 8.0f


def test_block_scale_exhaustive_matches_compiled_reference(ref_lib):
    """Every finite block max |y| >= 0: the oracle's block scale byte equals the
    reference's (amax/6 through its own encoder), all 2^31 - 2^23 inputs."""
    chunk = 1 << 27
    for lo in range(0, FINITE_POS_END, chunk):
        n = min(chunk, FINITE_POS_END - lo)
        a = ref_lib.block_scale_sweep(lo, n, 0)
        b = ref_lib.ref_block_scale_sweep(lo, n)
        bad = np.nonzero(a != b)[0]
        assert bad.size == 0, [(hex(lo + int(i)), int(a[i]), int(b[i])) for i in bad[:8]]


@pytest.mark.parametrize("sign", [0, 0x80000000])
def test_e2m1_exhaustive_matches_compiled_reference(ref_lib, sign):
    """Every float with |v| <= 6 of either sign (-0 included): the oracle's
    nearest-E2M1 scan equals the reference quantiser's, bit for bit."""
    chunk = 1 << 27
    for lo in range(0, SIX_BITS + 1, chunk):
        n = min(chunk, SIX_BITS + 1 - lo)
        a = ref_lib.e2m1_sweep(sign + lo, n)
        b = ref_lib.ref_e2m1_sweep(sign + lo, n)
        bad = np.nonzero(a != b)[0]
        assert bad.size == 0, [(hex(sign + lo + int(i)), int(a[i]), int(b[i])) for i in bad[:8]]


def test_quantise_matches_compiled_reference_random(ref_lib):
    rng = np.random.default_rng(7)
    for scale in (1e-6, 0.02, 1.0, 4.0, 300.0, 1e8):
        x = (rng.standard_normal(1 << 16) * scale).astype(np.float32)
        c0, s0 = ref_lib.quantise(x, 0)
        c1, s1 = ref_lib.ref_quantise(x)
        np.testing.assert_array_equal(s0, s1)
        np.testing.assert_array_equal(c0, c1)
        np.testing.assert_array_equal(ref_lib.dequantise(c0, s0, 0).view(np.uint32),
                                      ref_lib.ref_dequantise(c1, s1).view(np.uint32))


def test_fn448_equals_ref240_below_240(oracle_lib):
    rng = np.random.default_rng(8)
    # block amax/6 < 240 for every block: |x| < 1440
    x = rng.uniform(-1439, 1439, 1 << 14).astype(np.float32)
    c0, s0 = oracle_lib.quantise(x, 0)
    c1, s1 = oracle_lib.quantise(x, 1)
    np.testing.assert_array_equal(c0, c1)
    np.testing.assert_array_equal(s0, s1)
    # above 240 the modes diverge: fn448 keeps 448 = 0x7E
    o = oracle_lib.oracle()
    assert o.orc_scale_encode(300.0, 0) == 0x77
    assert o.orc_scale_encode(300.0, 1) == 0x79  # 288 (1.125 * 2^8), round half up of 1.171875
    assert o.orc_scale_encode(1e6, 1) == 0x7E
    assert o.orc_scale_decode(0x7E, 1) == 448.0


def test_global_scale_tile_roundtrip(oracle_lib):
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(4 * 16384) * 0.02).astype(np.float32)
    for mode in (0, 1):
        codes, scales, gs, y = oracle_lib.quantise_tiles(x, 16384, mode)
        # gs = amax / (6 * sat): the largest |y| of each tile is 6 * sat
        amax = np.abs(x.reshape(4, -1)).max(axis=1)
        np.testing.assert_allclose(gs, amax / (6.0 * (448.0 if mode else 240.0)), rtol=1e-7)
        # the codes are the reference quantiser applied to y exactly
        c2, s2 = oracle_lib.quantise(y, mode)
        np.testing.assert_array_equal(codes, c2)
        np.testing.assert_array_equal(scales, s2)
        xr = oracle_lib.dequantise_tiles(codes, scales, gs, mode)
        sq = oracle_lib.sqnr_db(x, xr)
        assert sq > 17.0, sq


def test_zero_tile_gets_unit_global_scale(oracle_lib):
    codes, scales, gs, _ = oracle_lib.quantise_tiles(np.zeros(16384, np.float32), 16384, 0)
    assert gs[0] == 1.0
    assert (codes == 0).all() and (scales == 0x38).all()


def test_m3_fixture_stream_is_the_libc_stream(oracle_lib):
    # srand(42); the first S value of the d=512 case must equal glibc's first rand()
    import ctypes
    libc = ctypes.CDLL("libc.so.6")
    libc.srand(42)
    r0 = libc.rand()
    d, S, k, v = next(oracle_lib.m3_fixture((16,)))
    expect = np.float32(-4.0) + np.float32(8.0) * (np.float32(r0) / np.float32(2147483647))
    assert S[0] == expect


def test_legacy_variants_agree_within_rounding(oracle_lib):
    d, S, k, v = next(oracle_lib.m3_fixture((64,)))
    kb, vb = oracle_lib.bf16_bits(k), oracle_lib.bf16_bits(v)
    outs = [oracle_lib.legacy_update_f32(S, kb, vb, 0.9, 0.1, var) for var in range(3)]
    for o in outs[1:]:
        np.testing.assert_allclose(o, outs[0], rtol=1e-6, atol=1e-6)
    exact = 0.9 * S.astype(np.float64) + 0.1 * np.outer(oracle_lib.bf16_to_f32(kb), oracle_lib.bf16_to_f32(vb)).reshape(-1)
    np.testing.assert_allclose(outs[0], exact, rtol=1e-6, atol=1e-6)


def _token_inputs(T, D, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, D)).astype(np.float32)
    k = rng.standard_normal((T, D)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    k /= np.linalg.norm(k, axis=1, keepdims=True)
    v = rng.standard_normal((T, D)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal(T)))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal(T) + 2.0))).astype(np.float32)
    return q, k, v, g, beta


@pytest.mark.parametrize("T", [1, 63, 64, 130])
def test_chunked_form_matches_recurrence(oracle_lib, T):
    D = 128
    q, k, v, g, beta = _token_inputs(T, D, T)
    S0 = np.random.default_rng(1).standard_normal((D, D)) * 0.02
    o1, S1 = oracle_lib.recurrent_f64(S0, q, k, v, g, beta, 1 / np.sqrt(D))
    o2, S2 = oracle_lib.chunked_f64(S0, q, k, v, g, beta, 1 / np.sqrt(D), 64)
    np.testing.assert_allclose(o2, o1, rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(S2, S1, rtol=1e-9, atol=1e-11)


def test_chunked_form_with_weak_decay(oracle_lib):
    # g close to 0 keeps the whole chunk coupled (the hard case for the WY form)
    D, T = 128, 128
    q, k, v, g, beta = _token_inputs(T, D, 5)
    g = (g * 0.01).astype(np.float32)
    S0 = np.zeros((D, D))
    o1, S1 = oracle_lib.recurrent_f64(S0, q, k, v, g, beta, 1 / np.sqrt(D))
    o2, S2 = oracle_lib.chunked_f64(S0, q, k, v, g, beta, 1 / np.sqrt(D), 64)
    np.testing.assert_allclose(o2, o1, rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(S2, S1, rtol=1e-8, atol=1e-10)


def test_decode_step_matches_f64_recurrence(oracle_lib):
    B, HK, HV, D = 2, 2, 4, 128
    rng = np.random.default_rng(3)
    states = (rng.standard_normal((3, HV, D, D)) * 0.02).astype(np.float32)
    codes, scales, gs, _ = oracle_lib.quantise_tiles(states.reshape(-1), D * D, 0)
    codes = codes.reshape(3, HV, D, D // 2).copy()
    scales = scales.reshape(3, HV, D, D // 16).copy()
    gs = gs.reshape(3, HV).copy()
    S_deq = oracle_lib.dequantise_tiles(codes.reshape(-1), scales.reshape(-1), gs.reshape(-1), 0).reshape(3, HV, D, D)
    qf = rng.standard_normal((B, HK, D)).astype(np.float32)
    kf = rng.standard_normal((B, HK, D)).astype(np.float32)
    qf /= np.linalg.norm(qf, axis=-1, keepdims=True)
    kf /= np.linalg.norm(kf, axis=-1, keepdims=True)
    vf = rng.standard_normal((B, HV, D)).astype(np.float32)
    q, k, v = oracle_lib.bf16_bits(qf), oracle_lib.bf16_bits(kf), oracle_lib.bf16_bits(vf)
    g = (-np.log1p(np.exp(rng.standard_normal((B, HV)) + 2))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, HV))))).astype(np.float32)
    slot = np.array([2, -1], np.int32)
    codes0 = codes.copy()
    o32, o16, y = oracle_lib.gdn_decode(q, k, v, g, beta, slot, codes, scales, gs, 1 / np.sqrt(D), want_y=True)
    for h in range(HV):
        hk = h // (HV // HK)
        o_ref, S_ref = oracle_lib.recurrent_f64(
            S_deq[2, h].astype(np.float64), oracle_lib.bf16_to_f32(q[0, hk])[None], oracle_lib.bf16_to_f32(k[0, hk])[None],
            oracle_lib.bf16_to_f32(v[0, h])[None], g[0, h:h + 1], beta[0, h:h + 1], 1 / np.sqrt(D))
        np.testing.assert_allclose(o32[0, h], o_ref[0], rtol=1e-5, atol=1e-6)
        # the new tile is the reference quantiser applied to y
        c2, s2 = oracle_lib.quantise(y[0, h], 0)
        np.testing.assert_array_equal(codes[2, h].reshape(-1), c2)
    # padding sequence: zero output, its (unused) slot untouched
    assert (o32[1] == 0).all()
    np.testing.assert_array_equal(codes[0], codes0[0])
    np.testing.assert_array_equal(codes[1], codes0[1])
