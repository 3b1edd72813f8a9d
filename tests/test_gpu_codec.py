"""GPU parity of the NVFP4 codec kernels (through the C ABI) with the
reference quantiser: bit-exact codes and scales on identical fp32 inputs."""
from __future__ import annotations

import pathlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _q(x_np, mode=0):
    from gdn_b200 import ops
    c, s = ops.nvfp4_quantize(torch.from_numpy(x_np).cuda(), mode)
    torch.cuda.synchronize()
    return c.cpu().numpy(), s.cpu().numpy()


def test_quantize_matches_reference_golden_vectors(cuda):
    g = np.load(GOLDEN / "ref_quantise_vectors.npz")
    c, s = _q(g["x"], 0)
    np.testing.assert_array_equal(s, g["scales"])
    np.testing.assert_array_equal(c, g["codes"])


@pytest.mark.parametrize("mode", [0, 1])
def test_quantize_matches_oracle_random(cuda, oracle_lib, mode):
    rng = np.random.default_rng(11 + mode)
    parts = [(rng.standard_normal(1 << 18) * s).astype(np.float32) for s in (1e-7, 0.02, 1.0, 50.0, 3e3, 1e9)]
    x = np.concatenate(parts)
    c, s = _q(x, mode)
    c0, s0 = oracle_lib.quantise(x, mode)
    np.testing.assert_array_equal(s, s0)
    np.testing.assert_array_equal(c, c0)


def _threshold_codes(a: np.ndarray) -> np.ndarray:
    # number of E2M1 midpoints strictly below |a| (ties keep the smaller magnitude)
    t = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    return np.searchsorted(t, a, side="left").astype(np.uint8)


def test_e2m1_fast_path_sweep(cuda):
    """Every 61st float in [0, 6] plus +-4 ulps around each midpoint, through the
    hardware converter: blocks carry 6.0 in element 0 so the block scale is
    exactly 1.0 (amax/6 = 1 -> 0x38)."""
    lo = np.float32(0).view(np.uint32)
    hi = np.float32(6.0).view(np.uint32)
    sweep = np.arange(lo, hi + 1, 61, dtype=np.uint32).view(np.float32)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32).view(np.uint32)
    near = (mids[:, None].astype(np.int64) + np.arange(-4, 5)[None, :]).reshape(-1).astype(np.uint32).view(np.float32)
    vals = np.concatenate([sweep, near, -sweep, -near])
    n15 = (vals.size + 14) // 15
    vals = np.concatenate([vals, np.zeros(n15 * 15 - vals.size, np.float32)]).reshape(n15, 15)
    x = np.concatenate([np.full((n15, 1), 6.0, np.float32), vals], axis=1).reshape(-1)
    c, s = _q(x, 0)
    assert (s == 0x38).all()
    nib = np.stack([c & 0xF, c >> 4], axis=1).reshape(n15, 16)[:, 1:].reshape(-1)
    a = vals.reshape(-1)
    expect = _threshold_codes(np.abs(a)) | np.where(a < 0, 8, 0).astype(np.uint8)
    bad = np.nonzero(nib != expect)[0]
    assert bad.size == 0, [(float(a[i]), int(nib[i]), int(expect[i])) for i in bad[:10]]


def test_e2m1_signs_and_zeros(cuda):
    x = np.array([6.0, -0.0, 0.0, -1e-30, -1e-40, 1e-40, -0.1, 0.1, -0.25, 0.25, -0.26, 0.26, -6.0, 5.0, -5.0,
                  -0.75], np.float32)
    c, s = _q(x, 0)
    c0, s0 = _q_oracle(x)
    np.testing.assert_array_equal(s, s0)
    np.testing.assert_array_equal(c, c0)


def _q_oracle(x):
    from oracle import bindings
    return bindings.quantise(x, 0)


def test_non_finite_and_huge_blocks(cuda, oracle_lib):
    g = np.load(GOLDEN / "ref_quantise_vectors.npz")
    x = g["x"][:2048]
    rng = np.random.default_rng(5)
    huge = (rng.standard_normal(4096) * 1e12).astype(np.float32)
    huge[::97] = np.float32(3e38)
    y = np.concatenate([x, huge])
    c, s = _q(y, 0)
    c0, s0 = oracle_lib.quantise(y, 0)
    np.testing.assert_array_equal(s, s0)
    np.testing.assert_array_equal(c, c0)


@pytest.mark.parametrize("mode", [0, 1])
def test_dequantize_bit_exact(cuda, oracle_lib, mode):
    from gdn_b200 import ops
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 256, 1 << 16, dtype=np.uint8)
    scales = rng.integers(0, 256, 1 << 13, dtype=np.uint8)
    out = ops.nvfp4_dequantize(torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda(), mode).cpu().numpy()
    ref = oracle_lib.dequantise(codes, scales, mode)
    # NaN scale codes give NaN either way; the payload bits of a NaN carry no value
    np.testing.assert_array_equal(np.isnan(out), np.isnan(ref))
    ok = ~np.isnan(ref)
    np.testing.assert_array_equal(out[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_dequantize_matches_compiled_reference(cuda, ref_lib):
    from gdn_b200 import ops
    rng = np.random.default_rng(4)
    codes = rng.integers(0, 256, 1 << 16, dtype=np.uint8)
    scales = rng.integers(0, 0x78, 1 << 13, dtype=np.uint8)
    out = ops.nvfp4_dequantize(torch.from_numpy(codes).cuda(), torch.from_numpy(scales).cuda(), 0).cpu().numpy()
    np.testing.assert_array_equal(out.view(np.uint32), ref_lib.ref_dequantise(codes, scales).view(np.uint32))


@pytest.mark.parametrize("mode", [0, 1])
def test_quantize_tiles_matches_oracle(cuda, oracle_lib, mode):
    from gdn_b200 import ops
    rng = np.random.default_rng(6)
    x = (rng.standard_normal(16 * 16384) * 0.02).astype(np.float32)
    x[5 * 16384:6 * 16384] = 0.0  # an all-zero tile
    codes, scales, gs = ops.nvfp4_quantize_tiles(torch.from_numpy(x).cuda(), 16384, mode)
    c0, s0, g0, _ = oracle_lib.quantise_tiles(x, 16384, mode)
    np.testing.assert_array_equal(gs.cpu().numpy().view(np.uint32), g0.view(np.uint32))
    np.testing.assert_array_equal(scales.cpu().numpy(), s0)
    np.testing.assert_array_equal(codes.cpu().numpy(), c0)
    back = ops.nvfp4_dequantize_tiles(codes, scales, gs, mode).cpu().numpy()
    np.testing.assert_array_equal(back.view(np.uint32),
                                  oracle_lib.dequantise_tiles(c0, s0, g0, mode).view(np.uint32))


def test_quantize_tiles_full_size_sampled_parity(cuda, oracle_lib):
    """Full pool size (256 slots x 32 heads of N(0, 0.02) states): 64 sampled
    tiles bit-exact with the oracle, and the round trip keeps SQNR > 17 dB on
    every tile.  (Requantising a dequantised tile is not an identity for the
    reference codec: a decoded scale of significand 1.875 re-encodes one binade
    up, gdn_fp4_intrinsics.cuh:97-100.)"""
    from gdn_b200 import ops
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    nt = 256 * 32
    x = torch.randn(nt * 16384, device="cuda", generator=gen) * 0.02
    c, s, g = ops.nvfp4_quantize_tiles(x, 16384)
    y = ops.nvfp4_dequantize_tiles(c, s, g)
    err = (y - x).view(nt, -1).pow(2).sum(1)
    sig = x.view(nt, -1).pow(2).sum(1)
    sqnr = 10 * torch.log10(sig / err)
    assert float(sqnr.min()) > 17.0
    pick = np.random.default_rng(1).choice(nt, 64, replace=False)
    xs = x.view(nt, -1)[pick].cpu().numpy()
    c0, s0, g0, _ = oracle_lib.quantise_tiles(xs.reshape(-1), 16384, 0)
    np.testing.assert_array_equal(c.view(nt, -1)[pick].cpu().numpy().reshape(-1), c0)
    np.testing.assert_array_equal(s.view(nt, -1)[pick].cpu().numpy().reshape(-1), s0)
    np.testing.assert_array_equal(g[pick].cpu().numpy(), g0)
