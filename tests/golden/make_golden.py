"""Regenerates the committed golden fixtures in tests/golden/.

Run in a checkout that has the reference (bojak83318/blackwell-kernel-sm_120)
at $GDN_REFERENCE_DIR (default: a checkout named `reference` beside this
repository) and the oracle built
(`make -C oracle && make -C oracle ref`):

    python tests/golden/make_golden.py

Writes:
  reference_decode_tables.json  the E2M1 and UE4M3 decode bit tables of the
                                reference's unit test, parsed from
                                tests/unit/m1_intrinsics.hpp:22-58
  ref_quantise_vectors.npz      inputs and the outputs of the reference's own
                                nvfp4_quantise_host (gdn_state_update_ref.cu:93-141)
                                and encode_f32_to_ue4m3 (gdn_fp4_intrinsics.cuh:71-123),
                                compiled from its sources into oracle/_ref
"""
from __future__ import annotations

import json
import os
import pathlib
import re
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import bindings as ob  # noqa: E402


def parse_tables(ref_dir: pathlib.Path) -> dict:
    text = (ref_dir / "tests" / "unit" / "m1_intrinsics.hpp").read_text()
    out = {}
    for name in ("kE2M1ExpectedBits", "kUE4M3ExpectedBits"):
        m = re.search(name + r"\s*=\s*\{(.*?)\};", text, re.S)
        vals = [int(v, 16) for v in re.findall(r"0x([0-9a-fA-F]+)u", m.group(1))]
        out[name] = vals
    assert len(out["kE2M1ExpectedBits"]) == 16 and len(out["kUE4M3ExpectedBits"]) == 256
    return out


def edge_blocks() -> np.ndarray:
    """Blocks of 16 aimed at every rounding rule of the reference quantiser."""
    blocks = []
    mags = np.array([0, .25, .5, .75, 1, 1.25, 1.5, 1.75, 2, 2.5, 3, 3.5, 4, 5, 6, 7], np.float32)
    for s in (1.0, 2.0 ** -8, 2.0 ** -12, 2.0 ** -20, 3.0, 240.0 / 6, 1000.0, 1e6, 1e10, 1e30):
        blocks.append(mags * np.float32(s))
        blocks.append(-mags * np.float32(s))
    # exact E2M1 midpoints relative to a power-of-two scale (ties)
    blocks.append(np.array([6, .25, .75, 1.25, 1.75, 2.5, 3.5, 5, -.25, -.75, -1.25, -1.75, -2.5, -3.5, -5, 0],
                           np.float32))
    # neighbours of midpoints (one ulp either side)
    mid = np.array([.25, .75, 1.25, 1.75, 2.5, 3.5, 5, 6], np.float32)
    up = np.nextafter(mid, np.float32(np.inf))
    dn = np.nextafter(mid, np.float32(0))
    blocks.append(np.concatenate([up, dn]))
    # zero block, negative zeros, tiny values, subnormal scales
    blocks.append(np.zeros(16, np.float32))
    blocks.append(-np.zeros(16, np.float32))
    blocks.append(np.full(16, 1e-40, np.float32) * np.arange(16, dtype=np.float32))
    blocks.append(np.linspace(0, 0.0936, 16, dtype=np.float32))
    # block amax in the [1.875, 2) significand band of amax/6
    for e in range(-6, 8):
        blocks.append(np.linspace(-1, 1, 16, dtype=np.float32) * np.float32(6 * 1.9 * 2.0 ** e))
    # saturation at 240 and far beyond
    blocks.append(np.linspace(0, 32000, 16, dtype=np.float32))
    # non-finite values
    b = np.linspace(-3, 3, 16, dtype=np.float32)
    b[3] = np.nan
    blocks.append(b.copy())
    b[7] = np.inf
    blocks.append(b.copy())
    b = np.linspace(-3, 3, 16, dtype=np.float32)
    b[0] = -np.inf
    blocks.append(b)
    return np.concatenate(blocks).astype(np.float32)


def main() -> None:
    ref_dir = pathlib.Path(os.environ.get("GDN_REFERENCE_DIR", HERE.parents[2] / "reference"))
    tables = parse_tables(ref_dir)
    tables["source"] = "tests/unit/m1_intrinsics.hpp:22-58 of bojak83318/blackwell-kernel-sm_120"
    tables["note"] = ("E2M1 entries 6, 7, 14, 15 of the unit test decode to inf/NaN; the product decoder "
                      "(src/intrinsics/gdn_fp4_intrinsics.cuh:27-45) gives 4 and 6, so only codes 0-5 and 8-13 "
                      "pin the decoder.")
    (HERE / "reference_decode_tables.json").write_text(json.dumps(tables, indent=1))

    rng = np.random.default_rng(20250101)
    parts = [
        edge_blocks(),
        rng.standard_normal(4096).astype(np.float32),
        (rng.standard_normal(2048) * 0.02).astype(np.float32),
        rng.uniform(-4, 4, 2048).astype(np.float32),
        (rng.standard_normal(1024) * np.exp(rng.uniform(-30, 30, 1024))).astype(np.float32),
    ]
    x = np.concatenate(parts).astype(np.float32)
    x = x[: x.size // 16 * 16]
    codes, scales = ob.ref_quantise(x)

    # scale-encoder inputs: every boundary neighbourhood plus a log-uniform spread
    enc_in = [np.float32(v) for v in (0, -1, np.inf, -np.inf, np.nan, 240, 239.99, 448, 2 ** -6, 2 ** -9, 2 ** -10)]
    for e in range(-12, 10):
        for m in np.arange(8, 16) / 8.0:
            base = np.float32(m * 2.0 ** e)
            for c in (base, np.nextafter(base, np.float32(0)), np.nextafter(base, np.float32(np.inf)),
                      np.float32(base * (1 + 1 / 16)), np.float32(base * (1 + 1 / 32))):
                enc_in.append(np.float32(c))
    enc_in = np.concatenate([np.array(enc_in, np.float32),
                             np.exp(rng.uniform(-25, 8, 8192)).astype(np.float32)])
    enc_out = np.array([ob.ref().ref_encode_ue4m3(float(v)) for v in enc_in], np.uint8)
    np.savez_compressed(HERE / "ref_quantise_vectors.npz", x=x, codes=codes, scales=scales,
                        enc_in=enc_in, enc_out=enc_out)
    print(f"wrote {x.size} quantiser inputs and {enc_in.size} scale-encoder inputs")


if __name__ == "__main__":
    main()
