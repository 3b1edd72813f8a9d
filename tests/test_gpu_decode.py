"""GPU parity of the fused NVFP4 gated-delta-rule decode (gdn_decode, through
the C ABI) with the CPU oracle.

* Exactness: the codes and scales the kernel writes are the reference
  quantiser applied to the kernel's own fp32 quantiser inputs (debug_y),
  bit for bit.
* Per-step parity (teacher forced: both sides start each step from the same
  pool): outputs and quantiser inputs agree to fp32 reduction-order error;
  codes differ only where that error crosses a rounding boundary.
* SQNR gate: over 64 free-running steps the GPU's outputs and final states,
  against the unquantised f64 recurrence, are within 0.1 dB of (or better
  than) the oracle's own quantised recurrence.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128
QS = 1.0 / np.sqrt(D)


def _pool(n_slots, mode, seed=1, std=0.02):
    from gdn_b200 import NVFP4StatePool, workloads
    states = workloads.initial_states(n_slots, HV, D, std=std, seed=seed)
    pool = NVFP4StatePool.zeros(n_slots, HV, D, "cuda", scale_mode=mode)
    pool.load_fp32(states.cuda())
    return pool, states


def _snap(pool):
    return (pool.codes.cpu().numpy().copy(), pool.scales.cpu().numpy().copy(), pool.gscale.cpu().numpy().copy())


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _inputs(B, steps, seed=0):
    from gdn_b200 import workloads
    return workloads.decode_steps(B, steps, HK, HV, D, seed=seed, device="cuda")


def _gpu_step(pool, x, t, slot, debug=False):
    from gdn_b200 import ops
    y = torch.empty((slot.numel(), HV, D, D), dtype=torch.float32, device="cuda") if debug else None
    o = ops.decode(x["q"][t], x["k"][t], x["v"][t], x["g"][t], x["beta"][t], slot, pool, debug_y=y)
    torch.cuda.synchronize()
    return o, y


def _assert_same_state(y, gs, y_ref, gs_ref, gden, what=""):
    """The new states gs * y agree to fp32 reduction order.  The global scale
    is c * 2^-k with k chosen from max |S' / c|, so the two sides may pick a k
    one apart when that maximum lies within rounding of a power-of-two step;
    gs must otherwise agree to rounding and never differ by more than 2x."""
    gs = np.asarray(gs, np.float64).reshape(-1)
    gs_ref = np.asarray(gs_ref, np.float64).reshape(-1)
    ratio = gs / gs_ref
    near = np.isclose(ratio, 1.0, rtol=2e-6)
    flipped = np.isclose(ratio, 2.0, rtol=2e-6) | np.isclose(ratio, 0.5, rtol=2e-6)
    assert (near | flipped).all(), (what, ratio[~(near | flipped)][:8])
    assert flipped.mean() < 0.02, (what, flipped.mean())
    n = gs.size
    S = y.reshape(n, -1) * gs[:, None]
    S_ref = y_ref.reshape(n, -1) * gs_ref[:, None]
    tol = 2e-4 * gden * np.maximum(gs, gs_ref)[:, None]
    assert (np.abs(S - S_ref) <= tol).all(), (what, float((np.abs(S - S_ref) / tol).max()))


def _oracle_step(oracle_lib, snap, x, t, slot_np, mode):
    codes, scales, gs = (a.copy() for a in snap)
    o32, o16, y = oracle_lib.gdn_decode(_bits(x["q"][t]), _bits(x["k"][t]), _bits(x["v"][t]),
                                        x["g"][t].cpu().numpy(), x["beta"][t].cpu().numpy(), slot_np,
                                        codes, scales, gs, QS, mode, want_y=True)
    return o32, y, (codes, scales, gs)


@pytest.mark.parametrize("mode", [0, 1])
def test_pool_initialisation_bit_exact(cuda, oracle_lib, mode):
    pool, states = _pool(4, mode)
    c0, s0, g0, _ = oracle_lib.quantise_tiles(states.numpy().reshape(-1), D * D, mode)
    codes, scales, gs = _snap(pool)
    np.testing.assert_array_equal(gs.reshape(-1).view(np.uint32), g0.view(np.uint32))
    np.testing.assert_array_equal(scales.reshape(-1), s0)
    np.testing.assert_array_equal(codes.reshape(-1), c0)


@pytest.mark.parametrize("mode", [0, 1])
def test_decode_teacher_forced(cuda, oracle_lib, mode):
    B, steps = 4, 6
    pool, _ = _pool(8, mode)
    slot = torch.tensor([5, 2, 7, 0], dtype=torch.int32, device="cuda")
    slot_np = slot.cpu().numpy()
    x = _inputs(B, steps)
    for t in range(steps):
        snap = _snap(pool)
        o, y = _gpu_step(pool, x, t, slot, debug=True)
        o_ref, y_ref, (c_ref, s_ref, g_ref) = _oracle_step(oracle_lib, snap, x, t, slot_np, mode)
        codes, scales, gs = _snap(pool)
        y_np = y.cpu().numpy()
        for b in range(B):
            s = int(slot_np[b])
            # exactness: codes/scales == reference quantiser(kernel's own y)
            c2, s2 = oracle_lib.quantise(y_np[b].reshape(-1), mode)
            np.testing.assert_array_equal(codes[s].reshape(-1), c2)
            np.testing.assert_array_equal(scales[s].reshape(-1), s2)
            # y spans (gden / 2, gden]: the power-of-two global scale
            gden = 6.0 * (448.0 if mode else 240.0)
            ymax = np.abs(y_np[b]).reshape(HV, -1).max(axis=1)
            assert ((ymax > gden / 2) & (ymax <= gden)).all(), ymax
        # the new state gs' * y: the same fp32 state up to reduction order
        _assert_same_state(y_np, gs[slot_np], y_ref, g_ref[slot_np], gden, f"step {t}")
        frac = float((codes != c_ref).mean())
        assert frac < 2e-3, frac
        # outputs: bf16 rounding of the same fp32 value
        o_np = o.float().cpu().numpy()
        err = np.abs(o_np - o_ref)
        assert (err <= 6e-3 * np.abs(o_ref) + 2e-4 * np.abs(o_ref).max()).all(), err.max()
        # unused slots untouched
        for s in (1, 3, 4, 6):
            np.testing.assert_array_equal(codes[s], snap[0][s])


def _f64_reference(states0, x, slot_np, steps):
    """Unquantised f64 recurrence per (sequence, head) from the fp32 initial states."""
    from oracle import bindings as ob
    B = slot_np.size
    o = np.zeros((steps, B, HV, D))
    S_end = np.zeros((B, HV, D, D))
    q = x["q"][:steps].float().cpu().numpy()
    k = x["k"][:steps].float().cpu().numpy()
    v = x["v"][:steps].float().cpu().numpy()
    g = x["g"][:steps].cpu().numpy()
    be = x["beta"][:steps].cpu().numpy()
    for b in range(B):
        for h in range(HV):
            hk = h // (HV // HK)
            ob_, S = ob.recurrent_f64(states0[slot_np[b], h].astype(np.float64), q[:, b, hk], k[:, b, hk], v[:, b, h],
                                      g[:, b, h], be[:, b, h], QS)
            o[:, b, h] = ob_
            S_end[b, h] = S
    return o, S_end


@pytest.mark.parametrize("mode", [0, 1])
def test_sqnr_gate_64_steps(cuda, oracle_lib, mode):
    B, steps = 4, 64
    pool, states = _pool(4, mode)
    slot = torch.tensor([2, 0, 3, 1], dtype=torch.int32, device="cuda")
    slot_np = slot.cpu().numpy()
    x = _inputs(B, steps, seed=10)
    o_ref, S_ref = _f64_reference(states.numpy(), x, slot_np, steps)
    # oracle quantised trajectory
    codes, scales, gs = _snap(pool)
    o_orc = np.zeros_like(o_ref)
    for t in range(steps):
        o32, _, _ = oracle_lib.gdn_decode(_bits(x["q"][t]), _bits(x["k"][t]), _bits(x["v"][t]),
                                          x["g"][t].cpu().numpy(), x["beta"][t].cpu().numpy(), slot_np,
                                          codes, scales, gs, QS, mode)
        o_orc[t] = o32
    S_orc = oracle_lib.dequantise_tiles(codes.reshape(-1), scales.reshape(-1), gs.reshape(-1), mode).reshape(4, HV, D, D)
    # GPU quantised trajectory
    o_gpu = np.zeros_like(o_ref)
    for t in range(steps):
        o, _ = _gpu_step(pool, x, t, slot)
        o_gpu[t] = o.float().cpu().numpy()
    S_gpu = pool.dequantize().cpu().numpy()
    sq = {
        "o_oracle": oracle_lib.sqnr_db(o_ref, o_orc), "o_gpu": oracle_lib.sqnr_db(o_ref, o_gpu),
        "S_oracle": oracle_lib.sqnr_db(S_ref, S_orc[slot_np]), "S_gpu": oracle_lib.sqnr_db(S_ref, S_gpu[slot_np]),
    }
    print(f"SQNR mode {mode}: {sq}")
    assert sq["o_gpu"] >= sq["o_oracle"] - 0.1, sq
    assert sq["S_gpu"] >= sq["S_oracle"] - 0.1, sq


def test_padding_and_out_of_range_slots(cuda, oracle_lib):
    from gdn_b200 import ops
    pool, _ = _pool(4, 0)
    ops.device_status(clear=True)
    before = _snap(pool)
    slot = torch.tensor([-1, 1, 9, 3], dtype=torch.int32, device="cuda")
    x = _inputs(4, 1)
    o, _ = _gpu_step(pool, x, 0, slot)
    o_np = o.float().cpu().numpy()
    assert (o_np[0] == 0).all() and (o_np[2] == 0).all()
    assert np.abs(o_np[1]).max() > 0
    after = _snap(pool)
    for s in (0, 2):
        np.testing.assert_array_equal(after[0][s], before[0][s])
        np.testing.assert_array_equal(after[1][s], before[1][s])
    assert (after[0][1] != before[0][1]).any()
    st = ops.device_status(clear=True)
    assert st & 0x2  # GDN_STATUS_BAD_SLOT
    assert ops.device_status(clear=True) == 0


def test_strided_qkv_views(cuda):
    """q, k, v as views of one fused projection row [B, (2HK + HV) * D]."""
    from gdn_b200 import ops
    B = 8
    x = _inputs(B, 1, seed=4)
    fused = torch.cat([x["q"][0].reshape(B, -1), x["k"][0].reshape(B, -1), x["v"][0].reshape(B, -1)], dim=1)
    qv = fused[:, :HK * D].view(B, HK, D)
    kv = fused[:, HK * D:2 * HK * D].view(B, HK, D)
    vv = fused[:, 2 * HK * D:].view(B, HV, D)
    slot = torch.arange(B, dtype=torch.int32, device="cuda")
    p1, _ = _pool(B, 0)
    p2, _ = _pool(B, 0)
    o1 = ops.decode(x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot, p1)
    o2 = ops.decode(qv, kv, vv, x["g"][0], x["beta"][0], slot, p2)
    assert torch.equal(o1, o2)
    assert torch.equal(p1.codes, p2.codes) and torch.equal(p1.scales, p2.scales)
    assert torch.equal(p1.gscale, p2.gscale)


def test_deterministic_bytes(cuda):
    from gdn_b200 import ops
    B = 64
    x = _inputs(B, 1, seed=5)
    slot = torch.arange(B, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(2):
        p, _ = _pool(B, 0)
        o = ops.decode(x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot, p)
        outs.append((o.clone(), p.codes.clone(), p.scales.clone(), p.gscale.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("B", [4, 256])
def test_back_to_back_steps_on_one_pool(cuda, B):
    """Consecutive decode launches on one pool, queued back to back with no
    host synchronisation, give the same bytes as the same steps with a
    synchronisation after each.  The kernel is a programmatic dependent
    launch whose set-up overlaps the previous launch: every step must still
    read the state the previous step wrote."""
    from gdn_b200 import ops
    steps = 12
    x = _inputs(B, steps, seed=21)
    slot = torch.randperm(B, generator=torch.Generator().manual_seed(3)).to(torch.int32).cuda()
    results = []
    for sync_each in (True, False):
        p, _ = _pool(B, 1, seed=4)
        out = torch.empty((steps, B, HV, D), dtype=torch.bfloat16, device="cuda")
        for t in range(steps):
            ops.decode(x["q"][t], x["k"][t], x["v"][t], x["g"][t], x["beta"][t], slot, p, out=out[t])
            if sync_each:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        results.append((out, p.codes.clone(), p.scales.clone(), p.gscale.clone()))
    assert ops.device_status(clear=True) == 0
    for a, b in zip(*results):
        assert torch.equal(a, b)


def test_full_size_batch256_with_random_slots(cuda, oracle_lib):
    """Batch-256 decode step over a 2048-slot pool addressed through a seeded
    random permutation: bit-exact codes against the reference quantiser on
    every tile, and teacher-forced parity on 48 sampled tiles."""
    from gdn_b200 import NVFP4StatePool, ops, workloads
    B, n_slots = 256, 2048
    pool = NVFP4StatePool.zeros(n_slots, HV, D, "cuda")
    slot = workloads.slot_permutation(B, n_slots, seed=3).cuda()
    slot_np = slot.cpu().numpy()
    states = workloads.initial_states(B, HV, D, seed=7).cuda()
    pool.load_fp32(states, slot)
    x = _inputs(B, 1, seed=6)
    snap_c = pool.codes[slot.long()].cpu().numpy()
    snap_s = pool.scales[slot.long()].cpu().numpy()
    snap_g = pool.gscale[slot.long()].cpu().numpy()
    o, y = _gpu_step(pool, x, 0, slot, debug=True)
    codes = pool.codes[slot.long()].cpu().numpy()
    scales = pool.scales[slot.long()].cpu().numpy()
    y_np = y.cpu().numpy()
    c2, s2 = oracle_lib.quantise(y_np.reshape(-1), 0)
    np.testing.assert_array_equal(scales.reshape(-1), s2)
    np.testing.assert_array_equal(codes.reshape(-1), c2)
    # sampled teacher-forced parity: oracle on a compact pool of the sampled sequences
    pick = np.random.default_rng(0).choice(B, 48, replace=False)
    sub_slot = np.arange(48, dtype=np.int32)
    cc, ss, gg = snap_c[pick].copy(), snap_s[pick].copy(), snap_g[pick].copy()
    sel = torch.from_numpy(pick).cuda().long()
    o32, _, y_ref = oracle_lib.gdn_decode(_bits(x["q"][0][sel]), _bits(x["k"][0][sel]), _bits(x["v"][0][sel]),
                                          x["g"][0][sel].cpu().numpy(), x["beta"][0][sel].cpu().numpy(), sub_slot,
                                          cc, ss, gg, QS, 0, want_y=True)
    o_np = o.float().cpu().numpy()[pick]
    assert np.abs(o_np - o32).max() <= 6e-3 * np.abs(o32).max()
    gs_k = pool.gscale[slot.long()].cpu().numpy()[pick]
    _assert_same_state(y_np[pick], gs_k, y_ref, gg, 1440.0, "batch 256")
    assert float((codes[pick] != cc).mean()) < 2e-3


def test_torch_op_decode_matches_c_abi(cuda):
    from gdn_b200 import gdn_op, ops
    B = 16
    x = _inputs(B, 1, seed=8)
    slot = torch.arange(B, dtype=torch.int32, device="cuda")
    p1, _ = _pool(B, 0)
    p2, _ = _pool(B, 0)
    o1 = ops.decode(x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot, p1)
    o2 = gdn_op.decode(x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot, p2)
    assert torch.equal(o1, o2)
    assert torch.equal(p1.codes, p2.codes)


def _twin_pools(n_slots, mode, slot, seed):
    """Two pools with identical bytes: random states loaded into `slot`."""
    from gdn_b200 import NVFP4StatePool, workloads
    states = workloads.initial_states(slot.numel(), HV, D, seed=seed).cuda()
    pools = []
    for _ in range(2):
        p = NVFP4StatePool.zeros(n_slots, HV, D, "cuda", scale_mode=mode)
        p.load_fp32(states, slot)
        pools.append(p)
    return pools


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("B,n_slots", [(4, 8), (256, 2048)])
def test_production_instance_writes_the_debug_instance_bytes(cuda, mode, B, n_slots):
    """The serving kernel (no debug_y) and the instance the bit-exact tests run
    (debug_y set) write identical codes, scales, global scales and outputs,
    over two consecutive steps, so the bit-exactness shown on the debug
    instance holds for the production one."""
    from gdn_b200 import workloads
    slot = workloads.slot_permutation(B, n_slots, seed=11 + B).cuda()
    prod, dbg = _twin_pools(n_slots, mode, slot, seed=12)
    x = _inputs(B, 2, seed=13)
    for t in range(2):
        o_p, _ = _gpu_step(prod, x, t, slot, debug=False)
        o_d, _ = _gpu_step(dbg, x, t, slot, debug=True)
        assert torch.equal(o_p, o_d)
        assert torch.equal(prod.codes, dbg.codes)
        assert torch.equal(prod.scales, dbg.scales)
        assert torch.equal(prod.gscale.view(torch.int32), dbg.gscale.view(torch.int32))


@pytest.mark.parametrize("mode", [0, 1])
def test_fused_norm_instance_writes_the_plain_instance_pool_bytes(cuda, mode):
    """The fused gated-norm instance changes only the output: its pool bytes
    equal the plain (production) instance's, at batch 256 on a random map."""
    from gdn_b200 import ops, workloads
    B, n_slots = 256, 2048
    slot = workloads.slot_permutation(B, n_slots, seed=21).cuda()
    plain, normed = _twin_pools(n_slots, mode, slot, seed=22)
    x = _inputs(B, 1, seed=23)
    gen = torch.Generator().manual_seed(24)
    z = torch.randn((B, HV, D), generator=gen).to(torch.bfloat16).cuda()
    w = (1.0 + 0.1 * torch.randn(D, generator=gen)).cuda()
    args = (x["q"][0], x["k"][0], x["v"][0], x["g"][0], x["beta"][0], slot)
    ops.decode(*args, plain)
    ops.decode(*args, normed, norm_weight=w, gate_z=z)
    torch.cuda.synchronize()
    assert torch.equal(plain.codes, normed.codes)
    assert torch.equal(plain.scales, normed.scales)
    assert torch.equal(plain.gscale.view(torch.int32), normed.gscale.view(torch.int32))


@pytest.mark.parametrize("mode", [0, 1])
def test_requantiser_rare_paths(cuda, oracle_lib, mode):
    """Tiles that leave the requantiser's common path, checked bit for bit
    against the reference quantiser on the kernel's own y and against the
    oracle's new state:
      * a rank-1 term thousands of times the decayed state (strong decay,
        g = -8): max |S'/c| exceeds gden and k < 0;
      * a decayed state below 1e-30 (g = -80): dropped, S' = k w^T;
      * rows whose key entry is 0 or 1e-20 over a zero state: all-zero
        blocks and blocks whose local scale is subnormal."""
    from gdn_b200 import NVFP4StatePool, ops, workloads
    B = 2
    x = workloads.decode_steps(B, 1, HK, HV, D, seed=40, device="cuda")
    g = x["g"][0].clone()
    g[0, 0:4] = -8.0
    g[0, 4:8] = -80.0
    k = x["k"][0].clone()
    k[1, :, 0:8] = 0.0
    k[1, :, 8:16] = 1e-20
    states = workloads.initial_states(B, HV, D, seed=41)
    states[1] = 0.0
    pool = NVFP4StatePool.zeros(B, HV, D, "cuda", scale_mode=mode)
    pool.load_fp32(states.cuda())
    slot = torch.arange(B, dtype=torch.int32, device="cuda")
    snap = _snap(pool)
    y = torch.empty((B, HV, D, D), dtype=torch.float32, device="cuda")
    ops.decode(x["q"][0], k, x["v"][0], g, x["beta"][0], slot, pool, debug_y=y)
    torch.cuda.synchronize()
    codes, scales, gs = _snap(pool)
    y_np = y.cpu().numpy()
    for b in range(B):
        c2, s2 = oracle_lib.quantise(y_np[b].reshape(-1), mode)
        np.testing.assert_array_equal(codes[b].reshape(-1), c2)
        np.testing.assert_array_equal(scales[b].reshape(-1), s2)
    # the zero-state sequence really has zero blocks (scale 0x38) and tiny ones
    assert (scales[1][:, 0:8] == 0x38).any()
    c_r, s_r, g_r = (a.copy() for a in snap)
    o32, _, y_ref = oracle_lib.gdn_decode(_bits(x["q"][0]), _bits(k), _bits(x["v"][0]), g.cpu().numpy(),
                                          x["beta"][0].cpu().numpy(), slot.cpu().numpy(), c_r, s_r, g_r, QS, mode,
                                          want_y=True)
    gden = 6.0 * (448.0 if mode else 240.0)
    _assert_same_state(y_np, gs, y_ref, g_r, gden, "rare paths")
    assert ops.device_status(clear=True) == 0
