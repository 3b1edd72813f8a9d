"""GPU parity of the chunked NVFP4 gated-delta-rule prefill (gdn_prefill,
through the C ABI) with the CPU oracle.

* Outputs and final fp32 states follow the unquantised f64 recurrence of the
  oracle (token by token, oracle/gdn_oracle.c orc_gdn_recurrent_f64) within
  the tolerance of the kernel's arithmetic (bf16 inputs and outputs, bf16
  chunk operands, tf32 state products): per (sequence, head)
  ||o - o_ref|| <= 1e-2 ||o_ref|| and max |o - o_ref| <= 4e-2 max |o_ref|.
* Exactness of the state write: the codes and scales stored in the pool are
  the reference quantiser applied to the kernel's own fp32 quantiser inputs
  (debug_y), bit for bit, and the global scale is amax / gden.
* Edge cases: one-token and partial chunks, empty sequences, chunk
  boundaries, zero and pool initial states, padding and out-of-range slots,
  invalid cu_seqlens, strided q/k/v views, determinism.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128
QS = 1.0 / np.sqrt(D)
O_NORM_TOL = 1e-2
O_MAX_TOL = 4e-2
S_NORM_TOL = 1e-2


def _inputs(lengths, seed=0):
    from gdn_b200 import workloads
    x = workloads.token_inputs(int(sum(lengths)), HK, HV, D, seed=seed, device="cuda")
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    return x, cu


def _pool(n_slots, mode, seed=1, std=0.02):
    from gdn_b200 import NVFP4StatePool, workloads
    states = workloads.initial_states(n_slots, HV, D, std=std, seed=seed)
    pool = NVFP4StatePool.zeros(n_slots, HV, D, "cuda", scale_mode=mode)
    pool.load_fp32(states.cuda())
    return pool


def _snap(pool):
    return (pool.codes.cpu().numpy().copy(), pool.scales.cpu().numpy().copy(), pool.gscale.cpu().numpy().copy())


def _run(x, cu, pool=None, slots=None, has=None, debug=False):
    from gdn_b200 import ops
    N = len(cu) - 1
    cu_t = torch.from_numpy(cu).cuda()
    slot_t = None if slots is None else torch.tensor(slots, dtype=torch.int32, device="cuda")
    has_t = None if has is None else torch.tensor(has, dtype=torch.bool, device="cuda")
    y = torch.full((N, HV, D, D), float("nan"), dtype=torch.float32, device="cuda") if debug else None
    o = ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu_t, pool=pool, slot_idx=slot_t,
                    has_initial_state=has_t, debug_y=y)
    torch.cuda.synchronize()
    return o, y


def _reference(x, cu, S0=None):
    """f64 recurrence per (sequence, head).  S0: [N, HV, D, D] initial states or None."""
    from oracle import bindings as ob
    q = x["q"].float().cpu().numpy()
    k = x["k"].float().cpu().numpy()
    v = x["v"].float().cpu().numpy()
    g = x["g"].cpu().numpy()
    be = x["beta"].cpu().numpy()
    N = len(cu) - 1
    o = np.zeros((int(cu[-1]), HV, D))
    S = np.zeros((N, HV, D, D))
    for n in range(N):
        b0, b1 = int(cu[n]), int(cu[n + 1])
        for h in range(HV):
            hk = h // (HV // HK)
            s0 = np.zeros((D, D)) if S0 is None else S0[n, h].astype(np.float64)
            if b1 == b0:
                S[n, h] = s0
                continue
            o[b0:b1, h], S[n, h] = ob.recurrent_f64(s0, q[b0:b1, hk], k[b0:b1, hk], v[b0:b1, h], g[b0:b1, h],
                                                   be[b0:b1, h], QS)
    return o, S


def _check_outputs(o_gpu, o_ref, cu):
    o = o_gpu.float().cpu().numpy()
    worst = (0.0, 0.0)
    for n in range(len(cu) - 1):
        b0, b1 = int(cu[n]), int(cu[n + 1])
        for h in range(HV):
            ref = o_ref[b0:b1, h]
            if ref.size == 0:
                continue
            err = o[b0:b1, h] - ref
            rel = np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30)
            mx = np.abs(err).max() / max(np.abs(ref).max(), 1e-30)
            worst = (max(worst[0], rel), max(worst[1], mx))
    assert worst[0] <= O_NORM_TOL and worst[1] <= O_MAX_TOL, worst
    return worst


def test_prefill_zero_state_varlen(cuda):
    lengths = [1, 81, 130, 64, 63, 65]
    x, cu = _inputs(lengths, seed=3)
    o, _ = _run(x, cu)
    o_ref, _ = _reference(x, cu)
    print("zero-state worst (norm, max):", _check_outputs(o, o_ref, cu))


@pytest.mark.parametrize("mode", [0, 1])
def test_prefill_pool_state(cuda, oracle_lib, mode):
    lengths = [70, 1, 128, 200, 0]
    slots = [5, 2, 7, 0, 3]
    has = [True, False, True, True, True]
    x, cu = _inputs(lengths, seed=5)
    pool = _pool(8, mode)
    before = _snap(pool)
    S_pool = oracle_lib.dequantise_tiles(before[0].reshape(-1), before[1].reshape(-1), before[2].reshape(-1),
                                         mode).reshape(8, HV, D, D)
    S0 = np.stack([S_pool[s] if hv else np.zeros((HV, D, D), np.float32) for s, hv in zip(slots, has)])
    o, y = _run(x, cu, pool, slots, has, debug=True)
    o_ref, S_ref = _reference(x, cu, S0)
    print(f"pool-state mode {mode} worst (norm, max):", _check_outputs(o, o_ref, cu))
    codes, scales, gs = _snap(pool)
    y_np = y.cpu().numpy()
    gden = 6.0 * (448.0 if mode else 240.0)
    for n, s in enumerate(slots):
        if lengths[n] == 0:
            # an empty sequence leaves its slot alone
            np.testing.assert_array_equal(codes[s], before[0][s])
            np.testing.assert_array_equal(scales[s], before[1][s])
            np.testing.assert_array_equal(gs[s], before[2][s])
            continue
        for h in range(HV):
            c2, s2 = oracle_lib.quantise(y_np[n, h].reshape(-1), mode)
            np.testing.assert_array_equal(codes[s, h].reshape(-1), c2)
            np.testing.assert_array_equal(scales[s, h].reshape(-1), s2)
        S_gpu = y_np[n].astype(np.float64) * gs[s][:, None, None]
        # global scale = amax / gden of the state that was quantised
        np.testing.assert_allclose(np.abs(S_gpu).reshape(HV, -1).max(axis=1) / gden, gs[s], rtol=1e-5)
        for h in range(HV):
            rel = np.linalg.norm(S_gpu[h] - S_ref[n, h]) / np.linalg.norm(S_ref[n, h])
            assert rel <= S_NORM_TOL, (n, h, rel)
    for s in (1, 4, 6):
        np.testing.assert_array_equal(codes[s], before[0][s])


def test_prefill_continues_from_its_own_state(cuda, oracle_lib):
    """Two prefill calls over halves of each sequence (the second starting from
    the pool state the first wrote) against the f64 recurrence over the whole
    sequence: the NVFP4 round trip between the calls costs no more than the
    state's quantisation error."""
    lengths = [150, 96, 40]
    x, cu = _inputs(lengths, seed=7)
    first = [l // 2 for l in lengths]
    second = [l - f for l, f in zip(lengths, first)]
    idx1 = np.concatenate([np.arange(cu[n], cu[n] + first[n]) for n in range(3)])
    idx2 = np.concatenate([np.arange(cu[n] + first[n], cu[n + 1]) for n in range(3)])
    x1 = {k: v[torch.from_numpy(idx1).cuda()].contiguous() for k, v in x.items()}
    x2 = {k: v[torch.from_numpy(idx2).cuda()].contiguous() for k, v in x.items()}
    cu1 = np.concatenate([[0], np.cumsum(first)]).astype(np.int32)
    cu2 = np.concatenate([[0], np.cumsum(second)]).astype(np.int32)
    from gdn_b200 import NVFP4StatePool
    pool = NVFP4StatePool.zeros(4, HV, D, "cuda")
    slots = [3, 0, 2]
    _run(x1, cu1, pool, slots, [False] * 3)
    o2, _ = _run(x2, cu2, pool, slots, [True] * 3)
    o_ref, _ = _reference(x, cu)
    o_ref2 = o_ref[idx2]
    o2n = o2.float().cpu().numpy()
    for n in range(3):
        b0, b1 = int(cu2[n]), int(cu2[n + 1])
        rel = np.linalg.norm(o2n[b0:b1] - o_ref2[b0:b1]) / np.linalg.norm(o_ref2[b0:b1])
        assert rel < 0.1, (n, rel)


def test_prefill_bad_slot_and_seqlens(cuda):
    from gdn_b200 import ops
    lengths = [20, 30, 10]
    x, cu = _inputs(lengths, seed=9)
    pool = _pool(4, 0)
    before = _snap(pool)
    ops.device_status(clear=True)
    # slot 9 >= num_slots: that sequence runs from zero and keeps no state
    o, _ = _run(x, cu, pool, [1, 9, -1], [True, True, True])
    assert ops.device_status(clear=True) & 0x2  # GDN_STATUS_BAD_SLOT
    o_ref, _ = _reference(x, cu)
    o_np = o.float().cpu().numpy()
    b0, b1 = int(cu[1]), int(cu[2])
    rel = np.linalg.norm(o_np[b0:b1] - o_ref[b0:b1]) / np.linalg.norm(o_ref[b0:b1])
    assert rel <= O_NORM_TOL
    after = _snap(pool)
    for s in (0, 2, 3):
        np.testing.assert_array_equal(after[0][s], before[0][s])
    assert (after[0][1] != before[0][1]).any()
    # invalid bounds: sequence 1 ends past the last token, sequence 2 ends before it starts
    bad = np.array([0, 10, 70, 60], np.int32)
    sentinel = torch.full((60, HV, D), 7.0, dtype=torch.bfloat16, device="cuda")
    cu_t = torch.from_numpy(bad).cuda()
    ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu_t, out=sentinel)
    torch.cuda.synchronize()
    assert ops.device_status(clear=True) & 0x4  # GDN_STATUS_BAD_SEQLENS
    assert (sentinel[10:].float() == 7.0).all()  # rows of the skipped sequences untouched
    assert (sentinel[:10].float() != 7.0).any()
    assert ops.device_status(clear=True) == 0


def test_prefill_strided_qkv_and_determinism(cuda):
    """q, k, v as views of one fused projection row [T, (2HK + HV) * D]."""
    from gdn_b200 import ops
    lengths = [100, 37]
    x, cu = _inputs(lengths, seed=11)
    T = int(cu[-1])
    fused = torch.cat([x["q"].reshape(T, -1), x["k"].reshape(T, -1), x["v"].reshape(T, -1)], dim=1)
    qv = fused[:, :HK * D].view(T, HK, D)
    kv = fused[:, HK * D:2 * HK * D].view(T, HK, D)
    vv = fused[:, 2 * HK * D:].view(T, HV, D)
    cu_t = torch.from_numpy(cu).cuda()
    o1 = ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu_t)
    o2 = ops.prefill(qv, kv, vv, x["g"], x["beta"], cu_t)
    o3 = ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu_t)
    assert torch.equal(o1, o2)
    assert torch.equal(o1, o3)


def test_prefill_long_sequence(cuda):
    """One 8192-token sequence (the long-prefill shape): a sample of heads
    against the f64 recurrence, every head finite."""
    from oracle import bindings as ob
    x, cu = _inputs([8192], seed=13)
    o, _ = _run(x, cu)
    on = o.float().cpu().numpy()
    assert np.isfinite(on).all()
    q = x["q"].float().cpu().numpy()
    k = x["k"].float().cpu().numpy()
    v = x["v"].float().cpu().numpy()
    g = x["g"].cpu().numpy()
    be = x["beta"].cpu().numpy()
    for h in (0, 13, 31):
        hk = h // (HV // HK)
        ref, _ = ob.recurrent_f64(np.zeros((D, D)), q[:, hk], k[:, hk], v[:, h], g[:, h], be[:, h], QS)
        rel = np.linalg.norm(on[:, h] - ref) / np.linalg.norm(ref)
        assert rel <= O_NORM_TOL, (h, rel)


def test_prefill_qk_l2norm_in_kernel(cuda):
    """qk_l2norm: q and k arrive unnormalised (each token scaled by 0.3 .. 3)
    and the kernel scales them to unit L2 norm, x / sqrt(sum x^2 + 1e-6) in
    fp32 (vLLM's use_qk_l2norm_in_kernel).  Outputs and final states follow
    the f64 recurrence of the normalised q, k; from a pool state too."""
    from gdn_b200 import ops
    lengths = [1, 70, 130, 64]
    x, cu = _inputs(lengths, seed=33)
    gen = torch.Generator().manual_seed(34)
    T = int(cu[-1])
    sq = (0.3 + 2.7 * torch.rand((T, HK, 1), generator=gen)).cuda()
    sk = (0.3 + 2.7 * torch.rand((T, HK, 1), generator=gen)).cuda()
    raw = dict(x, q=(x["q"].float() * sq).to(torch.bfloat16), k=(x["k"].float() * sk).to(torch.bfloat16))
    # the reference: the raw bf16 rows normalised in fp32
    ref_in = dict(x)
    for n in ("q", "k"):
        f = raw[n].float()
        ref_in[n] = f / torch.sqrt((f * f).sum(-1, keepdim=True) + 1e-6)
    pool = _pool(len(lengths), 1, seed=35)
    S0 = pool.dequantize().cpu().numpy()
    slots = list(range(len(lengths)))
    cu_t = torch.from_numpy(cu).cuda()
    o = ops.prefill(raw["q"], raw["k"], raw["v"], raw["g"], raw["beta"], cu_t, pool=pool,
                    slot_idx=torch.tensor(slots, dtype=torch.int32, device="cuda"),
                    has_initial_state=torch.ones(len(lengths), dtype=torch.bool, device="cuda"), qk_l2norm=True)
    torch.cuda.synchronize()
    o_ref, S_ref = _reference(ref_in, cu, S0)
    print("qk_l2norm worst (norm, max):", _check_outputs(o, o_ref, cu))
    S = pool.dequantize().cpu().numpy()
    for n in range(len(lengths)):
        for h in range(0, HV, 5):
            # the final state crosses NVFP4 once: the requantisation error dominates
            assert np.linalg.norm(S[n, h] - S_ref[n, h]) <= 0.15 * np.linalg.norm(S_ref[n, h])
    # without the flag the same raw inputs give a different result
    o_raw = ops.prefill(raw["q"], raw["k"], raw["v"], raw["g"], raw["beta"], cu_t)
    assert not torch.equal(o_raw, o)
