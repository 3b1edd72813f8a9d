"""GPU checks of the vLLM 0.22 seam (gdn_b200.vllm_seam) and of the
gdn_sm120.prefill torch op: same kernels as the C ABI, vLLM's argument
conventions ([1, T, H, D] inputs, [N, HV, V, K] dense states, PAD_SLOT_ID=-1)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128
QS = 1.0 / np.sqrt(D)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _inputs(lengths, seed):
    from gdn_b200 import workloads
    x = workloads.token_inputs(int(sum(lengths)), HK, HV, D, seed=seed, device="cuda")
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    return x, cu


def test_torch_prefill_op_matches_capi(cuda):
    from gdn_b200 import gdn_op, ops, NVFP4StatePool, workloads
    x, cu = _inputs([70, 5, 130], seed=21)
    o1 = ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu)
    o2 = gdn_op.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu)
    assert torch.equal(o1, o2)
    states = workloads.initial_states(4, HV, D, seed=3).cuda()
    p1 = NVFP4StatePool.zeros(4, HV, D, "cuda")
    p1.load_fp32(states)
    p2 = NVFP4StatePool.zeros(4, HV, D, "cuda")
    p2.load_fp32(states)
    slot = torch.tensor([2, 0, 3], dtype=torch.int32, device="cuda")
    has = torch.tensor([True, False, True], device="cuda")
    o1 = ops.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu, pool=p1, slot_idx=slot, has_initial_state=has)
    o2 = gdn_op.prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], cu, pool=p2, slot_idx=slot, has_initial_state=has)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    assert torch.equal(p1.codes, p2.codes) and torch.equal(p1.gscale, p2.gscale)


def test_seam_prefill(cuda):
    from gdn_b200 import ops, vllm_seam, workloads
    from oracle import bindings as ob
    lengths = [100, 33]
    x, cu = _inputs(lengths, seed=22)
    N = len(lengths)
    init = workloads.initial_states(N, HV, D, seed=4).cuda()      # S[k][v]
    init_vk = init.transpose(-1, -2).contiguous()                   # vLLM layout [V][K]
    o, final = vllm_seam.chunk_gated_delta_rule(
        x["q"].unsqueeze(0), x["k"].unsqueeze(0), x["v"].unsqueeze(0), x["g"].unsqueeze(0),
        x["beta"].unsqueeze(0), init_vk, True, cu_seqlens=cu, use_qk_l2norm_in_kernel=False)
    torch.cuda.synchronize()
    assert o.shape == (1, sum(lengths), HV, D) and final.shape == (N, HV, D, D)
    # reference: f64 recurrence from the NVFP4-rounded initial states
    from gdn_b200 import NVFP4StatePool
    pool = NVFP4StatePool.zeros(N, HV, D, "cuda")
    pool.load_fp32(init)
    S0 = pool.dequantize().cpu().numpy()
    q, k, v = (x[n].float().cpu().numpy() for n in ("q", "k", "v"))
    g, be = x["g"].cpu().numpy(), x["beta"].cpu().numpy()
    cun = cu.cpu().numpy()
    on = o[0].float().cpu().numpy()
    fin = final.transpose(-1, -2).cpu().numpy()
    for n in range(N):
        b0, b1 = cun[n], cun[n + 1]
        for h in range(0, HV, 7):
            ref, S = ob.recurrent_f64(S0[n, h], q[b0:b1, h // 2], k[b0:b1, h // 2], v[b0:b1, h], g[b0:b1, h],
                                      be[b0:b1, h], QS)
            assert np.linalg.norm(on[b0:b1, h] - ref) <= 1e-2 * np.linalg.norm(ref)
            # final state crosses NVFP4 once more on the way out
            assert np.linalg.norm(fin[n, h] - S) <= 0.15 * np.linalg.norm(S)


def test_seam_decode_in_place(cuda):
    from gdn_b200 import ops, vllm_seam, NVFP4StatePool, workloads
    B, slots = 6, 10
    x = workloads.decode_steps(B, 1, HK, HV, D, seed=23, device="cuda")
    gen = torch.Generator(device="cpu").manual_seed(5)
    A_log = torch.randn(HV, generator=gen).cuda()
    dt_bias = torch.randn(HV, generator=gen).cuda()
    a = torch.randn(B, HV, generator=gen).cuda()
    b = torch.randn(B, HV, generator=gen).cuda()
    ssm = workloads.initial_states(slots, HV, D, seed=6).cuda().transpose(-1, -2).contiguous()  # [slots, HV, V, K]
    before = ssm.clone()
    idx = torch.tensor([4, -1, 0, 9, 2, 7], dtype=torch.int32, device="cuda")  # <= 0: padding (0 = null block)
    o, st = vllm_seam.fused_sigmoid_gating_delta_rule_update(
        A_log, a, b, dt_bias, x["q"][0].unsqueeze(0), x["k"][0].unsqueeze(0), x["v"][0].unsqueeze(0),
        initial_state=ssm, inplace_final_state=True, ssm_state_indices=idx, use_qk_l2norm_in_kernel=False)
    torch.cuda.synchronize()
    assert st is ssm and o.shape == (1, B, HV, D)
    # same kernel (gating fused in, from the bf16 gate projections) through the C ABI on the same NVFP4 tiles
    pool = NVFP4StatePool.zeros(B, HV, D, "cuda", scale_mode=vllm_seam.SCALE_MODE)
    pool.load_fp32(before[idx.long().clamp(min=0)].transpose(-1, -2).contiguous())
    slot = torch.tensor([0, -1, -1, 3, 4, 5], dtype=torch.int32, device="cuda")
    o_ref = ops.decode(x["q"][0], x["k"][0], x["v"][0], None, None, slot, pool, A_log=A_log, dt_bias=dt_bias,
                       gate_a=a.to(torch.bfloat16), gate_b=b.to(torch.bfloat16))
    assert torch.equal(o[0], o_ref)
    # and the torch gating of the same bf16 projections agrees to the last bits of exp / log1p
    g, beta = vllm_seam.gating(A_log, a.to(torch.bfloat16), b.to(torch.bfloat16), dt_bias)
    pool2 = NVFP4StatePool.zeros(B, HV, D, "cuda", scale_mode=vllm_seam.SCALE_MODE)
    pool2.load_fp32(before[idx.long().clamp(min=0)].transpose(-1, -2).contiguous())
    o_host = ops.decode(x["q"][0], x["k"][0], x["v"][0], g, beta, slot, pool2)
    assert float((o_host.float() - o_ref.float()).abs().max()) <= 1e-2 * float(o_ref.float().abs().max())
    new = pool.dequantize().transpose(-1, -2)
    for i, s in enumerate(idx.tolist()):
        if s > 0:
            assert torch.equal(ssm[s], new[i])
    for s in (0, 1, 3, 5, 6, 8):
        assert torch.equal(ssm[s], before[s])


def test_seam_decode_out_of_place(cuda):
    """inplace_final_state=False: the cache is left alone and the states after
    the token come back in a fresh [B, HV, V, K] tensor (row i = sequence i,
    padding rows zero), as vLLM's own function returns them."""
    from gdn_b200 import vllm_seam, workloads
    B, slots = 5, 8
    x = workloads.decode_steps(B, 1, HK, HV, D, seed=31, device="cuda")
    gen = torch.Generator(device="cpu").manual_seed(7)
    A_log, dt_bias = torch.randn(HV, generator=gen).cuda(), torch.randn(HV, generator=gen).cuda()
    a, b = torch.randn(B, HV, generator=gen).cuda(), torch.randn(B, HV, generator=gen).cuda()
    ssm = workloads.initial_states(slots, HV, D, seed=8).cuda().transpose(-1, -2).contiguous()
    idx = torch.tensor([3, -1, 0, 7, 5], dtype=torch.int32, device="cuda")
    args = (A_log, a, b, dt_bias, x["q"][0].unsqueeze(0), x["k"][0].unsqueeze(0), x["v"][0].unsqueeze(0))
    cache = ssm.clone()
    o1, final = vllm_seam.fused_sigmoid_gating_delta_rule_update(*args, initial_state=cache,
                                                                 inplace_final_state=False, ssm_state_indices=idx)
    torch.cuda.synchronize()
    assert torch.equal(cache, ssm)
    assert final.shape == (B, HV, D, D) and final is not cache
    in_place = ssm.clone()
    o2, st = vllm_seam.fused_sigmoid_gating_delta_rule_update(*args, initial_state=in_place,
                                                              inplace_final_state=True, ssm_state_indices=idx)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    for i, s in enumerate(idx.tolist()):
        if s > 0:
            assert torch.equal(final[i], st[s])
            assert not torch.equal(final[i], ssm[s])
        else:  # padding: vLLM's null block 0 or a negative index
            assert int(final[i].count_nonzero()) == 0


def _sqnr(ref: np.ndarray, test: np.ndarray) -> float:
    ref = ref.astype(np.float64)
    err = test.astype(np.float64) - ref
    return float(10 * np.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300)))


def test_nvfp4_state_cache_prefill_then_8_decodes_matches_vllm(cuda, oracle_lib):
    """vLLM's own call sequence for a GDN layer (qwen_gdn_linear_attn.py
    _forward_core / _forward_core_decode_non_spec): a varlen prefill through
    the ChunkGatedDeltaRule op with the sequences' gathered states, the
    index_put of the final states into the cache, then 8 packed decode steps
    updating the cache in place at the state indices.  Patched: the cache is
    uint8 NVFP4 records and the seam runs the NVFP4 kernels.  Unpatched: vLLM's
    own FLA kernels on a dense fp32 cache.  The gate: the seam's outputs,
    measured against vLLM's, are within 0.1 dB of the oracle's quantised
    recurrence (same inputs, same NVFP4 state) measured the same way."""
    fla = pytest.importorskip("vllm.model_executor.layers.fla.ops")
    from gdn_b200 import vllm_seam, workloads
    from gdn_b200.pool import RECORD_BYTES, NVFP4StatePool
    lengths = [70, 130, 33, 200]
    N, steps, blocks = len(lengths), 8, 9
    block_idx = torch.tensor([3, 7, 1, 5], dtype=torch.int32, device="cuda")  # 0 is vLLM's null block
    x = workloads.token_inputs(sum(lengths), HK, HV, D, seed=70, device="cuda")  # q, k L2-normalised
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    gen = torch.Generator().manual_seed(71)
    A_log = (torch.rand(HV, generator=gen) * 2 - 1).cuda()
    dt_bias = torch.randn(HV, generator=gen).cuda()
    dec = workloads.decode_steps(N, steps, HK, HV, D, seed=72, device="cuda")
    a = torch.randn((steps, N, HV), generator=gen).to(torch.bfloat16).cuda()
    b = torch.randn((steps, N, HV), generator=gen).to(torch.bfloat16).cuda()
    qkv_raw = []  # decode inputs as vLLM's packed rows, q / k not normalised (the kernels normalise)
    for t in range(steps):
        scale = 0.5 + torch.rand((N, 1, 1), generator=gen).cuda()
        qkv_raw.append(torch.cat([(dec["q"][t] * scale).reshape(N, -1), (dec["k"][t] * scale).reshape(N, -1),
                                  dec["v"][t].reshape(N, -1)], dim=1).to(torch.bfloat16).contiguous())
    q1, k1, v1 = x["q"].unsqueeze(0), x["k"].unsqueeze(0), x["v"].unsqueeze(0)
    g1, b1 = x["g"].unsqueeze(0), x["beta"].unsqueeze(0)

    def run(cache, prefill_fn, decode_fn):
        idx = block_idx.long()
        init = cache[idx].contiguous()
        init[...] = 0  # no sequence has an initial state (vLLM zeroes those rows)
        o_pre, final = prefill_fn(q1, k1, v1, g1, b1, init)
        cache[idx] = final.to(cache.dtype)
        outs = [o_pre[0].float().cpu().numpy()]
        for t in range(steps):
            out = torch.empty((N, 1, HV, D), dtype=torch.bfloat16, device="cuda")
            decode_fn(qkv_raw[t], a[t], b[t], cache, out)
            outs.append(out[:, 0].float().cpu().numpy())
        torch.cuda.synchronize()
        return outs

    dense = torch.zeros((blocks, HV, D, D), dtype=torch.float32, device="cuda")
    ref = run(dense,
              lambda q, k, v, g, be, init: fla.chunk_gated_delta_rule(
                  q=q, k=k, v=v, g=g, beta=be, initial_state=init, output_final_state=True, cu_seqlens=cu,
                  use_qk_l2norm_in_kernel=False),
              lambda qkv, aa, bb, cache, out: fla.fused_recurrent_gated_delta_rule_packed_decode(
                  mixed_qkv=qkv, a=aa, b=bb, A_log=A_log, dt_bias=dt_bias, scale=D ** -0.5, initial_state=cache,
                  out=out, ssm_state_indices=block_idx, use_qk_l2norm_in_kernel=True))
    records = torch.zeros((blocks, HV, RECORD_BYTES), dtype=torch.uint8, device="cuda")
    got = run(records,
              lambda q, k, v, g, be, init: vllm_seam.chunk_gated_delta_rule(
                  q, k, v, g, be, init, True, cu_seqlens=cu, use_qk_l2norm_in_kernel=False),
              lambda qkv, aa, bb, cache, out: vllm_seam.fused_recurrent_gated_delta_rule_packed_decode(
                  qkv, aa, bb, A_log, dt_bias, D ** -0.5, cache, out, block_idx, use_qk_l2norm_in_kernel=True))
    assert records.dtype == torch.uint8 and records.shape == (blocks, HV, RECORD_BYTES)
    assert int(records[0].count_nonzero()) == 0  # the null block is never written

    # the oracle: f64 prefill from zero, its final state through the reference
    # quantiser (the prefill's global scale amax / (6 * 448)), then 8 oracle decode steps
    qf, kf, vf = (x[n].float().cpu().numpy() for n in ("q", "k", "v"))
    gf, bfv = x["g"].cpu().numpy(), x["beta"].cpu().numpy()
    cun = cu.cpu().numpy()
    S_end = np.zeros((N, HV, D, D))
    for n in range(N):
        s0, s1 = cun[n], cun[n + 1]
        for h in range(HV):
            _, S_end[n, h] = oracle_lib.recurrent_f64(np.zeros((D, D)), qf[s0:s1, h // 2], kf[s0:s1, h // 2],
                                                      vf[s0:s1, h], gf[s0:s1, h], bfv[s0:s1, h], QS)
    c0, s0_, g0, _ = oracle_lib.quantise_tiles(S_end.astype(np.float32).reshape(-1), D * D, 1)
    codes = c0.reshape(N, HV, D, D // 2).copy()
    scales = s0_.reshape(N, HV, D, D // 16).copy()
    gsc = g0.reshape(N, HV).copy()
    orc = [None]
    for t in range(steps):
        qkv = qkv_raw[t].view(N, 2 * HK + HV, D)
        qn = vllm_seam.l2norm(qkv[:, :HK])
        kn = vllm_seam.l2norm(qkv[:, HK:2 * HK])
        gt, bt = vllm_seam.gating(A_log, a[t], b[t], dt_bias)
        o32, _, _ = oracle_lib.gdn_decode(_bits(qn), _bits(kn), _bits(qkv[:, 2 * HK:]), gt.cpu().numpy(),
                                          bt.cpu().numpy(), np.arange(N, dtype=np.int32), codes, scales, gsc, QS, 1)
        orc.append(o32)
    pre = _sqnr(ref[0], got[0])
    assert pre >= 40.0, pre  # the prefill from a zero state: fp32 arithmetic only
    for t in range(1, steps + 1):
        s_gpu, s_orc = _sqnr(ref[t], got[t]), _sqnr(ref[t], orc[t])
        print(f"decode step {t}: SQNR vs vLLM, seam {s_gpu:.2f} dB, oracle {s_orc:.2f} dB")
        assert s_gpu >= s_orc - 0.1, (t, s_gpu, s_orc)
