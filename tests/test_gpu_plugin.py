"""GPU test of the TensorRT-LLM plugin face (libgdn_sm120_plugin.so): the
plugin's configurePlugin accepts the B200, and its enqueue, given TensorRT-style
descriptors and raw device pointers, writes the same output and pool bytes as
gdn_decode called through the Python front end on a twin pool."""
from __future__ import annotations

import ctypes

import pytest
import torch

import plugin_ctypes as pc

pytestmark = pytest.mark.gpu

HK, HV, D = 16, 32, 128


def test_plugin_enqueue_equals_decode(cuda):
    from gdn_b200 import NVFP4StatePool, ops, workloads
    lib = pc.load()
    B, S = 24, 40
    slot = workloads.slot_permutation(B, S, seed=51).cuda()
    states = workloads.initial_states(B, HV, D, seed=52).cuda()
    pools = []
    for _ in range(2):
        p = NVFP4StatePool.zeros(S, HV, D, "cuda", scale_mode=1)
        p.load_fp32(states, slot)
        pools.append(p)
    x = workloads.decode_steps(B, 1, HK, HV, D, seed=53, device="cuda")
    q, k, v, g, beta = (x[n][0].contiguous() for n in ("q", "k", "v", "g", "beta"))
    o_ref = ops.decode(q, k, v, g, beta, slot, pools[0])

    fc, keep = pc.fields(scale_mode=1)
    plugin = lib.gdn_trt_plugin_create(ctypes.byref(fc))
    assert plugin
    ins, outs = pc.decode_descs(B, HK, HV, D, S)
    assert lib.gdn_trt_plugin_configure(plugin, ins, 9, outs, 1) == 0  # sm_100 device accepted
    o = torch.empty((B, HV, D), dtype=torch.bfloat16, device="cuda")
    tensors = [q, k, v, g, beta, slot, pools[1].codes, pools[1].scales, pools[1].gscale]
    in_ptrs = (ctypes.c_void_p * 9)(*[t.data_ptr() for t in tensors])
    out_ptrs = (ctypes.c_void_p * 1)(o.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.gdn_trt_plugin_enqueue(plugin, ins, outs, in_ptrs, out_ptrs, stream) == 0
    torch.cuda.synchronize()
    lib.gdn_trt_plugin_destroy(plugin)
    assert torch.equal(o, o_ref)
    assert torch.equal(pools[0].codes, pools[1].codes) and torch.equal(pools[0].scales, pools[1].scales)
    assert torch.equal(pools[0].gscale, pools[1].gscale)
    assert ops.device_status(clear=True) == 0
