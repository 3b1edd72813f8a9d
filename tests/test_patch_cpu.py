"""The reference's Python integration surface (src/ops/qwen35_gdn_patch.py,
src/ops/gdn_op.py) mirrored by gdn_b200: names, defaults and errors, on CPU."""
from __future__ import annotations

import pytest
import torch


def test_state_cache_semantics():
    from gdn_b200.qwen35_gdn_patch import GDNStateCache
    c = GDNStateCache()
    d, s = c.get(3, 1, 64, torch.device("cpu"))
    assert d.shape == (64 * 64 // 2,) and s.shape == (64 * 64 // 16,)
    assert d.dtype == torch.uint8 and s.dtype == torch.uint8
    assert int(d.sum()) == 0 and int(s.sum()) == 0  # the zero state
    assert c.get(3, 1, 64, torch.device("cpu"))[0] is d  # cached
    nd, ns = torch.ones_like(d), torch.ones_like(s)
    c.update(3, 1, nd, ns)
    assert c.get(3, 1, 64, torch.device("cpu"))[0] is nd
    c.reset()
    assert len(c) == 0


def test_apply_missing_library(monkeypatch, tmp_path):
    from gdn_b200 import qwen35_gdn_patch as P
    assert P.get_patch_status() == {"patched": False, "so_path": None}
    with pytest.raises(FileNotFoundError):
        P.apply(so_path=str(tmp_path / "nope.so"))
    monkeypatch.setenv("GDN_OP_LIB", str(tmp_path / "also_missing.so"))
    with pytest.raises(FileNotFoundError):
        P.apply()
    assert P.get_patch_status()["patched"] is False


def test_load_gdn_op_missing_library(tmp_path):
    from gdn_b200 import gdn_op
    with pytest.raises(FileNotFoundError):
        gdn_op.load_gdn_op(str(tmp_path / "missing.so"))


def test_apply_routes_vllm_gdn_layer():
    """apply() swaps vLLM 0.22's prefill CustomOp and decode entry for the
    NVFP4 seam; remove() restores them."""
    pytest.importorskip("vllm")
    import importlib
    from gdn_b200 import qwen35_gdn_patch as P, vllm_seam
    try:
        mod = importlib.import_module(P._VLLM_GDN_MODULE)
    except Exception as e:  # vLLM present but its GDN layer does not import here
        pytest.skip(f"vLLM GDN layer not importable: {e}")
    orig_native = mod.ChunkGatedDeltaRule.forward_native
    orig_decode = mod.fused_sigmoid_gating_delta_rule_update
    orig_packed = mod.fused_recurrent_gated_delta_rule_packed_decode
    layer = mod.QwenGatedDeltaNetAttention
    had_shape = "get_state_shape" in layer.__dict__
    had_dtype = "get_state_dtype" in layer.__dict__
    had_forward = "forward" in mod.ChunkGatedDeltaRule.__dict__
    P.apply()
    try:
        st = P.get_patch_status()
        assert st["patched"] and st["so_path"].endswith("libgdn_sm120_op.so")
        assert mod.fused_sigmoid_gating_delta_rule_update is vllm_seam.fused_sigmoid_gating_delta_rule_update
        assert mod.fused_recurrent_gated_delta_rule_packed_decode is \
            vllm_seam.fused_recurrent_gated_delta_rule_packed_decode
        assert mod.ChunkGatedDeltaRule.forward_native is not orig_native
        assert hasattr(torch.ops.gdn_sm120, "state_update") and hasattr(torch.ops.gdn_sm120, "prefill")
        # the layer's state cache is sized as NVFP4 records
        assert "get_state_shape" in layer.__dict__ and "get_state_dtype" in layer.__dict__
    finally:
        P.remove()
    assert mod.ChunkGatedDeltaRule.forward_native is orig_native
    assert mod.fused_sigmoid_gating_delta_rule_update is orig_decode
    assert mod.fused_recurrent_gated_delta_rule_packed_decode is orig_packed
    assert ("get_state_shape" in layer.__dict__) == had_shape
    assert ("get_state_dtype" in layer.__dict__) == had_dtype
    assert ("forward" in mod.ChunkGatedDeltaRule.__dict__) == had_forward
    P.reset_state()


def test_nvfp4_state_cache_shape_hooks():
    """The patched shape/dtype hooks turn the dense [HV, V, K] temporal state
    into one NVFP4 record per value head, uint8, and leave the conv state."""
    pytest.importorskip("vllm")
    import importlib
    from gdn_b200 import qwen35_gdn_patch as P, vllm_seam
    from gdn_b200.pool import RECORD_BYTES
    try:
        mod = importlib.import_module(P._VLLM_GDN_MODULE)
    except Exception as e:
        pytest.skip(f"vLLM GDN layer not importable: {e}")

    import types

    class FakeLayer(mod.QwenGatedDeltaNetAttention):
        def __init__(self):  # the fields the hooks read, without a vLLM engine
            torch.nn.Module.__init__(self)
            self.tp_size, self.num_k_heads, self.num_v_heads = 2, 16, 32
            self.head_k_dim = self.head_v_dim = 128
            self.conv_kernel_size, self.num_spec = 4, 0
            self.model_config = types.SimpleNamespace(dtype=torch.bfloat16)
            self.cache_config = types.SimpleNamespace(mamba_cache_dtype="auto", mamba_ssm_cache_dtype="auto")

    dense_shape = mod.QwenGatedDeltaNetAttention.get_state_shape(FakeLayer())
    P.apply()
    try:
        layer = FakeLayer()
        conv_shape, temporal = mod.QwenGatedDeltaNetAttention.get_state_shape(layer)
        assert conv_shape == dense_shape[0]
        assert temporal == (16, RECORD_BYTES) == vllm_seam.state_shape(16)
        assert mod.QwenGatedDeltaNetAttention.get_state_dtype(layer) == (torch.bfloat16, torch.uint8)
    finally:
        P.remove()
