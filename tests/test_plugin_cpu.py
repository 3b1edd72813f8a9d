"""CPU tests of the TensorRT-LLM plugin face (include/gdn_trt_plugin.h,
libgdn_sm120_plugin.so): the header compiles on its own without TensorRT, and
the plugin's build-time methods (creator fields, output types and shapes,
format support, configure-time checks, workspace) answer as the interface
requires.  No GPU: configurePlugin's device check reports no device here."""
from __future__ import annotations

import ctypes
import pathlib
import subprocess

import pytest

import plugin_ctypes as pc

ROOT = pathlib.Path(__file__).resolve().parent.parent
B, HK, HV, D, S = 4, 16, 32, 128, 8


@pytest.fixture(scope="module")
def lib():
    if not pc.LIB.exists():
        pytest.skip("libgdn_sm120_plugin.so not built")
    return pc.load()


def test_header_compiles_without_tensorrt(tmp_path):
    src = tmp_path / "use_plugin.cpp"
    src.write_text('#include "gdn_trt_plugin.h"\n'
                   'int main() { gdn_trt::GdnDecodePluginCreator c; auto* p = c.createPlugin("x", nullptr);\n'
                   '  int ok = p && p->getNbOutputs() == 1; delete p; return ok ? 0 : 1; }\n')
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                    "-I/usr/local/cuda/include", str(src)], check=True)


def test_creator_fields_and_defaults(lib):
    nb = ctypes.c_int32(0)
    assert lib.gdn_trt_get_creators(ctypes.byref(nb)) and nb.value == 1
    p = lib.gdn_trt_plugin_create(None)
    assert p and lib.gdn_trt_plugin_name(p) == b"GdnNvfp4Decode"
    assert lib.gdn_trt_plugin_nb_outputs(p) == 1
    assert lib.gdn_trt_plugin_workspace(p) == 0
    c = lib.gdn_trt_plugin_clone(p)
    assert c and c != p
    lib.gdn_trt_plugin_destroy(c)
    lib.gdn_trt_plugin_destroy(p)
    fc, keep = pc.fields(scale_mode=0, q_scale=0.1, gscale_den=1440.0, qk_l2norm=1)
    p = lib.gdn_trt_plugin_create(ctypes.byref(fc))
    assert p
    lib.gdn_trt_plugin_destroy(p)
    bad, keep2 = pc.fields(scale_mode=5)
    assert not lib.gdn_trt_plugin_create(ctypes.byref(bad))
    wrong_type, keep3 = pc.fields(scale_mode=1.0)
    assert not lib.gdn_trt_plugin_create(ctypes.byref(wrong_type))


def test_output_types_shapes_and_formats(lib):
    p = lib.gdn_trt_plugin_create(None)
    ins, outs = pc.decode_descs(B, HK, HV, D, S)
    in_types = (ctypes.c_int32 * 9)(*[d.type for d in ins])
    out_types = (ctypes.c_int32 * 1)(-1)
    assert lib.gdn_trt_plugin_output_types(p, out_types, 1, in_types, 9) == 0
    assert out_types[0] == pc.BF16
    assert lib.gdn_trt_plugin_output_types(p, out_types, 2, in_types, 9) != 0
    in_dims = (pc.Dims * 9)(*[d.dims for d in ins])
    out_dims = (pc.Dims * 1)()
    assert lib.gdn_trt_plugin_output_shapes(p, in_dims, 9, out_dims, 1) == 0
    assert [out_dims[0].d[i] for i in range(out_dims[0].nbDims)] == [B, HV, D]
    both = (pc.PluginTensorDesc * 10)(*ins, *outs)
    for pos in range(10):
        assert lib.gdn_trt_plugin_supports(p, pos, both, 9, 1) == 1, pos
    both[3].type = pc.HALF  # g must be fp32
    assert lib.gdn_trt_plugin_supports(p, 3, both, 9, 1) == 0
    both[3].type = pc.FLOAT
    both[0].format = 1  # not linear
    assert lib.gdn_trt_plugin_supports(p, 0, both, 9, 1) == 0
    lib.gdn_trt_plugin_destroy(p)


def test_configure_checks_shapes_then_device(lib):
    p = lib.gdn_trt_plugin_create(None)
    ins, outs = pc.decode_descs(B, HK, HV, D, S)
    rc = lib.gdn_trt_plugin_configure(p, ins, 9, outs, 1)
    assert rc in (0, -2)  # shapes accepted; -2 where no sm_100 device is visible
    bad_d, outs2 = pc.decode_descs(B, HK, HV, 64, S)
    assert lib.gdn_trt_plugin_configure(p, bad_d, 9, outs2, 1) == -1  # head_dim must be 128
    ins3, outs3 = pc.decode_descs(B, 12, HV, D, S)
    assert lib.gdn_trt_plugin_configure(p, ins3, 9, outs3, 1) == -1  # HV % HK != 0
    ins4, outs4 = pc.decode_descs(B, HK, HV, D, S)
    ins4[7].dims.d[3] = 16  # scales must be D / 16 per row
    assert lib.gdn_trt_plugin_configure(p, ins4, 9, outs4, 1) == -1
    ins5, outs5 = pc.decode_descs(B, HK, HV, D, S)
    ins5[5].type = pc.INT64  # slot indices are int32
    assert lib.gdn_trt_plugin_configure(p, ins5, 9, outs5, 1) == -1
    lib.gdn_trt_plugin_destroy(p)
