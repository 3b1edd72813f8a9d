"""ctypes mirror of include/gdn_trt_plugin.h's descriptor types and the C entry
points of libgdn_sm120_plugin.so, shared by the plugin tests."""
from __future__ import annotations

import ctypes
import pathlib

LIB = pathlib.Path(__file__).resolve().parent.parent / "blackwell-kernel-sm_120_b200" / "lib" / "libgdn_sm120_plugin.so"

# nvinfer1::DataType values
FLOAT, HALF, INT8, INT32, BOOL, UINT8, FP8, BF16, INT64 = range(9)
FIELD_FLOAT32, FIELD_INT32 = 1, 2


class Dims(ctypes.Structure):
    _fields_ = [("nbDims", ctypes.c_int32), ("d", ctypes.c_int64 * 8)]


class PluginTensorDesc(ctypes.Structure):
    _fields_ = [("dims", Dims), ("type", ctypes.c_int32), ("format", ctypes.c_int32), ("scale", ctypes.c_float)]


class PluginField(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.c_void_p), ("type", ctypes.c_int32),
                ("length", ctypes.c_int32)]


class PluginFieldCollection(ctypes.Structure):
    _fields_ = [("nbFields", ctypes.c_int32), ("fields", ctypes.POINTER(PluginField))]


def load() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(LIB))
    p = ctypes.c_void_p
    lib.gdn_trt_get_creators.restype = p
    lib.gdn_trt_get_creators.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    lib.gdn_trt_plugin_create.restype = p
    lib.gdn_trt_plugin_create.argtypes = [ctypes.POINTER(PluginFieldCollection)]
    lib.gdn_trt_plugin_clone.restype = p
    lib.gdn_trt_plugin_clone.argtypes = [p]
    lib.gdn_trt_plugin_destroy.argtypes = [p]
    lib.gdn_trt_plugin_name.restype = ctypes.c_char_p
    lib.gdn_trt_plugin_name.argtypes = [p]
    lib.gdn_trt_plugin_nb_outputs.argtypes = [p]
    lib.gdn_trt_plugin_output_types.argtypes = [p, ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                                                ctypes.POINTER(ctypes.c_int32), ctypes.c_int32]
    lib.gdn_trt_plugin_output_shapes.argtypes = [p, ctypes.POINTER(Dims), ctypes.c_int32, ctypes.POINTER(Dims),
                                                 ctypes.c_int32]
    lib.gdn_trt_plugin_supports.argtypes = [p, ctypes.c_int32, ctypes.POINTER(PluginTensorDesc), ctypes.c_int32,
                                            ctypes.c_int32]
    lib.gdn_trt_plugin_configure.argtypes = [p, ctypes.POINTER(PluginTensorDesc), ctypes.c_int32,
                                             ctypes.POINTER(PluginTensorDesc), ctypes.c_int32]
    lib.gdn_trt_plugin_workspace.restype = ctypes.c_uint64
    lib.gdn_trt_plugin_workspace.argtypes = [p]
    lib.gdn_trt_plugin_enqueue.argtypes = [p, ctypes.POINTER(PluginTensorDesc), ctypes.POINTER(PluginTensorDesc),
                                           ctypes.POINTER(p), ctypes.POINTER(p), p]
    return lib


def fields(**kw) -> tuple[PluginFieldCollection, list]:
    """A field collection; ints become kINT32 fields, floats kFLOAT32."""
    keep = []
    arr = (PluginField * len(kw))()
    for i, (name, val) in enumerate(kw.items()):
        if isinstance(val, int):
            v, t = ctypes.c_int32(val), FIELD_INT32
        else:
            v, t = ctypes.c_float(val), FIELD_FLOAT32
        keep.append(v)
        arr[i] = PluginField(name.encode(), ctypes.cast(ctypes.pointer(v), ctypes.c_void_p), t, 1)
    keep.append(arr)
    return PluginFieldCollection(len(kw), arr), keep


def desc(shape, dtype) -> PluginTensorDesc:
    d = Dims()
    d.nbDims = len(shape)
    for i, s in enumerate(shape):
        d.d[i] = s
    return PluginTensorDesc(d, dtype, 0, 1.0)


def decode_descs(B, HK, HV, D, S):
    ins = [desc((B, HK, D), BF16), desc((B, HK, D), BF16), desc((B, HV, D), BF16), desc((B, HV), FLOAT),
           desc((B, HV), FLOAT), desc((B,), INT32), desc((S, HV, D, D // 2), UINT8), desc((S, HV, D, D // 16), UINT8),
           desc((S, HV), FLOAT)]
    outs = [desc((B, HV, D), BF16)]
    return (PluginTensorDesc * 9)(*ins), (PluginTensorDesc * 1)(*outs)
