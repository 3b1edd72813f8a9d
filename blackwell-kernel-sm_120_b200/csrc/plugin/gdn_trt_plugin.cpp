// gdn_trt_plugin.cpp -- libgdn_sm120_plugin.so: the TensorRT-LLM plugin face
// (include/gdn_trt_plugin.h) built as the library the reference names
// (PRD.md:29-44), linked against libgdn_b200.so.
//
// Exports, C types only:
//   gdn_trt_get_creators      the creator list a plugin library hands to the
//                             runtime (TensorRT's getCreators entry point,
//                             here with this header's creator type);
//   gdn_trt_plugin_*          each plugin method behind a plain C call, so
//                             that a host without TensorRT (ctypes, the tests)
//                             drives the same code a TensorRT build does.
#include "gdn_trt_plugin.h"

#define GDN_PLUGIN_API extern "C" __attribute__((visibility("default")))

using gdn_trt::DataType;
using gdn_trt::GdnDecodePlugin;
using gdn_trt::GdnDecodePluginCreator;
using gdn_trt::PluginFieldCollection;
using gdn_trt::PluginTensorDesc;

GDN_PLUGIN_API GdnDecodePluginCreator* const* gdn_trt_get_creators(int32_t* nb_creators) {
  static GdnDecodePluginCreator creator;
  static GdnDecodePluginCreator* const list[1] = {&creator};
  if (nb_creators) *nb_creators = 1;
  return list;
}

GDN_PLUGIN_API void* gdn_trt_plugin_create(const PluginFieldCollection* fields) {
  int32_t n = 0;
  return gdn_trt_get_creators(&n)[0]->createPlugin("GdnNvfp4Decode", fields);
}

GDN_PLUGIN_API void* gdn_trt_plugin_clone(const void* plugin) {
  return plugin ? static_cast<const GdnDecodePlugin*>(plugin)->clone() : nullptr;
}

GDN_PLUGIN_API void gdn_trt_plugin_destroy(void* plugin) { delete static_cast<GdnDecodePlugin*>(plugin); }

GDN_PLUGIN_API const char* gdn_trt_plugin_name(const void* plugin) {
  return static_cast<const GdnDecodePlugin*>(plugin)->getPluginName();
}

GDN_PLUGIN_API int32_t gdn_trt_plugin_nb_outputs(const void* plugin) {
  return static_cast<const GdnDecodePlugin*>(plugin)->getNbOutputs();
}

GDN_PLUGIN_API int32_t gdn_trt_plugin_output_types(const void* plugin, DataType* out_types, int32_t nb_outputs,
                                                   const DataType* in_types, int32_t nb_inputs) {
  return static_cast<const GdnDecodePlugin*>(plugin)->getOutputDataTypes(out_types, nb_outputs, in_types, nb_inputs);
}

GDN_PLUGIN_API int32_t gdn_trt_plugin_output_shapes(const void* plugin, const gdn_trt::Dims* in, int32_t nb_inputs,
                                                    gdn_trt::Dims* out, int32_t nb_outputs) {
  return static_cast<const GdnDecodePlugin*>(plugin)->getOutputShapes(in, nb_inputs, out, nb_outputs);
}

GDN_PLUGIN_API int32_t gdn_trt_plugin_supports(const void* plugin, int32_t pos, const PluginTensorDesc* in_out,
                                               int32_t nb_inputs, int32_t nb_outputs) {
  return static_cast<const GdnDecodePlugin*>(plugin)->supportsFormatCombination(pos, in_out, nb_inputs, nb_outputs)
             ? 1
             : 0;
}

GDN_PLUGIN_API int32_t gdn_trt_plugin_configure(void* plugin, const PluginTensorDesc* in, int32_t nb_inputs,
                                                const PluginTensorDesc* out, int32_t nb_outputs) {
  return static_cast<GdnDecodePlugin*>(plugin)->configurePlugin(in, nb_inputs, out, nb_outputs);
}

GDN_PLUGIN_API uint64_t gdn_trt_plugin_workspace(const void* plugin) {
  return static_cast<const GdnDecodePlugin*>(plugin)->getWorkspaceSize(nullptr, 0, nullptr, 0);
}

GDN_PLUGIN_API int32_t gdn_trt_plugin_enqueue(void* plugin, const PluginTensorDesc* in, const PluginTensorDesc* out,
                                              const void* const* inputs, void* const* outputs, cudaStream_t stream) {
  return static_cast<GdnDecodePlugin*>(plugin)->enqueue(in, out, inputs, outputs, nullptr, stream);
}
