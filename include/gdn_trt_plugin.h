/*
 * gdn_trt_plugin.h -- the TensorRT-LLM plugin face of the NVFP4 Gated DeltaNet
 * decode step: a C++ class with the IPluginV3 method set (IPluginV3OneCore,
 * IPluginV3OneBuild, IPluginV3OneRuntime) and a creator with the
 * IPluginCreatorV3One method set, whose enqueue calls gdn_decode
 * (gdn_b200.h).  It replaces the reference's empty plugin target
 * (src/trtllm/CMakeLists.txt:1-3) and follows the shape its PRD gives
 * (PRD.md:29-44): enqueue() calls the kernel, getOutputDataTypes() names the
 * output types, configurePlugin() checks the device capability, and the
 * library is libgdn_sm120_plugin.so.
 *
 * TensorRT is not a build dependency.  The descriptor types below carry the
 * same fields and enumerator values as nvinfer1's (DataType, Dims64,
 * PluginTensorDesc), so the adapter a TensorRT build adds derives from the
 * nvinfer1 interfaces and forwards each override to this class with a
 * reinterpret_cast of the descriptor pointers.
 *
 * Tensors (TensorRT linear format, row-major, contiguous):
 *   inputs  0 q            [B, HK, D]          bf16
 *           1 k            [B, HK, D]          bf16
 *           2 v            [B, HV, D]          bf16
 *           3 g            [B, HV]             fp32  log decay
 *           4 beta         [B, HV]             fp32
 *           5 slot_idx     [B]                 int32 (negative = padding)
 *           6 pool_codes   [S, HV, D, D/2]     uint8 (updated in place)
 *           7 pool_scales  [S, HV, D, D/16]    uint8 (updated in place)
 *           8 pool_gscale  [S, HV]             fp32  (updated in place)
 *   output  0 out          [B, HV, D]          bf16
 * D must be 128 and HV a multiple of HK.  The plugin needs no workspace: the
 * kernel allocates nothing.
 */
#ifndef GDN_TRT_PLUGIN_H_
#define GDN_TRT_PLUGIN_H_

#include <cstdint>
#include <cstring>
#include <string>

#include <cuda_runtime_api.h>

#include "gdn_b200.h"

namespace gdn_trt {

// nvinfer1::DataType enumerator values.
enum class DataType : int32_t {
  kFLOAT = 0,
  kHALF = 1,
  kINT8 = 2,
  kINT32 = 3,
  kBOOL = 4,
  kUINT8 = 5,
  kFP8 = 6,
  kBF16 = 7,
  kINT64 = 8,
};

// nvinfer1::TensorFormat::kLINEAR.
constexpr int32_t kFormatLinear = 0;

// nvinfer1::Dims64.
struct Dims {
  int32_t nbDims;
  int64_t d[8];
};

// nvinfer1::PluginTensorDesc.
struct PluginTensorDesc {
  Dims dims;
  DataType type;
  int32_t format;
  float scale;
};

// nvinfer1::PluginField / PluginFieldCollection (kFLOAT32 = 1, kINT32 = 2 as in PluginFieldType).
enum class FieldType : int32_t { kFLOAT32 = 1, kINT32 = 2 };
struct PluginField {
  const char* name;
  const void* data;
  FieldType type;
  int32_t length;
};
struct PluginFieldCollection {
  int32_t nbFields;
  const PluginField* fields;
};

// Return codes of the methods that TensorRT reads as int32 status (0 = ok).
constexpr int32_t kOk = 0;
constexpr int32_t kBadArgs = -1;
constexpr int32_t kBadDevice = -2;
constexpr int32_t kKernelFailed = -3;

class GdnDecodePlugin {
 public:
  static constexpr int32_t kNbInputs = 9;
  static constexpr int32_t kNbOutputs = 1;

  // Plugin fields: scale_mode (int32, GDN_SCALE_*), q_scale (float, <= 0:
  // 1/sqrt(D)), gscale_den (float, <= 0: 6 x saturation), qk_l2norm (int32).
  GdnDecodePlugin(int32_t scale_mode = GDN_SCALE_FN448, float q_scale = 0.0f, float gscale_den = 0.0f,
                  int32_t qk_l2norm = 0)
      : scale_mode_(scale_mode), q_scale_(q_scale), gscale_den_(gscale_den), qk_l2norm_(qk_l2norm) {}

  // ---- IPluginV3OneCore ----
  const char* getPluginName() const noexcept { return "GdnNvfp4Decode"; }
  const char* getPluginVersion() const noexcept { return "1"; }
  const char* getPluginNamespace() const noexcept { return namespace_.c_str(); }
  void setPluginNamespace(const char* ns) noexcept { namespace_ = ns ? ns : ""; }

  // ---- IPluginV3OneBuild ----
  int32_t getNbOutputs() const noexcept { return kNbOutputs; }

  // out = bf16; the pool tensors are inputs updated in place.
  int32_t getOutputDataTypes(DataType* outputTypes, int32_t nbOutputs, const DataType* inputTypes,
                             int32_t nbInputs) const noexcept {
    if (!outputTypes || nbOutputs != kNbOutputs || nbInputs != kNbInputs || !inputTypes) return kBadArgs;
    outputTypes[0] = DataType::kBF16;
    return kOk;
  }

  // out = [B, HV, D] from v = [B, HV, D].
  int32_t getOutputShapes(const Dims* inputs, int32_t nbInputs, Dims* outputs, int32_t nbOutputs) const noexcept {
    if (!inputs || !outputs || nbInputs != kNbInputs || nbOutputs != kNbOutputs || inputs[2].nbDims != 3)
      return kBadArgs;
    outputs[0] = inputs[2];
    return kOk;
  }

  // Linear format everywhere, with the dtype each position needs.
  bool supportsFormatCombination(int32_t pos, const PluginTensorDesc* inOut, int32_t nbInputs,
                                 int32_t nbOutputs) const noexcept {
    if (!inOut || nbInputs != kNbInputs || nbOutputs != kNbOutputs || pos < 0 || pos >= kNbInputs + kNbOutputs)
      return false;
    return inOut[pos].format == kFormatLinear && inOut[pos].type == expected_type(pos);
  }

  // Shapes and types of a concrete configuration, then the device: this
  // library is built for sm_100a (compute capability 10.0).
  int32_t configurePlugin(const PluginTensorDesc* in, int32_t nbInputs, const PluginTensorDesc* out,
                          int32_t nbOutputs) noexcept {
    if (!in || !out || nbInputs != kNbInputs || nbOutputs != kNbOutputs) return kBadArgs;
    for (int32_t i = 0; i < kNbInputs + kNbOutputs; ++i) {
      const PluginTensorDesc& t = i < kNbInputs ? in[i] : out[i - kNbInputs];
      if (t.type != expected_type(i) || t.format != kFormatLinear) return kBadArgs;
    }
    Shape s;
    if (!shape_of(in, out, &s)) return kBadArgs;
    return check_device();
  }

  size_t getWorkspaceSize(const PluginTensorDesc*, int32_t, const PluginTensorDesc*, int32_t) const noexcept {
    return 0;
  }

  // ---- IPluginV3OneRuntime ----
  int32_t enqueue(const PluginTensorDesc* inputDesc, const PluginTensorDesc* outputDesc, const void* const* inputs,
                  void* const* outputs, void* /*workspace*/, cudaStream_t stream) noexcept {
    if (!inputDesc || !outputDesc || !inputs || !outputs) return kBadArgs;
    Shape s;
    if (!shape_of(inputDesc, outputDesc, &s)) return kBadArgs;
    gdn_decode_params p;
    std::memset(&p, 0, sizeof(p));
    p.batch = (int32_t)s.B;
    p.num_k_heads = (int32_t)s.HK;
    p.num_v_heads = (int32_t)s.HV;
    p.head_dim = (int32_t)s.D;
    p.num_slots = s.S;
    p.q = static_cast<const gdn_bf16_t*>(inputs[0]);
    p.k = static_cast<const gdn_bf16_t*>(inputs[1]);
    p.v = static_cast<const gdn_bf16_t*>(inputs[2]);
    p.g = static_cast<const float*>(inputs[3]);
    p.beta = static_cast<const float*>(inputs[4]);
    p.slot_idx = static_cast<const int32_t*>(inputs[5]);
    // The pool is updated in place: TensorRT binds these inputs to the
    // state buffers the engine keeps across steps.
    p.pool_codes = static_cast<uint8_t*>(const_cast<void*>(inputs[6]));
    p.pool_scales = static_cast<uint8_t*>(const_cast<void*>(inputs[7]));
    p.pool_gscale = static_cast<float*>(const_cast<void*>(inputs[8]));
    p.out = static_cast<gdn_bf16_t*>(outputs[0]);
    p.q_scale = q_scale_;
    p.scale_mode = scale_mode_;
    p.gscale_den = gscale_den_;
    p.qk_l2norm = qk_l2norm_;
    return gdn_decode(&p, stream) == GDN_OK ? kOk : kKernelFailed;
  }

  GdnDecodePlugin* clone() const noexcept {
    GdnDecodePlugin* c = new GdnDecodePlugin(scale_mode_, q_scale_, gscale_den_, qk_l2norm_);
    c->setPluginNamespace(namespace_.c_str());
    return c;
  }

  int32_t scale_mode() const noexcept { return scale_mode_; }
  float q_scale() const noexcept { return q_scale_; }
  float gscale_den() const noexcept { return gscale_den_; }
  int32_t qk_l2norm() const noexcept { return qk_l2norm_; }

  // Compute capability 10.x on the current device, else kBadDevice.
  static int32_t check_device() noexcept {
    int dev = 0;
    cudaDeviceProp prop;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      (void)cudaGetLastError();
      return kBadDevice;
    }
    return prop.major == 10 ? kOk : kBadDevice;
  }

  static DataType expected_type(int32_t pos) noexcept {
    switch (pos) {
      case 0: case 1: case 2: case 9: return DataType::kBF16;
      case 3: case 4: case 8: return DataType::kFLOAT;
      case 5: return DataType::kINT32;
      default: return DataType::kUINT8;  // 6, 7
    }
  }

 private:
  struct Shape {
    int64_t B, HK, HV, D, S;
  };

  static bool shape_of(const PluginTensorDesc* in, const PluginTensorDesc* out, Shape* s) noexcept {
    const Dims& q = in[0].dims;
    if (q.nbDims != 3) return false;
    s->B = q.d[0];
    s->HK = q.d[1];
    s->D = q.d[2];
    const Dims& v = in[2].dims;
    if (v.nbDims != 3 || v.d[0] != s->B || v.d[2] != s->D) return false;
    s->HV = v.d[1];
    const Dims& codes = in[6].dims;
    if (codes.nbDims != 4) return false;
    s->S = codes.d[0];
    const int64_t D = s->D;
    auto is = [](const Dims& d, int n, int64_t a, int64_t b, int64_t c, int64_t e) {
      if (d.nbDims != n) return false;
      const int64_t want[4] = {a, b, c, e};
      for (int i = 0; i < n; ++i)
        if (d.d[i] != want[i]) return false;
      return true;
    };
    return D == 128 && s->HK > 0 && s->HV > 0 && s->HV % s->HK == 0 && s->B >= 0 && s->S >= 0 &&
           is(in[1].dims, 3, s->B, s->HK, D, 0) && is(in[3].dims, 2, s->B, s->HV, 0, 0) &&
           is(in[4].dims, 2, s->B, s->HV, 0, 0) && is(in[5].dims, 1, s->B, 0, 0, 0) &&
           is(codes, 4, s->S, s->HV, D, D / 2) && is(in[7].dims, 4, s->S, s->HV, D, D / 16) &&
           is(in[8].dims, 2, s->S, s->HV, 0, 0) && is(out[0].dims, 3, s->B, s->HV, D, 0);
  }

  int32_t scale_mode_;
  float q_scale_;
  float gscale_den_;
  int32_t qk_l2norm_;
  std::string namespace_;
};

// IPluginCreatorV3One method set.
class GdnDecodePluginCreator {
 public:
  const char* getPluginName() const noexcept { return "GdnNvfp4Decode"; }
  const char* getPluginVersion() const noexcept { return "1"; }
  const char* getPluginNamespace() const noexcept { return ""; }

  const PluginFieldCollection* getFieldNames() noexcept {
    static const PluginField fields[4] = {
        {"scale_mode", nullptr, FieldType::kINT32, 1},
        {"q_scale", nullptr, FieldType::kFLOAT32, 1},
        {"gscale_den", nullptr, FieldType::kFLOAT32, 1},
        {"qk_l2norm", nullptr, FieldType::kINT32, 1},
    };
    static const PluginFieldCollection fc = {4, fields};
    return &fc;
  }

  // Unknown fields are ignored; a field of the wrong type or length, or a
  // scale mode other than GDN_SCALE_*, gives nullptr.
  GdnDecodePlugin* createPlugin(const char* /*name*/, const PluginFieldCollection* fc) noexcept {
    int32_t mode = GDN_SCALE_FN448, l2 = 0;
    float qs = 0.0f, gden = 0.0f;
    for (int32_t i = 0; fc && i < fc->nbFields; ++i) {
      const PluginField& f = fc->fields[i];
      if (!f.name || !f.data || f.length != 1) return nullptr;
      if (!std::strcmp(f.name, "scale_mode") || !std::strcmp(f.name, "qk_l2norm")) {
        if (f.type != FieldType::kINT32) return nullptr;
        (!std::strcmp(f.name, "scale_mode") ? mode : l2) = *static_cast<const int32_t*>(f.data);
      } else if (!std::strcmp(f.name, "q_scale") || !std::strcmp(f.name, "gscale_den")) {
        if (f.type != FieldType::kFLOAT32) return nullptr;
        (!std::strcmp(f.name, "q_scale") ? qs : gden) = *static_cast<const float*>(f.data);
      }
    }
    if (mode != GDN_SCALE_REF240 && mode != GDN_SCALE_FN448) return nullptr;
    return new GdnDecodePlugin(mode, qs, gden, l2);
  }
};

}  // namespace gdn_trt

#endif  // GDN_TRT_PLUGIN_H_
