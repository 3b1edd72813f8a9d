// nvfp4_kernels.cu -- NVFP4 codec kernels and the legacy d x d state update.
//
// Reference counterparts (bojak83318/blackwell-kernel-sm_120):
//   gdn_nvfp4_quantize     nvfp4_quantise_host   src/kernel/gdn_state_update_ref.cu:93-141
//   gdn_nvfp4_dequantize   nvfp4_dequantise_host :75-89 and dequant_kernel_impl :178-197
//   launch_gdn_ref         :147-176 (dequantise kernel + fp32 update kernel + cudaMalloc/Free)
//   launch_gdn_state_update :202-262 (GPU fp32 update, stream sync, D2H, host
//                           quantise, H2D)
// Here each op is one stream-ordered kernel: one thread owns one 16-element
// scale block, loads it with vector loads, and writes whole bytes (8 code bytes
// + 1 scale byte), so no two threads ever touch the same byte.  These are
// HBM-bound elementwise kernels; grids are a multiple of the SM count.
#include <cstdint>
#include <cuda_bf16.h>

#include "../common.cuh"
#include "../intrinsics/nvfp4_codec.cuh"

namespace gdn {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t work_items, int per_sm = 8) {
  const int64_t cap = (int64_t)sm_count() * per_sm;
  int64_t g = (work_items + kThreads - 1) / kThreads;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

// 16 fp32 -> (w0, w1, scale) in the given mode.
template <bool kCheckRange>
__device__ __forceinline__ uint32_t quant_block(const float (&y)[16], int mode, uint2& codes) {
  float am = y[0];
#pragma unroll
  for (int i = 1; i < 16; ++i) am = absmax_nan(am, y[i]);
  uint32_t w0, w1;
  const uint32_t sc = quantize16<kCheckRange>(y, am, mode, w0, w1);
  codes = make_uint2(w0, w1);
  return sc;
}

// 8 code bytes + scale -> 16 fp32 (exact: e2m1 * scale has <= 6 significant bits).
__device__ __forceinline__ void dequant_block(uint2 codes, float dec, float (&x)[16]) {
  uint32_t h[4];
  cvt_e2m1x8_to_f16x2(codes.x, h);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = f16x2_to_f32x2(h[j]);
    x[2 * j] = f.x * dec;
    x[2 * j + 1] = f.y * dec;
  }
  cvt_e2m1x8_to_f16x2(codes.y, h);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = f16x2_to_f32x2(h[j]);
    x[8 + 2 * j] = f.x * dec;
    x[8 + 2 * j + 1] = f.y * dec;
  }
}

__device__ __forceinline__ void load16(const float* p, float (&x)[16]) {
  const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 t = __ldg(p4 + j);
    x[4 * j] = t.x; x[4 * j + 1] = t.y; x[4 * j + 2] = t.z; x[4 * j + 3] = t.w;
  }
}

__device__ __forceinline__ void store16(float* p, const float (&x)[16]) {
  float4* p4 = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int j = 0; j < 4; ++j) p4[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
}

template <int kMode>
__global__ void __launch_bounds__(kThreads) quantize_kernel(const float* __restrict__ x,
                                                            uint8_t* __restrict__ codes,
                                                            uint8_t* __restrict__ scales, int64_t nblk) {
  for (int64_t b = blockIdx.x * (int64_t)kThreads + threadIdx.x; b < nblk; b += (int64_t)gridDim.x * kThreads) {
    float y[16];
    load16(x + b * 16, y);
    uint2 c;
    scales[b] = (uint8_t)quant_block<true>(y, kMode, c);
    reinterpret_cast<uint2*>(codes)[b] = c;
  }
}

template <int kMode>
__global__ void __launch_bounds__(kThreads) dequantize_kernel(const uint8_t* __restrict__ codes,
                                                              const uint8_t* __restrict__ scales,
                                                              float* __restrict__ out, int64_t nblk) {
  for (int64_t b = blockIdx.x * (int64_t)kThreads + threadIdx.x; b < nblk; b += (int64_t)gridDim.x * kThreads) {
    float x[16];
    dequant_block(__ldg(reinterpret_cast<const uint2*>(codes) + b), scale_decode(__ldg(scales + b), kMode), x);
    store16(out + b * 16, x);
  }
}

// One CTA per tile: pass 1 finds amax (NaN-ignoring, as the reference's
// fmaxf), pass 2 quantises y = x * (1/gs) block by block.
template <int kMode>
__global__ void __launch_bounds__(kThreads) quantize_tiles_kernel(const float* __restrict__ x, int64_t tile_elems,
                                                                  uint8_t* __restrict__ codes,
                                                                  uint8_t* __restrict__ scales,
                                                                  float* __restrict__ gscale, float gden,
                                                                  int64_t ntiles) {
  __shared__ float red[kThreads / 32];
  const int64_t nblk = tile_elems / 16;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const float* xt = x + t * tile_elems;
    float am = 0.0f;
    for (int64_t i = threadIdx.x; i < tile_elems / 4; i += kThreads) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(xt) + i);
      am = fmaxf(am, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
    __syncthreads();
    am = red[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) am = fmaxf(am, red[w]);
    __syncthreads();
    const float gs = (am > 0.0f) ? __fdiv_rn(am, gden) : 1.0f;
    const float inv = __frcp_rn(gs);
    if (threadIdx.x == 0) gscale[t] = gs;
    for (int64_t b = threadIdx.x; b < nblk; b += kThreads) {
      float y[16];
      load16(xt + b * 16, y);
#pragma unroll
      for (int i = 0; i < 16; ++i) y[i] = __fmul_rn(y[i], inv);
      uint2 c;
      scales[t * nblk + b] = (uint8_t)quant_block<true>(y, kMode, c);
      reinterpret_cast<uint2*>(codes)[t * nblk + b] = c;
    }
  }
}

template <int kMode>
__global__ void __launch_bounds__(kThreads) dequantize_tiles_kernel(const uint8_t* __restrict__ codes,
                                                                    const uint8_t* __restrict__ scales,
                                                                    const float* __restrict__ gscale,
                                                                    int64_t blk_per_tile, float* __restrict__ out,
                                                                    int64_t nblk) {
  for (int64_t b = blockIdx.x * (int64_t)kThreads + threadIdx.x; b < nblk; b += (int64_t)gridDim.x * kThreads) {
    float x[16];
    dequant_block(__ldg(reinterpret_cast<const uint2*>(codes) + b), scale_decode(__ldg(scales + b), kMode), x);
    const float gs = __ldg(gscale + b / blk_per_tile);
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = __fmul_rn(x[i], gs);
    store16(out + b * 16, x);
  }
}

// Legacy update S' = alpha*S + beta*k[r]*v[c] (gdn_state_update_ref.cu:51-67,
// row r over k, column c over v).  The reference source line
//   alpha * s_prev + beta * k_fp32 * v_fp32
// leaves FMA contraction to the compiler; kVariant pins one of the three
// roundings so the result can be matched to the reference binary.
template <int kVariant>
__device__ __forceinline__ float legacy_elem(float s, float bk, float vc, float alpha) {
  if (kVariant == 0) return __fmaf_rn(alpha, s, __fmul_rn(bk, vc));
  if (kVariant == 1) return __fmaf_rn(bk, vc, __fmul_rn(alpha, s));
  return __fadd_rn(__fmul_rn(alpha, s), __fmul_rn(bk, vc));
}

// kOutF32: write the fp32 update (launch_gdn_ref); else requantise in place
// or out of place (launch_gdn_state_update).  kRowAligned: d % 16 == 0, so a
// scale block lies inside one row and v is read as two 16-byte vectors;
// otherwise (d % 4 == 0, the reference's d*d % 16 == 0) every element finds its
// own row and column.
template <int kVariant, bool kOutF32, bool kRowAligned>
__global__ void __launch_bounds__(kThreads) legacy_update_kernel(const uint8_t* S_data, const uint8_t* S_scales,
                                                                 const __nv_bfloat16* __restrict__ k,
                                                                 const __nv_bfloat16* __restrict__ v,
                                                                 uint8_t* out_data, uint8_t* out_scales,
                                                                 float* __restrict__ out_f32, float alpha,
                                                                 float beta, int d, int64_t nblk) {
  for (int64_t b = blockIdx.x * (int64_t)kThreads + threadIdx.x; b < nblk; b += (int64_t)gridDim.x * kThreads) {
    float x[16];
    dequant_block(reinterpret_cast<const uint2*>(S_data)[b], scale_decode(S_scales[b], kScaleRef240), x);
    if (kRowAligned) {
      const int bpr = d / 16;  // scale blocks per row
      const int r = (int)(b / bpr);
      const int c0 = (int)(b % bpr) * 16;
      const float bk = __fmul_rn(beta, bf2f(k[r]));
      const uint4* v4 = reinterpret_cast<const uint4*>(v + c0);
      __nv_bfloat16 vv[16];
      *reinterpret_cast<uint4*>(vv) = __ldg(v4);
      *reinterpret_cast<uint4*>(vv + 8) = __ldg(v4 + 1);
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = legacy_elem<kVariant>(x[i], bk, bf2f(vv[i]), alpha);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t e = b * 16 + i;
        const int r = (int)(e / d), c = (int)(e % d);
        x[i] = legacy_elem<kVariant>(x[i], __fmul_rn(beta, bf2f(k[r])), bf2f(v[c]), alpha);
      }
    }
    if (kOutF32) {
      store16(out_f32 + b * 16, x);
    } else {
      uint2 c;
      const uint32_t sc = quant_block<true>(x, kScaleRef240, c);
      reinterpret_cast<uint2*>(out_data)[b] = c;
      out_scales[b] = (uint8_t)sc;
    }
  }
}

// fmaf(beta*k, v, alpha*s): the rounding of the reference's compiled update
// line, found by comparing every variant bit for bit with the reference's
// launch_gdn_ref on a B200 (tests/test_gpu_legacy.py).  The reference entry
// points always use it; gdn_legacy_update_rounding takes a variant per call.
constexpr int kLegacyReferenceVariant = 1;

template <bool kOutF32>
int launch_legacy(const uint8_t* S_data, const uint8_t* S_scales, const __nv_bfloat16* k,
                  const __nv_bfloat16* v, uint8_t* out_data, uint8_t* out_scales, float* out_f32,
                  float alpha, float beta, int d, int variant, cudaStream_t stream) {
  const int64_t n = (int64_t)d * d;
  const int64_t nblk = n / 16;
  const int grid = grid_for(nblk);
#define GDN_LEGACY_LAUNCH(V, A)                                                                         \
  legacy_update_kernel<V, kOutF32, A><<<grid, kThreads, 0, stream>>>(S_data, S_scales, k, v, out_data, \
                                                                     out_scales, out_f32, alpha, beta, d, nblk)
  const bool aligned_rows = (d % 16 == 0) && aligned16(v);
  switch (variant * 2 + (aligned_rows ? 1 : 0)) {
    case 0: GDN_LEGACY_LAUNCH(0, false); break;
    case 1: GDN_LEGACY_LAUNCH(0, true); break;
    case 2: GDN_LEGACY_LAUNCH(1, false); break;
    case 3: GDN_LEGACY_LAUNCH(1, true); break;
    case 4: GDN_LEGACY_LAUNCH(2, false); break;
    default: GDN_LEGACY_LAUNCH(2, true); break;
  }
#undef GDN_LEGACY_LAUNCH
  return launch_status();
}

// Sweeps of the device codec over consecutive fp32 bit patterns lo, lo+1, ...
// (the exhaustive checks of the production paths against the reference):
//   which 0: out[i] = block_scale_code(f, mode), the scale byte the
//            requantisers write for a block whose max |y| is f;
//   which 1: out[i] = e2m1_encode8 nibble of f with inverse scale 1, the
//            per-element encoder every quantiser here uses.
// One thread per 8 values; the caller keeps lo + count <= 2^32.
__global__ void __launch_bounds__(kThreads) codec_selftest_kernel(int which, uint32_t lo, int64_t count, int mode,
                                                                  uint8_t* __restrict__ out) {
  for (int64_t t = blockIdx.x * (int64_t)kThreads + threadIdx.x; t * 8 < count; t += (int64_t)gridDim.x * kThreads) {
    const int64_t i0 = t * 8;
    const int n = count - i0 < 8 ? (int)(count - i0) : 8;
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(lo + (uint32_t)(i0 + (e < n ? e : 0)));
    uint8_t r[8];
    if (which == 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = (uint8_t)block_scale_code(f[e], mode);
    } else {
      const float2 y[4] = {make_float2(f[0], f[1]), make_float2(f[2], f[3]), make_float2(f[4], f[5]),
                           make_float2(f[6], f[7])};
      const uint32_t w = e2m1_encode8(y, make_float2(1.0f, 1.0f));
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = (uint8_t)((w >> (4 * e)) & 0xFu);
    }
    for (int e = 0; e < n; ++e) out[i0 + e] = r[e];
  }
}

bool legacy_args_ok(const void* a, const void* b, const void* k, const void* v, const void* c,
                    const void* e, int d) {
  return a && b && k && v && c && e && d > 0 && d % 4 == 0;
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int launch_gdn_state_update(const uint8_t* S_data, const uint8_t* S_scales, const __nv_bfloat16* k,
                                       const __nv_bfloat16* v, uint8_t* S_out_data, uint8_t* S_out_scales,
                                       float alpha, float beta, int d, cudaStream_t stream) {
  // Reference: code 1 for null pointers or d <= 0 (gdn_state_update_ref.cu:214-217).
  // d*d must be a multiple of 16 (the op's check, src/ops/gdn_op.cu:74); the
  // reference C entry point would read past the scale array otherwise.
  if (!legacy_args_ok(S_data, S_scales, k, v, S_out_data, S_out_scales, d)) return GDN_ERR_ARGS;
  if ((reinterpret_cast<uintptr_t>(S_data) & 7u) || (reinterpret_cast<uintptr_t>(S_out_data) & 7u))
    return GDN_ERR_ALIGN;
  return launch_legacy<false>(S_data, S_scales, k, v, S_out_data, S_out_scales, nullptr, alpha, beta, d,
                              kLegacyReferenceVariant, stream);
}

extern "C" void launch_gdn_ref(const uint8_t* S_data, const uint8_t* S_scales, const __nv_bfloat16* k,
                               const __nv_bfloat16* v, float* S_out, float alpha, float beta, int d,
                               cudaStream_t stream) {
  if (!legacy_args_ok(S_data, S_scales, k, v, S_out, S_out, d)) return;
  if ((reinterpret_cast<uintptr_t>(S_data) & 7u) || !aligned16(S_out)) return;
  launch_legacy<true>(S_data, S_scales, k, v, nullptr, nullptr, S_out, alpha, beta, d, kLegacyReferenceVariant,
                      stream);
}

extern "C" int gdn_legacy_update_rounding(const uint8_t* S_data, const uint8_t* S_scales, const __nv_bfloat16* k,
                                          const __nv_bfloat16* v, uint8_t* S_out_data, uint8_t* S_out_scales,
                                          float* S_out_f32, float alpha, float beta, int d, int rounding,
                                          cudaStream_t stream) {
  if (rounding < 0 || rounding > 2) return GDN_ERR_ARGS;
  if (S_out_f32) {
    if (!legacy_args_ok(S_data, S_scales, k, v, S_out_f32, S_out_f32, d)) return GDN_ERR_ARGS;
    if ((reinterpret_cast<uintptr_t>(S_data) & 7u) || !aligned16(S_out_f32)) return GDN_ERR_ALIGN;
    return launch_legacy<true>(S_data, S_scales, k, v, nullptr, nullptr, S_out_f32, alpha, beta, d, rounding,
                               stream);
  }
  if (!legacy_args_ok(S_data, S_scales, k, v, S_out_data, S_out_scales, d)) return GDN_ERR_ARGS;
  if ((reinterpret_cast<uintptr_t>(S_data) & 7u) || (reinterpret_cast<uintptr_t>(S_out_data) & 7u))
    return GDN_ERR_ALIGN;
  return launch_legacy<false>(S_data, S_scales, k, v, S_out_data, S_out_scales, nullptr, alpha, beta, d, rounding,
                              stream);
}

extern "C" int gdn_nvfp4_quantize(const float* x, uint8_t* codes, uint8_t* scales, int64_t n, int32_t mode,
                                  cudaStream_t stream) {
  if (!x || !codes || !scales || n <= 0 || n % 16) return GDN_ERR_ARGS;
  if (mode != kScaleRef240 && mode != kScaleFn448) return GDN_ERR_UNSUPPORTED;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(codes) & 7u)) return GDN_ERR_ALIGN;
  const int64_t nblk = n / 16;
  if (mode == kScaleRef240)
    quantize_kernel<kScaleRef240><<<grid_for(nblk), kThreads, 0, stream>>>(x, codes, scales, nblk);
  else
    quantize_kernel<kScaleFn448><<<grid_for(nblk), kThreads, 0, stream>>>(x, codes, scales, nblk);
  return launch_status();
}

extern "C" int gdn_nvfp4_dequantize(const uint8_t* codes, const uint8_t* scales, float* out, int64_t n,
                                    int32_t mode, cudaStream_t stream) {
  if (!out || !codes || !scales || n <= 0 || n % 16) return GDN_ERR_ARGS;
  if (mode != kScaleRef240 && mode != kScaleFn448) return GDN_ERR_UNSUPPORTED;
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(codes) & 7u)) return GDN_ERR_ALIGN;
  const int64_t nblk = n / 16;
  if (mode == kScaleRef240)
    dequantize_kernel<kScaleRef240><<<grid_for(nblk), kThreads, 0, stream>>>(codes, scales, out, nblk);
  else
    dequantize_kernel<kScaleFn448><<<grid_for(nblk), kThreads, 0, stream>>>(codes, scales, out, nblk);
  return launch_status();
}

extern "C" int gdn_nvfp4_quantize_tiles(const float* x, int64_t num_tiles, int64_t tile_elems, uint8_t* codes,
                                        uint8_t* scales, float* gscale, int32_t mode, float gden,
                                        cudaStream_t stream) {
  if (!x || !codes || !scales || !gscale || num_tiles <= 0 || tile_elems <= 0 || tile_elems % 16)
    return GDN_ERR_ARGS;
  if (mode != kScaleRef240 && mode != kScaleFn448) return GDN_ERR_UNSUPPORTED;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(codes) & 7u)) return GDN_ERR_ALIGN;
  if (!(gden > 0.0f)) gden = default_gden(mode);
  int64_t grid = num_tiles;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (grid > cap) grid = cap;
  if (mode == kScaleRef240)
    quantize_tiles_kernel<kScaleRef240><<<(int)grid, kThreads, 0, stream>>>(x, tile_elems, codes, scales, gscale,
                                                                            gden, num_tiles);
  else
    quantize_tiles_kernel<kScaleFn448><<<(int)grid, kThreads, 0, stream>>>(x, tile_elems, codes, scales, gscale,
                                                                           gden, num_tiles);
  return launch_status();
}

extern "C" int gdn_nvfp4_dequantize_tiles(const uint8_t* codes, const uint8_t* scales, const float* gscale,
                                          int64_t num_tiles, int64_t tile_elems, float* out, int32_t mode,
                                          cudaStream_t stream) {
  if (!out || !codes || !scales || !gscale || num_tiles <= 0 || tile_elems <= 0 || tile_elems % 16)
    return GDN_ERR_ARGS;
  if (mode != kScaleRef240 && mode != kScaleFn448) return GDN_ERR_UNSUPPORTED;
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(codes) & 7u)) return GDN_ERR_ALIGN;
  const int64_t nblk = num_tiles * (tile_elems / 16);
  if (mode == kScaleRef240)
    dequantize_tiles_kernel<kScaleRef240><<<grid_for(nblk), kThreads, 0, stream>>>(codes, scales, gscale,
                                                                                   tile_elems / 16, out, nblk);
  else
    dequantize_tiles_kernel<kScaleFn448><<<grid_for(nblk), kThreads, 0, stream>>>(codes, scales, gscale,
                                                                                  tile_elems / 16, out, nblk);
  return launch_status();
}

extern "C" int gdn_b200_selftest_codec(int32_t which, uint32_t lo_bits, int64_t count, int32_t scale_mode,
                                       uint8_t* out, cudaStream_t stream) {
  if (!out || count <= 0 || (which != 0 && which != 1)) return GDN_ERR_ARGS;
  if ((uint64_t)lo_bits + (uint64_t)count > (1ull << 32)) return GDN_ERR_ARGS;
  if (scale_mode != kScaleRef240 && scale_mode != kScaleFn448) return GDN_ERR_UNSUPPORTED;
  const int64_t threads = (count + 7) / 8;
  codec_selftest_kernel<<<grid_for(threads), kThreads, 0, stream>>>(which, lo_bits, count, scale_mode, out);
  return launch_status();
}
