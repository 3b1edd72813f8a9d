// nvfp4_codec.cuh -- NVFP4 state codec for sm_100a (host + device).
//
// Format (the reference's, src/kernel/gdn_state_update_ref.cu:16-18):
//   * E2M1 codes packed two per byte, the even element in the low nibble;
//   * one 8-bit E4M3-style scale per 16 contiguous elements;
//   * (new) one fp32 global scale per state tile, applied as y = x * (1/gs).
//
// Two scale modes:
//   kScaleRef240 -- the reference codec exactly: encoder saturates at 240
//                   (0x77), decoder reads exponent 15 as inf/NaN
//                   (src/intrinsics/gdn_fp4_intrinsics.cuh:48-123).
//   kScaleFn448  -- the same rounding rules extended to the E4M3FN range
//                   (saturation 448 = 0x7E, exponent 15 is a normal binade,
//                   0x7F is NaN).  Identical bytes to kScaleRef240 for every
//                   block whose local scale is below 240.
//
// Every encoder here is bit-exact with the reference quantiser
// nvfp4_quantise_host (src/kernel/gdn_state_update_ref.cu:93-141) given the
// same fp32 inputs.  The fast device path uses the Blackwell conversions
// cvt.rn.f16x2.e2m1x2 (decode) and cvt.rn.satfinite.e2m1x2.f32 (encode); the
// encode side corrects round-to-nearest-even into the reference's
// "ties go to the smaller magnitude" rule with one FMA per element (see
// e2m1_nudge below).
#pragma once

#include <cstdint>
#include <cstring>
#include <cmath>
#include <cuda_runtime.h>

namespace gdn {

enum ScaleMode : int { kScaleRef240 = 0, kScaleFn448 = 1 };

// Default global-scale denominators: gs = amax / (6 * saturation), so that the
// largest block of a tile lands on the largest finite scale.
__host__ __device__ constexpr float default_gden(int mode) { return mode ? 6.0f * 448.0f : 6.0f * 240.0f; }

__host__ __device__ inline float f32_bits(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f; std::memcpy(&f, &u, 4); return f;
#endif
}
__host__ __device__ inline uint32_t bits_f32(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u; std::memcpy(&u, &f, 4); return u;
#endif
}

// E2M1 nibble value; exact.  Follows gdn_fp4_intrinsics.cuh:27-45:
// magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, bit 3 is the sign.
__host__ __device__ inline float e2m1_value(uint32_t nib) {
  const uint32_t c = nib & 7u;
  // c >= 2: (1 + m/2) * 2^(e-1) has fp32 bits (c << 22) + (126 << 23).
  float mag = (c >= 2u) ? f32_bits((c << 22) + 0x3F000000u) : (c ? 0.5f : 0.0f);
  return (nib & 8u) ? -mag : mag;
}

// Scale byte -> float, gdn_fp4_intrinsics.cuh:48-68 (mode 0) or E4M3FN (mode 1).
__host__ __device__ inline float scale_decode(uint32_t b, int mode) {
  b &= 0xFFu;
  const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
  float mag;
  if (e == 0u) {
    mag = (float)m * 0.001953125f;  // m * 2^-9, exact
  } else if (e == 15u && (mode == kScaleRef240 || m == 7u)) {
    mag = (mode == kScaleRef240 && m == 0u) ? f32_bits(0x7F800000u) : f32_bits(0x7FC00000u);
  } else {
    mag = f32_bits(((e + 120u) << 23) | (m << 20));
  }
  return (b & 0x80u) ? -mag : mag;
}

// Reciprocal used by the quantiser: 1/dec if dec > 0, else 0
// (gdn_state_update_ref.cu:110-111).  Correctly rounded on both sides.
__host__ __device__ inline float scale_inverse(float dec) {
#ifdef __CUDA_ARCH__
  return (dec > 0.0f) ? __frcp_rn(dec) : 0.0f;
#else
  return (dec > 0.0f) ? (1.0f / dec) : 0.0f;
#endif
}

// float -> scale byte with the reference's rounding (gdn_fp4_intrinsics.cuh:71-123),
// restated on the fp32 bit pattern:
//   * not finite or <= 0                      -> 0
//   * below 2^-6 (subnormal scale)            -> min(7, int(x*512 + 0.5f))
//   * normal: round half up at 3 mantissa bits (add 2^19 to the bits), except
//     that a significand in [1.875, 2) always rounds up to the next binade
//     (the reference halves n >= 1.875 before rounding);
//   * saturate at 0x77 (mode 0) / 0x7E (mode 1).
// Checked exhaustively against the reference encoder over all positive floats.
__host__ __device__ inline uint32_t scale_encode(float x, int mode) {
  const uint32_t u = bits_f32(x);
  if (!(x > 0.0f) || u >= 0x7F800000u) return 0u;
  if (x < 0.015625f) {
#ifdef __CUDA_ARCH__
    const int m = (int)__fmaf_rn(x, 512.0f, 0.5f);
#else
    const int m = (int)std::fma(x, 512.0f, 0.5f);
#endif
    return (uint32_t)(m > 7 ? 7 : m);
  }
  const uint32_t add = ((u & 0x7FFFFFu) >= 0x700000u) ? 0x100000u : 0x80000u;
  const uint32_t code = ((u + add) >> 20) - 960u;  // 960 = (127 - 7) << 3
  const uint32_t sat = mode ? 0x7Eu : 0x77u;
  return code > sat ? sat : code;
}

// Local block scale input: amax/6, or 1.0 for an all-zero block
// (gdn_state_update_ref.cu:106-107).  The division is IEEE round-to-nearest.
__host__ __device__ inline float local_scale(float amax) {
#ifdef __CUDA_ARCH__
  return (amax > 0.0f) ? __fdiv_rn(amax, 6.0f) : 1.0f;
#else
  return (amax > 0.0f) ? (amax / 6.0f) : 1.0f;
#endif
}

// Exact reference E2M1 encoder (gdn_state_update_ref.cu:117-135): nearest
// magnitude with a strict '<' scan over rounded errors |a - m_k| (ties keep the
// smaller magnitude), sign from (x < 0).  Below 8 the scan equals a threshold
// count: for a in [m_k, m_k+1] the two candidate errors are exact (Sterbenz),
// so the larger magnitude wins iff a exceeds the midpoint.  From 2^25 up the
// rounded errors collide and the scan's answer depends on rounding, so large
// inputs run the literal scan.  NaN gives 0.
__host__ __device__ inline uint32_t e2m1_encode_exact(float x) {
  const float a = fabsf(x);
  uint32_t c;
  if (a < 8.0f) {
    c = (a > 0.25f) + (a > 0.75f) + (a > 1.25f) + (a > 1.75f) + (a > 2.5f) + (a > 3.5f) + (a > 5.0f);
  } else {
    const float mags[8] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    float best = fabsf(a - mags[0]);
    c = 0u;
    for (uint32_t k = 1; k < 8; ++k) {
      const float e = fabsf(a - mags[k]);
      if (e < best) { best = e; c = k; }
    }
  }
  return c | ((x < 0.0f) ? 8u : 0u);
}

// Tie correction for the hardware converter.  cvt.rn.satfinite.e2m1x2 rounds
// to nearest-even, which differs from the reference only at the three "odd"
// midpoints 0.75, 1.75, 3.5 (RNE rounds them up).  Feeding it
// n = RN(v - v*eps) with eps*2^23 in (1/3, 0.4) moves every value whose
// significand starts 1.1x (0.75, 1.75, 3.5) down by more than half an ulp and
// every value whose significand starts 1.0x or 1.01 (0.25, 1.25, 2.5, 5) by
// less than half an ulp, so RNE on n equals "ties to smaller" on v for every
// fp32 v.  It also turns -0.0 into +0.0, as the reference's (v < 0) sign test
// does.  Verified exhaustively for |v| < 8 (larger values saturate to 6 either
// way).
constexpr float kE2M1TieEps = 4.335e-8f;

#ifdef __CUDACC__
__device__ __forceinline__ float e2m1_nudge(float v) { return __fmaf_rn(v, -kE2M1TieEps, v); }

// amax/6 in three operations (Markstein's FMA correction of a quotient: q0 =
// a*RN(1/6), r = a - 6*q0 exactly, q = q0 + r*RN(1/6)).  Checked against IEEE
// division for every positive finite float: identical for a >= 2^-125; below
// that the quotient is subnormal and may differ in its last bits, but every
// such quotient (< 2^-127) encodes to scale code 0 either way, so the scale
// byte -- the only consumer -- is identical for all inputs.
__device__ __forceinline__ float div6_for_scale(float a) {
  const float y = 0.16666667163372039795f;  // RN(1/6)
  const float q0 = __fmul_rn(a, y);
  const float r = __fmaf_rn(-q0, 6.0f, a);
  return __fmaf_rn(r, y, q0);
}

__device__ __forceinline__ float local_scale_fast(float amax) {
  return (amax > 0.0f) ? div6_for_scale(amax) : 1.0f;
}

// scale_encode(local_scale_fast(amax), mode) for a finite amax >= 0, without
// the encoder's "<= 0 or not finite" test: amax / 6 of a finite amax is finite,
// a quotient that underflows to 0 takes the subnormal branch to code 0 as the
// test would, and a zero block takes the reference's local scale 1.0 (0x38).
__device__ __forceinline__ uint32_t block_scale_code(float amax, int mode) {
  if (!(amax > 0.0f)) return 0x38u;
  const float x = div6_for_scale(amax);
  if (x < 0.015625f) {
    const int m = (int)__fmaf_rn(x, 512.0f, 0.5f);
    return (uint32_t)(m > 7 ? 7 : m);
  }
  const uint32_t u = __float_as_uint(x);
  const uint32_t add = ((u & 0x7FFFFFu) >= 0x700000u) ? 0x100000u : 0x80000u;
  const uint32_t code = ((u + add) >> 20) - 960u;
  const uint32_t sat = mode ? 0x7Eu : 0x77u;
  return code > sat ? sat : code;
}

__device__ __forceinline__ float2 e2m1_nudge2(float2 v) {
  return __ffma2_rn(v, make_float2(-kE2M1TieEps, -kE2M1TieEps), v);
}

// Two fp32 -> one byte: low nibble from `lo`, high nibble from `hi`.
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint16_t r;
  asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %1, %2; cvt.u16.u8 %0, t; }"
      : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Eight fp32 (already scaled by the block inverse and nudged) -> 4 bytes.
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float* n) {
  uint32_t r;
  asm("{ .reg .b8 b0, b1, b2, b3;\n"
      "  cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
      "  cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      "  cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
      "  cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      "  mov.b32 %0, {b0, b1, b2, b3}; }"
      : "=r"(r)
      : "f"(n[0]), "f"(n[1]), "f"(n[2]), "f"(n[3]), "f"(n[4]), "f"(n[5]), "f"(n[6]), "f"(n[7]));
  return r;
}

// E2M1 codes of v = RN(y * inv) for 8 values (pairs y[0..3], element 0 in the
// low nibble) with the reference's rounding: nearest, ties to the smaller
// magnitude, sign from (v < 0).  The nudge also maps v = -0 to +0 (code 0x0),
// as the reference's sign test does.  Exact for every finite y * inv with
// |v| < 8 (larger values saturate to 6 either way); the whole domain is swept
// by gdn_b200_selftest_codec.
__device__ __forceinline__ uint32_t e2m1_encode8(const float2* y, float2 inv2) {
  float2 n[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) n[p] = e2m1_nudge2(__fmul2_rn(y[p], inv2));
  return cvt_e2m1x8(reinterpret_cast<const float*>(n));
}

// One code word (8 nibbles, element 0 in the low nibble) -> 8 raw E2M1 values as
// four f16x2 (element 2j in the low half of out[j]).  Exact.
__device__ __forceinline__ void cvt_e2m1x8_to_f16x2(uint32_t w, uint32_t (&out)[4]) {
  asm("{ .reg .b8 b0, b1, b2, b3;\n"
      "  mov.b32 {b0, b1, b2, b3}, %4;\n"
      "  cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "  cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "  cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "  cvt.rn.f16x2.e2m1x2 %3, b3; }"
      : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
      : "r"(w));
}

__device__ __forceinline__ float2 f16x2_to_f32x2(uint32_t h) {
  float lo, hi;
  asm("{ .reg .f16 a, b; mov.b32 {a, b}, %2; cvt.f32.f16 %0, a; cvt.f32.f16 %1, b; }"
      : "=f"(lo), "=f"(hi) : "r"(h));
  return make_float2(lo, hi);
}

// max(|a|, |b|) propagating NaN; the sign of the result is meaningless
// (callers take fabsf at the end).
__device__ __forceinline__ float absmax_nan(float a, float b) {
  float r;
  asm("max.NaN.xorsign.abs.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Exact path: reference semantics (NaN-ignoring amax, literal encoder).  Kept
// out of line: only blocks holding NaN/inf or huge ratios reach it.
static __device__ __noinline__ uint32_t quantize16_exact(const float* y, int mode, uint32_t& w0, uint32_t& w1) {
  float amax = 0.0f;
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(y[i]));
  const uint32_t sc = scale_encode(local_scale(amax), mode);
  const float inv = scale_inverse(scale_decode(sc, mode));
  uint32_t c[2] = {0u, 0u};
  for (int i = 0; i < 16; ++i) c[i >> 3] |= e2m1_encode_exact(__fmul_rn(y[i], inv)) << (4 * (i & 7));
  w0 = c[0];
  w1 = c[1];
  return sc;
}

// The same exact path on register pairs (y[p] = elements 2p, 2p+1), inline so
// that a kernel keeping its state in registers needs no call (and no spills)
// for the rare non-finite block.
__device__ __forceinline__ uint32_t quantize16_exact_pairs(const float2 (&y)[8], int mode, uint32_t& w0,
                                                           uint32_t& w1) {
  float amax = 0.0f;
#pragma unroll
  for (int p = 0; p < 8; ++p) amax = fmaxf(amax, fmaxf(fabsf(y[p].x), fabsf(y[p].y)));
  const uint32_t sc = scale_encode(local_scale(amax), mode);
  const float inv = scale_inverse(scale_decode(sc, mode));
  uint32_t c0 = 0u, c1 = 0u;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    c0 |= (e2m1_encode_exact(__fmul_rn(y[p].x, inv)) | (e2m1_encode_exact(__fmul_rn(y[p].y, inv)) << 4)) << (8 * p);
    c1 |= (e2m1_encode_exact(__fmul_rn(y[p + 4].x, inv)) | (e2m1_encode_exact(__fmul_rn(y[p + 4].y, inv)) << 4))
          << (8 * p);
  }
  w0 = c0;
  w1 = c1;
  return sc;
}

// Quantise 16 fp32 inputs (the reference quantiser's block) to 8 code bytes and
// one scale byte.  `amax_nan` is the NaN-propagating |max| of the block.  The
// fast path (hardware converter + tie nudge) is exact while the block is finite
// and every |y * inv| < 2^24; otherwise the block takes the exact scalar path.
// With a global scale (|y| <= gden) the second condition always holds: an
// unsaturated block has |y * inv| <= 6 * 16/15, the saturated top block
// |y * inv| <= gden / saturation = 6.  kCheckRange = false skips that test.
// Returns the scale byte; codes land in w0 (elements 0..7) and w1 (8..15).
template <bool kCheckRange>
__device__ __forceinline__ uint32_t quantize16(const float* y, float amax_nan, int mode,
                                               uint32_t& w0, uint32_t& w1) {
  const float am = fabsf(amax_nan);
  bool fast = am <= 3.0e38f;  // finite (NaN and inf fail the test)
  const float amax_ok = fast ? am : 0.0f;
  uint32_t sc = scale_encode(local_scale(amax_ok), mode);
  float inv = scale_inverse(scale_decode(sc, mode));
  if (kCheckRange) fast = fast && (amax_ok * inv < 16777216.0f);
  if (fast) {
    float2 yp[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) yp[p] = make_float2(y[2 * p], y[2 * p + 1]);
    const float2 inv2 = make_float2(inv, inv);
    w0 = e2m1_encode8(yp, inv2);
    w1 = e2m1_encode8(yp + 4, inv2);
    return sc;
  }
  return quantize16_exact(y, mode, w0, w1);
}
#endif  // __CUDACC__

}  // namespace gdn
