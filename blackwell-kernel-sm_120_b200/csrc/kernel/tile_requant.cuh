// tile_requant.cuh -- requantisation of whole 16-element scale blocks of a
// 128 x 128 NVFP4 state tile, shared by the decode and prefill kernels.
//
// Each thread owns whole 16-element scale blocks of one row (two or four,
// i.e. a quarter or a half row) as fp32 pairs.  The tile's global scale is
// gs = amax / gden
// (1.0 for an all-zero tile) and every block goes through the reference block
// quantiser (src/kernel/gdn_state_update_ref.cu:93-141) applied to
// y = x * RN(1/gs): local scale amax_blk / 6, scale byte by the reference
// encoder, E2M1 nearest with ties to the smaller magnitude.
#pragma once

#include <cstdint>

#include "../intrinsics/nvfp4_codec.cuh"

namespace gdn {

// Per-block max |x| of the four blocks (NaN ignored, as the reference's fmaxf
// scan does) and their maximum.  am[blk] may be NaN-free only; the return
// value feeds the tile amax.
__device__ __forceinline__ float block_amax4(const float2 (&x)[32], float (&am)[4]) {
  float tmax = 0.0f;
#pragma unroll
  for (int blk = 0; blk < 4; ++blk) {
    float mx = absmax_nan(x[8 * blk].x, x[8 * blk].y);
#pragma unroll
    for (int p = 1; p < 8; ++p) mx = absmax_nan(absmax_nan(mx, x[8 * blk + p].x), x[8 * blk + p].y);
    am[blk] = fabsf(mx);
    float ok_max = am[blk];
    if (isnan(ok_max)) {
      ok_max = 0.0f;
#pragma unroll
      for (int p = 0; p < 8; ++p) ok_max = fmaxf(ok_max, fmaxf(fabsf(x[8 * blk + p].x), fabsf(x[8 * blk + p].y)));
    }
    tmax = fmaxf(tmax, ok_max);
  }
  return tmax;
}

// Block max |x| with three-input max (sm_100): am[blk] = max |x| of block blk,
// NaN when the block holds one (the requantiser then takes its exact path);
// returns the NaN-ignoring maximum over the blocks.
template <int NB>
__device__ __forceinline__ float block_amax3(const float2 (&x)[8 * NB], float (&am)[NB]) {
  float tmax = 0.0f;
#pragma unroll
  for (int blk = 0; blk < NB; ++blk) {
    const float2* xb = x + 8 * blk;
    float m0, m1, mb;
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(xb[0].x), "f"(xb[0].y), "f"(xb[1].x));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(xb[1].y), "f"(xb[2].x), "f"(xb[2].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[3].x), "f"(xb[3].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(m1), "f"(xb[4].x), "f"(xb[4].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[5].x), "f"(xb[5].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(m1), "f"(xb[6].x), "f"(xb[6].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[7].x), "f"(xb[7].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(mb) : "f"(m0), "f"(m1), "f"(0.0f));
    am[blk] = mb;
    float ok_max = mb;
    if (isnan(mb)) {  // rare: the reference's amax ignores NaN
      ok_max = 0.0f;
#pragma unroll
      for (int p = 0; p < 8; ++p) ok_max = fmaxf(ok_max, fmaxf(fabsf(xb[p].x), fabsf(xb[p].y)));
    }
    tmax = fmaxf(tmax, ok_max);
  }
  return tmax;
}

// As block_amax3 without the per-block NaN test: am[blk] = max |x| of block
// blk, NaN when the block holds one.  The caller folds the block maxima with
// max3_nan and takes the NaN-ignoring maximum (amax_ignore_nan) only in the
// rare case that the fold is NaN.
template <int NB>
__device__ __forceinline__ void block_amax3_raw(const float2 (&x)[8 * NB], float (&am)[NB]) {
#pragma unroll
  for (int blk = 0; blk < NB; ++blk) {
    const float2* xb = x + 8 * blk;
    float m0, m1, mb;
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(xb[0].x), "f"(xb[0].y), "f"(xb[1].x));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(xb[1].y), "f"(xb[2].x), "f"(xb[2].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[3].x), "f"(xb[3].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(m1), "f"(xb[4].x), "f"(xb[4].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[5].x), "f"(xb[5].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m1) : "f"(m1), "f"(xb[6].x), "f"(xb[6].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(m0) : "f"(m0), "f"(xb[7].x), "f"(xb[7].y));
    asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(mb) : "f"(m0), "f"(m1), "f"(0.0f));
    am[blk] = mb;
  }
}

// max of three non-negative-or-NaN values, NaN if any is NaN.
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// max |x| over 16 pairs, NaN ignored (the reference's fmaxf scan); 0 if all are NaN.
__device__ __forceinline__ float amax_ignore_nan(const float2 (&x)[16]) {
  float m = 0.0f;
#pragma unroll
  for (int p = 0; p < 16; ++p) m = fmaxf(m, fmaxf(fabsf(x[p].x), fabsf(x[p].y)));
  return m;
}

// Quantises the NB 16-element blocks of x with the tile's inverse global
// scale.  am[blk] = max |x| of block blk (NaN when the block holds one).
// inv_tab[s] = 1 / decode(s) for every scale byte s.  Writes the 8 NB code
// bytes (2 NB words, element order) and the NB scale bytes (low bytes of
// scw, block order); debug_row, when set, receives the 16 NB fp32 quantiser
// inputs.
template <int kMode, int NB>
__device__ __forceinline__ void requant_blocks(const float2 (&x)[8 * NB], const float (&am)[NB], float inv_gs,
                                               const float* inv_tab, uint32_t (&words)[2 * NB], uint32_t& scw,
                                               float* debug_row) {
  const float2 r2 = make_float2(inv_gs, inv_gs);
  scw = 0;
#pragma unroll
  for (int blk = 0; blk < NB; ++blk) {
    float2 y[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) y[p] = __fmul2_rn(x[8 * blk + p], r2);
    // max |y| of the block = RN(max |x| * inv_gs): rounding is monotone.
    const float am_y = __fmul_rn(am[blk], inv_gs);
    uint32_t w0, w1, sc;
    if (am_y <= 3.0e38f) {
      sc = block_scale_code(am_y, kMode);
      const float inv = inv_tab[sc];
      const float2 inv2 = make_float2(inv, inv);
      w0 = e2m1_encode8(y, inv2);
      w1 = e2m1_encode8(y + 4, inv2);
    } else {  // NaN or inf in the block: exact scalar path
      sc = quantize16_exact_pairs(y, kMode, w0, w1);
    }
    words[2 * blk] = w0;
    words[2 * blk + 1] = w1;
    scw |= sc << (8 * blk);
    if (debug_row) {
      float4* dy = reinterpret_cast<float4*>(debug_row + 16 * blk);
#pragma unroll
      for (int p = 0; p < 4; ++p) dy[p] = make_float4(y[2 * p].x, y[2 * p].y, y[2 * p + 1].x, y[2 * p + 1].y);
    }
  }
}

// ---- power-of-two global scale ---------------------------------------------
//
// The decode requantiser picks the new global scale as gs' = c * 2^-k, where
// S' = c * D (D the fp32 tile it holds) and k >= 0 is the largest integer with
// max |D| * 2^k <= gden, and quantises y = D * 2^k.  Scaling by 2^k is exact,
// so everything the reference quantiser derives from y follows from D:
//   * a block's max |y| is am * 2^k and its local scale RN(am * 2^k / 6) is
//     2^k RN(am / 6) (am / 6 a normal float);
//   * the scale byte, while it lies in [8, saturation] (a normal E4M3 code
//     with no clamping), is the code of RN(am / 6) plus 8k: scale_w() - 960 + 8k;
//   * the inverse of that scale is RN(1 / dec) = scale_inv_w() * 2^-k, so
//     RN(y * inv) = RN(D * scale_inv_w()), which does not depend on k.
// The E2M1 codes of a block can therefore be computed before the tile max is
// known, with one multiply per element fewer than y = D * 2^k, v = y * inv.
// Blocks whose final scale byte falls outside [8, saturation] (a subnormal
// or zero local scale, saturation) or that hold a NaN take the exact path.

// The scale encoder's rounding of x = RN(am / 6) for a finite am > 0 with x a
// normal float, as (biased exponent << 3 | 3 mantissa bits): half up at the
// third mantissa bit, a significand >= 1.875 to the next binade
// (src/intrinsics/gdn_fp4_intrinsics.cuh:102-120).  For x >= 2^-6 the E4M3
// code is this value - 960; the decoded scale is the float with bits w << 20.
__device__ __forceinline__ uint32_t scale_w(float am) {
  const uint32_t u = __float_as_uint(div6_for_scale(am));
  const uint32_t add = ((u & 0x700000u) == 0x700000u) ? 0x100000u : 0x80000u;
  return (u + add) >> 20;
}

// rt[m] = bits of RN(1 / (1 + m/8)) + (127 << 23) for m = 0..7 (scale_inv_w_entry).
// RN(1 / dec) of the decoded scale with bits w << 20 is then
// rt[w & 7] - ((w >> 3) << 23): the reciprocal's significand from the table
// and its exponent 127 - (biased exponent of dec), exact while both are
// normal floats.
__device__ __forceinline__ float scale_inv_w(uint32_t w, const uint32_t* rt) {
  return __uint_as_float(rt[w & 7u] - ((w & ~7u) << 20));
}

// RN(1 / (1 + m / 8)) for m = 0..7, correctly rounded (the reciprocals of
// 8/8 .. 15/8), as float bit patterns plus 127 << 23.
__host__ __device__ constexpr uint32_t scale_inv_w_entry(int m) {
  return (m == 0 ? 0x3F800000u    // 1
          : m == 1 ? 0x3F638E39u  // 8/9
          : m == 2 ? 0x3F4CCCCDu  // 8/10
          : m == 3 ? 0x3F3A2E8Cu  // 8/11
          : m == 4 ? 0x3F2AAAABu  // 8/12
          : m == 5 ? 0x3F1D89D9u  // 8/13
          : m == 6 ? 0x3F124925u  // 8/14
                   : 0x3F088889u) // 8/15
         + (127u << 23);
}

// k = the largest integer with A * 2^k <= gden, for normal positive floats A
// and gden, from their bit patterns.
__device__ __forceinline__ int pow2_headroom(uint32_t a_bits, uint32_t gden_bits) {
  return (int)(gden_bits >> 23) - (int)(a_bits >> 23) - ((a_bits & 0x7FFFFFu) > (gden_bits & 0x7FFFFFu) ? 1 : 0);
}

// 2^e for an integer e in [-126, 127].
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// The 64-element form used by the prefill epilogue.
template <int kMode>
__device__ __forceinline__ void requant_half_row(const float2 (&x)[32], const float (&am)[4], float inv_gs,
                                                 const float* inv_tab, uint32_t (&words)[8], uint32_t& scw,
                                                 float* debug_row) {
  requant_blocks<kMode, 4>(x, am, inv_gs, inv_tab, words, scw, debug_row);
}

}  // namespace gdn
